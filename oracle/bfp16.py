"""bfp16ebs8 format oracle (numpy restatement) -- TEST INFRASTRUCTURE ONLY.

Restates the reference's 9-bit block-floating-point weight format (raon-npu
``quant/bfp16.py``) and the arithmetic of its GEMV (``kernels/gemv_bfp16/
reference.py``) so a GPU path for the format can be checked against it.  Each
function cites the reference lines whose behaviour it follows.

Format summary (``quant/bfp16.py:1-24``): the input (K) axis is cut into
groups of 8 values sharing one exponent byte ``e``; each value is an int8
mantissa ``m`` and decodes to ``m * 2**(e - 133)``.  The GEMV layout packs 32
output rows x 256 columns into a 9216-byte block: two halves of 16 rows, each
32 groups of [16 exponent bytes (one per row), 128 mantissa bytes stored
column-major as 8 columns x 16 rows].  Blocks follow the q4nx ordering
``((slice * k_blocks + k) * rows + row)`` with 4 block rows (128 output rows)
per slice.
"""

from __future__ import annotations

import numpy as np

GROUP = 8            # values per shared exponent   (quant/bfp16.py:36)
M_TILE = 32          # rows per GEMV block           (quant/bfp16.py:48)
K_TILE = 256         # columns per GEMV block        (quant/bfp16.py:49)
HALF_ROWS = 16       # rows per half block           (quant/bfp16.py:52)
GROUPS_PER_TILE = K_TILE // GROUP
GROUP_BYTES = HALF_ROWS + HALF_ROWS * GROUP          # 144 (quant/bfp16.py:58)
BLOCK_BYTES = 2 * GROUPS_PER_TILE * GROUP_BYTES      # 9216 (quant/bfp16.py:54-60)
E_MIN = 7            # smallest exponent the GEMV layout stores (quant/bfp16.py:43-45)


def encode(w) -> tuple[np.ndarray, np.ndarray]:
    """Round-to-nearest-even encoding along the last axis (the reference's
    default ``rounding="conv_even"``, ``quant/bfp16.py:75-125``).

    Per group of 8: e = the largest f32 exponent field of the group; the
    mantissas are rint(value / 2**(e - 133)) (ties to even, in f64, where the
    division by a power of two is exact); if any rounds above 127 the exponent
    goes up by one and the group is rounded again; finally the mantissas are
    clipped to [-128, 127] (so -128 is reachable, +128 is not).  Returns
    (exponents uint8 [..., K/8], mantissas int8 [..., K/8, 8]).
    """
    w = np.ascontiguousarray(w, dtype=np.float32)
    k = w.shape[-1]
    if k % GROUP:
        raise ValueError(f"last axis {k} is not a multiple of {GROUP}")
    if not np.isfinite(w).all():
        raise ValueError("inputs must be finite")
    groups = w.reshape(*w.shape[:-1], k // GROUP, GROUP)
    e = ((groups.view(np.uint32) >> 23) & 0xFF).max(axis=-1).astype(np.int64)
    vals = groups.astype(np.float64)
    m = np.rint(vals / np.ldexp(1.0, e - 133)[..., None])
    up = m.max(axis=-1) > 127
    if up.any():
        e = e + up
        m = np.rint(vals / np.ldexp(1.0, e - 133)[..., None])
    m = np.clip(m, -128, 127)
    return e.astype(np.uint8), m.astype(np.int8)


def decode(e, m) -> np.ndarray:
    """m * 2**(e - 133) as f32 (``quant/bfp16.py:128-141``)."""
    e = np.asarray(e, dtype=np.int64)
    return (np.asarray(m, dtype=np.float64) * np.ldexp(1.0, e - 133)[..., None]).astype(np.float32)


def flush_tiny(e, m) -> tuple[np.ndarray, np.ndarray]:
    """The GEMV layout's exponent floor (``quant/bfp16.py:252-268``): a group
    whose exponent is below 7 is stored as exponent 7 with zero mantissas."""
    e = np.asarray(e, dtype=np.uint8)
    tiny = e < E_MIN
    return np.where(tiny, np.uint8(E_MIN), e), np.where(tiny[..., None], np.int8(0), np.asarray(m, np.int8))


def pack_gemv(w, rows: int = 4) -> bytes:
    """GEMV layout bytes of an f32 matrix [M, K] (``quant/bfp16.py:190-292``,
    with the default ``flush_tiny=True``)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    M, K = w.shape
    if M % (rows * M_TILE) or K % K_TILE:
        raise ValueError(f"[{M}, {K}] must be a multiple of [{rows * M_TILE}, {K_TILE}]")
    e, m = flush_tiny(*encode(w))
    return pack_gemv_raw(e, m, rows)


def pack_gemv_raw(e, m, rows: int = 4) -> bytes:
    """Lay exponents [M, K/8] and mantissas [M, K/8, 8] out in GEMV blocks."""
    e = np.asarray(e, dtype=np.uint8)
    m = np.asarray(m, dtype=np.int8).view(np.uint8)
    M, G = e.shape
    kb, slices = G // GROUPS_PER_TILE, M // (rows * M_TILE)
    # (slice, row block, half, row, k block, group) -> (slice, k block, row block, half, group, row)
    ex = e.reshape(slices, rows, 2, HALF_ROWS, kb, GROUPS_PER_TILE).transpose(0, 4, 1, 2, 5, 3)
    # mantissas: (..., group, column) -> (..., group, column, row): column-major within a group
    mt = m.reshape(slices, rows, 2, HALF_ROWS, kb, GROUPS_PER_TILE, GROUP).transpose(0, 4, 1, 2, 5, 6, 3)
    mt = mt.reshape(slices, kb, rows, 2, GROUPS_PER_TILE, GROUP * HALF_ROWS)
    return np.ascontiguousarray(np.concatenate([ex, mt], axis=-1)).tobytes()


def parse_gemv(buf, K: int, M: int, rows: int = 4) -> tuple[np.ndarray, np.ndarray]:
    """Inverse of ``pack_gemv_raw``: (exponents [M, K/8], mantissas int8 [M, K])
    (``quant/bfp16.py:295-365``)."""
    kb, slices = K // K_TILE, M // (rows * M_TILE)
    raw = np.frombuffer(bytes(buf), dtype=np.uint8)[: slices * kb * rows * BLOCK_BYTES]
    raw = raw.reshape(slices, kb, rows, 2, GROUPS_PER_TILE, GROUP_BYTES)
    e = raw[..., :HALF_ROWS].transpose(0, 2, 3, 5, 1, 4).reshape(M, K // GROUP)
    mt = raw[..., HALF_ROWS:].reshape(slices, kb, rows, 2, GROUPS_PER_TILE, GROUP, HALF_ROWS)
    m = mt.transpose(0, 2, 3, 6, 1, 4, 5).reshape(M, K).view(np.int8)
    return np.ascontiguousarray(e), np.ascontiguousarray(m)


def gemv_weights(e, m) -> np.ndarray:
    """The GEMV's exact f32 weights (``kernels/gemv_bfp16/reference.py:25-46,
    160-167``): scale 2**(max(e, 7) - 133) (the kernel's defensive clamp),
    times the int8 mantissa; every product is exact in bf16."""
    e = np.maximum(np.asarray(e, dtype=np.int64), E_MIN)
    m = np.asarray(m, dtype=np.float64)
    M = e.shape[0]
    return (m.reshape(M, -1, GROUP) * np.ldexp(1.0, e - 133)[..., None]).reshape(M, -1).astype(np.float32)


def gemv(e, m, x_bits) -> np.ndarray:
    """y = bf16(sum_k w[:, k] * x[k]) for one bf16 row x (bit patterns):
    products exact, f32 accumulation in column order, round to nearest even
    (``kernels/gemv_bfp16/reference.py:118-182``).  Returns bf16 bits [M]."""
    w = gemv_weights(e, m)
    x = (np.asarray(x_bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
    acc = np.zeros(w.shape[0], dtype=np.float32)
    for k in range(w.shape[1]):
        acc = (acc + w[:, k] * x[k]).astype(np.float32)
    b = acc.view(np.uint32).astype(np.uint64)
    return (((b + 0x7FFF + ((b >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)
