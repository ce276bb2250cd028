"""q4nx format oracle (numpy restatement) -- TEST INFRASTRUCTURE ONLY.

Restates the reference's quantiser and GEMV packing (raon-npu ``quant/q4nx.py``)
so the CUDA upload/dequant path can be checked byte for byte.  Each function
cites the reference lines whose behaviour it follows.

Format summary (reference ``quant/q4nx.py:22-29``): a block covers 32 output
rows x 256 input columns in 5120 bytes = 512 B bf16 scales + 512 B bf16 mins
(both ``[group 8][row 32]``) + 4096 B of 4-bit codes; a weight dequantises to
``min + scale * code`` per 32-column group.
"""

from __future__ import annotations

import numpy as np

M_TILE = 32          # rows per block            (quant/q4nx.py:23)
K_TILE = 256         # columns per block         (quant/q4nx.py:24)
GROUP = 32           # columns per scale/min     (quant/q4nx.py:25)
BLOCK_BYTES = 5120   # 32*256*5/8                (quant/q4nx.py:28)
PARAM_BYTES = 1024   # scales + mins per block   (quant/q4nx.py:29)
GROUPS_PER_BLOCK = K_TILE // GROUP


# ---------------------------------------------------------------- bf16 bits --
def f32_to_bf16(x) -> np.ndarray:
    """f32 -> bf16 bit pattern, round-to-nearest-even, every NaN -> 0x7FC0.

    Follows ``quant/q4nx.py:32-44`` and ``host/weights.py:104-115``.
    """
    a = np.ascontiguousarray(x, dtype=np.float32)
    bits = a.view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    out = (rounded & 0xFFFF).astype(np.uint16)
    out[np.isnan(a)] = 0x7FC0
    return out


def bf16_to_f32(u) -> np.ndarray:
    """bf16 bit pattern -> f32 by a 16-bit left shift (``quant/q4nx.py:47-49``)."""
    return (np.asarray(u, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_round(x) -> np.ndarray:
    """Value of ``f32_to_bf16`` as f32 (``quant/q4nx.py:52-54``)."""
    return bf16_to_f32(f32_to_bf16(x))


def _to_f32_directed(x: np.ndarray, toward_neg: bool) -> np.ndarray:
    """Nearest f32 on the requested side of an f64 input (f32 input passes through)."""
    if x.dtype != np.float64:
        return np.asarray(x, dtype=np.float32)
    f = x.astype(np.float32)
    back = f.astype(np.float64)
    if toward_neg:
        return np.where(back > x, np.nextafter(f, np.float32(-np.inf)), f).astype(np.float32)
    return np.where(back < x, np.nextafter(f, np.float32(np.inf)), f).astype(np.float32)


def _bf16_directed(x, toward_neg: bool):
    arr = np.asarray(x)
    scalar = arr.ndim == 0
    f = np.atleast_1d(_to_f32_directed(arr, toward_neg))
    bits = np.ascontiguousarray(f).view(np.uint32)
    negative = (bits >> 31) == 1
    inexact = (bits & 0xFFFF) != 0
    # Truncation moves toward zero; one extra bf16 step away from zero is needed
    # when truncation went the wrong way (negative for floor, positive for ceil).
    step = inexact & (negative if toward_neg else ~negative)
    top = (bits >> 16) + step.astype(np.uint32)
    out = (top.astype(np.uint32) << 16).view(np.float32).copy()
    out[np.isnan(f)] = np.nan
    out = out.reshape(np.shape(f))
    return out.item() if scalar else out.reshape(arr.shape)


def bf16_floor(x):
    """Greatest bf16 <= x (``quant/q4nx.py:57-80``; f64 inputs handled exactly)."""
    return _bf16_directed(x, toward_neg=True)


def bf16_ceil(x):
    """Smallest bf16 >= x (``quant/q4nx.py:83-106``)."""
    return _bf16_directed(x, toward_neg=False)


def bf16_next_up(x):
    """Next bf16 toward +inf of an exact bf16 value; -0 counts as +0 (``quant/q4nx.py:109-124``)."""
    arr = np.asarray(x, dtype=np.float32)
    scalar = arr.ndim == 0
    top = (np.atleast_1d(arr).view(np.uint32) >> 16).astype(np.int64)
    top = np.where(top == 0x8000, 0, top)
    neg = top >= 0x8000
    nxt = np.where(top == 0, 1, np.where(neg, np.where(top == 0x8001, 0, top - 1), top + 1))
    out = (nxt.astype(np.uint32) << 16).view(np.float32).reshape(arr.shape)
    return out.item() if scalar else out


# ------------------------------------------------------------------ quantise --
def quantize(w: np.ndarray):
    """f32 [N, K] -> (codes u8 [N,K], scales f32 [N,K/32], mins f32 [N,K/32]).

    Steps of ``quant/q4nx.py:127-200``: per 32-column group, ``min_q`` is the bf16
    floor of the group minimum; ``scale_q`` the bf16 ceiling of
    ``(max - min_q) / 15`` (f64), stepped up one bf16 at a time until
    ``min_q + 15 * scale_q >= max`` (f64); a group whose max equals ``min_q``
    gets scale 0 and all codes 0; codes are ``clip(rint((w - min_q) / scale), 0, 15)``
    in f64.
    """
    arr = np.asarray(w)
    if arr.ndim != 2:
        raise ValueError(f"Weight matrix must be 2D, got shape {arr.shape}")
    if not np.isfinite(arr).all():
        raise ValueError("Input weight matrix contains non-finite values (NaN or Inf)")
    w32 = arr.astype(np.float32)
    n, k = w32.shape
    if k % GROUP:
        raise ValueError(f"Columns/in-features ({k}) must be a multiple of GROUP ({GROUP})")
    grouped = w32.reshape(n, k // GROUP, GROUP)
    lo = grouped.min(axis=2)
    hi = grouped.max(axis=2).astype(np.float64)

    min_q = np.asarray(bf16_floor(lo), dtype=np.float32)
    base = min_q.astype(np.float64)
    span = hi - base
    scale_q = np.asarray(bf16_ceil(span / 15.0), dtype=np.float32)
    for _ in range(64):
        short = base + 15.0 * scale_q.astype(np.float64) < hi
        if not short.any() or not np.isfinite(scale_q).all():
            break
        scale_q = np.where(short, bf16_next_up(scale_q), scale_q).astype(np.float32)
    flat = span == 0.0
    scale_q = np.where(flat, np.float32(0.0), scale_q).astype(np.float32)
    if not (np.isfinite(min_q).all() and np.isfinite(scale_q).all()):
        raise ValueError("Quantization parameters (scale_q or min_q) overflowed to non-finite values")

    divisor = np.where(flat, 1.0, scale_q.astype(np.float64))[..., None]
    q = np.rint((grouped.astype(np.float64) - base[..., None]) / divisor)
    codes = np.clip(q, 0, 15).astype(np.uint8)
    codes[np.broadcast_to(flat[..., None], codes.shape)] = 0
    return codes.reshape(n, k), scale_q, min_q


def dequantize_simple(codes, scales, mins) -> np.ndarray:
    """``f32(f64(min) + f64(scale) * code)`` per element (``quant/q4nx.py:203-223``)."""
    c = np.asarray(codes)
    g = np.arange(c.shape[1]) // GROUP
    s = np.asarray(scales, dtype=np.float32)[:, g].astype(np.float64)
    m = np.asarray(mins, dtype=np.float32)[:, g].astype(np.float64)
    return (m + s * c.astype(np.float64)).astype(np.float32)


def pad_gemv(w: np.ndarray, m_align: int = 128, k_align: int = 256):
    """Zero-pad rows/cols up to the alignments (``quant/q4nx.py:226-248,441-455``)."""
    if w.ndim != 2:
        raise ValueError(f"pad requires 2D array, got shape {w.shape}")
    r, c = w.shape
    pr, pc = (-r) % m_align, (-c) % k_align
    if pr == 0 and pc == 0:
        return w.copy(), (r, c)
    return np.pad(w, ((0, pr), (0, pc))), (r, c)


# ------------------------------------------------------------------ packing --
def _nibble_order(codes_blocks: np.ndarray) -> np.ndarray:
    """[..., 32 rows, 256 cols] codes -> [..., 4096] packed bytes in block order.

    In-block byte for row r (h = r // 16, rr = r % 16) and column k
    (g = k // 32, c = k % 32) is ``((h*8 + g)*32 + c)*8 + rr//2``; even rr is
    the low nibble (``quant/q4nx.py:384-390``).
    """
    lead = codes_blocks.shape[:-2]
    c = codes_blocks.reshape(*lead, 2, 16, K_TILE)          # h, rr, k
    c = np.moveaxis(c, -2, -1)                               # h, k, rr
    c = c.reshape(*lead, 2 * K_TILE, 8, 2)                   # (h,k), rr//2, rr%2
    return (c[..., 0] | (c[..., 1] << 4)).astype(np.uint8).reshape(*lead, 4096)


def _param_bytes(scales_blocks: np.ndarray, mins_blocks: np.ndarray) -> np.ndarray:
    """[..., 32 rows, 8 groups] scales/mins -> [..., 1024] bytes ([s|m][g][r] bf16)."""
    s = np.swapaxes(f32_to_bf16(scales_blocks), -1, -2)
    m = np.swapaxes(f32_to_bf16(mins_blocks), -1, -2)
    both = np.stack([s, m], axis=-3)                         # [..., 2, 8, 32]
    lead = both.shape[:-3]
    return np.ascontiguousarray(both).view(np.uint8).reshape(*lead, PARAM_BYTES)


def pack_gemv(codes, scales, mins, rows: int = 4) -> bytes:
    """The GEMV byte layout of ``quant/q4nx.py:335-393``.

    A slice is ``rows * 32`` output rows; blocks are ordered
    ``(slice * k_blocks + k) * rows + row``.  With ``rows=2`` this is also the
    ``pack_decode_proj`` layout (``quant/q4nx.py:257-297``).
    """
    codes = np.asarray(codes, dtype=np.uint8)
    m, k = codes.shape
    band = rows * M_TILE
    if m % band:
        raise ValueError(f"M ({m}) must be a multiple of {band} (rows={rows} * M_TILE={M_TILE})")
    if k % K_TILE:
        raise ValueError(f"K ({k}) must be a multiple of K_TILE ({K_TILE})")
    kb = k // K_TILE
    nslice = m // band
    # [slice, row, 32, kb, 256] -> [slice, kb, row, 32, 256]
    cb = codes.reshape(nslice, rows, M_TILE, kb, K_TILE).transpose(0, 3, 1, 2, 4)
    sb = np.asarray(scales, np.float32).reshape(nslice, rows, M_TILE, kb, 8).transpose(0, 3, 1, 2, 4)
    mb = np.asarray(mins, np.float32).reshape(nslice, rows, M_TILE, kb, 8).transpose(0, 3, 1, 2, 4)
    blocks = np.concatenate([_param_bytes(sb, mb), _nibble_order(cb)], axis=-1)
    return blocks.reshape(-1).tobytes()


def parse_gemv(buf, K: int, M: int, rows: int = 4):
    """Inverse of ``pack_gemv`` (``quant/q4nx.py:396-438``)."""
    raw = np.frombuffer(buf, dtype=np.uint8) if isinstance(buf, (bytes, bytearray)) else np.asarray(buf, np.uint8)
    kb = K // K_TILE
    nslice = M // (rows * M_TILE)
    blocks = raw[: nslice * kb * rows * BLOCK_BYTES].reshape(nslice, kb, rows, BLOCK_BYTES)
    params = bf16_to_f32(blocks[..., :PARAM_BYTES].copy().view("<u2").reshape(nslice, kb, rows, 2, 8, M_TILE))
    # [slice, kb, row, 8, 32] -> [slice, row, 32, kb, 8]
    scales = params[..., 0, :, :].transpose(0, 2, 4, 1, 3).reshape(M, K // GROUP)
    mins = params[..., 1, :, :].transpose(0, 2, 4, 1, 3).reshape(M, K // GROUP)
    nib = blocks[..., PARAM_BYTES:]
    pairs = np.stack([nib & 0x0F, nib >> 4], axis=-1).reshape(nslice, kb, rows, 2, K_TILE, 16)
    # [slice, kb, row, h, k, rr] -> [slice, row, h, rr, kb, k]
    codes = pairs.transpose(0, 2, 3, 5, 1, 4).reshape(M, K)
    return np.ascontiguousarray(codes), np.ascontiguousarray(scales), np.ascontiguousarray(mins)


def pack_decode_proj(codes, scales, mins) -> bytes:
    """``quant/q4nx.py:257-297``: pairs of 32-row bands -- identical to ``pack_gemv(rows=2)``."""
    codes = np.asarray(codes)
    if codes.shape[0] % (2 * M_TILE):
        raise ValueError(f"rows ({codes.shape[0]}) must be a multiple of 64 for decode projection packing")
    if codes.shape[1] % K_TILE:
        raise ValueError(f"cols ({codes.shape[1]}) must be a multiple of {K_TILE} (256)")
    return pack_gemv(codes, scales, mins, rows=2)


def packed_bytes(n: int, k: int) -> int:
    """Size of an n x k pack_gemv buffer."""
    return n * k * 5 // 8


def quantize_pack(w: np.ndarray):
    """quantize + pack_gemv; returns (packed bytes, codes, scales, mins)."""
    codes, scales, mins = quantize(w)
    return pack_gemv(codes, scales, mins), codes, scales, mins


def normal_weight_q4nx(n: int, k: int, seed: int, std: float = 0.02, chunk_rows: int = 8192):
    """Seeded ``N(0, std)`` f32 [n, k] weights, quantised and packed in row chunks.

    Draws the same numbers as one ``default_rng(seed).standard_normal((n, k))``
    call (the generator is consumed sequentially) but bounds host memory; since
    ``pack_gemv`` orders blocks slice-major, packing 128-row-aligned chunks and
    concatenating equals packing the whole matrix.  Returns
    (packed bytes, codes, scales, mins).
    """
    assert chunk_rows % 128 == 0
    rng = np.random.default_rng(seed)
    parts, cs, ss, ms = [], [], [], []
    for r0 in range(0, n, chunk_rows):
        rows = min(chunk_rows, n - r0)
        w = (rng.standard_normal((rows, k)) * std).astype(np.float32)
        c, s, m = quantize(w)
        parts.append(pack_gemv(c, s, m))
        cs.append(c)
        ss.append(s)
        ms.append(m)
    return b"".join(parts), np.concatenate(cs), np.concatenate(ss), np.concatenate(ms)


def dequantize_packed(buf, n: int, k: int) -> np.ndarray:
    """parse_gemv + dequantize_simple: the f32 weights the CPU path multiplies by."""
    return dequantize_simple(*parse_gemv(buf, K=k, M=n))
