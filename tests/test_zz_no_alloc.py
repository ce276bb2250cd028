"""The allocation-free GEMV entry point, ``rc_gemv_noalloc``.

Some callers must not allocate device memory while they run a GEMV: a
latency-critical serving thread cannot afford the device-wide synchronisation
that cudaMalloc/cudaFree may imply, and a host that reserved a fixed device
memory budget at start-up forbids later allocations.  ``rc_gemv`` may grow its
scratch on first use of a larger shape; ``rc_gemv_noalloc`` instead keeps its
split-K scratch in one static device array.  These tests call it through the
C ABI twice in a row and check each result against ``rc_gemv`` on the same
inputs -- bit for bit, since both run the same kernel with the same partition
-- and the f32 sums against the CPU oracle within the GEMV tolerance.

This file is named to be collected last, so that a run stopping at its first
failure has already run every other test; it creates its own context and
weights, so it passes alone in a fresh process as well as after the others.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import backend as ob
from oracle import q4nx as q

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3   # the north star's bar for the GEMV against the oracle (normwise, f32 sums)


@pytest.fixture(scope="module")
def torch():
    import torch as _t
    return _t


@pytest.fixture(scope="module")
def ctx():
    from raon_npu_b200.build import build
    build()
    from raon_npu_b200.device import Context
    c = Context(0)
    yield c
    c.close()


def _weight(ctx, n, k, seed):
    w = (np.random.default_rng(seed).standard_normal((n, k)) * 0.02).astype(np.float32)
    packed, codes, scales, mins = q.quantize_pack(w)
    return ctx.upload_q4nx(packed, n, k), q.dequantize_simple(codes, scales, mins)


def _stream(torch) -> int:
    h = int(torch.cuda.current_stream().cuda_stream)
    return h if h else 1   # cudaStreamLegacy for torch's default stream


def _call_noalloc(ctx, torch, wt, x, y, y_dtype, x_dtype=0, row0=0, nrows=None, bias=None):
    """rc_gemv_noalloc through the C ABI (no Python wrapper in between)."""
    nrows = wt.n if nrows is None else nrows
    status = ctx.lib.rc_gemv_noalloc(
        wt.handle, ctypes.c_void_p(x.data_ptr()), int(x_dtype), wt.k, x.shape[0], ctypes.c_void_p(y.data_ptr()),
        int(y_dtype), nrows, int(row0), int(nrows), ctypes.c_void_p(None if bias is None else bias.data_ptr()),
        ctypes.c_void_p(_stream(torch)))
    from raon_npu_b200._lib import check
    check(status, "rc_gemv_noalloc")


# (4096, 2048): whole-tile CTA partition; (2560, 4096): stream-K partition,
# whose split tiles reduce through the static scratch's counters and partials;
# the lm-head shape: the most tiles; T = 20: two launches (16 + 4 rows), each
# clearing the shared counters.
CASES = [
    dict(n=4096, k=2048, t=3),
    dict(n=2560, k=4096, t=5),
    dict(n=151936, k=2048, t=1),
    dict(n=2048, k=2048, t=20),
    dict(n=2560, k=4096, t=9, x_dtype=1),                          # f32 rows: two slots per row
    dict(n=4096, k=2048, t=4, row0=1024, nrows=512, bias=True),    # a row slice with its bias
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "-".join(f"{k}{v}" for k, v in c.items()))
def test_noalloc_matches_rc_gemv_twice_in_a_row(torch, ctx, case):
    """Both entry points run the same kernel with the same T-independent
    partition, so the results must be identical to the bit, on every call."""
    n, k, t = case["n"], case["k"], case["t"]
    x_dtype = case.get("x_dtype", 0)
    row0, nrows = case.get("row0", 0), case.get("nrows", n)
    wt, w32 = _weight(ctx, n, k, seed=n + k)
    rng = np.random.default_rng(t)
    xf = rng.standard_normal((t, k)).astype(np.float32)
    xh = xf if x_dtype else q.f32_to_bf16(xf)
    x = torch.from_numpy(xh if x_dtype else xh.view(np.int16)).cuda()
    bias = None
    if case.get("bias"):
        bias = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda()
    out_dtypes = (1,) if x_dtype else (0, 1)
    ref = {}
    for yd in out_dtypes:
        r = torch.empty((t, nrows), dtype=torch.float32 if yd else torch.int16, device="cuda")
        wt.gemv_into(x, r, t, x_dtype=x_dtype, row0=row0, nrows=nrows, bias_dev=bias, y_dtype=yd)
        ref[yd] = r
    torch.cuda.synchronize()
    ctx.sync()
    ref = {yd: r.cpu().numpy() for yd, r in ref.items()}

    # the f32 sums against the oracle (NumpyBackend.linear's f32 dot, before rounding)
    b = None if bias is None else bias.cpu().numpy()[row0:row0 + nrows]
    oracle = ob.linear_f32(w32[row0:row0 + nrows], xh, b)
    err = np.max(np.abs(ref[1].astype(np.float64) - oracle)) / np.max(np.abs(oracle))
    assert err <= REL_TOL, err

    for _ in range(2):
        for yd in out_dtypes:
            y = torch.full((t, nrows), -1, dtype=torch.float32 if yd else torch.int16, device="cuda")
            _call_noalloc(ctx, torch, wt, x, y, yd, x_dtype=x_dtype, row0=row0, nrows=nrows, bias=bias)
            torch.cuda.synchronize()
            ctx.sync()
            got = y.cpu().numpy()
            assert np.array_equal(got.view(np.uint32 if yd else np.uint16), ref[yd].view(np.uint32 if yd else
                                                                                         np.uint16)), \
                (yd, int(np.count_nonzero(got != ref[yd])))
    wt.free()


def test_noalloc_rejects_inputs_beyond_its_static_limits(torch, ctx):
    # K = 6144 cannot stage 16 bf16 rows in shared memory: a clear ValueError,
    # no launch, and the entry point stays usable for a supported call after it.
    wt, _ = _weight(ctx, 128, 6144, seed=3)
    x = torch.zeros((16, 6144), dtype=torch.int16, device="cuda")
    y = torch.empty((16, 128), dtype=torch.int16, device="cuda")
    with pytest.raises(ValueError, match="shared memory"):
        _call_noalloc(ctx, torch, wt, x, y, 0)
    # Eight rows fit at this K.
    _call_noalloc(ctx, torch, wt, x[:8], y[:8], 0)
    torch.cuda.synchronize()
    ctx.sync()
    assert (y[:8].cpu().numpy() == 0).all()   # x = 0 -> y = 0
    wt.free()
