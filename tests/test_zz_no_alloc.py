"""The allocation-free GEMV entry point, ``rc_gemv_noalloc``.

Some callers must not allocate device memory while they run a GEMV: a
latency-critical serving thread cannot afford the device-wide synchronisation
that cudaMalloc/cudaFree may imply, and a host that reserved a fixed device
memory budget at start-up forbids later allocations.  ``rc_gemv`` may grow its
scratch on first use of a larger shape; ``rc_gemv_noalloc`` instead keeps its
split-K scratch in one static device array.  These tests call it through the
C ABI twice in a row and check each result against ``rc_gemv`` on the same
inputs, with the tolerance the other GEMV tests use.

This file is named to be collected last, so that a run stopping at its first
failure has already run every other test; it creates its own context and
weights, so it passes alone in a fresh process as well as after the others.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import q4nx as q

pytestmark = pytest.mark.gpu

REL_TOL = 2e-3   # as tests/test_gemv_gpu.py: normwise, on the f32 sums


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
    return ctx.upload_q4nx(q.quantize_pack(w)[0], n, k)


def _stream(torch) -> int:
    h = int(torch.cuda.current_stream().cuda_stream)
    return h if h else 1   # cudaStreamLegacy for torch's default stream


def _call_noalloc(ctx, torch, wt, x, y, y_dtype):
    """rc_gemv_noalloc through the C ABI (no Python wrapper in between)."""
    status = ctx.lib.rc_gemv_noalloc(
        wt.handle, ctypes.c_void_p(x.data_ptr()), 0, wt.k, x.shape[0], ctypes.c_void_p(y.data_ptr()),
        int(y_dtype), wt.n, 0, wt.n, None, ctypes.c_void_p(_stream(torch)))
    from raon_npu_b200._lib import check
    check(status, "rc_gemv_noalloc")


def _rel(a, b):
    return float(np.max(np.abs(a.astype(np.float64) - b)) / max(np.max(np.abs(b)), 1e-30))


def _ulp(a, b):
    def key(u):
        u = u.astype(np.int32)
        return np.where(u & 0x8000, -(u & 0x7FFF), u & 0x7FFF)
    return np.abs(key(a) - key(b))


# (4096, 2048): whole-tile CTA partition; (2560, 4096): stream-K partition,
# whose split tiles reduce through the static scratch's counters and partials.
@pytest.mark.parametrize("n,k,t", [(4096, 2048, 3), (2560, 4096, 5), (151936, 2048, 1)])
def test_noalloc_matches_rc_gemv_twice_in_a_row(torch, ctx, n, k, t):
    wt = _weight(ctx, n, k, seed=n + k)
    xh = q.f32_to_bf16(np.random.default_rng(t).standard_normal((t, k)).astype(np.float32))
    x = torch.from_numpy(xh.view(np.int16)).cuda()

    ref16 = torch.empty((t, n), dtype=torch.int16, device="cuda")
    ref32 = torch.empty((t, n), dtype=torch.float32, device="cuda")
    wt.gemv_into(x, ref16, t)
    wt.gemv_into(x, ref32, t, y_dtype=1)
    torch.cuda.synchronize()
    ctx.sync()
    r16 = ref16.cpu().numpy().view(np.uint16)
    r32 = ref32.cpu().numpy()

    for _ in range(2):
        y16 = torch.full((t, n), -1, dtype=torch.int16, device="cuda")
        y32 = torch.full((t, n), float("nan"), dtype=torch.float32, device="cuda")
        _call_noalloc(ctx, torch, wt, x, y16, 0)
        _call_noalloc(ctx, torch, wt, x, y32, 1)
        torch.cuda.synchronize()
        ctx.sync()
        g32 = y32.cpu().numpy()
        g16 = y16.cpu().numpy().view(np.uint16)
        assert np.isfinite(g32).all()
        assert _rel(g32, r32) <= REL_TOL
        d = _ulp(g16, r16)
        assert d.max() <= 1 and np.count_nonzero(d) <= max(2, d.size // 100)
    wt.free()


def test_noalloc_rejects_inputs_beyond_its_static_limits(torch, ctx):
    # K = 6144 cannot stage 16 bf16 rows in shared memory: a clear ValueError,
    # no launch, and the entry point stays usable for a supported call after it.
    wt = _weight(ctx, 128, 6144, seed=3)
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
