"""GPU parity of the bfp16ebs8 GEMV (``rc_upload_bfp16`` + ``rc_gemv``)
against the reference's own outputs and the oracle.

Bar: every product of an int8 mantissa, its group's power-of-two scale and a
bf16 activation is exact, so the f32 result differs from the exact sum only by
f32 summation rounding: |y_f32 - y_exact| <= K * 2^-23 * sum |w x| per output.
The bf16 output must equal RTNE of the kernel's f32 output bit for bit, and
differ from the reference's bf16 output (``kernels/gemv_bfp16/reference.py``
``bfp16_gemv_bit_reference``: the same products summed in column order) by at
most 1 ulp, on at most 1 % of the outputs (only the summation order differs).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import bfp16 as b
from tests.golden.cases import BFP16_CASES, bfp16_input

pytestmark = pytest.mark.gpu
GOLD = np.load(Path(__file__).parent / "golden" / "bfp16.npz")


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


def _ulp(a, c):
    def key(u):
        u = u.astype(np.int32)
        return np.where(u & 0x8000, -(u & 0x7FFF), u & 0x7FFF)
    return np.abs(key(a) - key(c))


def _run(torch, ctx, w, x_bits, row0=0, nrows=None, bias=None):
    """(bf16 bits [T, nrows], f32 [T, nrows]) of rows [row0, row0+nrows)."""
    n, k = w.shape
    nrows = n if nrows is None else nrows
    wt = ctx.upload_bfp16(np.frombuffer(b.pack_gemv(w), np.uint8), n, k)
    bias_dev = wt.set_bias(bias) if bias is not None else 0
    x = torch.from_numpy(np.ascontiguousarray(x_bits).view(np.int16)).cuda()
    T = x.shape[0]
    y16 = torch.empty((T, nrows), dtype=torch.int16, device="cuda")
    y32 = torch.empty((T, nrows), dtype=torch.float32, device="cuda")
    import ctypes
    from raon_npu_b200._lib import check, RC_DTYPE_BF16, RC_DTYPE_F32
    for y, dt in ((y16, RC_DTYPE_BF16), (y32, RC_DTYPE_F32)):
        check(ctx.lib.rc_gemv(ctx.handle, wt.handle, ctypes.c_void_p(x.data_ptr()), RC_DTYPE_BF16, k, T,
                              ctypes.c_void_p(y.data_ptr()), dt, nrows, row0, nrows,
                              ctypes.c_void_p(bias_dev if bias_dev else None), None))
    torch.cuda.synchronize()
    ctx.sync()
    out = y16.cpu().numpy().view(np.uint16), y32.cpu().numpy()
    wt.free()
    return out


def _check(y16, y32, w, x_bits, row0, nrows, bias=None, ref16=None):
    e, m = b.parse_gemv(b.pack_gemv(w), K=w.shape[1], M=w.shape[0])
    wx = b.gemv_weights(e, m).astype(np.float64)[row0:row0 + nrows]
    xf = (x_bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    exact = xf @ wx.T
    mag = np.abs(xf) @ np.abs(wx).T
    if bias is not None:
        exact = exact + bias[row0:row0 + nrows]
        mag = mag + np.abs(bias[row0:row0 + nrows])
    bound = w.shape[1] * 2.0 ** -23 * mag + 1e-30
    assert (np.abs(y32 - exact) <= bound).all(), np.max(np.abs(y32 - exact) / bound)
    # bf16 output = RTNE of the f32 output
    u = y32.astype(np.float32).view(np.uint32).astype(np.uint64)
    np.testing.assert_array_equal(y16, (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16))
    if ref16 is not None:
        d = _ulp(y16, ref16)
        assert d.max() <= 1 and np.count_nonzero(d) <= max(1, y16.size // 100), (d.max(), np.count_nonzero(d))


@pytest.mark.parametrize("name", list(BFP16_CASES))
def test_reference_fixtures(torch, ctx, name):
    n, k, seed, kind, t = BFP16_CASES[name]
    w, x = bfp16_input(n, k, seed, kind, t)
    y16, y32 = _run(torch, ctx, w, x)
    _check(y16, y32, w, x, 0, n, ref16=GOLD[f"{name}/y"])


@pytest.mark.parametrize("n,k,T", [(2048, 4096, 1), (2048, 4096, 3), (4096, 2048, 8), (256, 2048, 16),
                                   (40960, 256, 2), (1024, 1280, 5)])
def test_shapes_against_oracle(torch, ctx, n, k, T):
    rng = np.random.default_rng(n + k + T)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    xf = rng.standard_normal((T, k)).astype(np.float32)
    u = xf.view(np.uint32).astype(np.uint64)
    x = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)
    y16, y32 = _run(torch, ctx, w, x)
    e, m = b.parse_gemv(b.pack_gemv(w), K=k, M=n)
    rows = np.random.default_rng(0).choice(n, size=min(n, 256), replace=False)
    ref = np.stack([b.gemv(e[rows], m[rows], x[t]) for t in range(T)])
    _check(y16, y32, w, x, 0, n)
    d = _ulp(y16[:, rows], ref)
    assert d.max() <= 1 and np.count_nonzero(d) <= max(1, d.size // 100)


def test_row_range_bias_and_repeat(torch, ctx):
    rng = np.random.default_rng(7)
    n, k, T = 1024, 1024, 4
    w = (rng.standard_normal((n, k)) * np.exp2(rng.integers(-6, 3, (n, 1)))).astype(np.float32)
    xf = rng.standard_normal((T, k)).astype(np.float32)
    u = xf.view(np.uint32).astype(np.uint64)
    x = (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)
    bias = rng.standard_normal(n).astype(np.float32)
    a16, a32 = _run(torch, ctx, w, x, row0=272, nrows=480, bias=bias)
    _check(a16, a32, w, x, 272, 480, bias=bias)
    c16, c32 = _run(torch, ctx, w, x, row0=272, nrows=480, bias=bias)
    np.testing.assert_array_equal(a16, c16)
    np.testing.assert_array_equal(a32, c32)


def test_rejects_what_it_does_not_compute(torch, ctx):
    import ctypes
    from raon_npu_b200._lib import RC_DTYPE_F32, RC_ERR_INVALID
    w = (np.random.default_rng(3).standard_normal((128, 256)) * 0.02).astype(np.float32)
    wt = ctx.upload_bfp16(np.frombuffer(b.pack_gemv(w), np.uint8), 128, 256)
    x = torch.zeros((1, 256), dtype=torch.float32, device="cuda")
    y = torch.zeros((1, 128), dtype=torch.float32, device="cuda")
    rc = ctx.lib.rc_gemv(ctx.handle, wt.handle, ctypes.c_void_p(x.data_ptr()), RC_DTYPE_F32, 256, 1,
                         ctypes.c_void_p(y.data_ptr()), RC_DTYPE_F32, 128, 0, 128, None, None)
    assert rc == RC_ERR_INVALID
    rc = ctx.lib.rc_dequant_q4nx(ctx.handle, wt.handle, ctypes.c_void_p(y.data_ptr()), None)
    assert rc == RC_ERR_INVALID
    with pytest.raises(ValueError):
        ctx.upload_bfp16(np.zeros(100, np.uint8), 128, 256)
    wt.free()
