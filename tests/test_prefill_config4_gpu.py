"""MoE prefill at BASELINE config 4's own shape, every token against the oracle.

Layer: hidden 2048, 128 routed experts + 1 shared, intermediate 768, softmax
top-8 of the logits plus a per-expert bias ``b_e = -1.1 ln(rank_e)`` (rank: a
seeded permutation of 1..128, so the expert load follows Zipf(1.1)), SwiGLU,
q4nx weights N(0, 0.02) quantised on the device.  Token counts: the 512 of
config 4 and the reference's grouped-parity counts T in {1, 7, 8, 9, 16, 17,
64} (``host/test_prefill_grouped_parity.py:27-40``), through both prefill
kernels, and a layer of the same shape whose down matrices are bfp16ebs8.

Oracle: ``NumpyBackend.moe_experts`` semantics (``host/backend.py:466-510``)
with the shared expert added as ``_moe_token`` does (``host/raon.py:1321-1327``),
computed expert by expert over the tokens routed to it (the bf16 roundings of
gate, up, activation and down of every token, then the ascending-ID f32
combine of each token).  Its f32 weights are the device dequantiser's output,
which is checked bit for bit against the oracle's own dequantiser on two
experts here (and on other shapes in test_gemv_gpu.py): dequantising all 129
experts with the numpy restatement would take over a minute of host time.
Bars: the selected ids bit-exact; the MoE output bars of
``tests.test_moe_gpu`` on every token (per element one bf16 step of its
terms' magnitude plus either side's last rounding, row RMS relative error
<= 4e-3, normwise max error <= 2^-6) and RMS relative error <= 2e-3 over
the call.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import backend as ob
from oracle import bfp16 as ob16
from oracle import q4nx as q
from tests.test_moe_gpu import _config3_layer, assert_bf16_outputs_close, assert_call_rms

pytestmark = pytest.mark.gpu

H, I, E, K = 2048, 768, 128, 8
T_CONFIG4 = 512
T_GROUPED = (1, 7, 8, 9, 16, 17, 64)


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


def zipf_bias(seed: int) -> np.ndarray:
    rank = np.random.default_rng(seed).permutation(E) + 1
    return (-1.1 * np.log(rank)).astype(np.float32)


def _dequant(ctx, torch, packed_dev, n, k):
    """f32 weights of pack_gemv bytes on the device (rc_dequant_q4nx)."""
    w = ctx.upload_q4nx(packed_dev, n, k)
    out = torch.empty((n, k), dtype=torch.float32, device="cuda")
    w.dequant_into(out)
    torch.cuda.synchronize()
    w.free()
    return out.cpu().numpy()


@pytest.fixture(scope="module")
def c4(torch, ctx):
    layer, wr, packed = _config3_layer(torch, ctx, n_experts=E, seed=410)
    bias = zipf_bias(411)
    layer.set_router(wr, bias)
    weights = {}
    for e in range(E + 1):
        pgu, pdn = packed[e]
        fgu = _dequant(ctx, torch, pgu, 2 * I, H)
        weights[e] = (fgu[:I], fgu[I:], _dequant(ctx, torch, pdn, H, I))
    for e in (0, E):   # the device dequantiser is the oracle's, bit for bit
        pgu, pdn = (t.cpu().numpy() for t in packed[e])
        np.testing.assert_array_equal(q.dequantize_packed(pgu, 2 * I, H), np.concatenate(weights[e][:2]))
        np.testing.assert_array_equal(q.dequantize_packed(pdn, H, I), weights[e][2])
    yield layer, wr, bias, weights, packed
    layer.close()


def oracle_layer(x, wr, bias, weights, k=K, act="swiglu"):
    """(out [T, H] bf16, ids [T, k] in router order, term magnitudes [T, H])."""
    T = x.shape[0]
    logits = (ob.router_logits(x, wr) + bias).astype(np.float32)
    ids = np.stack([ob.topk_lower_index_wins(logits[t], k) for t in range(T)])
    sel = np.take_along_axis(logits, ids, axis=1).astype(np.float64)
    ex = np.exp(sel - sel.max(axis=1, keepdims=True))
    w = (ex / ex.sum(axis=1, keepdims=True)).astype(np.float32)
    rows = {}
    for e in np.unique(ids):
        toks = np.nonzero((ids == e).any(axis=1))[0]
        wg, wu, wd = weights[int(e)]
        xs = x[toks]
        a = q.f32_to_bf16(ob.glu(ob.linear(wg, xs), ob.linear(wu, xs), act))
        d = ob.linear(wd, a)
        for j, t in enumerate(toks):
            rows[(int(t), int(e))] = d[j]
    wg, wu, wd = weights[E]
    shared = ob.linear(wd, q.f32_to_bf16(ob.glu(ob.linear(wg, x), ob.linear(wu, x), act)))
    out = np.empty((T, H), np.uint16)
    mag = np.empty((T, H), np.float64)
    for t in range(T):
        acc = np.zeros(H, np.float32)
        m = np.abs(q.bf16_to_f32(shared[t]).astype(np.float64))
        for r in np.argsort(ids[t], kind="stable"):       # ascending expert ID
            row = q.bf16_to_f32(rows[(t, int(ids[t, r]))])
            acc += row * np.float32(w[t, r])
            m = m + np.abs(row.astype(np.float64) * w[t, r])
        out[t] = ob.moe_token_with_shared(q.f32_to_bf16(acc), shared[t])
        mag[t] = m
    return out, ids, mag


def _run_prefill(torch, ctx, layer, x):
    T = x.shape[0]
    xd = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).cuda()
    out = torch.empty((T, H), dtype=torch.int16, device="cuda")
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    layer.prefill(xd, K, out, ids, act="swiglu")
    torch.cuda.synchronize()
    ctx.sync()
    return out.cpu().numpy().view(np.uint16), ids.cpu().numpy()


def _check_all_tokens(got, ids, ref, r_ids, mag):
    np.testing.assert_array_equal(ids, r_ids)
    for t in range(got.shape[0]):
        assert_bf16_outputs_close(got[t], ref[t], mag[t])
    assert_call_rms(got, ref)


@pytest.mark.parametrize("kernel", ["gemv", "tcgen05"])
@pytest.mark.parametrize("T", (T_CONFIG4,) + T_GROUPED)
def test_config4_prefill_every_token_matches_oracle(torch, ctx, c4, kernel, T):
    layer, wr, bias, weights, _ = c4
    layer.set_prefill_kernel(kernel)
    x = q.f32_to_bf16(np.random.default_rng(420 + T).standard_normal((T, H)).astype(np.float32))
    got, ids = _run_prefill(torch, ctx, layer, x)
    ref, r_ids, mag = oracle_layer(x, wr, bias, weights)
    _check_all_tokens(got, ids, ref, r_ids, mag)
    if T == T_CONFIG4:
        # the load is skewed as config 4 intends: the busiest expert takes many
        # times its even share of the 4096 routed rows
        counts = np.bincount(ids.ravel(), minlength=E)
        assert counts.max() >= 4 * (T * K // E)


def test_config4_prefill_bfp16_down_every_token_matches_oracle(torch, ctx, c4):
    """The same layer with bfp16ebs8 down matrices (the reference's moe_b2
    expert bundles): synthetic exponents 120..122 and int8 mantissas, packed by
    the oracle's GEMV packing, decoded by the oracle to the f32 weights."""
    from raon_npu_b200.device import MoeLayer
    _, wr, bias, weights, packed = c4
    rng = np.random.default_rng(430)
    layer = MoeLayer(ctx, H, I, E, has_shared=True)
    bf_weights = {}
    for e in range(E + 1):
        ex = rng.integers(120, 123, (H, I // 8)).astype(np.uint8)
        mt = rng.integers(-128, 128, (H, I)).astype(np.int8)
        layer.set_expert(e, packed[e][0].cpu().numpy(), np.frombuffer(ob16.pack_gemv_raw(ex, mt), np.uint8),
                         down_format="bfp16")
        bf_weights[e] = (weights[e][0], weights[e][1], ob16.gemv_weights(ex, mt))
    layer.set_router(wr, bias)
    for T in (17, T_CONFIG4):
        x = q.f32_to_bf16(np.random.default_rng(440 + T).standard_normal((T, H)).astype(np.float32))
        got, ids = _run_prefill(torch, ctx, layer, x)
        ref, r_ids, mag = oracle_layer(x, wr, bias, bf_weights)
        _check_all_tokens(got, ids, ref, r_ids, mag)
    layer.close()


def test_config4_prefill_equals_decode_bytes(torch, ctx, c4):
    """The register-fragment prefill kernel runs the decode GEMV's unit arithmetic on the
    same per-token staging: at config 4's shape its bytes are the decode
    path's (16 tokens per decode call)."""
    layer = c4[0]
    layer.set_prefill_kernel("gemv")
    T = 64
    x = q.f32_to_bf16(np.random.default_rng(450).standard_normal((T, H)).astype(np.float32))
    got, _ = _run_prefill(torch, ctx, layer, x)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    dec = torch.empty((T, H), dtype=torch.int16, device="cuda")
    for t0 in range(0, T, 16):
        layer.decode(xd[t0:t0 + 16], K, dec[t0:t0 + 16], act="swiglu")
    torch.cuda.synchronize()
    ctx.sync()
    np.testing.assert_array_equal(dec.cpu().numpy().view(np.uint16), got)
