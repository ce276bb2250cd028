"""GPU parity of the MoE prefill path (tcgen05 grouped GEMM) against the
oracle, the decode path and itself.

Bars: routing bit-exact (the decode router's ids); outputs against the oracle
with the MoE bars of tests/test_moe_gpu.py (per element one bf16 step of each
accumulated term plus either side's last rounding, row RMS relative error
<= 4e-3, call RMS <= 2e-3).
Bit-exact properties: a token's bytes do not depend on the other tokens of
the call (columns of the tensor-core GEMM do not interact), caller-supplied
routes reproduce the routed call, and the expert-parallel halves summed over
ranks reproduce the single-GPU bytes.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import backend as ob
from oracle import q4nx as q
from tests.golden import cases
from tests.test_moe_gpu import _config3_layer, _oracle_expert, assert_bf16_outputs_close, assert_call_rms, rms_rel

pytestmark = pytest.mark.gpu


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


def _dev(torch, a, dtype):
    return torch.from_numpy(np.ascontiguousarray(a).view(dtype)).cuda()


def _oracle_token(experts, shared, wr, x, k, act, bias=None):
    """Oracle layer output of one token (router with optional logit bias)."""
    logits = ob.router_logits(x, wr)
    if bias is not None:
        logits = (logits + bias).astype(np.float32)
    ids = ob.topk_lower_index_wins(logits, k)
    sel = logits[ids].astype(np.float64)
    e = np.exp(sel - sel.max())
    w = (e / e.sum()).astype(np.float32)
    ex = {int(i): experts(int(i)) for i in ids}
    routed = ob.moe_experts(ex, x, ids, w, act=act)
    out = routed
    mag = ob.moe_term_magnitude(ex, x, ids, w, act)
    if shared is not None:
        sh = ob.expert_forward(*shared, x, act)
        out = ob.moe_token_with_shared(routed, sh)
        mag = ob.moe_term_magnitude(ex, x, ids, w, act, shared_down_u16=sh)
    return out, ids, mag


KERNELS = ["gemv", "tcgen05"]


@pytest.mark.parametrize("kernel", KERNELS)
def test_prefill_small_layer_matches_oracle(torch, ctx, kernel):
    """hidden 256, intermediate 256, 6 experts + shared, top-3, SiTU, T = 37."""
    from raon_npu_b200.device import MoeLayer
    d = cases.moe_inputs(hidden=256, inter=256, experts=7, k=3, tokens=37, seed=201)
    layer = MoeLayer(ctx, 256, 256, 6, has_shared=True)
    layer.set_prefill_kernel(kernel)
    for e, (pgu, pdn) in d["packed"].items():
        layer.set_expert(e, pgu, pdn)            # expert 6 is the shared one
    rng = np.random.default_rng(202)
    wr = q.f32_to_bf16((rng.standard_normal((6, 256)) * 0.05).astype(np.float32))
    layer.set_router(wr)
    x = d["x"]
    out = torch.empty((37, 256), dtype=torch.int16, device="cuda")
    ids = torch.empty((37, 3), dtype=torch.int32, device="cuda")
    layer.prefill(_dev(torch, x, np.int16), 3, out, ids, act="situ")
    torch.cuda.synchronize()
    ctx.sync()
    got = out.cpu().numpy().view(np.uint16)
    refs = []
    for t in range(37):
        ref, r_ids, mag = _oracle_token(lambda e: d["experts"][e], d["experts"][6], wr, x[t], 3, "situ")
        np.testing.assert_array_equal(ids[t].cpu().numpy(), r_ids)
        assert_bf16_outputs_close(got[t], ref, mag)
        refs.append(ref)
    assert_call_rms(got, np.stack(refs))
    layer.close()


@pytest.fixture(scope="module")
def c4(torch, ctx):
    """Config-4 shapes with 32 experts: hidden 2048, I = 768, top-8, plus a
    per-expert logit bias skewing the load (Zipf-like, as BASELINE config 4)."""
    layer, wr, packed = _config3_layer(torch, ctx, n_experts=32, seed=96)
    rng = np.random.default_rng(97)
    rank = rng.permutation(32) + 1
    bias = (-1.1 * np.log(rank)).astype(np.float32)
    layer.set_router(wr, bias)
    yield layer, wr, packed, bias
    layer.close()


@pytest.mark.parametrize("kernel", KERNELS)
def test_prefill_config4_shapes_match_oracle_and_decode(torch, ctx, c4, kernel):
    layer, wr, packed, bias = c4
    layer.set_prefill_kernel(kernel)
    T = 200
    rng = np.random.default_rng(98)
    x = q.f32_to_bf16(rng.standard_normal((T, 2048)).astype(np.float32))
    xd = _dev(torch, x, np.int16)
    out = torch.empty((T, 2048), dtype=torch.int16, device="cuda")
    ids = torch.empty((T, 8), dtype=torch.int32, device="cuda")
    w = torch.empty((T, 8), dtype=torch.float32, device="cuda")
    layer.prefill(xd, 8, out, ids, w, act="swiglu")
    # the decode path (<= 16 tokens per call) on the same tokens
    dec = torch.empty((T, 2048), dtype=torch.int16, device="cuda")
    dids = torch.empty((T, 8), dtype=torch.int32, device="cuda")
    for t0 in range(0, T, 16):
        t1 = min(T, t0 + 16)
        layer.decode(xd[t0:t1], 8, dec[t0:t1], dids[t0:t1], act="swiglu")
    torch.cuda.synchronize()
    ctx.sync()
    assert torch.equal(ids, dids)
    got, ref_dec = out.cpu().numpy().view(np.uint16), dec.cpu().numpy().view(np.uint16)
    cache = {}

    def expert(e):
        if e not in cache:
            cache[e] = _oracle_expert(packed, e, 2048, 768)
        return cache[e]
    for t in (0, 1, 57, 199):
        ref, r_ids, mag = _oracle_token(expert, expert(32), wr, x[t], 8, "swiglu", bias)
        np.testing.assert_array_equal(ids[t].cpu().numpy(), r_ids)
        assert_bf16_outputs_close(got[t], ref, mag)
    # the tensor-core kernel sums in another order than the decode path:
    # their rows differ by rounding flips only
    for t in range(T):
        assert rms_rel(got[t], ref_dec[t]) <= 4e-3, t
    if kernel == "gemv":
        # the register-fragment path runs the decode's unit arithmetic on the
        # same per-token staging: the bytes are the decode's
        assert torch.equal(out, dec)


@pytest.mark.parametrize("kernel", KERNELS)
def test_prefill_tokens_are_batch_invariant(torch, ctx, c4, kernel):
    layer = c4[0]
    layer.set_prefill_kernel(kernel)
    rng = np.random.default_rng(99)
    x = q.f32_to_bf16(rng.standard_normal((300, 2048)).astype(np.float32))
    xd = _dev(torch, x, np.int16)
    a = torch.empty((300, 2048), dtype=torch.int16, device="cuda")
    b = torch.empty((71, 2048), dtype=torch.int16, device="cuda")
    c = torch.empty((1, 2048), dtype=torch.int16, device="cuda")
    layer.prefill(xd, 8, a, act="swiglu")
    layer.prefill(xd[100:171], 8, b, act="swiglu")
    layer.prefill(xd[5:6], 8, c, act="swiglu")
    torch.cuda.synchronize()
    ctx.sync()
    assert torch.equal(a[100:171], b)
    assert torch.equal(a[5:6], c)


@pytest.mark.parametrize("kernel", KERNELS)
def test_prefill_caller_routes_reproduce_routed_call(torch, ctx, c4, kernel):
    layer = c4[0]
    layer.set_prefill_kernel(kernel)
    rng = np.random.default_rng(100)
    x = q.f32_to_bf16(rng.standard_normal((90, 2048)).astype(np.float32))
    xd = _dev(torch, x, np.int16)
    out = torch.empty((90, 2048), dtype=torch.int16, device="cuda")
    ids = torch.empty((90, 8), dtype=torch.int32, device="cuda")
    w = torch.empty((90, 8), dtype=torch.float32, device="cuda")
    layer.prefill(xd, 8, out, ids, w, act="swiglu")
    out2 = torch.empty_like(out)
    layer.prefill_experts(xd, ids, w, 8, out2, act="swiglu", with_shared=True)
    torch.cuda.synchronize()
    ctx.sync()
    assert torch.equal(out, out2)


def test_prefill_expert_parallel_ranks_reproduce_single_gpu_bytes(torch, ctx):
    """4 'ranks' each holding 8 of 32 experts and the shared one: summed slot
    rows combined per rank's tokens give exactly the single-GPU bytes.  With
    routes each rank computed for its own 24 tokens only (the prefill router),
    ``prefill_local_routes`` gives the same slot rows and weights."""
    E, R, T = 32, 4, 96
    full, wr, _ = _config3_layer(torch, ctx, n_experts=E, seed=103)
    per = E // R
    ranks = [_config3_layer(torch, ctx, n_experts=E, seed=103, owned=set(range(r * per, (r + 1) * per)) | {E})[0]
             for r in range(R)]
    rng = np.random.default_rng(104)
    x = q.f32_to_bf16(rng.standard_normal((T, 2048)).astype(np.float32))
    xd = _dev(torch, x, np.int16)
    ref = torch.empty((T, 2048), dtype=torch.int16, device="cuda")
    full.prefill(xd, 8, ref, act="swiglu")
    total = torch.zeros((T, 9, 2048), dtype=torch.float32, device="cuda")
    sws = []
    M = T // R
    ids = torch.empty((T, 8), dtype=torch.int32, device="cuda")
    wts = torch.empty((T, 8), dtype=torch.float32, device="cuda")
    for r, layer in enumerate(ranks):
        layer.route(xd[r * M:(r + 1) * M], M, 8, ids[r * M:(r + 1) * M], wts[r * M:(r + 1) * M])
    for r, layer in enumerate(ranks):
        slots = torch.empty((T, 9, 2048), dtype=torch.int16, device="cuda")
        sw = torch.empty((T, 8), dtype=torch.float32, device="cuda")
        layer.prefill_local(xd, 8, slots, sw, experts=(r * per, (r + 1) * per), shared_tokens=(r * M, M),
                            act="swiglu")
        slots2 = torch.full((T, 9, 2048), 0x7FC0, dtype=torch.int16, device="cuda")
        sw2 = torch.full((T, 8), float("nan"), dtype=torch.float32, device="cuda")
        layer.prefill_local_routes(xd, ids, wts, 8, slots2, sw2, experts=(r * per, (r + 1) * per),
                                   shared_tokens=(r * M, M), act="swiglu")
        torch.cuda.synchronize()
        assert torch.equal(slots2, slots), r
        assert torch.equal(sw2, sw), r
        total += slots.view(torch.bfloat16).float()
        sws.append(sw)
    torch.cuda.synchronize()
    summed = total.to(torch.bfloat16).view(torch.int16)
    for r, layer in enumerate(ranks):
        assert torch.equal(sws[r], sws[0])
        out = torch.empty((M, 2048), dtype=torch.int16, device="cuda")
        layer.prefill_combine(summed[r * M:(r + 1) * M].contiguous(), sws[r][r * M:(r + 1) * M].contiguous(), 8,
                              out, tokens=M, with_shared=True)
        torch.cuda.synchronize()
        assert torch.equal(out, ref[r * M:(r + 1) * M]), r
    ctx.sync()
    for layer in [full] + ranks:
        layer.close()
