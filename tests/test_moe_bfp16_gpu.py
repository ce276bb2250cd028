"""MoE layers whose expert down matrices are bfp16ebs8 (the reference's
``moe_b2`` expert bundles, ``npu/backend.py:640-652``; gate/up stay q4nx as
its ``moe_b1``): ``rc_moe_set_expert`` with ``RC_UPLOAD_DOWN_BFP16``.

The oracle is ``NumpyBackend.moe_experts`` (``host/backend.py:466-510``) on
the exact f32 weights the bfp16ebs8 down matrices decode to
(``oracle.bfp16.gemv_weights``).  Bar: as for the q4nx layers, every output
within one bf16 step of the f32 combine's term magnitude of the oracle's
(each expert row is a bf16 value whose last rounding may fall either way
between two summation orders), and a small RMS error.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import backend as ob
from oracle import bfp16 as ob16
from oracle import q4nx as q
from tests.golden import cases
from tests.test_moe_gpu import assert_bf16_outputs_close

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


def _bfp16_experts(rng, hidden, inter, E):
    """Per expert: q4nx [gate; up] bytes, bfp16ebs8 bytes of the K-padded down
    matrix, and the oracle's f32 (gate, up, down) weights."""
    ip = (inter + 255) // 256 * 256
    packed, experts = {}, {}
    for e in range(E):
        gu = (rng.standard_normal((2 * inter, hidden)) * 0.02).astype(np.float32)
        dn = np.zeros((hidden, ip), np.float32)
        dn[:, :inter] = rng.standard_normal((hidden, inter)) * 0.02
        pgu, fgu = cases.q4nx_weight(gu, q)
        ex, mt = ob16.flush_tiny(*ob16.encode(dn))
        packed[e] = (pgu, ob16.pack_gemv_raw(ex, mt))
        experts[e] = (fgu[:inter], fgu[inter:], ob16.gemv_weights(ex, mt.reshape(hidden, ip))[:, :inter])
    return packed, experts


def _layer(ctx, packed, hidden, inter, E, has_shared=False):
    from raon_npu_b200.device import MoeLayer
    layer = MoeLayer(ctx, hidden, inter, E, has_shared=has_shared)
    for e, (pgu, pdn) in packed.items():
        layer.set_expert(e, pgu, pdn, down_format="bfp16")
    return layer


@pytest.mark.parametrize("hidden,inter,E,k,T", [(2048, 768, 16, 8, 1), (2048, 768, 16, 8, 6),
                                               (256, 1088, 6, 3, 12), (512, 512, 8, 2, 16)])
def test_experts_bfp16_down_match_oracle(ctx, hidden, inter, E, k, T):
    rng = np.random.default_rng(hidden + inter + T)
    packed, experts = _bfp16_experts(rng, hidden, inter, E)
    layer = _layer(ctx, packed, hidden, inter, E)
    x = q.f32_to_bf16(rng.standard_normal((T, hidden)).astype(np.float32))
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)])
    w = rng.uniform(0.05, 0.5, (T, k)).astype(np.float32)
    for act in ("swiglu", "situ"):
        out = layer.experts_host(x, ids, w, act=act)
        for t in range(T):
            ref = ob.moe_experts(experts, x[t], ids[t], w[t], act=act)
            mag = ob.moe_term_magnitude(experts, x[t], ids[t], w[t], act)
            assert_bf16_outputs_close(out[t], ref, mag)
        # batch invariance: one token alone gives the same bytes
        one = layer.experts_host(x[T - 1], ids[T - 1], w[T - 1], act=act)
        np.testing.assert_array_equal(one, out[T - 1])
    layer.close()


def test_decode_with_bfp16_down_routes_through_separate_launches(torch, ctx):
    """rc_moe_decode (fused requested) on a bfp16-down layer with a shared
    expert equals rc_moe_experts with the ids / weights the router chose plus
    the shared expert, and the oracle within the MoE bar."""
    hidden, inter, E, k, T = 1024, 512, 12, 4, 3
    rng = np.random.default_rng(23)
    packed, experts = _bfp16_experts(rng, hidden, inter, E + 1)
    layer = _layer(ctx, packed, hidden, inter, E, has_shared=True)
    wr = q.f32_to_bf16((rng.standard_normal((E, hidden)) * 0.02).astype(np.float32))
    layer.set_router(wr)
    x = q.f32_to_bf16(rng.standard_normal((T, hidden)).astype(np.float32))
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    out = torch.empty_like(xd)
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    layer.decode(xd, k, out, ids, w, act="swiglu")
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16)
    idh, wh = ids.cpu().numpy(), w.cpu().numpy()
    again = layer.experts_host(x, idh, wh, act="swiglu", with_shared=True)
    np.testing.assert_array_equal(got, again)
    for t in range(T):
        rid, rw, _ = ob.route_softmax(x[t], wr, k)
        assert sorted(rid.tolist()) == sorted(idh[t].tolist())
        routed = ob.moe_experts(experts, x[t], idh[t], wh[t], act="swiglu")
        sh = ob.expert_forward(*experts[E], x[t], "swiglu")
        ref = ob.moe_token_with_shared(routed, sh)
        mag = ob.moe_term_magnitude(experts, x[t], idh[t], wh[t], "swiglu", shared_down_u16=sh)
        assert_bf16_outputs_close(got[t], ref, mag)
    layer.close()


def test_bfp16_down_expert_parallel_halves_reproduce_single_gpu_bytes(torch, ctx):
    """The NCCL-transport halves (rc_moe_decode_local on two layers holding
    half of the experts each, rank 0 also the shared one; slot rows merged,
    then rc_moe_combine) give exactly the bytes of the whole layer's decode."""
    hidden, inter, E, k = 1024, 512, 16, 4
    rng = np.random.default_rng(41)
    packed, _ = _bfp16_experts(rng, hidden, inter, E + 1)
    wr = q.f32_to_bf16((rng.standard_normal((E, hidden)) * 0.02).astype(np.float32))
    full = _layer(ctx, packed, hidden, inter, E, has_shared=True)
    r0 = _layer(ctx, {e: packed[e] for e in list(range(E // 2)) + [E]}, hidden, inter, E, has_shared=True)
    r1 = _layer(ctx, {e: packed[e] for e in range(E // 2, E)}, hidden, inter, E, has_shared=True)
    for layer in (full, r0, r1):
        layer.set_router(wr)
    for _ in range(3):
        x = q.f32_to_bf16(rng.standard_normal(hidden).astype(np.float32))
        xd = torch.from_numpy(x.view(np.int16)).cuda()
        ref = torch.empty(hidden, dtype=torch.int16, device="cuda")
        full.decode(xd, k, ref, act="swiglu")
        slots = [torch.empty((k + 1, hidden), dtype=torch.int16, device="cuda") for _ in range(2)]
        sw = [torch.empty(k, dtype=torch.float32, device="cuda") for _ in range(2)]
        r0.decode_local(xd, k, slots[0], sw[0], experts=(0, E // 2), shared_tokens=(0, 1), act="swiglu")
        r1.decode_local(xd, k, slots[1], sw[1], experts=(E // 2, E), shared_tokens=(0, 0), act="swiglu")
        torch.cuda.synchronize()
        a, b = slots
        assert bool(((a == 0) | (b == 0)).all())
        assert torch.equal(sw[0], sw[1])
        out = torch.empty(hidden, dtype=torch.int16, device="cuda")
        r0.combine(torch.where(a != 0, a, b), sw[0], k, out, with_shared=True)
        torch.cuda.synchronize()
        ctx.sync()
        assert torch.equal(out, ref)
    for layer in (full, r0, r1):
        layer.close()


@pytest.mark.parametrize("kernel", ["gemv", "tcgen05"])
def test_prefill_with_bfp16_down_equals_decode_chain(torch, ctx, kernel):
    """rc_moe_prefill on a bfp16-down layer (either prefill kernel setting: the
    bfp16 down runs on the register-fragment path's 8-row blocks) gives the
    bytes of the decode chain on the routes it chose, 16 tokens at a time, and
    the oracle's outputs within the MoE bar."""
    hidden, inter, E, k, T = 1024, 768, 12, 4, 40
    rng = np.random.default_rng(31)
    packed, experts = _bfp16_experts(rng, hidden, inter, E + 1)
    layer = _layer(ctx, packed, hidden, inter, E, has_shared=True)
    layer.set_prefill_kernel(kernel)
    wr = q.f32_to_bf16((rng.standard_normal((E, hidden)) * 0.02).astype(np.float32))
    layer.set_router(wr)
    x = q.f32_to_bf16(rng.standard_normal((T, hidden)).astype(np.float32))
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    out = torch.empty_like(xd)
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    layer.prefill(xd, k, out, ids, w, act="swiglu")
    torch.cuda.synchronize()
    got = out.cpu().numpy().view(np.uint16)
    idh, wh = ids.cpu().numpy(), w.cpu().numpy()
    for t0 in range(0, T, 16):
        again = layer.experts_host(x[t0:t0 + 16], idh[t0:t0 + 16], wh[t0:t0 + 16], act="swiglu", with_shared=True)
        np.testing.assert_array_equal(got[t0:t0 + 16], again)
    for t in (0, T // 2, T - 1):
        routed = ob.moe_experts(experts, x[t], idh[t], wh[t], act="swiglu")
        sh = ob.expert_forward(*experts[E], x[t], "swiglu")
        mag = ob.moe_term_magnitude(experts, x[t], idh[t], wh[t], "swiglu", shared_down_u16=sh)
        assert_bf16_outputs_close(got[t], ob.moe_token_with_shared(routed, sh), mag)
    layer.close()


def test_bfp16_down_refusals(torch, ctx):
    """One down format per layer, and a down matrix of the wrong size, are refused."""
    from raon_npu_b200.device import MoeLayer
    hidden, inter, E = 256, 256, 4
    rng = np.random.default_rng(3)
    packed, _ = _bfp16_experts(rng, hidden, inter, E)
    layer = _layer(ctx, {0: packed[0]}, hidden, inter, E)
    dq, _ = cases.q4nx_weight((rng.standard_normal((hidden, inter)) * 0.02).astype(np.float32), q)
    with pytest.raises(ValueError, match="one format per layer"):
        layer.set_expert(1, packed[1][0], dq)
    with pytest.raises(ValueError):
        layer.set_expert(1, packed[1][0], packed[1][1][:-9], down_format="bfp16")
    layer.set_expert(0, packed[0][0], packed[0][1], down_format="bfp16")     # replacing the same expert is fine
    layer.close()
    q_layer = MoeLayer(ctx, hidden, inter, E, has_shared=False)
    with pytest.raises(ValueError, match="unknown down format"):
        q_layer.set_expert(0, packed[0][0], packed[0][1], down_format="bfp8")
    q_layer.close()
