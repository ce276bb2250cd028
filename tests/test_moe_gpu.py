"""GPU parity of the MoE decode path (router, grouped expert GEMVs, combine)
against the CPU oracle and the reference's own outputs.

Bars: top-k expert ids bit-exact (lower index wins ties) and router logits
equal to the oracle's f64-accumulated logits.  Outputs (bf16) against the
oracle's bf16 outputs: RMS relative error <= 2e-3 (the north star's
tolerance), and per element |y - y_ref| <= 2^-7 * m[h] + ulp(y_ref[h]) with
m[h] = sum_e |w_e down_e[h]| (+ |shared[h]|) (``oracle.backend.
moe_term_magnitude``): one bf16 step of every accumulated term (a step is at
most 2^-7 of the value) plus the final rounding.

Why not "bit-exact but for rare flips": both sides stage the reference's bf16
roundings (gate, up, act, down) but sum in different orders and use different
exp/tanh; a 1-ulp flip of one gate/up output flips an activation element,
which moves every down-projection output a little, so per-expert outputs
differ by one bf16 step on many elements, and the weighted sum over the
experts can cancel to a result smaller than its terms.  What is bit-exact:
the routing, the combine (restated by the oracle on the GPU's own expert
rows), batch invariance (a token's bytes do not depend on the other tokens of
the call) and expert parallelism (ranks reproduce the single-GPU bytes).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import backend as ob
from oracle import q4nx as q
from tests.golden import cases

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


def ulp_diff(a, b):
    def key(u):
        u = np.asarray(u).astype(np.int32)
        return np.where(u & 0x8000, -(u & 0x7FFF), u & 0x7FFF)
    return np.abs(key(a) - key(b))


def bf16_ulp_at(u16):
    """Spacing of bf16 values at each element (one step of the last place)."""
    f = np.abs(q.bf16_to_f32(u16).astype(np.float64))
    e = np.floor(np.log2(np.maximum(f, 2.0 ** -126)))
    return 2.0 ** (e - 7)


def rms_rel(got, ref):
    rf = q.bf16_to_f32(np.asarray(ref, np.uint16)).astype(np.float64)
    gf = q.bf16_to_f32(np.asarray(got, np.uint16)).astype(np.float64)
    return float(np.sqrt(np.mean((gf - rf) ** 2)) / max(np.sqrt(np.mean(rf ** 2)), 1e-30))


# Largest errors seen by the MoE output checks in this run (printed in the
# pytest terminal summary).
PARITY = {"outputs": 0, "rms_max": 0.0, "normwise_max": 0.0, "call_rms_max": 0.0}

# Bars on bf16 MoE outputs against the oracle (NumpyBackend semantics: the
# reference's bf16 roundings of gate, up, activation and down, f32 sums).
#  * RMS relative error <= 2e-3 over all rows of a call (the north star's
#    tolerance), <= 4e-3 on every single row;
#  * normwise max error max|y - y_ref| / max|y_ref| <= 2^-6 per row, two bf16
#    steps of the largest output;
#  * per element |y - y_ref| <= 2^-7 m + ulp(y_ref) + ulp(y), m the magnitude of
#    the terms the f32 combine sums (one bf16 step of each term, and the last
#    rounding of either side falling the other way).
# Why not tighter: both sides round to bf16 at four points per expert, and
# the device's q4nx unit arithmetic (scale * sum(code x) + min * sum(x), two
# terms that largely cancel, on tensor cores) leaves f32 sums ~1e-6 of |y|
# from exact -- far inside the GEMV bar, but enough to flip a bf16 rounding
# now and then; a flipped activation moves a few percent of that expert's
# down outputs by one step.  Neighbouring bf16 values are 2^-8..2^-7 of their
# magnitude apart, so single elements differ by that much.  Two correct
# numpy restatements that differ only in summation order (f32 vs f64 dot
# products) already differ by up to 1.2e-3 RMS on single rows and 4.3e-3
# normwise (tests/test_oracle_pins.py, the spread test).
ROW_RMS = 4e-3
CALL_RMS = 2e-3
MAX_NORMWISE = 2.0 ** -6


def assert_bf16_outputs_close(got, ref, magnitude=None, tol=ROW_RMS):
    got = np.asarray(got, np.uint16)
    ref = np.asarray(ref, np.uint16)
    rf = q.bf16_to_f32(ref).astype(np.float64)
    gf = q.bf16_to_f32(got).astype(np.float64)
    err = np.abs(gf - rf)
    if magnitude is not None:
        bound = 2.0 ** -7 * magnitude + bf16_ulp_at(ref) + bf16_ulp_at(got)
        bad = err > bound
        assert not bad.any(), (np.nonzero(bad)[0][:8], err[bad][:8], bound[bad][:8])
    else:
        assert ulp_diff(got, ref).max() <= 1
    rms = np.sqrt(np.mean(err ** 2)) / max(np.sqrt(np.mean(rf ** 2)), 1e-30)
    normwise = float(err.max() / max(np.abs(rf).max(), 1e-30))
    PARITY["outputs"] += 1
    PARITY["rms_max"] = max(PARITY["rms_max"], float(rms))
    PARITY["normwise_max"] = max(PARITY["normwise_max"], normwise)
    assert rms <= tol, rms
    assert normwise <= MAX_NORMWISE, normwise


def assert_call_rms(got, ref, tol=CALL_RMS):
    """RMS relative error over every row of a call (bf16 bits [T, H])."""
    rf = q.bf16_to_f32(np.asarray(ref, np.uint16)).astype(np.float64)
    gf = q.bf16_to_f32(np.asarray(got, np.uint16)).astype(np.float64)
    rms = float(np.sqrt(np.mean((gf - rf) ** 2)) / max(np.sqrt(np.mean(rf ** 2)), 1e-30))
    PARITY["call_rms_max"] = max(PARITY["call_rms_max"], rms)
    assert rms <= tol, rms


def make_layer(ctx, d, has_shared=False, shared=None):
    from raon_npu_b200.device import MoeLayer
    e0 = next(iter(d["packed"]))
    hidden = d["experts"][e0][2].shape[0]
    inter = d["experts"][e0][0].shape[0]
    layer = MoeLayer(ctx, hidden, inter, len(d["packed"]), has_shared=has_shared)
    for e, (pgu, pdn) in d["packed"].items():
        layer.set_expert(e, pgu, pdn)
    if shared is not None:
        layer.set_expert(len(d["packed"]), *shared)
    return layer


# ---------------------------------------------------------------- experts --
def test_moe_experts_matches_reference_fixture(ctx):
    """NumpyBackend.moe_experts outputs recorded from the reference (SiTU, two beta pairs)."""
    g = np.load(cases.__file__.replace("cases.py", "moe.npz"))
    d = cases.moe_inputs(**cases.MOE_CASE)
    layer = make_layer(ctx, d)
    for t in range(d["x"].shape[0]):
        for tag, kw in (("default", {}), ("betas", dict(gate_beta=2.0, value_beta=10.0))):
            out = layer.experts_host(d["x"][t], d["top_ids"][t], d["top_w"][t], act="situ", **kw)
            mag = ob.moe_term_magnitude(d["experts"], d["x"][t], d["top_ids"][t], d["top_w"][t], "situ", **kw)
            assert_bf16_outputs_close(out, g[f"tok{t}/{tag}"], mag)
    layer.close()


@pytest.mark.parametrize("act", ["swiglu", "situ"])
def test_moe_experts_matches_oracle_config3_shapes(ctx, act):
    """hidden 2048, intermediate 768, 8 of 16 experts (the config-3 expert shapes)."""
    d = cases.moe_inputs(hidden=2048, inter=768, experts=16, k=8, tokens=2, seed=61)
    layer = make_layer(ctx, d)
    for t in range(2):
        out = layer.experts_host(d["x"][t], d["top_ids"][t], d["top_w"][t], act=act)
        ref = ob.moe_experts(d["experts"], d["x"][t], d["top_ids"][t], d["top_w"][t], act=act)
        mag = ob.moe_term_magnitude(d["experts"], d["x"][t], d["top_ids"][t], d["top_w"][t], act)
        assert_bf16_outputs_close(out, ref, mag)
    layer.close()


def test_moe_experts_padded_intermediate(ctx):
    """Real-Raon-like intermediate 1088 (down K zero-padded to 1280, kernels/moe/pack.py:190-224)."""
    rng = np.random.default_rng(71)
    hidden, inter, E = 256, 1088, 4
    experts, packed = {}, {}
    for e in range(E):
        gu = (rng.standard_normal((2 * inter, hidden)) * 0.02).astype(np.float32)
        dn = (rng.standard_normal((hidden, inter)) * 0.02).astype(np.float32)
        dnp, _ = q.pad_gemv(dn, m_align=128, k_align=256)
        pgu, fgu = cases.q4nx_weight(gu, q)
        pdn, fdn = cases.q4nx_weight(dnp, q)
        experts[e] = (fgu[:inter], fgu[inter:], fdn[:, :inter])
        packed[e] = (pgu, pdn)
    from raon_npu_b200.device import MoeLayer
    layer = MoeLayer(ctx, hidden, inter, E, has_shared=False)
    for e, (a, b) in packed.items():
        layer.set_expert(e, a, b)
    x = q.f32_to_bf16(rng.standard_normal(hidden).astype(np.float32))
    ids = np.array([3, 0, 2])
    w = np.array([0.5, 0.3, 0.2], np.float32)
    out = layer.experts_host(x, ids, w, act="situ")
    assert_bf16_outputs_close(out, ob.moe_experts(experts, x, ids, w, act="situ"),
                              ob.moe_term_magnitude(experts, x, ids, w, "situ"))
    layer.close()


def test_moe_experts_rejects_unknown_expert(ctx):
    d = cases.moe_inputs(**cases.MOE_CASE)
    layer = make_layer(ctx, d)
    with pytest.raises(ValueError):
        layer.experts_host(d["x"][0], np.array([0, 99, 1]), d["top_w"][0])
    layer.close()


# ----------------------------------------------------------------- router --
def _router_layer(ctx, hidden, E, seed, dup=None):
    from raon_npu_b200.device import MoeLayer
    rng = np.random.default_rng(seed)
    wr = q.f32_to_bf16((rng.standard_normal((E, hidden)) * 0.02).astype(np.float32))
    if dup:
        for a, b in dup:
            wr[b] = wr[a]
    layer = MoeLayer(ctx, hidden, 64, E, has_shared=False)
    layer.set_router(wr)
    return layer, wr, rng


def test_softmax_router_matches_oracle(torch, ctx):
    layer, wr, rng = _router_layer(ctx, 2048, 128, seed=81)
    T, k = 16, 8
    x = q.f32_to_bf16(rng.standard_normal((T, 2048)).astype(np.float32))
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    lg = torch.empty((T, 128), dtype=torch.float32, device="cuda")
    layer.route(xd, T, k, ids, w, lg)
    torch.cuda.synchronize()
    ctx.sync()
    for t in range(T):
        r_ids, r_w, r_lg = ob.route_softmax(x[t], wr, k)
        np.testing.assert_array_equal(lg[t].cpu().numpy(), r_lg)
        np.testing.assert_array_equal(ids[t].cpu().numpy(), r_ids)
        np.testing.assert_allclose(w[t].cpu().numpy(), r_w, rtol=2e-6)
        # selection logic on the device's own logits is exact by construction
        np.testing.assert_array_equal(ids[t].cpu().numpy(), ob.topk_lower_index_wins(lg[t].cpu().numpy(), k))
    layer.close()


def test_router_ties_lower_index_wins(torch, ctx):
    # experts 9 and 40 duplicate expert 3 (identical logits); 77 duplicates 12
    layer, wr, rng = _router_layer(ctx, 256, 128, seed=82, dup=[(3, 9), (3, 40), (12, 77)])
    x = q.f32_to_bf16(rng.standard_normal((4, 256)).astype(np.float32))
    x[3] = 0                                    # every logit 0: all 128 experts tie
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    ids = torch.empty((4, 8), dtype=torch.int32, device="cuda")
    w = torch.empty((4, 8), dtype=torch.float32, device="cuda")
    lg = torch.empty((4, 128), dtype=torch.float32, device="cuda")
    layer.route(xd, 4, 8, ids, w, lg)
    torch.cuda.synchronize()
    for t in range(4):
        np.testing.assert_array_equal(ids[t].cpu().numpy(), ob.topk_lower_index_wins(ob.router_logits(x[t], wr), 8))
    np.testing.assert_array_equal(ids[3].cpu().numpy(), np.arange(8))
    np.testing.assert_allclose(w[3].cpu().numpy(), np.full(8, 0.125, np.float32), rtol=1e-6)
    layer.close()


def test_sigmoid_bias_router_matches_reference_fixture(torch, ctx):
    from raon_npu_b200.device import MoeLayer
    g = np.load(cases.__file__.replace("cases.py", "router.npz"))
    d = cases.router_inputs(**cases.ROUTER_CASE)
    E, H = d["router_w_bits"].shape
    layer = MoeLayer(ctx, H, 64, E, has_shared=False)
    layer.set_router(d["router_w_bits"], d["bias"])
    T, k = d["x"].shape[0], d["k"]
    xd = torch.from_numpy(d["x"].view(np.int16)).cuda()
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    layer.route(xd, T, k, ids, w, router="sigmoid_bias", scaling=d["scaling"])
    torch.cuda.synchronize()
    for t in range(T):
        np.testing.assert_array_equal(ids[t].cpu().numpy(), g[f"tok{t}/top"])
        np.testing.assert_allclose(w[t].cpu().numpy(), g[f"tok{t}/w"], rtol=1e-5)
    layer.close()


# ------------------------------------------------------- decode layer (cfg 3) --
def _config3_layer(torch, ctx, n_experts=128, hidden=2048, inter=768, seed=91, owned=None, has_shared=True):
    """Experts generated on the GPU (seeded), quantised by rc_quantize_q4nx.
    Returns (layer, router bits, host packed bytes of every expert)."""
    from raon_npu_b200.device import MoeLayer
    gen = torch.Generator(device="cuda")
    layer = MoeLayer(ctx, hidden, inter, n_experts, has_shared=has_shared)
    packed = {}
    ids = list(range(n_experts)) + ([n_experts] if has_shared else [])
    for e in ids:
        gen.manual_seed(seed * 1000 + e)
        gu = torch.randn((2 * inter, hidden), generator=gen, device="cuda") * 0.02
        dn = torch.randn((hidden, inter), generator=gen, device="cuda") * 0.02
        ip = (inter + 255) // 256 * 256          # down K zero-padded to the 256-column tile
        if ip != inter:
            dn = torch.nn.functional.pad(dn, (0, ip - inter))
        pgu = torch.empty(2 * inter * hidden * 5 // 8, dtype=torch.uint8, device="cuda")
        pdn = torch.empty(hidden * ip * 5 // 8, dtype=torch.uint8, device="cuda")
        ctx.quantize_q4nx(gu, pgu, 2 * inter, hidden)
        ctx.quantize_q4nx(dn, pdn, hidden, ip)
        packed[e] = (pgu, pdn)
        if owned is None or e in owned:
            layer.set_expert(e, pgu, pdn)
    rng = np.random.default_rng(seed)
    wr = q.f32_to_bf16((rng.standard_normal((n_experts, hidden)) * 0.02).astype(np.float32))
    layer.set_router(wr)
    return layer, wr, packed


def _oracle_expert(packed, e, hidden, inter):
    pgu, pdn = (t.cpu().numpy() for t in packed[e])
    fgu = q.dequantize_packed(pgu, 2 * inter, hidden)
    ip = (inter + 255) // 256 * 256
    return fgu[:inter], fgu[inter:], q.dequantize_packed(pdn, hidden, ip)[:, :inter]


def test_moe_decode_layer_config3(torch, ctx):
    """hidden 2048, 128 experts + shared, I=768, softmax top-8, SwiGLU."""
    layer, wr, packed = _config3_layer(torch, ctx)
    rng = np.random.default_rng(5)
    gots, refs = [], []
    for trial in range(3):
        x = q.f32_to_bf16(rng.standard_normal(2048).astype(np.float32))
        xd = torch.from_numpy(x.view(np.int16)).cuda()
        out = torch.empty(2048, dtype=torch.int16, device="cuda")
        ids = torch.empty(8, dtype=torch.int32, device="cuda")
        w = torch.empty(8, dtype=torch.float32, device="cuda")
        layer.decode(xd, 8, out, ids, w, act="swiglu")
        torch.cuda.synchronize()
        ctx.sync()
        r_ids, r_w, _ = ob.route_softmax(x, wr, 8)
        np.testing.assert_array_equal(ids.cpu().numpy(), r_ids)
        experts = {int(e): _oracle_expert(packed, int(e), 2048, 768) for e in r_ids}
        routed = ob.moe_experts(experts, x, r_ids, r_w, act="swiglu")
        sh = ob.expert_forward(*_oracle_expert(packed, 128, 2048, 768), x, "swiglu")
        ref = ob.moe_token_with_shared(routed, sh)
        mag = ob.moe_term_magnitude(experts, x, r_ids, r_w, "swiglu", shared_down_u16=sh)
        got = out.cpu().numpy().view(np.uint16)
        assert_bf16_outputs_close(got, ref, mag)
        gots.append(got)
        refs.append(ref)

        # Stage by stage: every expert's bf16 output row (8 routed slots in
        # ascending expert ID, then the shared expert) against the oracle's,
        # and the combine of the GPU's own rows, restated by the oracle, bit-exact.
        slots = torch.empty((9, 2048), dtype=torch.int16, device="cuda")
        sw = torch.empty(8, dtype=torch.float32, device="cuda")
        layer.decode_local(xd, 8, slots, sw, act="swiglu")
        torch.cuda.synchronize()
        rows = slots.cpu().numpy().view(np.uint16)
        order = np.argsort(r_ids, kind="stable")
        np.testing.assert_array_equal(sw.cpu().numpy(), w.cpu().numpy()[order])
        for s, e in enumerate(list(r_ids[order]) + [128]):
            e_ref = sh if e == 128 else ob.expert_forward(*experts[int(e)], x, "swiglu")
            # one expert row: a flipped activation element moves ~20% of the
            # down outputs by one bf16 step, so the bar is one step (2^-8) RMS
            assert rms_rel(rows[s], e_ref) <= 2.0 ** -8, (s, int(e), rms_rel(rows[s], e_ref))
        routed_gpu = ob.combine_ascending(rows[None, :8], r_ids[order][None], w.cpu().numpy()[order][None])[0]
        np.testing.assert_array_equal(ob.moe_token_with_shared(routed_gpu, rows[8]), got)
    assert_call_rms(np.stack(gots), np.stack(refs))
    layer.close()


def test_expert_parallel_halves_reproduce_single_gpu_bytes(torch, ctx):
    """Two 'ranks' on one GPU, each holding half of the experts (rank 0 also the
    shared one): summing the slot rows and combining gives exactly the bytes
    of the single-layer decode."""
    full, wr, _ = _config3_layer(torch, ctx, n_experts=32, seed=92)
    r0, _, _ = _config3_layer(torch, ctx, n_experts=32, seed=92, owned=set(range(16)) | {32})
    r1, _, _ = _config3_layer(torch, ctx, n_experts=32, seed=92, owned=set(range(16, 32)))
    rng = np.random.default_rng(6)
    for _ in range(4):
        x = q.f32_to_bf16(rng.standard_normal(2048).astype(np.float32))
        xd = torch.from_numpy(x.view(np.int16)).cuda()
        ref = torch.empty(2048, dtype=torch.int16, device="cuda")
        full.decode(xd, 8, ref, act="swiglu")
        slots = [torch.empty((9, 2048), dtype=torch.int16, device="cuda") for _ in range(2)]
        sw = [torch.empty(8, dtype=torch.float32, device="cuda") for _ in range(2)]
        r0.decode_local(xd, 8, slots[0], sw[0], experts=(0, 16), shared_tokens=(0, 1), act="swiglu")
        r1.decode_local(xd, 8, slots[1], sw[1], experts=(16, 32), shared_tokens=(0, 0), act="swiglu")
        torch.cuda.synchronize()
        # each slot row is produced by exactly one rank; the other rank's row is zero
        a = slots[0].view(torch.int16)
        b = slots[1].view(torch.int16)
        assert bool(((a == 0) | (b == 0)).all())
        merged = torch.where(a != 0, a, b)
        assert torch.equal(sw[0], sw[1])
        out = torch.empty(2048, dtype=torch.int16, device="cuda")
        r0.combine(merged, sw[0], 8, out, with_shared=True)
        torch.cuda.synchronize()
        ctx.sync()
        assert torch.equal(out, ref)
    for layer in (full, r0, r1):
        layer.close()


def test_decode_refuses_missing_experts(torch, ctx):
    layer, _, _ = _config3_layer(torch, ctx, n_experts=16, seed=93, owned=set(range(8)) | {16})
    xd = torch.zeros(2048, dtype=torch.int16, device="cuda")
    out = torch.empty(2048, dtype=torch.int16, device="cuda")
    with pytest.raises(ValueError):
        layer.decode(xd, 8, out, act="swiglu")
    slots = torch.empty((9, 2048), dtype=torch.int16, device="cuda")
    sw = torch.empty(8, dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):
        layer.decode_local(xd, 8, slots, sw, experts=(4, 12), act="swiglu")
    layer.close()


# --------------------------------------------------------- multi-token --
@pytest.mark.parametrize("T", [2, 5, 8, 9, 16])
def test_decode_tokens_are_batch_invariant_and_match_oracle(torch, ctx, T):
    """T tokens in one call: every token's output and routing equal the bytes of
    a one-token call (columns of the grouped GEMV do not interact), and match
    the oracle within the MoE bar."""
    layer, wr, packed = _config3_layer(torch, ctx, n_experts=32, seed=94)
    rng = np.random.default_rng(100 + T)
    x = q.f32_to_bf16(rng.standard_normal((T, 2048)).astype(np.float32))
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    out = torch.empty((T, 2048), dtype=torch.int16, device="cuda")
    ids = torch.empty((T, 8), dtype=torch.int32, device="cuda")
    w = torch.empty((T, 8), dtype=torch.float32, device="cuda")
    layer.decode(xd, 8, out, ids, w, act="swiglu")
    one = torch.empty(2048, dtype=torch.int16, device="cuda")
    for t in range(T):
        layer.decode(xd[t], 8, one, act="swiglu")
        torch.cuda.synchronize()
        assert torch.equal(one, out[t]), t
    ctx.sync()
    got = out.cpu().numpy().view(np.uint16)
    for t in range(min(T, 3)):
        r_ids, r_w, _ = ob.route_softmax(x[t], wr, 8)
        np.testing.assert_array_equal(ids[t].cpu().numpy(), r_ids)
        experts = {int(e): _oracle_expert(packed, int(e), 2048, 768) for e in r_ids}
        sh = ob.expert_forward(*_oracle_expert(packed, 32, 2048, 768), x[t], "swiglu")
        ref = ob.moe_token_with_shared(ob.moe_experts(experts, x[t], r_ids, r_w, act="swiglu"), sh)
        mag = ob.moe_term_magnitude(experts, x[t], r_ids, r_w, "swiglu", shared_down_u16=sh)
        assert_bf16_outputs_close(got[t], ref, mag)
    layer.close()


@pytest.mark.parametrize("ranks,M", [(4, 1), (4, 4), (8, 2)])
def test_expert_parallel_ranks_reproduce_single_gpu_bytes(torch, ctx, ranks, M):
    """Expert parallelism as the multi-GPU path runs it, emulated on one GPU:
    every rank holds experts [r*E/N, (r+1)*E/N) and the shared expert, routes
    all N*M gathered tokens, computes its experts for all of them and the
    shared expert for its own M tokens; the slot rows summed over ranks (the
    reduce-scatter) and combined per rank give exactly the single-GPU bytes."""
    E = 32
    T = ranks * M
    full, wr, _ = _config3_layer(torch, ctx, n_experts=E, seed=95)
    per = E // ranks
    layers = [_config3_layer(torch, ctx, n_experts=E, seed=95, owned=set(range(r * per, (r + 1) * per)) | {E})[0]
              for r in range(ranks)]
    rng = np.random.default_rng(7)
    x = q.f32_to_bf16(rng.standard_normal((T, 2048)).astype(np.float32))
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    ref = torch.empty((T, 2048), dtype=torch.int16, device="cuda")
    full.decode(xd, 8, ref, act="swiglu")
    total = torch.zeros((T, 9, 2048), dtype=torch.float32, device="cuda")
    sws = []
    for r, layer in enumerate(layers):
        slots = torch.empty((T, 9, 2048), dtype=torch.int16, device="cuda")
        sw = torch.empty((T, 8), dtype=torch.float32, device="cuda")
        layer.decode_local(xd, 8, slots, sw, experts=(r * per, (r + 1) * per), shared_tokens=(r * M, M),
                           act="swiglu")
        total += slots.view(torch.bfloat16).float()
        sws.append(sw)
    torch.cuda.synchronize()
    summed = total.to(torch.bfloat16).view(torch.int16)
    for r, layer in enumerate(layers):
        assert torch.equal(sws[r], sws[0])
        out = torch.empty((M, 2048), dtype=torch.int16, device="cuda")
        layer.combine(summed[r * M:(r + 1) * M].contiguous(), sws[r][r * M:(r + 1) * M].contiguous(), 8, out,
                      tokens=M, with_shared=True)
        torch.cuda.synchronize()
        assert torch.equal(out, ref[r * M:(r + 1) * M]), r
    ctx.sync()
    for layer in [full] + layers:
        layer.close()


def test_experts_multi_token_matches_oracle(torch, ctx):
    """rc_moe_experts with caller ids for T = 6 tokens, overlapping expert choices."""
    d = cases.moe_inputs(hidden=2048, inter=768, experts=16, k=8, tokens=6, seed=62)
    layer = make_layer(ctx, d)
    out = layer.experts_host(d["x"], d["top_ids"], d["top_w"], act="swiglu")
    for t in range(6):
        ref = ob.moe_experts(d["experts"], d["x"][t], d["top_ids"][t], d["top_w"][t], act="swiglu")
        mag = ob.moe_term_magnitude(d["experts"], d["x"][t], d["top_ids"][t], d["top_w"][t], "swiglu")
        assert_bf16_outputs_close(out[t], ref, mag)
        one = layer.experts_host(d["x"][t], d["top_ids"][t], d["top_w"][t], act="swiglu")
        np.testing.assert_array_equal(one, out[t])
    with pytest.raises(ValueError):
        bad = d["top_ids"].copy()
        bad[2, 1] = bad[2, 0]
        layer.experts_host(d["x"], bad, d["top_w"], act="swiglu")
    layer.close()


def test_experts_grouped_matches_oracle(torch, ctx):
    """``moe_experts_grouped``: routed sums and the shared expert's down rows from
    caller-supplied shared gate|up rows (SiTU), T = 4."""
    d = cases.moe_inputs(hidden=2048, inter=768, experts=16, k=8, tokens=4, seed=63)
    rng = np.random.default_rng(64)
    dn = (rng.standard_normal((2048, 768)) * 0.02).astype(np.float32)
    gu_dummy = (rng.standard_normal((2 * 768, 2048)) * 0.02).astype(np.float32)
    p_dn, f_dn = cases.q4nx_weight(dn, q)
    p_gu, _ = cases.q4nx_weight(gu_dummy, q)
    layer = make_layer(ctx, d, has_shared=True, shared=(p_gu, p_dn))
    shared_gu = q.f32_to_bf16((rng.standard_normal((4, 2 * 768)) * 2).astype(np.float32))
    dev = lambda a, dt: torch.from_numpy(np.ascontiguousarray(a).view(dt)).cuda()
    xd = dev(d["x"], np.int16)
    ids = dev(d["top_ids"].astype(np.int32), np.int32)
    w = dev(d["top_w"].astype(np.float32), np.float32)
    sgu = dev(shared_gu, np.int16)
    routed = torch.empty((4, 2048), dtype=torch.int16, device="cuda")
    shared = torch.empty((4, 2048), dtype=torch.int16, device="cuda")
    layer.experts_grouped(xd, ids, w, 8, routed, sgu, shared, act="situ")
    torch.cuda.synchronize()
    ctx.sync()
    r_ref, s_ref = ob.moe_experts_grouped(d["experts"], f_dn, d["x"], d["top_ids"], d["top_w"], shared_gu,
                                          act="situ")
    got_r = routed.cpu().numpy().view(np.uint16)
    got_s = shared.cpu().numpy().view(np.uint16)
    for t in range(4):
        mag = ob.moe_term_magnitude(d["experts"], d["x"][t], d["top_ids"][t], d["top_w"][t], "situ")
        assert_bf16_outputs_close(got_r[t], r_ref[t], mag)
        assert rms_rel(got_s[t], s_ref[t]) <= 2.0 ** -8
    layer.close()


# ------------------------------------------------------------- robustness --
@pytest.mark.parametrize("T", [3, 40])
def test_router_ranks_nan_logits_last(torch, ctx, T):
    """Experts whose router row holds a NaN get NaN logits; like numpy's stable
    argsort of the negated values they rank after every number, among
    themselves by index (T = 3: decode router, T = 40: prefill router)."""
    layer, wr, rng = _router_layer(ctx, 256, 64, seed=83)
    wr = wr.copy()
    for e in (0, 1, 5, 9, 33):
        wr[e, 7] = 0x7FC0
    layer.set_router(wr)
    x = q.f32_to_bf16(rng.standard_normal((T, 256)).astype(np.float32))
    x[T - 1] = 0x7FC0                       # a NaN token row: every logit NaN
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    k = 8
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    layer.route(xd, T, k, ids, w)
    torch.cuda.synchronize()
    ctx.sync()
    for t in range(T):
        ref = ob.topk_lower_index_wins(ob.router_logits(x[t], wr), k)
        np.testing.assert_array_equal(ids[t].cpu().numpy(), ref)
    np.testing.assert_array_equal(ids[T - 1].cpu().numpy(), np.arange(k))
    layer.close()


def test_caller_expert_id_out_of_range_is_an_error(torch, ctx):
    """Device-side routes are not validated on the host: an out-of-range id
    sets the device error word and the next synchronisation raises."""
    d = cases.moe_inputs(**cases.MOE_CASE)
    layer = make_layer(ctx, d)
    xd = torch.from_numpy(d["x"][:2].view(np.int16)).cuda()
    ids = torch.tensor([[0, 1, 2], [3, 99, 4]], dtype=torch.int32, device="cuda")
    w = torch.full((2, 3), 0.3, dtype=torch.float32, device="cuda")
    out = torch.empty((2, 256), dtype=torch.int16, device="cuda")
    layer.experts(xd, ids, w, 3, out, act="situ")
    torch.cuda.synchronize()
    with pytest.raises(ValueError):
        ctx.sync()
    layer.prefill_experts(xd, ids, w, 3, out, act="situ")
    torch.cuda.synchronize()
    with pytest.raises(ValueError):
        ctx.sync()
    ctx.sync()                              # the word was reported and cleared
    layer.close()


def test_residual_add_kernels_match_numpy(torch, ctx):
    from raon_npu_b200.device import add_bf16, add_rms_bf16
    rng = np.random.default_rng(9)
    a = q.f32_to_bf16(rng.standard_normal((3, 2048)).astype(np.float32))
    b = q.f32_to_bf16((rng.standard_normal((3, 2048)) * 3).astype(np.float32))
    ad, bd = (torch.from_numpy(v.view(np.int16)).cuda() for v in (a, b))
    out = torch.empty_like(ad)
    add_bf16(ctx, ad, bd, out)
    torch.cuda.synchronize()
    s = q.bf16_to_f32(a) + q.bf16_to_f32(b)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint16), q.f32_to_bf16(s))
    add_rms_bf16(ctx, ad, bd, out)
    torch.cuda.synchronize()
    ctx.sync()
    ref = s / np.sqrt(np.mean(s.astype(np.float64) ** 2, axis=1, keepdims=True) + 1e-6)
    got = q.bf16_to_f32(out.cpu().numpy().view(np.uint16))
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 1e-3)) <= 2 ** -7


# ------------------------------------------------ fused decode kernel --
def _decode_both_paths(torch, layer, xd, k, **kw):
    """(out, ids, w) of rc_moe_decode through the fused kernel and through the
    separate launches."""
    T = xd.shape[0]
    res = []
    for fused in (True, False):
        layer.set_fused(fused)
        out = torch.full((T, layer.hidden), 0x7FC0, dtype=torch.int16, device="cuda")
        ids = torch.full((T, k), -7, dtype=torch.int32, device="cuda")
        w = torch.full((T, k), float("nan"), dtype=torch.float32, device="cuda")
        layer.decode(xd, k, out, ids, w, **kw)
        torch.cuda.synchronize()
        res.append((out, ids, w))
    layer.set_fused(True)
    return res


@pytest.mark.parametrize("T", [1, 3, 8, 9, 16])
@pytest.mark.parametrize("router", ["softmax", "sigmoid_bias"])
def test_fused_decode_equals_separate_launches(torch, ctx, T, router):
    """The persistent fused decode kernel (router, gate/up, down, combine in one
    cooperative launch) gives exactly the bytes of the separate launches:
    outputs, top-k ids and weights, for 1..16 tokens and both routers."""
    layer, wr, _ = _config3_layer(torch, ctx)
    if router == "sigmoid_bias":
        rng_b = np.random.default_rng(31)
        layer.set_router(wr, (rng_b.standard_normal(128) * 0.01).astype(np.float32))
    rng = np.random.default_rng(200 + T)
    x = q.f32_to_bf16(rng.standard_normal((T, 2048)).astype(np.float32))
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    kw = dict(act="swiglu", router=router)
    if router == "sigmoid_bias":
        kw.update(renormalize=True, scaling=2.5)
    (fo, fi, fw), (so, si, sw) = _decode_both_paths(torch, layer, xd, 8, **kw)
    ctx.sync()
    assert torch.equal(fi, si)
    assert torch.equal(fw, sw)
    assert torch.equal(fo, so)
    layer.close()


@pytest.mark.parametrize("ranks,M", [(2, 1), (4, 4)])
def test_fused_decode_local_equals_separate_launches(torch, ctx, ranks, M):
    """Expert-parallel local halves: slot rows (zeros where another rank computes)
    and slot weights identical between the fused kernel and the separate
    launches."""
    E = 32
    T = ranks * M
    per = E // ranks
    rng = np.random.default_rng(300 + ranks)
    x = q.f32_to_bf16(rng.standard_normal((T, 2048)).astype(np.float32))
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    for r in range(ranks):
        layer, _, _ = _config3_layer(torch, ctx, n_experts=E, seed=96, owned=set(range(r * per, (r + 1) * per)) | {E})
        got = []
        for fused in (True, False):
            layer.set_fused(fused)
            slots = torch.full((T, 9, 2048), 0x7FC0, dtype=torch.int16, device="cuda")
            sw = torch.full((T, 8), float("nan"), dtype=torch.float32, device="cuda")
            layer.decode_local(xd, 8, slots, sw, experts=(r * per, (r + 1) * per), shared_tokens=(r * M, M),
                               act="situ")
            torch.cuda.synchronize()
            got.append((slots, sw))
        ctx.sync()
        assert torch.equal(got[0][1], got[1][1]), r
        assert torch.equal(got[0][0], got[1][0]), r
        layer.close()


@pytest.mark.parametrize("hidden,inter,E,k,T", [(512, 192, 8, 2, 5), (256, 64, 4, 4, 16), (2048, 768, 256, 16, 16),
                                                 (4096, 1536, 64, 6, 2)])
def test_fused_decode_edge_shapes(torch, ctx, hidden, inter, E, k, T):
    """Shapes at the fused kernel's edges: fewer experts than CTAs, padded
    intermediate size, k = E, the largest E / k / T, a wide hidden size."""
    layer, wr, _ = _config3_layer(torch, ctx, n_experts=E, hidden=hidden, inter=inter, seed=97)
    rng = np.random.default_rng(hidden + E)
    x = q.f32_to_bf16(rng.standard_normal((T, hidden)).astype(np.float32))
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    (fo, fi, fw), (so, si, sw) = _decode_both_paths(torch, layer, xd, k, act="swiglu")
    ctx.sync()
    assert torch.equal(fi, si)
    assert torch.equal(fw, sw)
    assert torch.equal(fo, so)
    layer.close()


@pytest.mark.parametrize("T", [1, 5, 16, 40, 300])
def test_host_entry_points_equal_device_calls(torch, ctx, T):
    """rc_moe_decode_host / rc_moe_prefill_host (and ExpertParallelMoe's host
    entry on one GPU) give the bytes, ids and weights of the device calls."""
    from raon_npu_b200.expert_parallel import ExpertParallelMoe
    E, k = 32, 8
    layer, _, _ = _config3_layer(torch, ctx, n_experts=E, seed=98)
    rng = np.random.default_rng(700 + T)
    x = q.f32_to_bf16(rng.standard_normal((T, 2048)).astype(np.float32))
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    out = torch.empty((T, 2048), dtype=torch.int16, device="cuda")
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    w = torch.empty((T, k), dtype=torch.float32, device="cuda")
    entries = ([("decode", layer.decode, layer.decode_host)] if T <= 16 else []) + \
        [("prefill", layer.prefill, layer.prefill_host)]
    host_out = {}
    for name, dev_call, host_call in entries:
        dev_call(xd, k, out, ids, w, act="situ", router="sigmoid_bias", scaling=1.5)
        torch.cuda.synchronize()
        ctx.sync()
        ho, hi, hw = host_call(x, k, routes=True, act="situ", router="sigmoid_bias", scaling=1.5)
        np.testing.assert_array_equal(ho, out.cpu().numpy().view(np.uint16), err_msg=name)
        np.testing.assert_array_equal(hi, ids.cpu().numpy(), err_msg=name)
        np.testing.assert_array_equal(hw, w.cpu().numpy(), err_msg=name)
        np.testing.assert_array_equal(host_call(x, k, act="situ", router="sigmoid_bias", scaling=1.5), ho,
                                      err_msg=name)
        host_out[name] = ho
    ep = ExpertParallelMoe(layer, k, act="situ", router="sigmoid_bias", scaling=1.5)
    if T <= 16:
        np.testing.assert_array_equal(ep.decode_host(x), host_out["decode"])
    np.testing.assert_array_equal(ep.prefill_host(x), host_out["prefill"])
    with pytest.raises(ValueError):
        layer.decode_host(np.zeros((17, 2048), np.uint16), k)
    with pytest.raises(ValueError):
        layer.decode_host(np.zeros((1, 1024), np.uint16), k)
    layer.close()
