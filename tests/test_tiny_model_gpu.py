"""The reference's host model on the tiny q4nx checkpoint, its path calls
replayed through ``CudaBackend`` on the GPU.

``tests/golden/tiny_model.npz`` holds what ``RaonModel.step`` (host/raon.py:
856-933) did over six decode steps of the tiny three-layer model (RDA + dense
MLP, MLA + MoE, RDA + MoE; 8 experts, top-2, one shared expert; sigmoid+bias
router with routed scaling 1.5; SiTU betas 2 / 9) with NumpyBackend
computing: every ``linear`` call (attention projections with K padded to
256, the dense MLP, the shared experts as row slices of their [gate; up]
bundle, the lm_head), every ``moe_experts`` call with the model's own routes,
and each MoE layer's ``_moe_token`` output.  The reference's model code does
not run here; its calls do, in the model's order, on the same inputs.

Bars: each linear output as the GEMV bar of tests/test_gemv_gpu.py against
the f32 sums of the same q4nx weights (at most 1 ulp where |y| >= 2^-8 max|y|,
at most 1% of the elements differ) and within 1 ulp of the model's own
output there; the lm_head output is the step's logits.  MoE outputs with the
MoE bars of tests/test_moe_gpu.py.  The device's sigmoid+bias router gives
the model's expert ids in the model's order and its weights within 1e-5
relative; the fused decode layer and the prefill layer (router on the
device, routed experts, shared expert, combine) give the model's
``_moe_token`` output within the MoE bars.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import backend as ob
from oracle import q4nx as q
from tests.golden import cases
from tests.test_gemv_gpu import assert_bf16_close
from tests.test_moe_gpu import assert_bf16_outputs_close, assert_call_rms, ulp_diff

pytestmark = pytest.mark.gpu

FIXTURE = Path(cases.__file__).with_name("tiny_model.npz")
CFG = cases.TINY_MODEL_CONFIG
E, K = CFG["num_experts"], CFG["num_experts_per_token"]
C, I = CFG["hidden_size"], CFG["moe_intermediate_size"]
GATE_BETA, VALUE_BETA = CFG["activation_situ_beta"], CFG["activation_situ_linear_beta"]
SCALING = CFG["routed_scaling_factor"]


@pytest.fixture(scope="module")
def torch():
    import torch as _t
    return _t


@pytest.fixture(scope="module")
def model():
    return cases.tiny_model()


@pytest.fixture(scope="module")
def trace():
    return cases.tiny_model_trace(FIXTURE)


@pytest.fixture(scope="module")
def be(model):
    """CudaBackend holding the tiny model: one bundle per projection (the
    shared experts' gate and up as the two halves of one [gate; up] bundle),
    the MoE layers with their routers and shared experts."""
    from raon_npu_b200.build import build
    build()
    from raon_npu_b200.backend import CudaBackend
    b = CudaBackend(0)
    for name, (packed, n, k) in model["bundles"].items():
        b.register_bundle(name, np.frombuffer(packed, np.uint8), n, k)
    for name, (bundle, r0, r1, k) in model["linears"].items():
        b.map_name(name, bundle, r0, r1, orig_k=k if k != model["bundles"][bundle][2] else None)
    b.tiny_layers = {}
    for layer, experts in model["experts"].items():
        m = b.register_moe_layer(layer, C, I, E, act="situ", has_shared=True)
        for e, (pgu, pdn) in experts.items():
            m.set_expert(e, np.frombuffer(pgu, np.uint8), np.frombuffer(pdn, np.uint8))
        m.set_router(*model["router"][layer])
        b.tiny_layers[layer] = m
    yield b
    b.close()


def _expert_weights(model, layer):
    h = model["host"]
    p = f"model.layers.{layer}.moe"
    return lambda e: tuple(h[f"{p}.{'experts.' + str(e) if e < E else 'shared_experts'}.{m}_proj.weight"]
                           for m in ("gate", "up", "down"))


def test_every_linear_call_of_the_model(be, model, trace):
    h = model["host"]
    n = 0
    for i, c in enumerate(trace["calls"]):
        if c["kind"] != "linear":
            continue
        got = be.linear(c["name"], c["x"])
        assert got.shape == c["y"].shape and got.dtype == np.uint16, (i, c["name"])
        ref32 = ob.linear_f32(h[c["name"]], c["x"])
        assert_bf16_close(got, ref32)
        big = np.abs(ref32) >= np.max(np.abs(ref32)) / 256
        assert ulp_diff(got, c["y"])[big].max(initial=0) <= 1, (i, c["name"])
        n += 1
    assert n == sum(1 for c in trace["calls"] if c["kind"] == "linear")


def test_logits_of_every_step(be, trace):
    """The lm_head call of each step on its recorded final norm: the logits
    within the GEMV bar, and the greedy token wherever the model's top two
    logits are more than two bf16 steps apart."""
    for s, (a, b) in enumerate(trace["steps"]):
        head = trace["calls"][b - 1]
        assert head["name"] == "lm_head.weight"
        got = q.bf16_to_f32(be.linear("lm_head.weight", head["x"]))
        ref = trace["logits"][s]
        d = ulp_diff(q.f32_to_bf16(got), q.f32_to_bf16(ref))
        big = np.abs(ref) >= np.max(np.abs(ref)) / 256
        assert d[big].max(initial=0) <= 1, s
        top2 = np.sort(ref)[-2:]
        if top2[1] - top2[0] > 2 * 2.0 ** (np.floor(np.log2(abs(top2[1]))) - 7):
            assert int(np.argmax(got)) == int(np.argmax(ref)), s


def test_every_moe_call_with_the_models_routes(be, model, trace):
    gots, refs = [], []
    for i, c in enumerate(trace["calls"]):
        if c["kind"] != "moe":
            continue
        assert c["betas"] == (GATE_BETA, VALUE_BETA)
        got = be.moe_experts(c["layer"], c["x"], c["top"], c["w"], gate_beta=c["betas"][0], value_beta=c["betas"][1])
        ex = _expert_weights(model, c["layer"])
        mag = ob.moe_term_magnitude({int(e): ex(int(e)) for e in c["top"]}, c["x"], c["top"], c["w"], "situ",
                                    GATE_BETA, VALUE_BETA)
        assert_bf16_outputs_close(got, c["y"], mag)
        gots.append(got)
        refs.append(c["y"])
    assert len(gots) == 2 * len(trace["steps"])
    assert_call_rms(np.stack(gots), np.stack(refs))


def _layer_inputs(trace, layer):
    calls = [c for c in trace["calls"] if c["kind"] == "moe" and c["layer"] == layer]
    return (np.stack([c["x"] for c in calls]), np.stack([c["top"] for c in calls]),
            np.stack([c["w"] for c in calls]), np.stack([c["layer_out"] for c in calls]))


@pytest.mark.parametrize("layer", [1, 2])
def test_device_router_gives_the_models_routes(torch, be, trace, layer):
    x, top, w, _ = _layer_inputs(trace, layer)
    T = x.shape[0]
    m = be.tiny_layers[layer]
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wd = torch.empty((T, K), dtype=torch.float32, device="cuda")
    m.route(xd, T, K, ids, wd, router="sigmoid_bias", renormalize=CFG["moe_renormalize"], scaling=SCALING)
    torch.cuda.synchronize()
    be.ctx.sync()
    np.testing.assert_array_equal(ids.cpu().numpy(), top)
    np.testing.assert_allclose(wd.cpu().numpy(), w, rtol=1e-5)


@pytest.mark.parametrize("path", ["decode", "prefill"])
@pytest.mark.parametrize("layer", [1, 2])
def test_moe_layer_on_the_device_gives_the_models_moe_token(torch, be, model, trace, layer, path):
    """All six steps' hidden rows of one MoE layer in one call: the device
    routes them (sigmoid+bias, scaling 1.5), runs the routed and shared
    experts with SiTU(2, 9) and combines, against ``_moe_token``."""
    x, top, w, want = _layer_inputs(trace, layer)
    T = x.shape[0]
    m = be.tiny_layers[layer]
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    out = torch.empty((T, C), dtype=torch.int16, device="cuda")
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    wd = torch.empty((T, K), dtype=torch.float32, device="cuda")
    getattr(m, path)(xd, K, out, ids, wd, router="sigmoid_bias", renormalize=CFG["moe_renormalize"],
                     scaling=SCALING, act="situ", gate_beta=GATE_BETA, value_beta=VALUE_BETA)
    torch.cuda.synchronize()
    be.ctx.sync()
    np.testing.assert_array_equal(ids.cpu().numpy(), top)
    got = out.cpu().numpy().view(np.uint16)
    ex = _expert_weights(model, layer)
    shared = ex(E)
    for t in range(T):
        sh = ob.expert_forward(*shared, x[t], "situ", GATE_BETA, VALUE_BETA)
        mag = ob.moe_term_magnitude({int(e): ex(int(e)) for e in top[t]}, x[t], top[t], w[t], "situ",
                                    GATE_BETA, VALUE_BETA, shared_down_u16=sh)
        assert_bf16_outputs_close(got[t], want[t], mag)
    assert_call_rms(got, want)
