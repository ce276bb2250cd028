"""The reference's host model on the tiny q4nx checkpoint, restated call by
call by the oracle (no GPU).

``tests/golden/tiny_model.npz`` records ``RaonModel.step`` (host/raon.py:
856-933) over six tokens of the tiny three-layer model (RDA + dense MLP,
MLA + MoE, RDA + MoE; sigmoid+bias router, SiTU betas 2 / 9) with
NumpyBackend computing: every ``linear`` and ``moe_experts`` call, the
model's own routes and each MoE layer's output.  Here the oracle reproduces
each recorded call bit for bit from the same inputs, so the GPU replay of the
same trace (tests/test_tiny_model_gpu.py) is checked against a pinned oracle.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle import backend as ob
from oracle import q4nx as q
from tests.golden import cases

FIXTURE = Path(cases.__file__).with_name("tiny_model.npz")


@pytest.fixture(scope="module")
def model():
    return cases.tiny_model()


@pytest.fixture(scope="module")
def trace():
    return cases.tiny_model_trace(FIXTURE)


def _experts(model, layer):
    h = model["host"]
    p = f"model.layers.{layer}.moe"
    return lambda e: tuple(h[f"{p}.experts.{e}.{m}_proj.weight"] for m in ("gate", "up", "down"))


def test_oracle_quantiser_reproduces_the_fixture_weights(model, trace):
    b = model["bundles"]
    assert hashlib.sha256(b"".join(b[n][0] for n in sorted(b))).hexdigest() == trace["bundles_sha"]
    ex = model["experts"]
    blob = b"".join(ex[L][e][i] for L in sorted(ex) for e in sorted(ex[L]) for i in (0, 1))
    assert hashlib.sha256(blob).hexdigest() == trace["experts_sha"]


def test_trace_has_the_model_structure(trace):
    """Per step: the three layers' linears (RDA 9 + dense MLP 3, MLA 6 +
    shared expert 3, RDA 9 + shared expert 3), two MoE calls and the lm_head,
    in the model's order; the lm_head output is the step's logits."""
    assert len(trace["steps"]) == len(cases.TINY_MODEL_TOKENS)
    for s, (a, b) in enumerate(trace["steps"]):
        calls = trace["calls"][a:b]
        assert [c["kind"] for c in calls].count("moe") == 2
        assert [c["layer"] for c in calls if c["kind"] == "moe"] == [1, 2]
        assert calls[-1]["name"] == "lm_head.weight"
        np.testing.assert_array_equal(q.bf16_to_f32(calls[-1]["y"]), trace["logits"][s])
        names = [c["name"] for c in calls if c["kind"] == "linear"]
        assert len(names) == 12 + 6 + 3 + 9 + 3 + 1
        for j, c in enumerate(calls):       # the shared expert's three linears follow the routed call
            if c["kind"] == "moe":
                sh = f"model.layers.{c['layer']}.moe.shared_experts"
                assert [d["name"] for d in calls[j + 1:j + 4]] == [f"{sh}.{m}_proj.weight" for m in ("gate", "up", "down")]


def test_oracle_linear_reproduces_every_recorded_call(model, trace):
    h = model["host"]
    for i, c in enumerate(trace["calls"]):
        if c["kind"] == "linear":
            np.testing.assert_array_equal(ob.linear(h[c["name"]], c["x"]), c["y"], err_msg=f"call {i} {c['name']}")


def test_oracle_router_and_experts_reproduce_the_model(model, trace):
    """Routes: the oracle's sigmoid+bias router (ids in the model's order;
    weights within 1e-6 relative, the router pin's bar: the oracle takes the
    sigmoid in f64, the model in f32); outputs: the routed experts with the model's SiTU
    betas, and routed + shared combined as ``_moe_token`` does."""
    cfg = cases.TINY_MODEL_CONFIG
    calls = trace["calls"]
    for i, c in enumerate(calls):
        if c["kind"] != "moe":
            continue
        bits, bias = model["router"][c["layer"]]
        ids, w, _ = ob.route_sigmoid_bias(c["x"], bits, bias, cfg["num_experts_per_token"],
                                          renormalize=cfg["moe_renormalize"], scaling=cfg["routed_scaling_factor"])
        np.testing.assert_array_equal(ids, c["top"])
        np.testing.assert_allclose(w, c["w"], rtol=1e-6)
        ex = _experts(model, c["layer"])
        got = ob.moe_experts({int(e): ex(int(e)) for e in ids}, c["x"], c["top"], c["w"], act="situ",
                             gate_beta=c["betas"][0], value_beta=c["betas"][1])
        np.testing.assert_array_equal(got, c["y"], err_msg=f"call {i}")
        shared_down = calls[i + 3]
        assert shared_down["name"] == f"model.layers.{c['layer']}.moe.shared_experts.down_proj.weight"
        np.testing.assert_array_equal(ob.moe_token_with_shared(c["y"], shared_down["y"]), c["layer_out"])
