"""Generate golden fixtures by running the reference's own CPU code.

Run from the repository root where the reference checkout is readable:

    RAON_REFERENCE=/path/to/raon-npu python tests/golden/make_golden.py

It imports the reference's ``quant.q4nx``, ``quant.bfp16``,
``kernels/gemv_bfp16/reference.py``, ``host.backend.NumpyBackend``,
``host.raon.RaonModel._route_token`` and ``kernels.moe_grouped.planner`` and
records their outputs on seeded inputs into ``tests/golden/*.npz``.  The tests
regenerate the same inputs from the seeds recorded here and check the oracle
(and through it the CUDA path) against these outputs.  The reference is never
needed at test time.
"""

from __future__ import annotations

import hashlib
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = os.environ.get("RAON_REFERENCE", "")
if not REF or not Path(REF).is_dir():
    raise SystemExit("set RAON_REFERENCE to the reference checkout")
sys.path.insert(0, REF)

from quant import q4nx as rq  # noqa: E402
from host.backend import NumpyBackend  # noqa: E402
from host.weights import Weights  # noqa: E402
from host.raon import RaonConfig, RaonModel  # noqa: E402
from kernels.moe_grouped.planner import build_plan, scatter_b2  # noqa: E402
from serve.engine import GenOptions, sample_token  # noqa: E402

sys.path.insert(0, str(HERE.parent.parent))
from tests.golden.cases import (  # noqa: E402
    QUANT_CASES, LINEAR_CASES, MOE_CASE, ROUTER_CASE, COMBINE_CASE, SAMPLE_CASES, BFP16_CASES,
    TINY_MODEL_CONFIG, TINY_MODEL_TOKENS,
    quant_input, linear_inputs, moe_inputs, router_inputs, combine_inputs, sample_inputs, bfp16_input,
    tiny_model,
)


class _Tensors(Weights):
    """In-memory weight store (the reference's own test double pattern)."""

    def __init__(self, tensors):
        self.tensors = dict(tensors)
        self.selected_layers = None
        self.load_global = True
        self.skip_moe_experts = False
        self._f32_cache = {}


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


def make_quant():
    out = {}
    for name, (n, k, seed, kind) in QUANT_CASES.items():
        w = quant_input(n, k, seed, kind)
        c, s, m = rq.quantize(w)
        packed = rq.pack_gemv(c, s, m)
        deq = rq.dequantize_simple(*rq.parse_gemv(packed, K=k, M=n))
        out[f"{name}/codes_sha"] = np.array(sha(c.tobytes()))
        out[f"{name}/scales"] = s
        out[f"{name}/mins"] = m
        out[f"{name}/packed_sha"] = np.array(sha(packed))
        out[f"{name}/deq_sha"] = np.array(sha(deq.astype(np.float32).tobytes()))
    np.savez_compressed(HERE / "quant.npz", **out)


def make_linear():
    out = {}
    for name, case in LINEAR_CASES.items():
        w_f32, x, bias = linear_inputs(**case, q=rq)
        tensors = {"w.weight": w_f32}
        if bias is not None:
            tensors["w.bias"] = bias
        y = NumpyBackend(_Tensors(tensors)).linear("w.weight", x)
        out[f"{name}/y"] = y
    np.savez_compressed(HERE / "linear.npz", **out)


def make_moe():
    d = moe_inputs(**MOE_CASE, q=rq)
    tensors = {}
    for e, (wg, wu, wd) in d["experts"].items():
        tensors[f"model.layers.0.moe.experts.{e}.gate_proj.weight"] = wg
        tensors[f"model.layers.0.moe.experts.{e}.up_proj.weight"] = wu
        tensors[f"model.layers.0.moe.experts.{e}.down_proj.weight"] = wd
    be = NumpyBackend(_Tensors(tensors))
    out = {}
    for t in range(d["x"].shape[0]):
        out[f"tok{t}/default"] = be.moe_experts(0, d["x"][t], d["top_ids"][t], d["top_w"][t])
        out[f"tok{t}/betas"] = be.moe_experts(0, d["x"][t], d["top_ids"][t], d["top_w"][t],
                                              gate_beta=2.0, value_beta=10.0)
    np.savez_compressed(HERE / "moe.npz", **out)


class _FakeModel:
    """Just enough of RaonModel for ``_route_token``."""

    class _Cfg:
        pass

    def __init__(self, router_w, bias, k, scaling):
        self._c = {"router_weight": router_w, "router_bias": bias}
        self.config = self._Cfg()
        self.config.num_experts_per_token = k
        self.config.moe_renormalize = True
        self.config.routed_scaling_factor = scaling

    def _layer_constants(self, layer_idx):
        return self._c


def make_router():
    d = router_inputs(**ROUTER_CASE)
    fake = _FakeModel(d["router_w_f32"], d["bias"], d["k"], d["scaling"])
    out = {}
    for t in range(d["x"].shape[0]):
        top, w, logits = RaonModel._route_token(fake, 0, d["x"][t])
        out[f"tok{t}/top"] = np.asarray(top)
        out[f"tok{t}/w"] = np.asarray(w, np.float32)
        out[f"tok{t}/logits"] = np.asarray(logits, np.float32)
    np.savez_compressed(HERE / "router.npz", **out)


def make_combine():
    d = combine_inputs(**COMBINE_CASE)
    plan = build_plan(d["top_ids"], include_shared=True)
    # Lay the per-(token, route) rows out in the planner's call/slot/row order.
    outputs = []
    for call in plan.calls:
        arr = np.zeros((8, 8, d["rows"].shape[-1]), np.uint16)
        for slot, job in enumerate(call.jobs):
            if job is None:
                continue
            for r, item in enumerate(job.assignments):
                arr[slot, r] = d["shared"][item.token] if job.shared else d["rows"][item.token, item.route]
        outputs.append(arr)
    routed, shared = scatter_b2(plan, outputs, d["top_ids"], d["top_w"])
    np.savez_compressed(HERE / "combine.npz", routed=routed, shared=shared)


def make_sample():
    """serve.engine.sample_token on seeded logits: 20 draws per case (generator
    seeds s, s+1, ...)."""
    out = {}
    for name, (vocab, seed, kind, opts) in SAMPLE_CASES.items():
        logits, seen, gseed = sample_inputs(vocab, seed, kind)
        o = GenOptions(**opts)
        out[f"{name}/tokens"] = np.array(
            [sample_token(logits, seen, o, np.random.default_rng(gseed + i)) for i in range(20)], np.int64)
    np.savez_compressed(HERE / "sample.npz", **out)


def make_bfp16():
    """quant/bfp16.py's codec and GEMV packing, and kernels/gemv_bfp16/
    reference.py's bit-level GEMV model, on seeded matrices.  The reference
    module is loaded from its file (its package imports the NPU toolchain)."""
    import importlib.util
    import warnings
    from quant import bfp16 as rb
    spec = importlib.util.spec_from_file_location("gemv_bfp16_reference",
                                                  Path(REF) / "kernels/gemv_bfp16/reference.py")
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    out = {}
    for name, (n, k, seed, kind, t) in BFP16_CASES.items():
        w, x = bfp16_input(n, k, seed, kind, t)
        enc = rb.bfp16ebs8_encode(w)
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            packed, stats = rb.pack_bfp16_gemv(w, return_stats=True)
        e, m = rb.parse_bfp16_gemv_raw(packed, K=k, M=n)
        out[f"{name}/encode_sha"] = np.array(sha(enc.tobytes()))
        out[f"{name}/packed_sha"] = np.array(sha(packed))
        out[f"{name}/exponents"] = e
        out[f"{name}/mantissas_sha"] = np.array(sha(m.tobytes()))
        out[f"{name}/flushed"] = np.array(stats["flushed_nonzero_blocks"])
        out[f"{name}/y"] = np.stack([ref.bfp16_gemv_bit_reference(w, (x[i].astype(np.uint32) << 16).view(
            np.float32))[1] for i in range(t)])
    np.savez_compressed(HERE / "bfp16.npz", **out)


class _RecordingBackend(NumpyBackend):
    """NumpyBackend that records the path calls the model makes: every
    ``linear`` and ``moe_experts`` call with its inputs and output (the
    experts' own linears inside ``moe_experts`` are not separate calls)."""

    def __init__(self, weights):
        super().__init__(weights)
        self.calls = []
        self._inside_moe = False

    def linear(self, name, x):
        y = super().linear(name, x)
        if not self._inside_moe:
            self.calls.append({"kind": "linear", "name": name, "x": np.array(x), "y": np.array(y)})
        return y

    def moe_experts(self, layer, x, top_ids, top_weights, gate_beta=4.0, value_beta=25.0, shared_gu=None):
        self._inside_moe = True
        try:
            y = super().moe_experts(layer, x, top_ids, top_weights, gate_beta=gate_beta, value_beta=value_beta,
                                    shared_gu=shared_gu)
        finally:
            self._inside_moe = False
        self.calls.append({"kind": "moe", "layer": layer, "x": np.array(x), "y": np.array(y),
                           "top": np.array(top_ids), "w": np.array(top_weights, np.float32),
                           "betas": np.array([gate_beta, value_beta], np.float64)})
        return y


def make_tiny_model():
    """``RaonModel.step`` (host/raon.py:856-933) over TINY_MODEL_TOKENS on the
    tiny model's q4nx weights, NumpyBackend computing: every path call of every
    step (inputs, outputs, the model's own sigmoid+bias routes), each MoE
    layer's output (``_moe_token``: routed + shared, host/raon.py:1293-1330)
    and the step's logits."""
    m = tiny_model(rq)
    cfg = RaonConfig.from_dict(dict(TINY_MODEL_CONFIG))
    be = _RecordingBackend(_Tensors(m["host"]))
    model = RaonModel(cfg, _Tensors(m["host"]), be)
    moe_token = model._moe_token
    layer_out = []

    def recording_moe_token(layer_idx, hidden, shared_gate_up=None):
        res = moe_token(layer_idx, hidden, shared_gate_up)
        layer_out.append(np.array(res[0]))
        return res
    model._moe_token = recording_moe_token
    out = {"bundles_sha": np.array(sha(b"".join(m["bundles"][n][0] for n in sorted(m["bundles"])))),
           "experts_sha": np.array(sha(b"".join(m["experts"][L][e][i] for L in sorted(m["experts"])
                                                for e in sorted(m["experts"][L]) for i in (0, 1))))}
    starts = []
    for s_i, tok in enumerate(TINY_MODEL_TOKENS):
        starts.append(len(be.calls))
        out[f"step{s_i}/logits"] = np.asarray(model.step(tok), np.float32)
    starts.append(len(be.calls))
    out["step_starts"] = np.array(starts, np.int32)
    # one flat array of every call's input and one of its output, with offsets
    xs = [c["x"].reshape(-1) for c in be.calls]
    ys = [c["y"].reshape(-1) for c in be.calls]
    out["x_flat"], out["y_flat"] = np.concatenate(xs), np.concatenate(ys)
    out["x_off"] = np.cumsum([0] + [a.size for a in xs]).astype(np.int32)
    out["y_off"] = np.cumsum([0] + [a.size for a in ys]).astype(np.int32)
    out["name"] = np.array([c.get("name", "") for c in be.calls])
    moe = [i for i, c in enumerate(be.calls) if c["kind"] == "moe"]
    assert len(moe) == len(layer_out)
    out["moe_call"] = np.array(moe, np.int32)
    out["moe_layer"] = np.array([be.calls[i]["layer"] for i in moe], np.int32)
    out["moe_top"] = np.stack([be.calls[i]["top"] for i in moe]).astype(np.int32)
    out["moe_w"] = np.stack([be.calls[i]["w"] for i in moe])
    out["moe_betas"] = np.stack([be.calls[i]["betas"] for i in moe])
    out["moe_layer_out"] = np.stack(layer_out)
    np.savez_compressed(HERE / "tiny_model.npz", **out)


if __name__ == "__main__":
    make_tiny_model()
    make_bfp16()
    make_sample()
    make_quant()
    make_linear()
    make_moe()
    make_router()
    make_combine()
    for p in sorted(HERE.glob("*.npz")):
        print(p.name, p.stat().st_size)
