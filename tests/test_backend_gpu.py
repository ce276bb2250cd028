"""The reference-facing boundary: ``CudaBackend`` (the ``Backend`` ABC of
host/backend.py:65-204) driven exactly as ``RaonModel`` drives a backend, on
the reference's own recorded outputs and the oracle.

Bars as for the kernels underneath: GEMV outputs within 1 bf16 ulp of the
reference's (where |y| >= 2^-8 max|y|) on at most 1 % of elements, f32
outputs within 1e-4 normwise; MoE outputs within the MoE bar of
tests/test_moe_gpu.py; ``linear_batch`` byte-identical to per-row ``linear``.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import backend as ob
from oracle import q4nx as q
from tests.golden import cases
from tests.test_gemv_gpu import assert_bf16_close, ulp_diff
from tests.test_moe_gpu import assert_bf16_outputs_close, rms_rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from raon_npu_b200.build import build
    build()
    from raon_npu_b200.backend import CudaBackend
    b = CudaBackend(0)
    yield b
    b.close()


# ------------------------------------------------------------------ linear --
def test_linear_matches_reference_fixture(be):
    """NumpyBackend.linear outputs recorded from the reference (bf16 and f32
    inputs, T = 1..16, with and without bias)."""
    g = np.load(cases.__file__.replace("cases.py", "linear.npz"))
    for name, case in cases.LINEAR_CASES.items():
        w_f32, x, b = cases.linear_inputs(**case)
        be.register_q4nx(name, cases.linear_packed(case["n"], case["k"], case["seed"]), case["n"], case["k"],
                         bias=b)
        y = be.linear(name, x)
        ref = g[f"{name}/y"]
        assert y.shape == ref.shape and y.dtype == ref.dtype, name
        if x.dtype == np.float32:
            assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) <= 1e-4, name
        else:
            big = np.abs(q.bf16_to_f32(ref)) >= np.max(np.abs(q.bf16_to_f32(ref))) / 256
            assert ulp_diff(y, ref)[big].max() <= 1, name
            assert_bf16_close(y, ob.linear_f32(w_f32, x, b))
        # one token row as a 1-D vector gives the same bytes as its batch row
        np.testing.assert_array_equal(be.linear(name, x[0]), y[0])


def test_linear_batch_is_rowwise_linear(be):
    """host/backend.py:71-74: linear_batch is byte-identical to stacking linear."""
    n, k = 512, 2048
    rng = np.random.default_rng(3)
    packed, _ = cases.q4nx_weight((rng.standard_normal((n, k)) * 0.02).astype(np.float32), q)
    be.register_q4nx("batch.w", packed, n, k)
    x = q.f32_to_bf16(rng.standard_normal((16, k)).astype(np.float32))
    yb = be.linear_batch("batch.w", x)
    np.testing.assert_array_equal(yb, np.stack([be.linear("batch.w", x[t]) for t in range(16)]))


def test_bundle_row_slices_and_padded_k(be):
    """Several projections in one bundle, addressed by name and row range
    (npu/backend.py:3575-3650); a K zero-padded to 256 accepts the unpadded row."""
    rng = np.random.default_rng(4)
    n, k_real, k_pad = 384, 300, 512
    w = (rng.standard_normal((n, k_real)) * 0.02).astype(np.float32)
    wp, _ = q.pad_gemv(w, m_align=128, k_align=256)
    assert wp.shape == (n, k_pad)
    packed, w_f32 = cases.q4nx_weight(wp, q)
    be.register_bundle("L00/qkv", packed, n, k_pad)
    be.map_name("q_proj", "L00/qkv", 0, 128, orig_k=k_real)
    be.map_name("kv_proj", "L00/qkv", 128, 384, orig_k=k_real)
    x = q.f32_to_bf16(rng.standard_normal((2, k_real)).astype(np.float32))
    full = ob.linear_f32(w_f32[:, :k_real], x)
    assert_bf16_close(be.linear("q_proj", x), full[:, :128])
    assert_bf16_close(be.linear("kv_proj", x), full[:, 128:])
    assert "q_proj" in be and "v_proj" not in be


def test_linear_errors(be):
    with pytest.raises(KeyError):
        be.linear("no.such.weight", np.zeros(256, np.uint16))
    n, k = 128, 256
    packed, _ = cases.q4nx_weight(np.ones((n, k), np.float32) * 0.01, q)
    be.register_q4nx("err.w", packed, n, k)
    with pytest.raises(ValueError):
        be.linear("err.w", np.zeros(k, np.float64))
    with pytest.raises(ValueError):
        be.linear("err.w", np.zeros(k + 1, np.uint16))


# ------------------------------------------------------------------- MoE --
def _moe_backend_layer(be, layer, d, act, shared=None):
    e0 = next(iter(d["packed"]))
    hidden = d["experts"][e0][2].shape[0]
    inter = d["experts"][e0][0].shape[0]
    E = len(d["packed"])
    be.register_moe_layer(layer, hidden, inter, E, act=act, has_shared=shared is not None)
    for e, (pgu, pdn) in d["packed"].items():
        be.register_moe_expert(layer, e, pgu, pdn)
    if shared is not None:
        be.register_moe_expert(layer, E, *shared)


def test_moe_experts_matches_reference_fixture(be):
    """NumpyBackend.moe_experts recorded from the reference (SiTU, default and
    custom betas), through the ABC call RaonModel makes."""
    g = np.load(cases.__file__.replace("cases.py", "moe.npz"))
    d = cases.moe_inputs(**cases.MOE_CASE)
    _moe_backend_layer(be, 3, d, "situ")
    for t in range(d["x"].shape[0]):
        for tag, kw in (("default", {}), ("betas", dict(gate_beta=2.0, value_beta=10.0))):
            out = be.moe_experts(3, d["x"][t], d["top_ids"][t], d["top_w"][t], **kw)
            mag = ob.moe_term_magnitude(d["experts"], d["x"][t], d["top_ids"][t], d["top_w"][t], "situ", **kw)
            assert out.dtype == np.uint16 and out.shape == (d["x"].shape[1],)
            assert_bf16_outputs_close(out, g[f"tok{t}/{tag}"], mag)
    # f32 token rows are rounded to bf16 first
    xf = q.bf16_to_f32(d["x"][0])
    np.testing.assert_array_equal(be.moe_experts(3, xf, d["top_ids"][0], d["top_w"][0]),
                                  be.moe_experts(3, d["x"][0], d["top_ids"][0], d["top_w"][0]))


def test_moe_experts_validation(be):
    d = cases.moe_inputs(**cases.MOE_CASE)
    _moe_backend_layer(be, 4, d, "situ")
    x, ids, w = d["x"][0], d["top_ids"][0], d["top_w"][0]
    with pytest.raises(ValueError):
        be.moe_experts(4, x, np.array([0, 0, 1]), w)           # duplicate expert
    with pytest.raises(ValueError):
        be.moe_experts(4, x, np.array([0, 6, 1]), w)           # out of range
    with pytest.raises(ValueError):
        be.moe_experts(4, x, ids, w.astype(np.float64))        # weight dtype
    with pytest.raises(ValueError):
        be.moe_experts(4, x[:100], ids, w)                     # row length
    with pytest.raises(ValueError):
        be.moe_experts(99, x, ids, w)                          # unknown layer


def test_moe_experts_grouped_matches_oracle(be):
    """moe_experts_grouped for T = 20 tokens (more than 16: the routed experts
    run on the prefill kernels in one call): routed sums and shared down rows
    against the oracle; the routed rows equal the per-token moe_experts bytes,
    and both halves equal a 16-token call (decode kernels) byte for byte."""
    d = cases.moe_inputs(hidden=2048, inter=768, experts=16, k=8, tokens=20, seed=65)
    rng = np.random.default_rng(66)
    gu = (rng.standard_normal((2 * 768, 2048)) * 0.02).astype(np.float32)
    dn = (rng.standard_normal((2048, 768)) * 0.02).astype(np.float32)
    p_gu, _ = cases.q4nx_weight(gu, q)
    p_dn, f_dn = cases.q4nx_weight(dn, q)
    _moe_backend_layer(be, 5, d, "situ", shared=(p_gu, p_dn))
    shared_gu = q.f32_to_bf16((rng.standard_normal((20, 2 * 768)) * 2).astype(np.float32))
    routed, shared = be.moe_experts_grouped(5, d["x"], d["top_ids"], d["top_w"], shared_gu)
    r_ref, s_ref = ob.moe_experts_grouped(d["experts"], f_dn, d["x"], d["top_ids"], d["top_w"], shared_gu,
                                          act="situ")
    for t in range(20):
        mag = ob.moe_term_magnitude(d["experts"], d["x"][t], d["top_ids"][t], d["top_w"][t], "situ")
        assert_bf16_outputs_close(routed[t], r_ref[t], mag)
        assert rms_rel(shared[t], s_ref[t]) <= 2.0 ** -8
    for t in (0, 7, 19):
        np.testing.assert_array_equal(be.moe_experts(5, d["x"][t], d["top_ids"][t], d["top_w"][t]), routed[t])
    r16, s16 = be.moe_experts_grouped(5, d["x"][:16], d["top_ids"][:16], d["top_w"][:16], shared_gu[:16])
    np.testing.assert_array_equal(r16, routed[:16])
    np.testing.assert_array_equal(s16, shared[:16])
    with pytest.raises(ValueError):
        be.moe_experts_grouped(5, d["x"], d["top_ids"], d["top_w"], shared_gu[:, :100])
