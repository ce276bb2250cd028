"""Pin the CPU oracle to the reference: golden hashes, KATs, and fixtures
produced by running the reference itself (``tests/golden/make_golden.py``).

CPU only.  Everything the CUDA tests compare against rests on these pins.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

from oracle import backend as ob
from oracle import q4nx as q
from tests.golden import cases

GOLDEN = Path(__file__).resolve().parent / "golden"


def sha(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()


# ---------------------------------------------------------- published pins --
@pytest.mark.parametrize("m,k,seed,digest,nbytes", [
    # bench/gemv/test_gemv_ref.py:80-95
    (1024, 256, 1234, "008a66c523441448ae9115edf7de8f1e41f891fe88a5581df47dbacd625071ac", 163840),
    (2048, 512, 1234, "0ecb33ce812482f45163d5f5743e3673ea4d5054741da78b8f420d605a20ffc6", 655360),
])
def test_pack_gemv_golden_sha256(m, k, seed, digest, nbytes):
    w = np.random.default_rng(seed).standard_normal((m, k)).astype(np.float32)
    c, s, mn = q.quantize(w)
    blob = q.pack_gemv(c, s, mn, rows=4)
    assert len(blob) == nbytes
    assert sha(blob) == digest
    pc, ps, pm = q.parse_gemv(blob, K=k, M=m)
    np.testing.assert_array_equal(pc, c)
    np.testing.assert_array_equal(ps, s)
    np.testing.assert_array_equal(pm, mn)


def _kat(rows, cols):
    """Known-answer inputs of quant/test_q4nx.py:250-258."""
    n = rows * cols
    codes = ((np.arange(n, dtype=np.int64) * 7 + 3) % 16).astype(np.uint8).reshape(rows, cols)
    i = np.arange(rows * (cols // 32), dtype=np.int64)
    scales = (((i % 97) - 48) * 1e-3).astype(np.float32).reshape(rows, cols // 32)
    mins = (((i % 89) - 44) * 3e-3).astype(np.float32).reshape(rows, cols // 32)
    return codes, scales, mins


@pytest.mark.parametrize("shape,nbytes,digest", [
    # quant/test_q4nx.py:263-268
    ((64, 256), 10240, "2f934f13747e9f5e261c226655ea811bbae8e45ff6784374d6dd31bd91a394fa"),
    ((1088, 2560), 1740800, "155407fbcfd7ba1b3ddd4a242ec7cb16d5725ad201fa001283180f11048af0bc"),
    ((2560, 1280), 2048000, "12846cb24767c9f150311cba31b9186a87df6fdf12d8c517553493be08181fee"),
    ((128, 768), 61440, "7815e5a5b40aafb908cbb0c774914520fed87cbc09a91a72bd76adab59ca5d7f"),
])
def test_pack_decode_proj_kat_sha256(shape, nbytes, digest):
    blob = q.pack_decode_proj(*_kat(*shape))
    assert len(blob) == nbytes
    assert sha(blob) == digest


def test_gemv_hand_calculated_640():
    """bench/gemv/test_gemv_ref.py:204-228: code 3, scale 0.5, min 1 -> w = 2.5; x = 1 -> y = 640."""
    m, k = 128, 256
    blob = q.pack_gemv(np.full((m, k), 3, np.uint8), np.full((m, 8), 0.5, np.float32),
                       np.full((m, 8), 1.0, np.float32))
    w = q.dequantize_packed(blob, m, k)
    np.testing.assert_array_equal(w, np.full((m, k), 2.5, np.float32))
    y = ob.linear(w, q.f32_to_bf16(np.ones(k, np.float32)))
    np.testing.assert_array_equal(q.bf16_to_f32(y), np.full(m, 640.0, np.float32))


def test_rne_boundary_259_rounds_to_260():
    """bench/gemv/test_gemv_ref.py:231-303: a dot of exactly 259 rounds (RNE) to 260, floor gives 258."""
    assert q.bf16_floor(np.float32(259.0)) == 258.0
    assert q.bf16_round(np.float32(259.0)) == 260.0
    m, k = 128, 256
    codes = np.zeros((m, k), np.uint8)
    codes[:, :31] = 8
    codes[:, 31] = 11
    scales = np.zeros((m, 8), np.float32)
    scales[:, 0] = 1.0
    w = q.dequantize_packed(q.pack_gemv(codes, scales, np.zeros((m, 8), np.float32)), m, k)
    y = ob.linear(w, q.f32_to_bf16(np.ones(k, np.float32)))
    np.testing.assert_array_equal(q.bf16_to_f32(y), np.full(m, 260.0, np.float32))


# ---------------------------------------------------- reference fixtures --
@pytest.mark.parametrize("name", list(cases.QUANT_CASES))
def test_quantize_pack_dequant_match_reference(name):
    g = np.load(GOLDEN / "quant.npz")
    n, k, seed, kind = cases.QUANT_CASES[name]
    w = cases.quant_input(n, k, seed, kind)
    c, s, m = q.quantize(w)
    assert sha(c.tobytes()) == str(g[f"{name}/codes_sha"])
    np.testing.assert_array_equal(s, g[f"{name}/scales"])
    np.testing.assert_array_equal(m, g[f"{name}/mins"])
    blob = q.pack_gemv(c, s, m)
    assert sha(blob) == str(g[f"{name}/packed_sha"])
    deq = q.dequantize_packed(blob, n, k)
    assert sha(deq.astype(np.float32).tobytes()) == str(g[f"{name}/deq_sha"])


@pytest.mark.parametrize("name", list(cases.LINEAR_CASES))
def test_linear_matches_reference_numpy_backend(name):
    g = np.load(GOLDEN / "linear.npz")
    w, x, b = cases.linear_inputs(**cases.LINEAR_CASES[name])
    y = ob.linear(w, x, b)
    ref = g[f"{name}/y"]
    assert y.dtype == ref.dtype and y.shape == ref.shape
    if y.dtype == np.float32:
        np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-6)
    else:
        # Both sides are one BLAS f32 dot + RTNE; allow a rare 1-ulp flip from a
        # different BLAS summation order but no more.
        diff = np.abs(y.astype(np.int32) - ref.astype(np.int32))
        assert diff.max() <= 1 and np.count_nonzero(diff) <= max(1, y.size // 200)


def test_moe_experts_matches_reference_numpy_backend():
    g = np.load(GOLDEN / "moe.npz")
    d = cases.moe_inputs(**cases.MOE_CASE)
    for t in range(d["x"].shape[0]):
        for tag, kw in (("default", {}), ("betas", dict(gate_beta=2.0, value_beta=10.0))):
            y = ob.moe_experts(d["experts"], d["x"][t], d["top_ids"][t], d["top_w"][t], act="situ", **kw)
            ref = g[f"tok{t}/{tag}"]
            diff = np.abs(y.astype(np.int32) - ref.astype(np.int32))
            assert diff.max() <= 1 and np.count_nonzero(diff) <= max(1, y.size // 100), (t, tag)


def test_sigmoid_bias_router_matches_reference():
    g = np.load(GOLDEN / "router.npz")
    d = cases.router_inputs(**cases.ROUTER_CASE)
    for t in range(d["x"].shape[0]):
        ids, w, logits = ob.route_sigmoid_bias(d["x"][t], d["router_w_bits"], d["bias"], d["k"],
                                               scaling=d["scaling"])
        np.testing.assert_array_equal(ids, g[f"tok{t}/top"])
        np.testing.assert_allclose(w, g[f"tok{t}/w"], rtol=1e-6)
        np.testing.assert_allclose(logits, g[f"tok{t}/logits"], rtol=1e-5, atol=1e-6)


def test_ascending_id_combine_matches_reference_scatter_b2():
    g = np.load(GOLDEN / "combine.npz")
    d = cases.combine_inputs(**cases.COMBINE_CASE)
    np.testing.assert_array_equal(ob.combine_ascending(d["rows"], d["top_ids"], d["top_w"]), g["routed"])
    np.testing.assert_array_equal(d["shared"], g["shared"])


# ------------------------------------------------- quantiser properties --
def test_quantize_error_within_half_scale():
    """quant/test_q4nx.py:111-131."""
    w = (np.random.default_rng(2026).standard_normal((64, 512)) * 2.5).astype(np.float32)
    c, s, m = q.quantize(w)
    assert c.max() <= 15
    err = np.abs(w - q.dequantize_simple(c, s, m))
    assert np.all(err <= 0.5 * np.repeat(s, 32, axis=1) + 1e-6)


@pytest.mark.parametrize("bad", [np.nan, np.inf, -np.inf])
def test_quantize_rejects_non_finite(bad):
    w = np.ones((32, 64), np.float32)
    w[0, 10] = bad
    with pytest.raises(ValueError, match="non-finite"):
        q.quantize(w)


def test_quantize_validation():
    with pytest.raises(ValueError, match="must be 2D"):
        q.quantize(np.ones(64, np.float32))
    with pytest.raises(ValueError, match="multiple of GROUP"):
        q.quantize(np.ones((32, 45), np.float32))
    with pytest.raises(ValueError, match="multiple of 128"):
        q.pack_gemv(np.zeros((100, 256), np.uint8), np.zeros((100, 8)), np.zeros((100, 8)))
    with pytest.raises(ValueError, match="multiple of K_TILE"):
        q.pack_gemv(np.zeros((128, 200), np.uint8), np.zeros((128, 6)), np.zeros((128, 6)))


def test_exact_constant_groups_have_zero_scale():
    """quant/test_q4nx.py:207-230."""
    w = np.zeros((32, 128), np.float32)
    w[:, 32:64] = 5.0
    w[:, 64:96] = -12.5
    w[:, 96:] = np.linspace(1.0, 10.0, 32, dtype=np.float32)
    c, s, m = q.quantize(w)
    assert np.all(s[:, :3] == 0) and np.all(s[:, 3] > 0) and np.all(c[:, :96] == 0)


def test_padding_invariance():
    """bench/gemv/test_gemv_ref.py:306-345: zero-padded K and N leave the live outputs unchanged."""
    rng = np.random.default_rng(9999)
    w = rng.standard_normal((2100, 576)).astype(np.float32)
    x = rng.standard_normal(576).astype(np.float32)
    wp, shape = q.pad_gemv(w)
    assert wp.shape == (2176, 768) and shape == (2100, 576)
    wdq = q.dequantize_simple(*q.quantize(wp))
    xp = np.zeros(768, np.float32)
    xp[:576] = x
    full = wdq.astype(np.float64) @ xp.astype(np.float64)
    live = wdq[:2100, :576].astype(np.float64) @ x.astype(np.float64)
    np.testing.assert_allclose(full[:2100], live, rtol=1e-12, atol=1e-12)


def test_bf16_directed_rounding():
    """quant/test_q4nx.py:56-103."""
    v = np.array([0.0, -0.0, 1.0, -1.0, 1001.0, 1001.1, -1001.1, 1 + 2 ** -20, 1 - 2 ** -20,
                  -1 - 2 ** -20, 3.3895314e38, -3.3895314e38, 1e-40, -1e-40], np.float32)
    fl, ce = q.bf16_floor(v), q.bf16_ceil(v)
    assert np.all(fl <= v) and np.all(ce >= v)
    assert np.all(q.bf16_round(fl) == fl) and np.all(q.bf16_round(ce) == ce)
    inexact = fl != ce
    assert np.all(q.bf16_next_up(fl[inexact]) == ce[inexact])
    v64 = np.array([1001.1, -1001.1, 1e-10, -1e-10, 1.23456789012345])
    assert np.all(np.asarray(q.bf16_floor(v64), np.float64) <= v64)
    assert np.all(np.asarray(q.bf16_ceil(v64), np.float64) >= v64)


def test_softmax_topk_lower_index_wins_ties():
    logits = np.array([0.5, 2.0, 2.0, -1.0, 2.0, 0.5], np.float32)
    np.testing.assert_array_equal(ob.topk_lower_index_wins(logits, 4), [1, 2, 4, 0])


# ---------------------------------------------------------------- sampler --
@pytest.mark.parametrize("name", list(cases.SAMPLE_CASES))
def test_sampler_restatement_matches_reference_draws(name):
    """serve/engine.py:84-140 run by the reference (tests/golden/sample.npz,
    20 generator seeds per case) vs the oracle's restatement fed the same
    generator's uniform draw."""
    from oracle.sampling import sample_token_u
    g = np.load(Path(cases.__file__).with_name("sample.npz"))
    vocab, seed, kind, opts = cases.SAMPLE_CASES[name]
    logits, seen, gseed = cases.sample_inputs(vocab, seed, kind)
    got = [sample_token_u(logits, seen, opts["top_k"], opts["top_p"], opts["temperature"],
                          opts["presence_penalty"], np.random.default_rng(gseed + i).random()) for i in range(20)]
    np.testing.assert_array_equal(got, g[f"{name}/tokens"])


# ------------------------------------------------- spread of the MoE bar --
def _moe_layer_rows(x, experts, shared, ids, w, f64_dots: bool):
    """The oracle's MoE layer (bf16 roundings of gate, up, activation, down;
    ascending-ID f32 combine; shared expert added) with every GEMV's dot
    products in f32 (numpy, as NumpyBackend) or in f64 rounded to f32."""
    def lin(wm, xb):
        xf = q.bf16_to_f32(xb)
        y = np.dot(xf.astype(np.float64), wm.T.astype(np.float64)).astype(np.float32) if f64_dots \
            else np.dot(xf, wm.T)
        return q.f32_to_bf16(y.astype(np.float32))

    def expert(e, xb):
        wg, wu, wd = experts[e] if e >= 0 else shared
        return lin(wd, q.f32_to_bf16(ob.glu(lin(wg, xb), lin(wu, xb), "swiglu")))
    out = []
    for t in range(x.shape[0]):
        acc = np.zeros(x.shape[1], np.float32)
        for r in np.argsort(ids[t], kind="stable"):
            acc += q.bf16_to_f32(expert(int(ids[t, r]), x[t])) * np.float32(w[t, r])
        out.append(ob.moe_token_with_shared(q.f32_to_bf16(acc), expert(-1, x[t])))
    return np.stack(out)


def test_moe_outputs_of_two_summation_orders_differ_within_the_bars():
    """Two correct restatements of the MoE layer that differ only in the order
    of the f32 sums (numpy f32 dot products vs f64 ones rounded to f32) give
    different bf16 outputs -- the bf16 roundings turn 1e-7 differences into
    one-step flips -- and stay inside the bars the GPU MoE tests apply."""
    from tests.test_moe_gpu import CALL_RMS, MAX_NORMWISE, ROW_RMS
    rng = np.random.default_rng(5)
    H, I, E, k, T = 2048, 768, 16, 8, 24

    def bfw(shape):
        return q.bf16_to_f32(q.f32_to_bf16((rng.standard_normal(shape) * 0.02).astype(np.float32)))
    experts = {e: (bfw((I, H)), bfw((I, H)), bfw((H, I))) for e in range(E)}
    shared = (bfw((I, H)), bfw((I, H)), bfw((H, I)))
    x = q.f32_to_bf16(rng.standard_normal((T, H)).astype(np.float32))
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)])
    w = rng.uniform(0.05, 0.3, (T, k)).astype(np.float32)
    a = _moe_layer_rows(x, experts, shared, ids, w, f64_dots=False)
    b = _moe_layer_rows(x, experts, shared, ids, w, f64_dots=True)
    af, bf = (q.bf16_to_f32(v).astype(np.float64) for v in (a, b))
    err = np.abs(af - bf)
    assert (a != b).any()                       # not bit-exact across summation orders
    row_rms = np.sqrt((err ** 2).mean(axis=1)) / np.sqrt((bf ** 2).mean(axis=1))
    assert row_rms.max() <= ROW_RMS
    assert np.sqrt((err ** 2).mean()) / np.sqrt((bf ** 2).mean()) <= CALL_RMS
    assert (err.max(axis=1) / np.abs(bf).max(axis=1)).max() <= MAX_NORMWISE
