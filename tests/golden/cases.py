"""Seeded input generators shared by ``make_golden.py`` (run against the
reference) and the tests (run against the oracle and the CUDA path).

Only numpy's seeded generator is used here; quantisation is done by whichever
q4nx module the caller passes (the reference's when making fixtures, the
oracle's in tests), so the fixtures also check that the two agree.
"""

from __future__ import annotations

import numpy as np

# name -> (rows N, cols K, seed, kind)
QUANT_CASES = {
    "normal_128x256": (128, 256, 11, "normal"),
    "normal_256x512": (256, 512, 12, "normal"),
    "wide_128x768": (128, 768, 13, "wide"),
    "edge_128x256": (128, 256, 14, "edge"),
}

# name -> kwargs of linear_inputs
LINEAR_CASES = {
    "t1_256x512": dict(n=256, k=512, t=1, seed=21, x_kind="bf16", bias=False),
    "t3_384x256": dict(n=384, k=256, t=3, seed=22, x_kind="bf16", bias=False),
    "t16_128x768": dict(n=128, k=768, t=16, seed=23, x_kind="bf16", bias=False),
    "f32_t2_256x256": dict(n=256, k=256, t=2, seed=24, x_kind="f32", bias=False),
    "bias_t1_128x512": dict(n=128, k=512, t=1, seed=25, x_kind="bf16", bias=True),
}

MOE_CASE = dict(hidden=256, inter=256, experts=6, k=3, tokens=3, seed=31)

# Sampler (serve/engine.py:84-140): name -> (vocab, seed, logit kind, options)
SAMPLE_CASES = {
    "vocab_k50_p09": (151936, 301, "normal", dict(temperature=1.0, top_p=0.9, top_k=50, presence_penalty=0.0)),
    "vocab_penalty": (151936, 302, "normal", dict(temperature=1.0, top_p=0.9, top_k=50, presence_penalty=1.5)),
    "temp07_k20_p095": (151936, 303, "normal", dict(temperature=0.7, top_p=0.95, top_k=20, presence_penalty=0.0)),
    "greedy_penalty": (151936, 304, "normal", dict(temperature=0.0, top_p=0.9, top_k=50, presence_penalty=1.5)),
    "ties_k5": (4096, 305, "ties", dict(temperature=1.0, top_p=0.99, top_k=5, presence_penalty=0.0)),
    "small_p05": (1000, 306, "normal", dict(temperature=1.3, top_p=0.5, top_k=100, presence_penalty=0.5)),
    "no_topk_p09": (3000, 307, "normal", dict(temperature=1.0, top_p=0.9, top_k=0, presence_penalty=0.0)),
}
ROUTER_CASE = dict(hidden=256, experts=16, k=4, tokens=8, seed=41, scaling=2.5)
# bfp16ebs8 (quant/bfp16.py): name -> (rows N, cols K, seed, kind, GEMV rows x)
BFP16_CASES = {
    "normal_128x256": (128, 256, 61, "normal", 3),
    "normal_256x512": (256, 512, 62, "normal", 2),
    "edge_128x512": (128, 512, 63, "edge", 3),
}
COMBINE_CASE = dict(tokens=20, k=4, hidden=64, seed=51)


def _bf16_bits(a: np.ndarray) -> np.ndarray:
    """RTNE f32 -> bf16 bits (the arithmetic both sides define identically)."""
    a = np.ascontiguousarray(a, np.float32)
    b = a.view(np.uint32).astype(np.uint64)
    return (((b + 0x7FFF + ((b >> 16) & 1)) >> 16) & 0xFFFF).astype(np.uint16)


def quant_input(n: int, k: int, seed: int, kind: str) -> np.ndarray:
    rng = np.random.default_rng(seed)
    if kind == "normal":
        return (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    if kind == "wide":
        w = (rng.standard_normal((n, k)) * 2.5).astype(np.float32)
        w[::7, 32:64] = 5.0                     # exact bf16 constant group
        w[1::7, 64:96] = 0.1                    # inexact constant group
        w[2::7, 96:128] = np.linspace(1001.0, 1001.1, 32, dtype=np.float32)
        w[3::7, 128:160] = np.linspace(-1001.1, -1001.0, 32, dtype=np.float32)
        return w
    if kind == "edge":
        w = rng.uniform(-1, 1, (n, k)).astype(np.float32)
        w[:, 0:32] = 0.0
        w[:, 32:64] = -12.5
        w[0, 64] = -3e38
        w[0, 65] = 3e38
        w[0, 66:96] = np.linspace(-1e38, 1e38, 30, dtype=np.float32)
        w[1, 96:128] = 1e-40                    # subnormal constant group
        return w
    raise ValueError(kind)


def bfp16_input(n: int, k: int, seed: int, kind: str, t: int) -> tuple[np.ndarray, np.ndarray]:
    """(f32 weights [n, k], bf16 bit rows x [t, k]) for a bfp16ebs8 case.  The
    edge kind mixes groups that round up to +128 (exponent carry), reach -128,
    are all zero, or are tiny enough for the layout's exponent floor."""
    rng = np.random.default_rng(seed)
    if kind == "normal":
        w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    elif kind == "edge":
        w = (rng.standard_normal((n, k)) * np.exp2(rng.integers(-12, 6, (n, 1)))).astype(np.float32)
        w[:, 0:8] = 1.9999                      # rounds to mantissa 128: exponent + 1
        w[:, 8:16] = -1.9999                    # rounds to -128: kept
        w[:, 16:24] = 0.0
        w[:, 24:32] = 3e-38                     # exponent field 1: below the layout's floor
        w[0::3, 32:40] = np.linspace(-7.0, 7.0, 8, dtype=np.float32)
        w[1::3, 40:48] = 2.5e-3                 # ties of the mantissa rounding at some exponents
    else:
        raise ValueError(kind)
    x = _bf16_bits(rng.standard_normal((t, k)).astype(np.float32))
    return w, x


def q4nx_weight(w: np.ndarray, q) -> tuple[bytes, np.ndarray]:
    """(pack_gemv bytes, dequantised f32 weights) using q4nx module ``q``."""
    c, s, m = q.quantize(w)
    packed = q.pack_gemv(c, s, m)
    return packed, q.dequantize_simple(*q.parse_gemv(packed, K=w.shape[1], M=w.shape[0]))


def linear_inputs(n, k, t, seed, x_kind, bias, q=None):
    """(w_f32 dequantised, x [t,k] bf16 bits or f32, bias f32 | None); w is q4nx-exact."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    if q is None:
        import oracle.q4nx as q
    _, w_f32 = q4nx_weight(w, q)
    xf = rng.standard_normal((t, k)).astype(np.float32)
    x = xf if x_kind == "f32" else _bf16_bits(xf)
    b = rng.standard_normal(n).astype(np.float32) if bias else None
    return w_f32, x, b


def linear_packed(n, k, seed, q=None) -> bytes:
    """The pack_gemv bytes behind ``linear_inputs`` with the same arguments."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    if q is None:
        import oracle.q4nx as q
    return q4nx_weight(w, q)[0]


def moe_inputs(hidden, inter, experts, k, tokens, seed, q=None):
    """Per-expert dequantised (gate, up, down) f32, x [T,H] bf16, top ids/weights.

    Gate and up are quantised together as the reference's expert packer does
    (``kernels/moe/pack.py:136-172``: ``vstack([gate; up])`` -> one q4nx matrix).
    """
    if q is None:
        import oracle.q4nx as q
    rng = np.random.default_rng(seed)
    ex, packed = {}, {}
    for e in range(experts):
        gu = (rng.standard_normal((2 * inter, hidden)) * 0.02).astype(np.float32)
        dn = (rng.standard_normal((hidden, inter)) * 0.02).astype(np.float32)
        pgu, fgu = q4nx_weight(gu, q)
        pdn, fdn = q4nx_weight(dn, q)
        ex[e] = (fgu[:inter], fgu[inter:], fdn)
        packed[e] = (pgu, pdn)
    x = _bf16_bits(rng.standard_normal((tokens, hidden)).astype(np.float32))
    ids = np.stack([rng.permutation(experts)[:k] for _ in range(tokens)]).astype(np.int64)
    w = rng.uniform(0.05, 0.5, (tokens, k)).astype(np.float32)
    return {"experts": ex, "packed": packed, "x": x, "top_ids": ids, "top_w": w}


def router_inputs(hidden, experts, k, tokens, seed, scaling):
    rng = np.random.default_rng(seed)
    wr_bits = _bf16_bits((rng.standard_normal((experts, hidden)) * 0.02).astype(np.float32))
    wr_f32 = (wr_bits.astype(np.uint32) << 16).view(np.float32)
    x = _bf16_bits(rng.standard_normal((tokens, hidden)).astype(np.float32))
    x[-1] = 0                                   # all logits 0: every choice ties
    bias = (rng.standard_normal(experts) * 0.01).astype(np.float32)
    bias[3] = bias[9]                           # a duplicated bias value
    return {"router_w_bits": wr_bits, "router_w_f32": wr_f32, "x": x, "bias": bias,
            "k": k, "scaling": scaling}


def combine_inputs(tokens, k, hidden, seed):
    rng = np.random.default_rng(seed)
    ids = np.stack([rng.permutation(128)[:k] for _ in range(tokens)]).astype(np.int64)
    rows = _bf16_bits(rng.standard_normal((tokens, k, hidden)).astype(np.float32))
    shared = _bf16_bits(rng.standard_normal((tokens, hidden)).astype(np.float32))
    w = rng.uniform(0.0, 1.0, (tokens, k)).astype(np.float32)
    return {"top_ids": ids, "rows": rows, "shared": shared, "top_w": w}


def sample_inputs(vocab, seed, kind):
    """(logits f32 holding bf16 values, seen token ids, the generator seed of the draw)."""
    rng = np.random.default_rng(seed)
    if kind == "ties":
        x = np.round(rng.standard_normal(vocab) * 2.0).astype(np.float32)   # few distinct levels
    else:
        x = (rng.standard_normal(vocab) * 2.5).astype(np.float32)
    bits = _bf16_bits(x)
    logits = (bits.astype(np.uint32) << 16).view(np.float32)
    order = np.argsort(-logits, kind="stable")
    seen = [int(order[0]), int(order[3]), int(order[17]), int(rng.integers(vocab)), int(rng.integers(vocab))]
    return logits, seen, seed + 1000


# ------------------------------------------------------------- tiny model --
# The reference's tiny three-layer model (host/test_host_small.py:103-133: RDA
# + dense MLP, MLA + MoE, RDA + MoE; 8 experts, top-2, one shared expert, the
# SiTU betas of its ``tiny_situ_model``), widened where the q4nx MoE kernels
# need it: hidden 256 (a whole q4nx K block) instead of 64 and an expert
# intermediate of 64 (the MoE layer's granularity) instead of 32.
TINY_MODEL_CONFIG = dict(
    vocab_size=256, hidden_size=256, intermediate_size=128, num_hidden_layers=3,
    num_attention_heads=4, head_dim=16, num_experts=8, num_experts_per_token=2,
    moe_intermediate_size=64, num_shared_experts=1, first_k_dense_replace=1,
    q_lora_rank=32, kv_lora_rank=32, qk_nope_head_dim=16, qk_rope_head_dim=8, v_head_dim=16,
    rda_decay_rank=16,
    rda_config={"num_heads": 4, "head_dim": 16, "conv_kernel_size": 4, "full_rank_gate": True,
                "gate_lower_bound": -5.0, "rda_layers": [1, 3], "mla_layers": [2]},
    activation_situ_beta=2.0, activation_situ_linear_beta=9.0,
    routed_scaling_factor=1.5, moe_renormalize=True,
    pad_token_id=0, eos_token_id=[2], max_position_embeddings=64,
)
TINY_MODEL_SEED = 701
TINY_MODEL_TOKENS = (1, 17, 42, 200, 7, 99)


def _tiny_linear_shapes(c: dict) -> dict:
    """name -> (out, in) of every matrix the model multiplies through
    ``Backend.linear`` (host/raon.py:1108-1134,1166-1222,1295-1327,932)."""
    C, H = c["hidden_size"], c["num_attention_heads"]
    rda = c["rda_config"]
    rp = rda["num_heads"] * rda["head_dim"]
    rda_layers = {x - 1 for x in rda["rda_layers"]}
    out = {}
    for L in range(c["num_hidden_layers"]):
        a = f"model.layers.{L}.self_attn"
        if L in rda_layers:
            for p in ("q", "k", "v", "g"):
                out[f"{a}.{p}_proj.weight"] = (rp, C)
            out[f"{a}.b_proj.weight"] = (rda["num_heads"], C)
            out[f"{a}.rda_w_proj.weight"] = (rda["num_heads"], C)
            out[f"{a}.f_a_proj.weight"] = (c["rda_decay_rank"], C)
            out[f"{a}.f_b_proj.weight"] = (rp, c["rda_decay_rank"])
            out[f"{a}.o_proj.weight"] = (C, rp)
        else:
            qd = c["qk_nope_head_dim"] + c["qk_rope_head_dim"]
            out[f"{a}.q_a_proj.weight"] = (c["q_lora_rank"], C)
            out[f"{a}.q_b_proj.weight"] = (H * qd, c["q_lora_rank"])
            out[f"{a}.kv_a_proj_with_mqa.weight"] = (c["kv_lora_rank"] + c["qk_rope_head_dim"], C)
            out[f"{a}.kv_b_proj.weight"] = (H * (c["qk_nope_head_dim"] + c["v_head_dim"]), c["kv_lora_rank"])
            out[f"{a}.g_proj.weight"] = (H * c["v_head_dim"], C)
            out[f"{a}.o_proj.weight"] = (C, H * c["v_head_dim"])
        if L < c["first_k_dense_replace"]:
            m, inter = f"model.layers.{L}.mlp", c["intermediate_size"]
            out[f"{m}.gate_proj.weight"] = (inter, C)
            out[f"{m}.up_proj.weight"] = (inter, C)
            out[f"{m}.down_proj.weight"] = (C, inter)
        # (the shared experts' gate/up/down are made with the routed experts)
    out["lm_head.weight"] = (c["vocab_size"], C)
    return out


def _q4nx_padded(w: np.ndarray, q):
    """Zero-pad to 128 rows / 256 columns (the exporter's GEMV alignment,
    quant/q4nx.py:226-248), quantise and pack; returns (packed, padded n, padded
    k, dequantised f32 weights of the unpadded [n, k])."""
    n, k = w.shape
    wp = np.pad(w, ((0, (-n) % 128), (0, (-k) % 256)))
    packed, f32 = q4nx_weight(wp, q)
    return packed, wp.shape[0], wp.shape[1], np.ascontiguousarray(f32[:n, :k])


def tiny_model(q=None):
    """Seeded weights of the tiny model in q4nx form.

    Returns ``host`` (name -> array, the weights the reference's host model
    and NumpyBackend read: the q4nx matrices as their dequantised f32 values,
    the rest as f32, the embedding as bf16 bits), ``bundles`` (bundle ->
    (packed, padded n, padded k)), ``linears`` (name -> (bundle, first row,
    end row, unpadded k): a shared expert's gate and up are the two row halves
    of its [gate; up] bundle, as the reference's exporter packs them),
    ``experts`` (MoE layer -> expert -> (packed [gate; up], packed K-padded
    down); the shared expert under id ``num_experts``, the same bytes as its
    bundles) and ``router`` (MoE layer -> (bf16 bits [E, C], correction bias
    f32 [E]))."""
    if q is None:
        import oracle.q4nx as q
    c = TINY_MODEL_CONFIG
    rng = np.random.default_rng(TINY_MODEL_SEED)
    C, V, n_mhc = c["hidden_size"], c["vocab_size"], 4
    E, I = c["num_experts"], c["moe_intermediate_size"]

    def normal(shape, std):
        return (rng.standard_normal(shape) * std).astype(np.float32)

    host, bundles, linears, experts, router = {}, {}, {}, {}, {}
    host["model.embed_tokens.weight"] = _bf16_bits(normal((V, C), 1.0))
    host["model.norm.weight"] = 1.0 + normal((C,), 0.1)
    for name, (n, k) in _tiny_linear_shapes(c).items():
        packed, n_pad, k_pad, f32 = _q4nx_padded(normal((n, k), k ** -0.5), q)
        bundles[name] = (packed, n_pad, k_pad)
        linears[name] = (name, 0, n, k)
        host[name] = f32
    rda_layers = {x - 1 for x in c["rda_config"]["rda_layers"]}
    rp, hd = 4 * 16, 16
    for L in range(c["num_hidden_layers"]):
        p = f"model.layers.{L}"
        host[f"{p}.input_layernorm.weight"] = 1.0 + normal((C,), 0.1)
        host[f"{p}.post_attention_layernorm.weight"] = 1.0 + normal((C,), 0.1)
        for site in ("self_attn_raon_mhc", "mlp_raon_mhc"):
            s = f"{p}.{site}"
            std = 0.5 * (n_mhc * C) ** -0.5
            host[f"{s}.phi_pre"] = normal((n_mhc, n_mhc * C), std)
            host[f"{s}.phi_post"] = normal((n_mhc, n_mhc * C), std)
            host[f"{s}.res.phi_z"] = normal(((n_mhc - 1) ** 2, n_mhc * C), std)
            for a in ("alpha_pre", "alpha_post", "res.alpha_z"):
                host[f"{s}.{a}"] = np.array([0.5], np.float32)
            host[f"{s}.b_pre"] = normal((n_mhc,), 0.1)
            host[f"{s}.b_post"] = normal((n_mhc,), 0.1)
            host[f"{s}.res.b_z"] = normal(((n_mhc - 1) ** 2,), 0.1)
            host[f"{s}.res.eta"] = np.array([0.0], np.float32)
        a = f"{p}.self_attn"
        if L in rda_layers:
            for kind in ("q", "k", "v"):
                host[f"{a}.{kind}_conv1d.weight"] = normal((rp, c["rda_config"]["conv_kernel_size"]), 0.5)
            host[f"{a}.dt_bias"] = normal((rp,), 0.1)
            host[f"{a}.A_log"] = np.log(rng.uniform(1.0, 4.0, 4)).astype(np.float32)
            host[f"{a}.o_norm.weight"] = 1.0 + normal((hd,), 0.1)
        else:
            host[f"{a}.q_a_layernorm.weight"] = 1.0 + normal((c["q_lora_rank"],), 0.1)
            host[f"{a}.kv_a_layernorm.weight"] = 1.0 + normal((c["kv_lora_rank"],), 0.1)
        if L < c["first_k_dense_replace"]:
            continue
        m = f"{p}.moe"
        bits = _bf16_bits(normal((E, C), C ** -0.5))
        bias = normal((E,), 0.05)
        router[L] = (bits, bias)
        host[f"{m}.gate.weight"] = (bits.astype(np.uint32) << 16).view(np.float32)
        host[f"{m}.gate.e_score_correction_bias"] = bias
        experts[L] = {}
        for e in range(E + 1):
            pgu, fgu = q4nx_weight(normal((2 * I, C), C ** -0.5), q)
            pdn, n_pad, k_pad, fdn = _q4nx_padded(normal((C, I), I ** -0.5), q)
            experts[L][e] = (pgu, pdn)
            ex = f"{m}.experts.{e}" if e < E else f"{m}.shared_experts"
            host[f"{ex}.gate_proj.weight"] = np.ascontiguousarray(fgu[:I])
            host[f"{ex}.up_proj.weight"] = np.ascontiguousarray(fgu[I:])
            host[f"{ex}.down_proj.weight"] = fdn
            if e == E:
                bundles[f"{ex}.gate_up"] = (pgu, 2 * I, C)
                bundles[f"{ex}.down_proj.weight"] = (pdn, n_pad, k_pad)
                linears[f"{ex}.gate_proj.weight"] = (f"{ex}.gate_up", 0, I, C)
                linears[f"{ex}.up_proj.weight"] = (f"{ex}.gate_up", I, 2 * I, C)
                linears[f"{ex}.down_proj.weight"] = (f"{ex}.down_proj.weight", 0, C, I)
    return {"host": host, "bundles": bundles, "linears": linears, "experts": experts, "router": router}


def tiny_model_trace(npz) -> dict:
    """The recorded ``RaonModel.step`` calls of ``tiny_model.npz`` as a list of
    dicts (kind "linear": name, x, y; kind "moe": layer, x, y, top, w, betas,
    layer_out), the per-step call ranges and the per-step logits."""
    z = np.load(npz)
    calls = []
    moe = {int(i): j for j, i in enumerate(z["moe_call"])}
    for i in range(len(z["name"])):
        c = {"x": z["x_flat"][z["x_off"][i]:z["x_off"][i + 1]],
             "y": z["y_flat"][z["y_off"][i]:z["y_off"][i + 1]]}
        if i in moe:
            j = moe[i]
            c.update(kind="moe", layer=int(z["moe_layer"][j]), top=z["moe_top"][j], w=z["moe_w"][j],
                     betas=tuple(float(b) for b in z["moe_betas"][j]), layer_out=z["moe_layer_out"][j])
        else:
            c.update(kind="linear", name=str(z["name"][i]))
        calls.append(c)
    starts = [int(s) for s in z["step_starts"]]
    return {"calls": calls, "steps": list(zip(starts[:-1], starts[1:])),
            "logits": [z[f"step{s}/logits"] for s in range(len(starts) - 1)],
            "bundles_sha": str(z["bundles_sha"]), "experts_sha": str(z["experts_sha"])}
