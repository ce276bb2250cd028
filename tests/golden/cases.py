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
