"""Numpy oracle for the GEMV / MoE entry points -- TEST INFRASTRUCTURE ONLY.

Restates the reference CPU backend (raon-npu ``host/backend.py`` ``NumpyBackend``)
plus the routing and activation arithmetic that surrounds it, so the CUDA
backend can be compared on identical inputs.  Weights are given as the f32
matrices the reference multiplies by (``oracle.q4nx.dequantize_packed``).
"""

from __future__ import annotations

import numpy as np

from .q4nx import bf16_to_f32, f32_to_bf16


# ------------------------------------------------------------------ linear --
def linear_f32(w_f32: np.ndarray, x: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """fp32 ``x @ W.T (+ b)`` before output rounding (``host/backend.py:402-414``)."""
    xf = x if x.dtype == np.float32 else bf16_to_f32(x)
    y = np.dot(xf, w_f32.T)
    if bias is not None:
        y = y + bias
    return y.astype(np.float32)


def linear(w_f32: np.ndarray, x: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """``NumpyBackend.linear`` (``host/backend.py:402-417``): bf16 (uint16) in ->
    RTNE bf16 out; f32 in -> f32 out.  Leading dimensions are kept."""
    y = linear_f32(w_f32, x, bias)
    return y if x.dtype == np.float32 else f32_to_bf16(y)


# -------------------------------------------------------------- activations --
def situ_glu(gate, value, gate_beta: float = 4.0, value_beta: float = 25.0) -> np.ndarray:
    """SiTU-GLU in f32: ``gb*tanh(g/gb)*sigmoid(g) * vb*tanh(v/vb)`` (``host/backend.py:47-62``)."""
    g = bf16_to_f32(gate) if np.asarray(gate).dtype == np.uint16 else np.asarray(gate, np.float32)
    v = bf16_to_f32(value) if np.asarray(value).dtype == np.uint16 else np.asarray(value, np.float32)
    sig = 1.0 / (1.0 + np.exp(-g))
    return (gate_beta * np.tanh(g / gate_beta) * sig) * (value_beta * np.tanh(v / value_beta))


def swiglu(gate, up) -> np.ndarray:
    """SiLU-GLU ``g*sigmoid(g)*u`` with the overflow-free sigmoid of
    ``kernels/moe/reference.py:160-170`` (the ``gate_beta=None`` branch)."""
    g = bf16_to_f32(gate) if np.asarray(gate).dtype == np.uint16 else np.asarray(gate, np.float32)
    u = bf16_to_f32(up) if np.asarray(up).dtype == np.uint16 else np.asarray(up, np.float32)
    e = np.exp(-np.abs(g))
    sig = np.where(g >= 0, 1.0 / (1.0 + e), e / (1.0 + e))
    return (g * sig) * u


def glu(gate, up, act: str, gate_beta: float = 4.0, value_beta: float = 25.0) -> np.ndarray:
    if act == "swiglu":
        return swiglu(gate, up)
    if act == "situ":
        return situ_glu(gate, up, gate_beta, value_beta)
    raise ValueError(f"unknown activation {act!r}")


# --------------------------------------------------------------------- MoE --
def expert_forward(w_gate, w_up, w_down, x, act, gate_beta=4.0, value_beta=25.0) -> np.ndarray:
    """One expert for one token: gate/up linear (bf16 each), act -> RTNE, down linear (bf16).

    The per-expert body of ``host/backend.py:496-507``.
    """
    g = linear(w_gate, x)
    u = linear(w_up, x)
    a = f32_to_bf16(glu(g, u, act, gate_beta, value_beta))
    return linear(w_down, a)


def moe_experts(experts, x, top_ids, top_weights, act="situ", gate_beta=4.0, value_beta=25.0) -> np.ndarray:
    """``NumpyBackend.moe_experts`` (``host/backend.py:466-510``) for one token.

    ``experts[e] = (w_gate, w_up, w_down)`` f32.  Experts are visited in
    ascending ID whatever the router order; the weighted sum is f32, then RTNE.
    """
    acc = np.zeros(experts[int(top_ids[0])][2].shape[0], np.float32)
    for eid, wt in sorted(((int(e), float(w)) for e, w in zip(top_ids, top_weights)), key=lambda p: p[0]):
        wg, wu, wd = experts[eid]
        acc += bf16_to_f32(expert_forward(wg, wu, wd, x, act, gate_beta, value_beta)) * np.float32(wt)
    return f32_to_bf16(acc)


def moe_term_magnitude(experts, x, top_ids, top_weights, act="situ", gate_beta=4.0, value_beta=25.0,
                       shared_down_u16=None) -> np.ndarray:
    """Per output h: sum_e |w_e * down_e[h]| (+ |shared[h]|), the magnitude of the
    terms the f32 combine accumulates.  Each expert output is a bf16 value
    whose last rounding step may fall either way between two implementations
    summing in different orders, so an implementation-independent bound on an
    MoE output is one bf16 step (at most 2^-7 relative) of this magnitude."""
    mag = None
    for eid, wt in zip(top_ids, top_weights):
        wg, wu, wd = experts[int(eid)]
        t = np.abs(bf16_to_f32(expert_forward(wg, wu, wd, x, act, gate_beta, value_beta)).astype(np.float64) * wt)
        mag = t if mag is None else mag + t
    if shared_down_u16 is not None:
        mag = mag + np.abs(bf16_to_f32(shared_down_u16).astype(np.float64))
    return mag


def moe_token_with_shared(routed_u16, shared_down_u16) -> np.ndarray:
    """``bf16(f32(routed) + f32(shared))`` (``host/raon.py:1321-1327``)."""
    return f32_to_bf16(bf16_to_f32(routed_u16) + bf16_to_f32(shared_down_u16))


def moe_decode_layer(experts, shared, router_w, x, top_k, act="swiglu", gate_beta=4.0, value_beta=25.0):
    """Config-3 MoE decode layer for one token: softmax router, routed experts, shared expert.

    Returns (out bf16, top_ids sorted by router rank, weights f32, logits f32).
    """
    ids, w, logits = route_softmax(x, router_w, top_k)
    routed = moe_experts(experts, x, ids, w, act, gate_beta, value_beta)
    sh = expert_forward(*shared, x, act, gate_beta, value_beta)
    return moe_token_with_shared(routed, sh), ids, w, logits


# ------------------------------------------------------------------ router --
def router_logits(x_u16: np.ndarray, router_w: np.ndarray) -> np.ndarray:
    """``x_f32 . Wr`` accumulated in f64 and rounded once to f32.

    ``router_w`` is bf16 bits [E, H] (the reference's ``x @ Wr.T`` orientation,
    ``host/raon.py:1230-1234``).  Products of two bf16 values are exact in f64,
    so the only roundings are the f64 additions and the final f32 cast; the
    CUDA router accumulates the same way, which makes its logits agree with
    these to the f32 bit except in vanishingly rare f64-rounding cases.
    """
    xf = bf16_to_f32(x_u16).astype(np.float64)
    wf = bf16_to_f32(router_w).astype(np.float64)
    return (xf @ wf.T).astype(np.float32)


def topk_lower_index_wins(values: np.ndarray, k: int) -> np.ndarray:
    """Indices of the k largest values, descending; equal values -> lower index first.

    A stable ``argsort`` of ``-values`` (the reference uses an unstable
    ``np.argsort(-choice)`` at ``host/raon.py:1239``; the restatement pins the
    tie rule to "lower index wins").
    """
    return np.argsort(-np.asarray(values, np.float64), kind="stable")[:k]


def route_softmax(x_u16, router_w, k):
    """softmax(x . Wr) -> top-k -> renormalised weights (BASELINE configs 3/4).

    Softmax is strictly increasing in the logit, so the top-k of the
    probabilities is the top-k of the logits; the renormalised weight of a
    selected expert is ``exp(l_i - l_max) / sum_top exp(l_j - l_max)`` (the
    full-softmax denominator cancels).  Weights are computed in f64 and
    returned as f32.
    """
    logits = router_logits(x_u16, router_w)
    ids = topk_lower_index_wins(logits, k)
    sel = logits[ids].astype(np.float64)
    e = np.exp(sel - sel.max())
    return ids, (e / e.sum()).astype(np.float32), logits


def route_sigmoid_bias(x_u16, router_w, bias, k, renormalize=True, scaling=1.0):
    """Reference router (``host/raon.py:1224-1247``): sigmoid scores, top-k of
    ``score + bias`` (lower index wins ties), weights = chosen scores
    renormalised by ``sum + 1e-20``, times the routed scaling factor."""
    logits = router_logits(x_u16, router_w)
    scores = (1.0 / (1.0 + np.exp(-logits.astype(np.float64)))).astype(np.float32)
    choice = scores + np.asarray(bias, np.float32)
    ids = topk_lower_index_wins(choice, k)
    chosen = scores[ids]
    if renormalize:
        chosen = chosen / (np.sum(chosen) + np.float32(1e-20))
    return ids, (chosen * np.float32(scaling)).astype(np.float32), logits


# ------------------------------------------------------------ grouped MoE --
def combine_ascending(rows_u16: np.ndarray, top_ids: np.ndarray, top_weights: np.ndarray) -> np.ndarray:
    """Per token: ``RTNE(sum over routes in ascending expert ID of f32(row) * w)``.

    The routed half of ``scatter_b2`` (``kernels/moe_grouped/planner.py:316-322``).
    ``rows_u16`` is [T, k, H] bf16 bits, one row per (token, route).
    """
    T, _, H = rows_u16.shape
    out = np.zeros((T, H), np.uint16)
    for t in range(T):
        acc = np.zeros(H, np.float32)
        for r in np.argsort(np.asarray(top_ids[t]), kind="stable"):
            acc += bf16_to_f32(rows_u16[t, r]) * np.float32(top_weights[t, r])
        out[t] = f32_to_bf16(acc)
    return out


def moe_experts_grouped(experts, shared_down_w, x, top_ids, top_weights, shared_gu, act="situ",
                        gate_beta=4.0, value_beta=25.0):
    """``moe_experts_grouped`` semantics (``npu/backend.py:4845-4979`` with the
    combine of ``kernels/moe_grouped/planner.py:286-322``): for every token the
    routed outputs are summed in ascending expert ID in f32 then RTNE; the
    shared output is ``linear(shared_down, RTNE(act(shared_gu)))``.

    Returns (routed [T, H] bf16, shared_down [T, H] bf16).
    """
    T = x.shape[0]
    routed = np.stack([moe_experts(experts, x[t], top_ids[t], top_weights[t], act, gate_beta, value_beta)
                       for t in range(T)])
    inter = shared_gu.shape[1] // 2
    a = f32_to_bf16(glu(shared_gu[:, :inter], shared_gu[:, inter:], act, gate_beta, value_beta))
    return routed, linear(shared_down_w, a)
