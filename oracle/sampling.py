"""Token sampler restated from the reference -- TEST INFRASTRUCTURE ONLY.

``sample_token`` of ``serve/engine.py:84-140`` (with ``_softmax`` of
``serve/engine.py:74-81``), with the generator's single uniform draw passed
in explicitly: numpy's ``Generator.choice(n, p=p)`` is
``cdf = p.cumsum(); cdf /= cdf[-1]; idx = cdf.searchsorted(rng.random(), 'right')``,
so the token is a pure function of (logits, options, u).
"""

from __future__ import annotations

import numpy as np


def softmax(x: np.ndarray) -> np.ndarray:
    """``_softmax`` (serve/engine.py:74-81): f64, argmax one-hot if the sum degenerates."""
    shifted = x - np.max(x)
    exp_x = np.exp(shifted)
    denom = np.sum(exp_x)
    if denom <= 0.0 or not np.isfinite(denom):
        probs = np.zeros_like(x, dtype=np.float64)
        probs[int(np.argmax(x))] = 1.0
        return probs
    return exp_x / denom


def sample_token_u(logits, seen, top_k: int, top_p: float, temperature: float, presence_penalty: float,
                   u: float) -> int:
    """serve/engine.py:84-140 step by step: presence penalty, greedy for
    temperature <= 0, top-k (ties with the k-th value kept), top-p (stable
    descending order, keep the top token), temperature, categorical draw."""
    scores = np.array(logits, dtype=np.float64, copy=True).ravel()
    V = scores.size
    if presence_penalty != 0.0 and seen:
        uniq = [int(t) for t in set(seen) if 0 <= int(t) < V]
        if uniq:
            scores[uniq] -= float(presence_penalty)
    if temperature <= 0.0:
        return int(np.argmax(scores))
    if 0 < top_k < V:
        kth = np.partition(scores, -top_k)[-top_k]
        scores[scores < kth] = -np.inf
    if 0.0 <= top_p < 1.0:
        order = np.argsort(-scores, kind="stable")
        probs = softmax(scores[order])
        cum = np.cumsum(probs)
        remove = (cum - probs) >= top_p
        remove[0] = False
        scores[order[remove]] = -np.inf
    if temperature != 1.0:
        scores = scores / float(temperature)
    p = softmax(scores)
    cdf = p.cumsum()
    cdf /= cdf[-1]
    return int(cdf.searchsorted(u, side="right"))
