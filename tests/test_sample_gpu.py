"""GPU token sampler (rc_sample_tokens) against the reference's own draws and
the oracle restatement of serve/engine.py:84-140.

Bar: the sampled token ids are identical.  (The f64 exp/sum order on the
device can differ from numpy's in the last bit, which could only change a
token whose uniform draw falls within ~1e-15 of a cumulative-probability
boundary; none of the cases here comes close.)
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import q4nx as q
from oracle.sampling import sample_token_u
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


def _gpu_sample(torch, ctx, logits_f32, seen_lists, us, top_k, top_p, temperature, penalty):
    from raon_npu_b200.device import sample_tokens
    T = len(us)
    bits = q.f32_to_bf16(np.ascontiguousarray(logits_f32, np.float32).reshape(-1, logits_f32.shape[-1]))
    if bits.shape[0] == 1 and T > 1:
        bits = np.repeat(bits, T, axis=0)
    ld = torch.from_numpy(bits.view(np.int16)).cuda()
    flat = [int(s) for sl in seen_lists for s in sl]
    off = np.cumsum([0] + [len(sl) for sl in seen_lists]).astype(np.int32)
    seen_d = torch.tensor(flat if flat else [0], dtype=torch.int32, device="cuda")
    off_d = torch.from_numpy(off).cuda()
    u_d = torch.tensor(np.asarray(us, np.float64), device="cuda")
    out = torch.empty(T, dtype=torch.int32, device="cuda")
    sample_tokens(ctx, ld, u_d, out, top_k=top_k, top_p=top_p, temperature=temperature,
                  presence_penalty=penalty, seen_dev=seen_d, seen_off_dev=off_d)
    torch.cuda.synchronize()
    ctx.sync()
    return out.cpu().numpy()


@pytest.mark.parametrize("name", [n for n in cases.SAMPLE_CASES if cases.SAMPLE_CASES[n][3]["top_k"] > 0])
def test_sampler_reproduces_reference_draws(torch, ctx, name):
    g = np.load(cases.__file__.replace("cases.py", "sample.npz"))
    vocab, seed, kind, o = cases.SAMPLE_CASES[name]
    logits, seen, gseed = cases.sample_inputs(vocab, seed, kind)
    us = [np.random.default_rng(gseed + i).random() for i in range(20)]
    got = _gpu_sample(torch, ctx, logits, [seen] * 20, us, o["top_k"], o["top_p"], o["temperature"],
                      o["presence_penalty"])
    np.testing.assert_array_equal(got, g[f"{name}/tokens"])


def test_sampler_matches_oracle_on_random_cases(torch, ctx):
    rng = np.random.default_rng(55)
    for case in range(40):
        V = int(rng.choice([151936, 32000, 777]))
        scale = float(rng.choice([0.5, 2.5, 8.0]))
        logits = q.bf16_to_f32(q.f32_to_bf16((rng.standard_normal(V) * scale).astype(np.float32)))
        top_k = int(rng.choice([1, 5, 50, 200, min(1024, V - 1)]))
        top_p = float(rng.choice([0.0, 0.5, 0.9, 0.99, 1.0]))
        temperature = float(rng.choice([0.0, 0.3, 1.0, 1.7]))
        penalty = float(rng.choice([0.0, 1.5, -0.5]))
        T = 6
        seen_lists = [list(rng.integers(0, V, size=int(rng.integers(0, 40)))) for _ in range(T)]
        us = list(rng.random(T))
        got = _gpu_sample(torch, ctx, logits, seen_lists, us, top_k, top_p, temperature, penalty)
        ref = [sample_token_u(logits, seen_lists[t], top_k, top_p, temperature, penalty, us[t]) for t in range(T)]
        np.testing.assert_array_equal(got, ref, err_msg=f"case {case}: V={V} k={top_k} p={top_p} "
                                                         f"T={temperature} pen={penalty}")


def test_sampler_rejects_vocabulary_wide_top_p(torch, ctx):
    from raon_npu_b200.device import sample_tokens
    ld = torch.zeros((1, 1000), dtype=torch.int16, device="cuda")
    u = torch.zeros(1, dtype=torch.float64, device="cuda")
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    with pytest.raises(ValueError):
        sample_tokens(ctx, ld, u, out, top_k=0, top_p=0.9)


def test_sampler_reports_too_many_ties(torch, ctx):
    """5000 equal logits with top-k 5: every token ties at the threshold, more
    than the 2048 candidates the device sorts -> an error, not a wrong token."""
    from raon_npu_b200.device import sample_tokens
    ld = torch.full((1, 5000), 0x3F80, dtype=torch.int16, device="cuda")
    u = torch.full((1,), 0.5, dtype=torch.float64, device="cuda")
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    sample_tokens(ctx, ld, u, out, top_k=5, top_p=0.9)
    torch.cuda.synchronize()
    with pytest.raises(ValueError):
        ctx.sync()
    assert int(out.item()) == -1


def test_sampler_reports_nan_logits(torch, ctx):
    from raon_npu_b200.device import sample_tokens
    ld = torch.full((1, 3000), 0x7FC0, dtype=torch.int16, device="cuda")
    u = torch.full((1,), 0.5, dtype=torch.float64, device="cuda")
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    sample_tokens(ctx, ld, u, out, top_k=50, top_p=0.9)
    torch.cuda.synchronize()
    with pytest.raises(ValueError):
        ctx.sync()
    assert int(out.item()) == -1
