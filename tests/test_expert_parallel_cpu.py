"""Host logic of the expert-parallel MoE decode on CPU (gloo, world size 2).

``raon_npu_b200.expert_parallel.ExpertParallelMoe`` drives an MoE layer
through all-gather -> local experts -> reduce-scatter -> combine.  Here the
layer is a stand-in built on the oracle (the same ``decode_local`` /
``combine`` contract as ``MoeLayer``, computed in numpy), so the test checks
the partition of experts and shared-expert tokens over the ranks, the token
order of the gather, the exactness of the summed exchange and the slicing of
the combine: every rank's outputs must equal the single-process oracle decode
of its tokens byte for byte.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

HIDDEN, INTER, E, K, M = 256, 256, 8, 3, 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(seed=11):
    """Experts (dequantised f32 gate, up, down; id E = shared) and router bits."""
    from oracle import q4nx as q
    from tests.golden import cases
    rng = np.random.default_rng(seed)
    experts = {}
    for e in range(E + 1):
        gu = (rng.standard_normal((2 * INTER, HIDDEN)) * 0.02).astype(np.float32)
        dn = (rng.standard_normal((HIDDEN, INTER)) * 0.02).astype(np.float32)
        _, fgu = cases.q4nx_weight(gu, q)
        _, fdn = cases.q4nx_weight(dn, q)
        experts[e] = (fgu[:INTER], fgu[INTER:], fdn)
    wr = q.f32_to_bf16((rng.standard_normal((E, HIDDEN)) * 0.02).astype(np.float32))
    return experts, wr


class OracleLayer:
    """CPU stand-in for ``MoeLayer`` (test infrastructure: numpy oracle)."""

    def __init__(self, experts, wr, owned):
        self.experts = {e: w for e, w in experts.items() if e in owned}
        self.wr = wr
        self.n_experts, self.hidden, self.has_shared = E, HIDDEN, True

    def decode_local(self, x, k, slots, sw, experts, shared_tokens, act, **_):
        from oracle import backend as ob
        xs = x.numpy().view(np.uint16)
        routes = [ob.route_softmax(xs[t], self.wr, k)[:2] for t in range(xs.shape[0])]
        self._local(xs, routes, k, slots, sw, experts, shared_tokens, act)

    def prefill_local_routes(self, x, ids, w, k, slots, sw, experts, shared_tokens, act, **_):
        xs = x.numpy().view(np.uint16)
        routes = list(zip(ids.numpy(), w.numpy()))
        self._local(xs, routes, k, slots, sw, experts, shared_tokens, act)

    def _local(self, xs, routes, k, slots, sw, experts, shared_tokens, act):
        import torch
        from oracle import backend as ob
        lo, hi = experts
        t0, tn = shared_tokens
        rows = np.zeros((xs.shape[0], k + 1, self.hidden), np.uint16)
        wts = np.zeros((xs.shape[0], k), np.float32)
        for t in range(xs.shape[0]):
            ids, w = routes[t]
            order = np.argsort(ids, kind="stable")
            for pos, r in enumerate(order):
                e = int(ids[r])
                wts[t, pos] = w[r]
                if lo <= e < hi:
                    rows[t, pos] = ob.expert_forward(*self.experts[e], xs[t], act)
            if t0 <= t < t0 + tn:
                rows[t, k] = ob.expert_forward(*self.experts[E], xs[t], act)
        slots.copy_(torch.from_numpy(rows.view(np.int16)))
        sw.copy_(torch.from_numpy(wts))

    def route(self, x, tokens, k, ids, w, **_):
        import torch
        from oracle import backend as ob
        xs = x.numpy().view(np.uint16)
        res = [ob.route_softmax(xs[t], self.wr, k) for t in range(tokens)]
        ids.copy_(torch.from_numpy(np.stack([r[0] for r in res]).astype(np.int32)))
        w.copy_(torch.from_numpy(np.stack([r[1] for r in res])))

    prefill_local = decode_local

    def prefill_experts(self, x, ids, w, k, out, act, with_shared=False, **_):
        import torch
        from oracle import backend as ob
        xs = x.numpy().view(np.uint16)
        ii, ww = ids.numpy(), w.numpy()
        res = np.stack([ob.moe_experts(self.experts, xs[t], ii[t], ww[t], act=act) for t in range(xs.shape[0])])
        out.copy_(torch.from_numpy(res.view(np.int16)))

    def prefill_combine(self, slots, sw, k, out, tokens, with_shared):
        self.combine(slots, sw, k, out, tokens, with_shared)

    def combine(self, slots, sw, k, out, tokens, with_shared):
        import torch
        from oracle import backend as ob
        rows = slots.numpy().view(np.uint16)
        w = sw.numpy()
        # slot rows are already in ascending-ID order: combine with ids 0..k-1
        routed = ob.combine_ascending(rows[:, :k], np.tile(np.arange(k), (tokens, 1)), w)
        res = np.stack([ob.moe_token_with_shared(routed[t], rows[t, k]) for t in range(tokens)])
        out.copy_(torch.from_numpy(res.view(np.int16)))


def _worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist
    from raon_npu_b200.expert_parallel import ExpertParallelMoe
    from oracle import q4nx as q
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        experts, wr = _model()
        per = E // world
        owned = set(range(rank * per, (rank + 1) * per)) | {E}
        ep = ExpertParallelMoe(OracleLayer(experts, wr, owned), K, act="swiglu")
        assert ep.experts == (rank * per, (rank + 1) * per)
        assert all(ep.owns(e) for e in owned) and not any(ep.owns(e) for e in set(range(E)) - owned)
        rng = np.random.default_rng(100 + rank)
        x = q.f32_to_bf16(rng.standard_normal((M, HIDDEN)).astype(np.float32))
        out = torch.empty((M, HIDDEN), dtype=torch.int16)
        ep.decode(torch.from_numpy(x.view(np.int16)), out)
        np.save(os.path.join(result_dir, f"x{rank}.npy"), x)
        np.save(os.path.join(result_dir, f"out{rank}.npy"), out.numpy().view(np.uint16))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_expert_parallel_two_ranks_match_single_process(tmp_path):
    import torch.multiprocessing as mp
    from oracle import backend as ob
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    experts, wr = _model()
    for rank in range(world):
        x = np.load(tmp_path / f"x{rank}.npy")
        out = np.load(tmp_path / f"out{rank}.npy")
        for t in range(M):
            ref, _, _, _ = ob.moe_decode_layer({e: experts[e] for e in range(E)}, experts[E], wr, x[t], K,
                                               act="swiglu")
            np.testing.assert_array_equal(out[t], ref)


def _prefill_worker(rank, world, port, result_dir, exchange, M):
    import torch
    import torch.distributed as dist
    from raon_npu_b200.expert_parallel import ExpertParallelMoe
    from oracle import q4nx as q
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        experts, wr = _model()
        per = E // world
        owned = set(range(rank * per, (rank + 1) * per)) | {E}
        ep = ExpertParallelMoe(OracleLayer(experts, wr, owned), K, act="swiglu", prefill_exchange=exchange)
        rng = np.random.default_rng(300 + rank)
        x = q.f32_to_bf16(rng.standard_normal((M, HIDDEN)).astype(np.float32))
        out = torch.empty((M, HIDDEN), dtype=torch.int16)
        ep.prefill(torch.from_numpy(x.view(np.int16)), out)
        np.save(os.path.join(result_dir, f"px{rank}.npy"), x)
        np.save(os.path.join(result_dir, f"pout{rank}.npy"), out.numpy().view(np.uint16))
        np.save(os.path.join(result_dir, f"pex{rank}.npy"), np.array([ep.last_prefill_exchange], dtype=object),
                allow_pickle=True)
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("exchange,M", [("a2a", 5), ("gather", 5), ("gather", 20)])
def test_expert_parallel_prefill_matches_single_process(tmp_path, exchange, M):
    """Prefill over two gloo ranks, either exchange: every rank's outputs
    equal the single-process oracle layer byte for byte; with "a2a" only the
    rows of remote routes cross (there and back); "gather" above 16 tokens
    per rank routes each rank's own tokens and gathers the routes with the
    rows."""
    import torch.multiprocessing as mp
    from oracle import backend as ob
    world = 2
    mp.start_processes(_prefill_worker, args=(world, _free_port(), str(tmp_path), exchange, M), nprocs=world,
                       start_method="spawn")
    experts, wr = _model()
    sent = 0
    for rank in range(world):
        x = np.load(tmp_path / f"px{rank}.npy")
        out = np.load(tmp_path / f"pout{rank}.npy")
        ex = np.load(tmp_path / f"pex{rank}.npy", allow_pickle=True)[0]
        remote = 0
        for t in range(x.shape[0]):
            ref, ids, _, _ = ob.moe_decode_layer({e: experts[e] for e in range(E)}, experts[E], wr, x[t], K,
                                                 act="swiglu")
            np.testing.assert_array_equal(out[t], ref)
            remote += int(sum(1 for e in ids if int(e) // (E // world) != rank))
        if exchange == "a2a":
            assert ex["rows_sent"] == remote
        sent += ex["rows_sent"]
    assert sent == sum(np.load(tmp_path / f"pex{r}.npy", allow_pickle=True)[0]["rows_received"] for r in range(world))


def test_single_process_owns_every_expert():
    from raon_npu_b200.expert_parallel import ExpertParallelMoe
    import torch.distributed as dist

    class L:
        n_experts, hidden, has_shared = 6, 256, True
    if dist.is_initialized():
        pytest.skip("needs a process without a default group")
    ep = ExpertParallelMoe(L(), 2)
    assert ep.world == 1 and ep.experts == (0, 6) and ep.active_transport == "none"
    assert all(ep.owns(e) for e in range(7))


class HandshakeLayer:
    """Stand-in with the peer-memory entry points of ``MoeLayer``: records the
    blobs it is given; ``fail_init`` makes ``ep_init`` raise on this rank."""
    EP_HANDLE_BYTES = 128

    def __init__(self, rank, fail_init=False):
        self.rank, self.fail_init = rank, fail_init
        self.n_experts, self.hidden, self.has_shared = E, HIDDEN, True
        self.opened, self.decoded = {}, []

    def ep_init(self, rank, world, m):
        if self.fail_init:
            raise RuntimeError("rc_moe_ep_init: injected failure")
        self.geometry = (rank, world, m)
        return bytes([rank, world, m]) + bytes(self.EP_HANDLE_BYTES - 3)

    def ep_open(self, peer, blob):
        assert len(blob) == self.EP_HANDLE_BYTES
        self.opened[peer] = bytes(blob[:3])

    def ep_decode(self, x, k, out, **_):
        self.decoded.append((tuple(x.shape), k))
        out.copy_(x)


def _handshake_worker(rank, world, port, result_dir, fail_rank):
    import torch
    import torch.distributed as dist
    from raon_npu_b200.expert_parallel import ExpertParallelMoe
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer = HandshakeLayer(rank, fail_init=rank == fail_rank)
        ep = ExpertParallelMoe(layer, K, transport="p2p")
        x = torch.arange(M * HIDDEN, dtype=torch.int16).reshape(M, HIDDEN) + rank
        out = torch.empty_like(x)
        try:
            ep.decode(x, out)
            ep.decode(x, out)          # set up once per token count
            res = {"ok": True, "opened": layer.opened, "decoded": layer.decoded, "geometry": layer.geometry,
                   "same": bool(torch.equal(out, x)), "active": ep.active_transport}
        except RuntimeError as e:
            res = {"ok": False, "error": str(e)}
        np.save(os.path.join(result_dir, f"h{rank}.npy"), np.array([res], dtype=object), allow_pickle=True)
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_peer_memory_handshake(tmp_path, fail_rank):
    """Every rank opens every rank's blob, in rank order, once per token count;
    a rank whose set-up fails makes every rank raise (no rank waits for it)."""
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_handshake_worker, args=(world, _free_port(), str(tmp_path), fail_rank), nprocs=world,
                       start_method="spawn")
    for rank in range(world):
        res = np.load(tmp_path / f"h{rank}.npy", allow_pickle=True)[0]
        if fail_rank >= 0:
            assert not res["ok"] and "peer-memory expert parallelism unavailable" in res["error"], res
            continue
        assert res["ok"], res
        assert res["geometry"] == (rank, world, M)
        assert res["opened"] == {r: bytes([r, world, M]) for r in range(world)}
        assert res["decoded"] == [((M, HIDDEN), K), ((M, HIDDEN), K)]
        assert res["same"]
        assert res["active"] == "p2p"


def _bfp16_down_worker(rank, world, port, result_dir):
    import torch
    import torch.distributed as dist
    from raon_npu_b200.expert_parallel import ExpertParallelMoe
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer = HandshakeLayer(rank)
        layer.down_format = "bfp16"
        x = torch.zeros((M, HIDDEN), dtype=torch.int16)
        try:
            ExpertParallelMoe(layer, K, transport="p2p").decode(x, torch.empty_like(x))
            res = {"ok": True}
        except RuntimeError as e:
            res = {"ok": False, "error": str(e), "opened": layer.opened}
        np.save(os.path.join(result_dir, f"b{rank}.npy"), np.array([res], dtype=object), allow_pickle=True)
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_peer_memory_transport_refuses_bfp16_down_layers(tmp_path):
    """A layer whose down matrices are bfp16ebs8 is refused by the peer-memory
    transport on every rank before any exchange (the persistent kernel computes
    q4nx down matrices only); transport='auto' takes NCCL for it."""
    import torch.multiprocessing as mp
    world = 2
    mp.start_processes(_bfp16_down_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       start_method="spawn")
    for rank in range(world):
        res = np.load(tmp_path / f"b{rank}.npy", allow_pickle=True)[0]
        assert not res["ok"] and "q4nx down" in res["error"] and res["opened"] == {}, res
