"""Expert-parallel MoE decode (and prefill) on 2+ GPUs of one box.

Each rank (one process per GPU) holds E/N routed experts and the shared
expert and decodes its own tokens through ``ExpertParallelMoe``, over both
transports: ``"nccl"`` (all-gather, grouped expert GEMVs, reduce-scatter,
combine) and ``"p2p"`` (one persistent kernel that exchanges token and expert
rows through the ranks' peer-mapped buffers).  Every rank's output must
equal, byte for byte, the single-GPU ``MoeLayer.decode`` of the same tokens
with all experts loaded; the prefill of 40 tokens per rank (all-to-all of
the routed rows) must equal the single-GPU prefill.  The p2p case also makes a peer wait run out on
purpose -- rank 1 skips one call, so rank 0's kernel waits for token rows
that never come -- and checks that rank 0 gets the timeout status after the
1 s bound and that the layer then refuses further exchange calls.  Skipped
with fewer than 2 GPUs.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

E, H, I, K, M = 32, 2048, 768, 8, 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _layer(torch, ctx, owned):
    from raon_npu_b200.device import MoeLayer
    layer = MoeLayer(ctx, H, I, E, has_shared=True)
    gen = torch.Generator(device="cuda")
    for e in sorted(owned):
        gen.manual_seed(31_000 + e)
        gu = torch.randn((2 * I, H), generator=gen, device="cuda") * 0.02
        dn = torch.randn((H, I), generator=gen, device="cuda") * 0.02
        pgu = torch.empty(2 * I * H * 5 // 8, dtype=torch.uint8, device="cuda")
        pdn = torch.empty(H * I * 5 // 8, dtype=torch.uint8, device="cuda")
        ctx.quantize_q4nx(gu, pgu, 2 * I, H)
        ctx.quantize_q4nx(dn, pdn, H, I)
        layer.set_expert(e, pgu, pdn)
    rng = np.random.default_rng(5)
    wr = ((rng.standard_normal((E, H)) * 0.02).astype(np.float32).view(np.uint32) + 0x8000) >> 16
    layer.set_router(wr.astype(np.uint16))
    return layer


def _worker(rank, world, port, out_dir, transport):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from raon_npu_b200.build import build
        from raon_npu_b200.device import Context
        from raon_npu_b200.expert_parallel import ExpertParallelMoe
        build()
        ctx = Context(rank)
        per = E // world
        layer = _layer(torch, ctx, set(range(rank * per, (rank + 1) * per)) | {E})
        ep = ExpertParallelMoe(layer, K, act="swiglu", transport=transport)
        full = _layer(torch, ctx, set(range(E + 1)))
        gen = torch.Generator(device="cuda")
        res = []
        for trial in range(3):
            gen.manual_seed(100 * trial + rank)
            x = torch.randn((M, H), generator=gen, device="cuda").to(torch.bfloat16).view(torch.int16).contiguous()
            out = torch.empty((M, H), dtype=torch.int16, device="cuda")
            ep.decode(x, out)
            ref = torch.empty((M, H), dtype=torch.int16, device="cuda")
            full.decode(x, K, ref, act="swiglu")
            torch.cuda.synchronize()
            res.append(bool(torch.equal(out, ref)))
        host = ep.decode_host(x.cpu().numpy().view(np.uint16))
        res.append(bool(np.array_equal(host, ref.cpu().numpy().view(np.uint16))))
        ctx.sync()
        if transport == "nccl":
            # prefill, both exchanges: the gathered tokens with the slot rows
            # reduce-scattered, and the routed rows of remote routes in an
            # all-to-all there and back
            gen.manual_seed(700 + rank)
            xp = torch.randn((40, H), generator=gen, device="cuda").to(torch.bfloat16).view(torch.int16).contiguous()
            refp = torch.empty_like(xp)
            full.prefill(xp, K, refp, act="swiglu")
            for exchange in ("gather", "a2a"):
                ep.prefill_exchange = exchange
                outp = torch.empty_like(xp)
                ep.prefill(xp, outp)
                torch.cuda.synchronize()
                res.append(bool(torch.equal(outp, refp)))
                res.append(ep.last_prefill_exchange["rows_sent"] > 0)
            ctx.sync()
        if transport == "p2p":
            res.append(ep._ep_M == M)           # the peer path really ran
            dist.barrier()
            # rank 1 skips this call: rank 0's wait for its token rows runs out
            if rank == 0:
                layer.ep_decode(x, K, out, act="swiglu")
                try:
                    ctx.sync()
                    res.append(False)
                except RuntimeError as e:
                    res.append("bounded wait" in str(e))
                try:
                    layer.ep_decode(x, K, out, act="swiglu")
                    res.append(False)
                except RuntimeError as e:
                    res.append("rc_moe_ep_init" in str(e))
            torch.cuda.synchronize()
            dist.barrier()
        np.save(os.path.join(out_dir, f"ok{rank}.npy"), np.array(res))
        layer.close()
        full.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("transport", ["nccl", "p2p"])
def test_expert_parallel_matches_single_gpu_bytes(tmp_path, transport):
    import torch
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2 or more GPUs")
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path), transport), nprocs=world,
                       start_method="spawn")
    for r in range(world):
        ok = np.load(tmp_path / f"ok{r}.npy")
        assert ok.all(), (r, ok)
