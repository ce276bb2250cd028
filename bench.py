"""Benchmark of raon-npu's q4nx GEMV / MoE hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one config-3 MoE decode layer (hidden 2048,
128 routed experts + 1 shared, intermediate 768, softmax top-8, SwiGLU, q4nx
weights N(0, 0.02), bf16 tokens N(0, 1); synthetic and seeded) over one token
per rank, the routed experts sharded expert-parallel over the N ranks (one
process per GPU, torchrun), the token and expert rows exchanged inside the
decode kernel over NVLink peer memory.  ``value`` = tokens of all ranks per
second over the slowest rank's device time ("weak" scaling: the per-rank
work stays put as N grows); ``roofline`` = each rank's algorithmic bytes (the
packed weights of the distinct experts it streams, the shared expert, the
router weights and token rows) over that time, against the measured HBM copy
bandwidth.  Steps rotate over distinct layers, so no step finds its experts
in L2.  At N > 1 ``ep_parity`` decodes 16 tokens through the expert-parallel
layer and through one GPU holding every expert and compares the bytes.

Sub-objects: ``gemv_sweep`` -- the q4nx GEMV decode sweep (configs[1]: T in
{1,2,4,8,16} over 2048->4096, 4096->2048, 2048->512 and the 2048->151936
lm-head; dense, replicas only), GB/s of algorithmic bytes (N*K*5/8 packed
weights + 2*T*K + 2*T*N); ``config1`` -- the 4096x2048 T = 1 GEMV
(configs[0]); ``moe_prefill`` -- 512 tokens with a Zipf(1.1) expert load
(configs[3]); ``decode_step`` -- 48 layers + lm-head + sampling;
``per_shape``, ``bfp16`` and ``moe_bfp16_down`` at N = 1.

``--impl reference`` times the reference's own CPU arithmetic for this path
(the numpy restatement in ``oracle/`` of ``NumpyBackend`` and the router,
f32-dequantised weights cached) on the host cores with every BLAS thread,
rank 0 only, on the same MoE decode layer.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SHAPES = [(4096, 2048), (2048, 4096), (512, 2048), (151936, 2048)]   # (N out, K in)
TOKENS = [1, 2, 4, 8, 16]
METRIC = "q4nx GEMV HBM GB/s vs 8 TB/s; MoE layer tokens/s at 1/2/4/8 B200"
HBM_FALLBACK_GBS = 6650.0


# DRAM traffic of the timed work, from ncu captures of the same commands on a
# B200 (dram__bytes_read.sum + dram__bytes_write.sum): the GEMV launches of
# one sweep step; one config-3 decode layer at T = 1 (rc_moe_decode_kernel); the
# two grouped tcgen05 GEMMs of one 512-token prefill layer.  Single-GPU figures.
MEASURED_TRAFFIC = {"gemv_step": 1033.4e6, "moe_layer_t1": 27.16e6, "prefill_gemms": 264.79e6}
TRAFFIC_SOURCE = {
    "gemv_step": "profiles/gemv_sweep_launch_list.md (all rc_q4nx_gemv_kernel launches of one step)",
    "moe_layer_t1": "profiles/moe_decode_layer_t1.md (one rc_moe_decode_kernel launch, T = 1)",
    "prefill_gemms": "profiles/moe_prefill_gemm_t512.md (the two rc_pf_tc_kernel launches of a 512-token layer)",
}


def algo_bytes(n: int, k: int, t: int) -> int:
    return n * k * 5 // 8 + 2 * t * k + 2 * t * n


def step_bytes() -> int:
    return sum(algo_bytes(n, k, t) for t in TOKENS for n, k in SHAPES)


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return HBM_FALLBACK_GBS, "fallback"


# --------------------------------------------------------------- clocks --
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ our arm --
def capture_graph(torch, fn):
    """Capture ``fn``'s launches (issued on torch's current stream) into a CUDA graph."""
    g = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()                      # one eager pass on the capture stream
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        fn()
    return g


def run_ours(args, rank: int, world: int, local_rank: int):
    """Our arm.  The JSON line's ``value`` is the config-3 MoE decode layer
    (the half of the metric that shards): tokens/s of all
    ranks, one token per rank per step, experts expert-parallel over the
    ranks.  The GEMV sweep and config 1 follow as sub-objects,
    then prefill and the 48-layer decode step."""
    import torch
    import torch.distributed as dist
    from raon_npu_b200.device import Context

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    ctx = Context(local_rank)

    def barrier():
        if world > 1:
            dist.barrier()

    moe = run_moe(args, ctx, torch, dev, rank, world, local_rank, barrier)
    sweep = None if args.no_gemv else run_gemv_sweep(args, ctx, torch, dev, rank, world, local_rank, barrier)
    prefill = None if args.no_prefill else run_moe_prefill(args, ctx, torch, dev, rank, world, local_rank, barrier)
    dstep = None if args.no_decode_step else run_decode_step(args, ctx, torch, dev, rank, world, local_rank,
                                                             barrier)
    moe_bf = None
    if world == 1 and not args.no_extras:
        moe_bf = measure_moe_bfp16_down(args, ctx, torch, dev)

    if rank == 0:
        line = {
            "metric": METRIC, "value": moe["value"], "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": moe["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "u4 codes (q4nx), bf16 act, f32 acc",
            "data": "synthetic: q4nx weights from N(0,0.02) f32 (torch cuda generator, seeded, quantised on the "
                    "GPU bit-identically to the reference quantiser), bf16 x N(0,1)",
            "config": moe["config"],
            "roofline": moe["roofline"],
            "e2e": moe["e2e"],
            "cpu_baseline": moe["cpu_baseline"],
            "gpu_launches": moe["gpu_launches"],
            "clocks": moe["clocks"],
            "ep_parity": moe["ep_parity"],
            "moe_phases_us": moe.get("phases_us"),
            "moe_prefill": prefill,
            "decode_step": dstep,
            "gemv_sweep": sweep["sweep"] if sweep else None,
            "config1": sweep["config1"] if sweep else None,
            "per_shape": sweep["per_shape"] if sweep else None,
            "bfp16": sweep["bfp16"] if sweep else None,
            "moe_bfp16_down": moe_bf,
        }
        print(json.dumps(line), flush=True)
    ctx.close()


def run_gemv_sweep(args, ctx, torch, dev, rank: int, world: int, local_rank: int, barrier):
    """the q4nx GEMV decode sweep (dense GEMV: replicas
    only, so at N GPUs each rank runs its own copy); config 1 as its own
    entry; the per-shape launch table and the bfp16ebs8 GEMV (rank 0, N = 1)."""
    import torch.distributed as dist
    stream = torch.cuda.current_stream(dev)
    gen = torch.Generator(device=dev)

    # Weights: seeded N(0, 0.02) f32 on the device -> q4nx (rc_quantize_q4nx,
    # bit-identical to the reference quantiser) -> uploaded copies.
    weights = {}      # (n, k) -> list of Q4nxWeight (one per T; distinct buffers)
    for si, (n, k) in enumerate(SHAPES):
        gen.manual_seed(1000 + si)
        w = torch.randn((n, k), generator=gen, device=dev, dtype=torch.float32) * 0.02
        packed = torch.empty(n * k * 5 // 8, dtype=torch.uint8, device=dev)
        ctx.quantize_q4nx(w, packed, n, k)
        del w
        copies = 1 if n * k > 100_000_000 else len(TOKENS)
        weights[(n, k)] = [ctx.upload_q4nx(packed, n, k) for _ in range(copies)]
        del packed
    xs, ys = {}, {}
    for t in TOKENS:
        for n, k in SHAPES:
            gen.manual_seed(7 * t + k)
            xf = torch.randn((t, k), generator=gen, device=dev, dtype=torch.float32)
            xs[(n, k, t)] = xf.to(torch.bfloat16).view(torch.int16).contiguous()
            ys[(n, k, t)] = torch.empty((t, n), dtype=torch.int16, device=dev)
    torch.cuda.synchronize()
    launches_per_step = len(TOKENS) * len(SHAPES)   # one fused GEMV kernel per matrix

    def step():
        for ti, t in enumerate(TOKENS):
            for n, k in SHAPES:
                cps = weights[(n, k)]
                cps[ti % len(cps)].gemv_into(xs[(n, k, t)], ys[(n, k, t)], t)

    # Eager warm-up (sizes the scratch), then capture one step in a CUDA graph:
    # a decode step is a fixed launch sequence, replayed without host overhead.
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.sync()
    step_graph = capture_graph(torch, step)
    for _ in range(args.warmup):
        step_graph.replay()
    torch.cuda.synchronize()
    ctx.sync()
    barrier()
    clocks = ClockSampler(_gpu_index(local_rank))
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step_graph.replay()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = _max_over_ranks(torch, dist, dev, world, ms)
    del step_graph
    ctx.sync()
    sb = step_bytes()
    peak, peak_kind = peaks()
    achieved = sb / (ms * 1e-3) / 1e9

    # Per-shape launch times (rank 0, one GPU): back-to-back launches over
    # rotating copies whose total exceeds L2, so each launch streams from HBM.
    per_shape, bfp16 = None, None
    if rank == 0 and world == 1 and not args.no_extras:
        per_shape = measure_per_shape(ctx, torch, dev, gen, stream, weights)
        bfp16 = measure_bfp16(ctx, torch, dev, gen)

    # End to end through the host-buffer C-ABI entry point (rc_gemv_host):
    # pinned host x -> device, GEMV, y -> host, every GEMV of the step.
    host_x = {key: x.cpu().numpy().view(np.uint16) for key, x in xs.items()}

    def e2e_pass():
        for ti, t in enumerate(TOKENS):
            for n, k in SHAPES:
                weights[(n, k)][ti % len(weights[(n, k)])].gemv_host(host_x[(n, k, t)])
    e2e_pass()
    barrier()
    e2e_steps = max(2, min(args.steps, 5))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_pass()
    e2e_s = _max_over_ranks(torch, dist, dev, world, (time.perf_counter() - t0) / e2e_steps)
    h2d = sum(2 * t * k for t in TOKENS for n, k in SHAPES)
    d2h = sum(2 * t * n for t in TOKENS for n, k in SHAPES)

    # Config 1 (4096 x 2048, T = 1) on its own: device time per launch from the
    # per-shape table, end to end through rc_gemv_host, the oracle's f32 GEMV.
    config1 = None
    if rank == 0 and world == 1:
        n1, k1 = 4096, 2048
        w1 = weights[(n1, k1)][0]
        x1 = host_x[(n1, k1, 1)]
        for _ in range(3):
            w1.gemv_host(x1)
        reps = 200
        t0 = time.perf_counter()
        for _ in range(reps):
            w1.gemv_host(x1)
        e2e1 = (time.perf_counter() - t0) / reps
        b1 = algo_bytes(n1, k1, 1)
        row = [e for e in (per_shape or []) if e["k_to_n"] == f"{k1}->{n1}" and e["t"] == 1]
        config1 = {"workload": "BASELINE configs[0]: q4nx GEMV 4096x2048 (out x in), T = 1",
                   "algorithmic_bytes": b1,
                   "us_per_launch": row[0]["us_per_launch"] if row else None,
                   "gbs": row[0]["gbs"] if row else None, "frac": row[0]["frac"] if row else None,
                   "timing": "back-to-back launches over rotating copies larger than L2 (CUDA events)",
                   "e2e": {"value": round(b1 / e2e1 / 1e9, 3), "unit": "GB/s", "us_per_call": round(e2e1 * 1e6, 2),
                           "h2d_bytes_per_step": 2 * k1, "d2h_bytes_per_step": 2 * n1,
                           "api": "rc_gemv_host (synchronous)"}}
        if not args.no_cpu_baseline:
            config1["cpu_baseline"] = cpu_config1(ctx, torch, dev, w1, x1, budget_s=min(5.0, args.cpu_seconds))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(ctx, torch, dev, weights, host_x, budget_s=args.cpu_seconds)
    for ws in weights.values():
        for w in ws:
            w.free()
    weights.clear()
    sweep = {
        "metric": "q4nx GEMV HBM GB/s (BASELINE configs[1] sweep)", "value": round(world * sb / (ms_max * 1e-3) / 1e9, 2),
        "unit": "GB/s", "ms_per_step": round(ms_max, 4), "steps": args.steps,
        "config": {"shapes_k_to_n": [f"{k}->{n}" for n, k in SHAPES], "tokens": TOKENS,
                   "parallelism": f"replicas x{world} (dense GEMV does not shard)",
                   "l2": "each step streams %.2f GB of distinct weights" % (sb / 1e9),
                   "algorithmic_bytes_per_step": sb},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "traffic": MEASURED_TRAFFIC["gemv_step"], "traffic_source": TRAFFIC_SOURCE["gemv_step"],
                     "kernel": "rc_q4nx_gemv_kernel (20 launches per step)"},
        "e2e": {"value": round(world * sb / e2e_s / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "api": "rc_gemv_host (synchronous per GEMV)"},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk,
        "cpu_baseline": cpu,
    }
    return {"sweep": sweep, "config1": config1, "per_shape": _compact_shapes(per_shape), "bfp16": bfp16}


def _max_over_ranks(torch, dist, dev, world: int, v: float) -> float:
    if world == 1:
        return v
    tt = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    return float(tt.item())


def _compact_shapes(rows):
    """Per-shape launch table as {"KxN": {T: [us per launch, fraction of peak]}}."""
    if rows is None:
        return None
    out = {}
    for e in rows:
        out.setdefault(e["k_to_n"], {})[e["t"]] = [e["us_per_launch"], e["frac"]]
    return out


def measure_bfp16(ctx, torch, dev, gen):
    """The bfp16ebs8 GEMV (the reference's second weight format, rc_upload_bfp16
    + rc_gemv) on the sweep's shapes: synthetic packed blocks made on the device
    (exponent bytes 118..124, i.e. weights around 2^-9..2^-3, random int8
    mantissas), back-to-back launches over rotating copies larger than L2."""
    peak, _ = peaks()
    out = []
    for n, k in SHAPES:
        nbytes = n * k * 9 // 8
        copies = max(1, min(64, (400 << 20) // nbytes))
        cps = []
        for c in range(copies):
            gen.manual_seed(9000 + n + k + c)
            blk = torch.randint(0, 256, (nbytes // 144, 144), generator=gen, device=dev, dtype=torch.uint8)
            blk[:, :16] = torch.randint(118, 125, (nbytes // 144, 16), generator=gen, device=dev, dtype=torch.uint8)
            cps.append(ctx.upload_bfp16(blk.view(-1), n, k))
            del blk
        launches = max(20, min(200, copies * 2))
        for t in TOKENS:
            x = torch.randn((t, k), generator=gen, device=dev).to(torch.bfloat16).view(torch.int16).contiguous()
            y = torch.empty((t, n), dtype=torch.int16, device=dev)
            for i in range(min(launches, 10)):
                cps[i % len(cps)].gemv_into(x, y, t)
            torch.cuda.synchronize()

            def seq():
                for i in range(launches):
                    cps[i % len(cps)].gemv_into(x, y, t)
            g = capture_graph(torch, seq)
            g.replay()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            st = torch.cuda.current_stream(dev)
            e0.record(st)
            g.replay()
            e1.record(st)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / launches
            del g
            gbs = (nbytes + 2 * t * (n + k)) / (us * 1e-6) / 1e9
            out.append({"k_to_n": f"{k}->{n}", "t": t, "us_per_launch": round(us, 3), "gbs": round(gbs, 1),
                        "frac": round(gbs / peak, 4), "copies": len(cps)})
        for w in cps:
            w.free()
    ctx.sync()
    return {"workload": "bfp16ebs8 GEMV (9-bit weights), synthetic blocks, rotating copies > L2",
            "kernel": "rc_bfp16_gemv_kernel", "per_shape_us_frac": _compact_shapes(out)}


def measure_per_shape(ctx, torch, dev, gen, stream, weights):
    out = []
    peak, _ = peaks()
    for n, k in SHAPES:
        packed_bytes = n * k * 5 // 8
        copies = max(1, min(512, (400 << 20) // packed_bytes))
        if copies > 1:
            gen.manual_seed(5000 + n + k)
            w = torch.randn((n, k), generator=gen, device=dev, dtype=torch.float32) * 0.02
            packed = torch.empty(packed_bytes, dtype=torch.uint8, device=dev)
            ctx.quantize_q4nx(w, packed, n, k)
            del w
            cps = [ctx.upload_q4nx(packed, n, k) for _ in range(copies)]
            del packed
        else:
            cps = weights[(n, k)][:1]
        launches = max(50, min(400, copies * 2))
        for t in TOKENS:
            x = torch.randn((t, k), generator=gen, device=dev).to(torch.bfloat16).view(torch.int16).contiguous()
            y = torch.empty((t, n), dtype=torch.int16, device=dev)
            for i in range(min(launches, 20)):
                cps[i % len(cps)].gemv_into(x, y, t)
            torch.cuda.synchronize()

            def seq():
                for i in range(launches):
                    cps[i % len(cps)].gemv_into(x, y, t)
            g = capture_graph(torch, seq)
            g.replay()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            stream = torch.cuda.current_stream(dev)
            e0.record(stream)
            g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / launches
            del g
            gbs = algo_bytes(n, k, t) / (us * 1e-6) / 1e9
            out.append({"k_to_n": f"{k}->{n}", "t": t, "us_per_launch": round(us, 3), "gbs": round(gbs, 1),
                        "frac": round(gbs / peak, 4), "copies": len(cps)})
        if copies > 1:
            for w in cps:
                w.free()
    ctx.sync()
    return out


# ---------------------------------------------------- MoE decode layer --
# hidden 2048, 128 routed experts + 1 shared, SwiGLU
# gate/up 2048->768 and down 768->2048 in q4nx, softmax router top-8, one
# token per rank per step, experts sharded expert-parallel over the ranks.
MOE = dict(hidden=2048, inter=768, experts=128, k=8, tokens_per_rank=1)


def moe_expert_bytes(hidden: int, inter: int) -> int:
    inter_pad = (inter + 255) // 256 * 256
    return 2 * inter * hidden * 5 // 8 + hidden * inter_pad * 5 // 8


def _moe_seed(layer: int, expert: int) -> int:
    return 7_000_000 + 1000 * layer + expert


def build_moe_layers(ctx, torch, dev, n_layers: int, first: int = 0, all_experts: bool = False):
    """n_layers distinct config-3 layers (layer ids first, first + 1, ...); this
    rank loads its own experts and the shared one, or every expert with
    ``all_experts`` (weights seeded per (layer, expert), so every rank agrees)."""
    from raon_npu_b200.device import MoeLayer
    from raon_npu_b200.expert_parallel import ExpertParallelMoe
    H, I, E, k = MOE["hidden"], MOE["inter"], MOE["experts"], MOE["k"]
    gen = torch.Generator(device=dev)
    eps = []
    for li in range(first, first + n_layers):
        layer = MoeLayer(ctx, H, I, E, has_shared=True)
        ep = ExpertParallelMoe(layer, k, act="swiglu", router="softmax")
        for e in range(E + 1):
            if not (all_experts or ep.owns(e)):
                continue
            gen.manual_seed(_moe_seed(li, e))
            gu = torch.randn((2 * I, H), generator=gen, device=dev) * 0.02
            dn = torch.randn((H, I), generator=gen, device=dev) * 0.02
            pgu = torch.empty(2 * I * H * 5 // 8, dtype=torch.uint8, device=dev)
            pdn = torch.empty(H * I * 5 // 8, dtype=torch.uint8, device=dev)
            ctx.quantize_q4nx(gu, pgu, 2 * I, H)
            ctx.quantize_q4nx(dn, pdn, H, I)
            layer.set_expert(e, pgu, pdn)
        gen.manual_seed(_moe_seed(li, 999))
        wr = (torch.randn((E, H), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        layer.set_router(wr.view(torch.int16).cpu().numpy().view(np.uint16))
        eps.append(ep)
    torch.cuda.synchronize()
    return eps


def build_bfp16_down_layers(ctx, torch, dev, n_layers: int):
    """n_layers config-3 layers with q4nx gate/up (seeded as the q4nx layers)
    and synthetic bfp16ebs8 down matrices made on the device (exponent bytes
    118..124, random int8 mantissas)."""
    from raon_npu_b200.device import MoeLayer
    H, I, E = MOE["hidden"], MOE["inter"], MOE["experts"]
    ip = (I + 255) // 256 * 256
    gen = torch.Generator(device=dev)
    layers = []
    for li in range(n_layers):
        layer = MoeLayer(ctx, H, I, E, has_shared=True)
        for e in range(E + 1):
            gen.manual_seed(_moe_seed(li, e))
            gu = torch.randn((2 * I, H), generator=gen, device=dev) * 0.02
            pgu = torch.empty(2 * I * H * 5 // 8, dtype=torch.uint8, device=dev)
            ctx.quantize_q4nx(gu, pgu, 2 * I, H)
            blk = torch.randint(0, 256, (H * ip * 9 // 8 // 144, 144), generator=gen, device=dev, dtype=torch.uint8)
            blk[:, :16] = torch.randint(118, 125, (blk.shape[0], 16), generator=gen, device=dev, dtype=torch.uint8)
            layer.set_expert(e, pgu, blk.view(-1), down_format="bfp16")
        gen.manual_seed(_moe_seed(li, 999))
        wr = (torch.randn((E, H), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        layer.set_router(wr.view(torch.int16).cpu().numpy().view(np.uint16))
        layers.append(layer)
    torch.cuda.synchronize()
    return layers


def measure_moe_bfp16_down(args, ctx, torch, dev):
    """The config-3 decode layer (T = 1) with the experts' down matrices in
    bfp16ebs8, as the reference's production bundles store them (moe_b2):
    router, q4nx gate/up with the GLU epilogue, the grouped bfp16 down kernel
    and the combine as separate launches in one CUDA graph per layer.
    Synthetic down blocks are made on the device (exponent bytes 118..124,
    random int8 mantissas); layers rotate as in the q4nx measurement."""
    H, I, E, k = MOE["hidden"], MOE["inter"], MOE["experts"], MOE["k"]
    ip = (I + 255) // 256 * 256
    eb = 2 * I * H * 5 // 8 + H * ip * 9 // 8
    touched = (k + 1) * eb
    n_layers = min(24, max(2, -(-3 * 126_000_000 // touched)))
    gen = torch.Generator(device=dev)
    layers = build_bfp16_down_layers(ctx, torch, dev, n_layers)
    gen.manual_seed(4343)
    xs = [torch.randn((1, H), generator=gen, device=dev).to(torch.bfloat16).view(torch.int16).contiguous()
          for _ in range(n_layers)]
    outs = [torch.empty((1, H), dtype=torch.int16, device=dev) for _ in range(n_layers)]
    for _ in range(args.warmup):
        for li in range(n_layers):
            layers[li].decode(xs[li], k, outs[li])
    torch.cuda.synchronize()
    ctx.sync()
    graphs = [capture_graph(torch, lambda li=li: layers[li].decode(xs[li], k, outs[li])) for li in range(n_layers)]
    for s in range(args.warmup * n_layers):
        graphs[s % n_layers].replay()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(st)
    for s in range(args.steps):
        graphs[s % n_layers].replay()
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    del graphs
    ctx.sync()
    step_bytes = []
    for li in range(n_layers):
        ids = torch.empty((1, k), dtype=torch.int32, device=dev)
        w = torch.empty((1, k), dtype=torch.float32, device=dev)
        layers[li].route(xs[li], 1, k, ids, w)
        torch.cuda.synchronize()
        step_bytes.append((len(set(ids.cpu().numpy().ravel().tolist())) + 1) * eb + E * H * 2 + 4 * H)
    b = sum(step_bytes[s % n_layers] for s in range(args.steps)) / args.steps
    # prefill of 512 tokens through the first two layers (register-fragment gate/up, bfp16 grouped down)
    xp = torch.randn((PREFILL_TOKENS, H), generator=gen, device=dev).to(torch.bfloat16).view(torch.int16)
    op = torch.empty_like(xp)
    for _ in range(args.warmup):
        layers[0].prefill(xp, k, op)
    pgraphs = [capture_graph(torch, lambda li=li: layers[li].prefill(xp, k, op)) for li in range(2)]
    torch.cuda.synchronize()
    e0.record(st)
    for s in range(args.steps):
        pgraphs[s % 2].replay()
    e1.record(st)
    torch.cuda.synchronize()
    pms = e0.elapsed_time(e1) / args.steps
    del pgraphs
    for layer in layers:
        layer.close()
    peak, peak_kind = peaks()
    gbs = b / (ms * 1e-3) / 1e9
    return {"metric": "MoE decode layer tokens/s", "value": round(1 / (ms * 1e-3), 1), "unit": "tokens/s",
            "ms_per_step": round(ms, 5), "steps": args.steps,
            "config": {"workload": "config-3 MoE decode layer, T = 1, down matrices bfp16ebs8 (9-bit), "
                                   "gate/up q4nx", "layers_rotated": n_layers,
                       "path": "separate launches (router, gate/up GEMV + GLU, grouped bfp16 down, combine) "
                               "in one CUDA graph per layer"},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 4), "peak_source": peak_kind,
                         "bytes_per_step": round(b), "expert_bytes": eb},
            "prefill": {"tokens": PREFILL_TOKENS, "ms_per_step": round(pms, 4),
                        "tokens_per_s": round(PREFILL_TOKENS / (pms * 1e-3), 1),
                        "router": "softmax, unbiased", "path": "router, plan, register-fragment gate/up GEMV, "
                        "bfp16 grouped down over 8-row expert blocks, combine (one CUDA graph)"}}


def cpu_threads() -> dict:
    """Give the CPU legs every host core: ``torchrun`` sets OMP_NUM_THREADS=1
    for its workers, so the BLAS thread pools are raised to os.cpu_count()
    explicitly.  Returns the threads each pool now uses."""
    n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info, threadpool_limits
        threadpool_limits(limits=n)
        pools = {f"{i.get('internal_api')}": i.get("num_threads") for i in threadpool_info()}
    except Exception as e:          # noqa: BLE001 - reported in the JSON line
        pools = {"threadpoolctl": f"unavailable: {type(e).__name__}"}
    nums = [v for v in pools.values() if isinstance(v, int)]
    return {"threads": max(nums) if nums else 1, "pools": pools}


_MOE_CPU_CACHE: dict = {}


def moe_cpu_sample(n_tokens: int, budget_s: float, bias: np.ndarray | None = None):
    """The reference's CPU arithmetic for one config-3 decode layer (oracle port:
    router, routed experts in ascending ID, shared expert), timed per token
    over f32-dequantised weights cached.  To bound the setup, 16 distinct
    expert weight sets are generated and expert e uses set e % 16 (every
    expert has the same shape, so the timed arithmetic is unchanged).
    Returns (tokens, seconds)."""
    from oracle import backend as ob
    from oracle import q4nx as q
    H, I, E, k = MOE["hidden"], MOE["inter"], MOE["experts"], MOE["k"]
    rng = np.random.default_rng(77)
    wr = q.f32_to_bf16((rng.standard_normal((E, H)) * 0.02).astype(np.float32))
    cache = _MOE_CPU_CACHE

    def expert(e):
        if e not in cache:
            _, c, s_, m = q.normal_weight_q4nx(2 * I, H, seed=_moe_seed(0, e))
            gu = q.dequantize_simple(c, s_, m)
            _, c, s_, m = q.normal_weight_q4nx(H, I, seed=_moe_seed(0, e) + 500)
            cache[e] = (gu[:I], gu[I:], q.dequantize_simple(c, s_, m))
        return cache[e]
    done, secs = 0, 0.0
    shared = expert(E)
    while done < n_tokens and (secs < budget_s or done == 0):
        x = q.f32_to_bf16(rng.standard_normal(H).astype(np.float32))
        t0 = time.perf_counter()
        if bias is None:
            ids, _, _ = ob.route_softmax(x, wr, k)
            experts = {int(e): expert(int(e) % 16) for e in ids}
            t0 = time.perf_counter()
            ob.moe_decode_layer(experts, shared, wr, x, k, act="swiglu")
        else:
            # the prefill router of config 4: softmax of the biased logits
            logits = (ob.router_logits(x, wr) + bias).astype(np.float32)
            ids = ob.topk_lower_index_wins(logits, k)
            sel = logits[ids].astype(np.float64)
            ew = np.exp(sel - sel.max())
            w = (ew / ew.sum()).astype(np.float32)
            experts = {int(e): expert(int(e) % 16) for e in ids}
            routed = ob.moe_experts(experts, x, ids, w, act="swiglu")
            ob.moe_token_with_shared(routed, ob.expert_forward(*shared, x, "swiglu"))
        secs += time.perf_counter() - t0
        done += 1
    return done, secs


def moe_cpu_baseline(budget_s: float) -> dict:
    th = cpu_threads()
    n_tok, secs = moe_cpu_sample(256, budget_s)
    return {"value": round(n_tok / secs, 2), "unit": "tokens/s", "cores": th["threads"], "kind": "port",
            "blas_threads": th["pools"],
            "sample": f"{n_tok} decode tokens through the oracle's numpy MoE layer (router, 8 routed + shared "
                      f"SwiGLU experts, ascending-ID combine; host/backend.py:466-510, host/raon.py:1224-1327 "
                      f"restated), f32 weights cached (16 weight sets, id mod 16)"}


def _gather_tokens(torch, dist, world, x):
    if world == 1:
        return x
    g = torch.empty((world * x.shape[0], x.shape[1]), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(g.view(torch.bfloat16), x.view(torch.bfloat16))
    return g


def moe_ep_parity(ctx, torch, dev, rank: int, world: int, ep) -> dict:
    """N > 1: the same 16 tokens through the expert-parallel layer (16/N per
    rank, its exchange inside the decode kernel over NVLink peer memory) and
    through a one-GPU ``rc_moe_decode`` of the same layer holding every expert
    (rank 0): ``equal`` when every byte agrees."""
    import torch.distributed as dist
    H, k = MOE["hidden"], MOE["k"]
    M = 16 // world
    gen = torch.Generator(device=dev)
    gen.manual_seed(6161)                       # the same 16 tokens on every rank
    xall = torch.randn((world * M, H), generator=gen, device=dev).to(torch.bfloat16).view(torch.int16)
    mine = xall[rank * M:(rank + 1) * M].contiguous()
    out = torch.empty((M, H), dtype=torch.int16, device=dev)
    torch.cuda.synchronize()
    dist.barrier()
    ep.decode(mine, out)
    transport = ep.active_transport
    torch.cuda.synchronize()
    ctx.sync()
    got = torch.empty((world * M, H), dtype=torch.int16, device=dev)
    dist.all_gather_into_tensor(got.view(torch.bfloat16), out.view(torch.bfloat16))
    ok, diff = 1, 0
    if rank == 0:
        full = build_moe_layers(ctx, torch, dev, 1, first=0, all_experts=True)[0]
        ref = torch.empty_like(got)
        full.layer.decode(xall, k, ref, act="swiglu")
        torch.cuda.synchronize()
        ctx.sync()
        diff = int((ref != got).sum().item())
        ok = int(diff == 0)
        full.layer.close()
    flag = torch.tensor([ok, diff], dtype=torch.int64, device=dev)
    dist.broadcast(flag, 0)
    return {"equal": bool(flag[0].item()), "tokens": world * M, "tokens_per_rank": M,
            "differing_values": int(flag[1].item()), "transport": transport,
            "reference": "rc_moe_decode of the same layer with all 129 experts on rank 0's GPU"}


def moe_phase_trace(ctx, torch, dev, eps, xs, outs, calls: int, barrier) -> dict:
    """Where a decode step's time goes in the timed loop's steady state: the
    decode kernel's global-timer phase stamps (rc_moe_set_trace) of the last
    of ``calls`` L2-cold steps (layers rotated as in the timed loop) replayed
    back to back in one CUDA graph, over a few replays.  Per phase: [median,
    max] over CTAs of the stamp, in us after the earliest CTA started,
    averaged over the replays (this rank)."""
    from raon_npu_b200.device import MoeLayer
    n = ctx.sm_count
    buf = torch.zeros(n * 16, dtype=torch.int64, device=dev)
    for ep in eps:
        ep.layer.set_trace(buf, n)

    def seq():
        for c in range(calls):
            li = c % len(eps)
            eps[li].decode(xs[li], outs[li])
    seq()
    torch.cuda.synchronize()
    g = capture_graph(torch, seq)
    rows = []
    for _ in range(3):
        barrier()
        g.replay()
        torch.cuda.synchronize()
        rows.append(buf.view(n, 16).cpu().numpy().astype(np.int64))
    del g
    for ep in eps:
        ep.layer.set_trace(None, 0)
    ctx.sync()
    res = {}
    for i, name in enumerate(MoeLayer.TRACE_PHASES):
        med, mx = [], []
        for st in rows:
            col = st[:, i]
            if not col.any():
                continue
            t0 = st[:, 0].min()
            med.append((np.median(col) - t0) / 1e3)
            mx.append((col.max() - t0) / 1e3)
        if med:
            res[name] = [round(float(np.mean(med)), 2), round(float(np.mean(mx)), 2)]
    return res


def run_moe(args, ctx, torch, dev, rank: int, world: int, local_rank: int, barrier):
    """Config-3 MoE decode layer, expert-parallel over the ranks: tokens/s of
    all ranks, per-rank HBM roofline of the experts each rank streams."""
    import torch.distributed as dist
    H, E, k, M = MOE["hidden"], MOE["experts"], MOE["k"], MOE["tokens_per_rank"]
    eb = moe_expert_bytes(H, MOE["inter"])
    # expert bytes one rank streams per step: its share of the experts the
    # world*M tokens select, plus the shared expert
    touched = (min(world * M * k, E) // world + 1) * eb
    # rotate over enough distinct layers (each with its own fixed tokens, so
    # its own experts) that a layer's experts left L2 long before it returns
    n_layers = min(24, max(2, -(-3 * 126_000_000 // touched)))
    eps = build_moe_layers(ctx, torch, dev, n_layers)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4242 + rank)
    xs = [torch.randn((M, H), generator=gen, device=dev).to(torch.bfloat16).view(torch.int16).contiguous()
          for _ in range(n_layers)]
    outs = [torch.empty((M, H), dtype=torch.int16, device=dev) for _ in range(n_layers)]

    # eager warm-up; it also creates the NCCL communicators before any capture
    for _ in range(args.warmup):
        for li in range(n_layers):
            eps[li].decode(xs[li], outs[li])
    torch.cuda.synchronize()
    ctx.sync()

    # The timed steps run as one CUDA graph of args.steps consecutive layer
    # decodes (step s decodes layer s % n_layers), as a decode step runs its
    # layers back to back; warm-up replays the same graph.
    def steps_fn():
        for s_ in range(args.steps):
            eps[s_ % n_layers].decode(xs[s_ % n_layers], outs[s_ % n_layers])
    graph, graph_err = None, None
    try:
        graph = capture_graph(torch, steps_fn)
    except Exception as e:                  # noqa: BLE001 - reported in the JSON line
        graph, graph_err = None, f"{type(e).__name__}: {e}"[:200]
    ok = torch.tensor([1 if graph is not None else 0], dtype=torch.int32, device=dev)
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if not int(ok.item()):
        graph = None
    run_steps = graph.replay if graph is not None else steps_fn
    for _ in range(max(1, -(-args.warmup // args.steps))):
        run_steps()
    torch.cuda.synchronize()
    ctx.sync()
    barrier()
    clocks = ClockSampler(_gpu_index(local_rank))
    clocks.start()
    time.sleep(0.3)
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    run_steps()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms_max = _max_over_ranks(torch, dist, dev, world, e0.elapsed_time(e1) / args.steps)
    del graph
    ctx.sync()

    # Algorithmic bytes of each step on this rank: the packed weights of the
    # distinct experts it owns that the gathered tokens chose, the shared
    # expert, the router weights and the token rows.
    lo, hi = eps[0].experts
    T = world * M
    layer_bytes = []
    for li in range(n_layers):
        xg = _gather_tokens(torch, dist, world, xs[li])
        ids = torch.empty((T, k), dtype=torch.int32, device=dev)
        w = torch.empty((T, k), dtype=torch.float32, device=dev)
        eps[li].layer.route(xg, T, k, ids, w)
        torch.cuda.synchronize()
        active = {int(e) for e in ids.cpu().numpy().ravel() if lo <= int(e) < hi}
        layer_bytes.append((len(active) + 1) * eb + E * H * 2 + 4 * T * H)
    rank_bytes = sum(layer_bytes[s % n_layers] for s in range(args.steps)) / args.steps
    rb = torch.tensor([rank_bytes], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(rb)
    avg_rank_bytes = float(rb.item()) / world
    peak, peak_kind = peaks()
    achieved = avg_rank_bytes / (ms_max * 1e-3) / 1e9

    # End to end through the host entry point: pinned host token rows -> device,
    # expert-parallel decode (exchange included), rows back to the host.
    host_x = [x.cpu().numpy().view(np.uint16) for x in xs]
    e2e_n = max(2 * n_layers, min(args.steps, 64))
    for li in range(n_layers):
        eps[li].decode_host(host_x[li])
    barrier()
    t0 = time.perf_counter()
    for s in range(e2e_n):
        eps[s % n_layers].decode_host(host_x[s % n_layers])
    e2e_s = _max_over_ranks(torch, dist, dev, world, (time.perf_counter() - t0) / e2e_n)

    transport = eps[0].active_transport
    phases = None
    if world == 1 or transport == "p2p":
        barrier()
        phases = moe_phase_trace(ctx, torch, dev, eps, xs, outs, calls=2 * n_layers, barrier=barrier)
    parity = moe_ep_parity(ctx, torch, dev, rank, world, eps[0]) if world > 1 else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = moe_cpu_baseline(args.cpu_seconds)
    if world == 1 or transport == "p2p":
        per_step, kdesc = 1, "rc_moe_decode_kernel: router, top-k, grouped gate/up and down GEMVs, combine" + (
            "; token and expert rows exchanged over NVLink peer stores inside it" if world > 1 else "")
    else:
        per_step, kdesc = 2, ("rc_moe_decode_kernel (local experts) + combine, NCCL all-gather and reduce-scatter "
                              "around them")
    barrier()
    for ep in eps:
        ep.layer.close()
    return {
        "value": round(world * M / (ms_max * 1e-3), 1), "ms_per_step": round(ms_max, 5),
        "config": {"workload": "MoE decode layer (BASELINE configs[2]): hidden 2048, 128 experts + 1 shared, "
                               "I=768, softmax top-8, SwiGLU, q4nx", "tokens_per_rank": M,
                   "parallelism": f"ep{world}", "experts_per_rank": E // world, "transport": transport,
                   "l2": "steps rotate over %d distinct layers; a layer's %.1f MB of experts return after "
                         "%.0f MB of other layers' (> L2 126 MB)" % (n_layers, touched / 1e6,
                                                                      (n_layers - 1) * touched / 1e6),
                   "cuda_graph": bool(int(ok.item())), "graph_error": graph_err,
                   "timing": "one CUDA graph of the K timed layer decodes, back to back"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "traffic": MEASURED_TRAFFIC["moe_layer_t1"] if world == 1 and M == 1 else None,
                     "traffic_source": TRAFFIC_SOURCE["moe_layer_t1"],
                     "per_rank_bytes_per_step": round(avg_rank_bytes), "kernel": kdesc},
        "e2e": {"value": round(world * M / e2e_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": 2 * M * H,
                "d2h_bytes_per_step": 2 * M * H, "api": "ExpertParallelMoe.decode_host -> rc_moe_decode_host / rc_moe_ep_decode_host (synchronous)"},
        "gpu_launches": per_step * args.steps,
        "clocks": clk,
        "cpu_baseline": cpu,
        "ep_parity": parity,
        "phases_us": phases,
    }


# ------------------------------------------------------- MoE prefill layer --
# 512 tokens x hidden 2048 through the config-3 layer,
# router logits biased b_e = -1.1 ln(rank_e) (rank: seeded permutation of
# 1..128) so the expert load follows Zipf(1.1); the tensor-core grouped GEMM;
# expert-parallel at N GPUs with the 512 tokens split over the ranks.
PREFILL_TOKENS = 512


def zipf_bias(n_experts: int) -> np.ndarray:
    rank = np.random.default_rng(4321).permutation(n_experts) + 1
    return (-1.1 * np.log(rank)).astype(np.float32)


def run_moe_prefill(args, ctx, torch, dev, rank: int, world: int, local_rank: int, barrier):
    import torch.distributed as dist
    H, I, E, k = MOE["hidden"], MOE["inter"], MOE["experts"], MOE["k"]
    T = PREFILL_TOKENS
    if T % world:
        return {"unavailable": f"{T} tokens do not split over {world} ranks"}
    M = T // world
    eb = moe_expert_bytes(H, I)
    n_layers = 2
    eps = build_moe_layers(ctx, torch, dev, n_layers)
    bias = zipf_bias(E)
    gen = torch.Generator(device=dev)
    for li, ep in enumerate(eps):
        gen.manual_seed(_moe_seed(li, 999))
        wr = (torch.randn((E, H), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        ep.layer.set_router(wr.view(torch.int16).cpu().numpy().view(np.uint16), bias)
    gen.manual_seed(9191 + rank)
    xs = [torch.randn((M, H), generator=gen, device=dev).to(torch.bfloat16).view(torch.int16).contiguous()
          for _ in range(n_layers)]
    outs = [torch.empty((M, H), dtype=torch.int16, device=dev) for _ in range(n_layers)]
    for _ in range(args.warmup):
        for li in range(n_layers):
            eps[li].prefill(xs[li], outs[li])
    torch.cuda.synchronize()
    ctx.sync()
    graphs, graph_err = [], None
    try:
        for li in range(n_layers):
            graphs.append(capture_graph(torch, lambda li=li: eps[li].prefill(xs[li], outs[li])))
    except Exception as e:                  # noqa: BLE001 - reported in the JSON line
        graphs, graph_err = [], f"{type(e).__name__}: {e}"[:200]
    ok = torch.tensor([1 if graphs else 0], dtype=torch.int32, device=dev)
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if not int(ok.item()):
        graphs = []

    def step(s):
        li = s % n_layers
        if graphs:
            graphs[li].replay()
        else:
            eps[li].prefill(xs[li], outs[li])
    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(_gpu_index(local_rank))
    clocks.start()
    time.sleep(0.3)
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s in range(args.steps):
        step(s)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = ms
    if world > 1:
        tt = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_max = float(tt.item())
    del graphs
    ctx.sync()
    # this rank's algorithmic work per step: distinct owned experts the 512
    # tokens hit (weights), and the rows it computes (flops)
    lo, hi = eps[0].experts
    per_layer = []
    for li in range(n_layers):
        xg = _gather_tokens(torch, dist, world, xs[li])
        ids = torch.empty((T, k), dtype=torch.int32, device=dev)
        w = torch.empty((T, k), dtype=torch.float32, device=dev)
        eps[li].layer.route(xg, T, k, ids, w)
        torch.cuda.synchronize()
        idn = ids.cpu().numpy()
        mine = (idn >= lo) & (idn < hi)
        rows = int(mine.sum()) + M
        hit = len(np.unique(idn[mine])) + 1
        nbytes = hit * eb + 2 * rows * H + 2 * rows * I + 2 * rows * H
        flops = 2.0 * rows * (2 * I * H + H * I)
        per_layer.append((nbytes, flops, rows, hit))
    avg = [sum(p[i] for p in per_layer) / n_layers for i in range(4)]
    tot = torch.tensor(avg[:2], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tot)
    avg_bytes, avg_flops = float(tot[0]) / world, float(tot[1]) / world
    peak, peak_kind = peaks()
    tflops_peak = _bf16_peak()
    hbm_frac = avg_bytes / (ms_max * 1e-3) / 1e9 / peak
    tc_frac = avg_flops / (ms_max * 1e-3) / 1e12 / tflops_peak

    # end to end: this rank's token rows from pinned host memory, the layer
    # (exchange included), its rows back to the host
    host_x = [x.cpu().numpy().view(np.uint16) for x in xs]
    for li in range(n_layers):
        eps[li].prefill_host(host_x[li])
    barrier()
    e2e_n = max(2, min(args.steps, 10))
    t0 = time.perf_counter()
    for s_ in range(e2e_n):
        eps[s_ % n_layers].prefill_host(host_x[s_ % n_layers])
    e2e_s = _max_over_ranks(torch, dist, dev, world, (time.perf_counter() - t0) / e2e_n)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        th = cpu_threads()
        n_tok, secs = moe_cpu_sample(PREFILL_TOKENS, args.cpu_seconds / 2, bias=bias)
        cpu = {"value": round(n_tok / secs, 2), "unit": "tokens/s", "cores": th["threads"], "kind": "port",
               "sample": f"{n_tok} of the layer's tokens through the oracle per token (biased softmax router, "
                         f"NumpyBackend.moe_experts restated + shared expert), f32 weights cached"}
    exchange = getattr(eps[0], "last_prefill_exchange", None) if world > 1 else None
    # the all-to-all exchange (only routed rows travel; eager: its split sizes
    # are read on the host), timed on the same layers for comparison
    a2a = None
    if world > 1:
        for ep in eps:
            ep.prefill_exchange = "a2a"
        for s_ in range(max(2, args.warmup)):
            eps[s_ % n_layers].prefill(xs[s_ % n_layers], outs[s_ % n_layers])
        torch.cuda.synchronize()
        barrier()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        n_a = max(2, min(args.steps, 10))
        a0.record(stream)
        for s_ in range(n_a):
            eps[s_ % n_layers].prefill(xs[s_ % n_layers], outs[s_ % n_layers])
        a1.record(stream)
        torch.cuda.synchronize()
        a_ms = _max_over_ranks(torch, dist, dev, world, a0.elapsed_time(a1) / n_a)
        a2a = {"value": round(T / (a_ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(a_ms, 4),
               "exchange_rank0": getattr(eps[0], "last_prefill_exchange", None),
               "how": "ExpertParallelMoe(prefill_exchange='a2a'): each rank routes its tokens, the token row of "
                      "every route goes to its expert's owner (all_to_all_single, split sizes read on the host), "
                      "one prefill pass over the received rows, the expert rows back; eager launches"}
        for ep in eps:
            ep.prefill_exchange = "gather"
    for ep in eps:
        ep.layer.close()
    return {
        "metric": "MoE prefill layer tokens/s", "value": round(T / (ms_max * 1e-3), 1), "unit": "tokens/s",
        "exchange_rank0": exchange, "a2a": a2a,
        "ms_per_step": round(ms_max, 4), "scaling": "strong",
        "config": {"workload": "MoE prefill layer (BASELINE configs[3]): 512 tokens, Zipf(1.1) expert load",
                   "parallelism": f"ep{world}", "tokens_per_rank": M, "kernel": prefill_kernel_desc(world),
                   "cuda_graph": bool(int(ok.item())), "graph_error": graph_err,
                   "rank0_rows_per_step": round(avg[2]), "rank0_experts_hit": round(avg[3], 1)},
        "roofline": {"bound": "hbm" if hbm_frac >= tc_frac else "tensor",
                     "achieved": round(avg_bytes / (ms_max * 1e-3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(hbm_frac, 4), "peak_source": peak_kind,
                     "traffic": MEASURED_TRAFFIC["prefill_gemms"] if world == 1 else None,
                     "traffic_source": TRAFFIC_SOURCE["prefill_gemms"],
                     "tensor_tflops": round(avg_flops / (ms_max * 1e-3) / 1e12, 1),
                     "tensor_peak_tflops": tflops_peak, "tensor_frac": round(tc_frac, 4),
                     "per_rank_bytes_per_step": round(avg_bytes), "per_rank_flops_per_step": round(avg_flops)},
        "e2e": {"value": round(T / e2e_s, 1), "unit": "tokens/s", "h2d_bytes_per_step": 2 * M * H,
                "d2h_bytes_per_step": 2 * M * H, "api": "ExpertParallelMoe.prefill_host (synchronous; rc_moe_prefill_host on one GPU)"},
        "gpu_launches": (8 if world == 1 else 9) * args.steps,
        "clocks": clk,
        "cpu_baseline": cpu,
    }


def prefill_kernel_desc(world: int) -> str:
    return ("router, plan, rows gathered into expert order, tcgen05 grouped gate/up + down GEMMs over 64-token "
            "chunks (q4nx codes expanded to bf16 in shared memory, TMEM accumulators), combine"
            + ("; expert-parallel: NCCL all-gather of the token rows, the rank's experts over all tokens, "
               "reduce-scatter of the slot rows (one CUDA graph per layer)" if world > 1 else ""))


# ------------------------------------------------------ full decode step --
# 48 layers, each a q4nx projection pair 2048->4096 ->
# 2048 and the config-3 MoE block (residual add + RMS normalisation after the
# MoE: a SwiGLU block is quadratic in its input, so an unnormalised residual
# stream of random layers overflows within ~20 layers), then the
# 2048->151936 lm-head and top-k 50 / top-p 0.9 sampling on the GPU; one token
# per rank per step; projections replicated, experts sharded over the ranks.
DECODE_LAYERS = 48
LM_HEAD = (151936, 2048)


def build_decode_model(ctx, torch, dev):
    """Seeded random-init model: projections N(0, 1/K) (the variance of the
    hidden stream stays put over 48 layers), experts and router N(0, 0.02)."""
    import math
    from raon_npu_b200.device import MoeLayer
    from raon_npu_b200.expert_parallel import ExpertParallelMoe
    H, I, E, k = MOE["hidden"], MOE["inter"], MOE["experts"], MOE["k"]
    gen = torch.Generator(device=dev)

    def q4(n, kk, seed, std):
        gen.manual_seed(seed)
        w = torch.randn((n, kk), generator=gen, device=dev) * std
        packed = torch.empty(n * kk * 5 // 8, dtype=torch.uint8, device=dev)
        ctx.quantize_q4nx(w, packed, n, kk)
        del w
        return packed

    layers = []
    for li in range(DECODE_LAYERS):
        projs = []
        for j, (n, kk) in enumerate([(4096, H), (H, 4096)]):
            packed = q4(n, kk, 8_000_000 + 10 * li + j, 1.0 / math.sqrt(kk))
            projs.append(ctx.upload_q4nx(packed, n, kk))
        layer = MoeLayer(ctx, H, I, E, has_shared=True)
        ep = ExpertParallelMoe(layer, k, act="swiglu", router="softmax")
        for e in range(E + 1):
            if ep.owns(e):
                layer.set_expert(e, q4(2 * I, H, _moe_seed(100 + li, e), 0.02), q4(H, I, _moe_seed(100 + li, e) + 500,
                                                                                  0.02))
        gen.manual_seed(_moe_seed(100 + li, 999))
        wr = (torch.randn((E, H), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
        layer.set_router(wr.view(torch.int16).cpu().numpy().view(np.uint16))
        layers.append((projs, ep))
    lm = ctx.upload_q4nx(q4(LM_HEAD[0], LM_HEAD[1], 8_999_999, 0.02), LM_HEAD[0], LM_HEAD[1])
    torch.cuda.synchronize()
    return layers, lm


def run_decode_step(args, ctx, torch, dev, rank: int, world: int, local_rank: int, barrier):
    import torch.distributed as dist
    from raon_npu_b200.device import add_rms_bf16, sample_tokens
    H = MOE["hidden"]
    layers, lm = build_decode_model(ctx, torch, dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5151 + rank)
    x0 = torch.randn((1, H), generator=gen, device=dev).to(torch.bfloat16).view(torch.int16).contiguous()
    h1 = torch.empty((1, 4096), dtype=torch.int16, device=dev)
    h = torch.empty((1, H), dtype=torch.int16, device=dev)
    mo = torch.empty((1, H), dtype=torch.int16, device=dev)
    xs = [torch.empty((1, H), dtype=torch.int16, device=dev) for _ in range(2)]
    logits = torch.empty((1, LM_HEAD[0]), dtype=torch.int16, device=dev)
    u = torch.tensor([np.random.default_rng(77 + rank).random()], dtype=torch.float64, device=dev)
    tok = torch.empty(1, dtype=torch.int32, device=dev)
    trace = []

    def step(record=False):
        cur = x0
        for li, ((wa, wb), ep) in enumerate(layers):
            wa.gemv_into(cur, h1, 1)
            wb.gemv_into(h1, h, 1)
            if record:
                trace.append(h.clone())
            ep.decode(h, mo)
            nxt = xs[li & 1]
            add_rms_bf16(ctx, h, mo, nxt)
            cur = nxt
        lm.gemv_into(cur, logits, 1)
        sample_tokens(ctx, logits, u, tok, top_k=50, top_p=0.9, temperature=1.0)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.sync()
    graph, graph_err = None, None
    try:
        graph = capture_graph(torch, step)
    except Exception as e:                  # noqa: BLE001 - reported in the JSON line
        graph, graph_err = None, f"{type(e).__name__}: {e}"[:200]
    ok = torch.tensor([1 if graph is not None else 0], dtype=torch.int32, device=dev)
    if world > 1:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    if not int(ok.item()):
        graph = None
    run = graph.replay if graph is not None else step
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(_gpu_index(local_rank))
    clocks.start()
    time.sleep(0.3)
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    steps = max(3, args.steps // 4)
    e0.record(stream)
    for _ in range(steps):
        run()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = e0.elapsed_time(e1) / steps
    ms_max = ms
    if world > 1:
        tt = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms_max = float(tt.item())
    ctx.sync()

    # end to end: host hidden row -> device, the step, the sampled id -> host
    host_x = x0.cpu().numpy()
    pin = torch.from_numpy(host_x.copy()).pin_memory()
    tok_host = torch.empty(1, dtype=torch.int32).pin_memory()
    barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        x0.copy_(pin, non_blocking=True)
        run()
        tok_host.copy_(tok, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
    e2e_s = (time.perf_counter() - t0) / steps
    if world > 1:
        tt = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_s = float(tt.item())
    del graph

    # algorithmic bytes of one step on this rank: projections, the distinct
    # owned experts the layer's gathered tokens chose, shared, router, lm-head
    step(record=True)
    torch.cuda.synchronize()
    E, k, eb = MOE["experts"], MOE["k"], moe_expert_bytes(H, MOE["inter"])
    lo, hi = layers[0][1].experts
    nbytes = LM_HEAD[0] * LM_HEAD[1] * 5 // 8
    for li, ((wa, wb), ep) in enumerate(layers):
        hg = _gather_tokens(torch, dist, world, trace[li])
        ids = torch.empty((hg.shape[0], k), dtype=torch.int32, device=dev)
        w = torch.empty((hg.shape[0], k), dtype=torch.float32, device=dev)
        ep.layer.route(hg, hg.shape[0], k, ids, w)
        torch.cuda.synchronize()
        idn = ids.cpu().numpy().ravel()
        active = len({int(e) for e in idn if lo <= int(e) < hi})
        nbytes += 2 * 4096 * H * 5 // 8 + (active + 1) * eb + E * H * 2
    rb = torch.tensor([float(nbytes)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(rb)
    avg_bytes = float(rb.item()) / world
    peak, peak_kind = peaks()
    achieved = avg_bytes / (ms_max * 1e-3) / 1e9
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = decode_step_cpu_sample(ctx, torch, dev, layers, lm, args.cpu_seconds)
    for (wa, wb), ep in layers:
        wa.free()
        wb.free()
        ep.layer.close()
    lm.free()
    # DRAM traffic of the step, scaled from single-kernel captures: the GEMV
    # launches move 0.995x their algorithmic bytes (sweep launch list) and one
    # T = 1 MoE layer moves MEASURED_TRAFFIC["moe_layer_t1"] (one GPU only)
    traffic = None
    if world == 1:
        gemv_ratio = MEASURED_TRAFFIC["gemv_step"] / step_bytes()
        traffic = round(DECODE_LAYERS * (2 * 4096 * H * 5 // 8 * gemv_ratio + MEASURED_TRAFFIC["moe_layer_t1"])
                        + LM_HEAD[0] * LM_HEAD[1] * 5 // 8 * gemv_ratio)
    return {
        "metric": "decode step tokens/s (48 layers + lm-head + sampling)", "value": round(world / (ms_max * 1e-3), 2),
        "unit": "tokens/s", "ms_per_step": round(ms_max, 4), "steps": steps, "scaling": "weak",
        "config": {"workload": "synthetic full decode step (BASELINE configs[4]): 48 x (q4nx 2048->4096->2048 + "
                               "config-3 MoE + residual/RMS), lm-head 2048->151936, top-k 50 / top-p 0.9",
                   "tokens_per_rank": 1, "parallelism": f"projections replicated, experts ep{world}",
                   "cuda_graph": graph_err is None and bool(int(ok.item())), "graph_error": graph_err},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind, "traffic": traffic,
                     "traffic_source": "scaled from the GEMV sweep and MoE layer captures (see those sources)",
                     "per_rank_bytes_per_step": round(avg_bytes)},
        "e2e": {"value": round(world / e2e_s, 2), "unit": "tokens/s", "h2d_bytes_per_step": 2 * H,
                "d2h_bytes_per_step": 4, "api": "graph replay with the hidden row copied in and the id copied out"},
        "gpu_launches": (DECODE_LAYERS * 7 + 2) * steps,
        "clocks": clk,
        "cpu_baseline": cpu,
    }


def decode_step_cpu_sample(ctx, torch, dev, layers, lm, budget_s: float):
    """The reference's CPU arithmetic for the step, timed on one layer (its
    two projections and the MoE block for one token) and on the lm-head plus
    sampler, extrapolated to 48 layers; f32 weights cached (dequantised on the
    GPU, bit-identical to the reference's dequantiser)."""
    from oracle import backend as ob
    from oracle.sampling import sample_token_u
    th = cpu_threads()

    def f32(w):
        out = torch.empty((w.n, w.k), dtype=torch.float32, device=dev)
        w.dequant_into(out)
        torch.cuda.synchronize()
        return out.cpu().numpy()
    (wa, wb), ep = layers[0]
    fa, fb = f32(wa), f32(wb)
    flm = f32(lm)
    moe_tokens, moe_secs = moe_cpu_sample(16, budget_s / 2)
    rng = np.random.default_rng(3)
    x = ob.f32_to_bf16(rng.standard_normal(MOE["hidden"]).astype(np.float32))
    t0 = time.perf_counter()
    for _ in range(3):
        ob.linear(fb, ob.linear(fa, x))
    proj_s = (time.perf_counter() - t0) / 3
    t0 = time.perf_counter()
    lg = ob.linear(flm, x)
    sample_token_u(ob.bf16_to_f32(lg), [], 50, 0.9, 1.0, 0.0, 0.5)
    head_s = time.perf_counter() - t0
    per_token = DECODE_LAYERS * (proj_s + moe_secs / moe_tokens) + head_s
    return {"value": round(1.0 / per_token, 3), "unit": "tokens/s", "cores": th["threads"], "kind": "port",
            "sample": f"one layer (2 projections x3, MoE layer x{moe_tokens}) and the lm-head + sampler once, "
                      f"numpy f32 with cached weights, extrapolated to {DECODE_LAYERS} layers"}


def _bf16_peak() -> float:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"])
    return 1590.0


def _gpu_index(local_rank: int) -> int:
    if "CUDA_VISIBLE_DEVICES" in os.environ:
        return int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local_rank])
    return local_rank


# ----------------------------------------------------------- CPU legs --
def cpu_gemv_sweep_sample(weights_f32: dict, xs_u16: dict, budget_s: float):
    """Time the oracle's f32 GEMV over the sweep (f32-dequantised weights
    cached, the reference's steady state) within a time budget."""
    from oracle import backend as ob
    done_bytes, t_total, passes = 0, 0.0, 0
    keys = [(n, k, t) for t in TOKENS for n, k in SHAPES if (n, k) in weights_f32]
    while t_total < budget_s or passes == 0:
        for n, k, t in keys:
            x = xs_u16[(n, k, t)]
            t0 = time.perf_counter()
            ob.linear(weights_f32[(n, k)], x)
            t_total += time.perf_counter() - t0
            done_bytes += algo_bytes(n, k, t)
        passes += 1
        if passes >= 50:
            break
    return done_bytes, t_total, passes, keys


def cpu_baseline(ctx, torch, dev, weights, host_x, budget_s: float):
    th = cpu_threads()
    w32 = {}
    for (n, k), cps in weights.items():
        out = torch.empty((n, k), dtype=torch.float32, device=dev)
        cps[0].dequant_into(out)
        torch.cuda.synchronize()
        w32[(n, k)] = out.cpu().numpy()
        del out
    done, secs, passes, keys = cpu_gemv_sweep_sample(w32, host_x, budget_s)
    return {"value": round(done / secs / 1e9, 3), "unit": "GB/s", "cores": th["threads"], "kind": "port",
            "sample": f"{passes} pass(es) of the full sweep ({len(keys)} GEMVs) through the oracle's numpy f32 "
                      f"GEMV (host/backend.py:402-417 restated), f32 weights cached"}


def cpu_config1(ctx, torch, dev, w, x_u16, budget_s: float) -> dict:
    """Config 1 through the oracle's f32 GEMV with the dequantised weights cached
    (the reference's steady state); GB/s of the same algorithmic bytes."""
    from oracle import backend as ob
    th = cpu_threads()
    out = torch.empty((w.n, w.k), dtype=torch.float32, device=dev)
    w.dequant_into(out)
    torch.cuda.synchronize()
    w32 = out.cpu().numpy()
    del out
    ob.linear(w32, x_u16)
    n, secs = 0, 0.0
    while secs < budget_s and n < 2000:
        t0 = time.perf_counter()
        ob.linear(w32, x_u16)
        secs += time.perf_counter() - t0
        n += 1
    return {"value": round(n * algo_bytes(w.n, w.k, 1) / secs / 1e9, 3), "unit": "GB/s",
            "us_per_call": round(secs / n * 1e6, 1), "cores": th["threads"], "kind": "port",
            "sample": f"{n} calls of the oracle's NumpyBackend.linear restatement, f32 weights cached"}


def run_reference(args, rank: int):
    """Reference arm: the reference's CPU implementation of the path (the
    oracle port of NumpyBackend and the router), on the host cores with every
    BLAS thread, rank 0 only.  ``value``: the config-3 MoE decode layer,
    tokens/s (our arm's headline metric and config); the GEMV sweep follows."""
    if rank != 0:
        return
    from oracle import q4nx as q
    th = cpu_threads()
    # MoE decode layer: warm-up tokens (they also build the cached weights),
    # then one token per step, as our arm's one token per rank per step
    moe_cpu_sample(max(1, args.warmup), 0.0)
    n_tok, secs = moe_cpu_sample(args.steps, float("inf"))
    v = n_tok / secs
    # GEMV sweep on a bounded sample
    rng = np.random.default_rng(0)
    w32, xs = {}, {}
    for si, (n, k) in enumerate(SHAPES):
        packed, codes, scales, mins = q.normal_weight_q4nx(n, k, seed=1000 + si)
        w32[(n, k)] = q.dequantize_simple(codes, scales, mins)
        del packed, codes
    for t in TOKENS:
        for n, k in SHAPES:
            xs[(n, k, t)] = q.f32_to_bf16(rng.standard_normal((t, k)).astype(np.float32))
    cpu_gemv_sweep_sample(w32, xs, 0.0)
    done, gsecs, passes, _ = cpu_gemv_sweep_sample(w32, xs, min(args.cpu_seconds, 10.0))
    gv = done / gsecs / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "tokens/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(secs / n_tok * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (dequantised weights)",
            "data": "synthetic: q4nx weights from N(0,0.02) f32 (numpy default_rng, seeded), bf16 x N(0,1)",
            "config": {"workload": "MoE decode layer (BASELINE configs[2]): hidden 2048, 128 experts + 1 shared, "
                                   "I=768, softmax top-8, SwiGLU, q4nx", "tokens_per_step": 1,
                       "parallelism": "host CPU (the reference has no multi-device path)"},
            "cpu_baseline": {"value": round(v, 3), "unit": "tokens/s", "cores": th["threads"], "kind": "port",
                             "blas_threads": th["pools"],
                             "sample": f"{n_tok} decode tokens, one per step, through the oracle's numpy MoE "
                                       f"layer (NumpyBackend.moe_experts + router + shared expert restated), "
                                       f"f32 weights cached (16 weight sets, id mod 16)"},
            "e2e": {"value": round(v, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "gemv_sweep": {"value": round(gv, 3), "unit": "GB/s", "passes": passes,
                           "sample": "the configs[1] sweep through the oracle's NumpyBackend.linear restatement, "
                                     "f32 weights cached"}}
    print(json.dumps(line), flush=True)


def run_profile_case(args):
    """A few plain launches of one GEMV shape (no timing) for an ncu capture:
    ``python bench.py --profile 4096x2048 --tokens 1 --launches 4`` (q4nx) or
    ``--profile bfp16:151936x2048`` (bfp16ebs8)."""
    import torch
    from raon_npu_b200.device import Context
    bfp16 = args.profile.startswith("bfp16:")
    n, k = (int(v) for v in args.profile.split(":")[-1].split("x"))
    dev = torch.device("cuda", 0)
    ctx = Context(0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1)
    if bfp16:   # ``--profile bfp16:NxK``: synthetic bfp16ebs8 blocks as in measure_bfp16
        nbytes = n * k * 9 // 8
        packed = torch.randint(0, 256, (nbytes // 144, 144), generator=gen, device=dev, dtype=torch.uint8)
        packed[:, :16] = torch.randint(118, 125, (nbytes // 144, 16), generator=gen, device=dev, dtype=torch.uint8)
        copies = max(1, min(64, (256 << 20) // nbytes))
        ws = [ctx.upload_bfp16(packed.view(-1), n, k) for _ in range(copies)]
    else:
        w = torch.randn((n, k), generator=gen, device=dev) * 0.02
        packed = torch.empty(n * k * 5 // 8, dtype=torch.uint8, device=dev)
        ctx.quantize_q4nx(w, packed, n, k)
        copies = max(1, min(64, (256 << 20) // (n * k * 5 // 8)))
        ws = [ctx.upload_q4nx(packed, n, k) for _ in range(copies)]
    x = torch.randn((args.tokens, k), generator=gen, device=dev).to(torch.bfloat16).view(torch.int16)
    y = torch.empty((args.tokens, n), dtype=torch.int16, device=dev)
    for i in range(args.launches):
        ws[i % copies].gemv_into(x, y, args.tokens)
    torch.cuda.synchronize()
    ctx.sync()
    print(json.dumps({"profile": args.profile, "tokens": args.tokens, "launches": args.launches, "copies": copies}))


def run_profile_moe(args):
    """A few plain config-3 MoE decode steps on one GPU (no timing) for an ncu
    capture: ``python bench.py --profile moe --launches 6``."""
    import torch
    from raon_npu_b200.device import Context
    dev = torch.device("cuda", 0)
    ctx = Context(0)
    eps = build_moe_layers(ctx, torch, dev, 2)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4242)
    xs = [torch.randn((args.tokens, MOE["hidden"]), generator=gen, device=dev).to(torch.bfloat16)
          .view(torch.int16).contiguous() for _ in range(2)]
    out = torch.empty((args.tokens, MOE["hidden"]), dtype=torch.int16, device=dev)
    for i in range(args.launches):
        eps[i % 2].decode(xs[i % 2], out)
    torch.cuda.synchronize()
    ctx.sync()
    for ep in eps:
        ep.layer.close()
    ctx.close()
    print(json.dumps({"profile": "moe", "tokens": args.tokens, "steps": args.launches}))


def run_profile_prefill(args):
    """A few plain config-4 prefill layers on one GPU (no timing) for an ncu
    capture: ``python bench.py --profile prefill --launches 3``."""
    import torch
    from raon_npu_b200.device import Context
    dev = torch.device("cuda", 0)
    ctx = Context(0)
    eps = build_moe_layers(ctx, torch, dev, 1)
    E, H = MOE["experts"], MOE["hidden"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(_moe_seed(0, 999))
    wr = (torch.randn((E, H), generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    eps[0].layer.set_router(wr.view(torch.int16).cpu().numpy().view(np.uint16), zipf_bias(E))
    gen.manual_seed(9191)
    x = torch.randn((PREFILL_TOKENS, H), generator=gen, device=dev).to(torch.bfloat16).view(torch.int16).contiguous()
    out = torch.empty_like(x)
    for _ in range(args.launches):
        eps[0].prefill(x, out)
    torch.cuda.synchronize()
    ctx.sync()
    eps[0].layer.close()
    ctx.close()
    print(json.dumps({"profile": "prefill", "tokens": PREFILL_TOKENS, "steps": args.launches}))


def run_profile_moe_bfp16(args):
    """One config-3 layer with bfp16ebs8 down matrices on one GPU (no timing)
    for an ncu capture: ``--launches`` decode calls of ``--tokens`` tokens,
    then ``--launches`` 512-token prefills."""
    import torch
    from raon_npu_b200.device import Context
    dev = torch.device("cuda", 0)
    ctx = Context(0)
    layer = build_bfp16_down_layers(ctx, torch, dev, 1)[0]
    H, k = MOE["hidden"], MOE["k"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(4343)
    x = torch.randn((args.tokens, H), generator=gen, device=dev).to(torch.bfloat16).view(torch.int16).contiguous()
    out = torch.empty_like(x)
    xp = torch.randn((PREFILL_TOKENS, H), generator=gen, device=dev).to(torch.bfloat16).view(torch.int16)
    op = torch.empty_like(xp)
    for _ in range(args.launches):
        layer.decode(x, k, out)
    for _ in range(args.launches):
        layer.prefill(xp, k, op)
    torch.cuda.synchronize()
    ctx.sync()
    layer.close()
    ctx.close()
    print(json.dumps({"profile": "moe_bfp16", "tokens": args.tokens, "prefill_tokens": PREFILL_TOKENS,
                      "steps": args.launches}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemv", action="store_true", help="skip the GEMV sweep and config 1 (configs[0], [1])")
    ap.add_argument("--no-prefill", action="store_true", help="skip the MoE prefill layer (configs[3])")
    ap.add_argument("--no-decode-step", action="store_true", help="skip the 48-layer decode step (configs[4])")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the per-shape launch table, the bfp16ebs8 GEMV and the bfp16-down MoE layer")
    ap.add_argument("--profile", default=None, help="NxK: run a few plain GEMV launches for ncu and exit; "
                    "'moe' / 'prefill': a few config-3 decode / config-4 prefill steps; 'moe_bfp16': decode "
                    "and prefill calls of a layer with bfp16ebs8 down matrices; 'bfp16:NxK': bfp16 GEMVs")
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--launches", type=int, default=4)
    args = ap.parse_args()
    if args.profile == "moe":
        run_profile_moe(args)
        return
    if args.profile == "prefill":
        run_profile_prefill(args)
        return
    if args.profile == "moe_bfp16":
        run_profile_moe_bfp16(args)
        return
    if args.profile:
        run_profile_case(args)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
