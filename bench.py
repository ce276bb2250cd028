"""Benchmark of the q4nx decode GEMV on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = one pass of the GEMV decode sweep: token rows T in {1,2,4,8,16} over
the shapes (K -> N) 2048->4096, 4096->2048, 2048->512 and the lm-head
2048->151936, q4nx weights from N(0, 0.02) f32, activations bf16 N(0, 1)
(synthetic, seeded).  The dense GEMV does not shard: at N GPUs every rank runs
an independent replica (one process per GPU, torchrun), and ``value`` is the
algorithmic bytes of all ranks over the slowest rank's time ("weak" scaling).

Metric: q4nx GEMV HBM GB/s = algorithmic bytes (N*K*5/8 packed weights +
2*T*K + 2*T*N activation/output bytes per GEMV) / device time.  Each GEMV of a
step reads a different copy of its matrix and a step streams ~1 GB, far more
than the 126 MB L2, so no timed GEMV is served from L2.

``--impl reference`` times the reference's own CPU arithmetic for this path
(the numpy restatement in ``oracle/``: f32-dequantised weights, f32 dot,
bf16 RTNE -- ``host/backend.py:402-417``) on the host cores, rank 0 only.
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
    import torch
    import torch.distributed as dist
    from raon_npu_b200.device import Context

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    ctx = Context(local_rank)
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

    def barrier():
        if world > 1:
            dist.barrier()

    # Eager warm-up (sizes the scratch), then capture one step in a CUDA graph:
    # a decode step is a fixed launch sequence, replayed without host overhead.
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ctx.sync()
    step_graph = capture_graph(torch, step)
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step_graph.replay()
    torch.cuda.synchronize()
    ctx.sync()
    barrier()
    step = step_graph.replay

    clocks = ClockSampler(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local_rank)).split(",")[local_rank])
                          if "CUDA_VISIBLE_DEVICES" in os.environ else local_rank)
    clocks.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
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
    ctx.sync()

    sb = step_bytes()
    value = world * sb / (ms_max * 1e-3) / 1e9
    peak, peak_kind = peaks()
    achieved = sb / (ms * 1e-3) / 1e9

    # Per-shape launch times (rank 0): back-to-back launches over rotating
    # copies whose total exceeds L2, so each launch streams from HBM.
    per_shape = []
    if rank == 0 and not args.no_per_shape:
        per_shape = measure_per_shape(ctx, torch, dev, gen, stream, weights)

    # End to end through the host-buffer C-ABI entry point (rc_gemv_host):
    # pinned host x -> device, GEMV, y -> host, every GEMV of the step.
    host_x = {key: x.cpu().numpy().view(np.uint16) for key, x in xs.items()}
    e2e_steps = max(2, min(args.steps, 5))
    for _ in range(1):
        for ti, t in enumerate(TOKENS):
            for n, k in SHAPES:
                weights[(n, k)][ti % len(weights[(n, k)])].gemv_host(host_x[(n, k, t)])
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        for ti, t in enumerate(TOKENS):
            for n, k in SHAPES:
                weights[(n, k)][ti % len(weights[(n, k)])].gemv_host(host_x[(n, k, t)])
    e2e_s = (time.perf_counter() - t0) / e2e_steps
    if world > 1:
        tt = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_s = float(tt.item())
    h2d = sum(2 * t * k for t in TOKENS for n, k in SHAPES)
    d2h = sum(2 * t * n for t in TOKENS for n, k in SHAPES)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(ctx, torch, dev, weights, host_x, budget_s=args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u4 codes, bf16 act, f32 acc",
            "data": "synthetic: q4nx weights from N(0,0.02) f32 (torch cuda generator, seeded), bf16 x N(0,1)",
            "config": {"workload": "q4nx GEMV decode sweep (BASELINE configs[1])",
                       "shapes_k_to_n": [f"{k}->{n}" for n, k in SHAPES], "tokens": TOKENS,
                       "parallelism": f"replicas x{world} (dense GEMV does not shard)",
                       "l2": "inputs larger than L2: each step streams %.2f GB of distinct weights" % (sb / 1e9),
                       "algorithmic_bytes_per_step": sb},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                         "traffic": None, "kernel": "q4nx_gemv (x-prep + stream-K GEMV pairs, event-timed step)"},
            "e2e": {"value": round(world * sb / e2e_s / 1e9, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "api": "rc_gemv_host (synchronous per GEMV)"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk,
            "per_shape": per_shape,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    for ws in weights.values():
        for w in ws:
            w.free()
    ctx.close()


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
    w32 = {}
    for (n, k), cps in weights.items():
        out = torch.empty((n, k), dtype=torch.float32, device=dev)
        cps[0].dequant_into(out)
        torch.cuda.synchronize()
        w32[(n, k)] = out.cpu().numpy()
        del out
    done, secs, passes, keys = cpu_gemv_sweep_sample(w32, host_x, budget_s)
    return {"value": round(done / secs / 1e9, 3), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{passes} pass(es) of the full sweep ({len(keys)} GEMVs) through the oracle's numpy f32 "
                      f"GEMV (host/backend.py:402-417 restated), f32 weights cached; "
                      f"OPENBLAS_NUM_THREADS={os.environ.get('OPENBLAS_NUM_THREADS', 'unset')}"}


def run_reference(args, rank: int):
    """Reference arm: the reference's CPU implementation of the path (oracle port)."""
    if rank != 0:
        return
    from oracle import q4nx as q
    rng = np.random.default_rng(0)
    w32, xs = {}, {}
    for si, (n, k) in enumerate(SHAPES):
        packed, codes, scales, mins = q.normal_weight_q4nx(n, k, seed=1000 + si)
        w32[(n, k)] = q.dequantize_simple(codes, scales, mins)
        del packed, codes
    for t in TOKENS:
        for n, k in SHAPES:
            xs[(n, k, t)] = q.f32_to_bf16(rng.standard_normal((t, k)).astype(np.float32))
    for _ in range(args.warmup):
        cpu_gemv_sweep_sample(w32, xs, 0.0)
    t0 = time.perf_counter()
    done = 0
    for _ in range(args.steps):
        d, _, _, _ = cpu_gemv_sweep_sample(w32, xs, 0.0)
        done += d
    secs = time.perf_counter() - t0
    v = done / secs / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(secs / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (dequantised weights)",
            "data": "synthetic: q4nx weights from N(0,0.02) f32 (numpy default_rng, seeded), bf16 x N(0,1)",
            "config": {"workload": "q4nx GEMV decode sweep (BASELINE configs[1])",
                       "shapes_k_to_n": [f"{k}->{n}" for n, k in SHAPES], "tokens": TOKENS},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                             "sample": "one full sweep per step through the numpy restatement of "
                                       "NumpyBackend.linear (host/backend.py:402-417), f32 weights cached"},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_profile_case(args):
    """A few plain launches of one GEMV shape (no timing) for an ncu capture:
    ``python bench.py --profile 4096x2048 --tokens 1 --launches 4``."""
    import torch
    from raon_npu_b200.device import Context
    n, k = (int(v) for v in args.profile.split("x"))
    dev = torch.device("cuda", 0)
    ctx = Context(0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1)
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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-shape", action="store_true", help="skip the per-shape launch table")
    ap.add_argument("--profile", default=None, help="NxK: run a few plain GEMV launches for ncu and exit")
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--launches", type=int, default=4)
    args = ap.parse_args()
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
