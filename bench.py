#!/usr/bin/env python3
"""bench.py -- the headline exact i8 GEMM at 8192^3 on 1..8 B200s.

Workload (the i8 headline): C = A B with A, B int8
8192 x 8192 drawn from the reference's recorded generator (salts 1 and 2),
C exact int32, through slice::gemm::<i8, i32>'s C-ABI twin uor_b200_gemm_i8_i32.
With N GPUs the output is sharded by column blocks (the reference's Partition
of C into independent tiles, partition.rs:34): rank r owns an 8192-column block
of an 8192 x 8192 x (8192 N) product and its own B block; A is replicated. No
collective runs on the data path, so the scaling is weak.

Metric: exact-i8 TOPS = 2 m k n / t, whole job (all ranks' units / max rank time).
L2: three rotating operand sets (3 x 128 MiB > the 126 MB L2) plus a 256 MiB
output written every step, so no step reads operands a previous step left in L2.

--impl reference times the reference's CPU path on the host cores instead (the
Rust crate cannot be built here, so its C restatement in oracle/ stands in).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "uor-matmul_b200"))
sys.path.insert(0, ROOT)

SIZE = 8192
METRIC = "exact i8 GEMM TOPS at 8192^3 (bit-exact, int32 out)"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--size", type=int, default=SIZE)
    p.add_argument("--e2e-steps", type=int, default=3)
    p.add_argument("--no-cpu-baseline", action="store_true")
    return p.parse_args()


def env_rank():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


class Clocks:
    """SM clock and throttle reasons sampled through NVML during the timed region."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = None
        self._thread = None

    def start(self):
        import threading
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:
            return
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    self.samples.append(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
                    r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    for name, bit in self.REASONS.items():
                        if r & bit:
                            self.reasons.add(name)
                except Exception:
                    pass
                time.sleep(0.002)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        time.sleep(0.01)

    def stop(self):
        if not self._thread:
            return None
        self._stop.set()
        self._thread.join()
        if not self.samples:
            return None
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples),
                "source": "NVML, every 2 ms during the timed region"}


def cpu_baseline(size, budget_s=12.0):
    """The reference's CPU path (C restatement, all host threads) on a row sample."""
    import numpy as np
    import uor_b200 as U
    from oracle import oracle as orc

    k = n = size
    b = U.corpus(2, U.CORPUS_I8, k * n)
    threads = orc.max_threads()
    rows = 8
    while True:
        a = U.corpus(1, U.CORPUS_I8, rows * k)
        c = np.zeros(rows * n, np.int32)
        t0 = time.perf_counter()
        orc.gemm_i8_blocked(a, b, c, rows, k, n, threads=threads)
        dt = time.perf_counter() - t0
        if dt * 4 > budget_s or rows >= size:
            break
        rows = min(size, max(rows * 2, int(rows * budget_s / max(dt, 1e-3) / 2)))
    tops = 2.0 * rows * k * n / dt / 1e12
    return {"value": tops, "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{rows} of {size} rows of the {size}^3 product ({dt:.2f} s), "
                      "blocked C restatement of gemm_auto's s8 path, OpenMP over rows"}


def reference_arm(args, rank):
    if rank != 0:
        return
    steps = []
    base = None
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(args.size, budget_s=4.0 if i < args.warmup else 8.0)
        if i >= args.warmup:
            steps.append(r["value"])
        base = r
    v = statistics.median(steps)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "TOPS",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (reference xorshift corpus, salts 1/2)",
            "config": {"workload": f"i8 x i8 -> i32 GEMM {args.size}^3 (configs[4] headline)",
                       "m": args.size, "k": args.size, "n": args.size},
            "cpu_baseline": dict(base, value=v),
            "e2e": {"value": v, "unit": "TOPS", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def load_traffic():
    path = os.path.join(ROOT, "profiles", "k1_i8_8192_traffic.json")
    try:
        return json.load(open(path))
    except Exception:
        return None


def run_e2e(args, U, torch, dist, ctx, stream, m, k, n, rank, world):
    """The same product through the public call with pinned HOST buffers: every
    step copies A and B in and C out inside the timed region."""
    ops_per_step = 2.0 * m * k * n
    Ah = torch.from_numpy(U.corpus(1, U.CORPUS_I8, m * k)).pin_memory()
    Bh = torch.from_numpy(U.corpus(2 + 1000 * rank, U.CORPUS_I8, k * n)).pin_memory()
    Ch = torch.empty(m * n, dtype=torch.int32).pin_memory()
    U.gemm_i8_i32(m, k, n, Ah, Bh, Ch, ctx=ctx)  # warm the staging buffers
    if dist:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.e2e_steps):
        U.gemm_i8_i32(m, k, n, Ah, Bh, Ch, ctx=ctx)
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([e2e_ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    return {"value": world * args.e2e_steps * ops_per_step / (e2e_ms / 1e3) / 1e12,
            "unit": "TOPS", "h2d_bytes_per_step": m * k + k * n, "d2h_bytes_per_step": 4 * m * n,
            "ms_per_step": e2e_ms / args.e2e_steps}


def main():
    args = parse()
    rank, world, local = env_rank()
    if args.impl == "reference":
        reference_arm(args, rank)
        return

    import numpy as np
    import torch
    import uor_b200 as U

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=180))
    m = k = n = args.size
    sets = 3
    A = [torch.from_numpy(U.corpus(1 + 100 * s, U.CORPUS_I8, m * k)).cuda() for s in range(sets)]
    B = [torch.from_numpy(U.corpus(2 + 100 * s + 1000 * rank, U.CORPUS_I8, k * n)).cuda()
         for s in range(sets)]
    C = torch.empty(m * n, dtype=torch.int32, device="cuda")
    ctx = U.Context(local)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)
    route = U.Route()

    def step(i):
        U.gemm_i8_i32(m, k, n, A[i % sets], B[i % sets], C, ctx=ctx, route=route,
                      asynchronous=True)

    for i in range(args.warmup):
        step(i)
    assert ctx.sync() == U.OK
    # correctness gate on the last warm-up output: Freivalds check in f64 (exact here)
    x = torch.randint(-1, 2, (n,), device="cuda", dtype=torch.float64)
    s = (args.warmup - 1) % sets
    lhs = C.view(m, n).double() @ x
    rhs = A[s].view(m, k).double() @ (B[s].view(k, n).double() @ x)
    assert torch.equal(lhs, rhs), "checksum mismatch"

    clocks = Clocks(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        ev[i][0].record(stream)
        step(args.warmup + i)
        ev[i][1].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = clocks.stop()
    assert ctx.sync() == U.OK
    elapsed_ms = t_start.elapsed_time(t_end)
    kernel_ms = [a.elapsed_time(b) for a, b in ev]
    if dist:
        t = torch.tensor([elapsed_ms], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ops_per_step = 2.0 * m * k * n
    value = world * args.steps * ops_per_step / (elapsed_ms / 1e3) / 1e12
    ms_per_step = elapsed_ms / args.steps

    # ---- end to end through the C ABI with pinned host buffers
    e2e = None
    if args.e2e_steps > 0:
        e2e = run_e2e(args, U, torch, dist, ctx, stream, m, k, n, rank, world)
    del A, B, C

    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except Exception:
        pass
    if "bf16_tflops" in peaks:
        peak = 2.0 * peaks["bf16_tflops"]
        peak_src = "2x measured bf16 burst (int8 dense issues at twice bf16 on B200), of measured"
    else:
        peak = 2.0 * 1590.0
        peak_src = "2x fallback bf16 1.59 PFLOP/s, of fallback"
    avg_kernel_ms = statistics.mean(kernel_ms)
    achieved = ops_per_step / (avg_kernel_ms / 1e3) / 1e12
    traffic = load_traffic()

    line = {
        "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
        "data": "synthetic (reference xorshift corpus)",
        "config": {"workload": f"i8 x i8 -> i32 GEMM {m}x{k}x{n} per GPU (configs[4] headline), "
                               "column-block sharded",
                   "m": m, "k": k, "n_per_gpu": n, "n_total": n * world,
                   "l2": "3 rotating operand sets (384 MiB) + 256 MiB output per step",
                   "parallelism": f"column blocks x{world}, no data-path collective"},
        "route": route.as_dict(),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOPS",
                     "frac": achieved / peak, "peak_source": peak_src,
                     "traffic": traffic.get("bytes_per_launch") if traffic else None,
                     "algorithmic_bytes": m * k + k * n + 4 * m * n},
        "e2e": e2e,
        "gpu_launches": args.steps,
        "clocks": clk,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.size)
    ctx.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
