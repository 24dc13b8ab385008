#!/usr/bin/env python3
"""bench.py -- exact GEMM throughput on 1..8 B200s.

Default workload (the i8 headline): C = A B with A, B
int8 8192 x 8192 drawn from the reference's recorded generator (salts 1 and 2),
C exact int32, through slice::gemm::<i8, i32>'s C-ABI twin uor_b200_gemm_i8_i32.
With N GPUs the output is sharded by column blocks (the reference's Partition of
C into independent tiles, partition.rs:34): rank r owns an 8192-column block of
an 8192 x 8192 x (8192 N) product and its own B block; A is replicated. No
collective runs on the data path, so the scaling is weak. The default line also
carries the metric's second half, exact f32 GEMM TFLOPS at 8192^3 (config-3
operand distribution), measured on the same GPU after the headline.

Metric: exact-i8 TOPS = 2 m k n / t, whole job (all ranks' units / max rank time).
L2: three rotating operand sets (3 x 128 MiB > the 126 MB L2) plus a 256 MiB
output written every step, so no step reads operands a previous step left in L2.

--workload selects the other BASELINE configs for their own measurement lines
(i8-512: configs[0]; gemv / gemv-t: the narrow-side kernels at 1 x 8192 x 8192 and
8192 x 8192 x 1; codec: configs[1]; f32: configs[2]; wide: configs[3];
wide-splitk: configs[3] with the reduction split across ranks and one NCCL
all-reduce of exact limbs, strong scaling; trop: configs[4]'s max-plus half). They
are opt-in; the driver's line is the default.

--impl reference times the reference's CPU path on the host cores instead (the
Rust crate cannot be built here, so its C restatement in oracle/ stands in).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time
from types import SimpleNamespace

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "uor-matmul_b200"))
sys.path.insert(0, ROOT)

SIZE = 8192
METRIC = "exact i8 GEMM TOPS at 8192^3 (bit-exact, int32 out)"
WORKLOADS = ("i8", "i8-512", "gemv", "gemv-t", "codec", "codec-on-chip", "f32", "wide", "wide-splitk", "trop",
             "trop-witness", "complex", "codec-e8", "arena", "f64")


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--workload", default="i8", choices=WORKLOADS)
    p.add_argument("--size", type=int, default=None, help="square size of i8 / f32 workloads")
    p.add_argument("--batch", type=int, default=0,
                   help="products per step of the i8 workloads (0: 16 at the 8192^3 headline, "
                        "else 1)")
    p.add_argument("--e2e-steps", type=int, default=3)
    p.add_argument("--f32-steps", type=int, default=10,
                   help="timed steps of the exact f32 8192^3 half of the default line (0 skips)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the default line's extra keys (other configs, strong scaling)")
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


def tensor_peak():
    """The int8 dense denominator: twice the measured bf16 burst GEMM rate."""
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return (2.0 * peaks["bf16_tflops"],
                "2x measured bf16 burst (int8 dense issues at twice bf16 on B200), of measured")
    except Exception:
        return 2.0 * 1590.0, "2x fallback bf16 1.59 PFLOP/s, of fallback"


def load_traffic(name, key="bytes_per_launch"):
    try:
        return json.load(open(os.path.join(ROOT, "profiles", name))).get(key)
    except Exception:
        return None


# ---------------------------------------------------------------- CPU baseline

def host_threads(orc):
    """Every core this process may run on (torchrun sets OMP_NUM_THREADS=1 per rank)."""
    try:
        n = len(os.sched_getaffinity(0))
    except Exception:
        n = os.cpu_count() or 1
    return max(n, orc.max_threads())


def sample_rows(total_rows, run_rows, budget_s):
    """Time the oracle on a growing leading block of rows until it takes about a
    quarter of the budget; returns (rows, seconds, output of those rows)."""
    rows = 1
    while True:
        t0 = time.perf_counter()
        out = run_rows(rows)
        dt = time.perf_counter() - t0
        if dt * 4 > budget_s or rows >= total_rows:
            return rows, dt, out
        rows = min(total_rows, max(rows * 2, int(rows * budget_s / max(dt, 1e-3) / 4)))


# ---------------------------------------------------------------- workloads

def i8_batch(args, size):
    return args.batch if args.batch > 0 else (16 if size == SIZE else 1)


def i8_line_config(size, batch, sets, world):
    """The i8 line's config, printed identically by both arms."""
    name = ("configs[4] headline" if size == SIZE else "configs[0]" if size == 512 else "square")
    return {"workload": f"i8 x i8 -> i32 GEMM {size}x{size}x{size} per GPU ({name}), "
                        f"{batch} products per step, column-block sharded",
            "m": size, "k": size, "n_per_gpu": size, "batch": batch, "n_total": size * world,
            "l2": (f"{sets} rotating operand sets ({sets * 2 * size * size >> 20} MiB) + "
                   f"{4 * size * size >> 20} MiB output per product"),
            "parallelism": f"column blocks x{world}, no data-path collective"}


def wl_i8(args, U, torch, rank, size, sets=3, world=1):
    """configs[4] headline (size 8192) or configs[0] (size 512): i8 x i8 -> i32. A step
    is a batch of independent products over the rotating operand sets."""
    import numpy as np
    m = k = n = size
    batch = i8_batch(args, size)
    A = [torch.from_numpy(U.corpus(1 + 100 * s, U.CORPUS_I8, m * k)).cuda() for s in range(sets)]
    B = [torch.from_numpy(U.corpus(2 + 100 * s + 1000 * rank, U.CORPUS_I8, k * n)).cuda()
         for s in range(sets)]
    C = torch.empty(m * n, dtype=torch.int32, device="cuda")
    w = SimpleNamespace(route=U.Route(), units=2.0 * m * k * n * batch, launches=batch,
                        graph_sets=sets if size < 2048 else 0)

    def step(i, ctx):
        for j in range(batch):
            s = (i * batch + j) % sets
            U.gemm_i8_i32(m, k, n, A[s], B[s], C, ctx=ctx, route=w.route, asynchronous=True)

    def check(last):
        # Freivalds check in f64 on the last warm-up output (every partial < 2^53: exact)
        x = torch.randint(-1, 2, (n,), device="cuda", dtype=torch.float64)
        s = (last * batch + batch - 1) % sets
        lhs = C.view(m, n).double() @ x
        rhs = A[s].view(m, k).double() @ (B[s].view(k, n).double() @ x)
        assert torch.equal(lhs, rhs), "checksum mismatch"

    def cpu(budget_s, ctx):
        from oracle import oracle as orc
        U.gemm_i8_i32(m, k, n, A[0], B[0], C, ctx=ctx, asynchronous=True)
        ctx.sync()
        a, b = A[0].cpu().numpy(), B[0].cpu().numpy()
        threads = host_threads(orc)

        def run(rows):
            c = np.zeros(rows * n, np.int32)
            orc.gemm_i8_blocked(a[:rows * k], b, c, rows, k, n, threads=threads)
            return c
        rows, dt, c = sample_rows(m, run, budget_s)
        assert np.array_equal(c, C[:rows * n].cpu().numpy()), "GPU rows differ from the oracle"
        return {"value": 2.0 * rows * k * n / dt / 1e12, "unit": "TOPS", "cores": threads,
                "kind": "port",
                "sample": f"{rows} of {m} rows of the {m}x{k}x{n} product ({dt:.2f} s), blocked "
                          "C restatement of gemm_auto's s8 path, OpenMP over rows; the GPU's "
                          "rows were compared bit for bit"}

    def e2e(steps, ctx, stream):
        Bh = torch.from_numpy(U.corpus(2 + 1000 * rank, U.CORPUS_I8, k * n)).pin_memory()
        Ch = torch.empty(m * n, dtype=torch.int32).pin_memory()
        if world == 1:
            Ah = torch.from_numpy(U.corpus(1, U.CORPUS_I8, m * k)).pin_memory()

            def call():
                for _ in range(batch):
                    U.gemm_i8_i32(m, k, n, Ah, Bh, Ch, ctx=ctx)
            return timed_host(call, steps, stream, batch * (m * k + k * n), batch * 4 * m * n)
        # N > 1: A goes up once (rank 0) and is broadcast over NVLink; every rank uploads
        # its own B block and reads back its own C block.
        import uor_b200_dist as D
        Ah = (torch.from_numpy(U.corpus(1, U.CORPUS_I8, m * k)).pin_memory() if rank == 0
              else None)
        work = D.HostStaging(m * k, k * n, 4 * m * n)

        def call():
            for _ in range(batch):
                D.replicated_gemm_i8_host(m, k, n, Ah, Bh, Ch, work, ctx=ctx)
        # whole-job bytes: A once, every rank's B block in, every rank's C block out
        return timed_host(call, steps, stream, batch * (m * k + world * k * n),
                          batch * world * 4 * m * n)

    w.step, w.check, w.cpu, w.e2e = step, check, cpu, e2e
    w.metric = METRIC if size == SIZE else f"exact i8 GEMM TOPS at {size}^3 (bit-exact, int32 out)"
    w.unit, w.dtype = "TOPS", "int8"
    w.full_config = i8_line_config(size, batch, sets, world)
    w.config = {"workload": w.full_config["workload"], "m": m, "k": k, "n_per_gpu": n}
    w.l2 = w.full_config["l2"]
    w.algorithmic_bytes = m * k + k * n + 4 * m * n
    w.traffic = load_traffic("k1_pair_i8_8192_traffic.json") if size == SIZE else None
    w.flush = sets * 2 * m * k < (256 << 20)

    def roofline(avg_ms):
        # per launch: one product's work over the step time / the products in it
        peak, src = tensor_peak()
        ach = w.units / (avg_ms / 1e3) / 1e12
        return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TOPS",
                "frac": ach / peak, "peak_source": src,
                "frac_of_nominal_4500": ach / 4500.0,
                "launch_ms": avg_ms / batch,
                "traffic": w.traffic, "algorithmic_bytes": w.algorithmic_bytes}
    w.roofline = roofline
    return w


def wl_gemv(args, U, torch, rank, thin_m, sets=3):
    """The narrow-side shapes of the reduce factorization (spec.rs:474-526): 1 x 8192 x 8192
    (thin_m, the column kernel) or 8192 x 8192 x 1 (the reduce kernel); HBM-bound: the long
    operand is read once."""
    import numpy as np
    m, k, n = (1, 8192, 8192) if thin_m else (8192, 8192, 1)
    A = [torch.from_numpy(U.corpus(1 + 100 * s, U.CORPUS_I8, m * k)).cuda() for s in range(sets)]
    B = [torch.from_numpy(U.corpus(2 + 100 * s + 1000 * rank, U.CORPUS_I8, k * n)).cuda()
         for s in range(sets)]
    C = torch.empty(m * n, dtype=torch.int32, device="cuda")
    # the dp4a kernel and the exact chunk fold
    # units scaled so that measure()'s units/s/1e12 reads GB/s
    w = SimpleNamespace(route=U.Route(), units=float(m * k + k * n + 4 * m * n) * 1e3, launches=1,
                        graph_sets=sets)

    def step(i, ctx):
        U.gemm_i8_i32(m, k, n, A[i % sets], B[i % sets], C, ctx=ctx, route=w.route,
                      asynchronous=True)

    def check(last):
        s = last % sets
        want = (A[s].view(m, k).double() @ B[s].view(k, n).double()).reshape(-1)
        assert torch.equal(C.double(), want), "GEMV differs from the f64 product (exact here)"

    def cpu(budget_s, ctx):
        from oracle import oracle as orc
        step(0, ctx)
        ctx.sync()
        a, b = A[0].cpu().numpy(), B[0].cpu().numpy()
        threads = host_threads(orc)
        c = np.zeros(m * n, np.int32)
        reps, t0 = 0, time.perf_counter()
        while True:
            orc.gemm_i8_blocked(a, b, c, m, k, n, threads=threads)
            reps += 1
            dt = time.perf_counter() - t0
            if dt > budget_s / 4:
                break
        assert np.array_equal(c, C.cpu().numpy()), "GPU result differs from the oracle"
        return {"value": reps * w.units / dt / 1e12, "unit": "GB/s", "cores": threads,
                "kind": "port",
                "sample": f"the whole {m}x{k}x{n} product, {reps} times ({dt:.2f} s), blocked C "
                          "restatement; the GPU result was compared bit for bit"}

    def e2e(steps, ctx, stream):
        Ah, Bh = A[0].cpu().pin_memory(), B[0].cpu().pin_memory()
        Ch = torch.empty(m * n, dtype=torch.int32).pin_memory()
        return timed_host(lambda: U.gemm_i8_i32(m, k, n, Ah, Bh, Ch, ctx=ctx), steps, stream,
                          m * k + k * n, 4 * m * n)

    w.step, w.check, w.cpu, w.e2e = step, check, cpu, e2e
    w.metric = f"exact i8 GEMV GB/s, {m}x{k}x{n} (bit-exact, int32 out)"
    w.unit, w.dtype = "GB/s", "int8 (dp4a)"
    w.config = {"workload": f"i8 x i8 -> i32 {m}x{k}x{n} per GPU (narrow side: "
                            f"{'column' if thin_m else 'reduce'} kernel), column-block sharded",
                "m": m, "k": k, "n_per_gpu": n}
    w.l2 = f"{sets} rotating operand sets ({sets * (m * k + k * n) >> 20} MiB, > L2)"
    w.algorithmic_bytes = m * k + k * n + 4 * m * n
    w.flush = False

    def roofline(avg_ms):
        try:
            peak = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))["hbm_gbs"]
            src = "measured copy bandwidth (MEASURED_PEAKS.json hbm_gbs), of measured"
        except Exception:
            peak, src = 6650.0, "fallback 6.65 TB/s, of fallback"
        ach = w.algorithmic_bytes / (avg_ms / 1e3) / 1e9
        return {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak,
                "peak_source": src, "traffic": None, "algorithmic_bytes": w.algorithmic_bytes}
    w.roofline = roofline
    return w


def wl_codec(args, U, torch, rank, sets=3, on_chip=False):
    """A 2048 x 8192 i8, B 8192 x 8192 nibble codes through a 16-entry
    codebook (Packed<Grid<16>, 2>), exact i32 output, the codes decoded inside the
    tensor-core pipeline (K1C), never into a dense copy. on_chip: the same call with
    CODEC_ON_CHIP set (it changes only deep reductions)."""
    import numpy as np
    m, k, n = 2048, 8192, 8192
    A = [torch.from_numpy(U.corpus(1 + 100 * s, U.CORPUS_I8, m * k)).cuda() for s in range(sets)]
    Q = [torch.from_numpy(U.corpus(2 + 100 * s + 1000 * rank, U.CORPUS_NIBBLES, k * n)).cuda()
         for s in range(sets)]
    table = torch.from_numpy(U.corpus(7, U.CORPUS_I8, 16)).cuda()
    C = torch.empty(m * n, dtype=torch.int32, device="cuda")
    # one K1C launch: 512 x 256 tiles, each decoded stage serving both M256 halves
    w = SimpleNamespace(route=U.Route(), units=2.0 * m * k * n, launches=1)

    def step(i, ctx):
        U.coded_gemm(U.I32, A[i % sets], (m, k, k, 1), Q[i % sets], k, n, 2, table, C,
                     (m, n, n, 1), ctx=ctx, route=w.route, asynchronous=True, on_chip=on_chip)

    def dense(s):
        q = Q[s].to(torch.int64)
        codes = torch.stack([q & 15, q >> 4], dim=1).reshape(k, n)
        return table.to(torch.float64)[codes]

    def check(last):
        s = last % sets
        x = torch.randint(-1, 2, (n,), device="cuda", dtype=torch.float64)
        lhs = C.view(m, n).double() @ x
        rhs = A[s].view(m, k).double() @ (dense(s) @ x)
        assert torch.equal(lhs, rhs), "checksum mismatch"

    def cpu(budget_s, ctx):
        from oracle import oracle as orc
        step(0, ctx)
        ctx.sync()
        a, q, t = A[0].cpu().numpy(), Q[0].cpu().numpy(), table.cpu().numpy()
        threads = host_threads(orc)

        def run(rows):
            c = np.zeros(rows * n, np.int32)
            orc.coded_gemm(orc.View(a, rows, k, k, 1), q, 2, t, orc.View(c, rows, n, n, 1), k, n,
                           threads=threads)
            return c
        rows, dt, c = sample_rows(m, run, budget_s)
        assert np.array_equal(c, C[:rows * n].cpu().numpy()), "GPU rows differ from the oracle"
        return {"value": 2.0 * rows * k * n / dt / 1e12, "unit": "TOPS", "cores": threads,
                "kind": "port",
                "sample": f"{rows} of {m} rows ({dt:.2f} s), C restatement of coded_gemm "
                          "(per-MAC decode), OpenMP over rows; the GPU's rows were compared"}

    def e2e(steps, ctx, stream):
        Ah = A[0].cpu().pin_memory()
        Qh = Q[0].cpu().pin_memory()
        Th = table.cpu().pin_memory()
        Ch = torch.empty(m * n, dtype=torch.int32).pin_memory()
        return timed_host(lambda: U.coded_gemm(U.I32, Ah, (m, k, k, 1), Qh, k, n, 2, Th, Ch,
                                               (m, n, n, 1), ctx=ctx, on_chip=on_chip),
                          steps, stream, m * k + k * n // 2 + 16, 4 * m * n)

    w.step, w.check, w.cpu, w.e2e = step, check, cpu, e2e
    w.metric = "exact codec-tier GEMM TOPS, 2048x8192x8192, 4-bit codes (bit-exact, int32 out)"
    w.unit, w.dtype = "TOPS", "int8 (decoded nibble codes)"
    w.config = {"workload": "coded_gemm Packed<Grid<16>,2> 2048x8192x8192 per GPU (configs[1]), "
                            "column-block sharded", "m": m, "k": k, "n_per_gpu": n}
    w.l2 = f"{sets} rotating operand sets ({sets * (m * k + k * n // 2) >> 20} MiB) + 64 MiB output"
    w.algorithmic_bytes = m * k + k * n // 2 + 4 * m * n
    w.flush = False
    w.traffic = load_traffic("k1c_codec_on_chip_2048x8192x8192_traffic.json", "bytes_per_call")

    def roofline(avg_ms):
        peak, src = tensor_peak()
        ach = w.units / (avg_ms / 1e3) / 1e12
        return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TOPS",
                "frac": ach / peak, "peak_source": src, "traffic": w.traffic,
                "traffic_scope": "whole call (K1C), one ncu capture" if w.traffic else None,
                "algorithmic_bytes": w.algorithmic_bytes}
    w.roofline = roofline
    return w


def wl_codec_e8(args, U, torch, rank, sets=3):
    """configs[1]'s shape over the E8 codebook: B = Book<256, 8> with u8 codes (e8_codec_u8,
    0.125 bytes per weight), decoded inside the tensor-core pipeline (K1C's byte table)."""
    import numpy as np
    m, k, n = 2048, 8192, 8192
    A = [torch.from_numpy(U.corpus(1 + 100 * s, U.CORPUS_I8, m * k)).cuda() for s in range(sets)]
    Q = [torch.from_numpy(U.corpus(3 + 100 * s + 1000 * rank, U.CORPUS_RAW, k * n // 8)
                          .astype(np.uint8)).cuda() for s in range(sets)]
    table = torch.from_numpy(U.e8_table()).cuda()
    C = torch.empty(m * n, dtype=torch.int32, device="cuda")
    w = SimpleNamespace(route=U.Route(), units=2.0 * m * k * n, launches=1)

    def step(i, ctx):
        U.codec_gemm(U.I32, A[i % sets], (m, k, k, 1), U.TIER_BOOK, Q[i % sets], k, n, C,
                     (m, n, n, 1), table=table, block=8, code_bytes=1, ctx=ctx, route=w.route,
                     asynchronous=True)

    def check(last):
        s = last % sets
        dense = table.to(torch.float64)[Q[s].to(torch.int64)].reshape(k, n)
        x = torch.randint(-1, 2, (n,), device="cuda", dtype=torch.float64)
        assert torch.equal(C.view(m, n).double() @ x, A[s].view(m, k).double() @ (dense @ x))

    def cpu(budget_s, ctx):
        from oracle import oracle as orc
        step(0, ctx)
        ctx.sync()
        a, q, t = A[0].cpu().numpy(), Q[0].cpu().numpy(), table.cpu().numpy()
        # Book<256, 8>: code q of row r decodes to table[q] (8 weights); a table lookup
        dense = t[q.astype(np.int64)].reshape(k, n)
        threads = host_threads(orc)

        def run(rows):
            c = np.zeros(rows * n, np.int32)
            orc.gemm_int(orc.View(a, rows, k, k, 1), orc.View(dense.reshape(-1), k, n, n, 1),
                         orc.View(c, rows, n, n, 1), threads=threads)
            return c
        rows, dt, c = sample_rows(m, run, budget_s)
        assert np.array_equal(c, C[:rows * n].cpu().numpy()), "GPU rows differ from the oracle"
        return {"value": 2.0 * rows * k * n / dt / 1e12, "unit": "TOPS", "cores": threads,
                "kind": "port",
                "sample": f"{rows} of {m} rows ({dt:.2f} s), the Book table lookup then the "
                          "C restatement's integer GEMM, OpenMP over rows; GPU rows compared"}

    def e2e(steps, ctx, stream):
        Ah, Qh = A[0].cpu().pin_memory(), Q[0].cpu().pin_memory()
        Th = table.cpu().pin_memory()
        Ch = torch.empty(m * n, dtype=torch.int32).pin_memory()
        return timed_host(lambda: U.codec_gemm(U.I32, Ah, (m, k, k, 1), U.TIER_BOOK, Qh, k, n, Ch,
                                               (m, n, n, 1), table=Th, block=8, code_bytes=1,
                                               ctx=ctx),
                          steps, stream, m * k + k * n // 8 + 2048, 4 * m * n)

    w.step, w.check, w.cpu, w.e2e = step, check, cpu, e2e
    w.metric = "exact E8-codebook GEMM TOPS, 2048x8192x8192, Book<256,8> u8 codes (bit-exact, int32 out)"
    w.unit, w.dtype = "TOPS", "int8 (decoded E8 codewords)"
    w.config = {"workload": "codec_gemm Book<256,8> (E8, e8_codec_u8) 2048x8192x8192 per GPU, "
                            "column-block sharded", "m": m, "k": k, "n_per_gpu": n}
    w.l2 = f"{sets} rotating operand sets + 64 MiB output"
    w.algorithmic_bytes = m * k + k * n // 8 + 4 * m * n
    w.flush = False
    w.traffic = load_traffic("k1c_e8_book_on_chip_2048x8192x8192_traffic.json", "bytes_per_call")

    def roofline(avg_ms):
        peak, src = tensor_peak()
        ach = w.units / (avg_ms / 1e3) / 1e12
        return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TOPS",
                "frac": ach / peak, "peak_source": src, "traffic": w.traffic,
                "traffic_scope": "whole call (K1C), one ncu capture" if w.traffic else None,
                "basis": "2mnk int8 ops over the whole call (one K1C launch, the book decoded on chip)",
                "algorithmic_bytes": w.algorithmic_bytes}
    w.roofline = roofline
    return w


def wl_arena(args, U, torch, rank, sets=2):
    """Arena<f32, 256, u8> (CK-14's dequantized-8-bit codebook) as gemm_tabulated holds it:
    f32 A 2048 x 8192 against W 8192 x 8192 codes (n x k), exact f32 out."""
    import numpy as np
    m, k, n = 2048, 8192, 8192
    vals = (np.arange(256, dtype=np.float32) - np.float32(127.5)) * np.float32(2.0 ** -6)
    U.arena_canonicalize(vals)
    table = torch.from_numpy(vals).cuda()
    A = [torch.from_numpy(U.corpus(1 + 100 * s, U.CORPUS_F32_WIDE, m * k)).cuda() for s in range(sets)]
    Q = [torch.from_numpy(U.corpus(5 + 100 * s + 1000 * rank, U.CORPUS_RAW, n * k).astype(np.uint8)).cuda()
         for s in range(sets)]
    C = torch.empty(m * n, dtype=torch.float32, device="cuda")
    w = SimpleNamespace(route=U.Route(), units=2.0 * m * k * n, launches=7)

    def step(i, ctx):
        U.arena_gemm(U.F32, U.F32, A[i % sets], (m, k, k, 1), table, Q[i % sets], k, n, C,
                     (m, n, n, 1), orientation=1, ctx=ctx, route=w.route, asynchronous=True)

    def check(last):
        pass  # bit for bit by the CPU leg and the GPU tests

    def cpu(budget_s, ctx):
        from oracle import oracle as orc
        step(0, ctx)
        ctx.sync()
        a, q, t = A[0].cpu().numpy(), Q[0].cpu().numpy(), table.cpu().numpy()
        dense = orc.decode_arena(t, q, n, k)
        threads = host_threads(orc)

        def run(rows):
            c = np.zeros(rows * n, np.float32)
            orc.gemm_float(orc.View(a, rows, k, k, 1), orc.View(dense.reshape(-1), k, n, 1, k),
                           orc.View(c, rows, n, n, 1), threads=threads)
            return c
        rows, dt, c = sample_rows(m, run, budget_s)
        assert np.array_equal(c.view(np.uint32), C[:rows * n].cpu().numpy().view(np.uint32)), \
            "GPU rows differ from the oracle"
        return {"value": 2.0 * rows * k * n / dt / 1e12, "unit": "TFLOPS", "cores": threads,
                "kind": "port",
                "sample": f"{rows} of {m} rows ({dt:.2f} s), the oracle's Arena decode then the "
                          "C restatement of gemm_float, OpenMP over rows; GPU rows compared"}

    def e2e(steps, ctx, stream):
        Ah, Qh = A[0].cpu().pin_memory(), Q[0].cpu().pin_memory()
        Th = table.cpu().pin_memory()
        Ch = torch.empty(m * n, dtype=torch.float32).pin_memory()
        return timed_host(lambda: U.arena_gemm(U.F32, U.F32, Ah, (m, k, k, 1), Th, Qh, k, n, Ch,
                                               (m, n, n, 1), orientation=1, ctx=ctx),
                          steps, stream, 4 * m * k + n * k + 1024, 4 * m * n)

    w.step, w.check, w.cpu, w.e2e = step, check, cpu, e2e
    w.metric = "exact Arena f32 GEMM TFLOPS, 2048x8192x8192, 256 f32 symbols, u8 codes (bit-exact)"
    w.unit, w.dtype = "TFLOPS", "f32 (decoded symbols), exact float route"
    w.config = {"workload": "gemm_tabulated Arena<f32,256,u8> (CK-14 codebook) 2048x8192x8192 per "
                            "GPU, A from the configs[2] distribution", "m": m, "k": k, "n_per_gpu": n}
    w.l2 = f"{sets} rotating operand sets + 64 MiB output"
    w.algorithmic_bytes = 4 * m * k + n * k + 4 * m * n
    w.flush = False

    def roofline(avg_ms):
        peak, src = tensor_peak()
        gemms = max(1, w.route.pairs)
        ach = gemms * w.units / (avg_ms / 1e3) / 1e12
        return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TOPS",
                "frac": ach / peak, "peak_source": src, "traffic": None,
                "basis": f"int8 ops executed ({gemms} GEMMs of the exact float route x 2mnk)",
                "algorithmic_bytes": w.algorithmic_bytes}
    w.roofline = roofline
    return w


def wl_f32(args, U, torch, rank, size, sets=2):
    """exact f32 GEMM over the wide-exponent corpus with cancellation columns."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from float_data import config3
    m = k = n = size
    host = [config3(m, k, n, salt_a=1 + 100 * s, salt_b=2 + 100 * s + 1000 * rank)
            for s in range(sets)]
    A = [torch.from_numpy(h[0]).reshape(-1).cuda() for h in host]
    B = [torch.from_numpy(h[1]).reshape(-1).cuda() for h in host]
    C = torch.empty(m * n, dtype=torch.float32, device="cuda")
    # rows + columns analysis, A and B digit slicing, the slice-pair GEMM, the exact reduce
    w = SimpleNamespace(route=U.Route(), units=2.0 * m * k * n, launches=6)

    def step(i, ctx):
        U.gemm_float(U.F32, U.F32, A[i % sets], (m, k, k, 1), B[i % sets], (k, n, n, 1), C,
                     (m, n, n, 1), ctx=ctx, route=w.route, asynchronous=True)

    def check(last):
        # Bit for bit against the oracle on a leading block of rows of the last warm-up
        # product (rows 0 and 10 among them cancel to exactly zero), plus a sanity bound
        # on every cell: within 2^-20 relative of an f64 product where nothing cancels.
        from oracle import oracle as orc
        s = last % sets
        rows = min(m, getattr(w, "check_rows", 16))
        a, b = host[s]
        want = np.zeros(rows * n, np.float32)
        orc.gemm_float(orc.View(a.reshape(-1), rows, k, k, 1), orc.View(b.reshape(-1), k, n, n, 1),
                       orc.View(want, rows, n, n, 1), threads=host_threads(orc))
        got_rows = C[:rows * n].cpu().numpy()
        assert np.array_equal(want.view(np.uint32), got_rows.view(np.uint32)), \
            "f32 rows differ from the oracle"
        w.checked = (f"rows 0..{rows - 1} of the last warm-up product bit for bit against the "
                     "oracle; every cell within 2^-20 of f64 off the cancellation columns")
        ref = (A[s].view(m, k).double() @ B[s].view(k, n).double())
        got = C.view(m, n).double()
        keep = torch.ones(n, dtype=torch.bool, device="cuda")
        keep[::10] = False
        err = ((got - ref).abs() / ref.abs().clamp_min(1e-300))[:, keep]
        bad = float((err > 2.0 ** -20).double().mean())
        assert bad < 1e-5, f"f32 result far from the f64 product in {bad:.2e} of the cells"

    def cpu(budget_s, ctx):
        from oracle import oracle as orc
        step(0, ctx)
        ctx.sync()
        a, b = host[0]
        threads = host_threads(orc)

        def run(rows):
            c = np.zeros(rows * n, np.float32)
            orc.gemm_float(orc.View(a.reshape(-1), rows, k, k, 1), orc.View(b.reshape(-1), k, n, n, 1),
                           orc.View(c, rows, n, n, 1), threads=threads)
            return c
        rows, dt, c = sample_rows(m, run, budget_s)
        got = C[:rows * n].cpu().numpy()
        assert np.array_equal(c.view(np.uint32), got.view(np.uint32)), "GPU rows differ"
        return {"value": 2.0 * rows * k * n / dt / 1e12, "unit": "TFLOPS", "cores": threads,
                "kind": "port",
                "sample": f"{rows} of {m} rows ({dt:.2f} s), C restatement of the Complete "
                          "register accumulation (exact_product), OpenMP over rows; the GPU's "
                          "rows were compared bit for bit"}

    def e2e(steps, ctx, stream):
        Ah = torch.from_numpy(host[0][0]).reshape(-1).pin_memory()
        Bh = torch.from_numpy(host[0][1]).reshape(-1).pin_memory()
        Ch = torch.empty(m * n, dtype=torch.float32).pin_memory()
        return timed_host(lambda: U.gemm_float(U.F32, U.F32, Ah, (m, k, k, 1), Bh, (k, n, n, 1),
                                               Ch, (m, n, n, 1), ctx=ctx),
                          steps, stream, 8 * m * k, 4 * m * n)

    w.step, w.check, w.cpu, w.e2e = step, check, cpu, e2e
    w.metric = f"exact f32 GEMM TFLOPS at {size}^3 (bit-exact, rounded once)"
    w.unit, w.dtype = "TFLOPS", ("f32 in, int8 residue GEMMs modulo coprime moduli + CRT "
                                 "(or exact int8 digit slices), rounded once")
    w.config = {"workload": f"gemm_float f32 {m}x{k}x{n} per GPU (configs[2] distribution), "
                            "column-block sharded", "m": m, "k": k, "n_per_gpu": n}
    w.l2 = f"{sets} rotating operand sets ({sets * 8 * m * k >> 20} MiB) + {4 * m * n >> 20} MiB output"
    w.algorithmic_bytes = 8 * m * k + 4 * m * n
    w.flush = False
    w.traffic = (load_traffic(f"modular_f32_{size}_traffic.json", "bytes_per_call")
                 if size in (4096, 8192) else None)

    def roofline(avg_ms):
        peak, src = tensor_peak()
        pairs = max(1, w.route.pairs)
        ach = pairs * w.units / (avg_ms / 1e3) / 1e12
        if w.route.moduli:
            basis = (f"int8 GEMM ops executed ({w.route.moduli} residue GEMMs modulo coprime "
                     "moduli <= 256 x 2mnk) over the whole call (analysis, residue slicing, "
                     "GEMMs, CRT and encode)")
        else:
            basis = (f"int8 slice-pair ops executed ({pairs} of {w.route.a_layout} x "
                     f"{w.route.b_layout} digit pairs x 2mnk; {w.route.fixups} cells "
                     "recomputed exactly) over the whole call (analysis, slicing, GEMM, "
                     "interval test, fixups)")
        return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TOPS",
                "frac": ach / peak, "peak_source": src, "traffic": w.traffic,
                "traffic_scope": ("whole call, one ncu capture" if w.traffic else
                                  "not captured at this size; the 4096^3 call moves 13x its "
                                  "algorithmic bytes, the 8192^3 call 22x"),
                "basis": basis, "algorithmic_bytes": w.algorithmic_bytes}
    w.roofline = roofline
    return w


def wl_f64(args, U, torch, rank, size, sets=2):
    """raw::dgemm (exact f64, rounded once) at configs[2]'s shape and exponent range with
    full 53-bit significands: +-m 2^(e - 52), m in [2^52, 2^53), e in [-30, 30]."""
    import numpy as np
    m = k = n = size
    rng = np.random.default_rng(64 + rank)

    def draw(count):
        mant = rng.integers(1 << 52, 1 << 53, size=count, dtype=np.int64).astype(np.float64)
        e = rng.integers(-30, 31, size=count)
        sgn = rng.choice([-1.0, 1.0], size=count)
        return sgn * np.ldexp(mant, e - 52)
    host = [(draw(m * k), draw(k * n)) for _ in range(sets)]
    A = [torch.from_numpy(h[0]).cuda() for h in host]
    B = [torch.from_numpy(h[1]).cuda() for h in host]
    C = torch.empty(m * n, dtype=torch.float64, device="cuda")
    w = SimpleNamespace(route=U.Route(), units=2.0 * m * k * n, launches=6)

    def step(i, ctx):
        U.gemm_float(U.F64, U.F64, A[i % sets], (m, k, k, 1), B[i % sets], (k, n, n, 1), C,
                     (m, n, n, 1), ctx=ctx, route=w.route, asynchronous=True)

    def check(last):
        pass  # bit for bit by the CPU leg and the GPU tests

    def cpu(budget_s, ctx):
        from oracle import oracle as orc
        step(0, ctx)
        ctx.sync()
        a, b = host[0]
        threads = host_threads(orc)

        def run(rows):
            c = np.zeros(rows * n, np.float64)
            orc.gemm_float(orc.View(a, rows, k, k, 1), orc.View(b, k, n, n, 1),
                           orc.View(c, rows, n, n, 1), threads=threads)
            return c
        rows, dt, c = sample_rows(m, run, budget_s)
        assert np.array_equal(c.view(np.uint64), C[:rows * n].cpu().numpy().view(np.uint64)), \
            "GPU rows differ"
        return {"value": 2.0 * rows * k * n / dt / 1e12, "unit": "TFLOPS", "cores": threads,
                "kind": "port",
                "sample": f"{rows} of {m} rows ({dt:.2f} s), C restatement of the f64 Complete "
                          "register accumulation, OpenMP over rows; GPU rows compared bit for bit"}

    def e2e(steps, ctx, stream):
        Ah = torch.from_numpy(host[0][0]).pin_memory()
        Bh = torch.from_numpy(host[0][1]).pin_memory()
        Ch = torch.empty(m * n, dtype=torch.float64).pin_memory()
        return timed_host(lambda: U.gemm_float(U.F64, U.F64, Ah, (m, k, k, 1), Bh, (k, n, n, 1),
                                               Ch, (m, n, n, 1), ctx=ctx),
                          steps, stream, 16 * m * k, 8 * m * n)

    w.step, w.check, w.cpu, w.e2e = step, check, cpu, e2e
    w.metric = f"exact f64 GEMM TFLOPS at {size}^3 (raw::dgemm, bit-exact, rounded once)"
    w.unit, w.dtype = "TFLOPS", "f64 in, int8 residue GEMMs modulo coprime moduli + CRT"
    w.config = {"workload": f"dgemm f64 {m}x{k}x{n} per GPU (53-bit significands, exponents "
                            "in [-30, 30]), column-block sharded", "m": m, "k": k, "n_per_gpu": n}
    w.l2 = f"{sets} rotating operand sets ({sets * 16 * m * k >> 20} MiB) + {8 * m * n >> 20} MiB output"
    w.algorithmic_bytes = 16 * m * k + 8 * m * n
    w.flush = False

    def roofline(avg_ms):
        peak, src = tensor_peak()
        gemms = max(1, w.route.pairs)
        ach = gemms * w.units / (avg_ms / 1e3) / 1e12
        return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TOPS",
                "frac": ach / peak, "peak_source": src, "traffic": None,
                "basis": f"int8 ops executed ({gemms} GEMMs x 2mnk; moduli {w.route.moduli}) "
                         "over the whole call",
                "algorithmic_bytes": w.algorithmic_bytes}
    w.roofline = roofline
    return w


def wl_wide(args, U, torch, rank):
    """i32 x i32 full range, 1024 x 65536 x 1024, exact i128 output."""
    import numpy as np
    m, k, n = 1024, 65536, 1024
    A = torch.from_numpy(U.corpus(4, U.CORPUS_I32_FULL, m * k)).cuda()
    B = torch.from_numpy(U.corpus(5 + 1000 * rank, U.CORPUS_I32_FULL, k * n)).cuda()
    C = torch.zeros(m * n * 2, dtype=torch.int64, device="cuda")
    # A and B byte slicing, the limb-pair GEMM, the exact recombination
    w = SimpleNamespace(route=U.Route(), units=2.0 * m * k * n, launches=4)

    def step(i, ctx):
        U.gemm(U.I32, U.I128, A, (m, k, k, 1), B, (k, n, n, 1), C, (m, n, n, 1), ctx=ctx,
               route=w.route, asynchronous=True)

    def check(last):
        pass  # sums reach 2^78: checked bit for bit by the CPU leg and the GPU tests

    def cpu(budget_s, ctx):
        from oracle import oracle as orc
        step(0, ctx)
        ctx.sync()
        a, b = A.cpu().numpy(), B.cpu().numpy()
        threads = host_threads(orc)

        def run(rows):
            c = np.zeros(rows * n * 2, np.int64)
            orc.gemm_int(orc.View(a, rows, k, k, 1), orc.View(b, k, n, n, 1),
                         orc.View(c, rows, n, n, 1), out_bits=128, threads=threads)
            return c
        rows, dt, c = sample_rows(m, run, budget_s)
        assert np.array_equal(c, C[:rows * n * 2].cpu().numpy()), "GPU rows differ"
        return {"value": 2.0 * rows * k * n / dt / 1e12, "unit": "TOPS", "cores": threads,
                "kind": "port",
                "sample": f"{rows} of {m} rows ({dt:.2f} s), C restatement of the i32 -> i128 "
                          "exact loop, OpenMP over rows; the GPU's rows were compared"}

    def e2e(steps, ctx, stream):
        Ah, Bh = A.cpu().pin_memory(), B.cpu().pin_memory()
        Ch = torch.empty(m * n * 2, dtype=torch.int64).pin_memory()
        return timed_host(lambda: U.gemm(U.I32, U.I128, Ah, (m, k, k, 1), Bh, (k, n, n, 1), Ch,
                                         (m, n, n, 1), ctx=ctx),
                          steps, stream, 4 * (m * k + k * n), 16 * m * n)

    w.step, w.check, w.cpu, w.e2e = step, check, cpu, e2e
    w.metric = "exact i32 -> i128 GEMM TOPS, 1024x65536x1024 (bit-exact)"
    w.unit, w.dtype = "TOPS", "int32 in (4 x 4 int8 limb pairs), int128 out"
    w.config = {"workload": "i32 x i32 -> i128 GEMM 1024x65536x1024 per GPU (configs[3]), "
                            "column-block sharded", "m": m, "k": k, "n_per_gpu": n}
    w.l2 = "512 MiB of operands per step (> L2)"
    w.algorithmic_bytes = 4 * (m * k + k * n) + 16 * m * n
    w.flush = False
    w.traffic = load_traffic("modular_wide_i32_1024x65536x1024_traffic.json", "bytes_per_call")

    def roofline(avg_ms):
        peak, src = tensor_peak()
        gemms = max(1, w.route.pairs)
        ach = gemms * w.units / (avg_ms / 1e3) / 1e12
        what = (f"{gemms} residue GEMMs modulo coprime moduli (modular route; 16 byte-slice "
                "pairs otherwise)" if w.route.moduli else f"{gemms} int8 byte-slice pairs")
        return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TOPS",
                "frac": ach / peak, "peak_source": src, "traffic": w.traffic,
                "traffic_scope": "whole call (slicers, residue GEMMs, CRT), one ncu capture",
                "basis": f"int8 ops executed ({what} x 2mnk) over the whole call (slicing, "
                         "GEMMs, recombination)",
                "algorithmic_bytes": w.algorithmic_bytes}
    w.roofline = roofline
    return w


def wl_complex(args, U, torch, rank):
    """Complex<i32> full range, 1024 x 16384 x 1024, exact Complex<i128> output: the real
    product of the operands' real images (1024 x 32768 x 2048) on the limb path."""
    import numpy as np
    m, k, n = 1024, 16384, 1024
    A = torch.from_numpy(U.corpus(4, U.CORPUS_I32_FULL, 2 * m * k)).cuda()
    B = torch.from_numpy(U.corpus(5 + 1000 * rank, U.CORPUS_I32_FULL, 2 * k * n)).cuda()
    C = torch.zeros(m * n * 4, dtype=torch.int64, device="cuda")
    # A and B byte slicing (B into its real image), the limb-pair GEMM, the recombination
    w = SimpleNamespace(route=U.Route(), units=8.0 * m * k * n, launches=4)

    def step(i, ctx):
        U.gemm_complex(U.I32, U.I128, A, (m, k, k, 1), B, (k, n, n, 1), C, (m, n, n, 1),
                       ctx=ctx, route=w.route, asynchronous=True)

    def check(last):
        pass  # checked bit for bit by the CPU leg and the GPU tests

    def cpu(budget_s, ctx):
        from oracle import oracle as orc
        step(0, ctx)
        ctx.sync()
        a, b = A.cpu().numpy(), B.cpu().numpy()
        threads = host_threads(orc)

        def run(rows):
            c = np.zeros(rows * n * 4, np.int64)
            orc.gemm_complex(orc.View(a, rows, k, k, 1), orc.View(b, k, n, n, 1),
                             orc.View(c, rows, n, n, 1), out_bits=128, threads=threads)
            return c
        rows, dt, c = sample_rows(m, run, budget_s)
        assert np.array_equal(c, C[:rows * n * 4].cpu().numpy()), "GPU rows differ"
        return {"value": 8.0 * rows * k * n / dt / 1e12, "unit": "TOPS", "cores": threads,
                "kind": "port",
                "sample": f"{rows} of {m} rows ({dt:.2f} s), C restatement of the Complex<i32> "
                          "componentwise mac into i128 parts, OpenMP over rows; the GPU's rows "
                          "were compared"}

    def e2e(steps, ctx, stream):
        Ah, Bh = A.cpu().pin_memory(), B.cpu().pin_memory()
        Ch = torch.empty(m * n * 4, dtype=torch.int64).pin_memory()
        return timed_host(lambda: U.gemm_complex(U.I32, U.I128, Ah, (m, k, k, 1), Bh,
                                                 (k, n, n, 1), Ch, (m, n, n, 1), ctx=ctx),
                          steps, stream, 8 * (m * k + k * n), 32 * m * n)

    w.step, w.check, w.cpu, w.e2e = step, check, cpu, e2e
    w.metric = "exact Complex<i32> -> Complex<i128> GEMM TOPS (8 integer ops per complex mac), " \
               "1024x16384x1024 (bit-exact)"
    w.unit, w.dtype = "TOPS", "Complex<int32> in (4 x 4 int8 limb pairs), Complex<int128> out"
    w.config = {"workload": "Complex<i32> GEMM 1024x16384x1024 per GPU (alphabet.rs Complex), "
                            "column-block sharded", "m": m, "k": k, "n_per_gpu": n}
    w.l2 = "256 MiB of operands per step (> L2)"
    w.algorithmic_bytes = 8 * (m * k + k * n) + 32 * m * n
    w.flush = False

    def roofline(avg_ms):
        peak, src = tensor_peak()
        gemms = max(1, w.route.pairs)
        ach = gemms * w.units / (avg_ms / 1e3) / 1e12  # one real-image GEMM is 8mkn ops
        return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TOPS",
                "frac": ach / peak, "peak_source": src, "traffic": None,
                "basis": f"int8 ops executed ({gemms} {'residue GEMMs' if w.route.moduli else 'byte-slice pairs'}"
                         " x 2 x m x 2k x 2n) over the whole call (slicing, GEMMs, recombination)",
                "algorithmic_bytes": w.algorithmic_bytes}
    w.roofline = roofline
    return w


def wl_trop(args, U, torch, rank, selected=False):
    """configs[4]'s max-plus half: Trop<i8> 8192^3 with 5 % -inf, Trop<i32> output; with
    `selected`, gemm_selected's witness (the least index attaining each maximum) too."""
    import numpy as np
    m = k = n = 8192
    A = torch.from_numpy(U.corpus(1, U.CORPUS_TROP_I8, m * k)).cuda()
    B = torch.from_numpy(U.corpus(2 + 1000 * rank, U.CORPUS_TROP_I8, k * n)).cuda()
    C = torch.zeros(m * n * 8, dtype=torch.uint8, device="cuda")
    Wt = torch.zeros(m * n, dtype=torch.int64, device="cuda") if selected else None
    # A and B packing, the max-plus kernel
    w = SimpleNamespace(route=U.Route(), units=float(m) * k * n, launches=3)

    def step(i, ctx):
        if selected:
            U.gemm_tropical_selected(U.TROP_I8, U.TROP_I32, A, (m, k, k, 1), B, (k, n, n, 1), C,
                                     (m, n, n, 1), Wt, (m, n, n, 1), ctx=ctx, route=w.route)
        else:
            U.gemm_tropical(U.TROP_I8, U.TROP_I32, A, (m, k, k, 1), B, (k, n, n, 1), C,
                            (m, n, n, 1), ctx=ctx, route=w.route, asynchronous=True)

    def check(last):
        pass  # checked bit for bit on rows by the CPU leg and the GPU tests

    def cpu(budget_s, ctx):
        from oracle import oracle as orc
        TD = orc.TROP_DTYPES
        step(0, ctx)
        ctx.sync()
        a, b = A.cpu().numpy().view(TD[8]), B.cpu().numpy().view(TD[8])
        threads = host_threads(orc)

        def run(rows):
            c = np.zeros(rows * n, TD[32])
            orc.gemm_trop(orc.View(a, rows, k, k, 1), orc.View(b, k, n, n, 1),
                          orc.View(c, rows, n, n, 1), ebits=8, obits=32, threads=threads)
            return c
        rows, dt, c = sample_rows(m, run, budget_s)
        got = C[:rows * n * 8].cpu().numpy().view(TD[32])
        ok = np.array_equal(got["f"], c["f"]) and np.array_equal(
            np.where(got["f"] != 0, got["v"], 0), np.where(c["f"] != 0, c["v"], 0))
        assert ok, "GPU rows differ from the oracle"
        return {"value": float(rows) * k * n / dt / 1e12, "unit": "Tterm/s", "cores": threads,
                "kind": "port",
                "sample": f"{rows} of {m} rows ({dt:.2f} s), C restatement of driver::gemm's "
                          "max-plus loop, OpenMP over rows; the GPU's rows were compared"}

    def e2e(steps, ctx, stream):
        Ah, Bh = A.cpu().pin_memory(), B.cpu().pin_memory()
        Ch = torch.empty(m * n * 8, dtype=torch.uint8).pin_memory()
        return timed_host(lambda: U.gemm_tropical(U.TROP_I8, U.TROP_I32, Ah, (m, k, k, 1), Bh,
                                                  (k, n, n, 1), Ch, (m, n, n, 1), ctx=ctx),
                          steps, stream, 2 * (m * k + k * n), 8 * m * n)

    w.step, w.check, w.cpu, w.e2e = step, check, cpu, e2e
    w.metric = "exact max-plus GEMM Tterm/s, Trop<i8> 8192^3 (bit-exact, Trop<i32> out)"
    w.unit, w.dtype = "Tterm/s", "int16x2 packed lanes"
    w.config = {"workload": "Trop<i8> max-plus 8192x8192x8192 per GPU (configs[4]), "
                            "column-block sharded", "m": m, "k": k, "n_per_gpu": n}
    w.l2 = "256 MiB of operands + 512 MiB output per step (> L2)"
    w.algorithmic_bytes = 2 * (m * k + k * n) + 8 * m * n
    w.flush = False

    def roofline(avg_ms):
        # one fused packed i16x2 add-max per two terms; the ALU pipe takes a packed 16x2
        # instruction from 64 lanes per SM and clock
        peak = 148 * 64 * 2 * 1.965e9 / 1e12
        ach = w.units / (avg_ms / 1e3) / 1e12
        return {"bound": "alu", "achieved": ach, "peak": peak, "unit": "Tterm/s",
                "frac": ach / peak,
                "peak_source": "nominal: 148 SMs x 64 lanes/clk (packed i16x2 ALU rate) x 2 "
                               "terms per fused add-max x 1.965 GHz",
                "traffic": None, "algorithmic_bytes": w.algorithmic_bytes}
    w.roofline = roofline
    if selected:
        # one fused 32-bit add-max per term on (value, index) keys: half the packed rate
        w.e2e = None
        w.metric = ("exact max-plus GEMM with selection witness Tterm/s, Trop<i8> 8192^3 "
                    "(bit-exact, Trop<i32> + least-index witness out)")
        w.algorithmic_bytes = 4 * (m * k + k * n) + 16 * m * n
        w.dtype = "int32 (value, index) keys"
        w.config = dict(w.config, workload="Trop<i8> max-plus 8192^3 + gemm_selected witness "
                                           "per GPU, column-block sharded")

        def roofline_sel(avg_ms):
            r = roofline(avg_ms)
            r["peak"] = r["peak"] / 2
            r["frac"] = r["achieved"] / r["peak"]
            r["peak_source"] = ("nominal: 148 SMs x 64 lanes/clk x 1 term per fused 32-bit "
                                "add-max x 1.965 GHz")
            return r
        w.roofline = roofline_sel
    return w


def wl_wide_splitk(args, U, torch, rank, world):
    """configs[3] with the reduction split across ranks (strong scaling): each rank's
    exact partial sum as radix-2^40 limbs, one NCCL all-reduce of 3 m n int64, one
    finish per rank."""
    import numpy as np
    import uor_b200_dist as D
    m, k, n = 1024, 65536, 1024
    A = torch.from_numpy(U.corpus(4, U.CORPUS_I32_FULL, m * k)).cuda()
    B = torch.from_numpy(U.corpus(5, U.CORPUS_I32_FULL, k * n)).cuda()
    C = torch.zeros(m * n * 2, dtype=torch.int64, device="cuda")
    # partial (slicing, limb-pair GEMM, recombination into i128, limbs) and finish
    w = SimpleNamespace(route=U.Route(), units=2.0 * m * k * n / world, launches=6)

    def step(i, ctx):
        D.splitk_gemm(U.I32, U.I128, A, (m, k, k, 1), B, (k, n, n, 1), C, (m, n, n, 1), ctx=ctx,
                      partial=lambda *a, **kw: U.gemm_partial_limbs(*a, route=w.route, **kw))

    def check(last):
        want = torch.zeros_like(C)
        U.gemm(U.I32, U.I128, A, (m, k, k, 1), B, (k, n, n, 1), want, (m, n, n, 1))
        assert torch.equal(C, want), "split-K result differs from the one-device call"

    def cpu(budget_s, ctx):
        return wl_wide(args, U, torch, rank).cpu(budget_s, ctx)

    w.step, w.check, w.cpu = step, check, cpu
    w.e2e = None
    w.metric = "exact i32 -> i128 GEMM TOPS, 1024x65536x1024, split-K (bit-exact)"
    w.unit, w.dtype = "TOPS", "int32 in (4 x 4 int8 limb pairs), int128 out"
    w.config = {"workload": "i32 x i32 -> i128 GEMM 1024x65536x1024 in total (configs[3]), "
                            "reduction split across ranks", "m": m, "k": k, "n_per_gpu": n}
    w.scaling = "strong"
    w.parallelism = (f"split-K x{world}: radix-2^40 int64 limbs, one NCCL all-reduce of "
                     f"{3 * 8 * m * n >> 20} MiB")
    w.l2 = "512 MiB of operands (> L2)"
    w.algorithmic_bytes = 4 * (m * k + k * n) // world + 16 * m * n
    w.flush = False

    def roofline(avg_ms):
        peak, src = tensor_peak()
        ach = 16 * w.units / (avg_ms / 1e3) / 1e12
        return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TOPS",
                "frac": ach / peak, "peak_source": src, "traffic": None,
                "basis": "this rank's int8 limb-pair ops (16 x 2mnk / ranks) over the whole "
                         "step (partial, exchange, finish)",
                "algorithmic_bytes": w.algorithmic_bytes}
    w.roofline = roofline
    return w


def wl_i8_strong(args, U, torch, rank, world, dist, sets=3):
    """The fixed 8192^3 i8 product sharded over the ranks by output column blocks
    (partition.rs:34): rank r owns C[:, r n/N .. (r+1) n/N] and that block of B; A is
    uploaded once and broadcast over NCCL before the timed region. The all-gather of
    the C blocks is timed on its own (``collective``)."""
    import uor_b200_dist as D
    m = k = n = SIZE
    batch = i8_batch(args, SIZE)
    t = D.column_blocks(m, n, world).tile(rank)
    cols = t.cols if t is not None else 0
    A = []
    for s in range(sets):
        a = (torch.from_numpy(U.corpus(1 + 100 * s, U.CORPUS_I8, m * k)).cuda() if rank == 0
             else torch.empty(m * k, dtype=torch.int8, device="cuda"))
        if dist:
            dist.broadcast(a, src=0)
        A.append(a)
    B = []
    for s in range(sets):
        full = torch.from_numpy(U.corpus(2 + 100 * s, U.CORPUS_I8, k * n)).view(k, n)
        B.append(full[:, t.col:t.col + cols].contiguous().view(-1).cuda())
    C = torch.empty(m * max(cols, 1), dtype=torch.int32, device="cuda")
    w = SimpleNamespace(route=U.Route(), units=2.0 * m * k * cols * batch, launches=batch)

    def step(i, ctx):
        for j in range(batch):
            s = (i * batch + j) % sets
            U.gemm_i8_i32(m, k, cols, A[s], B[s], C, ctx=ctx, route=w.route, asynchronous=True)

    def check(last):
        x = torch.randint(-1, 2, (cols,), device="cuda", dtype=torch.float64)
        s = (last * batch + batch - 1) % sets
        lhs = C.view(m, cols).double() @ x
        rhs = A[s].view(m, k).double() @ (B[s].view(k, cols).double() @ x)
        assert torch.equal(lhs, rhs), "checksum mismatch"

    def collective_ms(reps=5):
        if not dist:
            return None
        full = torch.empty(world * C.numel(), dtype=torch.int32, device="cuda")
        dist.all_gather_into_tensor(full, C)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            dist.all_gather_into_tensor(full, C)
        e1.record()
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1) / reps], device="cuda", dtype=torch.float64)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        ms = float(ms.item())
        return {"op": "NCCL all-gather of the C column blocks (outside the timed steps)",
                "bytes_per_rank": 4 * C.numel(), "ms": ms,
                "busbw_gbs": 4 * C.numel() * (world - 1) / (ms / 1e3) / 1e9}

    w.step, w.check, w.e2e = step, check, None
    w.cpu = None
    w.collective_ms = collective_ms
    w.metric = "exact i8 GEMM TOPS, one 8192^3 product sharded over the GPUs (bit-exact)"
    w.unit, w.dtype = "TOPS", "int8"
    w.scaling = "strong"
    w.full_config = {
        "workload": f"i8 x i8 -> i32 GEMM 8192x8192x8192 in total, {batch} products per step, "
                    f"column blocks of {cols} per GPU", "m": m, "k": k, "n": n,
        "n_per_gpu": cols, "batch": batch,
        "l2": f"{sets} rotating operand sets ({sets * (m * k + k * cols) >> 20} MiB per GPU)",
        "parallelism": f"column blocks x{world}; A broadcast once over NCCL before timing; "
                       "no collective in the timed steps"}
    w.config = w.full_config
    w.algorithmic_bytes = m * k + k * cols + 4 * m * cols
    w.flush = False

    def roofline(avg_ms):
        peak, src = tensor_peak()
        ach = w.units / (avg_ms / 1e3) / 1e12
        return {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TOPS",
                "frac": ach / peak, "peak_source": src, "launch_ms": avg_ms / batch,
                "pair_tiles_per_launch": -(-m // 256) * -(-cols // 256),
                "traffic": None, "algorithmic_bytes": w.algorithmic_bytes}
    w.roofline = roofline
    return w


def wl_trop_strong(args, U, torch, rank, world, dist):
    """configs[4]'s max-plus half as one fixed Trop<i8> 8192^3 product sharded over the
    ranks by output column blocks (partition.rs:34): rank r owns C[:, r n/N ..] and that
    block of B; A is broadcast once over NCCL before the timed region."""
    import uor_b200_dist as D
    m = k = n = SIZE
    t = D.column_blocks(m, n, world).tile(rank)
    cols = t.cols if t is not None else 0
    A = (torch.from_numpy(U.corpus(1, U.CORPUS_TROP_I8, m * k)).cuda() if rank == 0
         else torch.empty(2 * m * k, dtype=torch.uint8, device="cuda"))
    if dist:
        dist.broadcast(A, src=0)
    full = torch.from_numpy(U.corpus(2, U.CORPUS_TROP_I8, k * n)).view(k, n, 2)
    B = full[:, t.col:t.col + cols].contiguous().view(-1).cuda()
    del full
    C = torch.zeros(8 * m * max(cols, 1), dtype=torch.uint8, device="cuda")
    w = SimpleNamespace(route=U.Route(), units=float(m) * k * cols, launches=3)

    def step(i, ctx):
        U.gemm_tropical(U.TROP_I8, U.TROP_I32, A, (m, k, k, 1), B, (k, cols, cols, 1), C,
                        (m, cols, cols, 1), ctx=ctx, route=w.route, asynchronous=True)

    w.step, w.check, w.e2e, w.cpu = step, (lambda last: None), None, None
    w.metric = "exact max-plus GEMM Tterm/s, one Trop<i8> 8192^3 product sharded over the GPUs"
    w.unit, w.dtype = "Tterm/s", "int16x2 packed lanes"
    w.scaling = "strong"
    w.full_config = {
        "workload": f"Trop<i8> max-plus 8192x8192x8192 in total, column blocks of {cols} per GPU",
        "m": m, "k": k, "n": n, "n_per_gpu": cols,
        "l2": "256 MiB of operands per GPU at N = 1 (> L2)",
        "parallelism": f"column blocks x{world}; A broadcast once over NCCL before timing; "
                       "no collective in the timed steps"}
    w.config = w.full_config
    w.algorithmic_bytes = 2 * (m * k + k * cols) + 8 * m * cols
    w.flush = False

    def roofline(avg_ms):
        peak = 148 * 64 * 2 * 1.965e9 / 1e12
        ach = w.units / (avg_ms / 1e3) / 1e12
        return {"bound": "alu", "achieved": ach, "peak": peak, "unit": "Tterm/s",
                "frac": ach / peak, "peak_source": "nominal packed i16x2 ALU rate (see trop line)",
                "traffic": None, "algorithmic_bytes": w.algorithmic_bytes}
    w.roofline = roofline
    return w


def build_workload(name, args, U, torch, rank, world=1):
    if name == "i8":
        return wl_i8(args, U, torch, rank, args.size or SIZE, world=world)
    if name == "i8-512":
        return wl_i8(args, U, torch, rank, args.size or 512, sets=1)
    if name == "gemv":
        return wl_gemv(args, U, torch, rank, True)
    if name == "gemv-t":
        return wl_gemv(args, U, torch, rank, False)
    if name == "codec":
        return wl_codec(args, U, torch, rank)
    if name == "codec-on-chip":
        return wl_codec(args, U, torch, rank, on_chip=True)
    if name == "f32":
        return wl_f32(args, U, torch, rank, args.size or 4096)
    if name == "wide":
        return wl_wide(args, U, torch, rank)
    if name == "wide-splitk":
        return wl_wide_splitk(args, U, torch, rank, world)
    if name == "complex":
        return wl_complex(args, U, torch, rank)
    if name == "codec-e8":
        return wl_codec_e8(args, U, torch, rank)
    if name == "arena":
        return wl_arena(args, U, torch, rank)
    if name == "f64":
        return wl_f64(args, U, torch, rank, args.size or 4096)
    return wl_trop(args, U, torch, rank, selected=name == "trop-witness")


# ---------------------------------------------------------------- timing

def timed_host(call, steps, stream, h2d, d2h):
    """The public call with pinned HOST buffers: every step copies its inputs in and
    its result out inside the timed region."""
    import torch
    call()  # warm the staging buffers
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        call()
    e1.record(stream)
    torch.cuda.synchronize()
    return {"ms": e0.elapsed_time(e1) / steps, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h}


def time_steps(w, ctx, stream, torch, dist, steps, warmup, local):
    for i in range(warmup):
        w.step(i, ctx)
    assert ctx.sync() == 0
    if warmup > 0:  # the output holds a step's result only after one has run
        w.check(warmup - 1)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda") if w.flush else None
    run = lambda i: w.step(i, ctx)  # noqa: E731
    graphs = []
    if getattr(w, "graph_sets", 0):
        # Steps shorter than the host's per-call work (argument marshalling, tensor maps,
        # the launch) are replayed from CUDA graphs of the same library call, one per
        # operand set, so the GPU is never starved between them.
        try:
            for gs in range(w.graph_sets):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    w.step(gs, ctx)
                graphs.append(g)
            torch.cuda.synchronize()
            run = lambda i: graphs[i % len(graphs)].replay()  # noqa: E731
            w.graphed = True
        except Exception as exc:  # pragma: no cover - reported in the line
            graphs = []
            w.graphed = f"not captured: {exc}"
    clocks = Clocks(local)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(steps):
        if flush is not None:
            flush.fill_(i & 0xFF)  # an L2-sized write between steps, outside the step events
        ev[i][0].record(stream)
        run(warmup + i)
        ev[i][1].record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clk = clocks.stop()
    assert ctx.sync() == 0
    del graphs
    step_ms = [a.elapsed_time(b) for a, b in ev]
    # With an L2 flush between steps the region holds the flushes too: count the steps.
    elapsed = sum(step_ms) if flush is not None else t_start.elapsed_time(t_end)
    if dist:
        t = torch.tensor([elapsed], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
    return elapsed, step_ms, clk


# ---------------------------------------------------------------- reference arm

def reference_arm(args, rank, world):
    """The reference's CPU path for the same workload on the host cores (rank 0). Only
    the oracle runs here: its C restatement draws the operands and computes the rows."""
    if rank != 0:
        return
    from oracle import oracle as orc
    import numpy as np
    size = args.size or SIZE
    batch = i8_batch(args, size)
    k = n = size
    a = orc.corpus_i8(1, size * k)
    b = orc.corpus_i8(2, k * n)
    threads = host_threads(orc)

    def run(r):
        c = np.zeros(r * n, np.int32)
        orc.gemm_i8_blocked(a[:r * k], b, c, r, k, n, threads=threads)
        return c
    # One bounded sample per step, sized so the whole run stays near two minutes.
    per_step = max(0.2, min(3.0, 120.0 / (args.warmup + args.steps)))
    rows, dt, _ = sample_rows(size, run, 4 * per_step)
    steps = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        run(rows)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            steps.append(2.0 * rows * k * n / dt / 1e12)
    v = statistics.median(steps)
    base = {"value": v, "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"{rows} of {size} rows of one {size}^3 product per step ({dt:.2f} s), "
                      "blocked C restatement of gemm_auto's s8 path, OpenMP over rows"}
    line = {"impl": "reference", "metric": METRIC if size == SIZE else
            f"exact i8 GEMM TOPS at {size}^3 (bit-exact, int32 out)", "value": v, "unit": "TOPS",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (reference xorshift corpus)",
            "config": i8_line_config(size, batch, 3, world),
            "cpu_baseline": base,
            "e2e": {"value": v, "unit": "TOPS", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- main

def measure(w, args, U, torch, dist, ctx, stream, rank, world, local):
    elapsed, step_ms, clk = time_steps(w, ctx, stream, torch, dist, args.steps, args.warmup,
                                       local)
    value = world * args.steps * w.units / (elapsed / 1e3) / 1e12
    line = {
        "metric": w.metric, "value": value, "unit": w.unit, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps,
        "higher_is_better": True, "scaling": getattr(w, "scaling", "weak"), "vs_baseline": None,
        "dtype": w.dtype, "data": "synthetic (reference xorshift corpus)",
        "config": getattr(w, "full_config", None) or dict(
            w.config, n_total=w.config["n_per_gpu"] * (
                world if getattr(w, "scaling", "weak") == "weak" else 1), l2=w.l2,
            parallelism=getattr(w, "parallelism",
                                f"column blocks x{world}, no data-path collective")),
        "route": w.route.as_dict(),
        "roofline": w.roofline(statistics.mean(step_ms)),
        "cuda_graph": getattr(w, "graphed", False),
        "gpu_launches": w.launches * args.steps,
        "clocks": clk,
    }
    if getattr(w, "checked", None):
        line["checked"] = w.checked
    if getattr(w, "collective_ms", None) is not None:
        line["collective"] = w.collective_ms()
    if args.e2e_steps > 0 and w.e2e is not None:
        if dist:
            dist.barrier()
        r = w.e2e(args.e2e_steps, ctx, stream)
        ms = r.pop("ms")
        if dist:
            t = torch.tensor([ms], device="cuda", dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        line["e2e"] = dict(value=world * w.units / (ms / 1e3) / 1e12, unit=w.unit,
                           ms_per_step=ms, **r)
    else:
        line["e2e"] = None
    return line


def sub_line(fl, keys=("metric", "value", "unit", "ms_per_step", "steps", "warmup", "scaling",
                         "route", "roofline", "gpu_launches", "clocks", "config", "checked",
                         "collective", "e2e", "cpu_baseline")):
    return {k2: fl[k2] for k2 in keys if k2 in fl}


def main():
    args = parse()
    rank, world, local = env_rank()
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return

    import torch
    import uor_b200 as U

    torch.cuda.set_device(local)
    import uor_b200_dist as D
    # pinned host buffers of the e2e leg land in memory local to this GPU (first touch by a
    # thread on the GPU's NUMA node); the CPU baseline gets every core back below
    all_cpus = os.sched_getaffinity(0)
    D.bind_to_local_cpus(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=180))
    ctx = U.Context(local)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    ctx.set_stream(stream.cuda_stream)

    w = build_workload(args.workload, args, U, torch, rank, world)
    line = measure(w, args, U, torch, dist, ctx, stream, rank, world, local)
    if world == 1:
        os.sched_setaffinity(0, all_cpus)
    if rank == 0 and world == 1 and not args.no_cpu_baseline and w.cpu is not None:
        line["cpu_baseline"] = w.cpu(12.0, ctx)
    del w
    torch.cuda.empty_cache()

    def extra(build, steps, warmup=3, e2e_steps=0, cpu_budget=0.0):
        sub = argparse.Namespace(**vars(args))
        sub.steps, sub.warmup, sub.e2e_steps = steps, warmup, e2e_steps
        f = build()
        fl = measure(f, sub, U, torch, dist, ctx, stream, rank, world, local)
        if cpu_budget and rank == 0 and world == 1 and not args.no_cpu_baseline and f.cpu:
            fl["cpu_baseline"] = f.cpu(cpu_budget, ctx)
        del f
        torch.cuda.empty_cache()
        return sub_line(fl)

    headline = args.workload == "i8" and (args.size or SIZE) == SIZE
    # The metric's second half: exact f32 GEMM at 8192^3, on every rank's own columns.
    if headline and args.f32_steps > 0:
        line["f32_exact_8192"] = extra(lambda: wl_f32(args, U, torch, rank, SIZE, sets=1),
                                       args.f32_steps)
    if headline and not args.no_extras:
        # Multi-GPU paths at every N (strong scaling: the same total work at every N).
        line["i8_8192_sharded"] = extra(
            lambda: wl_i8_strong(args, U, torch, rank, world, dist), args.steps)
        line["wide_splitk"] = extra(
            lambda: wl_wide_splitk(args, U, torch, rank, world), max(args.steps, 20))
        line["trop_8192_sharded"] = extra(
            lambda: wl_trop_strong(args, U, torch, rank, world, dist), 6)
        if world == 1:
            # every other BASELINE config on the same GPU, each with its own bit-exact
            # row check against the oracle (the CPU leg)
            line["configs"] = {
                "configs[0] i8 512^3": extra(
                    lambda: wl_i8(args, U, torch, rank, 512, sets=1), 200, e2e_steps=20,
                    cpu_budget=2.0),
                "configs[1] codec 2048x8192x8192": extra(
                    lambda: wl_codec(args, U, torch, rank), 100, e2e_steps=3, cpu_budget=4.0),
                "configs[2] exact f32 4096^3": extra(
                    lambda: wl_f32(args, U, torch, rank, 4096), 60, e2e_steps=3,
                    cpu_budget=4.0),
                "configs[3] i32 -> i128 1024x65536x1024": extra(
                    lambda: wl_wide(args, U, torch, rank), 100, e2e_steps=3, cpu_budget=4.0),
                "configs[4] Trop<i8> 8192^3": extra(
                    lambda: wl_trop(args, U, torch, rank), 6, e2e_steps=1, cpu_budget=4.0),
            }

    ctx.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
