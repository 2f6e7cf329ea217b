#!/usr/bin/env python3
"""Benchmark of the B200 FP16 Linear path (one JSON line on rank 0).

Workload (per GPU): FP16 Linear Y = X W^T + b at M = N = K = 4096, X ~ N(0,1), W ~ N(0,1/K),
b = 0, FP32 accumulation, FP16 output -- the reference's headline square case. With N GPUs the
Linear is column-parallel: rank r owns W[r*4096:(r+1)*4096, :] and Y[:, r*4096:(r+1)*4096] of a
4096 x (4096*N) x 4096 problem, X is replicated and no collective touches the data path (weak
scaling, one process per GPU).

  value     whole-job TFLOP/s, inputs resident in HBM: K back-to-back launches of the tcgen05
            GEMM through b2_linear_run_device, timed with CUDA events on the launching stream,
            max over ranks. Four rotating X/W/Y sets (384 MiB) > 126 MiB L2, so every launch
            starts with cold L2.
  e2e       the same metric through co_linear_run with pinned HOST buffers: H2D of X, device
            finiteness scan, GEMM, status check, D2H of Y per step.
  roofline  GEMM kernel: 2*M*N*K FLOPs per launch / event-timed launch duration vs the measured
            dense 16-bit tensor peak; DRAM traffic per launch from the committed ncu summary.
  sharded   M=8192, N=16384, K=16384 over all ranks with the total fixed (strong scaling):
            column-parallel (no collective) and the K-split N=1024 variant (FP32 partials reduced
            by NCCL all-reduce / reduce-scatter, then the epilogue).
  gemv      M=1 decode projections of a SmolLM-135M-shaped layer (HBM GB/s per launch, weights
            rotated over > 4x L2).
  gemm_tile16  the same 4096^3 Linear with the reference's per-256-K FP16 running sum (the
            co_linear_* default numerics), device-resident like `value`.
  graph_ffn the SwiGLU FFN Y = X + Linear(SiLU(Linear(X, Wg, b)) * Linear(X, Wu), Wd) through the
            static graph compiler (co_graph_*) at m = d = h = 4096 and at m = 8 / m = 1: CO_CHAIN
            (fused gate·up GEMM + residual epilogue, one CUDA graph) against CO_SEPARATE, L2
            flushed between steps, plus co_graph_run end to end.
  cpu_baseline  the oracle's restatement of the reference arithmetic (per-256-K FP16 running
            sum, tile16_fast) on a bounded row sample, all host threads.

--impl reference  times only that CPU restatement on the same workload (rank 0; other ranks exit).
"""
import argparse
import ctypes
import importlib
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

M = N_PER_GPU = K = 4096
FLOPS_PER_GPU = 2 * M * N_PER_GPU * K
METRIC = "FP16 Linear TFLOP/s at 4096^3 + M=1 GEMV HBM GB/s, % of B200 peak, 1-8 GPUs"
WORKLOAD = ("FP16 Linear Y=XW^T+b, M=N=K=4096 per GPU, column-parallel over N (global N=4096*GPUs), "
            "X~N(0,1), W~N(0,1/K), b=0, FP32 accumulate, FP16 out")
GEMV_LAYER = [("q", 576, 576), ("k", 192, 576), ("v", 192, 576), ("o", 576, 576), ("gate", 1536, 576),
              ("up", 1536, 576), ("down", 576, 1536), ("lm_head", 49152, 576)]


def peaks():
    """(dense 16-bit burst TFLOP/s, sustained TFLOP/s, HBM GB/s, source)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        burst = float(p["bf16_tflops"])
        return burst, float(p.get("bf16_tflops_sustained", burst)), float(p["hbm_gbs"]), "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


def traffic_per_launch():
    """DRAM bytes (read + write) of one 4096^3 GEMM launch from the committed ncu summary."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return json.load(f).get("gemm_4096_fp32acc_bytes")
    except Exception:
        return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the timed region runs."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            pass
        self._stop = threading.Event()

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.02)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": len(self.samples),
                "source": "nvml" if self.ok else "unavailable"}


def cpu_sample(flops_target_s=10.0, max_rows=M):
    """Time the oracle's tile16 restatement on a row sample of the workload (all host threads)."""
    import numpy as np
    import oracle
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(1)
    w = oracle.Widened((rng.standard_normal((N_PER_GPU, K)) / np.sqrt(K)).astype(np.float16))
    b = np.zeros(N_PER_GPU, np.float16)
    rows = 16
    while True:
        x = rng.standard_normal((rows, K)).astype(np.float16)
        t0 = time.perf_counter()
        oracle.linear("tile16_fast", x, w, b, post=0, threads=threads)
        dt = time.perf_counter() - t0
        if dt >= flops_target_s or rows >= max_rows:
            break
        rows = min(max_rows, max(rows * 2, int(rows * flops_target_s / max(dt, 1e-3))))
    tflops = 2 * rows * N_PER_GPU * K / dt / 1e12
    return {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{rows} of {M} rows of X against the full W (N=K=4096), tile16_fast oracle, "
                      f"{dt:.2f} s"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    import numpy as np
    import oracle
    threads = os.cpu_count() or 1
    rng = np.random.default_rng(1)
    w = oracle.Widened((rng.standard_normal((N_PER_GPU, K)) / np.sqrt(K)).astype(np.float16))
    b = np.zeros(N_PER_GPU, np.float16)
    # size one step so the whole --steps/--warmup run stays near two minutes (<= 0.5 s a step)
    step_s = min(0.5, 120.0 / max(1, args.steps + args.warmup))
    rows = 16
    x = rng.standard_normal((rows, K)).astype(np.float16)
    t0 = time.perf_counter()
    oracle.linear("tile16_fast", x, w, b, post=0, threads=threads)
    dt = time.perf_counter() - t0
    rows = max(1, min(M, int(rows * step_s / max(dt, 1e-4))))
    x = rng.standard_normal((rows, K)).astype(np.float16)
    for _ in range(args.warmup):
        oracle.linear("tile16_fast", x, w, b, post=0, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.linear("tile16_fast", x, w, b, post=0, threads=threads)
    dt = (time.perf_counter() - t0) / args.steps
    value = 2 * rows * N_PER_GPU * K / dt / 1e12
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "m": M, "n_per_gpu": N_PER_GPU, "k": K,
                       "step": f"{rows} rows of X x full W per step (bounded sample)",
                       "parallelism": "none (host CPU)"},
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                             "sample": f"{rows} of {M} rows of X per step, tile16_fast oracle "
                                       f"(per-256-K FP16 running sum), {threads} threads"},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-gemv", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-sharded", action="store_true")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--graph-only", action="store_true", help="only the graph FFN section (diagnostics)")
    ap.add_argument("--graph-m", type=int, nargs="*", default=[4096, 8, 1], help="graph FFN row counts")
    ap.add_argument("--tile16-only", action="store_true", help="only the tile-16 GEMM section (diagnostics)")
    ap.add_argument("--linear-shape", type=int, nargs="+", metavar="M N K",
                    help="time tile-16 Linears of these shapes only, given as M N K triples (diagnostics)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import numpy as np
    import torch
    import torch.distributed as dist
    b2 = importlib.import_module("rockchip-npu-notes_b200")
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    warmup = max(3, args.warmup)
    steps = max(1, args.steps)
    peak_tflops, peak_sustained, peak_gbs, peak_src = peaks()

    fd = b2.open_device(local)
    stream = torch.cuda.ExternalStream(b2.lib().b2_get_stream(fd))
    gen = torch.Generator(device="cuda").manual_seed(1234 + rank)
    if args.linear_shape:   # diagnostics: Linear shapes (M N K triples), no headline line
        if len(args.linear_shape) % 3:
            raise SystemExit("--linear-shape takes M N K triples")
        for i in range(0, len(args.linear_shape), 3):
            m_, n_, k_ = args.linear_shape[i:i + 3]
            print(json.dumps({"linear_shape": bench_linear_shape(b2, fd, torch, stream, peak_tflops, peak_gbs, m_, n_,
                                                                 k_, args.steps)}), flush=True)
        b2.close(fd)
        return
    if args.tile16_only:   # diagnostics (profiling the tile-16 GEMM): no headline line
        print(json.dumps({"gemm_tile16": bench_tile16(b2, fd, torch, stream, peak_tflops, args.steps)}), flush=True)
        b2.close(fd)
        return
    if args.graph_only:   # diagnostics (profiling the graph section): no headline line
        print(json.dumps({"graph_ffn": bench_graph(b2, fd, torch, stream, peak_tflops, peak_gbs, args.graph_m)}),
              flush=True)
        b2.close(fd)
        return

    # ---------------------------------------------------------------- device-resident timing
    sets = []
    for s in range(4):
        x = torch.randn(M, K, device="cuda", dtype=torch.float32, generator=gen).half()
        w = (torch.randn(N_PER_GPU, K, device="cuda", dtype=torch.float32, generator=gen) / K ** 0.5).half()
        y = torch.empty(M, N_PER_GPU, device="cuda", dtype=torch.float16)
        op = b2.Linear(fd, M, K, N_PER_GPU, w.cpu().numpy(), np.zeros(N_PER_GPU, np.float16),
                       post=b2.CO_LINEAR_NONE, mode=b2.CO_CHAIN, acc=b2.ACC_FP32, compat=False)
        sets.append((x, w, y, op))
    torch.cuda.synchronize()

    def step(i):
        x, _, y, op = sets[i % 4]
        op.run_device(M, x.data_ptr(), K, y.data_ptr(), N_PER_GPU)

    for i in range(warmup):
        step(i)
    b2.sync(fd)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    launches0 = b2.counters()["launches"]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for i in range(steps):
            step(i)
        end.record(stream)
        end.synchronize()
    gpu_launches = b2.counters()["launches"] - launches0
    if b2.status(fd):
        raise RuntimeError("device status raised during the timed region")
    ms = start.elapsed_time(end) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    torch.cuda.synchronize()
    value = world * FLOPS_PER_GPU / (ms * 1e-3) / 1e12
    kernel_tflops = FLOPS_PER_GPU / (ms * 1e-3) / 1e12

    # correctness spot check of the timed configuration (sampled rows vs the FP64 oracle)
    import oracle
    x0, w0, y0, _ = sets[0]
    rows = torch.arange(0, M, 257, device="cuda")
    ref = oracle.linear("fp64", x0[rows].cpu().numpy(), w0.cpu().numpy(), np.zeros(N_PER_GPU, np.float16),
                        post=0, want=("act",))["act"]
    ok, worst = oracle.tolerance_ok(y0[rows].cpu().numpy(), ref)
    if not ok:
        raise RuntimeError(f"bench output outside tolerance (worst err/tol {worst:.3f})")
    gi = sets[0][3].info()
    kernel_desc = (f"tcgen05 persistent GEMM, {gi.tile_m}x{gi.tile_n} output tile per "
                   f"{'CTA pair (cta_group::2)' if gi.tile_m == 256 else 'CTA'}, K step {gi.tile_k}, "
                   f"{gi.stages}-stage TMA ring, {gi.grid} CTAs")
    for _, _, _, op in sets:
        op.destroy()
    del sets

    # ---------------------------------------------------------------- end to end (host buffers)
    op = b2.Linear(fd, M, K, N_PER_GPU, w0.cpu().numpy(), np.zeros(N_PER_GPU, np.float16),
                   post=b2.CO_LINEAR_NONE, mode=b2.CO_CHAIN, acc=b2.ACC_FP32, compat=True)
    hx = b2.lib().b2_host_alloc(M * K * 2)
    hy = b2.lib().b2_host_alloc(M * N_PER_GPU * 2)
    xh = np.ctypeslib.as_array(ctypes.cast(hx, ctypes.POINTER(ctypes.c_uint16)), shape=(M, K))
    xh[:] = x0.cpu().numpy().view(np.uint16)
    e2e_steps = max(3, min(steps, 200))
    for _ in range(3):
        b2.check("co_linear_run", b2.lib().co_linear_run(op.h, hx, hy))
    if world > 1:
        dist.barrier()
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    es.record(stream)
    for _ in range(e2e_steps):
        b2.check("co_linear_run", b2.lib().co_linear_run(op.h, hx, hy))
    ee.record(stream)
    ee.synchronize()
    e2e_ms = es.elapsed_time(ee) / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    op.destroy()
    b2.lib().b2_host_free(hx)
    b2.lib().b2_host_free(hy)

    # ---------------------------------------------------------------- M=8192,N=16384,K=16384 (all ranks)
    shard = None
    if not args.no_sharded:
        shard = bench_sharded(b2, fd, torch, dist, stream, world, rank, peak_tflops, warmup, steps)

    # ---------------------------------------------------------------- GEMV (rank 0, N=1 only)
    gemv = None
    if rank == 0 and world == 1 and not args.no_gemv:
        gemv = bench_gemv(b2, fd, torch, stream, peak_gbs)

    # ---------------------------------------------------------------- tile-16 GEMM (rank 0, N=1 only)
    tile16 = None
    if rank == 0 and world == 1:
        tile16 = bench_tile16(b2, fd, torch, stream, peak_tflops, min(steps, 400))

    # ---------------------------------------------------------------- graph FFN (rank 0, N=1 only)
    graph = None
    if rank == 0 and world == 1 and not args.no_graph:
        graph = bench_graph(b2, fd, torch, stream, peak_tflops, peak_gbs, args.graph_m)

    line = None
    if rank == 0:
        traffic = traffic_per_launch()
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "m": M, "n_per_gpu": N_PER_GPU, "k": K,
                       "accumulate": "fp32", "kernel": kernel_desc,
                       "l2": "inputs larger than L2: 4 rotating X/W/Y sets of 96 MiB",
                       "parallelism": f"column-parallel x{world}, no collective"},
            "e2e": {"value": world * FLOPS_PER_GPU / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
                    "ms_per_step": e2e_ms, "api": "co_linear_run (pinned host X/Y)",
                    "h2d_bytes_per_step": M * K * 2, "d2h_bytes_per_step": M * N_PER_GPU * 2},
            "roofline": {"bound": "tensor", "achieved": kernel_tflops, "peak": peak_tflops, "unit": "TFLOP/s",
                         "frac": kernel_tflops / peak_tflops, "traffic": traffic,
                         "peak_source": f"{peak_src} dense 16-bit (cuBLAS bf16 burst)",
                         "frac_of_sustained": kernel_tflops / peak_sustained,
                         "peak_sustained": peak_sustained,
                         "algorithmic_flops_per_launch": FLOPS_PER_GPU},
            "gpu_launches": gpu_launches,
            "clocks": clocks.summary(),
            "spot_check": {"rows": int(rows.numel()), "worst_err_over_tol_vs_fp64": worst},
        }
        if shard:
            line["sharded"] = shard
        if gemv:
            line["gemv"] = gemv
        if tile16:
            line["gemm_tile16"] = tile16
        if graph:
            line["graph_ffn"] = graph
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_sample()
    b2.close(fd)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if line:
        print(json.dumps(line), flush=True)


def _timed_steps(torch, dist, world, stream, fn, warmup, steps, flush=None):
    """Mean device ms of `fn` over `steps` (per-step CUDA events on `stream`; an optional L2 flush
    between steps, outside the events), max over ranks."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    pairs = []
    with ClockSampler(torch.cuda.current_device()) as clocks:
        for _ in range(steps):
            if flush is not None:
                # on the launching stream, before the start event: write a buffer larger than L2, then
                # read one (so the timed launch starts with a cold L2 that holds no dirty lines whose
                # write-back it would pay for)
                with torch.cuda.stream(stream):
                    flush.zero_()
                    flush.view(torch.float32).sum()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            fn()
            e.record(stream)
            pairs.append((s, e))
        torch.cuda.synchronize()
    ms = sum(s.elapsed_time(e) for s, e in pairs) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms, clocks.summary()


def bench_sharded(b2, fd, torch, dist, stream, world, rank, peak_tflops, warmup, steps):
    """Large sharded Linear M=8192, N=16384, K=16384 (X~N(0,1), W~N(0,1/K), no bias, FP32 accumulate)
    over all ranks with the total work fixed (strong scaling): column-parallel over N with no
    collective, and the K-split variant N=1024 (FP32 partial -> NCCL all-reduce or reduce-scatter
    over NVLink -> bias/activation epilogue). Every rank runs every step; max over ranks."""
    import numpy as np
    import oracle
    sharded = importlib.import_module("rockchip-npu-notes_b200.sharded")
    m, n, k, n_ks = 8192, 16384, 16384, 1024
    l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    flush = torch.empty(2 * l2 // 4, dtype=torch.float32, device="cuda")
    out = {}
    gen = torch.Generator(device="cuda")

    def w_rows(n0, n1, seed):
        """Rows [n0, n1) of a W whose 256-row blocks are seeded by block index (rank-independent)."""
        blocks = []
        for b0 in range(n0 - n0 % 256, n1, 256):
            gen.manual_seed(seed + b0 // 256)
            blk = torch.randn(256, k, device="cuda", generator=gen) / k ** 0.5
            blocks.append(blk[max(n0 - b0, 0):min(n1 - b0, 256)].half())
        return torch.cat(blocks).cpu().numpy()

    gen.manual_seed(77)
    x = torch.randn(m, k, device="cuda", generator=gen).half()
    torch.cuda.synchronize()

    # ---- column-parallel: rank r owns W[n0:n1], writes Y[:, n0:n1]; X replicated
    col = sharded.ColumnShard(fd, 1, n, k, lambda a, b: w_rows(a, b, 9000), None, world, rank)
    cols = col.n1 - col.n0
    y = torch.empty(m, max(cols, 8), device="cuda", dtype=torch.float16)
    csteps = max(5, min(steps, 40))
    ms, clk = _timed_steps(torch, dist, world, stream,
                           lambda: col.run_device(m, x.data_ptr(), k, y.data_ptr(), y.shape[1]), 3, csteps)
    if b2.status(fd):
        raise RuntimeError("device status raised in the column-parallel run")
    flops = 2 * m * n * k
    worst = 0.0
    if cols:
        c = min(cols, 512)
        rows = torch.tensor([0, 2049, 5000, m - 1], device="cuda")
        w_chk = w_rows(col.n0, col.n0 + c, 9000)
        ref = oracle.linear("fp64", x[rows].cpu().numpy(), w_chk, None, post=0, want=("act",))["act"]
        ok, worst = oracle.tolerance_ok(y[rows, :c].cpu().numpy(), ref)
        if not ok:
            raise RuntimeError(f"column-parallel output outside tolerance ({worst:.3f})")
    col.destroy()
    del y
    tflops = flops / (ms * 1e-3) / 1e12
    out["column_parallel"] = {
        "m": m, "n": n, "k": k, "scaling": "strong", "collective": None, "ms_per_step": ms, "steps": csteps,
        "tflops": tflops, "tflops_per_gpu": tflops / world, "frac_per_gpu": tflops / world / peak_tflops,
        "columns_per_gpu": cols, "worst_err_over_tol_vs_fp64": worst, "clocks_rank0": clk,
        "l2": "inputs larger than L2 (X 256 MiB + W and Y blocks)"}

    # ---- K-split N=1024: rank r owns X[:, k0:k1], W[:, k0:k1]; FP32 partial reduced over NVLink
    w_ks = w_rows(0, n_ks, 20000)
    ks = sharded.KSplitLinear(fd, m, w_ks, None, world, rank, torch, dist)
    kk = max(ks.k1 - ks.k0, 8)
    xs = x[:, ks.k0:ks.k0 + kk].contiguous() if ks.k1 > ks.k0 else torch.zeros(m, 8, device="cuda").half()
    y = torch.zeros(m, n_ks, device="cuda", dtype=torch.float16)
    torch.cuda.synchronize()
    flops = 2 * m * n_ks * k
    collectives = ["all_reduce", "reduce_scatter"] if world > 1 else ["none"]
    ksteps = max(10, min(steps, 100))
    for coll in collectives:
        name = "all_reduce" if coll == "none" else coll

        def fn():
            ks.forward(m, xs.data_ptr(), kk, y.data_ptr(), n_ks, collective=name)

        with torch.cuda.stream(stream):
            y.zero_()
            ms, clk = _timed_steps(torch, dist, world, stream, fn, 3, ksteps, flush=flush)
        if b2.status(fd):
            raise RuntimeError("device status raised in the K-split run")
        r0, r1 = (0, m) if coll != "reduce_scatter" else ks.row_shard(m)
        rows = torch.tensor(sorted({r0, (r0 + r1) // 2, r1 - 1}), device="cuda")
        ref = oracle.linear("fp64", x[rows].cpu().numpy(), w_ks, None, post=0, want=("act",))["act"]
        ok, worst = oracle.tolerance_ok(y[rows].cpu().numpy(), ref)
        if not ok:
            raise RuntimeError(f"K-split ({coll}) output outside tolerance ({worst:.3f})")
        tflops = flops / (ms * 1e-3) / 1e12
        partial_bytes = m * ks.ldp * 4
        out[f"k_split_{coll}"] = {
            "m": m, "n": n_ks, "k": k, "scaling": "strong", "collective": None if coll == "none" else coll,
            "ms_per_step": ms, "steps": ksteps, "tflops": tflops, "tflops_per_gpu": tflops / world,
            "frac_per_gpu": tflops / world / peak_tflops, "k_per_gpu": ks.k1 - ks.k0,
            "fp32_partial_bytes": partial_bytes, "worst_err_over_tol_vs_fp64": worst, "clocks_rank0": clk,
            "l2": "flushed between steps (write of 2x L2, outside the events)"}
    ks.destroy()

    # fused K-split: partial row blocks stored into their owner's memory by the GEMM epilogue
    # (NVLink), round signal, owner reduction + epilogue (b2_ksplit_*)
    fk = sharded.FusedKSplit(fd, m, w_ks, None, world, rank, torch, dist)
    y.zero_()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ms, clk = _timed_steps(torch, dist, world, stream,
                               lambda: fk.run(m, xs.data_ptr(), kk, y.data_ptr(), n_ks), 3, ksteps, flush=flush)
    if b2.status(fd):
        raise RuntimeError("device status raised in the fused K-split run")
    r0, r1 = fk.rows(m)
    rows = torch.tensor(sorted({r0, (r0 + r1) // 2, r1 - 1}), device="cuda")
    ref = oracle.linear("fp64", x[rows].cpu().numpy(), w_ks, None, post=0, want=("act",))["act"]
    ok, worst = oracle.tolerance_ok(y[rows].cpu().numpy(), ref)
    if not ok:
        raise RuntimeError(f"fused K-split output outside tolerance ({worst:.3f})")
    tflops = flops / (ms * 1e-3) / 1e12
    out["k_split_fused"] = {
        "m": m, "n": n_ks, "k": k, "scaling": "strong",
        "collective": "GEMM epilogue stores to the owner over NVLink + signal + owner reduction (b2_ksplit_run)",
        "ms_per_step": ms, "steps": ksteps, "tflops": tflops, "tflops_per_gpu": tflops / world,
        "frac_per_gpu": tflops / world / peak_tflops, "k_per_gpu": fk.k1 - fk.k0, "rows_per_gpu": r1 - r0,
        "worst_err_over_tol_vs_fp64": worst, "clocks_rank0": clk,
        "l2": "flushed between steps (write of 2x L2, outside the events)"}
    fk.destroy()
    del x, xs, y, flush
    torch.cuda.empty_cache()
    return out


def bench_tile16(b2, fd, torch, stream, peak_tflops, steps):
    """The same 4096^3 Linear with the reference's own numerics (per-256-K FP16 running sum,
    co_linear_create's default; the headline uses FP32 accumulation): 4 rotating X/W/Y sets,
    back-to-back b2_linear_run_device launches timed with CUDA events on the launching stream."""
    import numpy as np
    gen = torch.Generator(device="cuda").manual_seed(77)
    sets = []
    for _ in range(4):
        x = torch.randn(M, K, device="cuda", generator=gen).half()
        w = (torch.randn(N_PER_GPU, K, device="cuda", generator=gen) / K ** 0.5).half()
        y = torch.empty(M, N_PER_GPU, device="cuda", dtype=torch.float16)
        op = b2.Linear(fd, M, K, N_PER_GPU, w.cpu().numpy(), np.zeros(N_PER_GPU, np.float16),
                       post=b2.CO_LINEAR_NONE, mode=b2.CO_CHAIN, acc=b2.ACC_TILE16, compat=False)
        sets.append((x, y, op))
    torch.cuda.synchronize()

    def step(i):
        x, y, op = sets[i % 4]
        op.run_device(M, x.data_ptr(), K, y.data_ptr(), N_PER_GPU)

    for i in range(5):
        step(i)
    b2.sync(fd)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        s.record(stream)
        for i in range(steps):
            step(i)
        e.record(stream)
        e.synchronize()
    if b2.status(fd):
        raise RuntimeError("device status raised in the tile-16 GEMM")
    ms = s.elapsed_time(e) / steps
    tflops = FLOPS_PER_GPU / (ms * 1e-3) / 1e12
    for _, _, op in sets:
        op.destroy()
    return {"ms": ms, "tflops": tflops, "frac": tflops / peak_tflops, "steps": steps,
            "numerics": "per-256-K FP16 running sum (co_linear_create default)", "clocks": clocks.summary()}


def bench_linear_shape(b2, fd, torch, stream, peak_tflops, peak_gbs, m, n, k, steps):
    """Diagnostics: one tile-16 Linear [m, k] x [n, k]^T through b2_linear_run_device, weights
    rotated over >= 4x L2 (so every launch streams W from HBM), back-to-back launches timed with
    CUDA events on the launching stream."""
    import numpy as np
    l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    wbytes = 2 * n * k
    copies = max(2, min(64, -(-4 * l2 // wbytes)))
    w = (np.random.default_rng(n + k).standard_normal((n, k), np.float32) / np.sqrt(k)).astype(np.float16)
    ops = [b2.Linear(fd, m, k, n, w, None, post=b2.CO_LINEAR_NONE, mode=b2.CO_CHAIN, acc=b2.ACC_TILE16, compat=False)
           for _ in range(copies)]
    x = torch.randn(m, k, device="cuda").half()
    y = torch.empty(m, n, device="cuda", dtype=torch.float16)
    for op in ops:
        op.run_device(m, x.data_ptr(), k, y.data_ptr(), n)
    b2.sync(fd)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for i in range(steps):
        ops[i % copies].run_device(m, x.data_ptr(), k, y.data_ptr(), n)
    e.record(stream)
    e.synchronize()
    if b2.status(fd):
        raise RuntimeError("device status raised in the linear-shape run")
    ms = s.elapsed_time(e) / steps
    info = ops[0].info()
    for op in ops:
        op.destroy()
    return {"m": m, "n": n, "k": k, "us": ms * 1e3, "tflops": 2 * m * n * k / (ms * 1e-3) / 1e12,
            "weight_gb_s": wbytes / (ms * 1e-3) / 1e9, "frac_of_hbm": wbytes / (ms * 1e-3) / 1e9 / peak_gbs,
            "kernel": "gemv" if info.kernel == 1 else "gemm", "weight_copies": copies}


def bench_graph(b2, fd, torch, stream, peak_tflops, peak_gbs, rows=(4096, 8, 1)):
    """The SwiGLU FFN of the reference's graph CLI (research/custom-ops/tools/c/graph_cli.c:67-74),
    Y = X + Linear(SiLU(Linear(X, Wg, b)) * Linear(X, Wu), Wd), through the static graph compiler
    (co_graph_*) at the reference graph API's largest shape (m = d = h = 4096) and at decode (m = 8,
    m = 1). Device-resident: b2_graph_launch timed with CUDA events per step, L2 flushed between steps,
    in CO_CHAIN (gate·up pair as ONE tcgen05 GEMM with the SiLU product in its epilogue, the residual
    in the down projection's epilogue, replayed as one CUDA graph) and CO_SEPARATE (one kernel per node,
    Linear = GEMM + separate epilogue). End to end: co_graph_run with pinned host X / Y. Rows of Y are
    checked against the oracle (every node with the reference's arithmetic)."""
    import numpy as np
    import oracle
    G = importlib.import_module("rockchip-npu-notes_b200.graph")
    l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    flush = torch.empty(2 * l2, dtype=torch.uint8, device="cuda")
    d = h = 4096
    rng = np.random.default_rng(4096)
    wg = (rng.standard_normal((h, d), np.float32) / 64).astype(np.float16)
    wu = (rng.standard_normal((h, d), np.float32) / 64).astype(np.float16)
    wd = (rng.standard_normal((d, h), np.float32) / 64).astype(np.float16)
    bias = (rng.standard_normal(h, np.float32) * 0.1).astype(np.float16)
    out = {"d": d, "h": h, "timing": "b2_graph_launch, CUDA events per step, L2 flushed between steps",
           "cases": {}}
    for m in rows:
        x = (np.random.default_rng(m).standard_normal((m, d), np.float32) * 0.7).astype(np.float16)
        nodes, o = G.swiglu_ffn(m, d, h, wg, wu, wd, bias)
        flops = 6 * m * d * h
        wbytes = 3 * d * h * 2
        case, ys = {"m": m, "flops": flops}, {}
        for name, mode in (("chain", b2.CO_CHAIN), ("separate", b2.CO_SEPARATE)):
            g = G.Graph(fd, nodes, o, mode, budget=4 << 30)
            ys[name] = g.run({0: x})
            steps = 30 if m > 8 else 200
            ms, clocks = _timed_steps(torch, None, 1, stream, g.launch, 3, steps, flush)
            b2.sync(fd)
            if g.status():
                raise RuntimeError(f"graph FFN m={m} {name}: device status raised")
            info = g.info()
            case[name] = {"ms": ms, "tflops": flops / (ms * 1e-3) / 1e12, "kernels": info["kernels"],
                          "cuda_graph": bool(info["captured"]), "gated_fused": info["gated"],
                          "residual_fused": info["residual"], "clocks": clocks}
            if m <= 8:
                case[name]["weight_gb_s"] = wbytes / (ms * 1e-3) / 1e9
                case[name]["frac_of_hbm"] = wbytes / (ms * 1e-3) / 1e9 / peak_gbs
            else:
                case[name]["frac_of_peak"] = flops / (ms * 1e-3) / 1e12 / peak_tflops
            if name == "chain":
                hx = b2.lib().b2_host_alloc(m * d * 2)
                hy = b2.lib().b2_host_alloc(m * d * 2)
                xh = np.ctypeslib.as_array(ctypes.cast(hx, ctypes.POINTER(ctypes.c_uint16)), shape=(m, d))
                yh = np.ctypeslib.as_array(ctypes.cast(hy, ctypes.POINTER(ctypes.c_uint16)), shape=(m, d))
                xh[:] = x.view(np.uint16)
                for _ in range(3):
                    rc, _ = g.run_rc({0: xh.view(np.float16)}, {o: yh.view(np.float16)})
                    b2.check("co_graph_run_many", rc)
                reps = 10 if m > 8 else 100
                es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                es.record(stream)
                for _ in range(reps):
                    g.run_rc({0: xh.view(np.float16)}, {o: yh.view(np.float16)})
                ee.record(stream)
                ee.synchronize()
                e2e = es.elapsed_time(ee) / reps
                case["e2e"] = {"ms": e2e, "tflops": flops / (e2e * 1e-3) / 1e12, "api": "co_graph_run (pinned host X/Y)",
                               "h2d_bytes_per_step": m * d * 2, "d2h_bytes_per_step": m * d * 2}
                b2.lib().b2_host_free(hx)
                b2.lib().b2_host_free(hy)
            g.destroy()
        if not np.array_equal(ys["chain"].view(np.uint16), ys["separate"].view(np.uint16)):
            raise RuntimeError(f"graph FFN m={m}: CO_CHAIN and CO_SEPARATE differ")
        rows = np.arange(0, m, max(1, m // 4))[:4]
        t0 = time.time()
        ref = oracle.ffn(x[rows], wg, wu, wd, bias)
        cpu_s = time.time() - t0
        ok, worst = oracle.tolerance_ok(ys["chain"][rows], ref)
        if not ok:
            raise RuntimeError(f"graph FFN m={m} outside tolerance (worst err/tol {worst:.3f})")
        case["spot_check"] = {"rows": int(rows.size), "worst_err_over_tol": worst,
                              "chain_equals_separate": True}
        case["cpu_oracle"] = {"rows": int(rows.size), "s": cpu_s, "kind": "port",
                              "tflops": 6 * rows.size * d * h / cpu_s / 1e12, "cores": os.cpu_count()}
        out["cases"][str(m)] = case
    del flush
    return out


def _eager_and_graph_ms(torch, stream, launch, reps):
    """Mean ms per call of launch(i), i = 0..reps-1, issued eagerly and as one replayed CUDA graph
    (a decode step runs as a graph: no host launch overhead between kernels)."""
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for i in range(reps):
        launch(i)
    e.record(stream)
    e.synchronize()
    eager = s.elapsed_time(e) / reps
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for i in range(reps):
            launch(i)
    best = None
    with torch.cuda.stream(stream):          # replay() launches on the current stream
        g.replay()
        stream.synchronize()
        for _ in range(3):
            s.record(stream)
            g.replay()
            e.record(stream)
            e.synchronize()
            t = s.elapsed_time(e) / reps
            best = t if best is None else min(best, t)
    del g
    return eager, best


def bench_gemv(b2, fd, torch, stream, peak_gbs):
    """M=1 projections of a SmolLM-135M-shaped layer, weights rotated over >= 4x L2; each timed as
    eager launches and as a replayed CUDA graph of the same launches (the headline per projection)."""
    import numpy as np
    l2 = torch.cuda.get_device_properties(torch.cuda.current_device()).L2_cache_size
    out = {"l2_bytes": l2, "timing": "CUDA graph of back-to-back launches (us, gb_s); eager_us beside it",
           "projections": {}}
    layer_bytes, layer_ms = 0, 0.0
    gen = torch.Generator(device="cuda").manual_seed(7)
    for name, n, k in GEMV_LAYER:
        wbytes = 2 * n * k
        copies = min(2048, max(2, -(-4 * l2 // wbytes)))
        w_host = (np.random.default_rng(n * k).standard_normal((n, k)) * 0.02).astype(np.float16)
        # one operator per weight copy (same values, distinct HBM buffers): copies*bytes >= 4x L2
        ops = [b2.Linear(fd, 1, k, n, w_host, None, post=b2.CO_LINEAR_NONE, acc=b2.ACC_FP32, compat=False)
               for _ in range(copies)]
        x = torch.randn(1, k, device="cuda", generator=gen).half()
        y = torch.empty(1, n, device="cuda", dtype=torch.float16)
        torch.cuda.synchronize()
        for op in ops:
            op.run_device(1, x.data_ptr(), k, y.data_ptr(), n)
        b2.sync(fd)
        reps = max(64, min(4 * copies, 2048))
        eager, ms = _eager_and_graph_ms(
            torch, stream, lambda i: ops[i % copies].run_device(1, x.data_ptr(), k, y.data_ptr(), n), reps)
        if b2.status(fd):
            raise RuntimeError(f"device status raised in the {name} GEMV")
        nbytes = 2 * n * k + 2 * k + 2 * n
        gbs = nbytes / (ms * 1e-3) / 1e9
        out["projections"][name] = {"n": n, "k": k, "bytes": nbytes, "us": ms * 1e3, "gb_s": gbs,
                                    "frac": gbs / peak_gbs, "eager_us": eager * 1e3, "weight_copies": copies,
                                    "kernel": "streamed (bulk-copy ring, mma.sync)" if k <= 2048 else "per-lane"}
        if name != "lm_head":
            layer_bytes += nbytes
            layer_ms += ms
        for op in ops:
            op.destroy()
    out["layer_7_projections"] = {"bytes": layer_bytes, "us": layer_ms * 1e3,
                                  "gb_s": layer_bytes / (layer_ms * 1e-3) / 1e9,
                                  "frac": layer_bytes / (layer_ms * 1e-3) / 1e9 / peak_gbs,
                                  "launches": 7}

    # the same 7 projections as ONE grouped launch (b2_linear_group_run_device); q/k/v/gate/up read
    # one shared input, o and down their own; weight sets rotated over >= 4x L2
    layer = [(name, n, k) for name, n, k in GEMV_LAYER if name != "lm_head"]
    set_bytes = sum(2 * n * k for _, n, k in layer)
    copies = min(256, max(2, -(-4 * l2 // set_bytes)))
    rng = np.random.default_rng(5)
    w_host = {name: (rng.standard_normal((n, k)) * 0.02).astype(np.float16) for name, n, k in layer}
    sets = [[b2.Linear(fd, 1, k, n, w_host[name], None, post=b2.CO_LINEAR_NONE, acc=b2.ACC_FP32, compat=False)
             for name, n, k in layer] for _ in range(copies)]
    xin = {"h": torch.randn(1, 576, device="cuda", generator=gen).half(),
           "o": torch.randn(1, 576, device="cuda", generator=gen).half(),
           "f": torch.randn(1, 1536, device="cuda", generator=gen).half()}
    src = {"q": "h", "k": "h", "v": "h", "gate": "h", "up": "h", "o": "o", "down": "f"}
    ys = [torch.empty(1, n, device="cuda", dtype=torch.float16) for _, n, _ in layer]
    xp = [xin[src[name]].data_ptr() for name, _, _ in layer]
    ldx = [k for _, _, k in layer]
    yp = [y.data_ptr() for y in ys]
    ldy = [n for _, n, _ in layer]
    torch.cuda.synchronize()
    for ops in sets:
        b2.group_run_device(ops, 1, xp, ldx, yp, ldy)
    b2.sync(fd)
    reps = max(64, 4 * copies)
    launches0 = b2.counters()["launches"]
    b2.group_run_device(sets[0], 1, xp, ldx, yp, ldy)
    group_launches = b2.counters()["launches"] - launches0
    eager, ms = _eager_and_graph_ms(torch, stream, lambda i: b2.group_run_device(sets[i % copies], 1, xp, ldx, yp, ldy),
                                    reps)
    if b2.status(fd):
        raise RuntimeError("device status raised in the grouped GEMV run")
    gbytes = sum(2 * n * k + 2 * k + 2 * n for _, n, k in layer)
    out["layer_7_projections_grouped"] = {"bytes": gbytes, "us": ms * 1e3, "gb_s": gbytes / (ms * 1e-3) / 1e9,
                                          "frac": gbytes / (ms * 1e-3) / 1e9 / peak_gbs, "eager_us": eager * 1e3,
                                          "launches": group_launches, "weight_sets": copies}
    for ops in sets:
        for op in ops:
            op.destroy()
    out["peak_gbs"] = peak_gbs
    return out


if __name__ == "__main__":
    main()
