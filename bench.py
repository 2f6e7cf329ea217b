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
            by NCCL all-reduce / reduce-scatter, then the epilogue; or fused: the GEMM epilogue
            stores each row block into its owner's memory over NVLink, with per-phase times).
            K-split steps start together on every rank (one-element NCCL all-reduce first).
  gemv      M=1 decode projections of a SmolLM-135M-shaped layer (HBM GB/s per launch, weights
            rotated over > 4x L2): each alone, the layer's 7 as one grouped launch, all 8 with the
            LM head as one grouped launch and as a decode step's dependent chain in one CUDA
            graph, and long-K decode shapes (4096x4096, 11008x4096, 4096x11008).
  cfg1      the fused HardSigmoid at M=64, N=256, K=512 (the reference CLI's operator): device,
            CUDA-graph and end-to-end microseconds, beside the CPU oracle (C port, all threads)
            and the pure-Python form of the reference's file-gate oracle.
  cube_entry co_linear_run_tiled at 4096^3 with 16 x 16 input cube views and 256 output cubes (the
            GEMM reads and writes the cubes directly) beside b2_linear_run_device on row-major buffers.
  summary   the key figures of all sections, printed last so that a truncated log keeps them.
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
    ap.add_argument("--rk-plan-only", action="store_true", help="only the plan-ABI section (diagnostics)")
    ap.add_argument("--cfg1-only", action="store_true", help="only the config-1 section (diagnostics)")
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
    if args.rk_plan_only:   # diagnostics (profiling the plan-ABI section): no headline line
        print(json.dumps({"rk_plan": bench_rk_plan(b2, fd, args.steps)}), flush=True)
        b2.close(fd)
        return
    if args.cfg1_only:   # diagnostics (profiling the config-1 operator): no headline line
        print(json.dumps({"cfg1": bench_cfg1(b2, fd, torch, stream, args.steps)}), flush=True)
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

    # ---------------------------------------------------------------- config 1 (rank 0, N=1 only)
    cfg1 = None
    if rank == 0 and world == 1:
        cfg1 = bench_cfg1(b2, fd, torch, stream, steps)

    # ---------------------------------------------------------------- cube entry (rank 0, N=1 only)
    cube = None
    if rank == 0 and world == 1:
        cube = bench_cube(b2, fd, torch, stream, steps)

    # ---------------------------------------------------------------- plan ABI (rank 0, N=1 only)
    rkp = None
    if rank == 0 and world == 1:
        try:
            rkp = bench_rk_plan(b2, fd, steps)
        except Exception as e:   # a secondary surface: report it, keep the line
            rkp = {"error": f"{type(e).__name__}: {e}"}

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
        # detail first, then the compact summary last (what a truncated log tail still shows)
        if graph:
            line["graph_ffn"] = graph
        if tile16:
            line["gemm_tile16"] = tile16
        if gemv:
            line["gemv"] = gemv
        if shard:
            line["sharded"] = shard
        if cube:
            line["cube_entry"] = cube
        if cfg1:
            line["cfg1"] = cfg1
        if rkp:
            line["rk_plan"] = rkp
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_sample()
        line["summary"] = summarize(world, kernel_tflops, e2e_ms, tile16, cfg1, shard, gemv, graph, cube, rkp)
    b2.close(fd)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if line:
        print(json.dumps(line), flush=True)


def _r(v, digits=4):
    """Rounds to `digits` significant digits (None stays None)."""
    if v is None:
        return None
    return float(f"{v:.{digits}g}")


def summarize(world, kernel_tflops, e2e_ms, tile16, cfg1, shard, gemv, graph, cube=None, rkp=None):
    """The line's key figures in a few hundred bytes, printed as its last key."""
    out = {"n_gpus": world, "gemm_4096_fp32acc_tflops": _r(kernel_tflops), "e2e_ms": _r(e2e_ms)}
    if tile16:
        out["gemm_4096_tile16_tflops"] = _r(tile16["tflops"])
    if cube:
        out["cube_run_tiled_4096_ms"] = {"run_tiled": _r(cube["run_tiled_ms"]), "run_device": _r(cube["run_device_ms"])}
    if cfg1:
        out["cfg1_hsig_64x256x512_us"] = {"device": _r(cfg1["device_us"]), "graph": _r(cfg1["graph_us"]),
                                          "e2e": _r(cfg1["e2e_us"]), "cpu_c_port": _r(cfg1["cpu_c_port_us"]),
                                          "cpu_literal_s": _r(cfg1["cpu_oracle_literal_s"])}
    if rkp:
        out["rk_plan_hsig_64x256x512_e2e_us"] = _r(rkp["e2e_us"]) if "e2e_us" in rkp else rkp.get("error")
    if shard:
        cp = shard["column_parallel"]
        out["cfg5_8192x16384x16384_column_parallel"] = {"ms": _r(cp["ms_per_step"]),
                                                        "tflops_per_gpu": _r(cp["tflops_per_gpu"])}
        out["cfg5_ksplit_n1024_ms"] = {key[8:]: _r(v["ms_per_step"]) for key, v in shard.items()
                                       if key.startswith("k_split_")}
        phases = shard.get("k_split_fused", {}).get("phases_ms")
        if phases:
            out["cfg5_ksplit_fused_phases_ms"] = {key: _r(v) for key, v in phases.items()}
    if gemv:
        fr = {"set_8_grouped": gemv["set_8_grouped"]["frac"], "set_8_chain": gemv["set_8_decode_chain"]["frac"],
              "lm_head": gemv["projections"]["lm_head"]["frac"],
              "layer_7_grouped": gemv["layer_7_projections_grouped"]["frac"]}
        fr.update({key: v["frac"] for key, v in gemv["long_k"].items()})
        out["gemv_m1_frac_of_hbm"] = {key: _r(v, 3) for key, v in fr.items()}
        out["gemv_set_8_grouped_us"] = _r(gemv["set_8_grouped"]["us"])
    if graph:
        out["graph_ffn_chain_ms"] = {m: _r(c["chain"]["ms"]) for m, c in graph["cases"].items()}
    return out


def _timed_steps(torch, dist, world, stream, fn, warmup, steps, flush=None, align=False, after=None):
    """Mean device ms of `fn` over `steps` (per-step CUDA events on `stream`; an optional L2 flush
    between steps, outside the events), max over ranks. With `align` (steps that exchange data
    between ranks), each step's start event follows a one-element NCCL all-reduce on `stream`, so
    every rank's step starts when the slowest rank is ready: a rank's step time then holds its own
    work and the exchange, not another rank's L2 flush. `after(i)` runs on the host after step i
    (for per-step readouts; it may synchronise)."""
    token = torch.zeros(1, device="cuda") if align and world > 1 else None
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    pairs = []
    with ClockSampler(torch.cuda.current_device()) as clocks:
        for i in range(steps):
            if flush is not None:
                # on the launching stream, before the start event: write a buffer larger than L2, then
                # read one (so the timed launch starts with a cold L2 that holds no dirty lines whose
                # write-back it would pay for)
                with torch.cuda.stream(stream):
                    flush.zero_()
                    flush.view(torch.float32).sum()
            if token is not None:
                with torch.cuda.stream(stream):
                    dist.all_reduce(token)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            fn()
            e.record(stream)
            pairs.append((s, e))
            if after is not None:
                after(i)
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
            ms, clk = _timed_steps(torch, dist, world, stream, fn, 3, ksteps, flush=flush, align=True)
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
            "l2": "flushed between steps (write of 2x L2, outside the events)",
            "start": "ranks aligned by a one-element NCCL all-reduce before each step"}
    ks.destroy()

    # fused K-split: partial row blocks stored into their owner's memory by the GEMM epilogue
    # (NVLink), round signal, owner reduction + epilogue (b2_ksplit_*)
    fk = sharded.FusedKSplit(fd, m, w_ks, None, world, rank, torch, dist)
    y.zero_()
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        ms, clk = _timed_steps(torch, dist, world, stream,
                               lambda: fk.run(m, xs.data_ptr(), kk, y.data_ptr(), n_ks), 3, ksteps, flush=flush,
                               align=True)
    if b2.status(fd):
        raise RuntimeError("device status raised in the fused K-split run")
    # the same rounds again with phase events (GEMM + NVLink stores, signal, wait + reduction), read
    # after every step; mean per rank, then the max over ranks of each phase
    fk.set_timing(True)
    acc = [0.0, 0.0, 0.0]

    def read_phases(_i):
        for j, v in enumerate(fk.phase_ms()):
            acc[j] += v

    psteps = max(5, min(ksteps, 30))
    with torch.cuda.stream(stream):
        _timed_steps(torch, dist, world, stream, lambda: fk.run(m, xs.data_ptr(), kk, y.data_ptr(), n_ks), 2,
                     psteps, flush=flush, align=True, after=read_phases)
    fk.set_timing(False)
    phases = torch.tensor([v / psteps for v in acc], device="cuda")
    if world > 1:
        dist.all_reduce(phases, op=dist.ReduceOp.MAX)
    phases_ms = dict(zip(("gemm_and_stores", "signal", "wait_and_reduce"), phases.tolist()))
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
        "worst_err_over_tol_vs_fp64": worst, "clocks_rank0": clk, "phases_ms": phases_ms,
        "l2": "flushed between steps (write of 2x L2, outside the events)",
        "start": "ranks aligned by a one-element NCCL all-reduce before each step"}
    fk.destroy()
    del x, xs, y, flush
    torch.cuda.empty_cache()
    return out


def bench_cfg1(b2, fd, torch, stream, steps):
    """Fused FP16 HardSigmoid(X W^T + b) at M=64, N=256, K=512 (X ~ U(-1,1), W ~ U(-1/sqrt(K),
    1/sqrt(K)), b ~ U(-0.1,0.1), seed 0): the operator the reference's file CLI and host oracle run
    (research/custom-ops/tools/python/cli_gate.py:38-49). 16.8 MFLOP, so it is latency-bound and
    reported as absolute times, with the co_linear_* default numerics (per-256-K FP16 running sum):
      device_us  b2_linear_run_device, back-to-back launches on the library's stream (CUDA events)
      graph_us   the same launches replayed as one CUDA graph
      e2e_us     co_linear_hsig_run from pinned host X/Y (H2D, finiteness scan, GEMM, sync, status
                 check, D2H), CUDA events around the host calls
      cpu        the oracle's C restatement of the reference arithmetic (exact tile sums, all host
                 threads), and its pure-Python form of the file-gate oracle on one core (the same
                 per-element loop as cli_gate.oracle: math.fsum per 256-K tile, FP16 running sum)."""
    import numpy as np
    import oracle
    m, n, k = 64, 256, 512
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    w = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float16)
    b = rng.uniform(-0.1, 0.1, n).astype(np.float16)
    op = b2.Linear(fd, m, k, n, w, b, post=b2.CO_LINEAR_HSIG, mode=b2.CO_CHAIN, acc=b2.ACC_TILE16, compat=True)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(m, n, device="cuda", dtype=torch.float16)
    torch.cuda.synchronize()

    def launch(_i=0):
        op.run_device(m, xd.data_ptr(), k, yd.data_ptr(), n)

    for _ in range(10):
        launch()
    b2.sync(fd)
    reps = max(50, min(steps, 2000))
    eager, graph = _eager_and_graph_ms(torch, stream, launch, reps)
    if b2.status(fd):
        raise RuntimeError("device status raised in the config-1 run")
    ref = oracle.linear("tile16", x, w, b, post=1)["y16"]
    ok, worst = oracle.tolerance_ok(yd.cpu().numpy(), ref)
    if not ok:
        raise RuntimeError(f"config-1 output outside tolerance (worst err/tol {worst:.3f})")
    # end to end through the reference-facing entry, pinned host buffers
    hx = b2.lib().b2_host_alloc(m * k * 2)
    hy = b2.lib().b2_host_alloc(m * n * 2)
    xh = np.ctypeslib.as_array(ctypes.cast(hx, ctypes.POINTER(ctypes.c_uint16)), shape=(m, k))
    yh = np.ctypeslib.as_array(ctypes.cast(hy, ctypes.POINTER(ctypes.c_uint16)), shape=(m, n))
    xh[:] = x.view(np.uint16)
    run = b2.lib().co_linear_hsig_run
    for _ in range(10):
        b2.check("co_linear_hsig_run", run(op.h, hx, hy))
    e2e_reps = max(50, min(steps, 1000))
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    es.record(stream)
    for _ in range(e2e_reps):
        run(op.h, hx, hy)
    ee.record(stream)
    ee.synchronize()
    wall_us = (time.perf_counter() - t0) / e2e_reps * 1e6
    e2e_us = es.elapsed_time(ee) / e2e_reps * 1e3
    if not np.array_equal(yh, yd.cpu().numpy().view(np.uint16)):
        raise RuntimeError("config-1 host and device entries differ")
    b2.lib().b2_host_free(hx)
    b2.lib().b2_host_free(hy)
    op.destroy()
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    for _ in range(5):
        oracle.linear("tile16", x, w, b, post=1, threads=threads)
    c_s = (time.perf_counter() - t0) / 5
    xs, ws, bs = (a.astype(np.float64).ravel().tolist() for a in (x, w, b))
    t0 = time.perf_counter()
    oracle.linear_py(m, k, n, xs, ws, bs, post=1)
    py_s = time.perf_counter() - t0
    flops = 2 * m * n * k
    return {"m": m, "n": n, "k": k, "op": "HardSigmoid(XW^T+b), tile-16 numerics", "device_us": eager * 1e3,
            "graph_us": graph * 1e3, "e2e_us": e2e_us, "e2e_wall_us": wall_us,
            "device_tflops": flops / (graph * 1e-3) / 1e12, "worst_err_over_tol_vs_oracle": worst,
            "cpu_c_port_us": c_s * 1e6, "cpu_c_port_threads": threads, "cpu_oracle_literal_s": py_s,
            "cpu_oracle_literal": "pure-Python restatement of cli_gate.oracle (one core)"}


def bench_rk_plan(b2, fd, steps):
    """The config-1 shape through the plan/workspace ABI: the Linear + HardSigmoid plan the reference's
    own planner writes for M=64, N=256, K=512 (tests/golden/rk_plans.json, chain mode: two K-tile
    uploads, two weight uploads packed once, MM + MM_ACC + a HardSigmoid LUT task, one download),
    run end to end with rk_workspace_run from host arrays (copies in, the recorded CUDA graph of the
    schedule, copy out, finiteness and guard checks, publish). The plan has no bias; its output is
    checked against co_linear_hsig_run at b = 0 within the 2e-3 + 2e-3|ref| tolerance (the plan sums
    each 256-K tile exactly, the operator on the tensor cores in FP32, so an element may differ by
    one FP16 rounding)."""
    import importlib
    import numpy as np
    rk = importlib.import_module("rockchip-npu-notes_b200.rkplan")
    name = "linear_hardsigmoid_64x512x256/chain"
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "tests", "golden", "rk_plans.json")) as f:
        entry = json.load(f)[name]
    m, n, k = 64, 256, 512
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, (m, k)).astype(np.float16)
    w = rng.uniform(-1 / np.sqrt(k), 1 / np.sqrt(k), (n, k)).astype(np.float16)
    y = np.zeros((m, n), np.float16)
    ids = {bd["name"]: bd["id"] for bd in entry["bindings"]}
    L = rk.declare(b2.lib())
    plan = rk.Plan(L, entry)
    ws = rk.Workspace(L, fd, plan, {ids["B"]: w})
    prepared = ws.prepare({ids["A"]: x}, {ids["A1"]: y})
    for _ in range(20):
        report = ws.run(prepared)
    reps = max(50, min(steps, 2000))
    wait = 0.0
    t0 = time.perf_counter()
    for _ in range(reps):
        report = ws.run(prepared)
        wait += report.submit_wait_us
    e2e_us = (time.perf_counter() - t0) / reps * 1e6
    tasks, submits = report.task_count, report.submit_count
    ws.destroy()
    plan.destroy()
    op = b2.Linear(fd, m, k, n, w, np.zeros(n, np.float16), post=b2.CO_LINEAR_HSIG, mode=b2.CO_CHAIN,
                   acc=b2.ACC_TILE16, compat=True)
    y_op = op.run(x)
    op.destroy()
    a, r = y.astype(np.float64), np.asarray(y_op, np.float64)
    if not np.all(np.abs(a - r) <= 2e-3 + 2e-3 * np.abs(r)):
        raise RuntimeError("plan-ABI output outside tolerance of co_linear_hsig_run at b = 0")
    same = float(np.mean(y.view(np.uint16) == np.asarray(y_op, np.float16).view(np.uint16)))
    return {"plan": name, "source": "the reference planner's descriptors (tests/golden/rk_plans.json)",
            "tasks": tasks, "submits": submits, "e2e_us": e2e_us, "device_schedule_and_copy_out_us": wait / reps,
            "vs_co_linear_hsig_run": {"within_tolerance": True, "bit_identical_fraction": same,
                                      "max_abs_diff": float(np.max(np.abs(a - r)))}}


def bench_cube(b2, fd, torch, stream, steps):
    """co_linear_run_tiled at M = N = K = 4096 (the reference's cube entry used by its graph and
    attention callers: research/custom-ops/src/linear_hardsigmoid.c:325-352): X as 16 x 16 C2=8 cube
    views of 256 x 256 (co_tensor_matrix), Y as 16 x 16 output cubes, co_linear_create's default
    numerics. The GEMM reads the input cubes through 3-D tensor maps and writes the output cubes
    directly; the entry is synchronous (it also checks every caller buffer's guard). Beside it, the
    same operator on row-major device buffers (b2_linear_run_device), back to back."""
    import numpy as np
    m = n = k = 4096
    rng = np.random.default_rng(12)
    w = (rng.standard_normal((n, k), np.float32) / 64).astype(np.float16)
    x = rng.standard_normal((m, k), np.float32).astype(np.float16)
    op = b2.Linear(fd, m, k, n, w, np.zeros(n, np.float16), post=b2.CO_LINEAR_NONE, mode=b2.CO_CHAIN)
    t = b2.tensor_matrix(256, 256)
    xbuf, ybuf = b2.Buffer(fd, 256 * t.bytes), b2.Buffer(fd, 256 * t.bytes)
    xv = [xbuf.view(t, i * t.bytes) for i in range(256)]     # [m tile][k tile]
    yv = [ybuf.view(t, i * t.bytes) for i in range(256)]     # [m tile][n tile]
    for i, v in enumerate(xv):
        mi, ki = divmod(i, 16)
        b2.upload(v, np.ascontiguousarray(x[mi * 256:(mi + 1) * 256, ki * 256:(ki + 1) * 256]))
    xa, ya = b2.views_array(xv), b2.views_array(yv)   # the caller's view arrays, built once
    run = b2.lib().co_linear_run_tiled
    for _ in range(3):
        assert run(op.h, xa, len(xv), ya, len(yv)) == 0
    reps = max(10, min(steps, 100))
    es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    before = b2.counters()["launches"]
    es.record(stream)
    for _ in range(reps):
        run(op.h, xa, len(xv), ya, len(yv))
    ee.record(stream)
    ee.synchronize()
    tiled_ms = es.elapsed_time(ee) / reps
    launches = (b2.counters()["launches"] - before) / reps
    # device-resident row-major run of the same operator (back to back, one stream)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty(m, n, device="cuda", dtype=torch.float16)
    torch.cuda.synchronize()
    for _ in range(3):
        op.run_device(m, xd.data_ptr(), k, yd.data_ptr(), n)
    b2.sync(fd)
    es.record(stream)
    for _ in range(reps):
        op.run_device(m, xd.data_ptr(), k, yd.data_ptr(), n)
    ee.record(stream)
    ee.synchronize()
    dev_ms = es.elapsed_time(ee) / reps
    if b2.status(fd):
        raise RuntimeError("device status raised in the cube-entry run")
    # the two entries give the same bytes
    got = np.empty((m, n), np.float16)
    for i, v in enumerate(yv):
        mi, ni = divmod(i, 16)
        got[mi * 256:(mi + 1) * 256, ni * 256:(ni + 1) * 256] = b2.download(v)
    if not np.array_equal(got.view(np.uint16), yd.cpu().numpy().view(np.uint16)):
        raise RuntimeError("cube entry and row-major entry differ")
    op.destroy()
    xbuf.free()
    ybuf.free()
    return {"m": m, "n": n, "k": k, "views_in": 256, "views_out": 256, "run_tiled_ms": tiled_ms,
            "run_device_ms": dev_ms, "ratio": tiled_ms / dev_ms, "launches_per_call": launches,
            "tflops": 2 * m * n * k / (tiled_ms * 1e-3) / 1e12,
            "numerics": "per-256-K FP16 running sum (co_linear_create default)"}


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

    # the whole set -- the layer's 7 projections and the LM head (63.7 MB of weights) -- as ONE grouped
    # launch, the inputs as in a decode step (q/k/v/gate/up share the layer input; o, down and the LM
    # head read their own); weight sets rotated over >= 4x L2, replayed as a CUDA graph
    full = list(GEMV_LAYER)
    set_bytes = sum(2 * n * k for _, n, k in full)
    copies = min(64, max(2, -(-4 * l2 // set_bytes)))
    w_host = {name: (rng.standard_normal((n, k)) * 0.02).astype(np.float16) for name, n, k in full}
    sets = [[b2.Linear(fd, 1, k, n, w_host[name], None, post=b2.CO_LINEAR_NONE, acc=b2.ACC_FP32, compat=False)
             for name, n, k in full] for _ in range(copies)]
    xin["lm"] = torch.randn(1, 576, device="cuda", generator=gen).half()
    src["lm_head"] = "lm"
    ys = [torch.empty(1, n, device="cuda", dtype=torch.float16) for _, n, _ in full]
    xp = [xin[src[name]].data_ptr() for name, _, _ in full]
    ldx = [k for _, _, k in full]
    yp = [y.data_ptr() for y in ys]
    ldy = [n for _, n, _ in full]
    torch.cuda.synchronize()
    for ops in sets:
        b2.group_run_device(ops, 1, xp, ldx, yp, ldy)
    b2.sync(fd)
    launches0 = b2.counters()["launches"]
    b2.group_run_device(sets[0], 1, xp, ldx, yp, ldy)
    set_launches = b2.counters()["launches"] - launches0
    reps = max(64, 4 * copies)
    eager, ms = _eager_and_graph_ms(torch, stream, lambda i: b2.group_run_device(sets[i % copies], 1, xp, ldx, yp, ldy),
                                    reps)
    if b2.status(fd):
        raise RuntimeError("device status raised in the grouped set run")
    fbytes = sum(2 * n * k + 2 * k + 2 * n for _, n, k in full)
    out["set_8_grouped"] = {"bytes": fbytes, "us": ms * 1e3, "gb_s": fbytes / (ms * 1e-3) / 1e9,
                            "frac": fbytes / (ms * 1e-3) / 1e9 / peak_gbs, "eager_us": eager * 1e3,
                            "launches": set_launches, "weight_sets": copies}

    # the same set as a decode step's dependent chain, one CUDA graph: {q,k,v} -> o (input: q's output)
    # -> {gate, up} (input: o's output) -> down (input: gate's output) -> LM head (input: down's output)
    name_ix = {name: i for i, (name, _, _) in enumerate(full)}
    x0 = xin["h"]

    def chain(i):
        ops = sets[i % copies]
        b2.group_run_device([ops[name_ix[q]] for q in ("q", "k", "v")], 1, [x0.data_ptr()] * 3, [576] * 3,
                            [ys[name_ix[q]].data_ptr() for q in ("q", "k", "v")], [576, 192, 192])
        ops[name_ix["o"]].run_device(1, ys[name_ix["q"]].data_ptr(), 576, ys[name_ix["o"]].data_ptr(), 576)
        b2.group_run_device([ops[name_ix["gate"]], ops[name_ix["up"]]], 1, [ys[name_ix["o"]].data_ptr()] * 2,
                            [576, 576], [ys[name_ix["gate"]].data_ptr(), ys[name_ix["up"]].data_ptr()], [1536, 1536])
        ops[name_ix["down"]].run_device(1, ys[name_ix["gate"]].data_ptr(), 1536, ys[name_ix["down"]].data_ptr(), 576)
        ops[name_ix["lm_head"]].run_device(1, ys[name_ix["down"]].data_ptr(), 576, ys[name_ix["lm_head"]].data_ptr(),
                                           49152)

    for i in range(copies):
        chain(i)
    b2.sync(fd)
    creps = max(16, 2 * copies)
    eager, ms = _eager_and_graph_ms(torch, stream, chain, creps)
    if b2.status(fd):
        raise RuntimeError("device status raised in the decode chain run")
    out["set_8_decode_chain"] = {"bytes": fbytes, "us": ms * 1e3, "gb_s": fbytes / (ms * 1e-3) / 1e9,
                                 "frac": fbytes / (ms * 1e-3) / 1e9 / peak_gbs, "eager_us": eager * 1e3,
                                 "launches": 5, "weight_sets": copies}
    for ops in sets:
        for op in ops:
            op.destroy()
    del sets

    # long-K decode projections at M=1 (a 7B-class layer's attention and FFN shapes), weights rotated
    out["long_k"] = {}
    for n, k in ((4096, 4096), (11008, 4096), (4096, 11008)):
        wbytes = 2 * n * k
        copies = max(2, -(-4 * l2 // wbytes))
        w_host = (np.random.default_rng(n + 3 * k).standard_normal((n, k)) * 0.02).astype(np.float16)
        ops = [b2.Linear(fd, 1, k, n, w_host, None, post=b2.CO_LINEAR_NONE, acc=b2.ACC_TILE16, compat=False)
               for _ in range(copies)]
        x = torch.randn(1, k, device="cuda", generator=gen).half()
        y = torch.empty(1, n, device="cuda", dtype=torch.float16)
        torch.cuda.synchronize()
        for op in ops:
            op.run_device(1, x.data_ptr(), k, y.data_ptr(), n)
        b2.sync(fd)
        reps = max(32, 4 * copies)
        eager, ms = _eager_and_graph_ms(
            torch, stream, lambda i: ops[i % copies].run_device(1, x.data_ptr(), k, y.data_ptr(), n), reps)
        if b2.status(fd):
            raise RuntimeError(f"device status raised in the {n}x{k} GEMV")
        nbytes = wbytes + 2 * k + 2 * n
        info = ops[0].info()
        out["long_k"][f"{n}x{k}"] = {"us": ms * 1e3, "gb_s": nbytes / (ms * 1e-3) / 1e9,
                                      "frac": nbytes / (ms * 1e-3) / 1e9 / peak_gbs, "eager_us": eager * 1e3,
                                      "stages": info.stages, "grid": info.grid, "weight_copies": copies}
        for op in ops:
            op.destroy()
    out["peak_gbs"] = peak_gbs
    return out


if __name__ == "__main__":
    main()
