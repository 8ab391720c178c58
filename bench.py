"""Benchmark of the sdvk-b200 hot path: the Q8_0 dequant GEMM
Y[9216,1280] = X[9216,1280] . dequant(W[1280,1280])^T, fp16 X, GGUF Q8_0 W, fp32 Y.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl sdvk|reference]

One step = one GEMM launch over one set of synthetic inputs.  Four rotating input/output sets
(4 x 72 MB, larger than the 126 MB L2) keep every step's operands out of L2.  Steps are captured in
CUDA graphs and replayed; the timed region is bracketed by a barrier and a device synchronize and
timed with CUDA events on the launching stream; the job time is the max over ranks.  Multi-GPU
runs are independent replicas (images sharded one per GPU): weak scaling, no collective on the
data path.  Rank 0 prints one JSON line.

--impl reference times the reference's own GEMM arithmetic (the C++ restatement of
gemm_nt_q8_v.comp in oracle/, which is what the reference's Vulkan path computes; the Vulkan path
itself needs a graphics stack this machine does not have) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
M, N, K = 9216, 1280, 1280
FLOP = 2.0 * M * N * K
METRIC = "Q8_0 GEMM TFLOP/s @9216x1280x1280"
WORKLOAD = "Q8_0 dequant GEMM 9216x1280x1280 (BASELINE config 0): fp16 X ~N(0,1), Q8_0 W (int8 U[-127,127], scale |N(0,0.02)|/127), fp32 Y"
ROTATE = 4
GRAPH_LEN = 50
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"]))}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS, bf16_tflops_sustained=FALLBACK_PEAKS["bf16_tflops"]), "fallback"


def profile_traffic():
    """DRAM bytes per launch of the GEMM kernel from the committed ncu summary, if present."""
    try:
        with open(os.path.join(ROOT, "profiles", "gemm_q8_nt_9216x1280x1280.json")) as f:
            return float(json.load(f)["dram_bytes_per_launch"])
    except Exception:
        return None


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled while the timed region runs."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.05)
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        except Exception:
            pass
        finally:
            try:
                os.remove(self.path)
            except Exception:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3] not in ("", "[N/A]"))}


def make_inputs(torch, device, seed):
    """Config-0 inputs generated on the device with torch's RNG (seeded per rank and set)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn((M, K), generator=g, device=device, dtype=torch.float32).half()
    q = torch.randint(-127, 128, (N, K), generator=g, device=device, dtype=torch.int8)
    sc = (torch.randn((N * K // 32,), generator=g, device=device).abs() * 0.02 / 127).half().float()
    y = torch.empty((M, N), device=device, dtype=torch.float32)
    return x, q, sc, y


def cpu_reference(x_np, q_np, s_np, budget_s):
    """Time the reference arithmetic (oracle restatement of gemm_nt_q8_v.comp, fp32) on a bounded
    row sample of the workload; returns (TFLOP/s, rows, threads, seconds)."""
    from oracle import pyoracle

    threads = pyoracle.num_threads()
    a = np.ascontiguousarray(x_np.astype(np.float32))
    pyoracle.gemm_nt_q8_shader(a[:64], q_np, s_np)  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:  # whole GEMMs until the budget is spent
        pyoracle.gemm_nt_q8_shader(a, q_np, s_np)
        reps += 1
        dt = time.perf_counter() - t0
        if dt >= budget_s:
            break
    return 2.0 * M * N * K * reps / dt / 1e12, reps, threads, dt


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    rng = np.random.default_rng(0)
    x = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16)
    q = rng.integers(-127, 128, (N, K), dtype=np.int8)
    s = (np.abs(rng.standard_normal(N * K // 32)) * 0.02 / 127).astype(np.float16).astype(np.float32)
    from oracle import pyoracle

    threads = pyoracle.num_threads()
    # each step: a bounded row sample, sized so the whole run takes about a minute
    budget = 60.0 / max(1, args.steps + args.warmup)
    rows = 16
    a = np.ascontiguousarray(x[:rows].astype(np.float32))
    t0 = time.perf_counter()
    pyoracle.gemm_nt_q8_shader(a, q, s)
    per_row = (time.perf_counter() - t0) / rows
    rows = int(max(8, min(M, budget / max(per_row, 1e-9))))
    a = np.ascontiguousarray(x[:rows].astype(np.float32))
    for _ in range(args.warmup):
        pyoracle.gemm_nt_q8_shader(a, q, s)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        pyoracle.gemm_nt_q8_shader(a, q, s)
    dt = time.perf_counter() - t0
    value = 2.0 * rows * N * K * args.steps / dt / 1e12
    sample = f"{rows} of {M} rows per step (fp32 restatement of gemm_nt_q8_v.comp, BM128 variant's per-element order)"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": WORKLOAD, "sample_rows": rows},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference Vulkan path unavailable on this box (no graphics stack); its shader arithmetic is timed "
                "as the oracle's C++ restatement on the host cores",
    }
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=100)
    ap.add_argument("--impl", default="sdvk", choices=["sdvk", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch
    import torch.distributed as dist
    import datetime

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    sys.path.insert(0, ROOT)
    import sdvk_b200
    from sdvk_b200 import torch_ops

    sets = [make_inputs(torch, device, 1000 * rank + i) for i in range(ROTATE)]
    ctx = torch_ops.context(device)

    def step(i):
        x, q, s, y = sets[i % ROTATE]
        torch_ops.gemm_q8_nt(x, q, s, out=y)

    # warm-up (also the first launch's attribute setup), then graphs of GRAPH_LEN steps
    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    cap = torch.cuda.Stream(device)
    graphs = {}

    def graph_of(n):
        if n not in graphs:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                for i in range(n):
                    step(i)
            graphs[n] = g
        return graphs[n]

    full, rem = divmod(args.steps, GRAPH_LEN)
    if full:
        graph_of(GRAPH_LEN).replay()
    if rem:
        graph_of(rem).replay()
    torch.cuda.synchronize()
    ctx.synchronize()  # surfaces any device-side error from the warm-up

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        stream = torch.cuda.current_stream(device)
        ev0.record(stream)
        for _ in range(full):
            graph_of(GRAPH_LEN).replay()
        if rem:
            graph_of(rem).replay()
        ev1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = ev0.elapsed_time(ev1)
    ctx.synchronize()
    clocks = clk.summary()
    t = torch.tensor([ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    ms_per_step = ms_max / args.steps
    value = world * FLOP * args.steps / (ms_max * 1e-3) / 1e12

    # ---- end to end through the C ABI: pinned host X -> device, GEMM, device Y -> pinned host
    e2e_steps = min(args.steps, 100)
    xh = torch.empty((M, K), dtype=torch.float16, pin_memory=True)
    xh.copy_(sets[0][0].cpu())
    yh = torch.empty((M, N), dtype=torch.float32, pin_memory=True)
    xd, qd, sd, yd = sets[0]
    ctx.set_stream(torch.cuda.current_stream(device).cuda_stream)

    def e2e_step():
        ctx.upload_async(xd.data_ptr(), xh.data_ptr(), xh.numel() * 2)
        ctx.gemm_q8_nt(xd.data_ptr(), sdvk_b200.F16, qd.data_ptr(), sd.data_ptr(), None, yd.data_ptr(),
                       sdvk_b200.F32, M, N, K, K, N)
        ctx.download_async(yh.data_ptr(), yd.data_ptr(), yh.numel() * 4)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0.record()
    for _ in range(e2e_steps):
        e2e_step()
    ev1.record()
    torch.cuda.synchronize()
    t = torch.tensor([ev0.elapsed_time(ev1)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item()) / e2e_steps
    e2e_value = world * FLOP / (e2e_ms * 1e-3) / 1e12

    # ---- CPU baseline (rank 0, N = 1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        x_np = sets[0][0].cpu().numpy()
        q_np = sets[0][1].cpu().numpy()
        s_np = sets[0][2].cpu().numpy()
        tf, reps, threads, secs = cpu_reference(x_np, q_np, s_np, budget_s=10.0)
        cpu = {"value": tf, "unit": "TFLOP/s", "cores": threads, "kind": "port",
               "sample": f"{reps} whole {M}x{N}x{K} GEMMs on the same inputs (fp32 restatement of "
                         f"gemm_nt_q8_v.comp, OpenMP over tiles), {secs:.1f} s"}

    pk, pk_kind = peaks()
    achieved = FLOP / (ms_per_step * 1e-3) / 1e12
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "M": M, "N": N, "K": K, "parallelism": f"replicas x{world}",
                       "l2": f"{ROTATE} rotating input/output sets ({ROTATE * 72} MB > 126 MB L2)",
                       "timing": f"CUDA events over CUDA-graph replays of {GRAPH_LEN} launches"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": achieved / pk["bf16_tflops"], "traffic": profile_traffic(),
                         "peak_kind": f"{pk_kind} dense bf16 burst",
                         "algorithmic_flop_per_launch": FLOP,
                         "algorithmic_bytes_per_launch": M * K * 2 + M * N * 4 + N * K + N * K // 32 * 4},
            "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": M * K * 2,
                    "d2h_bytes_per_step": M * N * 4, "ms_per_step": e2e_ms,
                    "path": "sdvk_upload_async + sdvk_gemm_q8_nt + sdvk_download_async, pinned host buffers"},
            "gpu_launches": args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    for g in graphs.values():
        del g
    graphs.clear()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
