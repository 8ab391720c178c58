"""Benchmark of the sdvk-b200 hot path on one B200 per rank.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl sdvk|reference] [--workload NAME]

Workloads (synthetic seeded inputs of the stated shapes, random-init Q8_0 weights):
  unet             (default) one SDXL 1024^2 CFG denoising step: the whole UNet pass over the
                   cond/uncond pair (batch 2, 4x128x128 latent, 77x2048 context) + the device sampler
                   step (Euler, cfg 5.0, v-pred); metric images/s at 20 steps per image (configs 3/4:
                   --gpus N runs N independent images)
  unet-cfg-pair    the same step with the CFG halves on a GPU pair (NCCL all-gather), --gpus even
  gemm             Q8_0 dequant GEMM Y[9216,1280] = X[9216,1280] . dequant(W[1280,1280])^T,
                   fp16 X, GGUF Q8_0 W (int8 + per-32 scale), fp32 Y (config 0)
  block            one SDXL BasicTransformerBlock, batch 2 x 1024 tokens x 1280 channels (config 2)
  attn-self-4096   fused attention, batch 2, 4096 tokens, 10 heads x 64, fp16 (config 1a)
  attn-self-1024   fused attention, batch 2, 1024 tokens, 20 heads x 64, fp16 (config 1b)
  attn-cross-77    fused attention, batch 2, 1024 queries x 77 keys, 20 heads x 64, fp16 (config 1c)
  conv, groupnorm, sampler   the next-row kernels at SDXL level-0 shapes

One step = one launch of the hot-path kernel (for `block`, the block's launches; for `unet`, a
denoising step of about 1030 launches replayed from one CUDA graph) over one set of inputs.
Rotating input/output sets
whose total exceeds the 126 MB L2 keep every step's operands out of L2.  Steps are captured in CUDA
graphs and replayed; the timed region is bracketed by a barrier and a device synchronize and timed
with CUDA events on the launching stream; the job time is the max over ranks.  Multi-GPU runs are
independent replicas (one image per GPU): weak scaling, no collective on the data path.  Rank 0
prints one JSON line.

`e2e` is the same metric through the C ABI with pinned host buffers: each step uploads that step's
inputs, runs the kernel and downloads the result, all inside the timed region.

--impl reference times the reference's own CPU implementation on the host cores (all usable cores,
whatever OMP_NUM_THREADS the launcher set).  For the UNet workloads that is the reference's own
generation program -- src/Modules/Diffusion/main.cpp and sdvkgen.cpp compiled unchanged against the
host stub engine (oracle/_ref/sdvkgen_host), whose kernels restate the reference's shaders in C++ --
running its Euler / v-pred / CFG 5 loop on the same seeded UNet at a 16x16 latent, each of its steps
scaled to the 128x128 latent by the UNet's FLOP ratio (the program runs the full size about 20 %
slower per FLOP than the small one, so the scaled value flatters the reference).  For the kernel
workloads it is the oracle's C++ restatement of gemm_nt_q8_v.comp / fused_attn_tiled.comp /
fused_attn.comp.  The Vulkan path itself needs a graphics stack this machine does not have.

The default `unet` line also carries `kernels` (config 0's GEMM and config 1's three attentions,
CUDA-event timed in the same process, each with its roofline fraction) and, at N >= 2, `cfg_pair`:
the CFG halves of each image on a GPU pair through the C ABI (sdvk_comm_create / sdvk_allgather
inside the captured step graph), with the pair's all-gather time and a check that both ranks of
every pair end with bit-identical latents.
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
GRAPH_LEN = 50
L2_BYTES = 126 << 20
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"]),
                "bf16_tflops_sustained": float(p.get("bf16_tflops_sustained", p["bf16_tflops"]))}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS, bf16_tflops_sustained=FALLBACK_PEAKS["bf16_tflops"]), "fallback"


def profile_traffic(workload: str):
    """DRAM bytes (read + write) per launch of the workload's kernel, from the committed ncu
    summary profiles/traffic.json, if present."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            return float(json.load(f)[workload]["dram_bytes_per_launch"])
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




# ------------------------------------------------------------------------------------------ workloads
class GemmWorkload:
    """the Q8_0 NT GEMM (gemm_nt_q8_v.comp's operator)."""

    name = "gemm"
    M, N, K = 9216, 1280, 1280
    metric = "Q8_0 GEMM TFLOP/s @9216x1280x1280"
    describe = ("Q8_0 dequant GEMM 9216x1280x1280 (BASELINE config 0): fp16 X ~N(0,1), Q8_0 W (int8 U[-127,127], "
                "scale |N(0,0.02)|/127), fp32 Y")
    bound = "tensor"
    dtype = "f16"

    def __init__(self):
        M, N, K = self.M, self.N, self.K
        self.flop = 2.0 * M * N * K
        self.bytes = M * K * 2 + M * N * 4 + N * K + N * K // 32 * 4
        self.rotate = max(2, -(-2 * L2_BYTES // self.bytes))

    def make_set(self, torch, device, seed):
        M, N, K = self.M, self.N, self.K
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        x = torch.randn((M, K), generator=g, device=device, dtype=torch.float32).half()
        q = torch.randint(-127, 128, (N, K), generator=g, device=device, dtype=torch.int8)
        sc = (torch.randn((N * K // 32,), generator=g, device=device).abs() * 0.02 / 127).half().float()
        y = torch.empty((M, N), device=device, dtype=torch.float32)
        return x, q, sc, y

    def step(self, torch_ops, st):
        x, q, s, y = st
        torch_ops.gemm_q8_nt(x, q, s, out=y)

    def e2e(self, sdvk_b200, ctx, torch, st):
        """Per step: pinned X -> device, GEMM, device Y -> pinned host."""
        x, q, s, y = st
        xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        xh.copy_(x.cpu())
        yh = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
        M, N, K = self.M, self.N, self.K

        def run():
            ctx.upload_async(x.data_ptr(), xh.data_ptr(), xh.numel() * 2)
            ctx.gemm_q8_nt(x.data_ptr(), sdvk_b200.F16, q.data_ptr(), s.data_ptr(), None, y.data_ptr(),
                           sdvk_b200.F32, M, N, K, K, N)
            ctx.download_async(yh.data_ptr(), y.data_ptr(), yh.numel() * 4)

        return run, xh.numel() * 2, yh.numel() * 4, "sdvk_upload_async + sdvk_gemm_q8_nt + sdvk_download_async"

    def host_inputs(self):
        M, N, K = self.M, self.N, self.K
        rng = np.random.default_rng(0)
        x = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16).astype(np.float32)
        q = rng.integers(-127, 128, (N, K), dtype=np.int8)
        s = (np.abs(rng.standard_normal(N * K // 32)) * 0.02 / 127).astype(np.float16).astype(np.float32)
        return x, q, s

    def cpu_run(self, inputs, rows):
        """The reference arithmetic on the first `rows` rows of X; returns the FLOP it did."""
        from oracle import pyoracle

        x, q, s = inputs
        pyoracle.gemm_nt_q8_shader(np.ascontiguousarray(x[:rows]), q, s)
        return 2.0 * rows * self.N * self.K

    cpu_units = M
    cpu_what = "rows of X (fp32 restatement of gemm_nt_q8_v.comp, OpenMP over 128x64 output tiles)"


class AttnWorkload:
    """fusedAttention (fused_attn_tiled.comp / fused_attn.comp's operator)."""

    dtype = "f16"

    def __init__(self, name, B, Tq, Tk, heads, hd=64):
        self.name, self.B, self.Tq, self.Tk, self.heads, self.hd = name, B, Tq, Tk, heads, hd
        self.C = heads * hd
        self.flop = 4.0 * B * heads * Tq * Tk * hd
        self.bytes = 2 * (2 * B * Tq * self.C + 2 * B * Tk * self.C)
        self.bound = "tensor" if self.flop / self.bytes > 300 else "hbm"
        kind = "self" if Tq == Tk else "cross"
        self.metric = f"fused attention TFLOP/s @B{B} {kind} Tq{Tq} Tk{Tk} {heads}x{hd}"
        self.describe = (f"fused {kind}-attention (BASELINE config 1): batch {B}, Tq {Tq}, Tk {Tk}, {heads} heads x "
                         f"{hd}, fp16 Q/K/V ~N(0,1) token-major [B, T, {self.C}], scale 1/sqrt({hd}), fp16 O")
        self.rotate = max(2, -(-2 * L2_BYTES // self.bytes))
        self.cpu_units = Tq
        self.cpu_what = (f"query rows of batch 0, all {heads} heads (fp32 restatement of "
                         f"{'fused_attn_tiled.comp' if hd == 64 and Tk >= 256 else 'fused_attn.comp'})")

    def make_set(self, torch, device, seed):
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        B, C = self.B, self.C
        q = torch.randn((B, self.Tq, C), generator=g, device=device, dtype=torch.float32).half()
        k = torch.randn((B, self.Tk, C), generator=g, device=device, dtype=torch.float32).half()
        v = torch.randn((B, self.Tk, C), generator=g, device=device, dtype=torch.float32).half()
        o = torch.empty((B, self.Tq, C), device=device, dtype=torch.float16)
        return q, k, v, o

    def step(self, torch_ops, st):
        q, k, v, o = st
        torch_ops.attention(q, k, v, self.heads, out=o)

    def e2e(self, sdvk_b200, ctx, torch, st):
        """Per step: pinned Q, K, V -> device, attention, device O -> pinned host."""
        q, k, v, o = st
        hosts = []
        for t in (q, k, v):
            h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
            h.copy_(t.cpu())
            hosts.append(h)
        oh = torch.empty(o.shape, dtype=o.dtype, pin_memory=True)
        d = sdvk_b200.AttnDesc()
        d.q, d.k, d.v, d.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
        d.dtype = d.o_dtype = sdvk_b200.F16
        d.batch, d.heads, d.Tq, d.Tk, d.hd = self.B, self.heads, self.Tq, self.Tk, self.hd
        d.ldq = d.ldk = d.ldv = d.ldo = self.C
        d.sq, d.so = self.Tq * self.C, self.Tq * self.C
        d.sk = d.sv = self.Tk * self.C
        d.hq = d.hk = d.hv = d.ho = self.hd
        d.scale = 1.0 / math.sqrt(self.hd)
        d.causal = 0

        def run():
            for h, t in zip(hosts, (q, k, v)):
                ctx.upload_async(t.data_ptr(), h.data_ptr(), h.numel() * 2)
            ctx.attention(d)
            ctx.download_async(oh.data_ptr(), o.data_ptr(), oh.numel() * 2)

        h2d = sum(h.numel() * 2 for h in hosts)
        return run, h2d, oh.numel() * 2, "3x sdvk_upload_async + sdvk_attention + sdvk_download_async"

    def host_inputs(self):
        rng = np.random.default_rng(1)
        C = self.C
        f16 = lambda a: a.astype(np.float16).astype(np.float32)
        return (f16(rng.standard_normal((self.Tq, C), dtype=np.float32)),
                f16(rng.standard_normal((self.Tk, C), dtype=np.float32)),
                f16(rng.standard_normal((self.Tk, C), dtype=np.float32)))

    def cpu_run(self, inputs, rows):
        from oracle import pyoracle

        q, k, v = inputs
        pyoracle.fused_attention(np.ascontiguousarray(q[:rows]), k, v, rows, self.Tk, self.C, self.heads)
        return 4.0 * self.heads * rows * self.Tk * self.hd


class BlockWorkload:
    """one SDXL BasicTransformerBlock (spatialTransformer's layer body)."""

    name = "block"
    B, T, C, H, Tc, Cc, F = 2, 1024, 1280, 20, 77, 2048, 5120
    metric = "BasicTransformerBlock TFLOP/s @B2 T1024 C1280"
    describe = ("SDXL BasicTransformerBlock (BASELINE config 2): batch 2, 1024 tokens, 1280 channels, 20x64 heads, "
                "77x2048 context, GEGLU 1280->10240->1280; random Q8_0 weights (config-0 distribution), fp32 residual "
                "x ~N(0,1), fp16 context ~N(0,1), LN gamma 1 beta 0")
    bound = "tensor"
    dtype = "f16"
    # LN, QKV GEMM, attention, out GEMM; LN, Q GEMM, K|V GEMM (split-K + reduce), attention, out GEMM;
    # LN, FF1 with GEGLU in its epilogue, FF2
    launches_per_step = 13

    def __init__(self):
        B, T, C, H, Tc, Cc, F = self.B, self.T, self.C, self.H, self.Tc, self.Cc, self.F
        rows = B * T
        self.flop = (2.0 * rows * (3 * C * C + 3 * C * C + 2 * F * C + C * F) + 2.0 * B * Tc * 2 * C * Cc
                     + 4.0 * B * H * T * T * 64 + 4.0 * B * H * T * Tc * 64)
        self.weights = None
        # weights (34 MB int8) + per-step activations and workspace (~110 MB) exceed L2 with 2 sets
        self.bytes = int((3 * C * C + 3 * C * C + 2 * C * Cc + 3 * F * C) * 1.03 + rows * C * 8 + B * Tc * Cc * 2)
        self.rotate = 2
        self.l2_note = ("2 rotating sets; each step moves ~250 MB (34 MB of weights, x read/written 9x, 89 MB of fp16 "
                        "intermediates) > 126 MB L2")
        self.cpu_units = T
        self.cpu_what = ("query rows of image 0 (fp32 restatement of the reference's kernels: layernorm_fwd, "
                         "gemm_nt_q8_v(+bias), fused_attn(_tiled), unary_fwd GELU, mul2, add2)")

    def _make_weights(self, torch, device):
        g = torch.Generator(device=device)
        g.manual_seed(4)
        B, T, C, H, Tc, Cc, F = self.B, self.T, self.C, self.H, self.Tc, self.Cc, self.F

        def q8(n, k, bias):
            q = torch.randint(-127, 128, (n, k), generator=g, device=device, dtype=torch.int8)
            s = (torch.randn((n * k // 32,), generator=g, device=device).abs() * 0.02 / 127).half().float()
            b = torch.randn((n,), generator=g, device=device) * 0.02 if bias else None
            return q, s, b

        W = {}
        qkv = q8(3 * C, C, False)  # q, k, v back to back: one GEMM
        for i, n in enumerate(("q", "k", "v")):
            W[n] = (qkv[0][i * C:(i + 1) * C], qkv[1][i * C * C // 32:(i + 1) * C * C // 32], None)
        kv = q8(2 * C, Cc, False)
        for i, n in enumerate(("k2", "v2")):
            W[n] = (kv[0][i * C:(i + 1) * C], kv[1][i * C * Cc // 32:(i + 1) * C * Cc // 32], None)
        W["o"], W["q2"], W["o2"] = q8(C, C, True), q8(C, C, False), q8(C, C, True)
        W["ff1"], W["ff2"] = q8(2 * F, C, True), q8(C, F, True)
        for i in (1, 2, 3):
            W[f"ln{i}_w"] = torch.ones(C, device=device)
            W[f"ln{i}_b"] = torch.zeros(C, device=device)
        # the load-time repack that folds GEGLU into the ff.net.0 GEMM (the original stays for the CPU arm)
        from sdvk_b200 import torch_ops

        W["ff1_il"] = torch_ops.geglu_interleave(*W["ff1"])
        return W

    def make_set(self, torch, device, seed):
        if self.weights is None:
            self.weights = self._make_weights(torch, device)
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        x = torch.randn((self.B, self.T, self.C), generator=g, device=device)
        ctx = torch.randn((self.B, self.Tc, self.Cc), generator=g, device=device).half()
        need = self._workspace(torch, device, x, ctx)
        ws = torch.empty(need, dtype=torch.uint8, device=device)
        return x, ctx, ws

    def _desc(self, sdvk_b200, torch_ops, x, ctx):
        d = sdvk_b200.BlockDesc()
        d.x, d.ctx, d.ctx_dtype = x.data_ptr(), ctx.data_ptr(), sdvk_b200.F16
        d.batch, d.T, d.C, d.heads, d.Tctx, d.Cctx, d.ff_inner = self.B, self.T, self.C, self.H, self.Tc, self.Cc, self.F
        for n in ("ln1_w", "ln1_b", "ln2_w", "ln2_b", "ln3_w", "ln3_b"):
            setattr(d, n, self.weights[n].data_ptr())
        for n in ("q", "k", "v", "o", "q2", "k2", "v2", "o2", "ff2"):
            setattr(d, n, torch_ops.q8_linear(*self.weights[n]))
        d.ff1 = torch_ops.q8_linear(*self.weights["ff1_il"])
        d.ff1_geglu_interleaved = 1
        d.eps = 1e-5
        return d

    def _workspace(self, torch, device, x, ctx):
        import sdvk_b200
        from sdvk_b200 import torch_ops

        return sdvk_b200.Context.block_workspace(self._desc(sdvk_b200, torch_ops, x, ctx))

    def step(self, torch_ops, st):
        import sdvk_b200

        x, ctx, ws = st
        torch_ops.context(x.device).transformer_block(self._desc(sdvk_b200, torch_ops, x, ctx), ws.data_ptr(),
                                                      ws.numel())

    def e2e(self, sdvk_b200, ctx_, torch, st):
        """Per step: pinned x and context -> device, the block, device x -> pinned host."""
        from sdvk_b200 import torch_ops

        x, cx, ws = st
        xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        xh.copy_(x.cpu())
        ch = torch.empty(cx.shape, dtype=cx.dtype, pin_memory=True)
        ch.copy_(cx.cpu())
        d = self._desc(sdvk_b200, torch_ops, x, cx)

        def run():
            ctx_.upload_async(x.data_ptr(), xh.data_ptr(), xh.numel() * 4)
            ctx_.upload_async(cx.data_ptr(), ch.data_ptr(), ch.numel() * 2)
            ctx_.transformer_block(d, ws.data_ptr(), ws.numel())
            ctx_.download_async(xh.data_ptr(), x.data_ptr(), xh.numel() * 4)

        return run, xh.numel() * 4 + ch.numel() * 2, xh.numel() * 4, \
            "2x sdvk_upload_async + sdvk_transformer_block + sdvk_download_async"

    def host_inputs(self):
        W = {k: (tuple(a.cpu().numpy() if a is not None else None for a in v) if isinstance(v, tuple)
                 else v.cpu().numpy()) for k, v in self.weights.items()}
        rng = np.random.default_rng(4)
        x = rng.standard_normal((1, self.T, self.C), dtype=np.float32)
        ctx = rng.standard_normal((1, self.Tc, self.Cc), dtype=np.float32).astype(np.float16).astype(np.float32)
        return x, ctx, W

    def cpu_run(self, inputs, rows):
        from oracle import pyoracle

        x, ctx, W = inputs
        pyoracle.block_shader(x, ctx, self.H, W, np.arange(rows))
        T, C, Tc, Cc, F = self.T, self.C, self.Tc, self.Cc, self.F
        return (2.0 * rows * (C * C + C * C + C * C + C * C + 2 * F * C + C * F) + 2.0 * T * 2 * C * C
                + 2.0 * Tc * 2 * C * Cc + 4.0 * self.H * rows * (T + Tc) * 64)


class GroupNormWorkload:
    """The ResBlock's GroupNorm + SiLU (groupnorm.comp via gnInto, sdvkgen.cpp:1105-1113) at the first
    UNet level of a 1024^2 latent: 2 images, 320 channels, 128 x 128, 32 groups.  HBM-bound."""

    dtype = "f32"
    unit = "GB/s"
    launches_per_step = 2  # statistics, apply

    def __init__(self, B=2, C=320, H=128, W=128, G=32):
        self.name = "groupnorm"
        self.B, self.C, self.P, self.G = B, C, H * W, G
        self.bytes = 2.0 * 4 * B * C * self.P  # x read once, y written once
        self.work = self.bytes
        self.flop = 8.0 * B * C * self.P
        self.bound = "hbm"
        self.metric = f"GroupNorm+SiLU GB/s @B{B} C{C} {H}x{W} G{G}"
        self.describe = (f"GroupNorm + SiLU (groupnorm.comp, ResBlock): {B} images, {C} channels, {H}x{W}, {G} groups, "
                         f"fp32 x ~N(0,1) channel-major, gamma ~1, beta ~0, eps 1e-5")
        self.rotate = max(2, -(-2 * L2_BYTES // int(self.bytes)))
        self.cpu_units = G
        self.cpu_what = "groups of image 0 (fp32 restatement of groupnorm.comp)"

    def make_set(self, torch, device, seed):
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        x = torch.randn((self.B, self.C, self.P), generator=g, device=device, dtype=torch.float32)
        gamma = 1.0 + 0.1 * torch.randn((self.C,), generator=g, device=device, dtype=torch.float32)
        beta = 0.1 * torch.randn((self.C,), generator=g, device=device, dtype=torch.float32)
        y = torch.empty_like(x)
        import sdvk_b200

        nbytes = sdvk_b200.Context.groupnorm_workspace(self.B, self.C, self.P, self.G)
        ws = torch.empty((nbytes,), dtype=torch.uint8, device=device)
        return x, gamma, beta, y, ws

    def step(self, torch_ops, st):
        x, gamma, beta, y, ws = st
        torch_ops.context(x.device).groupnorm(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), y.data_ptr(), self.B,
                                              self.C, self.P, self.G, 1e-5, True, ws.data_ptr(), ws.numel())

    def e2e(self, sdvk_b200, ctx, torch, st):
        """Per step: pinned x -> device, GroupNorm + SiLU, device y -> pinned host."""
        x, gamma, beta, y, ws = st
        xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        xh.copy_(x.cpu())
        yh = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)

        def run():
            ctx.upload_async(x.data_ptr(), xh.data_ptr(), xh.numel() * 4)
            ctx.groupnorm(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), y.data_ptr(), self.B, self.C, self.P,
                          self.G, 1e-5, True, ws.data_ptr(), ws.numel())
            ctx.download_async(yh.data_ptr(), y.data_ptr(), yh.numel() * 4)

        return run, xh.numel() * 4, yh.numel() * 4, "sdvk_upload_async + sdvk_groupnorm + sdvk_download_async"

    def host_inputs(self):
        rng = np.random.default_rng(1)
        x = rng.standard_normal((1, self.C, self.P), dtype=np.float32)
        gamma = (1.0 + 0.1 * rng.standard_normal(self.C)).astype(np.float32)
        beta = (0.1 * rng.standard_normal(self.C)).astype(np.float32)
        return x, gamma, beta

    def cpu_run(self, inputs, groups):
        from oracle import pyoracle

        x, gamma, beta = inputs
        cg = self.C // self.G
        ch = groups * cg
        pyoracle.groupnorm_shader(np.ascontiguousarray(x[:, :ch]), gamma[:ch], beta[:ch], groups, 1e-5, 1)
        return 2.0 * 4 * ch * self.P


class ConvWorkload:
    """A ResBlock 3x3 convolution with a Q8_0 weight (conv3RawInto, sdvkgen.cpp:1133-1158) at the first
    UNet level of a 1024^2 latent: 2 images, 320 -> 320 channels, 128 x 128."""

    dtype = "f16"

    def __init__(self, B=2, cin=320, cout=320, H=128, W=128):
        self.name = "conv"
        self.B, self.cin, self.cout, self.H, self.W = B, cin, cout, H, W
        P, K = H * W, cin * 9
        self.flop = 2.0 * B * cout * P * K
        self.bytes = B * (2.0 * cin * P + 4.0 * cout * P) + cout * K * 2
        self.bound = "tensor"
        self.metric = f"Q8_0 conv3x3 TFLOP/s @B{B} {cin}->{cout} {H}x{W}"
        self.describe = (f"3x3 convolution, Q8_0 weight [{cout}, {cin}*9] (config-0 distribution), {B} images of "
                         f"{cin}x{H}x{W} fp16 ~N(0,1), fp32 out + bias; step: the implicit GEMM as the UNet runs it "
                         f"(sdvk_conv3x3_nhwc: TMA im2col loads from the channels-last input its producer writes, "
                         f"weights repacked to fp16 at load time); e2e: sdvk_conv3x3_q8 from channel-major x and "
                         f"the Q8_0 weight, both conversions inside every call")
        self.rotate = max(2, -(-2 * L2_BYTES // int(self.bytes)))
        self.cpu_units = cout
        self.cpu_what = "output channels of image 0 (fp32 restatement of im2col.comp + gemm_nn_q8_v.comp)"
        self.launches_per_step = 1

    def make_set(self, torch, device, seed):
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        x = torch.randn((self.B, self.cin, self.H, self.W), generator=g, device=device, dtype=torch.float32).half()
        K = self.cin * 9
        q = torch.randint(-127, 128, (self.cout, K), generator=g, device=device, dtype=torch.int8)
        s = torch.rand((self.cout * K // 32,), generator=g, device=device) * (0.02 / 127)
        bias = 0.02 * torch.randn((self.cout,), generator=g, device=device)
        y = torch.empty((self.B, self.cout, self.H, self.W), device=device, dtype=torch.float32)
        import sdvk_b200

        nbytes = sdvk_b200.Context.conv3x3_workspace(self.cin, self.H, self.W, 1, sdvk_b200.F16)
        ws = torch.empty((nbytes,), dtype=torch.uint8, device=device)
        from sdvk_b200 import torch_ops

        xcl = x.permute(0, 2, 3, 1).contiguous()  # what the producer (GroupNorm+SiLU) writes in the UNet
        w16 = torch_ops.conv3x3_weights_f16(q, s)  # the load-time repack
        return x, q, s, bias, y, ws, xcl, w16

    def step(self, torch_ops, st):
        import sdvk_b200

        x, q, s, bias, y, ws, xcl, w16 = st
        torch_ops.context(x.device).conv3x3_nhwc(xcl.data_ptr(), w16.data_ptr(), bias.data_ptr(), 0, False,
                                                 y.data_ptr(), sdvk_b200.F32, self.B, self.cin, self.cout, self.H,
                                                 self.W, 1, -1)

    def e2e(self, sdvk_b200, ctx, torch, st):
        """Per step: pinned x -> device, sdvk_conv3x3_q8 (channels-last copy, weight repack, implicit GEMM),
        device y -> pinned host."""
        x, q, s, bias, y, ws = st[:6]
        xh = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
        xh.copy_(x.cpu())
        yh = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)

        def run():
            ctx.upload_async(x.data_ptr(), xh.data_ptr(), xh.numel() * 2)
            ctx.conv3x3_q8(x.data_ptr(), sdvk_b200.F16, q.data_ptr(), s.data_ptr(), bias.data_ptr(), y.data_ptr(),
                           sdvk_b200.F32, self.B, self.cin, self.cout, self.H, self.W, 1, -1, ws.data_ptr(),
                           ws.numel())
            ctx.download_async(yh.data_ptr(), y.data_ptr(), yh.numel() * 4)

        return run, xh.numel() * 2, yh.numel() * 4, "sdvk_upload_async + sdvk_conv3x3_q8 + sdvk_download_async"

    def host_inputs(self):
        from oracle import pyoracle

        rng = np.random.default_rng(1)
        x = rng.standard_normal((1, self.cin, self.H, self.W), dtype=np.float32).astype(np.float16).astype(np.float32)
        q, _, s = pyoracle.q8_weights(3, 0, self.cout, self.cin * 9)
        return x, q, s

    def cpu_run(self, inputs, channels):
        from oracle import pyoracle

        x, q, s = inputs
        K = self.cin * 9
        col = pyoracle.im2col3x3(x[0], 1, -1)
        pyoracle.gemm_nn_q8_shader(q[:channels], s[:channels * K // 32], col)
        return 2.0 * channels * self.H * self.W * K


class SamplerWorkload:
    """One model evaluation's sampler work at the SDXL 1024^2 latent (4 x 128 x 128 floats): the
    guidance combine, x0, the Euler update and the next scaled model input (the reference's default
    sampler and cfg 7.5; sdvkgen.cpp:3806-3846, 3770-3776, 4011-4019), one sdvk_sampler_step call.
    The reference runs this on the host between downloading the model output and uploading the next
    input."""

    dtype = "f32"
    unit = "GB/s"
    launches_per_step = 2  # guide pass, update pass

    def __init__(self, n=4 * 128 * 128):
        self.name = "sampler"
        self.n = n
        # eps_c, eps_u and lat read; x0, lat and the model input written
        self.bytes = 6.0 * 4 * n
        self.work = self.bytes
        self.flop = 12.0 * n
        self.bound = "hbm"
        self.metric = f"sampler step GB/s @ latent {n} floats, Euler, cfg 7.5"
        self.describe = (f"sampler step (evalGuided + x0FromEps + finishX0 + Euler update + input scaling) of an SDXL "
                         f"1024x1024 latent, {n} fp32 values, cond/uncond model outputs ~N(0,1)")
        self.rotate = max(2, -(-2 * L2_BYTES // int(5 * 4 * n)))
        self.cpu_units = 64
        self.cpu_what = "sampler evaluations (C++ restatement of the host loop, one thread)"

    def make_set(self, torch, device, seed):
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        n = self.n
        ec = torch.randn((n,), generator=g, device=device)
        eu = torch.randn((n,), generator=g, device=device)
        lat = torch.randn((n,), generator=g, device=device) * 3.0
        x0 = torch.empty_like(lat)
        xm = torch.empty_like(lat)
        return ec, eu, lat, x0, xm

    def _desc(self, sdvk_b200, st):
        ec, eu, lat, x0, xm = st
        d = sdvk_b200.SamplerStepDesc()
        d.kind, d.phase, d.n = sdvk_b200.SAMPLER_EULER, 0, self.n
        d.eps_c, d.eps_u, d.cfg = ec.data_ptr(), eu.data_ptr(), 7.5
        d.lat, d.x0, d.x_model = lat.data_ptr(), x0.data_ptr(), xm.data_ptr()
        d.sigma, d.sigma_next = 3.0, 2.5
        return d

    def step(self, torch_ops, st):
        import sdvk_b200

        torch_ops.context(st[0].device).sampler_step(self._desc(sdvk_b200, st))

    def e2e(self, sdvk_b200, ctx, torch, st):
        """Per step: pinned cond/uncond model outputs -> device, the sampler step, the next model input
        -> pinned host (the reference's downloadNow / host loop / uploadNow, reversed in direction)."""
        ec, eu, lat, x0, xm = st
        ech = torch.empty(ec.shape, dtype=ec.dtype, pin_memory=True)
        euh = torch.empty(eu.shape, dtype=eu.dtype, pin_memory=True)
        ech.copy_(ec.cpu())
        euh.copy_(eu.cpu())
        xmh = torch.empty(xm.shape, dtype=xm.dtype, pin_memory=True)
        d = self._desc(sdvk_b200, st)
        nb = self.n * 4

        def run():
            ctx.upload_async(ec.data_ptr(), ech.data_ptr(), nb)
            ctx.upload_async(eu.data_ptr(), euh.data_ptr(), nb)
            ctx.sampler_step(d)
            ctx.download_async(xmh.data_ptr(), xm.data_ptr(), nb)

        return run, 2 * nb, nb, "sdvk_upload_async x2 + sdvk_sampler_step + sdvk_download_async"

    def host_inputs(self):
        rng = np.random.default_rng(1)
        n = self.n
        return (rng.standard_normal(n).astype(np.float32), rng.standard_normal(n).astype(np.float32),
                (rng.standard_normal(n) * 3).astype(np.float32))

    def cpu_run(self, inputs, evals):
        from oracle import pyoracle

        ec, eu, lat0 = inputs
        lat = lat0.copy()
        x0, xm = np.empty_like(lat), np.empty_like(lat)
        for _ in range(evals):
            pyoracle.sampler_eval(kind=0, phase=0, n=self.n, eps_c=ec, eps_u=eu, cfg=7.5, lat=lat, x0=x0,
                                  x_model=xm, sigma=3.0, sigma_next=2.5)
        return evals * self.bytes


class UnetWorkload:
    """one denoising step of an SDXL 1024^2 CFG generation -- the whole UNet pass
    over the cond/uncond pair (batch 2, 4 x 128 x 128 latent, sdvk_unet_forward: unetForward,
    sdvkgen.cpp:1875-1973) followed by the device sampler step (guidance, v-prediction x0, the Euler
    update and the next scaled model input, sdvk_sampler_step).  A generation is 20 such steps, so the
    metric is images/s = 1 / (20 x s/step) per GPU; GPUs run independent images (weak scaling)."""

    name = "unet"
    unit = "images/s"
    dtype = "f16"
    bound = "tensor"
    steps_per_image = 20
    graph_len = 1
    default_steps = 10
    cfg = 5.0

    def __init__(self, B=2, H=128, W=128):
        self.B, self.H, self.W = B, H, W
        self.n = 4 * H * W
        self.unet = None
        self.flop = None  # set once the UNet exists (sdvk_unet_flops)
        self.work = 1.0 / self.steps_per_image  # images per step
        self.metric = "SDXL 1024^2 CFG UNet images/s (20 Euler steps, v-pred, cfg 5.0)"
        self.describe = ("SDXL UNet (320/640/1280, depths 0/2/10, hd 64, ctx 2048, adm 2816, GN 32) with random "
                         "Q8_0 weights (int8 U[-127,127], scale |N(0,0.02)|/127), batch 2 (cond/uncond) latent "
                         "4x128x128 fp32 ~N(0,1), context 2x77x2048 fp16 ~N(0,1), adm N(0,1); one step = UNet pass "
                         "+ sdvk_sampler_step (Euler, cfg 5.0, v-pred)")
        self.rotate = 1
        self.l2_note = ("one UNet pass reads 2.9 GB of Q8_0 weights and scales and several GB of activations per "
                        "step (>> 126 MB L2)")
        self.cpu_units = 9216
        self.cpu_what = ("rows of the 9216x1280x1280 Q8_0 GEMM (fp32 restatement of gemm_nt_q8_v.comp, the pass's "
                         "dominant arithmetic), converted to images/s at the pass's FLOP per image")
        self.bytes = 0

    def _ensure(self, torch, device):
        if self.unet is None:
            from sdvk_b200.unet import Unet

            self.unet = Unet(self.B, self.H, self.W, device=device.index)
            self.unet.init_random(3)
            self.flop = float(self.unet.flops)
            self.launches_per_step = self.unet.launches + 2  # + the sampler's guide and update passes
            # lower bound of the pass's DRAM traffic: every Q8_0 weight (int8 + fp32 scale per 32) read once
            from sdvk_b200 import UNET_Q8
            from sdvk_b200.unet import plan

            tens = plan(self.B, self.H, self.W)["tensors"].values()
            self.bytes = float(sum(r * c * 1.125 for kind, r, c in tens if kind == UNET_Q8))

    def make_set(self, torch, device, seed):
        self._ensure(torch, device)
        g = torch.Generator(device=device)
        g.manual_seed(seed)
        B, n = self.B, self.n
        lat = torch.randn((n,), generator=g, device=device) * 14.6
        xin = torch.empty((B, 4, self.H, self.W), device=device)
        xin[:] = (lat / math.sqrt(14.6 ** 2 + 1)).view(1, 4, self.H, self.W)
        ts = torch.full((B,), 999.0, device=device)
        adm = torch.randn((B, 2816), generator=g, device=device)
        ctx = torch.randn((B, 77, 2048), generator=g, device=device).half()
        out = torch.empty_like(xin)
        x0 = torch.empty((n,), device=device)
        return lat, xin, ts, adm, ctx, out, x0

    def _desc(self, sdvk_b200, st):
        lat, xin, ts, adm, ctx, out, x0 = st
        n = self.n
        d = sdvk_b200.SamplerStepDesc()
        d.kind, d.phase, d.n = sdvk_b200.SAMPLER_EULER, 0, n
        d.eps_c, d.eps_u, d.cfg, d.vpred = out.data_ptr(), out.data_ptr() + 4 * n, self.cfg, 1
        d.lat, d.x0, d.x_model = lat.data_ptr(), x0.data_ptr(), xin.data_ptr()
        d.sigma, d.sigma_next = 14.6, 12.0
        return d

    def _run(self, ctx, st, d):
        lat, xin, ts, adm, cx, out, x0 = st
        ctx._check(sdvk_b200_lib().sdvk_unet_forward(ctx.handle, self.unet._h, xin.data_ptr(), ts.data_ptr(),
                                                     adm.data_ptr(), cx.data_ptr(), 1, out.data_ptr()),
                   "sdvk_unet_forward")
        ctx.sampler_step(d)
        ctx.copy(xin.data_ptr() + 4 * self.n, xin.data_ptr(), 4 * self.n)  # the uncond half's input

    def step(self, torch_ops, st):
        import sdvk_b200

        self._run(torch_ops.context(st[0].device), st, self._desc(sdvk_b200, st))

    def e2e(self, sdvk_b200, ctx, torch, st):
        """Per step: pinned latent -> device, the UNet pass and the sampler step, the updated latent ->
        pinned host."""
        lat = st[0]
        lh = torch.empty(lat.shape, dtype=lat.dtype, pin_memory=True)
        lh.copy_(lat.cpu())
        d = self._desc(sdvk_b200, st)
        nb = self.n * 4

        def run():
            ctx.upload_async(lat.data_ptr(), lh.data_ptr(), nb)
            self._run(ctx, st, d)
            ctx.download_async(lh.data_ptr(), lat.data_ptr(), nb)

        return run, nb, nb, "sdvk_upload_async + sdvk_unet_forward + sdvk_sampler_step + sdvk_download_async"

    def host_inputs(self):
        return GemmWorkload().host_inputs()

    def cpu_run(self, inputs, rows):
        return GemmWorkload().cpu_run(inputs, rows)

    def cpu_value(self, flop_per_s):
        """images/s at the CPU restatement's FLOP rate (FLOP per image = 20 passes of the batch-2 pass)."""
        flop = self.flop if self.flop else UNET_PASS_FLOP
        return flop_per_s / (flop * self.steps_per_image)


class UnetPairWorkload(UnetWorkload):
    """BASELINE config 4's second mode: the CFG halves of one image on a GPU pair.  Each rank runs the
    UNet pass over its half (batch 1: rank 0 of the pair the conditional context, rank 1 the
    unconditional one), the pair all-gathers the 4 x 128 x 128 fp32 predictions over NCCL
    (sdvk_b200.cfg.CfgPair, 256 KB per rank), and both ranks run the same sampler step on the same
    bytes.  This halves the per-step latency of one image; images/s counts one image per pair."""

    name = "unet-cfg-pair"
    graph_len = 0  # eager steps: the pass is a captured graph, the all-gather runs between it and the sampler

    def __init__(self):
        super().__init__(B=1)
        self.work = 1.0 / (2 * self.steps_per_image)  # a rank's share of an image per step
        self.metric = "SDXL 1024^2 CFG UNet images/s (20 Euler steps, v-pred, cfg 5.0; CFG pair on 2 GPUs)"
        self.describe = self.describe.replace("batch 2 (cond/uncond)", "batch 1 per rank (cond on pair rank 0, "
                                              "uncond on pair rank 1) + NCCL all-gather of the prediction")
        self.pair = None
        self.graph = None

    def make_set(self, torch, device, seed):
        import torch.distributed as dist

        from sdvk_b200.cfg import CfgPair, pair_groups

        if self.pair is None:
            world = dist.get_world_size() if dist.is_initialized() else 1
            if world % 2:
                raise SystemExit("unet-cfg-pair needs an even number of GPUs")
            groups = pair_groups(world)
            self.pair = CfgPair(groups[dist.get_rank() // 2], self.cfg)
        lat, xin, ts, adm, ctx, out, x0 = super().make_set(torch, device, 7 + seed // 1000 // 2)
        g = torch.Generator(device=device)
        g.manual_seed(seed // 1000)
        ctx = torch.randn((1, 77, 2048), generator=g, device=device).half()  # this rank's half of the pair
        return lat, xin, ts, adm, ctx, out, x0

    def _run(self, ctx, st, d):
        import torch

        lat, xin, ts, adm, cx, out, x0 = st
        fwd = lambda: ctx._check(sdvk_b200_lib().sdvk_unet_forward(ctx.handle, self.unet._h, xin.data_ptr(),
                                                                   ts.data_ptr(), adm.data_ptr(), cx.data_ptr(), 1,
                                                                   out.data_ptr()), "sdvk_unet_forward")
        if self.graph is None and getattr(self, "_warm", False):
            self.graph = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream(out.device)
            s.wait_stream(torch.cuda.current_stream(out.device))
            with torch.cuda.graph(self.graph, stream=s):
                ctx.set_stream(s.cuda_stream)
                fwd()
            torch.cuda.current_stream(out.device).wait_stream(s)
            ctx.set_stream(torch.cuda.current_stream(out.device).cuda_stream)
        if self.graph is not None:
            self.graph.replay()
        else:
            fwd()
            self._warm = True
        cond, uncond = self.pair.exchange(out)
        d.eps_c, d.eps_u = cond.data_ptr(), uncond.data_ptr()
        ctx.sampler_step(d)

    def release(self):
        self.graph = None


# FLOP of the batch-2 SDXL 1024^2 pass as sdvk_unet_flops counts it (for the reference arm, which
# builds no UNet); bench runs of the sdvk arm print the live count in config.
UNET_PASS_FLOP = 13.0e12


def sdvk_b200_lib():
    import sdvk_b200

    return sdvk_b200.lib()


def wl_unit(wl):
    return getattr(wl, "unit", "TFLOP/s")


def wl_work(wl):
    """The workload's unit of work per step: FLOP, or bytes for the GB/s workloads."""
    return getattr(wl, "work", wl.flop)


def wl_scale(wl):
    return {"TFLOP/s": 1e12, "GB/s": 1e9}.get(wl_unit(wl), 1.0)


def wl_cpu_value(wl, flop_per_s):
    """A CPU sample's rate in the workload's unit."""
    conv = getattr(wl, "cpu_value", None)
    return conv(flop_per_s) if conv else flop_per_s / wl_scale(wl)


WORKLOADS = {
    "gemm": GemmWorkload,
    "groupnorm": GroupNormWorkload,
    "conv": ConvWorkload,
    "sampler": SamplerWorkload,
    "block": BlockWorkload,
    "unet": UnetWorkload,
    "unet-cfg-pair": UnetPairWorkload,
    "attn-self-4096": lambda: AttnWorkload("attn-self-4096", 2, 4096, 4096, 10),
    "attn-self-1024": lambda: AttnWorkload("attn-self-1024", 2, 1024, 1024, 20),
    "attn-cross-77": lambda: AttnWorkload("attn-cross-77", 2, 1024, 77, 20),
}


def usable_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def oracle_threads() -> int:
    """Every usable host core for the oracle's OpenMP loops, whatever OMP_NUM_THREADS says (torchrun
    sets it to 1 per rank)."""
    from oracle import pyoracle

    n = usable_cores()
    pyoracle.lib().orc_set_num_threads(n)
    return n


REF_PROGRAM = os.path.join(ROOT, "oracle", "_ref", "sdvkgen_host")
REF_SEED = 3        # the UNet seed both arms use (UnetWorkload._ensure)
REF_LATENT = 16     # the reference program's sample latent edge


def ref_model_args(workdir: str):
    """The seeded SDXL UNet as a GGUF file the reference's loader reads (cached between runs in the
    temp directory: 2.7 GB) and seeded embeddings, as the reference program's CLI options."""
    sys.path.insert(0, ROOT)
    from oracle import pyoracle, unet_gguf

    gguf = os.path.join(tempfile.gettempdir(), f"sdvk_bench_unet_seed{REF_SEED}.gguf")
    if not (os.path.exists(gguf) and os.path.getsize(gguf) > 2_000_000_000):
        tmp = gguf + f".{os.getpid()}.part"
        unet_gguf.write_gguf(tmp, REF_SEED)
        os.replace(tmp, gguf)
    files = {}
    ctx = pyoracle.normal_f32(11, 1, (2, 77, 2048))
    pool = pyoracle.normal_f32(11, 2, (2, 1280))
    for k, a in (("c", ctx[0]), ("u", ctx[1]), ("p", pool[0]), ("pu", pool[1])):
        files[k] = os.path.join(workdir, k + ".f32")
        np.ascontiguousarray(a, "<f4").tofile(files[k])
    return ["--unet", gguf, "--te1", gguf, "--te2", gguf, "--vae", gguf, "--emb-cond", files["c"], "--emb-uncond",
            files["u"], "--emb-pool", files["p"], "--emb-poolu", files["pu"]]


def ref_unet_sample(warmup: int, steps: int):
    """warmup + steps steps of the reference's own generation loop (Euler, v-pred, CFG 5: two UNet
    passes, the host CFG combine and the update per step) at a REF_LATENT^2 latent, each step timed
    by the wall clock between the program's step lines.  Returns the mean of the timed steps in
    seconds, the FLOP scale to the 128^2 latent and the core count."""
    sys.path.insert(0, ROOT)
    from sdvk_b200.unet import plan

    cores = usable_cores()
    with tempfile.TemporaryDirectory() as td:
        args = ref_model_args(td)
        env = dict(os.environ, OMP_NUM_THREADS=str(cores))
        cmd = [REF_PROGRAM, "x"] + args + ["--width", str(8 * REF_LATENT), "--height", str(8 * REF_LATENT), "--seed",
                                           "1", "--no-vae", "--latent-out", os.path.join(td, "lat.bin"), "--sampler",
                                           "euler", "--steps", str(warmup + steps), "--cfg", "5", "--vpred"]
        p = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, env=env, cwd=td)
        times, t_prev, tail = [], None, []
        for line in p.stdout:
            now = time.perf_counter()
            tail = (tail + [line])[-20:]
            if line.startswith("sampler "):
                t_prev = now
            elif line.startswith("step ") and t_prev is not None:
                times.append(now - t_prev)
                t_prev = now
        rc = p.wait()
    if rc != 0 or len(times) != warmup + steps:
        raise RuntimeError("reference program failed:\n" + "".join(tail))
    scale = plan(1, 128, 128)["flops"] / plan(1, REF_LATENT, REF_LATENT)["flops"]
    return statistics.mean(times[warmup:]), scale, cores


def cpu_sample(wl, budget_s, steps=None):
    """Time the reference arithmetic on a bounded sample of the workload.  With `steps` given (the
    reference arm), each step runs the same number of whole units (rows of X, query rows), sized
    from a probe so that the steps take about `budget_s` together.  Without it, whole workloads (or
    the largest unit count that fits) repeat until `budget_s` has passed.  Returns
    (FLOP per s, units per run, runs, seconds, threads)."""
    threads = oracle_threads()
    inputs = wl.host_inputs()
    probe = min(wl.cpu_units, 64)
    t0 = time.perf_counter()
    wl.cpu_run(inputs, probe)
    per_unit = (time.perf_counter() - t0) / probe
    per_run = budget_s / (steps or 1)
    units = int(max(8, min(wl.cpu_units, per_run / max(per_unit, 1e-9))))
    wl.cpu_run(inputs, units)  # warm-up at the timed size
    flop, runs, t0 = 0.0, 0, time.perf_counter()
    while True:
        flop += wl.cpu_run(inputs, units)
        runs += 1
        dt = time.perf_counter() - t0
        if (steps is not None and runs >= steps) or (steps is None and dt >= budget_s):
            break
    return flop / dt, units, runs, dt, threads


def run_reference(args, rank, world, wl):
    if rank != 0:
        return 0
    if isinstance(wl, UnetWorkload) and os.path.exists(REF_PROGRAM):
        return run_reference_program(args, world, wl)
    budget = 60.0
    fps, units, _, dt, threads = cpu_sample(wl, budget, steps=args.steps)
    value = wl_cpu_value(wl, fps)
    sample = f"{units} of {wl.cpu_units} {wl.cpu_what} per step"
    line = {
        "impl": "reference", "metric": wl.metric, "value": value, "unit": wl_unit(wl), "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": wl.describe, "sample_units": units},
        "cpu_baseline": {"value": value, "unit": wl_unit(wl), "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": wl_unit(wl), "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference Vulkan path unavailable on this box (no graphics stack); its shader arithmetic is timed "
                "as the oracle's C++ restatement on the host cores",
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference_program(args, world, wl):
    """The reference arm of the UNet workloads: the reference's own generation loop (ref_unet_sample)."""
    s_sample, scale, cores = ref_unet_sample(args.warmup, args.steps)
    s_step = s_sample * scale  # one CFG step (two batch-1 passes) at the 128^2 latent
    value = 1.0 / (wl.steps_per_image * s_step)
    sample = (f"{args.steps} timed steps (after {args.warmup}) of the reference's own generation loop "
              f"(oracle/_ref/sdvkgen_host: main.cpp + sdvkgen.cpp unchanged, shaders restated in C++, "
              f"{cores} OpenMP threads) at a {REF_LATENT}x{REF_LATENT} latent, Euler / v-pred / CFG 5, "
              f"{s_sample * 1e3:.0f} ms per step, scaled to 128x128 by the UNet FLOP ratio {scale:.1f}")
    line = {
        "impl": "reference", "metric": wl.metric, "value": value, "unit": wl_unit(wl), "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": s_step * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": wl.describe, "sample_latent": REF_LATENT,
                                        "flop_scale_to_full": scale},
        "cpu_baseline": {"value": value, "unit": wl_unit(wl), "cores": cores, "kind": "reference",
                         "sample": sample},
        "e2e": {"value": value, "unit": wl_unit(wl), "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "the reference's Vulkan engine is unavailable on this box (no graphics stack); its own UNet walker "
                "and generation loop run on the host stub engine",
    }
    print(json.dumps(line), flush=True)
    return 0


def kernel_lines(torch, torch_ops, device):
    """Config 0's GEMM and config 1's attentions, CUDA-event timed over CUDA-graph replays in this
    process (rotating inputs larger than L2), each against its roofline."""
    pk, pk_kind = peaks()
    cases = [("gemm_9216x1280x1280", GemmWorkload(), 2000),
             ("attn_self_4096", AttnWorkload("attn-self-4096", 2, 4096, 4096, 10), 400),
             ("attn_self_1024", AttnWorkload("attn-self-1024", 2, 1024, 1024, 20), 2000),
             ("attn_cross_77", AttnWorkload("attn-cross-77", 2, 1024, 77, 20), 2000)]
    out = {}
    cap = torch.cuda.Stream(device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(device.index) as clk:
        for key, wl, steps in cases:
            sets = [wl.make_set(torch, device, 77 + i) for i in range(wl.rotate)]
            for i in range(2 * wl.rotate):
                wl.step(torch_ops, sets[i % wl.rotate])
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                for i in range(GRAPH_LEN):
                    wl.step(torch_ops, sets[i % wl.rotate])
            reps = max(1, steps // GRAPH_LEN)
            g.replay()
            torch.cuda.synchronize()
            stream = torch.cuda.current_stream(device)
            ev0.record(stream)
            for _ in range(reps):
                g.replay()
            ev1.record(stream)
            torch.cuda.synchronize()
            us = ev0.elapsed_time(ev1) * 1e3 / (reps * GRAPH_LEN)
            if wl.bound == "tensor":
                ach, peak, unit = wl.flop / (us * 1e-6) / 1e12, pk["bf16_tflops"], "TFLOP/s"
            else:
                ach, peak, unit = wl.bytes / (us * 1e-6) / 1e9, pk["hbm_gbs"], "GB/s"
            out[key] = {"us_per_launch": us, "achieved": ach, "unit": unit, "peak": peak, "frac": ach / peak,
                        "bound": wl.bound, "flop": wl.flop, "bytes": wl.bytes, "traffic": profile_traffic(wl.name),
                        "launches": reps * GRAPH_LEN}
            del g, sets
            torch.cuda.synchronize()
    out["peak_kind"] = f"{pk_kind} (MEASURED_PEAKS.json: dense bf16 burst / HBM copy)"
    out["clocks"] = clk.summary()
    return out


def cfg_pair_line(torch, dist, device, rank, world, steps, warmup):
    """BASELINE config 4's second mode through the C ABI: rank 2p runs image p's conditional half and
    rank 2p + 1 its unconditional half (batch-1 UNet passes); each step's captured CUDA graph is the
    pass, sdvk_allgather of the two 4x128x128 fp32 predictions over the pair's NCCL communicator
    (sdvk_comm_create), and the sampler step on the gathered [cond | uncond] -- so both ranks update
    the same latent from the same bytes.  Every rank takes the same collective steps."""
    import sdvk_b200
    from sdvk_b200 import torch_ops
    from sdvk_b200.unet import Unet

    ctx = torch_ops.context(device)
    pair, prank = rank // 2, rank % 2
    uid = sdvk_b200.comm_unique_id() if prank == 0 else bytes(sdvk_b200.COMM_ID_BYTES)
    ids = [None] * world
    dist.all_gather_object(ids, uid)
    comm = sdvk_b200.Comm(ctx, 2, prank, ids[2 * pair], timeout_ms=60000)
    u = Unet(1, 128, 128, device=device.index)
    u.init_random(REF_SEED)
    n = 4 * 128 * 128
    g = torch.Generator(device=device)
    g.manual_seed(500 + pair)  # the same image on both ranks of the pair
    lat = torch.randn((n,), generator=g, device=device) * 14.6
    adm = torch.randn((1, 2816), generator=g, device=device)
    ctxs = torch.randn((2, 77, 2048), generator=g, device=device).half()
    cx = ctxs[prank:prank + 1].contiguous()  # this rank's half: cond or uncond
    xin = (lat / math.sqrt(14.6 ** 2 + 1)).view(1, 4, 128, 128).contiguous()
    ts = torch.full((1,), 999.0, device=device)
    out = torch.empty_like(xin)
    gathered = torch.empty((2, n), device=device)
    x0 = torch.empty((n,), device=device)
    d = sdvk_b200.SamplerStepDesc()
    d.kind, d.phase, d.n = sdvk_b200.SAMPLER_EULER, 0, n
    d.eps_c, d.eps_u, d.cfg, d.vpred = gathered.data_ptr(), gathered.data_ptr() + 4 * n, 5.0, 1
    d.lat, d.x0, d.x_model = lat.data_ptr(), x0.data_ptr(), xin.data_ptr()
    d.sigma, d.sigma_next = 14.6, 12.0
    lib = sdvk_b200.lib()

    def one_step():
        ctx._check(lib.sdvk_unet_forward(ctx.handle, u._h, xin.data_ptr(), ts.data_ptr(), adm.data_ptr(),
                                         cx.data_ptr(), 1, out.data_ptr()), "sdvk_unet_forward")
        comm.allgather(out.data_ptr(), gathered.data_ptr(), n, sdvk_b200.F32)
        ctx.sampler_step(d)

    cur = torch.cuda.current_stream(device)
    for _ in range(max(2, warmup)):
        ctx.set_stream(cur.cuda_stream)
        one_step()
    comm.wait()
    torch.cuda.synchronize()
    cap = torch.cuda.Stream(device)
    step_graph, ag_graph = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    cap.wait_stream(cur)
    # thread-local capture: NCCL's own threads keep making CUDA calls while this thread captures
    with torch.cuda.graph(step_graph, stream=cap, capture_error_mode="thread_local"):
        ctx.set_stream(cap.cuda_stream)
        one_step()
    with torch.cuda.graph(ag_graph, stream=cap, capture_error_mode="thread_local"):
        ctx.set_stream(cap.cuda_stream)
        for _ in range(20):
            comm.allgather(out.data_ptr(), gathered.data_ptr(), n, sdvk_b200.F32)
    cur.wait_stream(cap)
    ctx.set_stream(cur.cuda_stream)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def timed(graph, reps):
        graph.replay()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        ev0.record(cur)
        for _ in range(reps):
            graph.replay()
        ev1.record(cur)
        torch.cuda.synchronize()
        t = torch.tensor([ev0.elapsed_time(ev1)], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with ClockSampler(device.index) as clk:
        ms = timed(step_graph, steps) / steps
    ag_us = timed(ag_graph, 5) * 1e3 / (5 * 20)
    # both ranks of every pair must hold the same latent bytes
    lats = [torch.empty_like(lat) for _ in range(world)]
    dist.all_gather(lats, lat)
    same = all(torch.equal(lats[2 * p], lats[2 * p + 1]) for p in range(world // 2))
    del step_graph, ag_graph
    torch.cuda.synchronize()
    dist.barrier()
    comm.close()
    u.close()
    pairs = world // 2
    return {"pairs": pairs, "ms_per_step": ms, "images_per_s": pairs / (UnetWorkload.steps_per_image * ms * 1e-3),
            "allgather_us": ag_us, "allgather_bytes_per_rank": 4 * n, "latents_bit_identical": bool(same),
            "nccl_ranks_per_communicator": 2, "communicators": pairs, "steps": steps, "clocks": clk.summary(),
            "path": "sdvk_unet_forward (batch 1) + sdvk_allgather (C ABI over NCCL) + sdvk_sampler_step, "
                    "one CUDA graph per step, CUDA events, max over ranks"}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="timed steps (default: about 1 s of GPU work)")
    ap.add_argument("--warmup", type=int, default=100)
    ap.add_argument("--impl", default="sdvk", choices=["sdvk", "reference"])
    ap.add_argument("--workload", default="unet", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-kernels", action="store_true", help="unet: leave out the GEMM/attention sub-line")
    ap.add_argument("--no-cfg-pair", action="store_true", help="unet at N >= 2: leave out the CFG-pair sub-line")
    args = ap.parse_args(argv)
    args.warmup = max(3, args.warmup)
    wl = WORKLOADS[args.workload]()
    if args.steps is None:
        args.steps = 3 if args.impl == "reference" else getattr(wl, "default_steps", None) or (
            20000 if wl.flop < 5e10 else 5000)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world, wl)

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

    sets = [wl.make_set(torch, device, 1000 * rank + i) for i in range(wl.rotate)]
    ctx = torch_ops.context(device)

    def step(i):
        wl.step(torch_ops, sets[i % wl.rotate])

    # warm-up (also the first launch's attribute setup), then graphs of GRAPH_LEN steps; each eager
    # warm-up step is an NVTX range "step", so a profiler can select one step's launches
    # (ncu --nvtx --nvtx-include "step/")
    for i in range(args.warmup):
        torch.cuda.nvtx.range_push("step")
        step(i)
        torch.cuda.nvtx.range_pop()
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

    glen = getattr(wl, "graph_len", GRAPH_LEN)
    if glen == 0:  # the workload captures what it can itself and runs its steps eagerly
        full, rem = 0, 0
        step(0)
    else:
        full, rem = divmod(args.steps, glen)
    if full:
        graph_of(glen).replay()
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
            graph_of(glen).replay()
        if rem:
            graph_of(rem).replay()
        if glen == 0:
            for i in range(args.steps):
                step(i)
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
    value = world * wl_work(wl) * args.steps / (ms_max * 1e-3) / wl_scale(wl)

    # ---- end to end through the C ABI with pinned host buffers
    e2e_steps = min(args.steps, 100)
    ctx.set_stream(torch.cuda.current_stream(device).cuda_stream)
    run_e2e, h2d, d2h, path = wl.e2e(sdvk_b200, ctx, torch, sets[0])
    for _ in range(3):
        run_e2e()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev0.record()
    for _ in range(e2e_steps):
        run_e2e()
    ev1.record()
    torch.cuda.synchronize()
    t = torch.tensor([ev0.elapsed_time(ev1)], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e_ms = float(t.item()) / e2e_steps
    e2e_value = world * wl_work(wl) / (e2e_ms * 1e-3) / wl_scale(wl)

    # ---- CPU baseline (rank 0, N = 1 only): a bounded sample of the same workload
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if isinstance(wl, UnetWorkload) and os.path.exists(REF_PROGRAM):
            s_sample, scale, cores = ref_unet_sample(1, 3)
            cpu = {"value": 1.0 / (wl.steps_per_image * s_sample * scale), "unit": wl_unit(wl), "cores": cores,
                   "kind": "reference",
                   "sample": (f"3 steps (after 1) of the reference's own generation loop (oracle/_ref/sdvkgen_host, "
                              f"main.cpp + sdvkgen.cpp unchanged on the host stub engine) at a {REF_LATENT}x"
                              f"{REF_LATENT} latent, {s_sample * 1e3:.0f} ms per step, scaled to 128x128 by the "
                              f"UNet FLOP ratio {scale:.1f}")}
        else:
            fps, units, runs, secs, threads = cpu_sample(wl, budget_s=15.0)
            cpu = {"value": wl_cpu_value(wl, fps), "unit": wl_unit(wl), "cores": threads, "kind": "port",
                   "sample": f"{runs} x {units} of {wl.cpu_units} {wl.cpu_what}, {secs:.1f} s"}

    # ---- the metric's kernel half (config 0 GEMM, config 1 attention) and, at N >= 2, the CFG pair
    kernels = None
    if wl.name == "unet" and rank == 0 and not args.no_kernels:
        kernels = kernel_lines(torch, torch_ops, device)
    pair_line = None
    if wl.name == "unet" and world >= 2 and world % 2 == 0 and not args.no_cfg_pair:
        pair_line = cfg_pair_line(torch, dist, device, rank, world, min(args.steps, 20), args.warmup)

    pk, pk_kind = peaks()
    achieved_tf = wl.flop / (ms_per_step * 1e-3) / 1e12
    achieved_gbs = wl.bytes / (ms_per_step * 1e-3) / 1e9
    if wl.bound == "tensor":
        roof = {"bound": "tensor", "achieved": achieved_tf, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                "frac": achieved_tf / pk["bf16_tflops"], "peak_kind": f"{pk_kind} dense bf16 burst"}
    else:
        roof = {"bound": "hbm", "achieved": achieved_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                "frac": achieved_gbs / pk["hbm_gbs"], "peak_kind": f"{pk_kind} HBM copy"}
    roof.update({"traffic": profile_traffic(wl.name), "algorithmic_flop_per_launch": wl.flop,
                 "algorithmic_bytes_per_launch": wl.bytes})
    if rank == 0:
        line = {
            "metric": wl.metric, "value": value, "unit": wl_unit(wl), "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": wl.dtype, "data": "synthetic",
            "config": {"workload": wl.describe,
                       "parallelism": (f"CFG pairs x{world // 2} (NCCL all-gather per step)"
                                       if getattr(wl, "pair", None) is not None else f"replicas x{world}"),
                       "l2": getattr(wl, "l2_note", None) or
                       f"{wl.rotate} rotating input/output sets ({wl.rotate * wl.bytes / 1e6:.0f} MB > 126 MB L2)",
                       "timing": (f"CUDA events over CUDA-graph replays of {glen} step(s)" if glen else
                                  "CUDA events over eager steps (the UNet pass replayed from a CUDA graph)")},
            "roofline": roof,
            "e2e": {"value": e2e_value, "unit": wl_unit(wl), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms, "path": path + ", pinned host buffers"},
            "gpu_launches": args.steps * getattr(wl, "launches_per_step", 1),
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        if kernels is not None:
            line["kernels"] = kernels
        if pair_line is not None:
            line["cfg_pair"] = pair_line
        print(json.dumps(line), flush=True)
    for g in graphs.values():
        del g
    graphs.clear()
    if hasattr(wl, "release"):
        wl.release()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
