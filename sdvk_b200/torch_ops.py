"""The sdvk hot-path calls on torch CUDA tensors.

torch provides device memory and the stream (the context runs on torch's current stream); the
arithmetic is libsdvk_b200.so's CUDA kernels.  One Context per device is cached.
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import torch

from . import BF16, F16, F32, AttnDesc, BlockDesc, Context, Q8Linear

_CTX: Dict[int, Context] = {}
_DT = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}


def context(device: Optional[torch.device] = None) -> Context:
    dev = torch.cuda.current_device() if device is None else torch.device(device).index
    if dev is None:
        dev = torch.cuda.current_device()
    ctx = _CTX.get(dev)
    if ctx is None:
        ctx = Context(dev)
        _CTX[dev] = ctx
    ctx.set_stream(torch.cuda.current_stream(dev).cuda_stream)
    return ctx


def _dt(t: torch.Tensor) -> int:
    if t.dtype not in _DT:
        raise TypeError(f"unsupported dtype {t.dtype}")
    return _DT[t.dtype]


def gemm_q8_nt(a: torch.Tensor, q: torch.Tensor, s: torch.Tensor, bias: Optional[torch.Tensor] = None,
               out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float32,
               accumulate: bool = False) -> torch.Tensor:
    """C[..., M, N] = A[..., M, K] . (q[N, K] * s)^T (+ bias).  A is 2-D or 3-D (batch, M, K)."""
    assert q.dtype == torch.int8 and s.dtype == torch.float32
    N, K = q.shape
    a3 = a if a.dim() == 3 else a.unsqueeze(0)
    B, M, Ka = a3.shape
    assert Ka == K and a3.stride(2) == 1
    if out is None:
        out = torch.empty((B, M, N) if a.dim() == 3 else (M, N), dtype=out_dtype, device=a.device)
    o3 = out if out.dim() == 3 else out.unsqueeze(0)
    ctx = context(a.device)
    ctx.gemm_q8_nt(a3.data_ptr(), _dt(a3), q.data_ptr(), s.data_ptr(), bias.data_ptr() if bias is not None else None,
                   o3.data_ptr(), _dt(o3), M, N, K, a3.stride(1), o3.stride(1), B, a3.stride(0) if B > 1 else 0,
                   o3.stride(0) if B > 1 else 0, accumulate)
    return out


def gemm_q8_nn(q: torch.Tensor, s: torch.Tensor, b: torch.Tensor, bias: Optional[torch.Tensor] = None,
               out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float32,
               accumulate: bool = False) -> torch.Tensor:
    """C[..., M, N] = (q[M, K] * s) . B[..., K, N] (+ bias[M])."""
    assert q.dtype == torch.int8 and s.dtype == torch.float32
    M, K = q.shape
    b3 = b if b.dim() == 3 else b.unsqueeze(0)
    Bt, Kb, N = b3.shape
    assert Kb == K and b3.stride(2) == 1
    if out is None:
        out = torch.empty((Bt, M, N) if b.dim() == 3 else (M, N), dtype=out_dtype, device=b.device)
    o3 = out if out.dim() == 3 else out.unsqueeze(0)
    ctx = context(b.device)
    ctx.gemm_q8_nn(q.data_ptr(), s.data_ptr(), b3.data_ptr(), _dt(b3), bias.data_ptr() if bias is not None else None,
                   o3.data_ptr(), _dt(o3), M, N, K, q.stride(0), b3.stride(1), o3.stride(1), Bt, 0,
                   b3.stride(0) if Bt > 1 else 0, o3.stride(0) if Bt > 1 else 0, accumulate)
    return out


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, scale: Optional[float] = None,
              causal: bool = False, out: Optional[torch.Tensor] = None,
              out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """Fused attention on token-major activations [B, T, heads*hd] (head h at columns h*hd..)."""
    q3 = q if q.dim() == 3 else q.unsqueeze(0)
    k3 = k if k.dim() == 3 else k.unsqueeze(0)
    v3 = v if v.dim() == 3 else v.unsqueeze(0)
    B, Tq, C = q3.shape
    Tk = k3.shape[1]
    hd = C // heads
    assert C == heads * hd and k3.shape[2] == C and v3.shape[2] == C
    if out is None:
        od = out_dtype or (torch.float32 if q.dtype == torch.float32 else torch.float16)
        out = torch.empty(q.shape, dtype=od, device=q.device)
    o3 = out if out.dim() == 3 else out.unsqueeze(0)
    d = AttnDesc()
    d.q, d.k, d.v, d.o = q3.data_ptr(), k3.data_ptr(), v3.data_ptr(), o3.data_ptr()
    d.dtype, d.o_dtype = _dt(q3), _dt(o3)
    d.batch, d.heads, d.Tq, d.Tk, d.hd = B, heads, Tq, Tk, hd
    d.ldq, d.ldk, d.ldv, d.ldo = q3.stride(1), k3.stride(1), v3.stride(1), o3.stride(1)
    d.sq, d.sk, d.sv, d.so = q3.stride(0), k3.stride(0), v3.stride(0), o3.stride(0)
    d.hq = d.hk = d.hv = d.ho = hd
    d.scale = (1.0 / math.sqrt(hd)) if scale is None else scale
    d.causal = int(causal)
    context(q.device).attention(d)
    return out


def layernorm(x: torch.Tensor, gamma: Optional[torch.Tensor], beta: Optional[torch.Tensor], eps: float = 1e-5,
              out_dtype: torch.dtype = torch.float16, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """LayerNorm over the last dim of fp32 x (layernorm_fwd.comp)."""
    assert x.dtype == torch.float32 and x.stride(-1) == 1
    d = x.shape[-1]
    x2 = x.reshape(-1, d)
    if out is None:
        out = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    o2 = out.view(-1, d)
    context(x.device).layernorm(x2.data_ptr(), gamma.data_ptr() if gamma is not None else None,
                                beta.data_ptr() if beta is not None else None, o2.data_ptr(), _dt(o2), x2.shape[0], d,
                                x2.stride(0), o2.stride(0), eps)
    return out


def geglu(h: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = h[..., :F] * gelu_erf(h[..., F:]) on f16 h of width 2F."""
    assert h.dtype == torch.float16 and h.stride(-1) == 1
    F = h.shape[-1] // 2
    h2 = h.reshape(-1, 2 * F)
    if out is None:
        out = torch.empty(h.shape[:-1] + (F,), dtype=torch.float16, device=h.device)
    o2 = out.view(-1, F)
    context(h.device).geglu(h2.data_ptr(), o2.data_ptr(), h2.shape[0], F, h2.stride(0), o2.stride(0))
    return out


def q8_linear(q: torch.Tensor, s: torch.Tensor, bias: Optional[torch.Tensor] = None) -> Q8Linear:
    return Q8Linear(q.data_ptr(), s.data_ptr(), bias.data_ptr() if bias is not None else None)


def transformer_block(x: torch.Tensor, ctx: torch.Tensor, heads: int, weights: dict,
                      workspace: Optional[torch.Tensor] = None, eps: float = 1e-5) -> torch.Tensor:
    """One BasicTransformerBlock on fp32 x [B, T, C] in place.  `weights` maps ln1_w ... ln3_b to fp32
    tensors and q, k, v, o, q2, k2, v2, o2, ff1, ff2 to (int8 [N, K], fp32 scales, fp32 bias or None)."""
    assert x.dtype == torch.float32 and x.is_contiguous() and ctx.is_contiguous()
    B, T, C = x.shape
    d = BlockDesc()
    d.x, d.ctx, d.ctx_dtype = x.data_ptr(), ctx.data_ptr(), _dt(ctx)
    d.batch, d.T, d.C, d.heads = B, T, C, heads
    d.Tctx, d.Cctx = ctx.shape[1], ctx.shape[2]
    d.ff_inner = weights["ff2"][0].shape[1]
    for name in ("ln1_w", "ln1_b", "ln2_w", "ln2_b", "ln3_w", "ln3_b"):
        t = weights.get(name)
        setattr(d, name, t.data_ptr() if t is not None else None)
    for name in ("q", "k", "v", "o", "q2", "k2", "v2", "o2", "ff1", "ff2"):
        setattr(d, name, q8_linear(*weights[name]))
    d.eps = eps
    d.ff1_geglu_interleaved = int(bool(weights.get("ff1_geglu_interleaved", False)))
    need = Context.block_workspace(d)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    context(x.device).transformer_block(d, workspace.data_ptr(), workspace.numel() * workspace.element_size())
    return x


def cfg_combine(cond: torch.Tensor, uncond: torch.Tensor, cfg: float, rescale: float = 0.0,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """uncond + cfg * (cond - uncond), with the optional spread rescale (sdvk_cfg_combine), fp32."""
    assert cond.dtype == torch.float32 and uncond.dtype == torch.float32 and cond.shape == uncond.shape
    c, u = cond.contiguous(), uncond.contiguous()
    if out is None:
        out = torch.empty_like(c)
    context(c.device).cfg_combine(c.data_ptr(), u.data_ptr(), out.data_ptr(), c.numel(), cfg, rescale)
    return out


def q8_0_ingest(blocks: torch.Tensor, rows: int, cols: int, ldq: int = 0):
    """Split raw GGUF Q8_0 blocks (uint8 on the device, rows*cols/32 blocks of 34 bytes) into the int8
    payload [rows, ldq or cols] and fp32 scales [rows * (ldq or cols) / 32] (sdvk_q8_0_ingest)."""
    assert blocks.dtype == torch.uint8 and blocks.is_contiguous() and blocks.numel() == rows * cols // 32 * 34
    ld = ldq or cols
    q = torch.zeros((rows, ld), dtype=torch.int8, device=blocks.device)
    s = torch.zeros((rows * ld // 32,), dtype=torch.float32, device=blocks.device)
    context(blocks.device).q8_0_ingest(blocks.data_ptr(), rows, cols, q.data_ptr(), ld, s.data_ptr())
    return q, s


def conv3x3_q8(x: torch.Tensor, q: torch.Tensor, s: torch.Tensor, bias: Optional[torch.Tensor] = None,
               stride: int = 1, pad_off: int = -1, out_dtype: torch.dtype = torch.float32,
               workspace_bytes: Optional[int] = None) -> torch.Tensor:
    """3x3 convolution of x [B, cin, H, W] with a Q8_0 weight q [cout, cin*9] (+ fp32 scales, bias)
    (sdvk_conv3x3_q8; conv3RawInto / conv3s2)."""
    assert x.is_contiguous() and x.dim() == 4 and q.dtype == torch.int8
    B, cin, H, W = x.shape
    cout = q.shape[0]
    OH, OW = (H, W) if stride == 1 else (H // 2, W // 2)
    y = torch.empty((B, cout, OH, OW), dtype=out_dtype, device=x.device)
    ctx = context(x.device)
    nbytes = workspace_bytes or ctx.conv3x3_workspace(cin, H, W, stride, _dt(x))
    ws = torch.empty((max(nbytes, 16),), dtype=torch.uint8, device=x.device)
    ctx.conv3x3_q8(x.data_ptr(), _dt(x), q.data_ptr(), s.data_ptr(), bias.data_ptr() if bias is not None else None,
                   y.data_ptr(), _dt(y), B, cin, cout, H, W, stride, pad_off, ws.data_ptr(), nbytes)
    return y


def conv3x3_weights_f16(q: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    """The fp16 tap-major repack of a Q8_0 conv weight q [cout, cin*9] for conv3x3_nhwc
    (sdvk_conv3x3_weights_f16; cin % 64 == 0)."""
    assert q.dtype == torch.int8 and q.is_contiguous() and q.dim() == 2 and q.shape[1] % 9 == 0
    cout, K = q.shape
    w16 = torch.empty((cout, K), dtype=torch.float16, device=q.device)
    context(q.device).conv3x3_weights_f16(q.data_ptr(), s.data_ptr(), cout, K // 9, w16.data_ptr())
    return w16


def conv3x3_nhwc(x: torch.Tensor, w16: torch.Tensor, bias: Optional[torch.Tensor] = None, stride: int = 1,
                 pad_off: int = -1, out_dtype: torch.dtype = torch.float32, bias_stride: int = 0,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The implicit-GEMM 3x3 convolution (sdvk_conv3x3_nhwc) of channels-last fp16 x [B, H, W, cin] with
    w16 from conv3x3_weights_f16: y [B, cout, OH, OW], or y += conv when `out` is given (fp32)."""
    assert x.dtype == torch.float16 and x.is_contiguous() and x.dim() == 4
    B, H, W, cin = x.shape
    cout = w16.shape[0]
    OH, OW = (H, W) if stride == 1 else (H // 2, W // 2)
    y = out if out is not None else torch.empty((B, cout, OH, OW), dtype=out_dtype, device=x.device)
    context(x.device).conv3x3_nhwc(x.data_ptr(), w16.data_ptr(), bias.data_ptr() if bias is not None else None,
                                   bias_stride, out is not None, y.data_ptr(), _dt(y), B, cin, cout, H, W, stride,
                                   pad_off)
    return y


def groupnorm_cl(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, groups: int = 32, eps: float = 1e-5,
                 silu: bool = False) -> torch.Tensor:
    """GroupNorm (+SiLU) of fp32 x [B, C, *spatial] written channels-last as fp16 [B, P, C]
    (sdvk_groupnorm_cl)."""
    assert x.dtype == torch.float32 and x.is_contiguous() and x.dim() >= 2
    B, C = x.shape[0], x.shape[1]
    P = x.numel() // (B * C)
    out = torch.empty((B, P, C), dtype=torch.float16, device=x.device)
    ctx = context(x.device)
    nbytes = ctx.groupnorm_workspace(B, C, P, groups)
    ws = torch.empty((max(nbytes, 16),), dtype=torch.uint8, device=x.device)
    ctx.groupnorm_cl(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), out.data_ptr(), B, C, P, groups, eps, silu,
                     ws.data_ptr(), ws.numel())
    return out


def groupnorm(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, groups: int = 32, eps: float = 1e-5,
              silu: bool = False, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """GroupNorm (+SiLU) of fp32 x [B, C, *spatial] (groupnorm.comp), via sdvk_groupnorm."""
    assert x.dtype == torch.float32 and x.is_contiguous() and x.dim() >= 2
    B, C = x.shape[0], x.shape[1]
    P = x.numel() // (B * C)
    if out is None:
        out = torch.empty_like(x)
    ctx = context(x.device)
    nbytes = ctx.groupnorm_workspace(B, C, P, groups)
    ws = torch.empty((max(nbytes, 16),), dtype=torch.uint8, device=x.device)
    ctx.groupnorm(x.data_ptr(), gamma.data_ptr(), beta.data_ptr(), out.data_ptr(), B, C, P, groups, eps, silu,
                  ws.data_ptr(), ws.numel())
    return out


def geglu_interleave(q: torch.Tensor, s: torch.Tensor, bias: Optional[torch.Tensor] = None):
    """Repack an ff.net.0.proj Q8_0 weight [2F, K] for the GEGLU epilogue (sdvk_geglu_interleave)."""
    two_f, K = q.shape
    F = two_f // 2
    qo, so = torch.empty_like(q), torch.empty_like(s)
    bo = torch.empty_like(bias) if bias is not None else None
    context(q.device).geglu_interleave(q.data_ptr(), s.data_ptr(), bias.data_ptr() if bias is not None else None,
                                       F, K, qo.data_ptr(), so.data_ptr(), bo.data_ptr() if bo is not None else None)
    return qo, so, bo


def gemm_q8_nt_geglu(a: torch.Tensor, q_il: torch.Tensor, s_il: torch.Tensor, bias_il: Optional[torch.Tensor] = None,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """a . W^T (+ bias) with GEGLU in the epilogue, for a weight repacked by geglu_interleave: [M, F] f16."""
    M, K = a.shape
    F = q_il.shape[0] // 2
    if out is None:
        out = torch.empty((M, F), dtype=torch.float16, device=a.device)
    context(a.device).gemm_q8_nt_geglu(a.data_ptr(), _dt(a), q_il.data_ptr(), s_il.data_ptr(),
                                       bias_il.data_ptr() if bias_il is not None else None, out.data_ptr(), M, F, K,
                                       a.stride(0), out.stride(0))
    return out
