"""TEST INFRASTRUCTURE ONLY: numpy/ctypes front end of liboracle.so (see oracle.h).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this module, as the
checker or the timed CPU baseline.  The product (sdvk_b200) never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_DIR = os.path.join(HERE, "_ref")
REF_GGUF = os.path.join(REF_DIR, "libref_gguf.so")

_lib = None
_P, _U32, _U64, _I, _F = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int, ctypes.c_float

_SIG = {
    "orc_mt19937_new": (_P, [_U32]),
    "orc_mt19937_free": (None, [_P]),
    "orc_mt19937_uniform_f32": (None, [_P, _F, _F, _P, _U64]),
    "orc_mt19937_uniform_int": (None, [_P, ctypes.c_int32, ctypes.c_int32, _P, _U64]),
    "orc_normal_f32": (None, [_U64, _U64, _F, _P, _U64]),
    "orc_normal_f16": (None, [_U64, _U64, _F, _P, _U64]),
    "orc_q8_weights": (None, [_U64, _U64, _U64, _U64, _P, _P, _P]),
    "orc_f32_to_f16": (None, [_P, _P, _U64]),
    "orc_f16_to_f32": (None, [_P, _P, _U64]),
    "orc_q8_0_pack_blocks": (None, [_P, _P, _U64, _P]),
    "orc_q8_0_split_blocks": (None, [_P, _U64, _P, _P]),
    "orc_gguf_write_q8": (_I, [ctypes.c_char_p, ctypes.c_char_p, _U64, _U64, _P]),
    "orc_gemm_nt_q8_shader": (None, [_P, _P, _P, _P, _P] + [_U32] * 9),
    "orc_gemm_nt_q8_f64": (None, [_P, _P, _P, _P, _P] + [_U32] * 8),
    "orc_gemm_nn_q8_shader": (None, [_P, _P, _P, _P] + [_U32] * 11),
    "orc_gemm_nn_q8_f64": (None, [_P, _P, _P, _P] + [_U32] * 9),
    "orc_attn_tiled_shader": (_I, [_P, _P, _P, _P] + [_U32] * 5 + [_F]),
    "orc_attn_simple_shader": (_I, [_P, _P, _P, _P] + [_U32] * 5 + [_F]),
    "orc_fused_attention": (_I, [_P, _P, _P, _P] + [_U32] * 5 + [_I]),
    "orc_attn_f64": (None, [_P, _P, _P, _P] + [_U32] * 5 + [_U64] * 8 + [_U32, ctypes.c_double]),
    "orc_layernorm_shader": (None, [_P, _P, _P, _P, _U32, _U32, _F, _U32]),
    "orc_groupnorm_shader": (None, [_P, _P, _P, _P, _U32, _U32, _U32, _F, _U32]),
    "orc_layernorm_f64": (None, [_P, _P, _P, _P, _U32, _U32, ctypes.c_double]),
    "orc_gelu_erf_shader": (None, [_P, _P, _U64]),
    "orc_cfg_combine": (None, [_P, _P, _P, _U64, _F, _F]),
    "orc_sampler_eval": (_U64, [_P]),
    "orc_add2_shader": (None, [_P, _P, _P, _U32]),
    "orc_bias_add_shader": (None, [_P, _P, _U32, _U32]),
    "orc_copy_nd_shader": (None, [_P, _P, _P]),
    "orc_ew2_shader": (None, [_P, _P, _P, _P]),
    "orc_unary_shader": (None, [_P, _P, _U32, _U32]),
    "orc_upsample2x_shader": (None, [_P, _P, _U32, _U32, _U32]),
    "orc_im2col_shader": (None, [_P, _P] + [_U32] * 5),
    "orc_im2col_s2_shader": (None, [_P, _P] + [_U32] * 5 + [ctypes.c_int32]),
    "orc_gemm_fp32_shader": (None, [_I, _P, _P, _P, _P, _U32]),
    "orc_softmax_shader": (None, [_P, _P, _U32, _U32]),
    "orc_causal_mask_shader": (None, [_P, _U32, _U32, _U32]),
    "orc_gen_rng_new": (_P, [_U32]),
    "orc_gen_rng_free": (None, [_P]),
    "orc_gen_rng_normal": (None, [_P, _P, _U64]),
    "orc_euler_schedule": (_F, [_I, _I, _I, _I, _I, _P, _P]),
    "orc_num_threads": (_I, []),
    "orc_set_num_threads": (None, [_I]),
}


def build() -> None:
    """Build liboracle.so (and, when the reference sources are present, the _ref/ checkers)."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True)
    ref = os.environ.get("SDVK_REFERENCE", "")
    if ref and os.path.isdir(ref):
        subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={ref}"], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        for k, (r, a) in _SIG.items():
            f = getattr(L, k)
            f.restype = r
            f.argtypes = a
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ------------------------------------------------------------------------------ RNG
class MT19937:
    """std::mt19937 with libstdc++'s uniform distributions (the reference tests' RNG)."""

    def __init__(self, seed: int):
        self.h = lib().orc_mt19937_new(seed)

    def uniform_f32(self, n: int, lo=-1.0, hi=1.0) -> np.ndarray:
        out = np.empty(n, np.float32)
        lib().orc_mt19937_uniform_f32(self.h, lo, hi, _p(out), n)
        return out

    def uniform_int(self, n: int, lo: int, hi: int) -> np.ndarray:
        out = np.empty(n, np.int32)
        lib().orc_mt19937_uniform_int(self.h, lo, hi, _p(out), n)
        return out

    def __del__(self):
        try:
            lib().orc_mt19937_free(self.h)
        except Exception:
            pass


def normal_f32(seed: int, stream: int, shape, std: float = 1.0) -> np.ndarray:
    out = np.empty(int(np.prod(shape)), np.float32)
    lib().orc_normal_f32(seed, stream, std, _p(out), out.size)
    return out.reshape(shape)


def normal_f16(seed: int, stream: int, shape, std: float = 1.0) -> np.ndarray:
    out = np.empty(int(np.prod(shape)), np.uint16)
    lib().orc_normal_f16(seed, stream, std, _p(out), out.size)
    return out.view(np.float16).reshape(shape)


def q8_weights(seed: int, stream: int, rows: int, cols: int):
    """BASELINE config-0 Q8_0 weight: (int8 [rows, cols], fp16 scales, fp32 scales [rows*cols/32])."""
    q = np.empty(rows * cols, np.int8)
    d16 = np.empty(rows * cols // 32, np.uint16)
    d32 = np.empty(rows * cols // 32, np.float32)
    lib().orc_q8_weights(seed, stream, rows, cols, _p(q), _p(d16), _p(d32))
    return q.reshape(rows, cols), d16.view(np.float16), d32


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = _c(x, np.float32)
    out = np.empty(x.size, np.uint16)
    lib().orc_f32_to_f16(_p(x), _p(out), x.size)
    return out.view(np.float16).reshape(x.shape)


def f16_to_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x).view(np.uint16)
    out = np.empty(x.size, np.float32)
    lib().orc_f16_to_f32(_p(x), _p(out), x.size)
    return out.reshape(x.shape)


# ------------------------------------------------------------------------------ GGUF Q8_0
def q8_0_pack(q: np.ndarray, d16: np.ndarray) -> np.ndarray:
    q = _c(q, np.int8).ravel()
    d = np.ascontiguousarray(d16).view(np.uint16).ravel()
    out = np.empty(d.size * 34, np.uint8)
    lib().orc_q8_0_pack_blocks(_p(q), _p(d), d.size, _p(out))
    return out


def q8_0_split(blocks: np.ndarray):
    blocks = _c(blocks, np.uint8)
    nb = blocks.size // 34
    q = np.empty(nb * 32, np.int8)
    s = np.empty(nb, np.float32)
    lib().orc_q8_0_split_blocks(_p(blocks), nb, _p(q), _p(s))
    return q, s


def gguf_write_q8(path: str, name: str, rows: int, cols: int, blocks: np.ndarray) -> None:
    blocks = _c(blocks, np.uint8)
    if lib().orc_gguf_write_q8(path.encode(), name.encode(), rows, cols, _p(blocks)) != 0:
        raise OSError(f"cannot write {path}")


# ------------------------------------------------------------------------------ GEMMs
def gemm_nt_q8_shader(A, q, s, bias=None, C=None, mode=0, batch=1, sA=0, sC=0, lda=0, ldc=0, M=None, N=None, K=None):
    A = _c(A, np.float32)
    q = _c(q, np.int8)
    s = _c(s, np.float32)
    N = q.shape[0] if N is None else N
    K = q.shape[1] if K is None else K
    M = (A.shape[-2] if A.ndim >= 2 else 1) if M is None else M
    if C is None:
        C = np.zeros((batch, M, ldc or N) if batch > 1 else (M, ldc or N), np.float32)
    b = _c(bias, np.float32) if bias is not None else None
    lib().orc_gemm_nt_q8_shader(_p(A), _p(q), _p(s), _p(b) if b is not None else None, _p(C), M, N, K, mode, sA, sC,
                                batch, lda, ldc)
    return C


def gemm_nt_q8_f64(A, q, s, bias=None, batch=1, sA=0, lda=0):
    A = _c(A, np.float32)
    q = _c(q, np.int8)
    s = _c(s, np.float32)
    N, K = q.shape
    M = A.shape[-2]
    C = np.zeros((batch, M, N) if batch > 1 else (M, N), np.float64)
    b = _c(bias, np.float32) if bias is not None else None
    lib().orc_gemm_nt_q8_f64(_p(A), _p(q), _p(s), _p(b) if b is not None else None, _p(C), M, N, K, sA or M * K,
                             M * N, batch, lda, 0)
    return C


def gemm_nn_q8_shader(q, s, B, mode=0, batch=1, sA=0, sB=0, sC=0, lda=0, ldb=0, ldc=0, C=None):
    q = _c(q, np.int8)
    s = _c(s, np.float32)
    B = _c(B, np.float32)
    M, K = q.shape[-2], q.shape[-1]
    N = B.shape[-1]
    if C is None:
        C = np.zeros((batch, M, N) if batch > 1 else (M, N), np.float32)
    lib().orc_gemm_nn_q8_shader(_p(q), _p(s), _p(B), _p(C), M, N, K, mode, sA, sB, sC, batch, lda, ldb, ldc)
    return C


def gemm_nn_q8_f64(q, s, B, batch=1):
    q = _c(q, np.int8)
    s = _c(s, np.float32)
    B = _c(B, np.float32)
    M, K = q.shape
    N = B.shape[-1]
    C = np.zeros((batch, M, N) if batch > 1 else (M, N), np.float64)
    lib().orc_gemm_nn_q8_f64(_p(q), _p(s), _p(B), _p(C), M, N, K, K * N, M * N, batch, 0, 0, 0)
    return C


# ------------------------------------------------------------------------------ 3x3 convolution
def im2col3x3(x, stride=1, off=-1):
    """im2col.comp (stride 1, pad 1) / im2col_s2.comp (stride 2, pad offset off) for one image x [C, H, W]:
    col[k, p], k = c*9 + ky*3 + kx, p = oh*OW + ow (pure data movement, exact)."""
    x = np.asarray(x)
    C, H, W = x.shape
    if stride == 1:
        off = -1
    OH, OW = (H, W) if stride == 1 else (H // 2, W // 2)
    pad = np.zeros((C, H + 3, W + 3), x.dtype)  # room for offsets -1..+2 on both axes
    pad[:, 1:H + 1, 1:W + 1] = x
    col = np.empty((C, 3, 3, OH, OW), x.dtype)
    for ky in range(3):
        for kx in range(3):
            ih = np.arange(OH) * stride + ky + off + 1
            iw = np.arange(OW) * stride + kx + off + 1
            col[:, ky, kx] = pad[:, ih][:, :, iw]
    return col.reshape(C * 9, OH * OW)


def conv3x3_shader(x, q, s, bias, stride=1, off=-1):
    """conv3RawInto / conv3s2 (sdvkgen.cpp:1133-1175) in fp32: im2col, gemm_nn_q8_v.comp, biasAddCh."""
    x = np.asarray(x, np.float32)
    out = []
    for xi in x:
        col = im2col3x3(xi, stride, off)
        y = gemm_nn_q8_shader(q, s, col)
        if bias is not None:
            y = y + np.asarray(bias, np.float32)[:, None]
        out.append(y)
    H, W = x.shape[2], x.shape[3]
    OH, OW = (H, W) if stride == 1 else (H // 2, W // 2)
    return np.stack(out).reshape(x.shape[0], -1, OH, OW)


def conv3x3_f64(x, q, s, bias, stride=1, off=-1):
    """The same convolution in float64 with the dequantised weight (the truth)."""
    x = np.asarray(x, np.float64)
    qf = np.asarray(q, np.float64)
    w = (qf.reshape(qf.shape[0], -1, 32) * np.asarray(s, np.float64).reshape(qf.shape[0], -1, 1)).reshape(qf.shape)
    out = []
    for xi in x:
        y = w @ im2col3x3(xi, stride, off)
        if bias is not None:
            y = y + np.asarray(bias, np.float64)[:, None]
        out.append(y)
    H, W = x.shape[2], x.shape[3]
    OH, OW = (H, W) if stride == 1 else (H // 2, W // 2)
    return np.stack(out).reshape(x.shape[0], -1, OH, OW)


# ------------------------------------------------------------------------------ attention
def fused_attention(Q, K, V, Tq, Tk, C, heads, causal=False, force_simple=False):
    Q, K, V = (_c(x, np.float32) for x in (Q, K, V))
    O = np.zeros((Tq, C), np.float32)
    rc = lib().orc_fused_attention(_p(Q), _p(K), _p(V), _p(O), Tq, Tk, C, heads, int(causal), int(force_simple))
    if rc:
        raise ValueError("shape not supported by the reference operator")
    return O


def attn_tiled_shader(Q, K, V, Tq, Tk, C, heads, causal, scale):
    Q, K, V = (_c(x, np.float32) for x in (Q, K, V))
    O = np.zeros((Tq, C), np.float32)
    if lib().orc_attn_tiled_shader(_p(Q), _p(K), _p(V), _p(O), Tq, Tk, C, heads, int(causal), scale):
        raise ValueError("tiled kernel needs hd == 64")
    return O


def attn_simple_shader(Q, K, V, Tq, Tk, C, heads, causal, scale):
    Q, K, V = (_c(x, np.float32) for x in (Q, K, V))
    O = np.zeros((Tq, C), np.float32)
    if lib().orc_attn_simple_shader(_p(Q), _p(K), _p(V), _p(O), Tq, Tk, C, heads, int(causal), scale):
        raise ValueError("simple kernel restated for 32 <= hd <= 64 only")
    return O


def attn_f64(Q, K, V, heads, causal=False, scale=None):
    """fp64 truth on token-major [B, T, C] (or [T, C]) arrays."""
    squeeze = Q.ndim == 2
    Q3, K3, V3 = (x[None] if x.ndim == 2 else x for x in (Q, K, V))
    Q3, K3, V3 = (_c(x, np.float32) for x in (Q3, K3, V3))
    B, Tq, C = Q3.shape
    Tk = K3.shape[1]
    hd = C // heads
    if scale is None:
        scale = float(np.float32(1.0) / np.sqrt(np.float32(hd)))
    O = np.zeros((B, Tq, C), np.float64)
    lib().orc_attn_f64(_p(Q3), _p(K3), _p(V3), _p(O), B, Tq, Tk, heads, hd, C, C, C, C, Tq * C, Tk * C, Tk * C,
                       Tq * C, int(causal), scale)
    return O[0] if squeeze else O


# ------------------------------------------------------------------------------ block glue
def layernorm_shader(x, gamma, beta, eps=1e-5):
    x = _c(x, np.float32)
    rows, d = x.reshape(-1, x.shape[-1]).shape
    y = np.empty_like(x)
    lib().orc_layernorm_shader(_p(x), _p(_c(gamma, np.float32)), _p(_c(beta, np.float32)), _p(y), rows, d, eps, 1)
    return y


def layernorm_f64(x, gamma, beta, eps=1e-5):
    x = _c(x, np.float64)
    rows, d = x.reshape(-1, x.shape[-1]).shape
    y = np.empty_like(x)
    lib().orc_layernorm_f64(_p(x), _p(_c(gamma, np.float32)), _p(_c(beta, np.float32)), _p(y), rows, d, eps)
    return y


def groupnorm_shader(x, gamma, beta, G, eps=1e-5, act=0):
    """groupnorm.comp restated in fp32 (oracle.cpp), per image of x [B, C, P...]."""
    x = _c(x, np.float32)
    B, C = x.shape[0], x.shape[1]
    P = x[0, 0].size
    y = np.empty_like(x)
    g, b = _c(gamma, np.float32), _c(beta, np.float32)
    for i in range(B):
        xi = np.ascontiguousarray(x[i])
        yi = np.empty_like(xi)
        lib().orc_groupnorm_shader(_p(xi), _p(g), _p(b), _p(yi), C, P, G, eps, act)
        y[i] = yi
    return y


def groupnorm_f64(x, gamma, beta, G, eps=1e-5, act=0):
    """GroupNorm (+SiLU) in float64 (the truth the kernels and the restatement are measured against)."""
    x = np.asarray(x, np.float64)
    B, C = x.shape[0], x.shape[1]
    xg = x.reshape(B, G, -1)
    mean = xg.mean(axis=2, keepdims=True)
    var = ((xg - mean) ** 2).mean(axis=2, keepdims=True)
    y = ((xg - mean) / np.sqrt(var + eps)).reshape(x.shape)
    shape = (1, C) + (1,) * (x.ndim - 2)
    y = y * np.asarray(gamma, np.float64).reshape(shape) + np.asarray(beta, np.float64).reshape(shape)
    if act:
        y = y / (1.0 + np.exp(-y))
    return y


def gelu_erf_shader(x):
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().orc_gelu_erf_shader(_p(x), _p(y), x.size)
    return y


def _gelu64(x):
    from scipy.special import erf

    return 0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))


def block_f64(x, ctx, heads, W, rows=None, eps=1e-5):
    """fp64 truth of one BasicTransformerBlock (spatialTransformer's layer body,
    src/Modules/Diffusion/sdvkgen.cpp:1739-1763; geglu :1710-1720; crossAttention :1283-1290) on
    x [B, T, C] and ctx [B, Tctx, Cctx]: LN1 -> to_q/k/v -> attention -> to_out (+bias) -> +res,
    LN2 -> cross-attention against ctx -> +res, LN3 -> GEGLU (gate = second half) -> ff.net.2 -> +res.
    W maps ln{1,2,3}_{w,b} to fp32 arrays and q,k,v,o,q2,k2,v2,o2,ff1,ff2 to (int8, scales, bias|None).
    `rows` (query-token indices) limits the output rows; keys/values still cover every token.
    Values pass between the fp64 stages as fp32 (the f64 kernels take fp32 operands)."""
    B, T, C = x.shape
    rows = np.arange(T) if rows is None else np.asarray(rows)
    f32 = lambda a: np.ascontiguousarray(a, np.float32)
    lin = lambda a, w: gemm_nt_q8_f64(f32(a), w[0], w[1], w[2])
    out = np.empty((B, len(rows), C))
    for b in range(B):
        xb = np.asarray(x[b], np.float64)
        n = layernorm_f64(xb, W["ln1_w"], W["ln1_b"], eps)
        q, k, v = lin(n[rows], W["q"]), lin(n, W["k"]), lin(n, W["v"])
        a = attn_f64(f32(q), f32(k), f32(v), heads)
        x1 = xb[rows] + lin(a, W["o"])
        n = layernorm_f64(x1, W["ln2_w"], W["ln2_b"], eps)
        q, k, v = lin(n, W["q2"]), lin(ctx[b], W["k2"]), lin(ctx[b], W["v2"])
        x2 = x1 + lin(attn_f64(f32(q), f32(k), f32(v), heads), W["o2"])
        n = layernorm_f64(x2, W["ln3_w"], W["ln3_b"], eps)
        g = lin(n, W["ff1"])
        F = g.shape[1] // 2
        out[b] = x2 + lin(g[:, :F] * _gelu64(g[:, F:]), W["ff2"])
    return out


def block_shader(x, ctx, heads, W, rows=None, eps=1e-5):
    """The reference's own fp32 arithmetic for the same block, kernel by kernel as sdvkgen.cpp
    dispatches it: layernorm_fwd, gemm_nt_q8_v(+bias), fusedAttention, unary_fwd erf-GELU, mul2, add2.
    `rows` as in block_f64."""
    B, T, C = x.shape
    rows = np.arange(T) if rows is None else np.asarray(rows)
    lin = lambda a, w: gemm_nt_q8_shader(np.ascontiguousarray(a, np.float32), w[0], w[1], w[2])
    out = np.empty((B, len(rows), C), np.float32)
    for b in range(B):
        xb = np.ascontiguousarray(x[b], np.float32)
        n = layernorm_shader(xb, W["ln1_w"], W["ln1_b"], eps)
        q, k, v = lin(n[rows], W["q"]), lin(n, W["k"]), lin(n, W["v"])
        a = fused_attention(q, k, v, len(rows), T, C, heads)
        x1 = xb[rows] + lin(a, W["o"])
        n = layernorm_shader(x1, W["ln2_w"], W["ln2_b"], eps)
        q, k, v = lin(n, W["q2"]), lin(ctx[b], W["k2"]), lin(ctx[b], W["v2"])
        x2 = x1 + lin(fused_attention(q, k, v, len(rows), k.shape[0], C, heads), W["o2"])
        n = layernorm_shader(x2, W["ln3_w"], W["ln3_b"], eps)
        g = lin(n, W["ff1"])
        F = g.shape[1] // 2
        out[b] = x2 + lin(np.ascontiguousarray(g[:, :F]) * gelu_erf_shader(np.ascontiguousarray(g[:, F:])), W["ff2"])
    return out


def cfg_combine(cond, uncond, cfg, rescale=0.0):
    c, u = _c(cond, np.float32), _c(uncond, np.float32)
    out = np.empty_like(c)
    lib().orc_cfg_combine(_p(c), _p(u), _p(out), c.size, cfg, rescale)
    return out


class SamplerArgs(ctypes.Structure):
    """orc_sampler_args (oracle.h)."""

    _fields_ = [
        ("kind", ctypes.c_int32), ("phase", ctypes.c_int32), ("n", _U64),
        ("eps_c", _P), ("eps_u", _P), ("cfg", _F), ("rescale", _F),
        ("vpred", ctypes.c_int32), ("dynthresh", ctypes.c_int32),
        ("mask", _P), ("mask_cells", _U64), ("init_lat", _P),
        ("lat", _P), ("x_tmp", _P), ("x0", _P), ("x0v", _P), ("x0_prev", _P), ("lms", _P * 4),
        ("lms_count", ctypes.c_int32), ("noise", _P),
        ("sigma", _F), ("sigma_next", _F), ("eta", _F), ("sigma_prev", _F), ("have_prev", ctypes.c_int32),
        ("x_model", _P), ("thr", _P),
    ]


def sampler_eval(**kw) -> int:
    """One evaluation of the generation loop on the CPU (orc_sampler_eval).  Array arguments are
    contiguous float32 numpy arrays (written in place where the step writes them), or None."""
    a = SamplerArgs()
    for name, _ in SamplerArgs._fields_:
        if name not in kw or kw[name] is None:
            continue
        v = kw[name]
        if name == "lms":
            for j, arr in enumerate(v):
                if arr is not None:
                    assert arr.dtype == np.float32 and arr.flags.c_contiguous
                    a.lms[j] = arr.ctypes.data
        elif isinstance(v, np.ndarray):
            assert v.dtype == np.float32 and v.flags.c_contiguous, name
            setattr(a, name, v.ctypes.data)
        else:
            setattr(a, name, v)
    return int(lib().orc_sampler_eval(ctypes.byref(a)))


def sampler_run(kind: int, lat: np.ndarray, sigmas, model, noise=None, cfg=7.5, rescale=0.0, eta=0.0,
                vpred=False, dynthresh=False, mask=None, init_lat=None):
    """The generation loop's sampler on the CPU (sdvkgen.cpp:3796-4026): the same driving order as
    sdvk_b200.sampler.DeviceSampler, each evaluation by orc_sampler_eval.  model(x_model, step,
    phase, sigma) -> (eps_c, eps_u or None) as float32 arrays; noise(step) -> n float32 normals.
    Returns (lat, x0 of the last evaluation)."""
    f32 = np.float32
    lat = np.array(lat, dtype=f32, copy=True)
    n = lat.size
    z = lambda: np.zeros(n, f32)
    x0, x0b, x_tmp = z(), z(), z()
    x0_prev = z()
    lms = [z() for _ in range(4)]
    lms_count, have_prev, sigma_prev = 0, False, 0.0
    inv0 = f32(1.0) / np.sqrt(f32(sigmas[0]) * f32(sigmas[0]) + f32(1.0))
    x_model = (lat * inv0).astype(f32)
    two = kind in (2, 4, 5)
    common = dict(n=n, cfg=cfg, rescale=rescale, vpred=int(vpred), dynthresh=int(dynthresh), mask=mask,
                  mask_cells=0 if mask is None else mask.size, init_lat=init_lat, lat=lat, x_tmp=x_tmp,
                  x0_prev=x0_prev, eta=eta, x_model=x_model)
    last_x0 = x0
    for i in range(len(sigmas) - 1):
        sigma, sn = float(sigmas[i]), float(sigmas[i + 1])
        last = sn <= 0.0
        if kind == 3 and not last:
            lms = [lms[-1]] + lms[:-1]
            lms_count = min(lms_count + 1, 4)
        ec, eu = model(x_model, i, 0, sigma)
        nz = noise(i) if (not last and kind in (1, 7)) else None
        bad = sampler_eval(kind=kind, phase=0, eps_c=ec, eps_u=eu, x0=x0, lms=lms, lms_count=lms_count, noise=nz,
                           sigma=sigma, sigma_next=sn, sigma_prev=sigma_prev, have_prev=int(have_prev), **common)
        if bad:
            raise FloatingPointError(f"non-finite model output at step {i + 1}")
        last_x0 = x0
        if two and not last:
            ec, eu = model(x_model, i, 1, sn)
            nz = noise(i) if kind == 5 else None
            bad = sampler_eval(kind=kind, phase=1, eps_c=ec, eps_u=eu, x0=x0b, x0v=x0, noise=nz, sigma=sigma,
                               sigma_next=sn, **common)
            if bad:
                raise FloatingPointError(f"non-finite model output at step {i + 1}")
            last_x0 = x0b
        if kind in (6, 7) and not last:
            have_prev, sigma_prev = True, sigma
    return lat, last_x0.copy()


# ------------------------------------------------------------------ the rest of the kernel table
# Each takes numpy float32 arrays and the kernel's push constants as a tuple of uint32 (the float
# fields of copy_nd's Pnd -- its last -- packed as their bits), exactly as the walker fills them.
def pack_push(fields, float_last: bool = False) -> bytes:
    import struct as _st

    if float_last:
        return _st.pack(f"<{len(fields) - 1}If", *fields)
    return _st.pack(f"<{len(fields)}I", *[int(v) & 0xFFFFFFFF for v in fields])


def table_kernel(name: str, bufs, push: bytes, gz: int = 1) -> None:
    """Runs the restatement of one kernel-table entry in place on the float32 arrays of `bufs`
    (the binding order of vk_engine.cpp:51-125)."""
    import struct as _st

    L = lib()
    P = [_p(b) for b in bufs]
    u = _st.unpack(f"<{len(push) // 4}I", push)
    pb = ctypes.create_string_buffer(push, len(push))
    pp = ctypes.cast(pb, ctypes.c_void_p)
    if name == "add2":
        L.orc_add2_shader(P[0], P[1], P[2], u[0])
    elif name == "bias_add":
        L.orc_bias_add_shader(P[0], P[1], u[0], u[1])
    elif name == "copy_nd":
        L.orc_copy_nd_shader(P[0], P[1], pp)
    elif name == "ew2":
        L.orc_ew2_shader(P[0], P[1], P[2], pp)
    elif name == "unary_fwd":
        L.orc_unary_shader(P[0], P[1], u[0], u[1])
    elif name == "upsample2x":
        L.orc_upsample2x_shader(P[0], P[1], u[0], u[1], u[2])
    elif name == "im2col":
        L.orc_im2col_shader(P[0], P[1], *u[:5])
    elif name == "im2col_s2":
        L.orc_im2col_s2_shader(P[0], P[1], *u[:5], _st.unpack("<i", push[20:24])[0])
    elif name in ("gemm_nt", "gemm_nn"):
        L.orc_gemm_fp32_shader(int(name == "gemm_nt"), P[0], P[1], P[2], pp, gz)
    elif name == "softmax_fwd":
        L.orc_softmax_shader(P[0], P[1], u[0], u[1])
    elif name == "causal_mask":
        L.orc_causal_mask_shader(P[0], u[0], u[1], u[2])
    else:
        raise KeyError(name)


class GenRng:
    """The generation loop's noise source: std::mt19937(seed) and one std::normal_distribution<float>
    for the whole run (sdvkgen.cpp:3732-3734), so successive calls continue the reference's sequence."""

    def __init__(self, seed: int):
        self.h = lib().orc_gen_rng_new(seed)

    def normal(self, n: int) -> np.ndarray:
        out = np.empty(n, np.float32)
        lib().orc_gen_rng_normal(self.h, _p(out), n)
        return out

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_gen_rng_free(self.h)
            self.h = None


def euler_schedule(steps: int, spacing: str = "leading", zsnr: bool = False, num_train: int = 1000, offset: int = 1):
    """buildEuler (sdvkgen.cpp:2723-2765): (timesteps [steps], sigmas [steps + 1], init noise sigma)."""
    ts = np.empty(steps, np.float32)
    sg = np.empty(steps + 1, np.float32)
    init = lib().orc_euler_schedule(steps, int(spacing == "trailing"), num_train, offset, int(zsnr), _p(ts), _p(sg))
    return ts, sg, float(np.float32(init))


def num_threads() -> int:
    return lib().orc_num_threads()


# ------------------------------------------------------------------------------ metrics
def err_stats(got, ref) -> dict:
    """max-abs and RMS error, relative to max|ref| and RMS(ref)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    d = got - ref
    max_ref = float(np.max(np.abs(ref))) if ref.size else 0.0
    rms_ref = float(np.sqrt(np.mean(ref * ref))) if ref.size else 0.0
    max_abs = float(np.max(np.abs(d))) if d.size else 0.0
    rms = float(np.sqrt(np.mean(d * d))) if d.size else 0.0
    return {
        "max_abs": max_abs,
        "rms": rms,
        "rel_max": max_abs / max(max_ref, 1e-30),
        "rel_max_rms": max_abs / max(rms_ref, 1e-30),
        "rel_rms": rms / max(rms_ref, 1e-30),
        "finite": bool(np.all(np.isfinite(got))),
    }
