"""sdvk-b200: B200-native CUDA back end for sdvk's UNet transformer-block hot path.

The product is libsdvk_b200.so (C ABI in include/sdvk_cuda.h).  This package is a thin ctypes
binding over it, used by the tests, bench.py and Python callers:

  * ``Context``      -- one per device: memory, copies, step protocol, and the hot-path calls
                        (``gemm_q8_nt``, ``gemm_q8_nn``, ``attention``, ``dispatch``,
                        ``fused_attention``) on raw device pointers.
  * ``sdvk_b200.torch_ops`` -- the same calls on torch CUDA tensors (torch's stream).

There is no CPU fallback: if the library is missing or fails to load, importing the binding
raises.  Build it with ``python -m sdvk_b200.build``.
"""
from __future__ import annotations

import ctypes
import os
import struct
from typing import Optional, Sequence

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsdvk_b200.so")

OK, E_OOM, E_SHAPE, E_CUDA, E_TIMEOUT, E_ARG, E_KERNEL, E_STATE, E_NOT_FINITE = range(9)
F32, F16, BF16 = 0, 1, 2
PRECISION_REFERENCE, PRECISION_FAST = 0, 1

_lib: Optional[ctypes.CDLL] = None


class SdvkError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"sdvk status {status}: {message}")
        self.status = status


class Buf(ctypes.Structure):
    """sdvk_buf: non-owning device view (the reference's BufRef{buffer, offset, size})."""

    _fields_ = [("ptr", ctypes.c_void_p), ("offset", ctypes.c_uint64), ("size", ctypes.c_uint64)]


class AttnDesc(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("o", ctypes.c_void_p),
        ("dtype", ctypes.c_int), ("o_dtype", ctypes.c_int),
        ("batch", ctypes.c_uint32), ("heads", ctypes.c_uint32), ("Tq", ctypes.c_uint32),
        ("Tk", ctypes.c_uint32), ("hd", ctypes.c_uint32),
        ("ldq", ctypes.c_uint64), ("ldk", ctypes.c_uint64), ("ldv", ctypes.c_uint64), ("ldo", ctypes.c_uint64),
        ("sq", ctypes.c_uint64), ("sk", ctypes.c_uint64), ("sv", ctypes.c_uint64), ("so", ctypes.c_uint64),
        ("hq", ctypes.c_uint64), ("hk", ctypes.c_uint64), ("hv", ctypes.c_uint64), ("ho", ctypes.c_uint64),
        ("scale", ctypes.c_float), ("causal", ctypes.c_int),
    ]


class SamplerStepDesc(ctypes.Structure):
    """sdvk_sampler_step_desc: one model evaluation's share of the generation loop."""

    _fields_ = [
        ("kind", ctypes.c_int32), ("phase", ctypes.c_int32), ("n", ctypes.c_uint64),
        ("eps_c", ctypes.c_void_p), ("eps_u", ctypes.c_void_p), ("cfg", ctypes.c_float), ("rescale", ctypes.c_float),
        ("vpred", ctypes.c_int32), ("dynthresh", ctypes.c_int32),
        ("mask", ctypes.c_void_p), ("mask_cells", ctypes.c_uint64), ("init_lat", ctypes.c_void_p),
        ("lat", ctypes.c_void_p), ("x_tmp", ctypes.c_void_p), ("x0", ctypes.c_void_p), ("x0v", ctypes.c_void_p),
        ("x0_prev", ctypes.c_void_p), ("lms", ctypes.c_void_p * 4), ("lms_count", ctypes.c_int32),
        ("noise", ctypes.c_void_p), ("sigma", ctypes.c_float), ("sigma_next", ctypes.c_float),
        ("eta", ctypes.c_float), ("sigma_prev", ctypes.c_float), ("have_prev", ctypes.c_int32),
        ("x_model", ctypes.c_void_p), ("thr", ctypes.c_void_p),
    ]


# Sampler kinds (SamplerKind, src/Modules/Diffusion/GenParams.hpp:16-26)
SAMPLER_EULER, SAMPLER_EULER_A, SAMPLER_HEUN, SAMPLER_LMS, SAMPLER_DPM2, SAMPLER_DPM2_A = range(6)
SAMPLER_DPMPP_2M, SAMPLER_DPMPP_2S_A, SAMPLER_DDIM = 6, 7, 8


class Q8Linear(ctypes.Structure):
    """sdvk_q8_linear: int8 weight [N][K], fp32 scale per 32 weights, optional fp32 bias [N]."""

    _fields_ = [("q", ctypes.c_void_p), ("s", ctypes.c_void_p), ("bias", ctypes.c_void_p)]


class BlockDesc(ctypes.Structure):
    """sdvk_block_desc: one SDXL BasicTransformerBlock (spatialTransformer's layer body)."""

    _fields_ = [
        ("x", ctypes.c_void_p), ("ctx", ctypes.c_void_p), ("ctx_dtype", ctypes.c_int),
        ("batch", ctypes.c_uint32), ("T", ctypes.c_uint32), ("C", ctypes.c_uint32), ("heads", ctypes.c_uint32),
        ("Tctx", ctypes.c_uint32), ("Cctx", ctypes.c_uint32), ("ff_inner", ctypes.c_uint32),
        ("ln1_w", ctypes.c_void_p), ("ln1_b", ctypes.c_void_p), ("ln2_w", ctypes.c_void_p),
        ("ln2_b", ctypes.c_void_p), ("ln3_w", ctypes.c_void_p), ("ln3_b", ctypes.c_void_p),
        ("q", Q8Linear), ("k", Q8Linear), ("v", Q8Linear), ("o", Q8Linear),
        ("q2", Q8Linear), ("k2", Q8Linear), ("v2", Q8Linear), ("o2", Q8Linear),
        ("ff1", Q8Linear), ("ff2", Q8Linear),
        ("eps", ctypes.c_float),
        ("ff1_geglu_interleaved", ctypes.c_uint32),
    ]


class UnetDesc(ctypes.Structure):
    """sdvk_unet_desc: the SDXL UNet's architecture and the pass's batch and latent size."""

    _fields_ = [
        ("model_ch", ctypes.c_uint32 * 3), ("depth", ctypes.c_uint32 * 3),
        ("ctx_dim", ctypes.c_uint32), ("adm_dim", ctypes.c_uint32), ("temb_dim", ctypes.c_uint32),
        ("head_dim", ctypes.c_uint32), ("Tctx", ctypes.c_uint32),
        ("batch", ctypes.c_uint32), ("H", ctypes.c_uint32), ("W", ctypes.c_uint32),
    ]


class UnetTensorInfo(ctypes.Structure):
    """sdvk_unet_tensor_info: one named parameter of the UNet's arena."""

    _fields_ = [
        ("name", ctypes.c_char_p), ("kind", ctypes.c_int), ("rows", ctypes.c_uint32), ("cols", ctypes.c_uint32),
        ("q", ctypes.c_void_p), ("s", ctypes.c_void_p), ("f", ctypes.c_void_p),
    ]


UNET_Q8, UNET_F32 = 0, 1


class UnetTensorLayout(ctypes.Structure):
    """sdvk_unet_param_layout: where a parameter lives in the arena and how the seeded init fills it."""

    _fields_ = [("q_off", ctypes.c_uint64), ("s_off", ctypes.c_uint64), ("f_off", ctypes.c_uint64),
                ("init", ctypes.c_int)]


# name -> (restype, argtypes) for every symbol include/sdvk_cuda.h declares
_P, _U32, _U64, _I = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int
SIGNATURES = {
    "sdvk_ctx_create": (_I, [_I, ctypes.POINTER(_P)]),
    "sdvk_ctx_destroy": (_I, [_P]),
    "sdvk_ctx_set_stream": (_I, [_P, _P]),
    "sdvk_ctx_reset_stream": (_I, [_P]),
    "sdvk_ctx_stream": (_P, [_P]),
    "sdvk_ctx_set_timeout_ms": (_I, [_P, _U32]),
    "sdvk_ctx_set_precision": (_I, [_P, _I]),
    "sdvk_device_report": (_I, [_P, ctypes.c_char_p, ctypes.c_size_t]),
    "sdvk_last_error": (ctypes.c_char_p, [_P]),
    "sdvk_status_string": (ctypes.c_char_p, [_I]),
    "sdvk_alloc": (_I, [_P, _U64, ctypes.POINTER(_P)]),
    "sdvk_free": (_I, [_P, _P]),
    "sdvk_host_alloc": (_I, [_P, _U64, ctypes.POINTER(_P)]),
    "sdvk_host_free": (_I, [_P, _P]),
    "sdvk_upload": (_I, [_P, _P, _P, _U64]),
    "sdvk_download": (_I, [_P, _P, _P, _U64]),
    "sdvk_upload_async": (_I, [_P, _P, _P, _U64]),
    "sdvk_download_async": (_I, [_P, _P, _P, _U64]),
    "sdvk_copy": (_I, [_P, _P, _P, _U64]),
    "sdvk_fill_u32": (_I, [_P, _P, _U32, _U64]),
    "sdvk_step_begin": (_I, [_P]),
    "sdvk_step_end": (_I, [_P]),
    "sdvk_step_wait": (_I, [_P, _U32]),
    "sdvk_synchronize": (_I, [_P]),
    "sdvk_dispatch": (_I, [_P, ctypes.c_char_p, ctypes.POINTER(Buf), _U32, _P, _U32, _U32, _U32, _U32]),
    "sdvk_fused_attention": (_I, [_P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _I]),
    "sdvk_fused_attn_supported": (_I, [_U32, _U32]),
    "sdvk_gemm_q8_nt": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _U32, _U32, _U32, _U32, _U32, _U32, _U64, _U64, _I]),
    "sdvk_gemm_q8_nn": (_I, [_P, _P, _P, _P, _I, _P, _P, _I, _U32, _U32, _U32, _U32, _U32, _U32, _U32,
                             _U64, _U64, _U64, _I]),
    "sdvk_attention": (_I, [_P, ctypes.POINTER(AttnDesc)]),
    "sdvk_check_finite": (_I, [_P, _P, _I, _U64]),
    "sdvk_cfg_combine": (_I, [_P, _P, _P, _P, _U64, ctypes.c_float, ctypes.c_float]),
    "sdvk_sampler_step": (_I, [_P, ctypes.POINTER(SamplerStepDesc)]),
    "sdvk_sampler_scale": (_I, [_P, _P, _P, _U64, ctypes.c_float]),
    "sdvk_q8_0_ingest": (_I, [_P, _P, _U64, _U64, _P, _U64, _P]),
    "sdvk_conv3x3_workspace": (_U64, [_U32, _U32, _U32, _I, _I]),
    "sdvk_conv3x3_q8": (_I, [_P, _P, _I, _P, _P, _P, _P, _I, _U32, _U32, _U32, _U32, _U32, _I, _I, _P, _U64]),
    "sdvk_groupnorm_workspace": (_U64, [_U32, _U32, _U32, _U32]),
    "sdvk_conv3x3_implicit_ok": (_I, [_U32, _U32, _U32, _U32, _I]),
    "sdvk_conv3x3_weights_f16": (_I, [_P, _P, _P, _U32, _U32, _P]),
    "sdvk_conv3x3_nhwc": (_I, [_P, _P, _P, _P, _U64, _I, _P, _I, _U32, _U32, _U32, _U32, _U32, _I, _I]),
    "sdvk_groupnorm": (_I, [_P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, ctypes.c_float, _I, _P, _U64]),
    "sdvk_groupnorm_cl": (_I, [_P, _P, _P, _P, _P, _U32, _U32, _U32, _U32, ctypes.c_float, _I, _P, _U64]),
    "sdvk_comm_unique_id": (_I, [_P]),
    "sdvk_comm_create": (_I, [_P, _I, _I, _P, _U32, ctypes.POINTER(_P)]),
    "sdvk_comm_destroy": (_I, [_P]),
    "sdvk_comm_abort": (_I, [_P]),
    "sdvk_allgather": (_I, [_P, _P, _P, _P, _U64, _I]),
    "sdvk_comm_wait": (_I, [_P, _P, _U32]),
    "sdvk_geglu_interleave": (_I, [_P, _P, _P, _P, _U32, _U32, _P, _P, _P]),
    "sdvk_gemm_q8_nt_geglu": (_I, [_P, _P, _I, _P, _P, _P, _P, _U32, _U32, _U32, _U32, _U32]),
    "sdvk_layernorm": (_I, [_P, _P, _P, _P, _P, _I, _U32, _U32, _U64, _U64, ctypes.c_float]),
    "sdvk_geglu": (_I, [_P, _P, _P, _U32, _U32, _U64, _U64]),
    "sdvk_transformer_block_workspace": (_U64, [ctypes.POINTER(BlockDesc)]),
    "sdvk_transformer_block": (_I, [_P, ctypes.POINTER(BlockDesc), _P, _U64]),
    "sdvk_transformer_block_static": (_I, [_P, ctypes.POINTER(BlockDesc)]),
    "sdvk_device_memory": (_I, [_P, ctypes.POINTER(_U64), ctypes.POINTER(_U64)]),
    "sdvk_selftest_wait": (_I, [_P]),
    "sdvk_unet_create": (_I, [_P, ctypes.POINTER(UnetDesc), ctypes.POINTER(_P)]),
    "sdvk_unet_plan": (_I, [ctypes.POINTER(UnetDesc), ctypes.POINTER(_P)]),
    "sdvk_unet_destroy": (_I, [_P]),
    "sdvk_unet_init_random": (_I, [_P, _P, _U64]),
    "sdvk_unet_prepare": (_I, [_P, _P]),
    "sdvk_unet_tensor_count": (_U32, [_P]),
    "sdvk_unet_tensor": (_I, [_P, _U32, ctypes.POINTER(UnetTensorInfo)]),
    "sdvk_unet_tensor_layout": (_I, [_P, _U32, ctypes.POINTER(UnetTensorLayout)]),
    "sdvk_unet_flops": (_U64, [_P]),
    "sdvk_unet_workspace_bytes": (_U64, [_P]),
    "sdvk_unet_launches": (_U64, [_P]),
    "sdvk_unet_parameter_bytes": (_U64, [_P]),
    "sdvk_unet_forward": (_I, [_P, _P, _P, _P, _P, _P, _I, _P]),
}


def lib() -> ctypes.CDLL:
    """Load libsdvk_b200.so (raises if it is missing: there is no fallback path)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing; build it with `python -m sdvk_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def fused_attn_supported(C: int, heads: int) -> bool:
    """fusedAttnSupported (src/Modules/GPU/fused_attn.cpp:34-38)."""
    return bool(lib().sdvk_fused_attn_supported(C, heads))


class Context:
    """One sdvk context on one CUDA device (the reference's ``Engine``)."""

    def __init__(self, device: int = 0):
        self._h = ctypes.c_void_p()
        st = lib().sdvk_ctx_create(device, ctypes.byref(self._h))
        if st != OK:
            raise SdvkError(st, f"sdvk_ctx_create(device={device}) failed: {lib().sdvk_status_string(st).decode()}")
        self.device = device

    # -- plumbing --------------------------------------------------------------------------
    @property
    def handle(self):
        return self._h

    def _check(self, st: int, what: str) -> None:
        if st != OK:
            msg = lib().sdvk_last_error(self._h)
            raise SdvkError(st, f"{what}: {(msg or b'').decode()} ({lib().sdvk_status_string(st).decode()})")

    def close(self) -> None:
        if self._h:
            lib().sdvk_ctx_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream_ptr: Optional[int]) -> None:
        """Queue work on a cudaStream_t (0/None = CUDA's legacy default stream)."""
        self._check(lib().sdvk_ctx_set_stream(self._h, stream_ptr or None), "set_stream")

    def reset_stream(self) -> None:
        """Return to the context's private non-blocking stream."""
        self._check(lib().sdvk_ctx_reset_stream(self._h), "reset_stream")

    def set_precision(self, precision: int) -> None:
        """PRECISION_REFERENCE (default): fp32 attention inputs computed in fp32; PRECISION_FAST: f16."""
        self._check(lib().sdvk_ctx_set_precision(self._h, precision), "set_precision")

    def set_timeout_ms(self, ms: int) -> None:
        self._check(lib().sdvk_ctx_set_timeout_ms(self._h, ms), "set_timeout_ms")

    def device_report(self) -> str:
        buf = ctypes.create_string_buffer(1024)
        self._check(lib().sdvk_device_report(self._h, buf, len(buf)), "device_report")
        return buf.value.decode()

    # -- memory ----------------------------------------------------------------------------
    def alloc(self, nbytes: int) -> int:
        p = ctypes.c_void_p()
        self._check(lib().sdvk_alloc(self._h, nbytes, ctypes.byref(p)), "alloc")
        return p.value

    def free(self, ptr: int) -> None:
        self._check(lib().sdvk_free(self._h, ptr), "free")

    def host_alloc(self, nbytes: int) -> int:
        p = ctypes.c_void_p()
        self._check(lib().sdvk_host_alloc(self._h, nbytes, ctypes.byref(p)), "host_alloc")
        return p.value

    def host_free(self, ptr: int) -> None:
        self._check(lib().sdvk_host_free(self._h, ptr), "host_free")

    def upload(self, dst: int, src_host: int, nbytes: int) -> None:
        self._check(lib().sdvk_upload(self._h, dst, src_host, nbytes), "upload")

    def download(self, dst_host: int, src: int, nbytes: int) -> None:
        self._check(lib().sdvk_download(self._h, dst_host, src, nbytes), "download")

    def upload_async(self, dst: int, src_host: int, nbytes: int) -> None:
        self._check(lib().sdvk_upload_async(self._h, dst, src_host, nbytes), "upload_async")

    def download_async(self, dst_host: int, src: int, nbytes: int) -> None:
        self._check(lib().sdvk_download_async(self._h, dst_host, src, nbytes), "download_async")

    def copy(self, dst: int, src: int, nbytes: int) -> None:
        self._check(lib().sdvk_copy(self._h, dst, src, nbytes), "copy")

    def synchronize(self) -> None:
        self._check(lib().sdvk_synchronize(self._h), "synchronize")

    def selftest_wait(self) -> None:
        """Queue the failure-path self-test: a bounded wait that runs out (sdvk_selftest_wait)."""
        self._check(lib().sdvk_selftest_wait(self._h), "selftest_wait")

    # -- step protocol (beginStep / endStep / waitStep) --------------------------------------
    def step_begin(self) -> None:
        self._check(lib().sdvk_step_begin(self._h), "step_begin")

    def step_end(self) -> None:
        self._check(lib().sdvk_step_end(self._h), "step_end")

    def step_wait(self, timeout_ms: int = 0) -> None:
        self._check(lib().sdvk_step_wait(self._h, timeout_ms), "step_wait")

    # -- hot path ----------------------------------------------------------------------------
    def gemm_q8_nt(self, A: int, a_dtype: int, q: int, s: int, bias: Optional[int], C: int, c_dtype: int,
                   M: int, N: int, K: int, lda: int = 0, ldc: int = 0, batch: int = 1, sA: int = 0, sC: int = 0,
                   accumulate: bool = False) -> None:
        self._check(lib().sdvk_gemm_q8_nt(self._h, A, a_dtype, q, s, bias or None, C, c_dtype, M, N, K, lda, ldc,
                                          batch, sA, sC, int(accumulate)), "gemm_q8_nt")

    def gemm_q8_nn(self, q: int, s: int, B: int, b_dtype: int, bias: Optional[int], C: int, c_dtype: int,
                   M: int, N: int, K: int, lda: int = 0, ldb: int = 0, ldc: int = 0, batch: int = 1, sA: int = 0,
                   sB: int = 0, sC: int = 0, accumulate: bool = False) -> None:
        self._check(lib().sdvk_gemm_q8_nn(self._h, q, s, B, b_dtype, bias or None, C, c_dtype, M, N, K, lda, ldb,
                                          ldc, batch, sA, sB, sC, int(accumulate)), "gemm_q8_nn")

    def attention(self, desc: AttnDesc) -> None:
        self._check(lib().sdvk_attention(self._h, ctypes.byref(desc)), "attention")

    def fused_attention(self, q: int, k: int, v: int, out: int, Tq: int, Tk: int, C: int, heads: int,
                        causal: bool = False) -> None:
        """fusedAttention(Engine&, FusedAttnArgs) (src/Modules/GPU/fused_attn.cpp:40-61), fp32 buffers."""
        self._check(lib().sdvk_fused_attention(self._h, q, k, v, out, Tq, Tk, C, heads, int(causal)),
                    "fused_attention")

    def dispatch(self, kernel: str, bufs: Sequence[Buf], push: bytes, gx: int, gy: int = 1, gz: int = 1) -> None:
        """Engine::dispatch (src/Modules/GPU/vk_engine.hpp:111-112) for the hot-path kernel names."""
        arr = (Buf * len(bufs))(*bufs)
        pbuf = ctypes.create_string_buffer(push, len(push))
        self._check(lib().sdvk_dispatch(self._h, kernel.encode(), arr, len(bufs), pbuf, len(push), gx, gy, gz),
                    f"dispatch({kernel})")

    def layernorm(self, x: int, gamma: Optional[int], beta: Optional[int], y: int, y_dtype: int, rows: int, d: int,
                  ldx: int = 0, ldy: int = 0, eps: float = 1e-5) -> None:
        self._check(lib().sdvk_layernorm(self._h, x, gamma or None, beta or None, y, y_dtype, rows, d, ldx or d,
                                         ldy or d, eps), "layernorm")

    def geglu_interleave(self, q: int, s: int, bias: Optional[int], F: int, K: int, q_out: int, s_out: int,
                         bias_out: Optional[int]) -> None:
        self._check(lib().sdvk_geglu_interleave(self._h, q, s, bias or None, F, K, q_out, s_out, bias_out or None),
                    "geglu_interleave")

    def gemm_q8_nt_geglu(self, A: int, a_dtype: int, q: int, s: int, bias: Optional[int], C: int, M: int, F: int,
                         K: int, lda: int = 0, ldc: int = 0) -> None:
        self._check(lib().sdvk_gemm_q8_nt_geglu(self._h, A, a_dtype, q, s, bias or None, C, M, F, K, lda, ldc),
                    "gemm_q8_nt_geglu")

    def geglu(self, h: int, y: int, rows: int, F: int, ldh: int = 0, ldy: int = 0) -> None:
        self._check(lib().sdvk_geglu(self._h, h, y, rows, F, ldh or 2 * F, ldy or F), "geglu")

    @staticmethod
    def block_workspace(desc: "BlockDesc") -> int:
        return int(lib().sdvk_transformer_block_workspace(ctypes.byref(desc)))

    def transformer_block(self, desc: "BlockDesc", workspace: int, nbytes: int) -> None:
        self._check(lib().sdvk_transformer_block(self._h, ctypes.byref(desc), workspace, nbytes), "transformer_block")

    def transformer_block_static(self, desc: "BlockDesc") -> None:
        """The block on the library's fixed device scratch array (no workspace, no allocation)."""
        self._check(lib().sdvk_transformer_block_static(self._h, ctypes.byref(desc)), "transformer_block_static")

    def cfg_combine(self, cond: int, uncond: int, out: int, n: int, cfg: float, rescale: float = 0.0) -> None:
        self._check(lib().sdvk_cfg_combine(self._h, cond, uncond, out, n, cfg, rescale), "cfg_combine")

    def q8_0_ingest(self, blocks: int, rows: int, cols: int, q: int, ldq: int, scales: int) -> None:
        self._check(lib().sdvk_q8_0_ingest(self._h, blocks, rows, cols, q, ldq, scales), "q8_0_ingest")

    @staticmethod
    def conv3x3_workspace(cin: int, H: int, W: int, stride: int, x_dtype: int) -> int:
        return lib().sdvk_conv3x3_workspace(cin, H, W, stride, x_dtype)

    def conv3x3_q8(self, x: int, x_dtype: int, q: int, s: int, bias: Optional[int], y: int, y_dtype: int, batch: int,
                   cin: int, cout: int, H: int, W: int, stride: int, pad_off: int, workspace: int,
                   workspace_bytes: int) -> None:
        self._check(lib().sdvk_conv3x3_q8(self._h, x, x_dtype, q, s, bias or None, y, y_dtype, batch, cin, cout, H, W,
                                          stride, pad_off, workspace or None, workspace_bytes), "conv3x3_q8")

    @staticmethod
    def conv3x3_implicit_ok(batch: int, cin: int, H: int, W: int, stride: int) -> bool:
        return bool(lib().sdvk_conv3x3_implicit_ok(batch, cin, H, W, stride))

    def conv3x3_weights_f16(self, q: int, s: int, cout: int, cin: int, w16: int) -> None:
        self._check(lib().sdvk_conv3x3_weights_f16(self._h, q, s, cout, cin, w16), "conv3x3_weights_f16")

    def conv3x3_nhwc(self, x: int, w16: int, bias: Optional[int], bias_stride: int, accumulate: bool, y: int,
                     y_dtype: int, batch: int, cin: int, cout: int, H: int, W: int, stride: int, pad_off: int) -> None:
        self._check(lib().sdvk_conv3x3_nhwc(self._h, x, w16, bias or None, bias_stride, int(accumulate), y, y_dtype,
                                            batch, cin, cout, H, W, stride, pad_off), "conv3x3_nhwc")

    @staticmethod
    def groupnorm_workspace(batch: int, C: int, P: int, G: int) -> int:
        return lib().sdvk_groupnorm_workspace(batch, C, P, G)

    def groupnorm(self, x: int, gamma: int, beta: int, y: int, batch: int, C: int, P: int, G: int, eps: float,
                  silu: bool, workspace: int, workspace_bytes: int) -> None:
        self._check(lib().sdvk_groupnorm(self._h, x, gamma, beta, y, batch, C, P, G, eps, int(silu), workspace or None,
                                         workspace_bytes), "groupnorm")

    def groupnorm_cl(self, x: int, gamma: int, beta: int, y: int, batch: int, C: int, P: int, G: int, eps: float,
                     silu: bool, workspace: int, workspace_bytes: int) -> None:
        self._check(lib().sdvk_groupnorm_cl(self._h, x, gamma, beta, y, batch, C, P, G, eps, int(silu),
                                            workspace or None, workspace_bytes), "groupnorm_cl")

    def sampler_step(self, desc: SamplerStepDesc) -> None:
        """sdvk_sampler_step: guidance, x0 and the sampler update of one model evaluation."""
        self._check(lib().sdvk_sampler_step(self._h, ctypes.byref(desc)), "sampler_step")

    def sampler_scale(self, x: int, out: int, n: int, sigma: float) -> None:
        """out = x / sqrt(sigma^2 + 1), the first evaluation's model input."""
        self._check(lib().sdvk_sampler_scale(self._h, x, out, n, sigma), "sampler_scale")

    def check_finite(self, ptr: int, dtype: int, n: int) -> bool:
        st = lib().sdvk_check_finite(self._h, ptr, dtype, n)
        if st == E_NOT_FINITE:
            return False
        self._check(st, "check_finite")
        return True


def pack_pg(M, N, K, mode=0, sA=0, sB=0, sC=0, batch=1, lda=0, ldb=0, ldc=0) -> bytes:
    """Pg push constants of the Q8 GEMM kernels (sdvkgen.cpp:901-903)."""
    return struct.pack("<12I", M, N, K, mode, sA, sB, sC, batch, lda, ldb, ldc, 0)


def pack_gn(C, P, G, eps=1e-5, act=0) -> bytes:
    """groupnorm.comp push constants {C, P, G, eps, act} (sdvkgen.cpp:1107-1111)."""
    return struct.pack("<IIIfI", C, P, G, eps, act)


def pack_ln(rows, d, eps=1e-5, affine=1) -> bytes:
    """layernorm_fwd push constants {rows, d, eps, affine} (sdvkgen.cpp:1096-1100)."""
    return struct.pack("<IIfI", rows, d, eps, affine)


def pack_fa(Tq, Tk, C, heads, hd, causal, scale) -> bytes:
    """FaPush of the fused attention kernels (fused_attn.cpp:15-26)."""
    return struct.pack("<8If", Tq, Tk, C, heads, hd, int(causal), 0, 0, scale)


COMM_ID_BYTES = 128
STATIC_SCRATCH_BYTES = 64 << 20


def comm_unique_id() -> bytes:
    """A fresh NCCL unique id (made on one rank, passed to the others out of band)."""
    buf = ctypes.create_string_buffer(COMM_ID_BYTES)
    st = lib().sdvk_comm_unique_id(buf)
    if st != OK:
        raise SdvkError(st, "sdvk_comm_unique_id failed (is libnccl.so.2 available?)")
    return buf.raw


class Comm:
    """An NCCL communicator over a context's device (sdvk_comm)."""

    def __init__(self, ctx: Context, nranks: int, rank: int, uid: bytes, timeout_ms: int = 30000):
        self._ctx = ctx
        self._h = ctypes.c_void_p()
        idb = ctypes.create_string_buffer(uid, COMM_ID_BYTES)
        ctx._check(lib().sdvk_comm_create(ctx.handle, nranks, rank, idb, timeout_ms, ctypes.byref(self._h)),
                   "comm_create")

    def allgather(self, send: int, recv: int, count: int, dtype: int) -> None:
        self._ctx._check(lib().sdvk_allgather(self._ctx.handle, self._h, send, recv, count, dtype), "allgather")

    def wait(self, timeout_ms: int = 30000) -> None:
        self._ctx._check(lib().sdvk_comm_wait(self._ctx.handle, self._h, timeout_ms), "comm_wait")

    def abort(self) -> None:
        if self._h:
            lib().sdvk_comm_abort(self._h)

    def close(self) -> None:
        if self._h:
            lib().sdvk_comm_destroy(self._h)
            self._h = ctypes.c_void_p()
