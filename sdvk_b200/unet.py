"""The SDXL UNet pass (sdvk_unet_*, unetForward in src/Modules/Diffusion/sdvkgen.cpp:1875-1973) on
torch CUDA tensors.

``Unet`` owns the C-side object: its parameter arena (the reference checkpoint's tensor names) and a
workspace sized for one batch and latent size.  ``forward`` runs one denoiser pass on torch's current
stream through libsdvk_b200.so; there is no other path.
"""
from __future__ import annotations

import ctypes
from typing import Dict, Iterator, Optional, Tuple

import torch

from . import UNET_Q8, UnetDesc, UnetTensorInfo, lib
from .torch_ops import _dt, context

SDXL = dict(model_ch=(320, 640, 1280), depth=(0, 2, 10), ctx_dim=2048, adm_dim=2816, temb_dim=1280, head_dim=64,
            Tctx=77)


def _desc(batch: int, H: int, W: int, arch: dict) -> UnetDesc:
    d = UnetDesc()
    d.model_ch[:] = list(arch["model_ch"])
    d.depth[:] = list(arch["depth"])
    for k in ("ctx_dim", "adm_dim", "temb_dim", "head_dim", "Tctx"):
        setattr(d, k, arch[k])
    d.batch, d.H, d.W = batch, H, W
    return d


def plan(batch: int, H: int, W: int, **arch) -> dict:
    """The UNet's plan without a device (sdvk_unet_plan): {"tensors": {name: (kind, rows, cols)},
    "flops", "launches", "workspace_bytes", "parameter_bytes"}; internal groups (names in
    parentheses) are left out of "tensors"."""
    a = dict(SDXL)
    a.update(arch)
    h = ctypes.c_void_p()
    st = lib().sdvk_unet_plan(ctypes.byref(_desc(batch, H, W, a)), ctypes.byref(h))
    if st != 0:
        from . import SdvkError

        raise SdvkError(st, "sdvk_unet_plan rejected the description")
    try:
        tensors = {}
        for i in range(lib().sdvk_unet_tensor_count(h)):
            info = UnetTensorInfo()
            lib().sdvk_unet_tensor(h, i, ctypes.byref(info))
            name = info.name.decode()
            if not name.startswith("("):
                tensors[name] = (info.kind, info.rows, info.cols)
        return {"tensors": tensors, "flops": int(lib().sdvk_unet_flops(h)), "launches": int(lib().sdvk_unet_launches(h)),
                "workspace_bytes": int(lib().sdvk_unet_workspace_bytes(h)),
                "parameter_bytes": int(lib().sdvk_unet_parameter_bytes(h))}
    finally:
        lib().sdvk_unet_destroy(h)


class Unet:
    def __init__(self, batch: int, H: int, W: int, device: int = 0, **arch):
        a = dict(SDXL)
        a.update(arch)
        self.arch = a
        self.batch, self.H, self.W = batch, H, W
        d = _desc(batch, H, W, a)
        self.desc = d
        with torch.cuda.device(device):
            self.ctx = context(torch.device("cuda", device))
        self.device = device
        self._h = ctypes.c_void_p()
        self.ctx._check(lib().sdvk_unet_create(self.ctx.handle, ctypes.byref(d), ctypes.byref(self._h)),
                        "sdvk_unet_create")

    def close(self) -> None:
        if self._h:
            lib().sdvk_unet_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def flops(self) -> int:
        return int(lib().sdvk_unet_flops(self._h))

    @property
    def launches(self) -> int:
        return int(lib().sdvk_unet_launches(self._h))

    @property
    def workspace_bytes(self) -> int:
        return int(lib().sdvk_unet_workspace_bytes(self._h))

    def init_random(self, seed: int) -> None:
        self.ctx._check(lib().sdvk_unet_init_random(self.ctx.handle, self._h, seed), "sdvk_unet_init_random")

    def prepare(self) -> None:
        self.ctx._check(lib().sdvk_unet_prepare(self.ctx.handle, self._h), "sdvk_unet_prepare")

    def tensors(self) -> Iterator[Tuple[str, UnetTensorInfo]]:
        for i in range(lib().sdvk_unet_tensor_count(self._h)):
            info = UnetTensorInfo()
            self.ctx._check(lib().sdvk_unet_tensor(self._h, i, ctypes.byref(info)), "sdvk_unet_tensor")
            yield info.name.decode(), info

    def read(self, info: UnetTensorInfo) -> Dict[str, torch.Tensor]:
        """Copies of one parameter: {"q": int8 [rows, cols], "s": fp32 [rows, cols/32]} or {"f": fp32 [rows]}."""
        dev = torch.device("cuda", self.device)
        torch.cuda.current_stream(dev).synchronize()
        out = {}
        if info.kind == UNET_Q8:
            q = torch.empty((info.rows, info.cols), dtype=torch.int8, device=dev)
            s = torch.empty((info.rows, info.cols // 32), dtype=torch.float32, device=dev)
            self.ctx.copy(q.data_ptr(), info.q, q.numel())
            self.ctx.copy(s.data_ptr(), info.s, s.numel() * 4)
            out = {"q": q, "s": s}
        else:
            f = torch.empty((info.rows,), dtype=torch.float32, device=dev)
            self.ctx.copy(f.data_ptr(), info.f, f.numel() * 4)
            out = {"f": f}
        self.ctx.synchronize()
        return out

    def forward(self, x: torch.Tensor, timesteps: torch.Tensor, adm: torch.Tensor, context_: torch.Tensor,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """x fp32 [B, 4, H, W], timesteps fp32 [B], adm fp32 [B, adm_dim], context [B, Tctx, ctx_dim]."""
        B, H, W = self.batch, self.H, self.W
        assert x.shape == (B, 4, H, W) and x.dtype == torch.float32 and x.is_contiguous()
        assert timesteps.shape == (B,) and timesteps.dtype == torch.float32
        assert adm.shape == (B, self.arch["adm_dim"]) and adm.dtype == torch.float32 and adm.is_contiguous()
        assert context_.shape == (B, self.arch["Tctx"], self.arch["ctx_dim"]) and context_.is_contiguous()
        if out is None:
            out = torch.empty_like(x)
        ctx = context(x.device)
        ctx._check(lib().sdvk_unet_forward(ctx.handle, self._h, x.data_ptr(), timesteps.data_ptr(), adm.data_ptr(),
                                           context_.data_ptr(), _dt(context_), out.data_ptr()), "sdvk_unet_forward")
        return out
