"""The generation loop's sampler on the device: the reference's per-step host work
(src/Modules/Diffusion/sdvkgen.cpp:3759-4021) driven through sdvk_sampler_step, so the latent, the
x0 estimates and the sampler history stay in device memory between model evaluations.

The reference downloads each model output, combines and updates on the host, and uploads the next
scaled input (runPass / evalGuided, :3749-3758 and :3806-3846).  Here the model callback receives
the device tensor of the scaled input and returns device tensors, and one kernel per evaluation
does the rest.  Ancestral noise keeps the reference's draw order: ``noise(i)`` is called once per
step that consumes noise and must return the n normals the reference's nd(rng) would produce there.
"""
from __future__ import annotations

from typing import Callable, Optional, Sequence, Tuple

import torch

from . import SAMPLER_DPM2, SAMPLER_DPM2_A, SAMPLER_DPMPP_2M, SAMPLER_DPMPP_2S_A, SAMPLER_EULER_A, SAMPLER_HEUN
from . import SAMPLER_LMS, SamplerStepDesc
from .torch_ops import context

NAMES = {"euler": 0, "euler_a": 1, "heun": 2, "lms": 3, "dpm2": 4, "dpm2_a": 5, "dpmpp_2m": 6, "dpmpp_2s_a": 7,
         "ddim": 8}
TWO_EVALS = (SAMPLER_HEUN, SAMPLER_DPM2, SAMPLER_DPM2_A)  # samplerModelEvals (GenParams.hpp:92-101)
ANCESTRAL = (SAMPLER_EULER_A, SAMPLER_DPM2_A, SAMPLER_DPMPP_2S_A)

# model(x_model, step, phase, sigma) -> (eps_c, eps_u or None), fp32 device tensors of n values
Model = Callable[[torch.Tensor, int, int, float], Tuple[torch.Tensor, Optional[torch.Tensor]]]


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


class DeviceSampler:
    """Runs a sampler over a sigma schedule with every per-element step on the device.

    kind: SDVK_SAMPLER_* or a name of NAMES.  The options are the reference's GenParams fields
    (cfg, rescale, eta, vpred, dynthresh) and the inpaint blend (mask of mask_cells values indexed
    by k % mask_cells, init_lat)."""

    def __init__(self, kind, n: int, device="cuda", cfg: float = 7.5, rescale: float = 0.0, eta: float = 0.0,
                 vpred: bool = False, dynthresh: bool = False, mask: Optional[torch.Tensor] = None,
                 init_lat: Optional[torch.Tensor] = None):
        self.kind = NAMES[kind] if isinstance(kind, str) else int(kind)
        self.n = int(n)
        self.cfg, self.rescale, self.eta = float(cfg), float(rescale), float(eta)
        self.vpred, self.dynthresh = bool(vpred), bool(dynthresh)
        self.mask, self.init_lat = mask, init_lat
        self.ctx = context(torch.device(device))
        f = lambda: torch.zeros(self.n, dtype=torch.float32, device=device)
        self.x0, self.x0b, self.x_tmp, self.x_model = f(), f(), f(), f()
        self.x0_prev = f() if self.kind in (SAMPLER_DPMPP_2M, SAMPLER_DPMPP_2S_A) else None
        self.lms = [f() for _ in range(4)] if self.kind == SAMPLER_LMS else None
        self.thr = torch.zeros(1, dtype=torch.float32, device=device)
        self.lms_count = 0
        self.have_prev = False
        self.sigma_prev = 0.0

    def _desc(self, phase: int, eps_c, eps_u, lat, sigma: float, sigma_next: float, noise) -> SamplerStepDesc:
        d = SamplerStepDesc()
        d.kind, d.phase, d.n = self.kind, phase, self.n
        d.eps_c, d.eps_u = _ptr(eps_c), _ptr(eps_u)
        d.cfg, d.rescale = self.cfg, self.rescale
        d.vpred, d.dynthresh = int(self.vpred), int(self.dynthresh)
        if self.mask is not None:
            d.mask, d.mask_cells, d.init_lat = _ptr(self.mask), self.mask.numel(), _ptr(self.init_lat)
        d.lat, d.x_tmp = _ptr(lat), _ptr(self.x_tmp)
        d.x0 = _ptr(self.x0 if phase == 0 else self.x0b)
        d.x0v = _ptr(self.x0) if phase == 1 else None
        d.x0_prev = _ptr(self.x0_prev)
        if self.lms is not None:
            for j in range(4):
                d.lms[j] = self.lms[j].data_ptr()
            d.lms_count = self.lms_count
        d.noise = _ptr(noise)
        d.sigma, d.sigma_next, d.eta = sigma, sigma_next, self.eta
        d.sigma_prev, d.have_prev = self.sigma_prev, int(self.have_prev)
        d.x_model, d.thr = _ptr(self.x_model), _ptr(self.thr)
        return d

    def step(self, i: int, lat: torch.Tensor, sigmas: Sequence[float], model: Model,
             noise: Optional[Callable[[int], torch.Tensor]] = None) -> None:
        """Step i of the loop (sdvkgen.cpp:3796-4026), updating lat in place.  self.x_model must hold
        the step's scaled model input (begin() or the previous step leaves it there)."""
        sigma, sn = float(sigmas[i]), float(sigmas[i + 1])
        last = sn <= 0.0
        if self.lms is not None and not last:  # newest first; the oldest buffer is reused
            self.lms = [self.lms[-1]] + self.lms[:-1]
            self.lms_count = min(self.lms_count + 1, 4)
        eps_c, eps_u = model(self.x_model, i, 0, sigma)
        nz = None
        if not last and self.kind in (SAMPLER_EULER_A, SAMPLER_DPMPP_2S_A):
            nz = noise(i)
        self.ctx.sampler_step(self._desc(0, eps_c, eps_u, lat, sigma, sn, nz))
        if self.kind in TWO_EVALS and not last:
            eps_c2, eps_u2 = model(self.x_model, i, 1, sn)
            nz = noise(i) if self.kind == SAMPLER_DPM2_A else None
            self.ctx.sampler_step(self._desc(1, eps_c2, eps_u2, lat, sigma, sn, nz))
        if self.kind in (SAMPLER_DPMPP_2M, SAMPLER_DPMPP_2S_A) and not last:
            self.have_prev, self.sigma_prev = True, sigma

    def begin(self, lat: torch.Tensor, sigma0: float) -> None:
        """The first evaluation's model input, lat / sqrt(sigma0^2 + 1)."""
        self.ctx.sampler_scale(lat.data_ptr(), self.x_model.data_ptr(), self.n, float(sigma0))

    def run(self, lat: torch.Tensor, sigmas: Sequence[float], model: Model,
            noise: Optional[Callable[[int], torch.Tensor]] = None) -> torch.Tensor:
        """The whole schedule (len(sigmas) - 1 steps, sigmas[-1] == 0), lat updated in place."""
        assert lat.dtype == torch.float32 and lat.is_contiguous() and lat.numel() == self.n
        self.begin(lat, sigmas[0])
        for i in range(len(sigmas) - 1):
            self.step(i, lat, sigmas, model, noise)
        return lat
