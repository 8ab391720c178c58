"""Classifier-free guidance across a GPU pair.

The reference evaluates both guidance passes on one device, one after the other
(runPass(cond), runPass(uncond), src/Modules/Diffusion/sdvkgen.cpp:3812-3813), and combines them on the
host (:3825-3845).  With two GPUs per image the pair's rank 0 runs the conditional pass and rank 1
the unconditional one.  After each evaluation the two predictions are all-gathered, so every rank
holds [cond, uncond]; both ranks then run the same combine on the same bytes and keep bit-identical
latents, with no broadcast.  torch.distributed carries the all-gather (NCCL between GPUs, gloo on the
host); the combine on the device is libsdvk_b200's CUDA kernel (sdvk_cfg_combine).

Failure handling: the process group carries a timeout.  A partner that raises, exits or never joins
ends the next all-gather with an error on the surviving rank instead of a hang; `guided` re-raises it
as PairFailure, between steps, with no kernel of ours in flight.
"""
from __future__ import annotations

from typing import Callable, List, Optional

import torch
import torch.distributed as dist


class PairFailure(RuntimeError):
    """The partner rank failed or stopped answering during a guidance exchange."""


def device_combine(cond: torch.Tensor, uncond: torch.Tensor, cfg: float, rescale: float) -> torch.Tensor:
    """sdvk_cfg_combine on the device (fp32)."""
    from . import torch_ops

    return torch_ops.cfg_combine(cond, uncond, cfg, rescale)


def pair_groups(world: int) -> List[Optional["dist.ProcessGroup"]]:
    """One process group per rank pair (2i, 2i+1).  Every rank must call this, in the same order."""
    if world % 2:
        raise ValueError("the CFG-pair mode needs an even number of ranks")
    return [dist.new_group([2 * i, 2 * i + 1]) for i in range(world // 2)]


class CfgPair:
    """The guidance exchange of one rank pair.

    rank 0 of the pair evaluates the conditional pass, rank 1 the unconditional one; `guided` takes
    this rank's prediction and returns the combined guidance on both ranks."""

    def __init__(self, group: Optional["dist.ProcessGroup"], cfg: float, rescale: float = 0.0,
                 combine: Optional[Callable[[torch.Tensor, torch.Tensor, float, float], torch.Tensor]] = None):
        if dist.get_world_size(group) != 2:
            raise ValueError("a CFG pair has exactly two ranks")
        self.group = group
        self.rank = dist.get_rank(group)
        self.cfg = float(cfg)
        self.rescale = float(rescale)
        self.combine = combine or device_combine

    @property
    def is_cond(self) -> bool:
        return self.rank == 0

    def exchange(self, eps_local: torch.Tensor):
        """All-gather this rank's prediction: (cond, uncond), flat, the same bytes on both ranks."""
        flat = eps_local.contiguous().view(-1)
        both = torch.empty(2 * flat.numel(), dtype=flat.dtype, device=flat.device)
        try:
            dist.all_gather_into_tensor(both, flat, group=self.group)
        except Exception as e:  # partner raised, exited or timed out
            raise PairFailure(f"guidance exchange failed on pair rank {self.rank}: {e}") from e
        cond, uncond = both.view(2, -1)
        return cond, uncond

    def guided(self, eps_local: torch.Tensor) -> torch.Tensor:
        cond, uncond = self.exchange(eps_local)
        return self.combine(cond, uncond, self.cfg, self.rescale).view(eps_local.shape)

    def sampler_model(self, unet: Callable[[torch.Tensor, int, int, float], torch.Tensor]):
        """A model callback for sdvk_b200.sampler.DeviceSampler: this rank evaluates its own pass with
        unet(x_model, step, phase, sigma), the pair exchanges the two predictions, and each rank's
        sampler step (sdvk_sampler_step, guidance combine included) runs on the same bytes, so the
        latents stay bit-identical (sdvkgen.cpp:3806-3846 with the two passes on two GPUs)."""

        def model(x_model, step, phase, sigma):
            return self.exchange(unet(x_model, step, phase, sigma))

        return model
