"""Shared helpers of the GPU parity tests: stated tolerances and error reporting.

Tolerances are against the fp64 dequantised truth computed by the oracle on the SAME inputs the GPU
saw (fp16/bf16 inputs are converted exactly to fp64).  They follow from the operand precision:
  f16 operands   (10-bit mantissa)  rel_rms <= 1e-3,  max|err| / RMS(ref) <= 1e-2
  bf16 operands  (7-bit mantissa)   rel_rms <= 8e-3,  max|err| / RMS(ref) <= 8e-2
  tf32 (fp32 in, 10-bit mantissa)   rel_rms <= 2e-3,  max|err| / RMS(ref) <= 2e-2
Attention (f16/bf16 P.V, fp32 accumulation): max|err| / max|ref| <= 5e-3 (f16), 3e-2 (bf16);
fp32 inputs at the default (reference) precision are computed in fp32 and meet the reference's 2e-5.
The reference's own fp32 shader math meets 2e-5; its error is printed next to ours.
"""
import json
import os

import numpy as np
import torch

GEMM_TOL = {"f16": (1e-3, 1e-2), "bf16": (8e-3, 8e-2), "f32": (2e-3, 2e-2)}
# "f32_ref": fp32 inputs under SDVK_PRECISION_REFERENCE (the default) meet the reference's own bar
ATTN_TOL = {"f16": 5e-3, "bf16": 3e-2, "f32": 5e-3, "f32_ref": 2e-5}
REPORT = os.environ.get("SDVK_PARITY_REPORT")


def dev(x) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    torch.cuda.synchronize()
    if t.dtype == torch.bfloat16:
        t = t.float()
    return t.cpu().numpy()


def record(name: str, stats: dict, reference_stats: dict = None) -> None:
    """Append a parity line (used to build the published parity table); `reference_stats` is the
    restated reference fp32 arithmetic's error against the same truth, where the test has it."""
    line = {"case": name, **stats}
    if reference_stats is not None:
        line["reference_fp32"] = reference_stats
    print("PARITY", json.dumps(line))
    if REPORT:
        with open(REPORT, "a") as f:
            f.write(json.dumps(line) + "\n")


def check_gemm(orc, name, got, ref, kind):
    st = orc.err_stats(got, ref)
    record(name, st)
    rms_tol, max_tol = GEMM_TOL[kind]
    assert st["finite"], (name, st)
    assert st["rel_rms"] <= rms_tol and st["rel_max_rms"] <= max_tol, (name, st)
    return st


def check_attn(orc, name, got, ref, kind):
    st = orc.err_stats(got, ref)
    record(name, st)
    assert st["finite"], (name, st)
    assert st["rel_max"] <= ATTN_TOL[kind], (name, st)
    return st
