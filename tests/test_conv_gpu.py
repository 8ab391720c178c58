"""3x3 convolutions with Q8_0 weights (conv3RawInto / conv3s2: im2col + the NN GEMM + bias) on the
B200 against the float64 convolution, with the fp32 restatement of the reference's im2col and
gemm_nn_q8_v.comp reported beside."""
import numpy as np
import pytest
import torch

import sdvk_b200
from sdvk_b200 import torch_ops
from tests._gpu_util import check_gemm, dev, host, record

pytestmark = pytest.mark.gpu

CONV_CASES = [
    # (B, cin, cout, H, W, stride, off, x dtype, out dtype)
    (2, 32, 64, 16, 16, 1, -1, "f16", "f32"),
    (1, 64, 96, 20, 24, 2, -1, "f16", "f16"),
    (1, 32, 64, 16, 24, 2, 0, "f32", "f32"),
    (2, 320, 320, 32, 32, 1, -1, "f16", "f32"),  # an SDXL level-1 conv at a 256^2 latent
    (1, 96, 128, 24, 40, 2, -1, "bf16", "f32"),
    # the row-segment im2col (OW % 8 == 0): both stride-2 paddings and an fp32 input
    (2, 64, 64, 32, 48, 2, -1, "f16", "f32"),
    (1, 32, 64, 32, 32, 2, 0, "bf16", "f32"),
    (1, 32, 32, 16, 16, 1, -1, "f32", "f32"),
]
_TT = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}


@pytest.mark.parametrize("B,cin,cout,H,W,stride,off,dt,out", CONV_CASES)
def test_conv3x3_q8(orc, cuda_ok, B, cin, cout, H, W, stride, off, dt, out):
    x = orc.normal_f32(51, 0, (B, cin, H, W))
    xt = torch.from_numpy(x).cuda().to(_TT[dt])
    xr = xt.float().cpu().numpy()  # the values the kernel sees
    q, _, s = orc.q8_weights(51, 1, cout, cin * 9)
    bias = orc.normal_f32(51, 2, (cout,)) * 0.1
    y = torch_ops.conv3x3_q8(xt, dev(q), dev(s), dev(bias), stride, off, _TT[out])
    ref = orc.conv3x3_f64(xr, q, s, bias, stride, off)
    assert tuple(y.shape) == ref.shape
    st_ref = orc.err_stats(orc.conv3x3_shader(xr, q, s, bias, stride, off), ref)
    record(f"conv3x3 B{B} {cin}->{cout} {H}x{W} s{stride} off{off} {dt}->{out} (reference fp32 beside)", st_ref)
    check_gemm(orc, f"conv3x3 B{B} {cin}->{cout} {H}x{W} s{stride} off{off} {dt}->{out}", host(y).astype(np.float64),
               ref, dt if out == "f32" else "bf16" if dt == "bf16" else "f16")


def test_conv3x3_bands_match_one_pass(orc, cuda_ok):
    """A workspace of a few output rows (several bands, a short last one) gives the bitwise result of
    one whole-image band."""
    B, cin, cout, H, W = 1, 64, 64, 21, 16
    x = torch.from_numpy(orc.normal_f32(52, 0, (B, cin, H, W))).cuda().half()
    q, _, s = orc.q8_weights(52, 1, cout, cin * 9)
    full = torch_ops.conv3x3_q8(x, dev(q), dev(s), None)
    band = torch_ops.conv3x3_q8(x, dev(q), dev(s), None, workspace_bytes=cin * 9 * W * 2 * 4)  # 4 rows per band
    assert torch.equal(full, band)


def test_conv3x3_errors(cuda_ok):
    ctx = torch_ops.context()
    x = torch.zeros((1, 4, 8, 8), device="cuda", dtype=torch.float16)
    q = torch.zeros((8, 36), device="cuda", dtype=torch.int8)
    s = torch.zeros((8,), device="cuda")
    y = torch.zeros((1, 8, 8, 8), device="cuda")
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    with pytest.raises(sdvk_b200.SdvkError) as e:  # cin*9 = 36: not whole Q8_0 blocks
        ctx.conv3x3_q8(x.data_ptr(), sdvk_b200.F16, q.data_ptr(), s.data_ptr(), None, y.data_ptr(), sdvk_b200.F32,
                       1, 4, 8, 8, 8, 1, -1, ws.data_ptr(), ws.numel())
    assert e.value.status == sdvk_b200.E_SHAPE
    with pytest.raises(sdvk_b200.SdvkError) as e:  # stride 3
        ctx.conv3x3_q8(x.data_ptr(), sdvk_b200.F16, q.data_ptr(), s.data_ptr(), None, y.data_ptr(), sdvk_b200.F32,
                       1, 32, 8, 8, 8, 3, -1, ws.data_ptr(), ws.numel())
    assert e.value.status == sdvk_b200.E_SHAPE
