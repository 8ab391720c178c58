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


# ---------------------------------------------------------------------------- the implicit-GEMM form
# (conv_tc2.cuh): TMA im2col-mode loads from channels-last fp16 x, weights repacked to fp16 tap-major.
IMPLICIT_CASES = [
    # (B, cin, cout, H, W, stride, off, out dtype)
    (2, 320, 320, 32, 32, 1, -1, "f32"),   # the level-0 channel count; BN 160
    (2, 64, 64, 16, 48, 1, -1, "f32"),     # 128-position blocks start mid-row (the pixel box wraps rows)
    (1, 192, 640, 24, 16, 1, -1, "f32"),   # 1.5 pair tiles: the last tile's odd CTA lies past the last image
    (3, 128, 160, 16, 16, 1, -1, "f16"),   # fp16 output
    (2, 128, 4, 16, 16, 1, -1, "f32"),     # conv_out's 4 channels (BN 32, 28 rows of the tile clipped)
    (2, 64, 64, 32, 48, 2, -1, "f32"),     # the UNet downsampler's symmetric ring
    (1, 128, 96, 32, 32, 2, 0, "f32"),     # right/bottom padding only
]


def _implicit_inputs(orc, seed, B, cin, cout, H, W):
    x = orc.normal_f32(seed, 0, (B, cin, H, W))
    xt = torch.from_numpy(x).cuda().half()
    q, _, s = orc.q8_weights(seed, 1, cout, cin * 9)
    bias = orc.normal_f32(seed, 2, (cout,)) * 0.1
    return xt, xt.float().cpu().numpy(), q, s, bias


@pytest.mark.parametrize("B,cin,cout,H,W,stride,off,out", IMPLICIT_CASES)
def test_conv3x3_implicit(orc, cuda_ok, B, cin, cout, H, W, stride, off, out):
    assert sdvk_b200.Context.conv3x3_implicit_ok(B, cin, H, W, stride)
    xt, xr, q, s, bias = _implicit_inputs(orc, 61, B, cin, cout, H, W)
    w16 = torch_ops.conv3x3_weights_f16(dev(q), dev(s))
    xcl = xt.permute(0, 2, 3, 1).contiguous()
    y = torch_ops.conv3x3_nhwc(xcl, w16, dev(bias), stride, off, _TT[out])
    ref = orc.conv3x3_f64(xr, q, s, bias, stride, off)
    assert tuple(y.shape) == ref.shape
    check_gemm(orc, f"conv3x3 implicit B{B} {cin}->{cout} {H}x{W} s{stride} off{off} f16->{out}",
               host(y).astype(np.float64), ref, "f16")


def test_conv3x3_weights_f16_exact(orc, cuda_ok):
    """The repack is w16[o][(cb*9 + tap)*64 + j] = fp16(q[o][(cb*64 + j)*9 + tap] * scale), bit for bit."""
    cout, cin = 96, 128
    q, _, s = orc.q8_weights(62, 1, cout, cin * 9)
    w16 = host(torch_ops.conv3x3_weights_f16(dev(q), dev(s)))
    K = cin * 9
    w = (q.reshape(cout, -1, 32).astype(np.float32) * s.reshape(cout, -1, 1)).reshape(cout, cin, 9)
    want = w.reshape(cout, cin // 64, 64, 9).transpose(0, 1, 3, 2).reshape(cout, K).astype(np.float16)
    assert np.array_equal(w16.view(np.uint16), want.view(np.uint16))


def test_conv3x3_implicit_tile_widths_agree(orc, cuda_ok, monkeypatch):
    """Every pair-tile width sums each output over the same stages in the same order: the same bits."""
    B, cin, cout, H, W = 2, 128, 320, 16, 32
    xt, _, q, s, bias = _implicit_inputs(orc, 63, B, cin, cout, H, W)
    w16 = torch_ops.conv3x3_weights_f16(dev(q), dev(s))
    xcl = xt.permute(0, 2, 3, 1).contiguous()
    outs = []
    for bn in (32, 64, 128, 160, 192, 256):
        monkeypatch.setenv("SDVK_CONV_BN", str(bn))
        outs.append(torch_ops.conv3x3_nhwc(xcl, w16, dev(bias)))
    monkeypatch.delenv("SDVK_CONV_BN")
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def test_conv3x3_q8_takes_the_implicit_form(orc, cuda_ok, monkeypatch):
    """sdvk_conv3x3_q8 on an fp16 input goes the implicit way when it can (workspace: x channels-last and
    the repacked weights); against the im2col form the difference is fp32 summation order."""
    B, cin, cout, H, W = 2, 320, 320, 32, 32
    xt, xr, q, s, bias = _implicit_inputs(orc, 64, B, cin, cout, H, W)
    got = torch_ops.conv3x3_q8(xt, dev(q), dev(s), dev(bias))
    monkeypatch.setenv("SDVK_CONV_IMPLICIT", "0")
    assert not sdvk_b200.Context.conv3x3_implicit_ok(B, cin, H, W, 1)
    explicit = torch_ops.conv3x3_q8(xt, dev(q), dev(s), dev(bias))
    monkeypatch.delenv("SDVK_CONV_IMPLICIT")
    st = orc.err_stats(host(got).astype(np.float64), host(explicit).astype(np.float64))
    record("conv3x3 implicit vs im2col form", st)
    assert 0.0 < st["rel_rms"] <= 1e-5, st  # different summation order, same products
    check_gemm(orc, "conv3x3_q8 implicit form", host(got).astype(np.float64), orc.conv3x3_f64(xr, q, s, bias), "f16")


def test_conv3x3_implicit_accumulates_with_image_bias(orc, cuda_ok):
    """y += conv(x) + bias[b] (the ResBlock's conv2 into the skip path, conv1's per-image bias)."""
    B, cin, cout, H, W = 2, 128, 192, 16, 16
    xt, xr, q, s, _ = _implicit_inputs(orc, 65, B, cin, cout, H, W)
    bias = orc.normal_f32(65, 3, (B, 200)) * 0.1  # per-image rows of 200 (stride), first cout used
    y0 = orc.normal_f32(65, 4, (B, cout, H, W))
    y = dev(y0)
    w16 = torch_ops.conv3x3_weights_f16(dev(q), dev(s))
    torch_ops.conv3x3_nhwc(xt.permute(0, 2, 3, 1).contiguous(), w16, dev(bias), bias_stride=200, out=y)
    ref = orc.conv3x3_f64(xr, q, s, None) + y0 + bias[:, :cout, None, None]
    check_gemm(orc, "conv3x3 implicit accumulate + per-image bias", host(y).astype(np.float64), ref, "f16")


def test_conv3x3_implicit_rejects_shapes(cuda_ok):
    ctx = torch_ops.context()
    x = torch.zeros((1, 16, 16, 96), device="cuda", dtype=torch.float16)
    w = torch.zeros((64, 96 * 9), device="cuda", dtype=torch.float16)
    y = torch.zeros((1, 64, 16, 16), device="cuda")
    assert not sdvk_b200.Context.conv3x3_implicit_ok(1, 96, 16, 16, 1)  # cin % 64
    with pytest.raises(sdvk_b200.SdvkError) as e:
        ctx.conv3x3_nhwc(x.data_ptr(), w.data_ptr(), None, 0, False, y.data_ptr(), sdvk_b200.F32, 1, 96, 64, 16, 16,
                         1, -1)
    assert e.value.status == sdvk_b200.E_SHAPE
    assert not sdvk_b200.Context.conv3x3_implicit_ok(1, 64, 12, 10, 1)  # 120 positions
    assert not sdvk_b200.Context.conv3x3_implicit_ok(1, 64, 16, 16, 1)  # a 32 KB input


def test_groupnorm_channels_last_matches_channel_major(orc, cuda_ok):
    """sdvk_groupnorm_cl writes the values of sdvk_groupnorm, rounded to fp16 and transposed, bit for bit."""
    B, C, H, W = 2, 320, 24, 40
    x = dev(orc.normal_f32(66, 0, (B, C, H, W)) * 3 + 0.5)
    gamma = dev(orc.normal_f32(66, 1, (C,)))
    beta = dev(orc.normal_f32(66, 2, (C,)))
    for silu in (False, True):
        ref = torch_ops.groupnorm(x, gamma, beta, 32, 1e-5, silu)
        got = torch_ops.groupnorm_cl(x, gamma, beta, 32, 1e-5, silu)
        want = ref.reshape(B, C, H * W).transpose(1, 2).half()
        assert torch.equal(got, want), (silu, (got.float() - want.float()).abs().max())
