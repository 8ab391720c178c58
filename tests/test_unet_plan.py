"""The SDXL UNet's architecture as sdvk_unet_plan lays it out, on the CPU (no device): the
parameter table under the reference checkpoint's names (unetForward and its modules,
src/Modules/Diffusion/sdvkgen.cpp:1669-1973; weight dims as linearDims reads them, conv weights
[cout][cin*9]), the parameter count, and the FLOP count against a closed-form restatement."""
import pytest

import sdvk_b200
from sdvk_b200.unet import SDXL, plan

SDXL_UNET_PARAMS = 2_567_463_684  # the SDXL base UNet's published parameter count
CONV_IN_PAD = 320 * (32 - 4) * 9  # conv_in runs its 4 latent channels zero-padded to 32


@pytest.fixture(scope="module")
def sdxl():
    return plan(2, 128, 128)


def test_parameter_count_is_sdxl(sdxl):
    n = sum(r * c if kind == sdvk_b200.UNET_Q8 else r for kind, r, c in sdxl["tensors"].values())
    assert n == SDXL_UNET_PARAMS + CONV_IN_PAD
    assert len(sdxl["tensors"]) == 1680


@pytest.mark.parametrize("name,rows,cols", [
    ("time_embed.0.weight", 1280, 320),
    ("label_emb.0.0.weight", 1280, 2816),
    ("input_blocks.0.0.weight", 320, 32 * 9),
    ("input_blocks.3.0.op.weight", 320, 320 * 9),
    ("input_blocks.4.0.skip_connection.weight", 640, 320),
    ("input_blocks.4.1.proj_in.weight", 640, 640),
    ("input_blocks.4.1.transformer_blocks.1.attn2.to_k.weight", 640, 2048),
    ("input_blocks.8.1.transformer_blocks.9.ff.net.0.proj.weight", 10240, 1280),
    ("input_blocks.8.1.transformer_blocks.9.ff.net.2.weight", 1280, 5120),
    ("middle_block.0.emb_layers.1.weight", 1280, 1280),
    ("middle_block.1.transformer_blocks.9.attn1.to_out.0.weight", 1280, 1280),
    ("middle_block.2.out_layers.3.weight", 1280, 1280 * 9),
    ("output_blocks.0.0.in_layers.2.weight", 1280, 2560 * 9),
    ("output_blocks.0.0.skip_connection.weight", 1280, 2560),
    ("output_blocks.2.2.conv.weight", 1280, 1280 * 9),
    ("output_blocks.3.0.in_layers.2.weight", 640, 1920 * 9),
    ("output_blocks.5.2.conv.weight", 640, 640 * 9),
    ("output_blocks.6.0.in_layers.2.weight", 320, 960 * 9),
    ("output_blocks.8.0.skip_connection.weight", 320, 640),
    ("out.2.weight", 4, 320 * 9),
])
def test_named_weights(sdxl, name, rows, cols):
    assert sdxl["tensors"][name] == (sdvk_b200.UNET_Q8, rows, cols)


def test_no_attention_at_level_0_and_no_qkv_bias(sdxl):
    t = sdxl["tensors"]
    assert not any(k.startswith(("input_blocks.1.1.", "input_blocks.2.1.", "output_blocks.6.1.")) for k in t)
    assert "input_blocks.7.1.transformer_blocks.0.attn1.to_q.bias" not in t
    assert t["input_blocks.7.1.transformer_blocks.0.attn1.to_out.0.bias"] == (sdvk_b200.UNET_F32, 1280, 1)
    assert t["middle_block.1.norm.weight"] == (sdvk_b200.UNET_F32, 1280, 1)


def _flops(B, H, W, ch=(320, 640, 1280), depth=(0, 2, 10), ctx=2048, Tc=77, E=1280):
    """2 M N K per GEMM / convolution (conv_in at its 4 real channels) + 4 B Tq Tk C per attention."""
    f = 0

    def conv(cin, cout, h, w):
        return 2 * B * h * w * cout * cin * 9

    def block(C, T):
        F = 4 * C
        return 2 * B * (T * 3 * C * C + 3 * T * C * C + Tc * 2 * C * ctx + T * 2 * F * C + T * C * F) \
            + 4 * B * T * T * C + 4 * B * T * Tc * C

    def res(cin, cout, h, w):
        return conv(cin, cout, h, w) + conv(cout, cout, h, w) + (2 * B * h * w * cout * cin if cin != cout else 0) \
            + 2 * B * cout * E

    def st(C, P, d):
        return 2 * 2 * B * P * C * C + d * block(C, P)

    f += 2 * B * (E * ch[0] + E * E + E * 2816 + E * E)  # time and label embeddings
    h, w, c = H, W, ch[0]
    f += conv(4, c, h, w)
    skips = [c]
    for lv in range(3):
        for _ in range(2):
            f += res(c, ch[lv], h, w)
            c = ch[lv]
            if depth[lv]:
                f += st(c, h * w, depth[lv])
            skips.append(c)
        if lv < 2:
            f += 2 * B * (h // 2) * (w // 2) * c * c * 9
            h, w = h // 2, w // 2
            skips.append(c)
    f += res(c, c, h, w) + st(c, h * w, depth[2]) + res(c, c, h, w)
    for j in range(9):
        lv = 2 - j // 3
        f += res(c + skips.pop(), ch[lv], h, w)
        c = ch[lv]
        if depth[lv]:
            f += st(c, h * w, depth[lv])
        if j in (2, 5):
            h, w = 2 * h, 2 * w
            f += conv(c, c, h, w)
    return f + conv(c, 4, h, w)


def test_flops_match_the_architecture(sdxl):
    assert sdxl["flops"] == _flops(2, 128, 128)
    assert abs(sdxl["flops"] / 1e12 - 13.52) < 0.01


def test_plan_rejects_bad_shapes():
    with pytest.raises(sdvk_b200.SdvkError):
        plan(2, 18, 16)
    with pytest.raises(sdvk_b200.SdvkError):
        plan(2, 16, 16, model_ch=(48, 128, 192))
