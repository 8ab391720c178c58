"""The SDXL UNet pass (sdvk_unet_forward: unetForward, src/Modules/Diffusion/sdvkgen.cpp:1875-1973)
on the B200 against a plain PyTorch fp32 composition of the same architecture over the same
dequantised Q8_0 parameters (TF32 off), read back from the UNet's arena by name.

The torch composition follows the reference's modules: resBlock (:1669-1707), spatialTransformer
(:1722-1777) with the BasicTransformerBlock body (:1739-1763), GEGLU as a * gelu(gate) (:1710-1720),
concatCh (:1791-1796), buildTemb (:1982-1995) and timeEmbHost (:1779-1789)."""
import math

import pytest
import torch
import torch.nn.functional as F

from tests._gpu_util import record

pytestmark = pytest.mark.gpu

SMALL = dict(model_ch=(64, 128, 192), depth=(0, 1, 2), ctx_dim=96, adm_dim=96, temb_dim=256, head_dim=64, Tctx=77)


def _params(unet):
    P = {}
    for name, info in unet.tensors():
        if name.startswith("("):
            continue
        r = unet.read(info)
        if "q" in r:
            q, s = r["q"], r["s"]
            P[name] = (q.float().view(q.shape[0], -1, 32) * s.unsqueeze(-1)).view(q.shape)
        else:
            P[name] = r["f"]
    return P


def torch_unet(P, arch, x, t, adm, ctx):
    """fp32 torch forward of the SDXL UNet over the parameter dict P (dequantised)."""
    ch, depth, hd = arch["model_ch"], arch["depth"], arch["head_dim"]

    def lin(h, name, bias=True):
        y = h @ P[name + ".weight"].t()
        b = P.get(name + ".bias")
        return y + b if (bias and b is not None) else y

    def conv(h, name, stride=1, cin=None):
        w = P[name + ".weight"]
        cout = w.shape[0]
        w = w.view(cout, w.shape[1] // 9, 3, 3)
        if cin is not None:
            w = w[:, :cin]
        return F.conv2d(h, w, P.get(name + ".bias"), stride=stride, padding=1)

    def gn(h, name, eps, silu):
        y = F.group_norm(h, 32, P[name + ".weight"], P[name + ".bias"], eps)
        return F.silu(y) if silu else y

    half = ch[0] // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, device=x.device, dtype=torch.float32) / half)
    args = t[:, None] * freqs[None]
    sin = torch.cat([torch.cos(args), torch.sin(args)], dim=1)
    emb = lin(F.silu(lin(sin, "time_embed.0")), "time_embed.2") + \
        lin(F.silu(lin(adm, "label_emb.0.0")), "label_emb.0.2")
    emb_s = F.silu(emb)

    def res(h, p):
        y = conv(gn(h, p + ".in_layers.0", 1e-5, True), p + ".in_layers.2")
        y = y + lin(emb_s, p + ".emb_layers.1")[:, :, None, None]
        y = conv(gn(y, p + ".out_layers.0", 1e-5, True), p + ".out_layers.3")
        if p + ".skip_connection.weight" in P:
            w = P[p + ".skip_connection.weight"]
            h = F.conv2d(h, w[:, :, None, None], P[p + ".skip_connection.bias"])
        return h + y

    def attn(q, k, v, heads):
        B, Tq, C = q.shape
        Tk = k.shape[1]
        q = q.view(B, Tq, heads, hd).transpose(1, 2)
        k = k.view(B, Tk, heads, hd).transpose(1, 2)
        v = v.view(B, Tk, heads, hd).transpose(1, 2)
        a = torch.softmax((q @ k.transpose(-1, -2)) / math.sqrt(hd), dim=-1) @ v
        return a.transpose(1, 2).reshape(B, Tq, C)

    def block(tk, p, C):
        heads = C // hd
        n = F.layer_norm(tk, (C,), P[p + ".norm1.weight"], P[p + ".norm1.bias"], 1e-5)
        a = attn(lin(n, p + ".attn1.to_q", False), lin(n, p + ".attn1.to_k", False), lin(n, p + ".attn1.to_v", False),
                 heads)
        tk = tk + lin(a, p + ".attn1.to_out.0")
        n = F.layer_norm(tk, (C,), P[p + ".norm2.weight"], P[p + ".norm2.bias"], 1e-5)
        a = attn(lin(n, p + ".attn2.to_q", False), lin(ctx, p + ".attn2.to_k", False),
                 lin(ctx, p + ".attn2.to_v", False), heads)
        tk = tk + lin(a, p + ".attn2.to_out.0")
        n = F.layer_norm(tk, (C,), P[p + ".norm3.weight"], P[p + ".norm3.bias"], 1e-5)
        g = lin(n, p + ".ff.net.0.proj")
        a_, gate = g.chunk(2, dim=-1)
        return tk + lin(a_ * F.gelu(gate), p + ".ff.net.2")

    def st(h, p, n):
        B, C, H, W = h.shape
        g = F.group_norm(h, 32, P[p + ".norm.weight"], P[p + ".norm.bias"], 1e-6)
        tk = lin(g.flatten(2).transpose(1, 2), p + ".proj_in")
        for i in range(n):
            tk = block(tk, f"{p}.transformer_blocks.{i}", C)
        return h + lin(tk, p + ".proj_out").transpose(1, 2).reshape(B, C, H, W)

    h = conv(x, "input_blocks.0.0", cin=4)
    hs = [h]
    names = ["input_blocks.1", "input_blocks.2", "input_blocks.4", "input_blocks.5", "input_blocks.7",
             "input_blocks.8"]
    for lv in range(3):
        for k in range(2):
            p = names[2 * lv + k]
            h = res(h, p + ".0")
            if depth[lv]:
                h = st(h, p + ".1", depth[lv])
            hs.append(h)
        if lv < 2:
            h = conv(h, f"input_blocks.{3 * lv + 3}.0.op", stride=2)
            hs.append(h)
    h = res(h, "middle_block.0")
    if depth[2]:
        h = st(h, "middle_block.1", depth[2])
    h = res(h, "middle_block.2")
    for j in range(9):
        lv = 2 - j // 3
        h = torch.cat([h, hs.pop()], dim=1)
        p = f"output_blocks.{j}"
        h = res(h, p + ".0")
        if depth[lv]:
            h = st(h, p + ".1", depth[lv])
        if j in (2, 5):
            h = F.interpolate(h, scale_factor=2, mode="nearest")
            h = conv(h, p + (".2.conv" if depth[lv] else ".1.conv"))
    return conv(gn(h, "out.0", 1e-5, True), "out.2")


def _inputs(arch, B, H, W, seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn((B, 4, H, W), generator=g, device=device)
    t = torch.tensor([999.0, 500.0, 1.0, 250.0][:B], device=device)
    adm = torch.randn((B, arch["adm_dim"]), generator=g, device=device)
    ctx = torch.randn((B, arch["Tctx"], arch["ctx_dim"]), generator=g, device=device).half()
    return x, t, adm, ctx


def _compare(unet, arch, B, H, W, seed, bar_rms, bar_max):
    dev = torch.device("cuda", 0)
    x, t, adm, ctx = _inputs(arch, B, H, W, seed, dev)
    out = unet.forward(x, t, adm, ctx)
    out2 = unet.forward(x, t, adm, ctx)
    torch.cuda.synchronize()
    unet.ctx.synchronize()
    assert torch.isfinite(out).all()
    assert torch.equal(out, out2), "two passes over the same inputs differ"
    P = _params(unet)
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = torch.backends.cudnn.allow_tf32 = False
    try:
        with torch.no_grad():
            ref = torch_unet(P, arch, x, t, adm, ctx.float())
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old
    err = (out - ref).double()
    rms = ref.double().pow(2).mean().sqrt().item()
    rel_rms = err.pow(2).mean().sqrt().item() / rms
    rel_max = err.abs().max().item() / rms
    record(f"unet {tuple(arch['model_ch'])} depth {tuple(arch['depth'])} B{B} {H}x{W} vs torch fp32",
           {"rel_rms": rel_rms, "rel_max_rms": rel_max, "ref_rms": rms, "gflop": unet.flops / 1e9,
            "launches": unet.launches})
    assert rel_rms < bar_rms and rel_max < bar_max, (rel_rms, rel_max)


def test_unet_small_vs_torch_fp32():
    """A reduced UNet (every module kind, 16 x 16 latent) against the torch fp32 composition."""
    from sdvk_b200.unet import Unet

    u = Unet(2, 16, 16, device=0, **SMALL)
    u.init_random(11)
    _compare(u, u.arch, 2, 16, 16, 5, 5e-3, 5e-2)
    u.close()


def test_unet_sdxl_1024_vs_torch_fp32():
    """The SDXL architecture at the 1024^2 latent (128 x 128), batch 2 (config 3's pass)."""
    from sdvk_b200.unet import SDXL, Unet

    u = Unet(2, 128, 128, device=0)
    u.init_random(3)
    _compare(u, dict(SDXL), 2, 128, 128, 7, 5e-3, 5e-2)
    u.close()


def test_unet_graph_replay_matches_eager():
    """The pass captured in a CUDA graph replays to the eager result bit for bit (fixed addresses)."""
    from sdvk_b200.unet import Unet

    u = Unet(2, 16, 16, device=0, **SMALL)
    u.init_random(12)
    dev = torch.device("cuda", 0)
    x, t, adm, ctx = _inputs(u.arch, 2, 16, 16, 9, dev)
    eager = u.forward(x, t, adm, ctx).clone()
    torch.cuda.synchronize()
    out = torch.empty_like(x)
    s = torch.cuda.Stream(dev)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        u.forward(x, t, adm, ctx, out=out)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    del g
    u.close()


def test_unet_forward_replays_its_own_graph(monkeypatch):
    """sdvk_unet_forward runs the launches themselves on a first call, captures a CUDA graph on a second
    call with the same buffers and replays it after that; the graph reads the buffers' new contents at
    every replay, new buffers start over, and every result equals the launches made one by one
    (SDVK_UNET_GRAPH=0) bit for bit."""
    from sdvk_b200.unet import Unet

    u = Unet(2, 16, 16, device=0, **SMALL)
    u.init_random(13)
    dev = torch.device("cuda", 0)
    x, t, adm, ctx = _inputs(u.arch, 2, 16, 16, 3, dev)
    x2 = x * 0.5 + 0.1
    monkeypatch.setenv("SDVK_UNET_GRAPH", "0")
    eager1 = u.forward(x, t, adm, ctx).clone()
    eager2 = u.forward(x2, t, adm, ctx).clone()
    monkeypatch.delenv("SDVK_UNET_GRAPH")
    out = torch.empty_like(x)
    runs = [u.forward(x, t, adm, ctx, out=out).clone() for _ in range(3)]  # launches, capture, replay
    x_keep = x.clone()
    x.copy_(x2)  # the same buffer, new contents
    replayed = u.forward(x, t, adm, ctx, out=out).clone()
    other = torch.empty_like(x)
    fresh = u.forward(x_keep, t, adm, ctx, out=other).clone()  # new buffers
    torch.cuda.synchronize()
    u.ctx.synchronize()
    for r in runs:
        assert torch.equal(r, eager1)
    assert torch.equal(replayed, eager2)
    assert torch.equal(fresh, eager1)
    u.close()


def test_unet_rejects_bad_shapes():
    import sdvk_b200
    from sdvk_b200.unet import Unet

    with pytest.raises(sdvk_b200.SdvkError):
        Unet(2, 18, 16, device=0, **SMALL)  # latent sides must be multiples of 4
    with pytest.raises(sdvk_b200.SdvkError):
        Unet(2, 16, 16, device=0, **dict(SMALL, model_ch=(48, 128, 192)))  # 48 is not a multiple of head_dim


def test_unet_error_paths():
    """A device-less plan cannot run a pass (SDVK_E_STATE), and a UNet whose parameters were never
    prepared refuses to run rather than reading uninitialised repacks."""
    import ctypes

    import sdvk_b200
    from sdvk_b200 import lib
    from sdvk_b200.torch_ops import context
    from sdvk_b200.unet import Unet, _desc

    dev = torch.device("cuda", 0)
    x, t, adm, ctx = _inputs(SMALL, 2, 16, 16, 3, dev)
    out = torch.empty_like(x)
    h = ctypes.c_void_p()
    assert lib().sdvk_unet_plan(ctypes.byref(_desc(2, 16, 16, dict(SMALL))), ctypes.byref(h)) == sdvk_b200.OK
    c = context(dev)
    st = lib().sdvk_unet_forward(c.handle, h, x.data_ptr(), t.data_ptr(), adm.data_ptr(), ctx.data_ptr(),
                                 sdvk_b200.F16, out.data_ptr())
    assert st == sdvk_b200.E_STATE
    lib().sdvk_unet_destroy(h)
    u = Unet(2, 16, 16, device=0, **SMALL)  # created, never initialised or prepared
    with pytest.raises(sdvk_b200.SdvkError) as e:
        u.forward(x, t, adm, ctx)
    assert e.value.status == sdvk_b200.E_STATE
    u.close()
