"""The transformer block and its LayerNorm / GEGLU operators on the B200 against
the oracle: fp64 truth, with the restated reference fp32 arithmetic's own error reported beside ours."""
import numpy as np
import pytest
import torch

import sdvk_b200
from sdvk_b200 import torch_ops
from tests._gpu_util import dev, host, record

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,d,out", [(2048, 1280, "f16"), (333, 1280, "f32"), (77, 320, "f16"), (5, 2048, "f32")])
def test_layernorm(orc, cuda_ok, rows, d, out):
    x = orc.normal_f32(11, 0, (rows, d)) * 3.0 + 0.5
    g = orc.normal_f32(11, 1, (d,)) * 0.2 + 1.0
    b = orc.normal_f32(11, 2, (d,)) * 0.1
    y = torch_ops.layernorm(dev(x), dev(g), dev(b), out_dtype=torch.float16 if out == "f16" else torch.float32)
    ref = orc.layernorm_f64(x.astype(np.float64), g, b)
    st = orc.err_stats(host(y), ref)
    record(f"layernorm {rows}x{d} ->{out}", st)
    assert st["finite"] and st["rel_max"] <= (1e-3 if out == "f16" else 2e-6), st


def test_layernorm_dispatch_matches_reference_shader(orc, cuda_ok):
    """Engine::dispatch("layernorm_fwd", {x, gamma, beta, y}, {rows, d, eps, affine}) in fp32."""
    rows, d = 300, 1280
    x = orc.normal_f32(12, 0, (rows, d)) * 2.0
    g = orc.normal_f32(12, 1, (d,))
    b = orc.normal_f32(12, 2, (d,))
    xd, gd, bd = dev(x), dev(g), dev(b)
    y = torch.full_like(xd, float("nan"))
    bufs = [sdvk_b200.Buf(t.data_ptr(), 0, t.numel() * 4) for t in (xd, gd, bd, y)]
    torch_ops.context().dispatch("layernorm_fwd", bufs, sdvk_b200.pack_ln(rows, d, 1e-5, 1), rows)
    st = orc.err_stats(host(y), orc.layernorm_shader(x, g, b))
    record("layernorm_fwd dispatch vs reference shader", st)
    assert st["rel_max"] <= 2e-6, st


@pytest.mark.parametrize("rows,F", [(2048, 5120), (37, 1280)])
def test_geglu(orc, cuda_ok, rows, F):
    h = torch.from_numpy(orc.normal_f16(13, 0, (rows, 2 * F)) * 2).cuda()
    y = torch_ops.geglu(h)
    hf = h.float().cpu().numpy().astype(np.float64)
    ref = hf[:, :F] * orc._gelu64(hf[:, F:])
    st = orc.err_stats(host(y), ref)
    record(f"geglu {rows}x{F}", st)
    assert st["rel_max"] <= 2e-3, st


@pytest.mark.parametrize("rows,F,K", [(2048, 5120, 1280), (300, 256, 640)])
def test_gemm_geglu_epilogue(orc, cuda_ok, rows, F, K):
    """ff.net.0 with GEGLU in the GEMM epilogue (weight repacked by sdvk_geglu_interleave) against
    fp64: a * gelu(gate) for (a | gate) = x W^T + b."""
    x = orc.normal_f16(14, 0, (rows, K))
    q, _, sc = orc.q8_weights(14, 1, 2 * F, K)
    b = orc.normal_f32(14, 2, (2 * F,)) * 0.05
    qi, si, bi = torch_ops.geglu_interleave(dev(q), dev(sc), dev(b))
    y = torch_ops.gemm_q8_nt_geglu(torch.from_numpy(x).cuda(), qi, si, bi)
    g = orc.gemm_nt_q8_f64(x.astype(np.float32), q, sc, b)
    ref = g[:, :F] * orc._gelu64(g[:, F:])
    st = orc.err_stats(host(y), ref)
    record(f"gemm+geglu epilogue {rows}x{2 * F}x{K}", st)
    # the output is heavy-tailed and stored as f16: its largest values round by 2^-11 of max|ref|,
    # so the max error is bounded against max|ref| (as for the standalone GEGLU kernel)
    assert st["finite"] and st["rel_rms"] <= 1e-3 and st["rel_max"] <= 2e-3, st


def _weights(orc, seed, C, Cc, F, fused=True, ln_random=False, qkv_bias=False):
    """Random Q8_0 weights of BASELINE config 0's distribution for every linear of the block."""
    W, Wd = {}, {}

    def q8(stream, n, k, bias):
        q, _, s = orc.q8_weights(seed, stream, n, k)
        b = orc.normal_f32(seed, 100 + stream, (n,)) * 0.02 if bias else None
        return q, s, b

    def put(name, w):
        W[name] = w
        Wd[name] = tuple(dev(a) if a is not None else None for a in w)

    if fused:  # q, k, v (and k2, v2) as row blocks of one weight: the single-GEMM path
        q, s, b = q8(1, 3 * C, C, qkv_bias)
        qd, sd, bd = dev(q), dev(s), (dev(b) if b is not None else None)
        for i, name in enumerate(("q", "k", "v")):
            W[name] = (q[i * C:(i + 1) * C], s[i * C * C // 32:(i + 1) * C * C // 32],
                       b[i * C:(i + 1) * C] if b is not None else None)
            Wd[name] = (qd[i * C:(i + 1) * C], sd[i * C * C // 32:(i + 1) * C * C // 32],
                        bd[i * C:(i + 1) * C] if bd is not None else None)
        q, s, _ = q8(2, 2 * C, Cc, False)
        qd, sd = dev(q), dev(s)
        for i, name in enumerate(("k2", "v2")):
            W[name] = (q[i * C:(i + 1) * C], s[i * C * Cc // 32:(i + 1) * C * Cc // 32], None)
            Wd[name] = (qd[i * C:(i + 1) * C], sd[i * C * Cc // 32:(i + 1) * C * Cc // 32], None)
    else:
        put("q", q8(1, C, C, qkv_bias))
        put("k", q8(3, C, C, qkv_bias))
        put("v", q8(4, C, C, qkv_bias))
        put("k2", q8(5, C, Cc, False))
        put("v2", q8(6, C, Cc, False))
    put("o", q8(7, C, C, True))
    put("q2", q8(8, C, C, False))
    put("o2", q8(9, C, C, True))
    put("ff1", q8(10, 2 * F, C, True))
    put("ff2", q8(11, C, F, True))
    for i in (1, 2, 3):
        g = (orc.normal_f32(seed, 200 + i, (C,)) * 0.1 + 1.0) if ln_random else np.ones(C, np.float32)
        b = (orc.normal_f32(seed, 210 + i, (C,)) * 0.1) if ln_random else np.zeros(C, np.float32)
        W[f"ln{i}_w"], W[f"ln{i}_b"] = g, b
        Wd[f"ln{i}_w"], Wd[f"ln{i}_b"] = dev(g), dev(b)
    return W, Wd


BLOCK_CASES = [
    # (B, T, C, heads, Tctx, Cctx, F, fused weights, random LN / q-k-v biases, GEGLU epilogue)
    (2, 1024, 1280, 20, 77, 2048, 5120, True, False, True),  # config 2
    (2, 1024, 1280, 20, 77, 2048, 5120, True, False, False),
    (1, 300, 640, 10, 77, 1024, 1280, False, True, False),
]


@pytest.mark.parametrize("B,T,C,heads,Tc,Cc,F,fused,rnd,il", BLOCK_CASES)
def test_transformer_block(orc, cuda_ok, B, T, C, heads, Tc, Cc, F, fused, rnd, il):
    """x += attn1(LN1 x); x += attn2(LN2 x, ctx); x += ff2(geglu(ff1(LN3 x))), checked on a sample of
    query rows per image (keys and values cover every token)."""
    W, Wd = _weights(orc, 21, C, Cc, F, fused=fused, ln_random=rnd, qkv_bias=rnd)
    if il:  # GEGLU folded into the ff1 GEMM's epilogue (the oracle keeps the original weight)
        Wd["ff1"] = torch_ops.geglu_interleave(*Wd["ff1"])
        Wd["ff1_geglu_interleaved"] = True
    x = orc.normal_f32(22, 0, (B, T, C))
    ctx = orc.normal_f16(22, 1, (B, Tc, Cc))
    xd = dev(x)
    torch_ops.transformer_block(xd, torch.from_numpy(ctx).cuda(), heads, Wd)
    torch.cuda.synchronize()
    torch_ops.context().synchronize()
    rows = np.sort(np.random.default_rng(3).choice(T, size=min(T, 96), replace=False))
    ctx32 = ctx.astype(np.float32)
    ref = orc.block_f64(x, ctx32, heads, W, rows)
    got = host(xd)[:, rows]
    # compare the block's update (x_out - x_in): the residual itself is carried exactly
    delta_ref = ref - x[:, rows]
    st = orc.err_stats(got - x[:, rows], delta_ref)
    shader = orc.block_shader(x, ctx32, heads, W, rows)
    st_ref = orc.err_stats(shader - x[:, rows], delta_ref)
    record(f"block B{B} T{T} C{C} h{heads} ctx{Tc}x{Cc} F{F} fused={fused} geglu_epilogue={il}", st, st_ref)
    assert st["finite"], st
    assert st["rel_rms"] <= 5e-3 and st["rel_max_rms"] <= 5e-2, (st, st_ref)


def test_transformer_block_workspace_and_errors(cuda_ok):
    d = sdvk_b200.BlockDesc()
    d.batch, d.T, d.C, d.heads, d.Tctx, d.Cctx, d.ff_inner = 2, 1024, 1280, 20, 77, 2048, 5120
    need = sdvk_b200.Context.block_workspace(d)
    assert need >= 2 * 1024 * (1280 * 5 + 5120 * 3) * 2
    ctx = torch_ops.context()
    x = torch.zeros((2, 1024, 1280), device="cuda")
    d.x = x.data_ptr()
    ws = torch.empty(need // 2, dtype=torch.uint8, device="cuda")
    with pytest.raises(sdvk_b200.SdvkError) as e:
        ctx.transformer_block(d, ws.data_ptr(), ws.numel())  # workspace too small
    assert e.value.status == sdvk_b200.E_ARG
    d.heads = 10  # head dim 128
    with pytest.raises(sdvk_b200.SdvkError) as e:
        ctx.transformer_block(d, ws.data_ptr(), need)
    assert e.value.status == sdvk_b200.E_SHAPE
