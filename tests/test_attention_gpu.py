"""Fused attention parity on the B200 through the C ABI vs the oracle and the reference's golden
outputs."""
import json
import os

import numpy as np
import pytest
import torch

import sdvk_b200
from sdvk_b200 import torch_ops
from tests._gpu_util import check_attn, dev, host

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _golden_cases(orc):
    with open(os.path.join(GOLDEN, "manifest.json")) as f:
        man = json.load(f)
    rng = orc.MT19937(20261101)
    for e in man["attention"]:
        Tq, Tk, C = e["Tq"], e["Tk"], e["C"]
        q = rng.uniform_f32(Tq * C).reshape(Tq, C)
        k = rng.uniform_f32(Tk * C).reshape(Tk, C)
        v = rng.uniform_f32(Tk * C).reshape(Tk, C)
        ref = np.fromfile(os.path.join(GOLDEN, e["file"]), np.float32).reshape(Tq, C)
        yield e, q, k, v, ref


@pytest.mark.parametrize("precision", ["reference", "fast"])
def test_reference_test_shapes_fused_attention(orc, cuda_ok, precision):
    """tests/fused_attn_test.cpp's four shapes (fp32 buffers) through fusedAttention's replacement,
    against the reference's own fp64 outputs (golden).  At the default precision fp32 inputs are
    computed in fp32 and meet the reference's own 2e-5; in fast mode they run as f16 operands on the
    tensor cores (bar 5e-3)."""
    ctx = torch_ops.context()
    ctx.set_precision(sdvk_b200.PRECISION_FAST if precision == "fast" else sdvk_b200.PRECISION_REFERENCE)
    try:
        for e, q, k, v, ref in _golden_cases(orc):
            qd, kd, vd = dev(q), dev(k), dev(v)
            o = torch.full_like(qd, float("nan"))
            ctx.fused_attention(qd.data_ptr(), kd.data_ptr(), vd.data_ptr(), o.data_ptr(), e["Tq"], e["Tk"], e["C"],
                                e["heads"], e["causal"])
            check_attn(orc, f"fusedAttention[{precision}] golden Tq={e['Tq']} Tk={e['Tk']} C={e['C']} h={e['heads']}",
                       host(o), ref, "f32_ref" if precision == "reference" else "f32")
    finally:
        ctx.set_precision(sdvk_b200.PRECISION_REFERENCE)


def test_reference_test_shapes_dispatch(orc, cuda_ok):
    """Same shapes through Engine::dispatch("fused_attn" / "fused_attn_tiled", FaPush)."""
    ctx = torch_ops.context()
    for e, q, k, v, ref in _golden_cases(orc):
        hd = e["C"] // e["heads"]
        qd, kd, vd = dev(q), dev(k), dev(v)
        o = torch.full_like(qd, float("nan"))
        bufs = [sdvk_b200.Buf(t.data_ptr(), 0, t.numel() * 4) for t in (qd, kd, vd, o)]
        name = "fused_attn_tiled" if hd == 64 and e["Tk"] >= 256 else "fused_attn"
        push = sdvk_b200.pack_fa(e["Tq"], e["Tk"], e["C"], e["heads"], hd, e["causal"],
                                 float(np.float32(1) / np.sqrt(np.float32(hd))))
        ctx.dispatch(name, bufs, push, (e["Tq"] + 63) // 64, e["heads"], 1)
        check_attn(orc, f"dispatch {name} golden Tq={e['Tq']}", host(o), ref, "f32_ref")


CONFIG1 = [
    # (B, Tq, Tk, heads, hd, causal, dtype, out)      BASELINE config 1
    (2, 4096, 4096, 10, 64, False, "f16", "f16"),  # (a) self-attention at level 1
    (2, 1024, 1024, 20, 64, False, "f16", "f16"),  # (b) self-attention at level 2
    (2, 1024, 77, 20, 64, False, "f16", "f16"),  # (c) cross-attention against the 77-token context
    (2, 1000, 1000, 10, 64, True, "f16", "f32"),  # causal, ragged
    (1, 333, 77, 8, 40, False, "bf16", "f32"),  # hd 40 (fused_attn_test.cpp:77), bf16
    (1, 64, 1, 4, 64, False, "f16", "f32"),  # a single key
    (3, 1, 300, 2, 32, False, "f32", "f32"),  # a single query, fp32 in
]


@pytest.mark.parametrize("B,Tq,Tk,heads,hd,causal,dt,out", CONFIG1)
def test_attention_shapes(orc, cuda_ok, B, Tq, Tk, heads, hd, causal, dt, out):
    C = heads * hd
    q = orc.normal_f32(1, 0, (B, Tq, C))
    k = orc.normal_f32(1, 1, (B, Tk, C))
    v = orc.normal_f32(1, 2, (B, Tk, C))
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[dt]
    qt, kt, vt = (dev(x).to(tdt) for x in (q, k, v))
    q, k, v = (t.float().cpu().numpy() for t in (qt, kt, vt))  # exactly what the GPU sees
    o = torch_ops.attention(qt, kt, vt, heads, causal=causal,
                            out_dtype=torch.float32 if out == "f32" else torch.float16)
    got = host(o).astype(np.float64)
    if causal:
        rows = np.arange(Tq)
    else:
        rows = np.sort(np.random.default_rng(0).choice(Tq, size=min(Tq, 128), replace=False))
    ref = orc.attn_f64(q[:, rows], k, v, heads, causal=False) if not causal else orc.attn_f64(q, k, v, heads, True)
    check_attn(orc, f"attn B{B} Tq{Tq} Tk{Tk} h{heads}x{hd} causal={causal} {dt}->{out}", got[:, rows], ref, dt)


def test_attention_empty_keys_gives_zero(orc, cuda_ok):
    q = torch.randn((1, 70, 128), device="cuda", dtype=torch.float16)
    k = torch.zeros((1, 0, 128), device="cuda", dtype=torch.float16)
    o = torch_ops.attention(q, k, k, 2, out_dtype=torch.float32)
    assert torch.count_nonzero(o) == 0


def test_attention_strided_head_major_layout(orc, cuda_ok):
    """[B, H, T, D] layout through the explicit-stride descriptor equals the token-major result."""
    B, H, T, D = 2, 4, 200, 64
    x = [torch.randn((B, T, H * D), device="cuda", dtype=torch.float16) for _ in range(3)]
    ref = torch_ops.attention(*x, H, out_dtype=torch.float32)
    hm = [t.view(B, T, H, D).permute(0, 2, 1, 3).contiguous() for t in x]
    o = torch.empty((B, H, T, D), device="cuda", dtype=torch.float32)
    d = sdvk_b200.AttnDesc()
    d.q, d.k, d.v, d.o = hm[0].data_ptr(), hm[1].data_ptr(), hm[2].data_ptr(), o.data_ptr()
    d.dtype, d.o_dtype = sdvk_b200.F16, sdvk_b200.F32
    d.batch, d.heads, d.Tq, d.Tk, d.hd = B, H, T, T, D
    d.ldq = d.ldk = d.ldv = d.ldo = D
    d.sq = d.sk = d.sv = d.so = H * T * D
    d.hq = d.hk = d.hv = d.ho = T * D
    d.scale = 0.125
    torch_ops.context().attention(d)
    torch.cuda.synchronize()
    assert torch.equal(o.permute(0, 2, 1, 3).reshape(B, T, H * D), ref)


def test_attention_unsupported_head_dim(orc, cuda_ok):
    ctx = torch_ops.context()
    q = torch.zeros((4, 1280), device="cuda")
    with pytest.raises(sdvk_b200.SdvkError) as e:
        ctx.fused_attention(q.data_ptr(), q.data_ptr(), q.data_ptr(), q.data_ptr(), 4, 4, 1280, 10)  # hd 128
    assert e.value.status == sdvk_b200.E_SHAPE


KERNEL_CASES = [
    # (B, Tq, Tk, heads, causal, dtype, out)   head dim 64: the tensor-core (tcgen05) kernel's domain
    (2, 4096, 4096, 10, False, "f16", "f16"),
    (1, 1000, 77, 20, False, "f16", "f32"),
    (1, 300, 300, 4, True, "f16", "f32"),
    (2, 257, 129, 3, False, "bf16", "f32"),
    (1, 640, 640, 2, True, "bf16", "f16"),
    (3, 1, 2, 1, False, "f16", "f32"),
    # the persistent tensor-core kernel walks several items per CTA: causal items of 1 to 8 key tiles,
    # and items of an odd key-tile count (the two softmax groups get unequal shares)
    (2, 1024, 1024, 40, True, "f16", "f16"),
    (2, 1024, 384, 100, False, "f16", "f32"),
]


@pytest.mark.parametrize("kernel", ["tc", "mma", "auto"])
@pytest.mark.parametrize("B,Tq,Tk,heads,causal,dt,out", KERNEL_CASES + [
    # at most 128 non-causal keys: the short-key tcgen05 kernel under "auto"; many items per CTA
    (4, 1100, 128, 40, False, "f16", "f16"),
    (2, 130, 1, 3, False, "bf16", "f32"),
    (1, 64, 16, 5, False, "f16", "f32"),
])
def test_attention_kernel_variants(orc, cuda_ok, monkeypatch, kernel, B, Tq, Tk, heads, causal, dt, out):
    """The attention kernels (SDVK_ATTN_KERNEL=tc: tcgen05/TMEM; =mma: warp-level; auto: the default
    choice, which sends at most 128 non-causal keys to the short-key tcgen05 kernel) against fp64."""
    if kernel == "auto":
        monkeypatch.delenv("SDVK_ATTN_KERNEL", raising=False)
    else:
        monkeypatch.setenv("SDVK_ATTN_KERNEL", kernel)
    C = heads * 64
    tdt = {"f16": torch.float16, "bf16": torch.bfloat16}[dt]
    qt, kt, vt = (dev(orc.normal_f32(5, i, (B, T, C))).to(tdt) for i, T in enumerate((Tq, Tk, Tk)))
    q, k, v = (t.float().cpu().numpy() for t in (qt, kt, vt))
    o = torch_ops.attention(qt, kt, vt, heads, causal=causal,
                            out_dtype=torch.float32 if out == "f32" else torch.float16)
    got = host(o).astype(np.float64)
    rows = np.arange(Tq) if (causal or Tq <= 256) else np.sort(
        np.random.default_rng(1).choice(Tq, size=256, replace=False))
    ref = orc.attn_f64(q, k, v, heads, True) if causal else orc.attn_f64(q[:, rows], k, v, heads, False)
    check_attn(orc, f"attn[{kernel}] B{B} Tq{Tq} Tk{Tk} h{heads} causal={causal} {dt}->{out}", got[:, rows],
               ref if not causal else ref[:, rows], dt)
