"""GGUF Q8_0 ingest on the device and GroupNorm (+SiLU) on the B200, against the oracle: the ingest
bit for bit against the reference reader's recorded output (Gguf.cpp readQ8Into) and its fp16ToFp32
over every binary16 pattern; GroupNorm against fp64 with the fp32 restatement of groupnorm.comp
reported beside."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

import sdvk_b200
from sdvk_b200 import torch_ops
from tests._gpu_util import dev, host, record

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _blocks_dev(blocks: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(blocks, np.uint8)).cuda()


def test_ingest_matches_reference_reader_golden(cuda_ok):
    """The recorded readQ8Into output of the reference's own loader, reproduced on the device."""
    g = np.load(os.path.join(GOLDEN, "gguf_q8.npz"))
    nb = g["blocks"].size // 34
    q, s = torch_ops.q8_0_ingest(_blocks_dev(g["blocks"]), 1, nb * 32)
    assert np.array_equal(host(q).ravel(), g["q"])
    assert np.array_equal(host(s).view(np.uint32), g["scales"].view(np.uint32))


def test_ingest_every_fp16_scale_pattern(cuda_ok):
    """One block per binary16 pattern (65536): the fp32 scales hash to the reference's fp16ToFp32 of all
    patterns (subnormals, signed zeros, infinities, NaN payloads)."""
    m = json.load(open(os.path.join(GOLDEN, "manifest.json")))["gguf"]
    n = 65536
    blocks = np.zeros((n, 34), np.uint8)
    blocks[:, 0:2] = np.arange(n, dtype=np.uint32).astype(np.uint16).view(np.uint8).reshape(n, 2)
    blocks[:, 2:] = (np.arange(n * 32, dtype=np.int64).reshape(n, 32) * 37 % 256).astype(np.uint8)
    q, s = torch_ops.q8_0_ingest(_blocks_dev(blocks), n, 32)
    assert hashlib.sha256(host(s).tobytes()).hexdigest() == m["all_fp16_scales_sha256"]
    assert np.array_equal(host(q).view(np.uint8), blocks[:, 2:])


@pytest.mark.parametrize("rows,cols,pad", [(3, 32, 0), (1000, 96, 0), (257, 1280, 32), (5, 64, 64)])
def test_ingest_matches_oracle_split(orc, cuda_ok, rows, cols, pad):
    """Random tensors (odd block counts, padded payload rows) against the oracle's split, bit for bit;
    padding stays untouched."""
    qv, d16, _ = orc.q8_weights(31, rows, rows, cols)
    blocks = orc.q8_0_pack(qv, d16)
    ldq = cols + pad
    q, s = torch_ops.q8_0_ingest(_blocks_dev(blocks), rows, cols, ldq)
    rq, rs = orc.q8_0_split(blocks)
    hq, hs = host(q), host(s).reshape(rows, ldq // 32)
    assert np.array_equal(hq[:, :cols], rq.reshape(rows, cols))
    assert np.array_equal(hs[:, :cols // 32].ravel().view(np.uint32), rs.view(np.uint32))
    if pad:
        assert not hq[:, cols:].any() and not hs[:, cols // 32:].any()


def test_ingested_weights_feed_the_gemm(orc, cuda_ok):
    """Raw blocks -> device split -> Q8_0 GEMM equals the GEMM on the host-split weights, bitwise."""
    M, N, K = 512, 384, 640
    qv, d16, d32 = orc.q8_weights(7, 2, N, K)
    q, s = torch_ops.q8_0_ingest(_blocks_dev(orc.q8_0_pack(qv, d16)), N, K)
    x = dev(orc.normal_f16(7, 3, (M, K)))
    a = torch_ops.gemm_q8_nt(x, q, s)
    b = torch_ops.gemm_q8_nt(x, dev(qv), dev(d32))
    assert torch.equal(a, b)


def test_ingest_errors(cuda_ok):
    ctx = torch_ops.context()
    buf = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    q = torch.zeros(1024, dtype=torch.int8, device="cuda")
    s = torch.zeros(64, dtype=torch.float32, device="cuda")
    with pytest.raises(sdvk_b200.SdvkError) as e:
        ctx.q8_0_ingest(buf.data_ptr(), 2, 48, q.data_ptr(), 48, s.data_ptr())  # cols % 32
    assert e.value.status == sdvk_b200.E_SHAPE
    with pytest.raises(sdvk_b200.SdvkError) as e:
        ctx.q8_0_ingest(buf.data_ptr() + 1, 1, 32, q.data_ptr(), 32, s.data_ptr())  # odd block address
    assert e.value.status == sdvk_b200.E_SHAPE


GN_CASES = [
    # (B, C, H*W, G, silu)
    (2, 320, 128 * 128, 32, True),   # SDXL level 1 at a 1024^2 latent
    (2, 1280, 32 * 32, 32, False),   # level 3
    (1, 640, 64 * 64, 32, True),
    (2, 64, 300, 8, False),          # ragged
    (3, 12, 7, 3, True),
]


@pytest.mark.parametrize("B,C,P,G,silu", GN_CASES)
def test_groupnorm(orc, cuda_ok, B, C, P, G, silu):
    x = orc.normal_f32(41, 0, (B, C, P)) * 1.7 + 0.4
    g = orc.normal_f32(41, 1, (C,)) * 0.2 + 1.0
    b = orc.normal_f32(41, 2, (C,)) * 0.1
    y = torch_ops.groupnorm(dev(x), dev(g), dev(b), G, 1e-5, silu)
    ref = orc.groupnorm_f64(x, g, b, G, 1e-5, int(silu))
    st = orc.err_stats(host(y), ref)
    st_ref = orc.err_stats(orc.groupnorm_shader(x, g, b, G, 1e-5, int(silu)), ref)
    record(f"groupnorm B{B} C{C} P{P} G{G} silu={silu}", st, st_ref)
    assert st["finite"] and st["rel_max"] <= 2e-5, (st, st_ref)


def test_groupnorm_in_place_and_dispatch(orc, cuda_ok):
    """y may alias x; Engine::dispatch("groupnorm", {x, gamma, beta, y}, {C, P, G, eps, act}) runs the
    same kernels at batch 1 (the reference's form)."""
    C, P, G = 320, 4096, 32
    x = orc.normal_f32(42, 0, (1, C, P))
    g = orc.normal_f32(42, 1, (C,)) * 0.2 + 1.0
    b = orc.normal_f32(42, 2, (C,)) * 0.1
    xd = dev(x)
    want = host(torch_ops.groupnorm(xd, dev(g), dev(b), G, 1e-5, True))
    torch_ops.groupnorm(xd, dev(g), dev(b), G, 1e-5, True, out=xd)
    assert np.array_equal(host(xd), want)
    xd2, gd, bd = dev(x), dev(g), dev(b)
    y = torch.full_like(xd2, float("nan"))
    bufs = [sdvk_b200.Buf(t.data_ptr(), 0, t.numel() * 4) for t in (xd2, gd, bd, y)]
    torch_ops.context().dispatch("groupnorm", bufs, sdvk_b200.pack_gn(C, P, G, 1e-5, 1), G)
    assert np.array_equal(host(y), want)
