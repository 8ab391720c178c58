"""Pins of the CPU oracle against the reference's own tests, readers and golden vectors (CPU only).

The oracle (oracle/) is the checker every GPU parity test uses, so it is pinned first:
  * the reference's tests/fused_attn_test.cpp and tests/gemm_q8_bench.cpp, compiled from the
    reference sources with the oracle restatement as their device, must pass their own checks;
  * golden outputs of the reference's fp64 attention reference() must be reproduced;
  * the reference GGUF reader must decode the oracle's Q8_0 encoding bit for bit.
"""
import json
import os
import re
import subprocess

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _manifest():
    with open(os.path.join(GOLDEN, "manifest.json")) as f:
        return json.load(f)


def _ref_bin(orc, name):
    path = os.path.join(orc.REF_DIR, name)
    if not os.path.exists(path):
        pytest.skip(f"{path} not built (needs the reference sources: make -C oracle ref)")
    return path


def _attn_inputs(orc):
    """Regenerate the reference test's inputs: mt19937(20261101), U(-1,1), q, k, v per shape."""
    rng = orc.MT19937(20261101)
    out = []
    for e in _manifest()["attention"]:
        Tq, Tk, C = e["Tq"], e["Tk"], e["C"]
        q = rng.uniform_f32(Tq * C).reshape(Tq, C)
        k = rng.uniform_f32(Tk * C).reshape(Tk, C)
        v = rng.uniform_f32(Tk * C).reshape(Tk, C)
        ref = np.fromfile(os.path.join(GOLDEN, e["file"]), np.float32).reshape(Tq, C)
        out.append((e, q, k, v, ref))
    return out


def test_reference_fused_attn_harness_passes_on_oracle(orc):
    """tests/fused_attn_test.cpp (reference) judges the restatement with its own 2e-5 bar."""
    r = subprocess.run([_ref_bin(orc, "fused_attn_test")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL PASS (0 failures)" in r.stdout
    assert len(re.findall(r"^PASS ", r.stdout, re.M)) == 4


def test_reference_gemm_harness_on_oracle(orc):
    """tests/gemm_q8_bench.cpp (reference) correctness probe: 100x100x96, mt19937(7).

    The harness prints rel = max|got-ref|/max|ref| with no pass bar.  Its own CPU loop rounds the
    product before adding (no FMA); the restatement contracts like the shader, so the two differ
    by a few fp32 ulps.  Bar here: rel <= 1e-6."""
    r = subprocess.run([_ref_bin(orc, "gemm_q8_bench")], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    rels = [float(x) for x in re.findall(r"^check \S+\s+rel=(\S+)", r.stdout, re.M)]
    assert len(rels) == 5
    assert max(rels) <= 1e-6


def test_golden_attention_reference_outputs(orc):
    """The oracle's fp64 attention reproduces the reference's fp64 reference() outputs, and the
    fp32 restatement of fused_attn*.comp meets the reference test's bar (2e-5) against them."""
    for e, q, k, v, ref in _attn_inputs(orc):
        f64 = orc.attn_f64(q, k, v, e["heads"], causal=e["causal"]).astype(np.float32)
        assert np.array_equal(f64, ref) or np.max(np.abs(f64 - ref)) <= 2 * np.finfo(np.float32).eps * np.abs(ref).max()
        got = orc.fused_attention(q, k, v, e["Tq"], e["Tk"], e["C"], e["heads"], causal=e["causal"])
        st = orc.err_stats(got, ref)
        assert st["rel_max"] <= 2e-5, (e, st)


def test_golden_files_match_manifest():
    import hashlib

    for e in _manifest()["attention"]:
        data = open(os.path.join(GOLDEN, e["file"]), "rb").read()
        assert hashlib.sha256(data).hexdigest() == e["sha256"]


def test_gguf_q8_split_matches_reference_reader_golden(orc):
    """Gguf.cpp readQ8Into / readFloat outputs (recorded by make_golden.py) are reproduced."""
    m = _manifest()["gguf"]
    g = np.load(os.path.join(GOLDEN, "gguf_q8.npz"))
    q, s = orc.q8_0_split(g["blocks"])
    assert np.array_equal(q, g["q"]) and np.array_equal(s.view(np.uint32), g["scales"].view(np.uint32))
    deq = (q.astype(np.float32).reshape(-1, 32) * s[:, None]).ravel()  # d * (float)q, Gguf.cpp:520
    assert np.array_equal(deq.view(np.uint32), g["floats"].view(np.uint32))
    # all 65536 fp16 scale bit patterns decode exactly as the reference's fp16ToFp32
    allh = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    import hashlib

    f = orc.f16_to_f32(allh.view(np.float16))
    assert hashlib.sha256(f.tobytes()).hexdigest() == m["all_fp16_scales_sha256"]


def test_gguf_q8_live_reference_reader(orc, tmp_path):
    """Same pin live: a fresh seeded tensor through the compiled reference reader."""
    import ctypes

    path = os.path.join(orc.REF_DIR, "libref_gguf.so")
    if not os.path.exists(path):
        pytest.skip("reference GGUF reader not built")
    L = ctypes.CDLL(path)
    L.ref_gguf_read_q8.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_void_p]
    rows, cols = 40, 320
    q, d16, d32 = orc.q8_weights(123, 4, rows, cols)
    blocks = orc.q8_0_pack(q, d16)
    f = str(tmp_path / "t.gguf")
    orc.gguf_write_q8(f, "t", rows, cols, blocks)
    rq = np.empty(rows * cols, np.int8)
    rs = np.empty(rows * cols // 32, np.float32)
    assert L.ref_gguf_read_q8(f.encode(), b"t", rq.ctypes.data, rs.ctypes.data) == 0
    assert np.array_equal(rq, q.ravel()) and np.array_equal(rs.view(np.uint32), d32.view(np.uint32))


def test_fp16_conversion_matches_numpy(orc):
    allh = np.arange(65536, dtype=np.uint32).astype(np.uint16).view(np.float16)
    mine = orc.f16_to_f32(allh)
    ref = allh.astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(mine[~nan].view(np.uint32), ref[~nan].view(np.uint32))
    assert np.all(np.isnan(mine[nan]))
    x = np.concatenate([np.random.default_rng(0).standard_normal(100000).astype(np.float32) * 3000,
                        np.array([65504, 65519.99, 65520, 1e-8, 6e-8, 3e-8, 2.98e-8, -0.0, 5.96e-8, np.inf],
                                 np.float32)])
    assert np.array_equal(orc.f32_to_f16(x).view(np.uint16), x.astype(np.float16).view(np.uint16))


def test_q8_weight_generator(orc):
    q, d16, d32 = orc.q8_weights(0, 0, 64, 1280)
    assert q.min() >= -127 and q.max() <= 127 and abs(float(q.mean())) < 0.5
    assert np.all(d32 >= 0) and np.array_equal(d16.astype(np.float32), d32)
    # |N(0, 0.02)| / 127 has mean 0.02*sqrt(2/pi)/127
    assert abs(float(d32.mean()) / (0.02 * np.sqrt(2 / np.pi) / 127) - 1) < 0.05
    z = orc.normal_f32(0, 1, (200000,))
    assert abs(float(z.mean())) < 0.01 and abs(float(z.std()) - 1) < 0.01


@pytest.mark.parametrize("M,N,K", [(100, 100, 96), (77, 64, 2048), (130, 96, 32)])
def test_gemm_nt_restatement_vs_f64(orc, M, N, K):
    rng = np.random.default_rng(M * N + K)
    A = rng.standard_normal((M, K)).astype(np.float32)
    q, _, s = orc.q8_weights(5, M, N, K)
    bias = rng.standard_normal(N).astype(np.float32)
    got = orc.gemm_nt_q8_shader(A, q, s, bias)
    ref = orc.gemm_nt_q8_f64(A, q, s, bias)
    assert orc.err_stats(got, ref)["rel_max"] < 1e-5


def test_gemm_nt_restatement_modes_batch(orc):
    rng = np.random.default_rng(1)
    M, N, K, B = 33, 40, 64, 3
    A = rng.standard_normal((B, M, K)).astype(np.float32)
    q, _, s = orc.q8_weights(2, 0, N, K)
    C0 = rng.standard_normal((B, M, N)).astype(np.float32)
    got = orc.gemm_nt_q8_shader(A, q, s, None, C=C0.copy(), mode=1, batch=B, sA=M * K, sC=M * N, M=M)
    ref = C0 + orc.gemm_nt_q8_f64(A, q, s, None, batch=B, sA=M * K)
    assert orc.err_stats(got, ref)["rel_max"] < 1e-5


def test_gemm_nt_restatement_k_tail_quirk(orc):
    """gemm_nt_q8_v.comp stages A/B in groups of 4 along K and zero-fills a group unless
    gc + 3 < K (:69, :86): with K % 4 != 0 the last K % 4 columns never contribute."""
    rng = np.random.default_rng(3)
    M, N, K = 8, 8, 34  # scales indexed flat, (n*K + k) >> 5
    A = rng.standard_normal((M, K)).astype(np.float32)
    q = rng.integers(-127, 128, (N, K)).astype(np.int8)
    s = np.full((N * K + 31) // 32, 0.01, np.float32)
    got = orc.gemm_nt_q8_shader(A, q, s)
    w = q.astype(np.float64) * s[(np.arange(N)[:, None] * K + np.arange(K)[None, :]) >> 5]
    ref = A[:, :32].astype(np.float64) @ w[:, :32].T
    assert orc.err_stats(got, ref)["rel_max"] < 1e-5


@pytest.mark.parametrize("M,N,K", [(64, 100, 96), (1280, 64, 64), (96, 7, 32)])
def test_gemm_nn_restatement_vs_f64(orc, M, N, K):
    rng = np.random.default_rng(M + N + K)
    q, _, s = orc.q8_weights(9, N, M, K)
    B = rng.standard_normal((K, N)).astype(np.float32)
    got = orc.gemm_nn_q8_shader(q, s, B)
    ref = orc.gemm_nn_q8_f64(q, s, B)
    if N % 4:  # gemm_nn_q8_v.comp:207 zero-fills B groups with gc + 3 >= N
        ref[:, N & ~3:] = 0
    assert orc.err_stats(got, ref)["rel_max"] < 1e-5


def test_attention_restatements_vs_f64(orc):
    rng = np.random.default_rng(7)
    for Tq, Tk, C, heads, causal in [(100, 300, 128, 2, False), (70, 70, 128, 2, True), (40, 77, 256, 4, False)]:
        q, k, v = (rng.uniform(-1, 1, (t, C)).astype(np.float32) for t in (Tq, Tk, Tk))
        ref = orc.attn_f64(q, k, v, heads, causal)
        got_t = orc.attn_tiled_shader(q, k, v, Tq, Tk, C, heads, causal, 0.125)
        got_s = orc.attn_simple_shader(q, k, v, Tq, Tk, C, heads, causal, 0.125)
        assert orc.err_stats(got_t, ref)["rel_max"] < 2e-5
        assert orc.err_stats(got_s, ref)["rel_max"] < 2e-5


def test_layernorm_and_gelu_restatements(orc):
    import math

    rng = np.random.default_rng(11)
    x = (rng.standard_normal((17, 1280)) * 3 + 1).astype(np.float32)
    g = rng.standard_normal(1280).astype(np.float32)
    b = rng.standard_normal(1280).astype(np.float32)
    st = orc.err_stats(orc.layernorm_shader(x, g, b), orc.layernorm_f64(x, g, b))
    assert st["rel_max"] < 1e-5
    xs = np.linspace(-8, 8, 10001).astype(np.float32)
    ref = np.array([0.5 * t * (1 + math.erf(t / math.sqrt(2))) for t in xs.astype(np.float64)])
    assert np.max(np.abs(orc.gelu_erf_shader(xs) - ref)) < 2e-6 * 8  # A&S 7.1.26: |eps| <= 1.5e-7 in erf


def test_block_restatement_vs_f64(orc):
    """The reference's fp32 block arithmetic (kernel by kernel) against the fp64 block composition on a
    small BasicTransformerBlock: the two oracle paths agree to fp32 rounding."""
    rng_seed, C, Cc, F, heads, T, Tc = 31, 128, 64, 96, 2, 70, 9
    W = {}
    for i, (name, n, k, bias) in enumerate([("q", C, C, False), ("k", C, C, False), ("v", C, C, False),
                                             ("o", C, C, True), ("q2", C, C, False), ("k2", C, Cc, False),
                                             ("v2", C, Cc, False), ("o2", C, C, True), ("ff1", 2 * F, C, True),
                                             ("ff2", C, F, True)]):
        q, _, s = orc.q8_weights(rng_seed, i, n, k)
        W[name] = (q, s, orc.normal_f32(rng_seed, 50 + i, (n,)) * 0.05 if bias else None)
    for i in (1, 2, 3):
        W[f"ln{i}_w"] = orc.normal_f32(rng_seed, 60 + i, (C,)) * 0.1 + 1
        W[f"ln{i}_b"] = orc.normal_f32(rng_seed, 70 + i, (C,)) * 0.1
    x = orc.normal_f32(rng_seed, 80, (1, T, C))
    ctx = orc.normal_f32(rng_seed, 81, (1, Tc, Cc))
    ref = orc.block_f64(x, ctx, heads, W)
    got = orc.block_shader(x, ctx, heads, W)
    st = orc.err_stats(got - x, ref - x)
    assert st["rel_rms"] < 1e-5 and st["rel_max_rms"] < 1e-4, st


@pytest.mark.parametrize("B,C,P,G,act", [(1, 64, 300, 8, 0), (2, 12, 7, 3, 1), (1, 320, 1024, 32, 1)])
def test_groupnorm_restatement_against_f64(orc, B, C, P, G, act):
    """The fp32 restatement of groupnorm.comp (lane-strided partial sums, a tree over 256 lanes, two
    passes) stays within fp32 rounding of the float64 GroupNorm (+SiLU)."""
    x = orc.normal_f32(43, 0, (B, C, P)) * 2.0 + 0.5
    g = orc.normal_f32(43, 1, (C,)) * 0.2 + 1.0
    b = orc.normal_f32(43, 2, (C,)) * 0.1
    st = orc.err_stats(orc.groupnorm_shader(x, g, b, G, 1e-5, act), orc.groupnorm_f64(x, g, b, G, 1e-5, act))
    assert st["rel_max"] <= 2e-6, st


def test_im2col_restatement_matches_shader_loops(orc):
    """The oracle's im2col equals a line-by-line transcription of im2col.comp / im2col_s2.comp."""
    def loop(x, stride, off):
        C, H, W = x.shape
        OH, OW = (H, W) if stride == 1 else (H // 2, W // 2)
        if stride == 1:
            off = -1
        P = OH * OW
        col = np.zeros((C * 9, P), x.dtype)
        for i in range(C * 9 * P):
            k = i // P
            p = i - k * P
            c = k // 9
            r = k - c * 9
            ky, kx = r // 3, r - (r // 3) * 3
            oh, ow = p // OW, p % OW
            ih, iw = oh * stride + ky + off, ow * stride + kx + off
            if 0 <= ih < H and 0 <= iw < W:
                col[k, p] = x[c, ih, iw]
        return col

    x = orc.normal_f32(44, 0, (3, 7, 9))
    for stride, off in ((1, -1), (2, -1), (2, 0)):
        assert np.array_equal(loop(x, stride, off), orc.im2col3x3(x, stride, off))
