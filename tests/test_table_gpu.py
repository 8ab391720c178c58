"""The rest of the reference's kernel table through sdvk_dispatch (table.cu) against the oracle's
restatement of each shader (oracle/refkernels.cpp), with the walker's own push layouts and bindings
(src/Modules/GPU/vk_engine.cpp:51-125; push blocks sdvkgen.cpp:901-1206).

Layout and elementwise kernels (add2, ew2, copy_nd, bias_add, upsample2x, im2col, im2col_s2,
causal_mask) are exact copies or single IEEE operations: bit for bit.  The kernels with an
exponential (unary_fwd, softmax_fwd) use the device's expf: within 4e-7 relative.  The fp32 GEMMs
accumulate in the same k order with fused multiply-adds: within 1e-6 of max |ref|.  The in-place
forms the walker uses (add2 into an operand, copy_nd scaling in place, ew2's bias add into its own
input, softmax over its input) are covered too."""
import numpy as np
import pytest
import torch

import sdvk_b200
from oracle import pyoracle as po
from tests._gpu_util import dev, host, record

pytestmark = pytest.mark.gpu


def run_dev(name, arrays, push, gz=1, alias=None):
    """Dispatch `name` on device copies of `arrays` (alias: {i: j} binds buffer i to buffer j's
    memory); returns the host copies of every buffer after the call."""
    ctx = sdvk_b200.torch_ops.context()
    ts = [dev(a) for a in arrays]
    if alias:
        for i, j in alias.items():
            ts[i] = ts[j]
    torch.cuda.synchronize()
    bufs = [sdvk_b200.Buf(t.data_ptr(), 0, t.numel() * 4) for t in ts]
    ctx.dispatch(name, bufs, push, 1, 1, gz)
    ctx.synchronize()
    return [host(t) for t in ts]


def run_ref(name, arrays, push, gz=1, alias=None):
    hs = [np.array(a, np.float32, copy=True) for a in arrays]
    if alias:
        for i, j in alias.items():
            hs[i] = hs[j]
    po.table_kernel(name, hs, push, gz)
    return hs


def rnd(*shape, seed=0):
    return np.random.default_rng(seed).standard_normal(shape).astype(np.float32)


def both(name, arrays, push, out, gz=1, alias=None, exact=True, tol=0.0):
    got = run_dev(name, arrays, push, gz, alias)[out]
    ref = run_ref(name, arrays, push, gz, alias)[out]
    if exact:
        assert np.array_equal(got, ref), (name, np.abs(got - ref).max())
    else:
        st = po.err_stats(got, ref)
        record(f"table_{name}", st)
        assert st["rel_max"] <= tol, (name, st)


def test_add2_and_in_place(cuda_ok):
    n = 5003
    both("add2", [np.zeros(n, np.float32), rnd(n, seed=1), rnd(n, seed=2)], po.pack_push([n]), 0)
    # spatialTransformer's residual: add2 {t, t, a} (sdvkgen.cpp:1746)
    both("add2", [rnd(4096, seed=3), np.zeros(1, np.float32), rnd(4096, seed=4)], po.pack_push([4096]), 0,
         alias={1: 0})


def test_copy_nd_transpose_split_heads_and_scale(cuda_ok):
    outer, inner = 320, 257
    # transpose2(x, outer, inner) (sdvkgen.cpp:1072-1074): the tiled fast path
    push = po.pack_push([outer * inner, inner, outer, 1, 1, outer, 1, 0, 0, 1, inner, 0, 0, 0, 1.0], float_last=True)
    both("copy_nd", [np.zeros(outer * inner, np.float32), rnd(outer * inner, seed=5)], push, 0)
    # geglu's half split (:1714-1716)
    rows, F = 33, 96
    push = po.pack_push([rows * F, F, rows, 1, 1, 1, F, 0, 0, 1, 2 * F, 0, 0, 0, 1.0], float_last=True)
    both("copy_nd", [np.zeros(rows * F, np.float32), rnd(rows * 2 * F, seed=6)], push, 0)
    # headsView with a scale (:1212-1217): [T][C] -> [h][T][hd]
    T, heads, hd = 40, 5, 64
    C = heads * hd
    push = po.pack_push([heads * T * hd, hd, T, heads, 1, 1, hd, T * hd, 0, 1, C, hd, 0, 0, 0.125], float_last=True)
    both("copy_nd", [np.zeros(heads * T * hd, np.float32), rnd(T * C, seed=7)], push, 0)
    # scaleInPlace (:1066-1069) and the accumulate mode (headsMergeInto writes with mode 0; mode 1 here)
    n = 1000
    push = po.pack_push([n, n, 1, 1, 1, 1, 0, 0, 0, 1, 0, 0, 0, 0, 0.3], float_last=True)
    both("copy_nd", [rnd(n, seed=8), np.zeros(1, np.float32)], push, 0, alias={1: 0})
    push = po.pack_push([n, n, 1, 1, 1, 1, 0, 0, 0, 1, 0, 0, 0, 1, 2.0], float_last=True)
    both("copy_nd", [rnd(n, seed=9), rnd(n, seed=10)], push, 0)


def test_ew2_mul_and_bias_last(cuda_ok):
    n = 7777
    # mul2 (:1003-1019)
    both("ew2", [np.zeros(n, np.float32), rnd(n, seed=11), rnd(n, seed=12)],
         po.pack_push([n, n, 1, 1, 1, 1, 0, 0, 0, 1, 0, 0, 0, 1]), 0)
    # biasAddLast {y, y, b} (:1043-1059)
    rows, d = 77, 640
    both("ew2", [rnd(rows * d, seed=13), np.zeros(1, np.float32), rnd(d, seed=14)],
         po.pack_push([rows * d, d, rows, 1, 1, 1, d, 0, 0, 1, 0, 0, 0, 0]), 0, alias={1: 0})


@pytest.mark.parametrize("mode", [0, 1, 2, 3, 4])
def test_unary_modes(cuda_ok, mode):
    n = 4099
    x = rnd(n, seed=20 + mode) * 4
    both("unary_fwd", [x, np.zeros(n, np.float32)], po.pack_push([n, mode]), 1, exact=False, tol=1e-6)


def test_bias_add_upsample_causal(cuda_ok):
    C, P = 320, 1031
    both("bias_add", [rnd(C * P, seed=30), rnd(C, seed=31)], po.pack_push([C, P]), 0)
    C, H, W = 64, 9, 13
    both("upsample2x", [rnd(C * H * W, seed=32), np.zeros(C * 4 * H * W, np.float32)], po.pack_push([C, H, W]), 1)
    b, r, c = 3, 37, 41
    both("causal_mask", [rnd(b * r * c, seed=33)], po.pack_push([b, r, c]), 0)


def test_im2col_both_strides(cuda_ok):
    C, H, W = 19, 23, 17
    x = rnd(C * H * W, seed=40)
    for row0, rows in ((0, H), (5, 7)):
        both("im2col", [x, np.zeros(C * 9 * rows * W, np.float32)], po.pack_push([C, H, W, row0, rows]), 1)
    for off in (-1, 0):
        OH, OW = H // 2, W // 2
        push = po.pack_push([C, H, W, OH, OW, off & 0xFFFFFFFF])
        both("im2col_s2", [x, np.zeros(C * 9 * OH * OW, np.float32)], push, 1)


@pytest.mark.parametrize("nt", [True, False])
def test_gemm_fp32(cuda_ok, nt):
    M, N, K, batch = 100, 70, 36, 3
    name = "gemm_nt" if nt else "gemm_nn"
    A = rnd(batch * M * K, seed=50)
    B = rnd(batch * N * K, seed=51)
    push = po.pack_push([M, N, K, 0, M * K, N * K, M * N, batch, 0, 0, 0, 0])
    both(name, [A, B, np.zeros(batch * M * N, np.float32)], push, 2, gz=batch, exact=False, tol=1e-6)
    # conv_in's form: ldc = P over a row band, accumulate mode
    push = po.pack_push([M, N, K, 1, 0, 0, 0, 1, 0, 0, N + 5, 0])
    both(name, [A, B, rnd(M * (N + 5), seed=52)], push, 2, exact=False, tol=1e-6)


def test_softmax_rows_and_in_place(cuda_ok):
    rows, cols = 57, 1000
    x = rnd(rows * cols, seed=60) * 3
    both("softmax_fwd", [x, np.zeros(rows * cols, np.float32)], po.pack_push([rows, cols]), 1, exact=False, tol=1e-6)
    both("softmax_fwd", [x, np.zeros(1, np.float32)], po.pack_push([rows, cols]), 1, alias={1: 0}, exact=False,
         tol=1e-6)


def test_table_rejects_short_buffers(cuda_ok):
    ctx = sdvk_b200.torch_ops.context()
    a = torch.zeros(100, device="cuda")
    bufs = [sdvk_b200.Buf(a.data_ptr(), 0, 400)] * 3
    with pytest.raises(sdvk_b200.SdvkError) as e:
        ctx.dispatch("add2", bufs, po.pack_push([101]), 1)
    assert e.value.status == sdvk_b200.E_ARG
    with pytest.raises(sdvk_b200.SdvkError) as e:
        ctx.dispatch("no_such_kernel", bufs, po.pack_push([1]), 1)
    assert e.value.status == sdvk_b200.E_KERNEL
