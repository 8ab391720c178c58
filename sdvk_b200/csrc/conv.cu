// conv.cu -- the UNet's 3x3 convolutions with Q8_0 weights: im2col + the Q8_0 NN GEMM, the
// reference's structure (conv3RawInto and conv3s2, sdvkgen.cpp:1133-1175; im2col.comp and
// im2col_s2.comp; gemmNnQ8 with ldc = P; biasAddCh).
//
// x [batch][cin][H][W] (channel-major), weight [cout][cin*9] with k = c*9 + ky*3 + kx, output
// [batch][cout][OH][OW].  Stride 1 pads 1 on every side; stride 2 gives OH = H/2, OW = W/2 with either
// the symmetric pad-1 ring (off = -1, the UNet downsamplers) or padding on the right/bottom only
// (off = 0, the VAE encoder's Downsample2D).  The column matrix col[k][p] (p over a band of output rows)
// goes to a caller-provided workspace in the GEMM's activation type, in bands of output rows that fit
// it; the GEMM writes the band's output columns with the row stride OH*OW and adds the bias in its
// epilogue.  An implicit-GEMM form that never materialises col (TMA im2col loads) is the next step.
#include <algorithm>

#include "backend.hpp"
#include "ptx.cuh"

namespace sdvk {
namespace {

constexpr int kColThreads = 256;

// grid (ceil(np / (256 * 8)), K, images): thread = 8 consecutive output positions p of column-matrix row k,
// col[k][p] = x[c][oh*stride + ky + off][ow*stride + kx + off] (0 outside), stored with 16-byte
// vector stores (rows of col ld elements apart, ld % 8 == 0; positions in [np, round_up(np, 8)) are
// written with values the GEMM never reads).
template <class T>
__global__ void __launch_bounds__(kColThreads) im2col3x3_kernel(const T* __restrict__ x, T* __restrict__ col,
                                                                uint32_t H, uint32_t W, uint32_t OW, uint32_t row0,
                                                                uint32_t np, uint64_t ld, uint32_t stride, int off,
                                                                uint64_t xbs, uint64_t cbs) {
    grid_dependency_wait();
    grid_launch_dependents();
    x += blockIdx.z * xbs;  // image z: its input, and its column matrix cbs elements further on
    col += blockIdx.z * cbs;
    const uint32_t k = blockIdx.y;
    const uint32_t p0 = (blockIdx.x * kColThreads + threadIdx.x) * 8;
    if (p0 >= np) return;
    const uint32_t c = k / 9, r = k - c * 9, ky = r / 3, kx = r - ky * 3;
    uint32_t oh = row0 + p0 / OW, ow = p0 % OW;
    const T* xc = x + (uint64_t)c * H * W;
    T v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int ih = (int)(oh * stride + ky) + off, iw = (int)(ow * stride + kx) + off;
        v[j] = (ih >= 0 && ih < (int)H && iw >= 0 && iw < (int)W) ? xc[(uint64_t)ih * W + iw] : T(0.0f);
        if (++ow == OW) ow = 0, ++oh;
    }
    T* dst = col + (uint64_t)k * ld + p0;
    if constexpr (sizeof(T) == 2) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            w[j] = (uint32_t)__builtin_bit_cast(uint16_t, v[2 * j]) |
                   ((uint32_t)__builtin_bit_cast(uint16_t, v[2 * j + 1]) << 16);
        *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
}

// 8 consecutive values of T from a 16-byte aligned address, widened to float
template <class T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
    if constexpr (sizeof(T) == 4) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
        v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
    } else {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(p));
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            v[2 * j] = (float)__builtin_bit_cast(T, (uint16_t)(u[j] & 0xFFFFu));
            v[2 * j + 1] = (float)__builtin_bit_cast(T, (uint16_t)(u[j] >> 16));
        }
    }
}

// 8 floats stored as T (exact: every value came from a T) to a 16-byte aligned address
template <class T>
__device__ __forceinline__ void store8(T* p, const float (&v)[8]) {
    if constexpr (sizeof(T) == 4) {
        reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
            w[j] = (uint32_t)__builtin_bit_cast(uint16_t, T(v[2 * j])) |
                   ((uint32_t)__builtin_bit_cast(uint16_t, T(v[2 * j + 1])) << 16);
        *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// Row-segment im2col: grid (ceil(rows * OW/8 / 256), cin, images); a thread owns 8 consecutive output
// positions of one output row and one input channel c.  It reads the three input rows it needs once
// (the aligned 8*S values under the segment as 16-byte vectors, plus a one-value halo on either side)
// and writes all nine column-matrix rows k = c*9 + ky*3 + kx for its positions, 16 bytes each.
// Requires OW % 8 == 0, W % 8 == 0 and a 16-byte aligned x (every row and segment start aligned).
template <class T, int S, int OFF>
__global__ void __launch_bounds__(kColThreads) im2col3x3_rows_kernel(const T* __restrict__ x, T* __restrict__ col,
                                                                     uint32_t H, uint32_t W, uint32_t OW,
                                                                     uint32_t row0, uint32_t nrows, uint64_t ld,
                                                                     uint64_t xbs, uint64_t cbs) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint32_t segs = OW / 8, seg = blockIdx.x * kColThreads + threadIdx.x;
    if (seg >= nrows * segs) return;
    const uint32_t c = blockIdx.y, r = seg / segs, ow0 = (seg - r * segs) * 8, oh = row0 + r;
    const T* xc = x + blockIdx.z * xbs + (uint64_t)c * H * W;
    T* dst = col + blockIdx.z * cbs + (uint64_t)c * 9 * ld + (uint64_t)r * OW + ow0;
    const uint32_t a0 = ow0 * S;  // first input column under the segment (8-aligned)
    constexpr int NV = 8 * S + 2;  // v[i] holds input column a0 - 1 + i
#pragma unroll
    for (int ky = 0; ky < 3; ++ky) {
        const int ih = (int)(oh * S) + ky + OFF;
        float v[NV];
        if (ih >= 0 && ih < (int)H) {
            const T* row = xc + (uint64_t)ih * W;
            v[0] = a0 >= 1 ? (float)row[a0 - 1] : 0.0f;
#pragma unroll
            for (int h = 0; h < S; ++h) {
                float t[8];
                load8(row + a0 + 8 * h, t);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[1 + 8 * h + j] = t[j];
            }
            v[NV - 1] = a0 + 8 * S < W ? (float)row[a0 + 8 * S] : 0.0f;
        } else {
#pragma unroll
            for (int i = 0; i < NV; ++i) v[i] = 0.0f;
        }
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
            float o[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = v[j * S + kx + OFF + 1];
            store8(dst + (uint64_t)(ky * 3 + kx) * ld, o);
        }
    }
}

// im2col of output rows [row0, row0 + nrows) of `images` images into col (row pitch ld elements; image z
// at x + z*xbs, its columns at col + z*cbs): the row-segment kernel where the shape allows, else the
// per-element one.
template <class T>
int im2col_launch(const T* x, T* col, uint32_t cin, uint32_t H, uint32_t W, uint32_t OW, uint32_t row0,
                  uint32_t nrows, uint64_t ld, uint32_t stride, int off, uint32_t images, uint64_t xbs, uint64_t cbs,
                  const LaunchEnv& env) {
    const bool rows_ok = OW % 8 == 0 && W % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 &&
                         (xbs * sizeof(T)) % 16 == 0 && ld % 8 == 0 && (cbs * sizeof(T)) % 16 == 0;
    if (rows_ok) {
        const dim3 grid((nrows * (OW / 8) + kColThreads - 1) / kColThreads, cin, images);
        auto kern = stride == 1 ? im2col3x3_rows_kernel<T, 1, -1>
                                : off == 0 ? im2col3x3_rows_kernel<T, 2, 0> : im2col3x3_rows_kernel<T, 2, -1>;
        return launch_pdl(kern, grid, dim3(kColThreads), 0, env, "im2col3x3_rows_kernel launch", x, col, H, W, OW, row0,
                          nrows, ld, xbs, cbs);
    }
    const uint32_t np = nrows * OW;
    const dim3 grid((np + 8 * kColThreads - 1) / (8 * kColThreads), cin * 9, images);
    return launch_pdl(im2col3x3_kernel<T>, grid, dim3(kColThreads), 0, env, "im2col3x3_kernel launch", x, col, H, W,
                      OW, row0, np, ld, stride, off, xbs, cbs);
}

int im2col_any(const void* x, int x_dtype, void* col, uint32_t cin, uint32_t H, uint32_t W, uint32_t OW,
               uint32_t row0, uint32_t nrows, uint64_t ld, uint32_t stride, int off, uint32_t images, uint64_t xbs,
               uint64_t cbs, const LaunchEnv& env) {
    if (x_dtype == SDVK_F32)
        return im2col_launch(static_cast<const float*>(x), static_cast<float*>(col), cin, H, W, OW, row0, nrows, ld,
                             stride, off, images, xbs, cbs, env);
    if (x_dtype == SDVK_F16)
        return im2col_launch(static_cast<const __half*>(x), static_cast<__half*>(col), cin, H, W, OW, row0, nrows, ld,
                             stride, off, images, xbs, cbs, env);
    return im2col_launch(static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(col), cin, H, W, OW, row0,
                         nrows, ld, stride, off, images, xbs, cbs, env);
}

}  // namespace

uint64_t conv3x3_workspace(uint32_t cin, uint32_t H, uint32_t W, uint32_t stride, int dtype) {
    if (stride != 1 && stride != 2) return 0;
    const uint32_t OH = stride == 1 ? H : H / 2, OW = stride == 1 ? W : W / 2;
    return (uint64_t)cin * 9 * OH * OW * dtype_size(dtype);
}

int conv3x3_q8(const void* x, int x_dtype, const int8_t* q, const float* s, const float* bias, void* y, int y_dtype,
               uint32_t batch, uint32_t cin, uint32_t cout, uint32_t H, uint32_t W, uint32_t stride, int off,
               void* workspace, uint64_t ws_bytes, const LaunchEnv& env) {
    return conv3x3_q8_ex(x, x_dtype, q, s, bias, 0, false, y, y_dtype, batch, cin, cout, H, W, stride, off, workspace,
                         ws_bytes, env);
}

int conv3x3_q8_ex(const void* x, int x_dtype, const int8_t* q, const float* s, const float* bias, uint64_t bias_stride,
                  bool accumulate, void* y, int y_dtype, uint32_t batch, uint32_t cin, uint32_t cout, uint32_t H,
                  uint32_t W, uint32_t stride, int off, void* workspace, uint64_t ws_bytes, const LaunchEnv& env) {
    if (!x || !q || !s || !y) return fail(env, SDVK_E_ARG, "null pointer");
    if (accumulate && y_dtype != SDVK_F32) return fail(env, SDVK_E_ARG, "an accumulating conv needs an F32 output");
    if (x_dtype != SDVK_F16 && x_dtype != SDVK_BF16 && x_dtype != SDVK_F32)
        return fail(env, SDVK_E_ARG, "conv input must be F16, BF16 or F32");
    if (y_dtype != SDVK_F16 && y_dtype != SDVK_F32) return fail(env, SDVK_E_ARG, "conv output must be F16 or F32");
    if (stride != 1 && stride != 2) return fail(env, SDVK_E_SHAPE, "conv stride must be 1 or 2");
    if (stride == 1) off = -1;
    if (off != -1 && off != 0) return fail(env, SDVK_E_SHAPE, "conv padding offset must be -1 or 0");
    if (batch == 0 || cout == 0 || H == 0 || W == 0) return SDVK_OK;
    const uint32_t K = cin * 9;
    if (cin == 0 || K % 32) return fail(env, SDVK_E_SHAPE, "conv needs cin*9 % 32 == 0 (whole Q8_0 blocks)");
    const uint32_t OH = stride == 1 ? H : H / 2, OW = stride == 1 ? W : W / 2;
    if (OH == 0 || OW == 0) return SDVK_OK;
    const uint64_t P = (uint64_t)OH * OW, es = dtype_size(x_dtype);
    // Bands of output rows: a band's column matrix (pitch rows*OW elements, a multiple of 8 so that
    // the GEMM's TMA rows and every band's output columns start 16-byte aligned) must fit the
    // workspace.  The last band may be shorter; it keeps the pitch.
    const uint64_t row_bytes = (uint64_t)K * OW * es;
    uint32_t rows = (uint32_t)std::min<uint64_t>(OH, workspace ? ws_bytes / row_bytes : 0);
    while (rows > 0 && ((uint64_t)rows * OW) % 8 && rows < OH) --rows;
    if (rows < OH && ((uint64_t)rows * OW) % 8) rows = 0;
    if (rows == 0 || (reinterpret_cast<uintptr_t>(workspace) & 15u))
        return fail(env, SDVK_E_ARG, "conv workspace too small for one aligned band of output rows, or misaligned");
    const uint64_t pitch = (uint64_t)rows * OW;
    const uint64_t xs = (uint64_t)cin * H * W * es, ys = (uint64_t)cout * P * dtype_size(y_dtype);
    if (rows == OH && batch > 1 && ws_bytes / ((uint64_t)K * P * es) >= batch && P % 8 == 0) {
        // Every image's column matrix fits: one im2col launch over the images and one batched GEMM
        // (image z's columns at z*K*P, its output at z*cout*P, its bias at z*bias_stride).
        const uint64_t xbe = (uint64_t)cin * H * W, cbe = (uint64_t)K * P;
        int rc = im2col_any(x, x_dtype, workspace, cin, H, W, OW, 0u, OH, P, stride, off, batch, xbe, cbe, env);
        if (rc) return rc;
        GemmQ8Desc d{};
        d.x = workspace;
        d.x_dtype = x_dtype;
        d.ldx = P;
        d.sx = cbe;
        d.wq = q;
        d.ws = s;
        d.ldw = K;
        d.bias = bias;
        d.sbias = bias ? bias_stride : 0;
        d.c = y;
        d.c_dtype = y_dtype;
        d.ldc = P;
        d.sc = (uint64_t)cout * P;
        d.xrows = (uint32_t)P;
        d.wrows = cout;
        d.K = K;
        d.batch = batch;
        d.nn = true;
        d.accumulate = accumulate;
        return gemm_q8(d, env);
    }
    for (uint32_t bi = 0; bi < batch; ++bi) {
        const uint8_t* xb = static_cast<const uint8_t*>(x) + bi * xs;
        uint8_t* yb = static_cast<uint8_t*>(y) + bi * ys;
        for (uint32_t r0 = 0; r0 < OH; r0 += rows) {
            const uint32_t rr = std::min(rows, OH - r0), np = rr * OW;
            int rc = im2col_any(xb, x_dtype, workspace, cin, H, W, OW, r0, rr, pitch, stride, off, 1u, 0, 0, env);
            if (rc) return rc;
            GemmQ8Desc d{};
            d.x = workspace;
            d.x_dtype = x_dtype;
            d.ldx = pitch;
            d.wq = q;
            d.ws = s;
            d.ldw = K;
            d.bias = bias ? bias + (uint64_t)bi * bias_stride : nullptr;
            d.accumulate = accumulate;
            d.c = yb + (uint64_t)r0 * OW * dtype_size(y_dtype);
            d.c_dtype = y_dtype;
            d.ldc = P;
            d.xrows = np;
            d.wrows = cout;
            d.K = K;
            d.batch = 1;
            d.nn = true;
            if ((rc = gemm_q8(d, env))) return rc;
        }
    }
    return SDVK_OK;
}

}  // namespace sdvk
