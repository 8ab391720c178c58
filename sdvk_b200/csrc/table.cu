// table.cu -- the rest of the reference's kernel table (src/Modules/GPU/vk_engine.cpp:51-125) that its
// UNet walker, generation loop and attention fallback dispatch around the hot path: elementwise and
// layout kernels (add2, ew2, copy_nd, unary_fwd, bias_add, upsample2x), the convolution helpers
// (im2col, im2col_s2), the fp32 GEMMs (gemm_nt, gemm_nn) and the unfused-attention pieces
// (softmax_fwd, causal_mask).  Each keeps its shader's semantics, including the 32-bit index
// arithmetic and which operands may alias (the walker runs add2 / ew2 / copy_nd in place).
//
// All of them are HBM-bound glue except the fp32 GEMMs, which the walker uses only for weights it
// holds in fp32 (conv_in of a Q8_0 GGUF) and the fallback attention of head dims above 64.  Layout:
// grid-stride loops sized to the SM count, 16-byte vectors where the operands allow, and a 32 x 32
// shared-memory tile for copy_nd's 2-D transposes (transpose2, sdvkgen.cpp:1072-1074).
#include <cuda_runtime.h>

#include <cstdint>

#include "backend.hpp"
#include "ptx.cuh"

namespace sdvk {
namespace {

constexpr int kThreads = 256;

uint32_t grid_for(uint64_t n, int num_sms) {
    const uint64_t want = (n + kThreads - 1) / kThreads;
    const uint64_t cap = (uint64_t)(num_sms > 0 ? num_sms : 148) * 16;
    return (uint32_t)(want < 1 ? 1 : (want > cap ? cap : want));
}

__device__ __forceinline__ uint64_t gtid() { return blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; }
__device__ __forceinline__ uint64_t gstride() { return (uint64_t)gridDim.x * blockDim.x; }

// add2.comp: c = a + b (c may be a or b)
__global__ void add2_kernel(float* c, const float* a, const float* b, uint32_t n, bool vec4) {
    grid_dependency_wait();
    grid_launch_dependents();
    if (vec4) {
        const uint32_t n4 = n / 4;
        for (uint64_t i = gtid(); i < n4; i += gstride()) {
            const float4 x = reinterpret_cast<const float4*>(a)[i], y = reinterpret_cast<const float4*>(b)[i];
            reinterpret_cast<float4*>(c)[i] = make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w);
        }
        return;
    }
    for (uint64_t i = gtid(); i < n; i += gstride()) c[i] = a[i] + b[i];
}

struct NdIdx {
    uint32_t d0, d1, d2;
    __device__ __forceinline__ void split(uint32_t i, uint32_t& c0, uint32_t& c1, uint32_t& c2, uint32_t& c3) const {
        c0 = i % d0;
        uint32_t t = i / d0;
        c1 = t % d1;
        t /= d1;
        c2 = t % d2;
        c3 = t / d2;
    }
};

// copy_nd.comp: dst[sum c*os] (=|+=) scale * src[sum c*ss]
__global__ void copy_nd_kernel(float* d, const float* s, TablePnd p) {
    grid_dependency_wait();
    grid_launch_dependents();
    const NdIdx ix{p.d0, p.d1, p.d2};
    for (uint64_t g = gtid(); g < p.n; g += gstride()) {
        uint32_t c0, c1, c2, c3;
        ix.split((uint32_t)g, c0, c1, c2, c3);
        const uint32_t so = p.ss0 * c0 + p.ss1 * c1 + p.ss2 * c2 + p.ss3 * c3;
        const uint32_t dof = p.os0 * c0 + p.os1 * c1 + p.os2 * c2 + p.os3 * c3;
        const float v = p.scale * s[so];
        if (p.mode == 0u) d[dof] = v;
        else d[dof] += v;
    }
}

// copy_nd in its 2-D transpose form (d2 = d3 = 1, os1 = ss0 = 1): dst[c0 * os0 + c1] = scale *
// src[c0 + c1 * ss1] for c0 < d0, c1 < d1.  32 x 32 tiles through shared memory so both the reads
// (along c0) and the writes (along c1) are coalesced.  grid (ceil(d0/32), ceil(d1/32)), block (32, 8).
__global__ void __launch_bounds__(256) transpose_kernel(float* d, const float* s, uint32_t d0, uint32_t d1,
                                                        uint32_t os0, uint32_t ss1, float scale, uint32_t mode) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ float tile[32][33];
    const uint32_t c0b = blockIdx.x * 32, c1b = blockIdx.y * 32;
    for (uint32_t r = threadIdx.y; r < 32; r += 8) {
        const uint32_t c1 = c1b + r, c0 = c0b + threadIdx.x;
        if (c0 < d0 && c1 < d1) tile[r][threadIdx.x] = s[c0 + c1 * ss1];
    }
    __syncthreads();
    for (uint32_t r = threadIdx.y; r < 32; r += 8) {
        const uint32_t c0 = c0b + r, c1 = c1b + threadIdx.x;
        if (c0 < d0 && c1 < d1) {
            const float v = scale * tile[threadIdx.x][r];
            float* o = d + (uint64_t)c0 * os0 + c1;
            if (mode == 0u) *o = v;
            else *o += v;
        }
    }
}

// ew2.comp: c[i] = a[ai] + b[bi] (mode 0) or a[ai] * b[bi] (mode 1)
__global__ void ew2_kernel(float* c, const float* a, const float* b, TablePew2 p) {
    grid_dependency_wait();
    grid_launch_dependents();
    const NdIdx ix{p.d0, p.d1, p.d2};
    for (uint64_t g = gtid(); g < p.n; g += gstride()) {
        uint32_t c0, c1, c2, c3;
        ix.split((uint32_t)g, c0, c1, c2, c3);
        const uint32_t ai = p.as0 * c0 + p.as1 * c1 + p.as2 * c2 + p.as3 * c3;
        const uint32_t bi = p.bs0 * c0 + p.bs1 * c1 + p.bs2 * c2 + p.bs3 * c3;
        c[g] = (p.mode == 0u) ? (a[ai] + b[bi]) : (a[ai] * b[bi]);
    }
}

// unary_fwd.comp: 0 tanh-GELU, 1 sigmoid, 2 SiLU, 3 quick GELU, otherwise erf GELU (Abramowitz and
// Stegun 7.1.26, the shader's published polynomial)
__global__ void unary_kernel(const float* x, float* y, uint32_t n, uint32_t mode) {
    grid_dependency_wait();
    grid_launch_dependents();
    for (uint64_t i = gtid(); i < n; i += gstride()) {
        const float v = x[i];
        float r;
        if (mode == 0u) {
            const float t = 0.7978845608028654f * (v + 0.044715f * v * v * v);
            const float e = expf(-2.0f * fabsf(t));
            float th = (1.0f - e) / (1.0f + e);
            if (t < 0.0f) th = -th;
            r = 0.5f * v * (1.0f + th);
        } else if (mode == 1u) {
            r = 1.0f / (1.0f + expf(-v));
        } else if (mode == 2u) {
            r = v / (1.0f + expf(-v));
        } else if (mode == 3u) {
            r = v / (1.0f + expf(-1.702f * v));
        } else {
            const float xs = v * 0.70710678118654752440f;
            const float ax = fabsf(xs);
            const float t = 1.0f / (1.0f + 0.3275911f * ax);
            const float poly =
                (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
            const float e = 1.0f - poly * expf(-ax * ax);
            r = 0.5f * v * (1.0f + (xs >= 0.0f ? e : -e));
        }
        y[i] = r;
    }
}

// bias_add.comp: x[i] += b[i / P]
__global__ void bias_add_kernel(float* x, const float* __restrict__ b, uint32_t C, uint32_t P) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint64_t n = (uint64_t)C * P;
    for (uint64_t i = gtid(); i < n; i += gstride()) x[i] += b[(uint32_t)i / P];
}

// upsample2x.comp: nearest 2x of [C][H][W]
__global__ void upsample2x_kernel(const float* __restrict__ x, float* __restrict__ y, uint32_t C, uint32_t H,
                                  uint32_t W) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint32_t W2 = W * 2u, H2 = H * 2u;
    const uint64_t n = (uint64_t)C * W2 * H2;
    for (uint64_t g = gtid(); g < n; g += gstride()) {
        const uint32_t i = (uint32_t)g;
        const uint32_t c = i / (W2 * H2), r = i - c * (W2 * H2);
        const uint32_t oh = r / W2, ow = r - oh * W2;
        y[i] = x[(c * H + oh / 2u) * W + ow / 2u];
    }
}

// im2col.comp (stride 1, pad 1, output rows row0 .. row0 + rows - 1) and im2col_s2.comp (stride 2,
// pad offset off): col[k * P + p], k = c*9 + ky*3 + kx.  stride2 selects the second form; then
// (row0, rows) carry (OH, OW).
__global__ void im2col_kernel(const float* __restrict__ x, float* __restrict__ col, uint32_t C, uint32_t H, uint32_t W,
                              uint32_t a, uint32_t bdim, int off, bool stride2) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint32_t OW = stride2 ? bdim : W;
    const uint32_t P = stride2 ? a * bdim : bdim * W;
    const uint64_t n = (uint64_t)C * 9u * P;
    for (uint64_t g = gtid(); g < n; g += gstride()) {
        const uint32_t i = (uint32_t)g;
        const uint32_t k = i / P, p = i - k * P;
        const uint32_t c = k / 9u, r = k - c * 9u;
        const uint32_t ky = r / 3u, kx = r - ky * 3u;
        int ih, iw;
        if (stride2) {
            const uint32_t oh = p / OW, ow = p - oh * OW;
            ih = (int)(oh * 2u) + (int)ky + off;
            iw = (int)(ow * 2u) + (int)kx + off;
        } else {
            const uint32_t oh = a + p / W, ow = p % W;
            ih = (int)oh + (int)ky - 1;
            iw = (int)ow + (int)kx - 1;
        }
        float v = 0.0f;
        if (ih >= 0 && ih < (int)H && iw >= 0 && iw < (int)W) v = x[(c * H + (uint32_t)ih) * W + (uint32_t)iw];
        col[i] = v;
    }
}

// gemm_nt.comp / gemm_nn.comp in fp32: C (=|+=) A . B^T or A . B, batched over z.  64 x 64 output
// tiles, 256 threads with 4 x 4 outputs each, K in steps of 16 through shared memory; every output
// accumulates k in ascending order with fused multiply-adds.  NT reads B rows at stride K whatever
// ldb says (gemm_nt.comp:52).
template <bool NT>
__global__ void __launch_bounds__(256) gemm_fp32_kernel(const float* __restrict__ A, const float* __restrict__ B,
                                                        float* __restrict__ C, TablePg p) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ float As[16][64 + 4];
    __shared__ float Bs[16][64 + 4];
    const uint32_t M = p.M, N = p.N, K = p.K;
    const uint32_t lda = p.lda ? p.lda : K;
    const uint32_t ldb = NT ? K : (p.ldb ? p.ldb : N);
    const uint32_t ldc = p.ldc ? p.ldc : N;
    const uint32_t z = blockIdx.z;
    const float* Az = A + (uint64_t)z * p.sA;
    const float* Bz = B + (uint64_t)z * p.sB;
    float* Cz = C + (uint64_t)z * p.sC;
    const uint32_t m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    const uint32_t tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    float acc[4][4] = {};
    for (uint32_t k0 = 0; k0 < K; k0 += 16) {
        for (uint32_t e = threadIdx.x; e < 64 * 16; e += 256) {
            const uint32_t r = e / 16, kk = e % 16;  // A tile [64 rows][16 k], stored k-major
            const uint32_t gr = m0 + r, gk = k0 + kk;
            As[kk][r] = (gr < M && gk < K) ? Az[(uint64_t)gr * lda + gk] : 0.0f;
        }
        for (uint32_t e = threadIdx.x; e < 64 * 16; e += 256) {
            uint32_t nn, kk;
            float v = 0.0f;
            if (NT) {
                nn = e / 16;
                kk = e % 16;
                if (n0 + nn < N && k0 + kk < K) v = Bz[(uint64_t)(n0 + nn) * ldb + k0 + kk];
            } else {
                kk = e / 64;
                nn = e % 64;
                if (n0 + nn < N && k0 + kk < K) v = Bz[(uint64_t)(k0 + kk) * ldb + n0 + nn];
            }
            Bs[kk][nn] = v;
        }
        __syncthreads();
#pragma unroll
        for (uint32_t kk = 0; kk < 16; ++kk) {
            float av[4], bv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) av[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t gr = m0 + ty * 4 + i, gc = n0 + tx * 4 + j;
            if (gr < M && gc < N) {
                float* o = Cz + (uint64_t)gr * ldc + gc;
                *o = p.mode == 0u ? acc[i][j] : *o + acc[i][j];
            }
        }
}

// softmax_fwd.comp: one CTA per row; the row max, the sum of exp(x - max), y = exp(x - max) / sum.
// x and y may be the same row (attnCore runs it in place): every thread reads its elements before
// it writes them.
__global__ void __launch_bounds__(256) softmax_kernel(const float* x, float* y, uint32_t cols) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ float red[32];
    const float* xr = x + (uint64_t)blockIdx.x * cols;
    float* yr = y + (uint64_t)blockIdx.x * cols;
    float mx = -3.0e38f;
    for (uint32_t j = threadIdx.x; j < cols; j += blockDim.x) mx = fmaxf(mx, xr[j]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = mx;
    __syncthreads();
    mx = red[0];
    for (uint32_t w = 1; w < blockDim.x / 32; ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();
    float s = 0.0f;
    for (uint32_t j = threadIdx.x; j < cols; j += blockDim.x) s += expf(xr[j] - mx);
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = s;
    __syncthreads();
    s = 0.0f;
    for (uint32_t w = 0; w < blockDim.x / 32; ++w) s += red[w];
    const float ir = 1.0f / s;
    for (uint32_t j = threadIdx.x; j < cols; j += blockDim.x) yr[j] = expf(xr[j] - mx) * ir;
}

// causal_mask.comp: s[b][r][c] = -3e38 for c > r
__global__ void causal_mask_kernel(float* s, uint32_t batch, uint32_t rows, uint32_t cols) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint64_t n = (uint64_t)batch * rows * cols;
    for (uint64_t g = gtid(); g < n; g += gstride()) {
        const uint32_t i = (uint32_t)g;
        if (i % cols > (i / cols) % rows) s[i] = -3.0e38f;
    }
}

}  // namespace

int table_add2(float* c, const float* a, const float* b, uint32_t n, const LaunchEnv& env) {
    if (!n) return SDVK_OK;
    const bool vec4 = n % 4 == 0 && ((uintptr_t)a | (uintptr_t)b | (uintptr_t)c) % 16 == 0;
    return launch_pdl(add2_kernel, dim3(grid_for(vec4 ? n / 4 : n, env.num_sms)), dim3(kThreads), 0, env, "add2", c, a,
                      b, n, vec4);
}

int table_copy_nd(float* d, const float* s, const TablePnd& p, const LaunchEnv& env) {
    if (!p.n) return SDVK_OK;
    const bool transpose2d = p.d2 == 1 && p.d3 == 1 && p.os1 == 1 && p.ss0 == 1 && p.d0 > 1 && p.d1 > 1 &&
                             (uint64_t)p.d0 * p.d1 == p.n && d != s;
    if (transpose2d)
        return launch_pdl(transpose_kernel, dim3((p.d0 + 31) / 32, (p.d1 + 31) / 32), dim3(32, 8), 0, env, "copy_nd",
                          d, s, p.d0, p.d1, p.os0, p.ss1, p.scale, p.mode);
    return launch_pdl(copy_nd_kernel, dim3(grid_for(p.n, env.num_sms)), dim3(kThreads), 0, env, "copy_nd", d, s, p);
}

int table_ew2(float* c, const float* a, const float* b, const TablePew2& p, const LaunchEnv& env) {
    if (!p.n) return SDVK_OK;
    return launch_pdl(ew2_kernel, dim3(grid_for(p.n, env.num_sms)), dim3(kThreads), 0, env, "ew2", c, a, b, p);
}

int table_unary(const float* x, float* y, uint32_t n, uint32_t mode, const LaunchEnv& env) {
    if (!n) return SDVK_OK;
    return launch_pdl(unary_kernel, dim3(grid_for(n, env.num_sms)), dim3(kThreads), 0, env, "unary_fwd", x, y, n, mode);
}

int table_bias_add(float* x, const float* b, uint32_t C, uint32_t P, const LaunchEnv& env) {
    if (!C || !P) return SDVK_OK;
    return launch_pdl(bias_add_kernel, dim3(grid_for((uint64_t)C * P, env.num_sms)), dim3(kThreads), 0, env,
                      "bias_add", x, b, C, P);
}

int table_upsample2x(const float* x, float* y, uint32_t C, uint32_t H, uint32_t W, const LaunchEnv& env) {
    if (!C || !H || !W) return SDVK_OK;
    return launch_pdl(upsample2x_kernel, dim3(grid_for((uint64_t)C * H * W * 4, env.num_sms)), dim3(kThreads), 0, env,
                      "upsample2x", x, y, C, H, W);
}

int table_im2col(const float* x, float* col, uint32_t C, uint32_t H, uint32_t W, uint32_t a, uint32_t b, int off,
                 bool stride2, const LaunchEnv& env) {
    const uint64_t P = stride2 ? (uint64_t)a * b : (uint64_t)b * W;
    const uint64_t n = (uint64_t)C * 9 * P;
    if (!n) return SDVK_OK;
    return launch_pdl(im2col_kernel, dim3(grid_for(n, env.num_sms)), dim3(kThreads), 0, env,
                      stride2 ? "im2col_s2" : "im2col", x, col, C, H, W, a, b, off, stride2);
}

int table_gemm_fp32(bool nt, const float* A, const float* B, float* C, const TablePg& p, uint32_t batch,
                    const LaunchEnv& env) {
    if (!p.M || !p.N || !batch) return SDVK_OK;
    const dim3 grid((p.N + 63) / 64, (p.M + 63) / 64, batch);
    if (nt) return launch_pdl(gemm_fp32_kernel<true>, grid, dim3(256), 0, env, "gemm_nt", A, B, C, p);
    return launch_pdl(gemm_fp32_kernel<false>, grid, dim3(256), 0, env, "gemm_nn", A, B, C, p);
}

int table_softmax(const float* x, float* y, uint32_t rows, uint32_t cols, const LaunchEnv& env) {
    if (!rows || !cols) return SDVK_OK;
    return launch_pdl(softmax_kernel, dim3(rows), dim3(256), 0, env, "softmax_fwd", x, y, cols);
}

int table_causal_mask(float* s, uint32_t batch, uint32_t rows, uint32_t cols, const LaunchEnv& env) {
    const uint64_t n = (uint64_t)batch * rows * cols;
    if (!n) return SDVK_OK;
    return launch_pdl(causal_mask_kernel, dim3(grid_for(n, env.num_sms)), dim3(kThreads), 0, env, "causal_mask", s,
                      batch, rows, cols);
}

}  // namespace sdvk
