// ingest.cu -- the model-side kernels next to the transformer block: GGUF Q8_0 block ingest on the
// device and GroupNorm (+ SiLU).
//
// Q8_0 ingest (Gguf.cpp:559-583, GgufFile::readQ8Into): a GGUF Q8_0 tensor is a sequence of 34-byte
// blocks, a little-endian IEEE binary16 scale d followed by 32 int8 values.  The loader splits it
// into the int8 payload and fp32 scales that the GEMMs take; here the raw blocks are uploaded once
// and split on the device.  fp16 -> fp32 is exact (Gguf.cpp:11-35: subnormals normalised, inf and
// NaN keep their payload bits), so the split is bit-identical to the host loader's.
//
// GroupNorm (groupnorm.comp, called by gnInto, sdvkgen.cpp:1105-1113): x [B][C][P] (channel-major,
// P = H*W), G groups of C/G channels; per (batch, group) mean and variance over C/G*P values,
// y = (x - mean) / sqrt(var + eps) * gamma[c] + beta[c], optionally SiLU v / (1 + e^-v).  A group of a
// 128x128 latent holds up to 655 k values, so the statistics are split over CTAs: each CTA reduces a
// chunk to (count, mean, M2) with a two-pass sum over its chunk (the reference's two-pass form), and
// each apply CTA (one channel row) merges its group's chunks with Chan's pairwise update before
// normalising.  Both are HBM-bound: x is read twice (the second stats pass hits L2) and y written
// once.
#include <algorithm>
#include <cmath>

#include "backend.hpp"
#include "ptx.cuh"

namespace sdvk {
namespace {

// IEEE binary16 bits -> binary32, exact (the same mapping as the reference's fp16ToFp32).
__device__ __forceinline__ float half_bits_to_f32(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
    uint32_t f;
    if (exp == 0) {
        if (man == 0) {
            f = sign;
        } else {  // subnormal: shift the leading 1 into the implicit bit
            const int lz = __clz(man) - 21;  // leading zeros within the 10-bit field, plus 1
            f = sign | ((uint32_t)(113 - lz) << 23) | (((man << lz) & 0x3FFu) << 13);
        }
    } else if (exp == 31) {
        f = sign | 0x7F800000u | (man << 13);
    } else {
        f = sign | ((exp + 112u) << 23) | (man << 13);
    }
    return __uint_as_float(f);
}

constexpr int kIngestBlocks = 256;  // Q8_0 blocks per CTA (one per thread)

// blocks -> q[row * ldq + k], scales[row * (ldq / 32) + k / 32].  The CTA's 256 blocks (8704 bytes)
// are staged through shared memory with coalesced 2-byte loads; each thread then splits one block.
__global__ void __launch_bounds__(kIngestBlocks) q8_0_split_kernel(const uint16_t* __restrict__ src, uint64_t nblocks,
                                                                   uint64_t blocks_per_row, int8_t* __restrict__ q,
                                                                   uint64_t ldq, float* __restrict__ scales,
                                                                   bool vec_store) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ uint16_t stage[kIngestBlocks * 17];
    const uint64_t b0 = (uint64_t)blockIdx.x * kIngestBlocks;
    const uint64_t nb = min((uint64_t)kIngestBlocks, nblocks - b0);
    const uint16_t* base = src + b0 * 17;
    for (uint32_t i = threadIdx.x; i < nb * 17; i += kIngestBlocks) stage[i] = base[i];
    __syncthreads();
    if (threadIdx.x >= nb) return;
    const uint64_t b = b0 + threadIdx.x;
    const uint64_t row = b / blocks_per_row, kb = b % blocks_per_row;
    const uint16_t* blk = stage + threadIdx.x * 17;
    scales[row * (ldq / 32) + kb] = half_bits_to_f32(blk[0]);
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = (uint32_t)blk[1 + 2 * i] | ((uint32_t)blk[2 + 2 * i] << 16);
    int8_t* dst = q + row * ldq + kb * 32;
    if (vec_store) {
        reinterpret_cast<uint4*>(dst)[0] = make_uint4(w[0], w[1], w[2], w[3]);
        reinterpret_cast<uint4*>(dst)[1] = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) dst[i] = (int8_t)((w[i >> 2] >> (8 * (i & 3))) & 0xFF);
    }
}

// ---------------------------------------------------------------------------------- GroupNorm
constexpr int kGnThreads = 256;
// Positions per CTA of the channels-last apply: 128 (two 64-position sub-tiles).  Each CTA keeps one
// sub-tile of loads in flight, so the bytes in flight per SM grow with the CTAs per SM (UNet pass at
// batch 1: 14.46 ms with 256 positions per CTA, 14.37 ms with 128; batch 2 unchanged).
#ifndef SDVK_GN_CL_POS
#define SDVK_GN_CL_POS 128
#endif
constexpr uint32_t kGnClPos = SDVK_GN_CL_POS;
constexpr uint32_t kGnChunk = 16384;  // values per statistics CTA

struct GnStat {
    float n, mean, m2;
};

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();  // red is free (a previous call's readers are done)
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kGnThreads / 32; ++i) s += red[i];
    return s;
}

// grid (chunks, G, B): (count, mean, M2) of chunk c of group g of image b, two passes over the chunk
// (the second from L2).  vec: 16-byte loads (x 16-byte aligned and P % 4 == 0, so every group,
// chunk and channel row starts on a 16-byte boundary).
__global__ void __launch_bounds__(kGnThreads) gn_stats_kernel(const float* __restrict__ x, uint32_t C, uint32_t P,
                                                              uint32_t G, bool vec, GnStat* __restrict__ stats) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ float red[kGnThreads / 32];
    const uint32_t g = blockIdx.y, b = blockIdx.z, chunks = gridDim.x;
    const uint64_t cnt = (uint64_t)(C / G) * P;
    const float* xg = x + (uint64_t)b * C * P + (uint64_t)g * cnt;
    const uint64_t lo = (uint64_t)blockIdx.x * kGnChunk, hi = min(cnt, lo + kGnChunk);
    float s = 0.0f;
    if (vec) {
#pragma unroll 4
        for (uint64_t i = lo + 4 * threadIdx.x; i < hi; i += 4 * kGnThreads) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(xg + i));
            s += (v.x + v.y) + (v.z + v.w);
        }
    } else {
        for (uint64_t i = lo + threadIdx.x; i < hi; i += kGnThreads) s += xg[i];
    }
    const float n = (float)(hi - lo);
    const float mean = block_sum(s, red) / n;
    float ss = 0.0f;
    if (vec) {
#pragma unroll 4
        for (uint64_t i = lo + 4 * threadIdx.x; i < hi; i += 4 * kGnThreads) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(xg + i));
            const float d0 = v.x - mean, d1 = v.y - mean, d2 = v.z - mean, d3 = v.w - mean;
            ss = fmaf(d0, d0, fmaf(d1, d1, fmaf(d2, d2, fmaf(d3, d3, ss))));
        }
    } else {
        for (uint64_t i = lo + threadIdx.x; i < hi; i += kGnThreads) {
            const float d = xg[i] - mean;
            ss = fmaf(d, d, ss);
        }
    }
    const float m2 = block_sum(ss, red);
    if (threadIdx.x == 0) stats[((uint64_t)b * G + g) * chunks + blockIdx.x] = GnStat{n, mean, m2};
}

// One warp: (mean, 1/sqrt(var + eps)) of a group from its chunk statistics.  Lane l merges chunks l,
// l+32, ... in order (Chan et al.'s pairwise update of count, mean and M2), then a fixed butterfly over
// the lanes in which both partners merge the pair in the same order (lower lane first), so every lane,
// and every CTA that merges the same group, gets the same result.
__device__ __forceinline__ float2 gn_group_norm(const GnStat* __restrict__ st, uint32_t chunks, float eps) {
    const uint32_t lane = threadIdx.x & 31;
    float n = 0.0f, m = 0.0f, m2 = 0.0f;
    auto merge = [](float& n, float& m, float& m2, float on, float om, float om2) {
        if (on == 0.0f) return;
        const float nn = n + on, d = om - m;
        m += d * (on / nn);
        m2 += om2 + d * d * (n * on / nn);
        n = nn;
    };
    for (uint32_t k = lane; k < chunks; k += 32) merge(n, m, m2, st[k].n, st[k].mean, st[k].m2);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float on = __shfl_xor_sync(0xffffffffu, n, o), om = __shfl_xor_sync(0xffffffffu, m, o),
                    om2 = __shfl_xor_sync(0xffffffffu, m2, o);
        if ((lane & o) == 0) {
            merge(n, m, m2, on, om, om2);
        } else {
            float pn = on, pm = om, pm2 = om2;
            merge(pn, pm, pm2, n, m, m2);
            n = pn, m = pm, m2 = pm2;
        }
    }
    return make_float2(m, 1.0f / sqrtf(m2 / n + eps));
}

// GroupNorm's output value (x - mean) * sc + sh, then SiLU v / (1 + e^-v) with the fast exponential and a
// correctly rounded reciprocal (a few ulp, against a full division and expf that made the apply pass
// issue-bound rather than HBM-bound).
__device__ __forceinline__ float gn_out(float v, float mean, float sc, float sh, uint32_t act) {
    v = (v - mean) * sc + sh;
    return act ? v * __frcp_rn(1.0f + __expf(-v)) : v;
}

// grid (C, B): one channel row of one image per CTA.  Warp 0 merges the channel's group statistics
// (Chan et al.'s pairwise update of count, mean and M2, in a fixed order) into (mean,
// 1/sqrt(var + eps)), then the CTA writes y = (x - mean) * rstd * gamma[c] + beta[c] (+ SiLU
// v / (1 + e^-v)).
template <class TY>
__global__ void __launch_bounds__(kGnThreads) gn_apply_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                              const float* __restrict__ beta, TY* __restrict__ y,
                                                              uint32_t C, uint32_t P, uint32_t G, float eps,
                                                              uint32_t act, const GnStat* __restrict__ stats,
                                                              uint32_t chunks, bool vec) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ float2 norm;
    const uint32_t c = blockIdx.x, b = blockIdx.y, g = c / (C / G);
    if (threadIdx.x < 32) {
        const float2 r = gn_group_norm(stats + ((uint64_t)b * G + g) * chunks, chunks, eps);
        if (threadIdx.x == 0) norm = r;
    }
    __syncthreads();
    const float mean = norm.x, sc = norm.y * gamma[c], sh = beta[c];
    const uint64_t off = ((uint64_t)b * C + c) * P;
    const float* xr = x + off;
    TY* yr = y + off;
    auto f = [&](float v) { return gn_out(v, mean, sc, sh, act); };
    if (vec) {
#pragma unroll 4
        for (uint32_t i = 4 * threadIdx.x; i < P; i += 4 * kGnThreads) {
            const float4 v = __ldcs(reinterpret_cast<const float4*>(xr + i));  // last use of x
            if constexpr (sizeof(TY) == 4) {
                *reinterpret_cast<float4*>(yr + i) = make_float4(f(v.x), f(v.y), f(v.z), f(v.w));
            } else {
                const __half2 lo = __floats2half2_rn(f(v.x), f(v.y)), hi = __floats2half2_rn(f(v.z), f(v.w));
                *reinterpret_cast<uint2*>(yr + i) = make_uint2(*reinterpret_cast<const uint32_t*>(&lo),
                                                               *reinterpret_cast<const uint32_t*>(&hi));
            }
        }
    } else {
        for (uint32_t i = threadIdx.x; i < P; i += kGnThreads) yr[i] = TY(f(xr[i]));
    }
}

// The same values written channels-last, y[b][p][c] fp16 (the implicit convolution's input and the
// spatial transformer's token layout).  grid (ceil(P / kGnClPos), C / CT, B), 256 threads: CT channels
// x kGnClPos positions per CTA in sub-tiles of 64 positions through shared memory.  The warps first merge the
// statistics of the tile's groups (gn_group_norm, so the values equal gn_apply_kernel's bit for bit);
// x is read as float4 rows along P (vec: P % 4 == 0 and x 16-byte aligned), y written as 16-byte rows
// of 8 channels (CT * 2 contiguous bytes per position).  C % CT == 0, y 16-byte aligned.
template <int CT>
__global__ void __launch_bounds__(kGnThreads) gn_apply_cl_kernel(const float* __restrict__ x,
                                                                 const float* __restrict__ gamma,
                                                                 const float* __restrict__ beta, __half* __restrict__ y,
                                                                 uint32_t C, uint32_t P, uint32_t G, float eps,
                                                                 uint32_t act, const GnStat* __restrict__ stats,
                                                                 uint32_t chunks, bool vec) {
    __shared__ float2 gnorm[CT];
    __shared__ float cm[CT], csc[CT], csh[CT];
    __shared__ float tile[CT][65];
    const uint32_t t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const uint32_t b = blockIdx.z, c0 = blockIdx.y * CT, p0 = blockIdx.x * kGnClPos, cpg = C / G;
    const uint32_t p_end = min(P, p0 + kGnClPos);
    const float* xb = x + ((uint64_t)b * C + c0) * P;
    __half* yb = y + (uint64_t)b * P * C + c0;
    // x[c][ps + q .. q+3] of this thread's CT/16 rows: the first sub-tile's loads are in flight while the
    // warps merge the statistics, each next sub-tile's while the current one is stored
    float v[CT / 16][4];
    auto load = [&](uint32_t ps) {
#pragma unroll
        for (uint32_t i = 0; i < CT / 16; ++i) {
            const uint32_t r = t / 16 + 16 * i, pp = ps + (t % 16) * 4;
            const float* src = xb + (uint64_t)r * P + pp;
            if (vec && pp + 3 < P) {
                const float4 f = __ldcs(reinterpret_cast<const float4*>(src));
                v[i][0] = f.x, v[i][1] = f.y, v[i][2] = f.z, v[i][3] = f.w;
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) v[i][j] = pp + j < P ? __ldcs(src + j) : 0.0f;
            }
        }
    };
    // x is complete before this kernel's statistics kernel started (both come from one groupnorm
    // call, statistics first), so the first loads go out before waiting for the statistics
    load(p0);
    grid_dependency_wait();
    grid_launch_dependents();
    const uint32_t g_lo = c0 / cpg, g_hi = (c0 + CT - 1) / cpg;
    for (uint32_t g = g_lo + warp; g <= g_hi; g += kGnThreads / 32) {
        const float2 r = gn_group_norm(stats + ((uint64_t)b * G + g) * chunks, chunks, eps);
        if (lane == 0) gnorm[g - g_lo] = r;
    }
    __syncthreads();
    if (t < CT) {
        const uint32_t c = c0 + t;
        const float2 r = gnorm[c / cpg - g_lo];
        cm[t] = r.x, csc[t] = r.y * gamma[c], csh[t] = beta[c];
    }
    __syncthreads();
    constexpr uint32_t kChunks = CT / 8;  // 16-byte rows of 8 channels per position
#pragma unroll 1
    for (uint32_t ps = p0; ps < p_end; ps += 64) {
        // normalised x[c][ps .. ps+63] -> tile[c][0..63]
#pragma unroll
        for (uint32_t i = 0; i < CT / 16; ++i) {
            const uint32_t r = t / 16 + 16 * i, q = (t % 16) * 4;
#pragma unroll
            for (int j = 0; j < 4; ++j) tile[r][q + j] = gn_out(v[i][j], cm[r], csc[r], csh[r], act);
        }
        if (ps + 64 < p_end) load(ps + 64);
        __syncthreads();
        // tile[c][p] -> y[ps + p][c0 + 8k .. 8k+7] as 16-byte stores
#pragma unroll
        for (uint32_t i = 0; i < CT / 32; ++i) {
            const uint32_t k = t % kChunks, p = t / kChunks + (kGnThreads / kChunks) * i, pp = ps + p;
            if (pp < P) {
                uint32_t w[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const __half2 h = __floats2half2_rn(tile[8 * k + 2 * j][p], tile[8 * k + 2 * j + 1][p]);
                    w[j] = *reinterpret_cast<const uint32_t*>(&h);
                }
                *reinterpret_cast<uint4*>(yb + (uint64_t)pp * C + 8 * k) = make_uint4(w[0], w[1], w[2], w[3]);
            }
        }
        __syncthreads();
    }
}

}  // namespace

int q8_0_ingest(const void* blocks, uint64_t rows, uint64_t cols, int8_t* q, uint64_t ldq, float* scales,
                const LaunchEnv& env) {
    if (!blocks || !q || !scales) return fail(env, SDVK_E_ARG, "null pointer");
    if (rows == 0 || cols == 0) return SDVK_OK;
    if (cols % 32 || ldq < cols || ldq % 32 || (reinterpret_cast<uintptr_t>(blocks) & 1u) ||
        (reinterpret_cast<uintptr_t>(scales) & 3u))
        return fail(env, SDVK_E_SHAPE,
                    "Q8_0 ingest needs cols % 32 == 0, ldq >= cols, ldq % 32 == 0, 2-byte aligned blocks and "
                    "4-byte aligned scales");
    const uint64_t bpr = cols / 32, nblocks = rows * bpr;
    const bool vec = (reinterpret_cast<uintptr_t>(q) & 15u) == 0 && ldq % 16 == 0;
    const uint64_t grid = (nblocks + kIngestBlocks - 1) / kIngestBlocks;
    if (grid > 0x7FFFFFFFull) return fail(env, SDVK_E_SHAPE, "Q8_0 tensor too large");
    return launch_pdl(q8_0_split_kernel, dim3((uint32_t)grid), dim3(kIngestBlocks), 0, env, "q8_0_split_kernel launch",
                      static_cast<const uint16_t*>(blocks), nblocks, bpr, q, ldq, scales, vec);
}

uint64_t groupnorm_workspace(uint32_t batch, uint32_t C, uint32_t P, uint32_t G) {
    if (G == 0 || C % G) return 0;
    const uint64_t cnt = (uint64_t)(C / G) * P;
    const uint64_t chunks = (cnt + kGnChunk - 1) / kGnChunk;
    return (uint64_t)batch * G * chunks * sizeof(GnStat);
}

int groupnorm(const float* x, const float* gamma, const float* beta, float* y, uint32_t batch, uint32_t C, uint32_t P,
              uint32_t G, float eps, uint32_t act, void* workspace, uint64_t ws_bytes, const LaunchEnv& env) {
    return groupnorm_ex(x, gamma, beta, y, SDVK_F32, batch, C, P, G, eps, act, workspace, ws_bytes, env);
}

int groupnorm_ex(const float* x, const float* gamma, const float* beta, void* y, int y_dtype, uint32_t batch,
                 uint32_t C, uint32_t P, uint32_t G, float eps, uint32_t act, void* workspace, uint64_t ws_bytes,
                 const LaunchEnv& env, bool channels_last) {
    if (!x || !gamma || !beta || !y) return fail(env, SDVK_E_ARG, "null pointer");
    if (y_dtype != SDVK_F32 && y_dtype != SDVK_F16) return fail(env, SDVK_E_ARG, "GroupNorm output must be F32 or F16");
    if (channels_last && (y_dtype != SDVK_F16 || C % 32 || (C / 32) > 65535 || batch > 65535 ||
                          (reinterpret_cast<uintptr_t>(y) & 15u)))
        return fail(env, SDVK_E_SHAPE,
                    "the channels-last GroupNorm writes F16 to a 16-byte aligned y and needs C % 32 == 0");
    if (batch == 0 || C == 0 || P == 0) return SDVK_OK;
    if (G == 0 || C % G || G > 65535 || batch > 65535)
        return fail(env, SDVK_E_SHAPE, "GroupNorm needs C % G == 0 and at most 65535 groups and images");
    const uint64_t need = groupnorm_workspace(batch, C, P, G);
    if (!workspace || ws_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 15u))
        return fail(env, SDVK_E_ARG, "GroupNorm workspace too small or misaligned (sdvk_groupnorm_workspace)");
    const uint64_t cnt = (uint64_t)(C / G) * P;
    const uint32_t chunks = (uint32_t)((cnt + kGnChunk - 1) / kGnChunk);
    if (chunks > 0x7FFFFFFFu) return fail(env, SDVK_E_SHAPE, "GroupNorm group too large");
    GnStat* st = static_cast<GnStat*>(workspace);
    const bool vec = P % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
    if (int rc = launch_pdl(gn_stats_kernel, dim3(chunks, G, batch), dim3(kGnThreads), 0, env, "gn_stats_kernel launch",
                            x, C, P, G, vec, st))
        return rc;
    if (channels_last) {
        const bool xvec = P % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0;
        if (C % 64 == 0)
            return launch_pdl(gn_apply_cl_kernel<64>, dim3((P + kGnClPos - 1) / kGnClPos, C / 64, batch), dim3(kGnThreads), 0, env,
                              "gn_apply_cl_kernel launch", x, gamma, beta, static_cast<__half*>(y), C, P, G, eps, act,
                              (const GnStat*)st, chunks, xvec);
        return launch_pdl(gn_apply_cl_kernel<32>, dim3((P + kGnClPos - 1) / kGnClPos, C / 32, batch), dim3(kGnThreads), 0, env,
                          "gn_apply_cl_kernel launch", x, gamma, beta, static_cast<__half*>(y), C, P, G, eps, act,
                          (const GnStat*)st, chunks, xvec);
    }
    if (y_dtype == SDVK_F16)
        return launch_pdl(gn_apply_kernel<__half>, dim3(C, batch), dim3(kGnThreads), 0, env, "gn_apply_kernel launch",
                          x, gamma, beta, static_cast<__half*>(y), C, P, G, eps, act, (const GnStat*)st, chunks,
                          vec && (reinterpret_cast<uintptr_t>(y) & 7u) == 0);
    return launch_pdl(gn_apply_kernel<float>, dim3(C, batch), dim3(kGnThreads), 0, env, "gn_apply_kernel launch", x,
                      gamma, beta, static_cast<float*>(y), C, P, G, eps, act, (const GnStat*)st, chunks, vec);
}

}  // namespace sdvk
