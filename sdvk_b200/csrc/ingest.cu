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
// chunk to (count, mean, M2) with a two-pass sum over its chunk (the reference's two-pass form), a
// one-warp kernel merges a group's chunks with Chan's pairwise update, and the apply kernel
// normalises.  All three are HBM-bound: x is read twice (the second stats pass hits L2) and y
// written once.
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
// (the second from L2).
__global__ void __launch_bounds__(kGnThreads) gn_stats_kernel(const float* __restrict__ x, uint32_t C, uint32_t P,
                                                              uint32_t G, GnStat* __restrict__ stats) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ float red[kGnThreads / 32];
    const uint32_t g = blockIdx.y, b = blockIdx.z, chunks = gridDim.x;
    const uint64_t cnt = (uint64_t)(C / G) * P;
    const float* xg = x + (uint64_t)b * C * P + (uint64_t)g * cnt;
    const uint64_t lo = (uint64_t)blockIdx.x * kGnChunk, hi = min(cnt, lo + kGnChunk);
    float s = 0.0f;
    for (uint64_t i = lo + threadIdx.x; i < hi; i += kGnThreads) s += xg[i];
    const float n = (float)(hi - lo);
    const float mean = block_sum(s, red) / n;
    float ss = 0.0f;
    for (uint64_t i = lo + threadIdx.x; i < hi; i += kGnThreads) {
        const float d = xg[i] - mean;
        ss = fmaf(d, d, ss);
    }
    const float m2 = block_sum(ss, red);
    if (threadIdx.x == 0) stats[((uint64_t)b * G + g) * chunks + blockIdx.x] = GnStat{n, mean, m2};
}

// grid (G, B), one warp: merge the group's chunk statistics in a fixed order (Chan et al.'s
// pairwise update of count, mean and M2) into (mean, 1 / sqrt(var + eps)).
__global__ void gn_finalize_kernel(const GnStat* __restrict__ stats, uint32_t chunks, float eps,
                                   float2* __restrict__ norm) {
    grid_dependency_wait();
    grid_launch_dependents();
    if (threadIdx.x != 0) return;
    const uint64_t gi = (uint64_t)blockIdx.y * gridDim.x + blockIdx.x;
    const GnStat* st = stats + gi * chunks;
    float n = st[0].n, m = st[0].mean, m2 = st[0].m2;
    for (uint32_t c = 1; c < chunks; ++c) {
        const GnStat o = st[c];
        const float nn = n + o.n, d = o.mean - m;
        m += d * (o.n / nn);
        m2 += o.m2 + d * d * (n * o.n / nn);
        n = nn;
    }
    norm[gi] = make_float2(m, 1.0f / sqrtf(m2 / n + eps));
}

// grid (blocks over C*P, B): y = (x - mean) * rstd * gamma + beta (+ SiLU v / (1 + e^-v)).
__global__ void __launch_bounds__(kGnThreads) gn_apply_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                              const float* __restrict__ beta, float* __restrict__ y,
                                                              uint32_t C, uint32_t P, uint32_t G, uint32_t act,
                                                              const float2* __restrict__ norm) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint32_t b = blockIdx.y;
    const uint64_t per = (uint64_t)C * P, cnt = (uint64_t)(C / G) * P;
    const float* xb = x + (uint64_t)b * per;
    float* yb = y + (uint64_t)b * per;
    const float2* nb = norm + (uint64_t)b * G;
    for (uint64_t i = (uint64_t)blockIdx.x * kGnThreads + threadIdx.x; i < per; i += (uint64_t)gridDim.x * kGnThreads) {
        const float2 mr = nb[i / cnt];
        const uint32_t ch = (uint32_t)(i / P);
        float v = (xb[i] - mr.x) * mr.y * gamma[ch] + beta[ch];
        if (act) v = v / (1.0f + expf(-v));
        yb[i] = v;
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
    const uint64_t stats = (uint64_t)batch * G * chunks * sizeof(GnStat);
    return ((stats + 15) / 16) * 16 + (uint64_t)batch * G * sizeof(float2);
}

int groupnorm(const float* x, const float* gamma, const float* beta, float* y, uint32_t batch, uint32_t C, uint32_t P,
              uint32_t G, float eps, uint32_t act, void* workspace, uint64_t ws_bytes, const LaunchEnv& env) {
    if (!x || !gamma || !beta || !y) return fail(env, SDVK_E_ARG, "null pointer");
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
    const uint64_t stat_bytes = (uint64_t)batch * G * chunks * sizeof(GnStat);
    float2* norm = reinterpret_cast<float2*>(static_cast<uint8_t*>(workspace) + ((stat_bytes + 15) / 16) * 16);
    if (int rc = launch_pdl(gn_stats_kernel, dim3(chunks, G, batch), dim3(kGnThreads), 0, env, "gn_stats_kernel launch",
                            x, C, P, G, st))
        return rc;
    if (int rc = launch_pdl(gn_finalize_kernel, dim3(G, batch), dim3(32), 0, env, "gn_finalize_kernel launch",
                            (const GnStat*)st, chunks, eps, norm))
        return rc;
    const uint64_t per = (uint64_t)C * P;
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((per + kGnThreads - 1) / kGnThreads, 8ull * env.num_sms);
    return launch_pdl(gn_apply_kernel, dim3(blocks, batch), dim3(kGnThreads), 0, env, "gn_apply_kernel launch", x, gamma,
                      beta, y, C, P, G, act, (const float2*)norm);
}

}  // namespace sdvk
