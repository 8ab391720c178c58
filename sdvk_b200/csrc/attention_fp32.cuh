// attention_fp32.cuh -- fused attention computed in fp32 on the CUDA cores, for fp32 Q/K/V at the
// reference's precision.  fused_attn_tiled.comp and fused_attn.comp compute in fp32 and the
// reference's test holds them to 2e-5 of max|ref| (tests/fused_attn_test.cpp:123-124); the tensor-core
// kernels round Q/K/V and P to 16 bits, which costs about 3e-4.  This kernel keeps every operand in
// fp32: it is the default for fp32 inputs (SDVK_PRECISION_REFERENCE), and the tensor-core kernels
// serve them under SDVK_PRECISION_FAST.
//
// CTA = 128 threads = 128 query rows of one (batch, head); thread = one query row, whose scaled Q
// row and O accumulator stay in registers.  K/V stream through shared memory in 32-key tiles read
// as broadcasts.  Online softmax in the exp2 domain, one rescale of O per tile.
#pragma once

#include "attention.cuh"  // AttnParams

namespace sdvk {

constexpr int kF32Rows = 128;
constexpr int kF32Keys = 32;

template <class TOut>
__global__ void __launch_bounds__(kF32Rows) attn_fp32_kernel(const AttnParams p) {
    grid_dependency_wait();
    grid_launch_dependents();
    __shared__ float sK[kF32Keys][64];
    __shared__ float sV[kF32Keys][64];
    const uint32_t b = blockIdx.z, h = blockIdx.y;
    const uint32_t row = blockIdx.x * kF32Rows + threadIdx.x;
    const uint32_t hd = p.hd;
    const float* Q = static_cast<const float*>(p.q) + (uint64_t)b * p.sq + (uint64_t)h * p.hq;
    const float* K = static_cast<const float*>(p.k) + (uint64_t)b * p.sk + (uint64_t)h * p.hk;
    const float* V = static_cast<const float*>(p.v) + (uint64_t)b * p.sv + (uint64_t)h * p.hv;
    const bool live = row < p.Tq;
    float q[64], o[64];
#pragma unroll
    for (int d = 0; d < 64; ++d) {
        q[d] = (live && (uint32_t)d < hd) ? Q[(uint64_t)row * p.ldq + d] * p.scale_log2 : 0.0f;
        o[d] = 0.0f;
    }
    float m = -INFINITY, l = 0.0f;
    // keys this CTA needs: all of them, or (causal) up to its last query row
    const uint32_t last_row = min(p.Tq, (blockIdx.x + 1) * kF32Rows) - 1;
    const uint32_t kv_end = p.causal ? min(p.Tk, last_row + 1) : p.Tk;
    for (uint32_t k0 = 0; k0 < kv_end; k0 += kF32Keys) {
        for (uint32_t i = threadIdx.x; i < kF32Keys * 64; i += kF32Rows) {
            const uint32_t j = i / 64, d = i % 64, key = k0 + j;
            const bool ok = key < p.Tk && d < hd;
            sK[j][d] = ok ? K[(uint64_t)key * p.ldk + d] : 0.0f;
            sV[j][d] = ok ? V[(uint64_t)key * p.ldv + d] : 0.0f;
        }
        __syncthreads();
        float s[kF32Keys];
        float mt = -INFINITY;
#pragma unroll
        for (int j = 0; j < kF32Keys; ++j) {
            float acc = 0.0f;
#pragma unroll
            for (int d = 0; d < 64; ++d) acc = fmaf(q[d], sK[j][d], acc);
            const uint32_t key = k0 + j;
            s[j] = (key >= p.Tk || (p.causal && key > row)) ? -INFINITY : acc;
            mt = fmaxf(mt, s[j]);
        }
        const float m_new = fmaxf(m, mt);
        if (m_new != -INFINITY) {  // a row that has seen no key yet keeps m = -inf, l = 0, o = 0
            const float corr = exp2f(m - m_new);  // 0 on the first tile (m = -inf)
            l *= corr;
#pragma unroll
            for (int d = 0; d < 64; ++d) o[d] *= corr;
#pragma unroll
            for (int j = 0; j < kF32Keys; ++j) {
                const float pj = exp2f(s[j] - m_new);  // 0 for a masked key
                l += pj;
#pragma unroll
                for (int d = 0; d < 64; ++d) o[d] = fmaf(pj, sV[j][d], o[d]);
            }
            m = m_new;
        }
        __syncthreads();
    }
    if (!live) return;
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    TOut* O = static_cast<TOut*>(p.o) + (uint64_t)b * p.so + (uint64_t)h * p.ho + (uint64_t)row * p.ldo;
#pragma unroll
    for (int d = 0; d < 64; ++d)
        if ((uint32_t)d < hd) O[d] = (TOut)(o[d] * inv);
}

}  // namespace sdvk
