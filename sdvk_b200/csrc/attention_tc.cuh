// attention_tc.cuh -- fused flash attention on the 5th-generation tensor cores (tcgen05 + TMEM) for
// head dim 64 and 16-bit Q/K/V: O = softmax(Q K^T * scale) V per (batch, head), the operator of
// fused_attn_tiled.comp / fused_attn.comp.
//
// CTA = 128 query rows of one (batch, head).  The key/value sequence streams through shared memory
// in 128-key tiles loaded by TMA; tile t goes to softmax group t % 2, so two groups of 128 threads
// work on alternate tiles while the tensor core serves the other one:
//   warp 8     TMA: the Q tile once, then K/V tiles into a 4-stage ring
//   warp 9     TMEM allocation and the MMA issuer (one thread) (warps 10-11 only hold registers back):
//                S_g = Q . K_t^T            (M 128, N 128, K 64; A and B from shared memory)
//                O_g += P_g . V_t           (M 128, N 64, K 128; A = P from tensor memory)
//   warps 0-3  softmax group A (even tiles), warps 4-7 group B (odd tiles): thread = one query row
//              = one TMEM lane.  It reads its row of S from TMEM, applies the mask and the online
//              softmax (exp2 domain), writes P as 16-bit values back over S in TMEM, and rescales
//              its O row in TMEM only when the running maximum grew by more than 2^8.
// TMEM columns: S_A [0,128), S_B [128,256), O_A [256,320), O_B [320,384).
// At the end the two groups merge (O_A, m_A, l_A) and (O_B, m_B, l_B) row by row, normalise by
// 1/l (0 for a row that saw no key, as the reference) and store O with vector stores.
// Registers: 384 threads launch with 168 each (64512).  The control warpgroup (warps 8-11) drops to
// 56 and the two softmax warpgroups rise to 224, which holds a full 128-column row of S in
// registers: 2 x 128 x 224 + 128 x 56 = 64512, exactly the launch's pool.
// Every wait is bounded by p.timeout_ns: on expiry the kernel records kErrTimeout, drains what it
// issued and frees TMEM.
#pragma once

#include "gemm_q8.cuh"  // OperandTraits, kErrTimeout
#include "ptx.cuh"

namespace sdvk {

template <class T>
struct Half16Pack;
template <>
struct Half16Pack<__half> {  // low half = a
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};
template <>
struct Half16Pack<__nv_bfloat16> {
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
};

struct TcAttnParams {
    void* o;
    uint64_t ldo, so, ho;  // output strides, elements
    uint32_t Tq, Tk, heads, batch;
    float scale_log2;  // softmax scale * log2(e), > 0
    uint32_t causal;
    uint32_t* err;
    uint64_t timeout_ns;
};

struct TcAttnCfg {
    static constexpr int kBM = 128;  // query rows per CTA
    static constexpr int kBN = 128;  // keys per tile
    static constexpr int kHD = 64;
    static constexpr int kStages = 4;
    static constexpr int kTileBytes = kBN * kHD * 2;  // 16 KB (K or V tile; also the Q tile)
    static constexpr int kOffQ = 0;
    static constexpr int kOffKV = kOffQ + kTileBytes;
    static constexpr int kOffBar = kOffKV + kStages * 2 * kTileBytes;
    static constexpr int kNumBars = 1 + 2 * kStages + 2 + 2 + 1;
    static constexpr int kOffX = kOffBar + kNumBars * 8 + 8;  // TMEM slot + per-row (m, l) exchange
    static constexpr int kSmemBytes = kOffX + 4 * kBM * 4 + 1024;
    static constexpr int kThreads = 384;
    static constexpr uint32_t kRegsSoftmax = 224, kRegsControl = 56;
    static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsControl <= kThreads * 168, "register split exceeds the pool");
    // TMEM columns of group g's S (and P) and O
    static __device__ __forceinline__ uint32_t col_s(uint32_t g) { return g * 128u; }
    static __device__ __forceinline__ uint32_t col_o(uint32_t g) { return 256u + g * 64u; }
};

template <class T, class TO>
__global__ void __launch_bounds__(384, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const TcAttnParams p) {
    using Cfg = TcAttnCfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem + Cfg::kOffQ;
    uint8_t* sKV = smem + Cfg::kOffKV;  // stage s: K at s*32K, V at s*32K + 16K
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* q_full = bars;
    uint64_t* kv_full = q_full + 1;
    uint64_t* kv_empty = kv_full + Cfg::kStages;
    uint64_t* s_full = kv_empty + Cfg::kStages;
    uint64_t* p_full = s_full + 2;
    uint64_t* o_final = p_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_final + 1);
    float* xm = reinterpret_cast<float*>(smem + Cfg::kOffX);  // [2][128] running maxima
    float* xl = xm + 2 * Cfg::kBM;                              // [2][128] running sums

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t q0 = blockIdx.x * Cfg::kBM, head = blockIdx.y, b = blockIdx.z;
    // key tiles this CTA needs: all of them, or (causal) up to its last query row
    const uint32_t kv_end = p.causal ? min(p.Tk, q0 + Cfg::kBM) : p.Tk;
    const uint32_t n_kv = (kv_end + Cfg::kBN - 1) / Cfg::kBN;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < Cfg::kStages; ++i) {
            mbar_init(&kv_full[i], 1);
            mbar_init(&kv_empty[i], 1);
        }
        for (int g = 0; g < 2; ++g) {
            mbar_init(&s_full[g], 1);
            mbar_init(&p_full[g], 4);  // one arrival per softmax warp
        }
        mbar_init(o_final, 1);
        fence_mbar_init();
    }
    if (warp == 8 && lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 9) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool ok = true;
    auto fail = [&]() {
        atomicOr(p.err, kErrTimeout);
        ok = false;
    };

    if (warp >= 8) {
        regs_decrease<Cfg::kRegsControl>();
        if (warp == 8 && lane == 0) {
            // -------------------------------------------------------------- TMA producer
            mbar_arrive_expect_tx(q_full, Cfg::kTileBytes);
            tma_load_4d(sQ, &tmQ, q_full, 0, (int)q0, (int)head, (int)b);
            uint32_t t = 0;
            for (; t < n_kv; ++t) {
                const uint32_t s = t % Cfg::kStages, ph = (t / Cfg::kStages) & 1;
                if (!mbar_wait(&kv_empty[s], ph ^ 1, p.timeout_ns)) {
                    fail();
                    break;
                }
                uint8_t* dst = sKV + s * 2 * Cfg::kTileBytes;
                mbar_arrive_expect_tx(&kv_full[s], 2 * Cfg::kTileBytes);
                tma_load_4d(dst, &tmK, &kv_full[s], 0, (int)(t * Cfg::kBN), (int)head, (int)b);
                tma_load_4d(dst + Cfg::kTileBytes, &tmV, &kv_full[s], 0, (int)(t * Cfg::kBN), (int)head, (int)b);
            }
            // drain: every load issued has landed before the CTA can exit
            if (!mbar_wait(q_full, 0, p.timeout_ns)) fail();
            for (uint32_t i = (t > Cfg::kStages ? t - Cfg::kStages : 0); i < t; ++i)
                if (!mbar_wait(&kv_full[i % Cfg::kStages], (i / Cfg::kStages) & 1, p.timeout_ns)) fail();
        } else if (warp == 9 && lane == 0) {
            // -------------------------------------------------------------- MMA issuer
            constexpr uint32_t fmt = OperandTraits<T>::kFmt;
            constexpr uint32_t idesc_s = make_idesc(fmt, fmt, 0, 0, Cfg::kBM, Cfg::kBN);
            constexpr uint32_t idesc_o = make_idesc(fmt, fmt, 0, 1, Cfg::kBM, Cfg::kHD);
            const uint32_t q_addr = smem_u32(sQ);
            auto issue_s = [&](uint32_t t) -> bool {
                const uint32_t s = t % Cfg::kStages;
                if (!mbar_wait(&kv_full[s], (t / Cfg::kStages) & 1, p.timeout_ns)) return false;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(sKV + s * 2 * Cfg::kTileBytes);
#pragma unroll
                for (int kk = 0; kk < Cfg::kHD / 16; ++kk)
                    mma_f16(tmem + Cfg::col_s(t & 1), smem_desc_sw128(q_addr + kk * 32, 16, 1024),
                            smem_desc_sw128(k_addr + kk * 32, 16, 1024), idesc_s, kk > 0 ? 1u : 0u);
                mma_commit(&s_full[t & 1]);
                return true;
            };
            if (!mbar_wait(q_full, 0, p.timeout_ns)) fail();
            for (uint32_t t = 0; ok && t < n_kv && t < 2; ++t)
                if (!issue_s(t)) fail();
            for (uint32_t t = 0; ok && t < n_kv; ++t) {
                const uint32_t g = t & 1, i = t >> 1;
                if (!mbar_wait(&p_full[g], i & 1, p.timeout_ns)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t v_addr = smem_u32(sKV + (t % Cfg::kStages) * 2 * Cfg::kTileBytes + Cfg::kTileBytes);
#pragma unroll
                for (int kk = 0; kk < Cfg::kBN / 16; ++kk)
                    mma_f16_ts(tmem + Cfg::col_o(g), tmem + Cfg::col_s(g) + kk * 8,
                               smem_desc_sw128(v_addr + kk * 2048, Cfg::kTileBytes, 1024), idesc_o,
                               (i > 0 || kk > 0) ? 1u : 0u);
                mma_commit(&kv_empty[t % Cfg::kStages]);
                if (t + 2 < n_kv && !issue_s(t + 2)) {
                    fail();
                    break;
                }
            }
            mma_commit(o_final);
            if (!mbar_wait(o_final, 0, p.timeout_ns)) fail();
        }
    } else {
        // ------------------------------------------------------------------ softmax groups
        regs_increase<Cfg::kRegsSoftmax>();
        const uint32_t g = warp >> 2;             // 0: even key tiles, 1: odd key tiles
        const uint32_t r = (warp & 3) * 32 + lane;  // query row in the tile = TMEM lane
        const uint32_t lane_bits = ((warp & 3) * 32u) << 16;
        const uint32_t qrow = q0 + r;
        const float sl = p.scale_log2;
        float m_run = -INFINITY, l_run = 0.0f;
        for (uint32_t t = g, i = 0; t < n_kv; t += 2, ++i) {
            if (!__all_sync(0xffffffffu, mbar_wait(&s_full[g], i & 1, p.timeout_ns))) {
                fail();
                break;
            }
            tc_fence_after();
            uint32_t sr[128];
#pragma unroll
            for (int c = 0; c < 4; ++c)
                tmem_ld_32x32b_x32(tmem + lane_bits + Cfg::col_s(g) + c * 32,
                                   *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
            tmem_wait_ld();
            float* s = reinterpret_cast<float*>(sr);
            const uint32_t key0 = t * Cfg::kBN;
            if (key0 + Cfg::kBN > p.Tk || (p.causal && key0 + Cfg::kBN - 1 > q0)) {
#pragma unroll
                for (int j = 0; j < 128; ++j) {
                    const uint32_t key = key0 + j;
                    if (key >= p.Tk || (p.causal && key > qrow)) s[j] = -INFINITY;
                }
            }
            float mx = s[0];
#pragma unroll
            for (int j = 1; j < 128; ++j) mx = fmaxf(mx, s[j]);
            const float m_new = fmaxf(m_run, mx * sl);
            // Rescale only when the maximum grew by more than 2^8; P values up to 2^8 are exact
            // enough in 16 bits and the final 1/l uses the same stale maximum.
            const bool need = m_new - m_run > 8.0f;  // false for NaN (row still fully masked)
            if (__any_sync(0xffffffffu, need)) {
                const float f = need ? ex2_approx(m_run - m_new) : 1.0f;
                if (i > 0) {
                    uint32_t o[32];
#pragma unroll
                    for (int c = 0; c < 2; ++c) {
                        const uint32_t col = tmem + lane_bits + Cfg::col_o(g) + c * 32;
                        tmem_ld_32x32b_x32(col, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * f);
                        tmem_st_32x32b_x32(col, o);
                    }
                }
                l_run *= f;
                if (need) m_run = m_new;
            }
            const float mb = (m_run == -INFINITY) ? 0.0f : m_run;
            float sum = 0.0f;
#pragma unroll
            for (int h = 0; h < 2; ++h) {  // P over S: 16-bit pairs, columns [32h, 32h + 32)
                uint32_t pk[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const float p0 = ex2_approx(fmaf(s[64 * h + 2 * j], sl, -mb));
                    const float p1 = ex2_approx(fmaf(s[64 * h + 2 * j + 1], sl, -mb));
                    pk[j] = Half16Pack<T>::pack(p0, p1);
                    sum += p0 + p1;
                }
                tmem_st_32x32b_x32(tmem + lane_bits + Cfg::col_s(g) + 32 * h, pk);
            }
            l_run += sum;
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&p_full[g]);
        }
        // ---- merge the two groups and store
        xm[g * Cfg::kBM + r] = m_run;
        xl[g * Cfg::kBM + r] = l_run;
        __syncwarp();
        named_barrier(1, 256);
        const float mA = xm[r], lA = xl[r], mB = xm[Cfg::kBM + r], lB = xl[Cfg::kBM + r];
        const float m = fmaxf(mA, mB);
        const float fa = lA > 0.0f ? ex2_approx(mA - m) : 0.0f;
        const float fb = lB > 0.0f ? ex2_approx(mB - m) : 0.0f;
        const float l = lA * fa + lB * fb;
        const float inv = l > 0.0f ? 1.0f / l : 0.0f;
        const bool got = mbar_wait(o_final, 0, p.timeout_ns);
        if (!__all_sync(0xffffffffu, got)) {
            fail();
        } else {
            tc_fence_after();
            uint32_t oa[32], ob[32];
            tmem_ld_32x32b_x32(tmem + lane_bits + Cfg::col_o(0) + g * 32, oa);
            tmem_ld_32x32b_x32(tmem + lane_bits + Cfg::col_o(1) + g * 32, ob);
            tmem_wait_ld();
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                float acc = fa > 0.0f ? __uint_as_float(oa[j]) * fa : 0.0f;
                if (fb > 0.0f) acc = fmaf(__uint_as_float(ob[j]), fb, acc);
                v[j] = acc * inv;
            }
            if (qrow < p.Tq) {
                TO* dst = reinterpret_cast<TO*>(p.o) + (uint64_t)b * p.so + (uint64_t)head * p.ho +
                          (uint64_t)qrow * p.ldo + g * 32;
                if constexpr (sizeof(TO) == 4) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4)
                        *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; j += 8) {
                        uint4 w;
                        w.x = Half16Pack<__half>::pack(v[j], v[j + 1]);
                        w.y = Half16Pack<__half>::pack(v[j + 2], v[j + 3]);
                        w.z = Half16Pack<__half>::pack(v[j + 4], v[j + 5]);
                        w.w = Half16Pack<__half>::pack(v[j + 6], v[j + 7]);
                        *reinterpret_cast<uint4*>(dst + j) = w;
                    }
                }
            }
        }
    }

    // ---------------------------------------------------------------- teardown
    __syncwarp();
    __syncthreads();
    if (warp == 9) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace sdvk
