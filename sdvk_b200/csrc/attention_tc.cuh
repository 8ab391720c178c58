// attention_tc.cuh -- fused flash attention on the 5th-generation tensor cores (tcgen05 + TMEM) for
// head dim 64 and 16-bit Q/K/V: O = softmax(Q K^T * scale) V per (batch, head), the operator of
// fused_attn_tiled.comp / fused_attn.comp.
//
// CTA = 128 query rows of one (batch, head).  The key/value sequence streams through shared memory
// in 128-key tiles loaded by TMA; tile t goes to softmax group t % 2, so two groups of 128 threads
// work on alternate tiles while the tensor core serves the other one:
//   warp 8     TMA: the Q tile once, then K tiles into a 5-stage ring
//   warp 10    TMA: V tiles into a 7-stage ring (a K tile is free once S is computed, a V tile only
//              after P.V, so the two rings are separate to keep both far enough ahead)
//   warp 9     TMEM allocation and the MMA issuer (one thread) (warp 11 only holds registers back):
//                S_g = Q . K_t^T            (M 128, N 128, K 64; A and B from shared memory)
//                O_g += P_g . V_t           (M 128, N 64, K 128; A = P from tensor memory)
//   warps 0-3  softmax group A (even tiles), warps 4-7 group B (odd tiles): thread = one query row
//              = one TMEM lane.  It reads its row of S from TMEM, applies the mask and the online
//              softmax (exp2 domain; a quarter of the exponentials by polynomial on the FMA pipe),
//              writes P as 16-bit values back over S in TMEM, and rescales
//              its O row in TMEM only when the running maximum grew by more than 2^8.
// S is triple-buffered (tile t in buffer t % 3), so the MMA computes S for the next tile of a group
// while that group is still turning its current S into P: a group waits for the tensor core only
// when the tensor core is behind.
// TMEM columns: S buffers [0,128), [128,256), [256,384); O_A [384,448), O_B [448,512).
// At the end the two groups merge (O_A, m_A, l_A) and (O_B, m_B, l_B) row by row, normalise by
// 1/l (0 for a row that saw no key, as the reference) and store O with vector stores.
// Registers: 384 threads launch with 168 each (64512).  The control warpgroup (warps 8-11) drops to
// 72 and the two softmax warpgroups rise to 216, which holds a full 128-column row of S in
// registers: 2 x 128 x 216 + 128 x 72 = 64512, exactly the launch's pool.
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
    static constexpr int kKStages = 5, kVStages = 7;
    static constexpr int kTileBytes = kBN * kHD * 2;  // 16 KB (K or V tile; also the Q tile)
    static constexpr int kOffQ = 0;
    static constexpr int kOffK = kOffQ + kTileBytes;
    static constexpr int kOffV = kOffK + kKStages * kTileBytes;
    static constexpr int kOffBar = kOffV + kVStages * kTileBytes;
    static constexpr int kNumBars = 1 + 2 * kKStages + 2 * kVStages + 2 + 1;
    static constexpr int kOffX = kOffBar + kNumBars * 8 + 8;  // TMEM slot + per-row (m, l) exchange
    static constexpr int kSmemBytes = kOffX + 4 * kBM * 4 + 1024;
    static constexpr int kThreads = 384;
    static constexpr uint32_t kRegsSoftmax = 216, kRegsControl = 72;
    static_assert(2 * 128 * kRegsSoftmax + 128 * kRegsControl <= kThreads * 168, "register split exceeds the pool");
    // TMEM columns of S (and P) buffer b, and of group g's O
    static __device__ __forceinline__ uint32_t col_s(uint32_t b) { return b * 128u; }
    static __device__ __forceinline__ uint32_t col_o(uint32_t g) { return 384u + g * 64u; }
};

template <class T, class TO>
__global__ void __launch_bounds__(384, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const TcAttnParams p) {
    using Cfg = TcAttnCfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem + Cfg::kOffQ;
    uint8_t* sK = smem + Cfg::kOffK;
    uint8_t* sV = smem + Cfg::kOffV;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* q_full = bars;
    uint64_t* k_full = q_full + 1;
    uint64_t* k_empty = k_full + Cfg::kKStages;
    uint64_t* v_full = k_empty + Cfg::kKStages;
    uint64_t* v_empty = v_full + Cfg::kVStages;
    // k_empty[s] completing for tile t also says S(t) is in TMEM, and v_empty[s] completing says
    // P(t).V is in O: the softmax groups wait on those instead of on extra commits.
    uint64_t* p_full = v_empty + Cfg::kVStages;  // per group
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
        for (int i = 0; i < Cfg::kKStages; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
        }
        for (int i = 0; i < Cfg::kVStages; ++i) {
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        for (int g = 0; g < 2; ++g) mbar_init(&p_full[g], 4);  // one arrival per softmax warp
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
    // Everything above overlaps the previous kernel's tail; global memory is touched only after it.
    grid_dependency_wait();
    grid_launch_dependents();
    bool ok = true;
    auto fail = [&]() {
        atomicOr(p.err, kErrTimeout);
        ok = false;
    };

    if (warp >= 8) {
        regs_decrease<Cfg::kRegsControl>();
        if ((warp == 8 || warp == 10) && lane == 0) {
            // -------------------------------------------------------------- TMA producers (K; V)
            const bool is_k = warp == 8;
            const uint32_t nst = is_k ? Cfg::kKStages : Cfg::kVStages;
            uint64_t* full = is_k ? k_full : v_full;
            uint64_t* empty = is_k ? k_empty : v_empty;
            uint8_t* ring = is_k ? sK : sV;
            const CUtensorMap* map = is_k ? &tmK : &tmV;
            if (is_k) {
                mbar_arrive_expect_tx(q_full, Cfg::kTileBytes);
                tma_load_4d(sQ, &tmQ, q_full, 0, (int)q0, (int)head, (int)b);
            }
            uint32_t t = 0;
            for (; t < n_kv; ++t) {
                const uint32_t s = t % nst, ph = (t / nst) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1, p.timeout_ns)) {
                    fail();
                    break;
                }
                mbar_arrive_expect_tx(&full[s], Cfg::kTileBytes);
                tma_load_4d(ring + s * Cfg::kTileBytes, map, &full[s], 0, (int)(t * Cfg::kBN), (int)head, (int)b);
            }
            // drain: every load issued has landed before the CTA can exit
            if (is_k && !mbar_wait(q_full, 0, p.timeout_ns)) fail();
            for (uint32_t i = (t > nst ? t - nst : 0); i < t; ++i)
                if (!mbar_wait(&full[i % nst], (i / nst) & 1, p.timeout_ns)) fail();
        } else if (warp == 9) {
            // -------------------------------------------------------------- MMA issuer
            // The whole warp runs the loop (warp-uniform control flow and operands); one elected
            // lane issues each tcgen05 instruction.
            constexpr uint32_t fmt = OperandTraits<T>::kFmt;
            constexpr uint32_t idesc_s = make_idesc(fmt, fmt, 0, 0, Cfg::kBM, Cfg::kBN);
            constexpr uint32_t idesc_o = make_idesc(fmt, fmt, 0, 1, Cfg::kBM, Cfg::kHD);
            // Descriptors are built once; a K step advances the start-address field (16-byte
            // units) by 2 for K-major Q/K (32 bytes) and by 128 for MN-major V (16 rows of 128 B).
            const uint64_t q_desc = smem_desc_sw128(smem_u32(sQ), 16, 1024);
            const uint64_t k_desc0 = smem_desc_sw128(smem_u32(sK), 16, 1024);
            const uint64_t v_desc0 = smem_desc_sw128(smem_u32(sV), Cfg::kTileBytes, 1024);
            constexpr uint64_t kTileDesc = Cfg::kTileBytes >> 4;
            // The issuing thread keeps no divisions on its path: stage indices and phases advance
            // incrementally (every cycle it spends here the tensor pipe may sit idle).
            uint32_t ks = 0, kph = 0;  // K stage / phase of the next S to issue
            uint32_t vs = 0, vph = 0;  // V stage / phase of tile t
            auto issue_s = [&](uint32_t buf) -> bool {
                if (!__all_sync(0xffffffffu, mbar_spin_wait(&k_full[ks], kph, p.timeout_ns))) return false;
                tc_fence_after();
                const uint64_t k_desc = k_desc0 + ks * kTileDesc;
                const uint32_t d = tmem + Cfg::col_s(buf);
                if (elect_one()) {
#pragma unroll
                    for (int kk = 0; kk < Cfg::kHD / 16; ++kk)
                        mma_f16(d, q_desc + 2 * kk, k_desc + 2 * kk, idesc_s, kk > 0 ? 1u : 0u);
                    mma_commit(&k_empty[ks]);
                }
                __syncwarp();
                if (++ks == Cfg::kKStages) ks = 0, kph ^= 1;
                return true;
            };
            if (!__all_sync(0xffffffffu, mbar_wait(q_full, 0, p.timeout_ns))) fail();
            for (uint32_t t = 0; ok && t < n_kv && t < 3; ++t)
                if (!issue_s(t)) fail();
            uint32_t sb = 0;  // S buffer of tile t (t % 3)
            for (uint32_t t = 0; ok && t < n_kv; ++t) {
                const uint32_t g = t & 1, i = t >> 1;
                if (!__all_sync(0xffffffffu, mbar_spin_wait(&p_full[g], i & 1, p.timeout_ns) &&
                                                 mbar_spin_wait(&v_full[vs], vph, p.timeout_ns))) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint64_t v_desc = v_desc0 + vs * kTileDesc;
                const uint32_t d = tmem + Cfg::col_o(g), a = tmem + Cfg::col_s(sb);
                if (elect_one()) {
#pragma unroll
                    for (int kk = 0; kk < Cfg::kBN / 16; ++kk)
                        mma_f16_ts(d, a + kk * 8, v_desc + 128 * kk, idesc_o, (i > 0 || kk > 0) ? 1u : 0u);
                    mma_commit(&v_empty[vs]);
                }
                __syncwarp();
                if (++vs == Cfg::kVStages) vs = 0, vph ^= 1;
                // S(t + 3) reuses this buffer: the tensor core runs in issue order, so P(t) is read
                // by the P.V above before S(t + 3) overwrites it.
                if (t + 3 < n_kv && !issue_s(sb)) {
                    fail();
                    break;
                }
                sb = sb == 2 ? 0 : sb + 1;
            }
            if (elect_one()) mma_commit(o_final);
            __syncwarp();
            if (!__all_sync(0xffffffffu, mbar_wait(o_final, 0, p.timeout_ns))) fail();
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
            const uint32_t sb = t % 3;
            // S(t) has landed when K stage t % kKStages is released (at most that phase is pending:
            // S(t + kKStages) needs P(t + 2) of this group first).
            if (!__all_sync(0xffffffffu, mbar_wait(&k_empty[t % Cfg::kKStages], (t / Cfg::kKStages) & 1,
                                                   p.timeout_ns))) {
                fail();
                break;
            }
            tc_fence_after();
            uint32_t sr[128];
#pragma unroll
            for (int c = 0; c < 4; ++c)
                tmem_ld_32x32b_x32(tmem + lane_bits + Cfg::col_s(sb) + c * 32,
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
            // The softmax warps share each SMSP's issue slots with the MMA-issuing warp, so their
            // instruction count is what paces the tensor core: three-input max, packed f32x2
            // FMA/add, one convert per pair.
            float m4[4] = {s[0], s[1], s[2], s[3]};  // four independent chains
#pragma unroll
            for (int j = 4; j < 128; j += 2) m4[(j >> 1) & 3] = fmax3(m4[(j >> 1) & 3], s[j], s[j + 1]);
            const float mx = fmaxf(fmax3(m4[0], m4[1], m4[2]), m4[3]);
            const float m_new = fmaxf(m_run, mx * sl);
            // Rescale only when the maximum grew by more than 2^8; P values up to 2^8 are exact
            // enough in 16 bits and the final 1/l uses the same stale maximum.
            const bool need = m_new - m_run > 8.0f;  // false for NaN (row still fully masked)
            if (__any_sync(0xffffffffu, need)) {
                const float f = need ? ex2_approx(m_run - m_new) : 1.0f;
                // O holds this group's P.V up to its previous tile t - 2, which may still be running
                // (S(t) can complete before it); its V stage's release says it is done.  Only that
                // phase can be pending: P.V(t - 2 + kVStages) needs P(t + 2) of this group first.
                const uint32_t pt = t - 2;
                if (i > 0 && !__all_sync(0xffffffffu, mbar_wait(&v_empty[pt % Cfg::kVStages],
                                                                (pt / Cfg::kVStages) & 1, p.timeout_ns))) {
                    fail();
                    break;
                }
                if (i > 0) {
                    tc_fence_after();
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
            const uint64_t sl2 = f2_pack(sl, sl), nmb2 = f2_pack(-mb, -mb);
            uint64_t sum2[4] = {0, 0, 0, 0};  // packed pairs of partial sums (0 bits = 0.0f, 0.0f)
#pragma unroll
            for (int h = 0; h < 2; ++h) {  // P over S: 16-bit pairs, columns [32h, 32h + 32)
                uint32_t pk[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    float x0, x1, p0, p1;
                    f2_unpack(ffma2(f2_pack(s[64 * h + 2 * j], s[64 * h + 2 * j + 1]), sl2, nmb2), x0, x1);
                    // one pair in four on the FMA pipe, the rest on the MUFU: the MUFU is the
                    // softmax's busiest pipe and the FMA pipe has room
                    if ((j & 3) == 3) exp2_poly_pair(x0, x1, p0, p1);
                    else p0 = ex2_approx(x0), p1 = ex2_approx(x1);
                    pk[j] = Half16Pack<T>::pack(p0, p1);
                    sum2[j & 3] = fadd2(sum2[j & 3], f2_pack(p0, p1));
                }
                tmem_st_32x32b_x32(tmem + lane_bits + Cfg::col_s(sb) + 32 * h, pk);
            }
            float s_lo, s_hi;
            f2_unpack(fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3])), s_lo, s_hi);
            l_run += s_lo + s_hi;
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
