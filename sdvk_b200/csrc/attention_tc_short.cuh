// attention_tc_short.cuh -- tcgen05 attention for at most 128 keys (the 77-token cross-attention of
// fused_attn.comp), head dim 64, 16-bit Q/K/V.
//
// The work is HBM-bound (Q in, O out; K/V come from L2) and per item tiny, so the kernel is built
// for latency: 128-thread CTAs, two per SM, persistent over work items (batch, head, 128-query tile),
// with the next item's Q/K/V TMA-loaded into the other half of a double buffer while this item
// computes.  Per item:
//   S = Q K^T        one elected lane, M128 x N(keys rounded up to 16) x K64, into TMEM [0, 128)
//   softmax          thread = query row = TMEM lane: keys past Tk masked, exp2 domain, P written as
//                    16-bit pairs over S
//   O = P V          M128 x N64 x K(keys rounded up to 16), A (P) from TMEM, V MN-major from shared
//                    memory, into TMEM [128, 192)
//   epilogue         O row * 1/l, 16-byte vector stores from registers
// Every wait is bounded (TcAttnParams::timeout_ns): a wait that runs out records kErrTimeout and
// the CTA stops taking items, drains its loads and frees TMEM.
#pragma once

#include "attention_tc.cuh"

namespace sdvk {

struct TcShortCfg {
    static constexpr int kBM = 128;  // query rows per item
    static constexpr int kBN = 128;  // keys (at most)
    static constexpr int kHD = 64;
    static constexpr int kTile = kBM * kHD * 2;  // 16 KB: one Q, K or V tile
    static constexpr int kBuf = 3 * kTile;       // Q, K, V of one item
    static constexpr int kOffBar = 2 * kBuf;
    static constexpr int kSmemBytes = kOffBar + 64 + 1024;
    static constexpr int kThreads = 128;
    static constexpr uint32_t kTmemCols = 256;
    static constexpr uint32_t kColO = 128;
};

template <class T, class TO>
__global__ void __launch_bounds__(TcShortCfg::kThreads, 2)
    attn_tc_short_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const TcAttnParams p) {
    using Cfg = TcShortCfg;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* ld_full = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);  // [2]
    uint64_t* s_done = ld_full + 2;
    uint64_t* o_done = s_done + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t n_qt = (p.Tq + Cfg::kBM - 1) / Cfg::kBM;
    const uint32_t items = n_qt * p.heads * p.batch;
    const uint32_t n_s = ((p.Tk + 15) / 16) * 16;  // S columns computed (keys rounded up to 16)
    const uint32_t n_k16 = n_s / 16;               // K steps of P.V

    if (threadIdx.x == 0) {
        mbar_init(&ld_full[0], 1);
        mbar_init(&ld_full[1], 1);
        mbar_init(s_done, 1);
        mbar_init(o_done, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
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
    auto decode = [&](uint32_t item, uint32_t& qt, uint32_t& head, uint32_t& b) {
        qt = item % n_qt;
        const uint32_t rest = item / n_qt;
        head = rest % p.heads;
        b = rest / p.heads;
    };
    auto issue = [&](uint32_t item, int buf) {  // thread 0
        uint32_t qt, head, b;
        decode(item, qt, head, b);
        uint8_t* dst = smem + buf * Cfg::kBuf;
        mbar_arrive_expect_tx(&ld_full[buf], 3 * Cfg::kTile);
        tma_load_4d(dst, &tmQ, &ld_full[buf], 0, (int)(qt * Cfg::kBM), (int)head, (int)b);
        tma_load_4d(dst + Cfg::kTile, &tmK, &ld_full[buf], 0, 0, (int)head, (int)b);
        tma_load_4d(dst + 2 * Cfg::kTile, &tmV, &ld_full[buf], 0, 0, (int)head, (int)b);
    };

    constexpr uint32_t fmt = OperandTraits<T>::kFmt;
    const uint32_t idesc_s = make_idesc(fmt, fmt, 0, 0, Cfg::kBM, n_s);
    constexpr uint32_t idesc_o = make_idesc(fmt, fmt, 0, 1, Cfg::kBM, Cfg::kHD);
    const uint32_t r = (uint32_t)warp * 32 + lane;  // query row in the item = TMEM lane
    const uint32_t lane_bits = ((uint32_t)warp * 32u) << 16;
    const float sl = p.scale_log2;

    uint32_t j = 0, issued = 0;  // items consumed and issued by this CTA
    if (threadIdx.x == 0 && blockIdx.x < items) {
        issue(blockIdx.x, 0);
        issued = 1;
    }
    for (uint32_t item = blockIdx.x; item < items; item += gridDim.x, ++j) {
        const int buf = j & 1;
        // The other buffer's last reader (the previous item's MMAs) has completed: prefetch into it.
        if (threadIdx.x == 0 && ok && item + gridDim.x < items) {
            issue(item + gridDim.x, buf ^ 1);
            ++issued;
        }
        uint8_t* sQ = smem + buf * Cfg::kBuf;
        if (warp == 0) {
            if (!__all_sync(0xffffffffu, mbar_wait(&ld_full[buf], (j >> 1) & 1, p.timeout_ns))) fail();
            if (ok) {
                tc_fence_after();
                const uint64_t qd = smem_desc_sw128(smem_u32(sQ), 16, 1024);
                const uint64_t kd = smem_desc_sw128(smem_u32(sQ + Cfg::kTile), 16, 1024);
                if (elect_one()) {
#pragma unroll
                    for (int kk = 0; kk < Cfg::kHD / 16; ++kk) mma_f16(tmem, qd + 2 * kk, kd + 2 * kk, idesc_s, kk > 0);
                    mma_commit(s_done);
                }
                __syncwarp();
            }
        }
        if (!__syncthreads_and(ok)) {
            ok = false;
            break;
        }
        // ---- softmax over the row's keys
        if (!mbar_wait(s_done, j & 1, p.timeout_ns)) fail();
        if (!__syncthreads_and(ok)) {
            ok = false;
            break;
        }
        tc_fence_after();
        uint32_t sr[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            if ((uint32_t)c * 32 < n_s) {
                tmem_ld_32x32b_x32(tmem + lane_bits + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[c * 32]));
            } else {
#pragma unroll
                for (int e = 0; e < 32; ++e) sr[c * 32 + e] = __float_as_uint(-INFINITY);
            }
        }
        tmem_wait_ld();
        float* s = reinterpret_cast<float*>(sr);
#pragma unroll
        for (int k = 0; k < 128; ++k)
            if ((uint32_t)k >= p.Tk) s[k] = -INFINITY;
        float m4[4] = {s[0], s[1], s[2], s[3]};
#pragma unroll
        for (int k = 4; k < 128; k += 2) m4[(k >> 1) & 3] = fmax3(m4[(k >> 1) & 3], s[k], s[k + 1]);
        const float mb = fmaxf(fmax3(m4[0], m4[1], m4[2]), m4[3]) * sl;  // Tk >= 1: finite
        const uint64_t sl2 = f2_pack(sl, sl), nmb2 = f2_pack(-mb, -mb);
        uint64_t sum2[4] = {0, 0, 0, 0};
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // P over S: 16-bit pairs, columns [32h, 32h + 32)
            uint32_t pk[32];
#pragma unroll
            for (int q = 0; q < 32; ++q) {
                float x0, x1;
                f2_unpack(ffma2(f2_pack(s[64 * h + 2 * q], s[64 * h + 2 * q + 1]), sl2, nmb2), x0, x1);
                const float p0 = ex2_approx(x0), p1 = ex2_approx(x1);
                pk[q] = Half16Pack<T>::pack(p0, p1);
                sum2[q & 3] = fadd2(sum2[q & 3], f2_pack(p0, p1));
            }
            tmem_st_32x32b_x32(tmem + lane_bits + 32 * h, pk);
        }
        float s_lo, s_hi;
        f2_unpack(fadd2(fadd2(sum2[0], sum2[1]), fadd2(sum2[2], sum2[3])), s_lo, s_hi);
        const float l = s_lo + s_hi;
        tmem_wait_st();
        tc_fence_before();
        __syncthreads();  // every row's P is in TMEM
        // ---- O = P V
        if (warp == 0) {
            tc_fence_after();
            const uint64_t vd = smem_desc_sw128(smem_u32(sQ + 2 * Cfg::kTile), Cfg::kTile, 1024);
            if (elect_one()) {
                for (uint32_t kk = 0; kk < n_k16; ++kk)
                    mma_f16_ts(tmem + Cfg::kColO, tmem + kk * 8, vd + 128 * kk, idesc_o, kk > 0 ? 1u : 0u);
                mma_commit(o_done);
            }
            __syncwarp();
        }
        // ---- epilogue
        if (!mbar_wait(o_done, j & 1, p.timeout_ns)) fail();
        if (!__syncthreads_and(ok)) {
            ok = false;
            break;
        }
        tc_fence_after();
        uint32_t o[64];
        tmem_ld_32x32b_x32(tmem + lane_bits + Cfg::kColO, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
        tmem_ld_32x32b_x32(tmem + lane_bits + Cfg::kColO + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
        tmem_wait_ld();
        uint32_t qt, head, b;
        decode(item, qt, head, b);
        const uint32_t qrow = qt * Cfg::kBM + r;
        const float inv = 1.0f / l;
        if (qrow < p.Tq) {
            TO* dst = reinterpret_cast<TO*>(p.o) + (uint64_t)b * p.so + (uint64_t)head * p.ho + (uint64_t)qrow * p.ldo;
            if constexpr (sizeof(TO) == 4) {
#pragma unroll
                for (int e = 0; e < 64; e += 4)
                    *reinterpret_cast<float4*>(dst + e) =
                        make_float4(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv,
                                    __uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
            } else {
#pragma unroll
                for (int e = 0; e < 64; e += 8) {
                    uint4 w;
                    w.x = Half16Pack<__half>::pack(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
                    w.y = Half16Pack<__half>::pack(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
                    w.z = Half16Pack<__half>::pack(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
                    w.w = Half16Pack<__half>::pack(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
                    *reinterpret_cast<uint4*>(dst + e) = w;
                }
            }
        }
        tc_fence_before();
        __syncthreads();  // TMEM S/P/O and this buffer are free for the next items
    }
    // ---- teardown: every load issued has landed before the CTA exits
    if (threadIdx.x == 0) {
        for (uint32_t i = j; i < issued; ++i)
            if (!mbar_wait(&ld_full[i & 1], (i >> 1) & 1, p.timeout_ns)) fail();
    }
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, Cfg::kTmemCols);
    }
}

}  // namespace sdvk
