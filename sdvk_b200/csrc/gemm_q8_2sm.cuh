// gemm_q8_2sm.cuh -- the Q8_0 GEMM on CTA pairs (tcgen05 cta_group::2).
//
// A cluster of two CTAs on one TPC computes a 256 (x rows) x BNP (w rows) tile with one
// tcgen05.mma.cta_group::2 per 16-element K step, issued by the even CTA.  Each CTA stages its own
// 128 activation rows and dequantises only its own BNP/2 weight rows, so per SM the dequantisation
// work and the weight traffic are half of the single-CTA kernel's for the same tensor-core work.
// The accumulator rows each CTA owns land in its own TMEM; each CTA runs its own epilogue.
//
// The tensor pipe idles whenever the issuing thread polls a barrier that is not yet complete, so
// its per-stage control path is one CTA-scope poll of one barrier and one commit:
//   full[s]   (even CTA)  activation TMA bytes of both CTAs (cta_group::2 TMA) + the 16
//                         dequantiser warps of both CTAs; the even CTA's producer sets the tx count
//   empty[s]  (each CTA)  one MMA commit multicast to both CTAs frees activation and operand slot s
//   acc_full  (each CTA)  MMA commit multicast;  acc_empty (even CTA): the 8 epilogue warps
//   w_full, w_empty (each CTA)  the local raw int8 weight ring (TMA -> dequantisers)
// Warp roles per CTA: 0 activation TMA, 1 TMEM + MMA (even CTA issues), 2 weight TMA,
// 4-11 dequantisers, 12-15 epilogue (3 idle).
//
// Every wait is bounded (GemmQ8Params::timeout_ns): a wait that runs out records kErrTimeout, the
// CTA drains what it issued, both CTAs meet at the final cluster barrier and free TMEM.
#pragma once

#include "gemm_q8.cuh"

namespace sdvk {

template <class TA, int BNP>
struct Gemm2Config {
    static constexpr int kBM = 128;       // activation rows per CTA (pair: 256)
    static constexpr int kBNP = BNP;      // weight rows per pair tile (tensor-core N)
    static constexpr int kBNC = BNP / 2;  // weight rows dequantised by each CTA
    static constexpr int kES = sizeof(TA);
    static constexpr int kBK = 128 / kES;
    static constexpr int kUmmaK = 32 / kES;
    static constexpr int kS = 5;          // stages of (activation tile, dequantised weight tile)
    static constexpr int kSW = 4;         // raw int8 weight stages
    static constexpr int kAcc = 2;
    static constexpr int kABytes = kBM * 128;
    static constexpr int kBBytes = kBNC * 128;
    static constexpr int kStageBytes = kABytes + ((kBBytes + 1023) / 1024) * 1024;
    static constexpr int kWBytes = kBNC * kBK;
    static constexpr int kEpiBytes = 4 * 2 * 4096;  // 4 epilogue warps x 2 buffers x 32x32 fp32
    static constexpr uint32_t kTmemCols = 512;
    static constexpr int kOffStage = 0;
    static constexpr int kOffW = kOffStage + kS * kStageBytes;
    static constexpr int kOffEpi = kOffW + ((kSW * kWBytes + 1023) / 1024) * 1024;
    static constexpr int kOffBar = kOffEpi + kEpiBytes;
    static constexpr int kNumBars = 2 * kS + 2 * kSW + 2 * kAcc + 1;
    static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
    static constexpr int kThreads = 512;
    static constexpr int kConvThreads = 256;
    static constexpr int kChunksPerRow = kBK / 16;
    static constexpr int kTasksPerThread = (kBNC * kChunksPerRow + kConvThreads - 1) / kConvThreads;
    static constexpr int kRowStep = kConvThreads / kChunksPerRow;
    static_assert(kSmemBytes <= 232448, "shared memory");
    static_assert(BNP % 32 == 0 && BNP >= 128 && BNP <= 256, "pair tile N");
};

template <class TA, int BNP, bool NN, class TC>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(512, 1)
    gemm_q8_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmC, const GemmQ8Params p) {
    using Cfg = Gemm2Config<TA, BNP>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sStage = smem + Cfg::kOffStage;  // stage s: activation tile, then dequantised weights
    uint8_t* sW = smem + Cfg::kOffW;
    uint8_t* sEpi = smem + Cfg::kOffEpi;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* full = bars;
    uint64_t* empty = full + Cfg::kS;
    uint64_t* w_full = empty + Cfg::kS;
    uint64_t* w_empty = w_full + Cfg::kSW;
    uint64_t* acc_full = w_empty + Cfg::kSW;
    uint64_t* acc_empty = acc_full + Cfg::kAcc;
    uint64_t* mma_done = acc_empty + Cfg::kAcc;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const uint32_t cid = cluster_id_x(), ncl = nclusters_x();

    if (threadIdx.x == 0) {
        for (int i = 0; i < Cfg::kS; ++i) {
            mbar_init(&full[i], 1 + 16);  // producer's expect_tx + 16 dequantiser warps
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < Cfg::kSW; ++i) {
            mbar_init(&w_full[i], 1);
            mbar_init(&w_empty[i], 8);
        }
        for (int i = 0; i < Cfg::kAcc; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 8);
        }
        mbar_init(mma_done, 1);
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmW);
        tma_prefetch_desc(&tmC);
    }
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish_pair();
        tc_fence_before();
    }
    __syncwarp();
    cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    // Everything above overlaps the previous kernel's tail; global memory is touched only after it.
    grid_dependency_wait();
    grid_launch_dependents();

    bool ok = true;
    auto fail = [&]() {
        atomicOr(p.err, kErrTimeout);
        ok = false;
    };
    // Pair tiles: tiles_x counts 256-row pair tiles.
    auto decode = [&](uint32_t tile, uint32_t& z, uint32_t& xt, uint32_t& wt) {
        wt = tile % p.tiles_w;
        const uint32_t rest = tile / p.tiles_w;
        xt = rest % p.tiles_x;
        z = rest / p.tiles_x;
    };
    const uint32_t my_tiles = (p.num_tiles > cid) ? (p.num_tiles - cid + ncl - 1) / ncl : 0;
    const uint32_t my_iters = my_tiles * p.k_stages;

    if (warp == 0) {
        // ------------------------------------------------------------ activation TMA producer (both CTAs)
        if (lane == 0) {
            uint32_t it = 0;
            for (uint32_t i = 0; ok && i < my_tiles; ++i) {
                uint32_t z, xt, wt;
                decode(cid + i * ncl, z, xt, wt);
                const int x0 = (int)(xt * 2 * Cfg::kBM + rank * Cfg::kBM);
                for (uint32_t ks = 0; ks < p.k_stages; ++ks, ++it) {
                    const uint32_t s = it % Cfg::kS, ph = (it / Cfg::kS) & 1;
                    const int k0 = (int)(ks * Cfg::kBK);
                    if (!mbar_wait(&empty[s], ph ^ 1, p.timeout_ns)) {
                        fail();
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(&full[s], 2 * Cfg::kABytes);  // both CTAs' bytes
                    const uint32_t full_l = mapa_shared(&full[s], 0);
                    uint8_t* a_dst = sStage + s * Cfg::kStageBytes;
                    if constexpr (!NN) {
                        tma_load_3d_pair(a_dst, &tmA, full_l, k0, x0, (int)z);
                    } else {
#pragma unroll
                        for (int j = 0; j < Cfg::kBM / Cfg::kBK; ++j)
                            tma_load_3d_pair(a_dst + j * Cfg::kBK * 128, &tmA, full_l, x0 + j * Cfg::kBK, k0, (int)z);
                    }
                }
            }
            // The activation loads are drained by the MMA (it waits for every one it consumes).
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------ raw weight TMA producer (both CTAs)
        if (lane == 0) {
            uint32_t it = 0;
            for (uint32_t i = 0; ok && i < my_tiles; ++i) {
                uint32_t z, xt, wt;
                decode(cid + i * ncl, z, xt, wt);
                const int zw = p.sW ? (int)z : 0;
                for (uint32_t ks = 0; ks < p.k_stages; ++ks, ++it) {
                    const uint32_t sw = it % Cfg::kSW, pw = (it / Cfg::kSW) & 1;
                    if (!mbar_wait(&w_empty[sw], pw ^ 1, p.timeout_ns)) {
                        fail();
                        break;
                    }
                    mbar_arrive_expect_tx(&w_full[sw], Cfg::kWBytes);
                    tma_load_3d(sW + sw * Cfg::kWBytes, &tmW, &w_full[sw], (int)(ks * Cfg::kBK),
                                (int)(wt * Cfg::kBNP + rank * Cfg::kBNC), zw);
                }
            }
            for (uint32_t i = (it > Cfg::kSW ? it - Cfg::kSW : 0); i < it; ++i)  // drain
                if (!mbar_wait(&w_full[i % Cfg::kSW], (i / Cfg::kSW) & 1, p.timeout_ns)) fail();
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (even CTA)
        // The whole warp runs the loop (warp-uniform control flow and operands, no divisions on
        // the path); one elected lane issues each tcgen05 instruction.  Every cycle this warp
        // spends between MMAs can be tensor-pipe idle time.
        if (leader) {
            constexpr uint32_t idesc =
                make_idesc(OperandTraits<TA>::kFmt, OperandTraits<TA>::kFmt, NN ? 1 : 0, 0, 2 * Cfg::kBM, Cfg::kBNP);
            // Operand descriptors of stage 0; a stage adds kStageBytes, a K step of kUmmaK elements
            // adds 32 bytes (K-major) or kUmmaK rows of 128 bytes (MN-major activations).
            const uint32_t a0 = smem_u32(sStage);
            uint64_t adesc0;
            if constexpr (!NN) adesc0 = smem_desc_sw128(a0, 16, 1024);
            else if constexpr (!OperandTraits<TA>::kTf32) adesc0 = smem_desc_sw128(a0, Cfg::kBK * 128, 1024);
            else adesc0 = smem_desc(a0, Cfg::kBK * 128, 512, kLayoutSw128Base32);
            const uint64_t bdesc0 = smem_desc_sw128(a0 + Cfg::kABytes, 16, 1024);
            constexpr uint64_t kStageDesc = Cfg::kStageBytes >> 4;
            constexpr uint64_t kAStep = NN ? (Cfg::kUmmaK * 128) >> 4 : 2;
            uint32_t s = 0, ph = 0;
            for (uint32_t i = 0; ok && i < my_tiles; ++i) {
                const uint32_t acc = i & (Cfg::kAcc - 1), aph = (i / Cfg::kAcc) & 1;
                if (!__all_sync(0xffffffffu, mbar_wait(&acc_empty[acc], aph ^ 1, p.timeout_ns))) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * Cfg::kBNP;
                for (uint32_t ks = 0; ks < p.k_stages; ++ks) {
                    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph, p.timeout_ns))) {
                        fail();
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = adesc0 + s * kStageDesc, bd = bdesc0 + s * kStageDesc;
                    if (elect_one()) {
#pragma unroll
                        for (int kk = 0; kk < Cfg::kBK / Cfg::kUmmaK; ++kk) {
                            const uint32_t accum = (ks > 0 || kk > 0) ? 1u : 0u;
                            if constexpr (OperandTraits<TA>::kTf32)
                                mma_tf32_pair(d_tmem, ad + kk * kAStep, bd + 2 * kk, idesc, accum);
                            else mma_f16_pair(d_tmem, ad + kk * kAStep, bd + 2 * kk, idesc, accum);
                        }
                        mma_commit_pair_mc(&empty[s], 0x3);
                    }
                    __syncwarp();
                    if (++s == Cfg::kS) s = 0, ph ^= 1;
                }
                if (!ok) break;
                if (elect_one()) mma_commit_pair_mc(&acc_full[acc], 0x3);
                __syncwarp();
            }
            if (elect_one()) mma_commit_pair(mma_done);
            __syncwarp();
            if (!__all_sync(0xffffffffu, mbar_wait(mma_done, 0, p.timeout_ns))) fail();
        }
    } else if (warp >= 4 && warp < 12) {
        // ------------------------------------------------------------ dequantisers (both CTAs)
        const int ct = threadIdx.x - 128;
        const int chunk = ct % Cfg::kChunksPerRow;
        const int row0 = ct / Cfg::kChunksPerRow;
        constexpr int T = Cfg::kTasksPerThread;
        // Scales come from L2 two stages ahead of use (latency hidden).
        WeightCursor<T> cur;
        cur.init(&p, cid, ncl, row0, Cfg::kRowStep, Cfg::kBK, chunk * 16, Cfg::kBNP, rank * Cfg::kBNC, Cfg::kBNC);
        float sc0[T], sc1[T], sc2[T];
        uint4 unused[T];
        cur.load<false>(sc0, unused);
        cur.advance();
        cur.load<false>(sc1, unused);
        cur.advance();
        for (uint32_t it = 0; ok && it < my_iters; ++it) {
            cur.load<false>(sc2, unused);
            cur.advance();
            const uint32_t s = it % Cfg::kS, ph = (it / Cfg::kS) & 1;
            const uint32_t sw = it % Cfg::kSW, pw = (it / Cfg::kSW) & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&w_full[sw], pw, p.timeout_ns))) {  // leave together
                fail();
                break;
            }
            const uint8_t* wsrc = sW + sw * Cfg::kWBytes;
            uint8_t* bdst = sStage + s * Cfg::kStageBytes + Cfg::kABytes;
            uint4 raw[T];
#pragma unroll
            for (int t = 0; t < T; ++t) {
                const int r = row0 + t * Cfg::kRowStep;
                raw[t] = (r < Cfg::kBNC) ? *reinterpret_cast<const uint4*>(wsrc + r * Cfg::kBK + chunk * 16)
                                         : make_uint4(0, 0, 0, 0);
            }
            // The raw slot is free as soon as its bytes are in registers: hand it back to the weight
            // TMA before waiting for the operand stage (the arrive orders the warp's reads before
            // the next load into the slot), so the weight ring keeps moving while the stage ring is
            // full and its depth covers the TMA latency alone.
            __syncwarp();
            if (lane == 0) mbar_arrive(&w_empty[sw]);
            if (!__all_sync(0xffffffffu, mbar_wait(&empty[s], ph ^ 1, p.timeout_ns))) {
                fail();
                break;
            }
#pragma unroll
            for (int t = 0; t < T; ++t) {
                const int r = row0 + t * Cfg::kRowStep;
                if (r < Cfg::kBNC) dequant16<TA>(raw[t], sc0[t], bdst + r * 128, r, chunk * Cfg::kES);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(&full[s], 0));
#pragma unroll
            for (int t = 0; t < T; ++t) {
                sc0[t] = sc1[t];
                sc1[t] = sc2[t];
            }
        }
    } else if (warp >= 12) {
        // ------------------------------------------------------------ epilogue (both CTAs)
        const int q = warp & 3;
        uint8_t* ebuf = sEpi + q * (2 * 4096);
        uint32_t nstore = 0;
        for (uint32_t i = 0; ok && i < my_tiles; ++i) {
            uint32_t z, xt, wt;
            decode(cid + i * ncl, z, xt, wt);
            const uint32_t acc = i % Cfg::kAcc, aph = (i / Cfg::kAcc) & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[acc], aph, p.timeout_ns))) {
                fail();
                break;
            }
            tc_fence_after();
            const int x0 = (int)(xt * 2 * Cfg::kBM + rank * Cfg::kBM) + q * 32;
#pragma unroll 1
            for (int cc = 0; cc < Cfg::kBNP / 32; ++cc, ++nstore) {
                const int w0 = (int)(wt * Cfg::kBNP) + cc * 32;
                uint32_t raw[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * Cfg::kBNP + cc * 32, raw);
                tmem_wait_ld();
                if (cc + 1 == Cfg::kBNP / 32) {  // accumulator fully read: hand it back to the MMA
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));
                }
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]);
                if (p.bias) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const uint32_t n = (uint32_t)w0 + j;
                        v[j] += (n < p.wrows) ? __ldg(p.bias + n) : 0.0f;
                    }
                }
                uint8_t* buf = ebuf + (nstore & 1) * 4096;
                if (lane == 0) bulk_wait_read<1>();  // the store that last used `buf` has read it
                __syncwarp();
                if constexpr (!NN && sizeof(TC) == 2) {
                    if (p.geglu) {  // chunk = [a(16) | gate(16)] -> 16 outputs, a 32-byte row per lane
                        uint32_t h[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            __half2 t2 = __floats2half2_rn(v[2 * j] * gelu_erf_as_fast(v[16 + 2 * j]),
                                                           v[2 * j + 1] * gelu_erf_as_fast(v[17 + 2 * j]));
                            h[j] = *reinterpret_cast<uint32_t*>(&t2);
                        }
                        *reinterpret_cast<uint4*>(buf + lane * 32) = make_uint4(h[0], h[1], h[2], h[3]);
                        *reinterpret_cast<uint4*>(buf + lane * 32 + 16) = make_uint4(h[4], h[5], h[6], h[7]);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_3d(&tmC, buf, w0 / 2, x0, (int)z);
                            bulk_commit();
                        }
                        continue;
                    }
                }
                if constexpr (!NN) store_epi_row<TC>(buf, lane, v);
                else store_epi_col<TC>(buf, lane, v);
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if constexpr (!NN) {
                        if (p.accumulate) tma_reduce_add_3d(&tmC, buf, w0, x0, (int)z);
                        else tma_store_3d(&tmC, buf, w0, x0, (int)z);
                    } else {
                        if (p.accumulate) tma_reduce_add_3d(&tmC, buf, x0, w0, (int)z);
                        else tma_store_3d(&tmC, buf, x0, w0, (int)z);
                    }
                    bulk_commit();
                }
            }
        }
        if (lane == 0) bulk_wait_all();
    }

    // ---------------------------------------------------------------- teardown
    __syncwarp();
    cluster_sync();  // both CTAs done with TMEM and with each other's shared memory
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
    }
}

}  // namespace sdvk
