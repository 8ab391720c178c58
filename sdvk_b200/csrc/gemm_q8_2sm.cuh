// gemm_q8_2sm.cuh -- the Q8_0 GEMM on CTA pairs (tcgen05 cta_group::2).
//
// A cluster of two CTAs on one TPC computes a 256 (x rows) x 256 (w rows) tile with one
// tcgen05.mma.cta_group::2 per 16-element K step, issued by the even CTA.  Each CTA stages its own
// 128 activation rows and dequantises only its own 128 weight rows, so per SM the dequantisation
// work and the weight traffic are half of the single-CTA kernel's for the same tensor-core work.
// The accumulator rows each CTA owns land in its own TMEM; each CTA runs its own epilogue.
//
// Cross-CTA signalling (all waits bounded, see GemmQ8Params::timeout_ns):
//   a_full   (even CTA)  both CTAs' activation TMA loads complete_tx here (cta_group::2 TMA)
//   b_full   (even CTA)  the 16 dequant warps of both CTAs arrive here
//   acc_empty(even CTA)  the 8 epilogue warps of both CTAs arrive here
//   a_empty, b_empty, acc_full (each CTA)  the MMA commit multicasts to both CTAs
//   w_full, w_empty (each CTA)  the local raw-weight ring
#pragma once

#include "gemm_q8.cuh"

namespace sdvk {

template <class TA>
struct Gemm2Config {
    static constexpr int kBM = 128;      // activation rows per CTA (pair: 256)
    static constexpr int kBNP = 256;     // weight rows per pair tile
    static constexpr int kBNC = 128;     // weight rows dequantised by each CTA
    static constexpr int kES = sizeof(TA);
    static constexpr int kBK = 128 / kES;
    static constexpr int kUmmaK = 32 / kES;
    static constexpr int kSA = 5;        // activation stages
    static constexpr int kSW = 4;        // raw int8 weight stages
    static constexpr int kSB = 4;        // dequantised weight stages
    static constexpr int kAcc = 2;
    static constexpr int kABytes = kBM * 128;
    static constexpr int kWBytes = kBNC * kBK;
    static constexpr int kBBytes = kBNC * 128;
    static constexpr int kEpiBytes = 4 * 2 * 4096;
    static constexpr uint32_t kTmemCols = 512;
    static constexpr int kOffA = 0;
    static constexpr int kOffB = kOffA + kSA * kABytes;
    static constexpr int kOffW = kOffB + kSB * kBBytes;
    static constexpr int kOffEpi = kOffW + kSW * kWBytes;
    static constexpr int kOffBar = kOffEpi + kEpiBytes;
    static constexpr int kNumBars = 2 * kSA + 2 * kSW + 2 * kSB + 2 * kAcc + 1;
    static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
    static constexpr int kThreads = 512;
    static constexpr int kConvThreads = 256;
    static constexpr int kChunksPerRow = kBK / 16;
    static constexpr int kTasksPerThread = kBNC * kChunksPerRow / kConvThreads;
    static constexpr int kRowStep = kConvThreads / kChunksPerRow;
    static_assert(kSmemBytes <= 232448, "shared memory");
    static_assert(kTasksPerThread >= 1 && (kBNC * kChunksPerRow) % kConvThreads == 0, "dequant split");
};

template <class TA, bool NN, class TC>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(512, 1)
    gemm_q8_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmC, const GemmQ8Params p) {
    using Cfg = Gemm2Config<TA>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem + Cfg::kOffA;
    uint8_t* sB = smem + Cfg::kOffB;
    uint8_t* sW = smem + Cfg::kOffW;
    uint8_t* sEpi = smem + Cfg::kOffEpi;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* a_full = bars;
    uint64_t* a_empty = a_full + Cfg::kSA;
    uint64_t* w_full = a_empty + Cfg::kSA;
    uint64_t* w_empty = w_full + Cfg::kSW;
    uint64_t* b_full = w_empty + Cfg::kSW;
    uint64_t* b_empty = b_full + Cfg::kSB;
    uint64_t* acc_full = b_empty + Cfg::kSB;
    uint64_t* acc_empty = acc_full + Cfg::kAcc;
    uint64_t* mma_done = acc_empty + Cfg::kAcc;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const uint32_t cid = cluster_id_x(), ncl = nclusters_x();

    if (threadIdx.x == 0) {
        for (int i = 0; i < Cfg::kSA; ++i) {
            mbar_init(&a_full[i], 1);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < Cfg::kSW; ++i) {
            mbar_init(&w_full[i], 1);
            mbar_init(&w_empty[i], 8);
        }
        for (int i = 0; i < Cfg::kSB; ++i) {
            mbar_init(&b_full[i], 16);
            mbar_init(&b_empty[i], 1);
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

    bool ok = true;
    auto fail = [&]() {
        atomicOr(p.err, kErrTimeout);
        ok = false;
    };
    // Pair tiles: tiles_x counts 256-row pair tiles here.
    auto decode = [&](uint32_t tile, uint32_t& z, uint32_t& xt, uint32_t& wt) {
        wt = tile % p.tiles_w;
        const uint32_t rest = tile / p.tiles_w;
        xt = rest % p.tiles_x;
        z = rest / p.tiles_x;
    };
    const uint32_t my_tiles = (p.num_tiles > cid) ? (p.num_tiles - cid + ncl - 1) / ncl : 0;
    const uint32_t my_iters = my_tiles * p.k_stages;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            uint32_t it = 0;
            for (uint32_t i = 0; ok && i < my_tiles; ++i) {
                uint32_t z, xt, wt;
                decode(cid + i * ncl, z, xt, wt);
                const int zw = p.sW ? (int)z : 0;
                const int x0 = (int)(xt * 2 * Cfg::kBM + rank * Cfg::kBM);
                for (uint32_t ks = 0; ks < p.k_stages; ++ks, ++it) {
                    const uint32_t sa = it % Cfg::kSA, pa = (it / Cfg::kSA) & 1;
                    const uint32_t sw = it % Cfg::kSW, pw = (it / Cfg::kSW) & 1;
                    const int k0 = (int)(ks * Cfg::kBK);
                    if (!mbar_wait(&a_empty[sa], pa ^ 1, p.timeout_ns)) {
                        fail();
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(&a_full[sa], 2 * Cfg::kABytes);  // both CTAs' bytes
                    const uint32_t afull_l = mapa_shared(&a_full[sa], 0);
                    uint8_t* a_dst = sA + sa * Cfg::kABytes;
                    if constexpr (!NN) {
                        tma_load_3d_pair(a_dst, &tmA, afull_l, k0, x0, (int)z);
                    } else {
#pragma unroll
                        for (int j = 0; j < Cfg::kBM / Cfg::kBK; ++j)
                            tma_load_3d_pair(a_dst + j * Cfg::kBK * 128, &tmA, afull_l, x0 + j * Cfg::kBK, k0, (int)z);
                    }
                    if (!mbar_wait(&w_empty[sw], pw ^ 1, p.timeout_ns)) {
                        fail();
                        break;
                    }
                    mbar_arrive_expect_tx(&w_full[sw], Cfg::kWBytes);
                    tma_load_3d(sW + sw * Cfg::kWBytes, &tmW, &w_full[sw], k0,
                                (int)(wt * Cfg::kBNP + rank * Cfg::kBNC), zw);
                }
            }
            // Drain this CTA's raw-weight loads (the activation loads are drained by the MMA).
            for (uint32_t i = (it > Cfg::kSW ? it - Cfg::kSW : 0); i < it; ++i)
                if (!mbar_wait(&w_full[i % Cfg::kSW], (i / Cfg::kSW) & 1, p.timeout_ns)) fail();
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (even CTA)
        if (leader && lane == 0) {
            constexpr uint32_t idesc =
                make_idesc(OperandTraits<TA>::kFmt, OperandTraits<TA>::kFmt, NN ? 1 : 0, 0, 2 * Cfg::kBM, Cfg::kBNP);
            uint32_t it = 0;
            for (uint32_t i = 0; ok && i < my_tiles; ++i) {
                const uint32_t acc = i % Cfg::kAcc, aph = (i / Cfg::kAcc) & 1;
                if (!mbar_wait_cluster(&acc_empty[acc], aph ^ 1, p.timeout_ns)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * Cfg::kBNP;
                for (uint32_t ks = 0; ks < p.k_stages; ++ks, ++it) {
                    const uint32_t sa = it % Cfg::kSA, pa = (it / Cfg::kSA) & 1;
                    const uint32_t sb = it % Cfg::kSB, pb = (it / Cfg::kSB) & 1;
                    if (!mbar_wait_cluster(&a_full[sa], pa, p.timeout_ns) ||
                        !mbar_wait_cluster(&b_full[sb], pb, p.timeout_ns)) {
                        fail();
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + sa * Cfg::kABytes);
                    const uint32_t b_addr = smem_u32(sB + sb * Cfg::kBBytes);
#pragma unroll
                    for (int kk = 0; kk < Cfg::kBK / Cfg::kUmmaK; ++kk) {
                        uint64_t adesc;
                        if constexpr (!NN)
                            adesc = smem_desc_sw128(a_addr + kk * 32, 16, 1024);
                        else if constexpr (!OperandTraits<TA>::kTf32)
                            adesc = smem_desc_sw128(a_addr + kk * Cfg::kUmmaK * 128, Cfg::kBK * 128, 1024);
                        else
                            adesc = smem_desc(a_addr + kk * Cfg::kUmmaK * 128, Cfg::kBK * 128, 512, kLayoutSw128Base32);
                        const uint64_t bdesc = smem_desc_sw128(b_addr + kk * 32, 16, 1024);
                        const uint32_t accum = (ks > 0 || kk > 0) ? 1u : 0u;
                        if constexpr (OperandTraits<TA>::kTf32) mma_tf32_pair(d_tmem, adesc, bdesc, idesc, accum);
                        else mma_f16_pair(d_tmem, adesc, bdesc, idesc, accum);
                    }
                    mma_commit_pair_mc(&a_empty[sa], 0x3);
                    mma_commit_pair_mc(&b_empty[sb], 0x3);
                }
                if (!ok) break;
                mma_commit_pair_mc(&acc_full[acc], 0x3);
            }
            mma_commit_pair(mma_done);
            if (!mbar_wait(mma_done, 0, p.timeout_ns)) fail();
        }
    } else if (warp >= 4 && warp < 12) {
        // ------------------------------------------------------------ dequantisers (both CTAs)
        const int ct = threadIdx.x - 128;
        const int chunk = ct % Cfg::kChunksPerRow;
        const int row0 = ct / Cfg::kChunksPerRow;
        const uint64_t kblocks = p.K / 32;
        const uint64_t ldw_blocks = p.ldw / 32;
        constexpr int T = Cfg::kTasksPerThread;
        // Scales for iteration j (two iterations ahead of use, so their L2 latency is hidden).
        auto load_scales = [&](uint32_t j, float (&sc)[T]) {
#pragma unroll
            for (int t = 0; t < T; ++t) sc[t] = 0.0f;
            if (j >= my_iters) return;
            uint32_t z, xt, wt;
            decode(cid + (j / p.k_stages) * ncl, z, xt, wt);
            const uint64_t kb = ((uint64_t)(j % p.k_stages) * Cfg::kBK + (uint64_t)chunk * 16) / 32;
            if (kb >= kblocks) return;
            const float* ws = p.ws + (p.sW ? (uint64_t)z * (p.sW / 32) : 0);
#pragma unroll
            for (int t = 0; t < T; ++t) {
                const uint32_t n = wt * Cfg::kBNP + rank * Cfg::kBNC + row0 + t * Cfg::kRowStep;
                if (n < p.wrows) sc[t] = __ldg(ws + (uint64_t)n * ldw_blocks + kb);
            }
        };
        float sc0[T], sc1[T], sc2[T];
        load_scales(0, sc0);
        load_scales(1, sc1);
        for (uint32_t it = 0; ok && it < my_iters; ++it) {
            load_scales(it + 2, sc2);
            const uint32_t sw = it % Cfg::kSW, pw = (it / Cfg::kSW) & 1;
            const uint32_t sb = it % Cfg::kSB, pb = (it / Cfg::kSB) & 1;
            const bool got = mbar_wait(&w_full[sw], pw, p.timeout_ns) && mbar_wait(&b_empty[sb], pb ^ 1, p.timeout_ns);
            if (!__all_sync(0xffffffffu, got)) {  // the warp leaves the loop together
                fail();
                break;
            }
            const uint8_t* wsrc = sW + sw * Cfg::kWBytes;
            uint8_t* bdst = sB + sb * Cfg::kBBytes;
            uint4 raw[T];
#pragma unroll
            for (int t = 0; t < T; ++t)
                raw[t] = *reinterpret_cast<const uint4*>(wsrc + (row0 + t * Cfg::kRowStep) * Cfg::kBK + chunk * 16);
#pragma unroll
            for (int t = 0; t < T; ++t) {
                const int r = row0 + t * Cfg::kRowStep;
                dequant16<TA>(raw[t], sc0[t], bdst + r * 128, r, chunk * Cfg::kES);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&w_empty[sw]);
                mbar_arrive_cluster(mapa_shared(&b_full[sb], 0));
            }
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
                if (lane == 0) bulk_wait_read<1>();
                __syncwarp();
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
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));
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
