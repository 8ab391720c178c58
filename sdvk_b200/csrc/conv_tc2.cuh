// conv_tc2.cuh -- the 3x3 convolution as an implicit GEMM on CTA pairs (tcgen05 cta_group::2).
//
// y[z][o][p] = bias[z][o] + sum_{c,ky,kx} w[o][c][ky][kx] * x[z][c][oh*S + ky + lo][ow*S + kx + lo]
// (0 outside the image; lo = -1 for the symmetric pad-1 ring, 0 for right/bottom padding), the
// reference's conv3RawInto / conv3s2 (sdvkgen.cpp:1133-1175), without the column matrix:
//   A (tensor-core M: 128 output positions per CTA, 256 per pair)  the input windows, straight from
//        the channels-last fp16 input [z][h][w][c] by TMA in im2col mode.  One load per stage brings
//        128 consecutive output positions x 64 channels at one tap's offset from each position's
//        window corner; what falls outside the image reads as zero (the padding).  The rows land
//        128B-swizzled, K-major: the layout the tensor core reads.
//   B (tensor-core N: BN/2 output channels per CTA)  the weights as fp16 [cout][K'], K' =
//        (cblock * 9 + tap) * 64 + channel-in-block, stage ks = cblock * 9 + tap (repacked once
//        from the Q8_0 payload: q*s rounded to fp16, the value the GEMM's dequantiser produces).
// Both operands arrive by TMA, so the stage's only arrival is the even CTA's producer with the byte
// count of all four loads; the odd CTA's loads complete on the even CTA's barrier.
// D[position][channel] (TMEM lane = position, column = output channel) is stored transposed: tiles
// of [32 channels][32 positions] into the channel-major output, bias added, stored or reduce-added.
//
// Warp roles per CTA: 0 both TMA loads, 1 TMEM + MMA (even CTA issues), 4-7 epilogue.  Every wait is
// bounded (ConvParams::timeout_ns); a wait that runs out records kErrTimeout and the CTA leaves its
// loop, both CTAs meet at the final cluster barrier and free TMEM.
#pragma once

#include "gemm_q8.cuh"

namespace sdvk {

struct ConvParams {
    const float* bias;  // per output channel, image z's at bias + z * sbias (or null)
    uint64_t sbias;
    uint32_t P, OW;     // output positions per image (a multiple of 128), output width
    uint32_t batch, cout;
    int stride, lower;  // input coordinate of output (0, 0)'s window corner is (lower, lower)
    uint32_t k_stages;  // 9 * cin / 64
    uint32_t tiles_n, num_tiles;
    uint32_t accumulate;
    uint32_t* err;
    uint64_t timeout_ns;
};

#ifndef SDVK_CONV_EPI_BUFS
#define SDVK_CONV_EPI_BUFS 2
#endif
#ifndef SDVK_CONV_MAX_STAGES
#define SDVK_CONV_MAX_STAGES 8
#endif

template <int BN>
struct ConvCfg {
    static constexpr int kABytes = 128 * 128;        // 128 positions x 64 fp16 channels
    static constexpr int kBBytes = (BN / 2) * 128;   // BN/2 output channels x 64 fp16
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kEpiBufs = SDVK_CONV_EPI_BUFS;  // 32x32 fp32 staging buffers per epilogue warp
    static constexpr int kEpiBytes = 4 * kEpiBufs * 4096;
    static constexpr int kMaxSmem = 232448;
    static constexpr int kSFit = (kMaxSmem - 1024 - 256 - kEpiBytes) / kStageBytes;
    static constexpr int kS = kSFit > SDVK_CONV_MAX_STAGES ? SDVK_CONV_MAX_STAGES : kSFit;
    static constexpr int kAcc = 2;
    static constexpr uint32_t kTmemCols = (kAcc * BN <= 64) ? 64 : (kAcc * BN <= 128) ? 128 : (kAcc * BN <= 256) ? 256 : 512;
    static constexpr int kOffEpi = kS * kStageBytes;
    static constexpr int kOffBar = kOffEpi + kEpiBytes;
    static constexpr int kNumBars = 2 * kS + 2 * kAcc + 1;
    static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
    static constexpr int kThreads = 256;
    static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "pair tile N");
    static_assert(kBBytes % 1024 == 0, "B stage: whole 8-row swizzle atoms");
    static_assert(kS >= 3 && kSmemBytes <= kMaxSmem, "shared memory");
};

template <int BN, class TC>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 1)
    conv3x3_tc2_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                       const __grid_constant__ CUtensorMap tmC, const ConvParams p) {
    using Cfg = ConvCfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sEpi = smem + Cfg::kOffEpi;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* full = bars;
    uint64_t* empty = full + Cfg::kS;
    uint64_t* acc_full = empty + Cfg::kS;
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
            mbar_init(&full[i], 1);  // the even CTA's producer (expect_tx of both CTAs' bytes)
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < Cfg::kAcc; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 8);
        }
        mbar_init(mma_done, 1);
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmX);
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
    grid_dependency_wait();
    grid_launch_dependents();

    bool ok = true;
    auto fail = [&]() {
        atomicOr(p.err, kErrTimeout);
        ok = false;
    };
    // Tiles: 256 consecutive output positions (over images and rows) x BN output channels, the
    // channel tiles fastest so that the clusters working at one time read the same input windows.
    const uint32_t my_tiles = (p.num_tiles > cid) ? (p.num_tiles - cid + ncl - 1) / ncl : 0;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            uint32_t it = 0;
            for (uint32_t i = 0; ok && i < my_tiles; ++i) {
                const uint32_t tile = cid + i * ncl, nt = tile % p.tiles_n, mt = tile / p.tiles_n;
                const uint64_t g0 = (uint64_t)mt * 256 + rank * 128;  // this CTA's first position
                const uint32_t z = (uint32_t)(g0 / p.P), pp = (uint32_t)(g0 % p.P);
                const int wc = (int)(pp % p.OW) * p.stride + p.lower, hc = (int)(pp / p.OW) * p.stride + p.lower;
                const int n_row = (int)(nt * BN + rank * (BN / 2));
                uint32_t cb = 0, tap = 0;  // stage ks = cb * 9 + tap
                for (uint32_t ks = 0; ks < p.k_stages; ++ks, ++it) {
                    const uint32_t s = it % Cfg::kS, ph = (it / Cfg::kS) & 1;
                    if (!mbar_wait(&empty[s], ph ^ 1, p.timeout_ns)) {
                        fail();
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(&full[s], 2 * Cfg::kStageBytes);  // both CTAs' bytes
                    const uint32_t full_l = mapa_shared(&full[s], 0);
                    uint8_t* dst = smem + s * Cfg::kStageBytes;
                    const uint16_t kx = (uint16_t)(tap % 3), ky = (uint16_t)(tap / 3);
                    tma_load_im2col_4d_pair(dst, &tmX, full_l, (int)(cb * 64), wc, hc, (int)z, kx, ky);
                    tma_load_3d_pair(dst + Cfg::kABytes, &tmW, full_l, (int)(ks * 64), n_row, 0);
                    if (++tap == 9) tap = 0, ++cb;
                }
            }
            // The loads are drained by the MMA (it waits for every one it consumes).
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (even CTA)
        if (leader) {
            constexpr uint32_t idesc = make_idesc(0, 0, 0, 0, 256, BN);  // f16 x f16, both K-major
            const uint32_t a0 = smem_u32(smem);
            const uint64_t adesc0 = smem_desc_sw128(a0, 16, 1024);
            const uint64_t bdesc0 = smem_desc_sw128(a0 + Cfg::kABytes, 16, 1024);
            constexpr uint64_t kStageDesc = Cfg::kStageBytes >> 4;
            uint32_t s = 0, ph = 0;
            for (uint32_t i = 0; ok && i < my_tiles; ++i) {
                const uint32_t acc = i & (Cfg::kAcc - 1), aph = (i / Cfg::kAcc) & 1;
                if (!__all_sync(0xffffffffu, mbar_wait(&acc_empty[acc], aph ^ 1, p.timeout_ns))) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (uint32_t ks = 0; ks < p.k_stages; ++ks) {
                    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], ph, p.timeout_ns))) {
                        fail();
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = adesc0 + s * kStageDesc, bd = bdesc0 + s * kStageDesc;
                    if (elect_one()) {
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)  // 4 x 16 channels, 32 bytes apart in the swizzled rows
                            mma_f16_pair(d_tmem, ad + 2 * kk, bd + 2 * kk, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
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
    } else if (warp >= 4) {
        // ------------------------------------------------------------ epilogue (both CTAs)
        // Warp q reads TMEM lanes 32q..32q+31: output positions g0 + 32q + lane of this CTA's 128
        // (one image: P is a multiple of 128); each 32-column chunk is 32 output channels.
        const int q = warp & 3;
        uint8_t* ebuf = sEpi + q * (Cfg::kEpiBufs * 4096);
        uint32_t nstore = 0;
        for (uint32_t i = 0; ok && i < my_tiles; ++i) {
            const uint32_t tile = cid + i * ncl, nt = tile % p.tiles_n, mt = tile / p.tiles_n;
            const uint32_t acc = i % Cfg::kAcc, aph = (i / Cfg::kAcc) & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[acc], aph, p.timeout_ns))) {
                fail();
                break;
            }
            tc_fence_after();
            const uint64_t g = (uint64_t)mt * 256 + rank * 128 + q * 32;
            const uint32_t z = (uint32_t)(g / p.P), p0 = (uint32_t)(g % p.P);
            const bool live = z < p.batch;  // a last pair tile may end past the last image
#pragma unroll 1
            for (int cc = 0; cc < BN / 32; ++cc, ++nstore) {
                const uint32_t o0 = nt * BN + cc * 32;
                uint32_t raw[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + cc * 32, raw);
                tmem_wait_ld();
                if (cc + 1 == BN / 32) {  // accumulator fully read: hand it back to the MMA
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));
                }
                if (!live || o0 >= p.cout) continue;
                const uint32_t o = o0 + lane;
                const float bl = (p.bias && o < p.cout) ? __ldg(p.bias + z * p.sbias + o) : 0.0f;
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]) + __shfl_sync(0xffffffffu, bl, j);
                uint8_t* buf = ebuf + (nstore % Cfg::kEpiBufs) * 4096;
                if (lane == 0) bulk_wait_read<Cfg::kEpiBufs - 1>();  // the store that last used `buf` has read it
                __syncwarp();
                store_epi_col<TC>(buf, lane, v);  // [32 channels][32 positions]
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    if (p.accumulate) tma_reduce_add_3d(&tmC, buf, (int)p0, (int)o0, (int)z);
                    else tma_store_3d(&tmC, buf, (int)p0, (int)o0, (int)z);
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
