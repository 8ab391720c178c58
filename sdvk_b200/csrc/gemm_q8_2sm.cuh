// gemm_q8_2sm.cuh -- the Q8_0 GEMM on CTA pairs (tcgen05 cta_group::2).
//
// A cluster of two CTAs on one TPC computes a 256 (w rows) x BNX (x rows) tile with one
// tcgen05.mma.cta_group::2 per 16-element K step, issued by the even CTA.  Operand roles:
//   A (tensor-core M, 128 rows per CTA)  the dequantised weights: each CTA dequantises its own 128
//                                        weight rows into its own shared memory, and only its own
//                                        SM's tensor core reads them;
//   B (tensor-core N, BNX/2 rows per CTA) the activations, staged by TMA; both SMs' tensor cores
//                                        read both halves.
// With the operand written by generic stores (the dequantised weights) on the per-CTA side, the
// data a tensor core reads from generic stores is always its own SM's, ordered by a CTA-scope
// proxy fence; the activations that both SMs read arrive by TMA.  The 256 weight rows of a tile
// also divide the model's widths (1280, 10240) exactly.
// The accumulator D[w][x] (TMEM lane = weight row, column = activation row) is stored transposed
// for NT (C[x][w]) and directly for NN (C[w][x]).
//
// Two rings, sized independently: the dequantised-weight ring (one slot per dequantiser group) and the
// activation ring (6 slots: 8 measured slower in the UNet pass; the shared memory a raw-weight ring
// used to take is left unused).  The raw int8 weights do not pass through shared memory: the kernel
// is bound by shared-memory bandwidth (a k-stage moved about 745 128-byte wavefronts per SM at tile
// width 224: tensor-core operand reads, TMA writes, the dequantised tile's stores, the epilogue), and
// a TMA write plus a load of the raw tile were 128 of them.  Each dequantiser thread loads its
// 16-byte chunks of raw weights and their scales from global memory SDVK_GEMM2_RAW_AHEAD of its
// group's stages ahead, into registers.
// The tensor pipe idles whenever the issuing thread polls a barrier that is not yet complete, so its
// per-stage control path is two CTA-scope polls and two commits:
//   x_full[sx]  (even CTA)  activation TMA bytes of both CTAs (cta_group::2 TMA); the even CTA's
//                           producer sets the tx count
//   a_full[sa]  (even CTA)  one dequantiser group's warps of both CTAs
//   x_empty[sx], a_empty[sa] (each CTA)  an MMA commit multicast to both CTAs frees the slot
//   acc_full  (each CTA)  MMA commit multicast;  acc_empty (even CTA): the 8 epilogue warps
// Warp roles per CTA: 0 activation TMA, 1 TMEM + MMA (even CTA issues), 4-11 dequantisers in groups
// that take stages round-robin, 12-15 epilogue (2 and 3 idle).  One warp's pass over a stage is a
// chain of waits, shared-memory stores, a proxy fence and a remote arrive that lasts several times
// the stage's MMA time, so several groups keep several stages in flight.
//
// Every wait is bounded (GemmQ8Params::timeout_ns): a wait that runs out records kErrTimeout, the
// CTA drains what it issued, both CTAs meet at the final cluster barrier and free TMEM.
#pragma once

#include <type_traits>

#include "gemm_q8.cuh"

namespace sdvk {

template <class TA, int BNX>
struct Gemm2Config {
    static constexpr int kBW = 128;       // weight rows per CTA (pair: 256, tensor-core M)
    static constexpr int kBNX = BNX;      // activation rows per pair tile (tensor-core N)
    static constexpr int kBXC = BNX / 2;  // activation rows staged by each CTA
    static constexpr int kES = sizeof(TA);
    static constexpr int kBK = 128 / kES;
    static constexpr int kUmmaK = 32 / kES;
#ifndef SDVK_GEMM2_A_STAGES
#define SDVK_GEMM2_A_STAGES 4
#endif
#ifndef SDVK_GEMM2_RAW_AHEAD
#define SDVK_GEMM2_RAW_AHEAD 2
#endif
#ifndef SDVK_GEMM2_X_STAGES
#define SDVK_GEMM2_X_STAGES 6
#endif
#ifndef SDVK_GEMM2_EPI_BUFS
#define SDVK_GEMM2_EPI_BUFS 2
#endif
    static constexpr int kSA = SDVK_GEMM2_A_STAGES;    // dequantised weight tiles
    static constexpr int kRawAhead = SDVK_GEMM2_RAW_AHEAD;  // own stages of raw weights in registers
    static constexpr int kAcc = 2;
    static constexpr int kABytes = kBW * 128;
    static constexpr int kXBytes = ((kBXC * 128 + 1023) / 1024) * 1024;
    static constexpr int kEpiBufs = SDVK_GEMM2_EPI_BUFS;  // 32x32 fp32 staging buffers per epilogue warp
    static constexpr int kEpiBytes = 4 * kEpiBufs * 4096;
    static constexpr int kMaxSmem = 232448;
    static constexpr int kFixed = kSA * kABytes + kEpiBytes + 1024 + 512;
    static constexpr int kSXFit = (kMaxSmem - kFixed) / kXBytes;
    static constexpr int kSX = kSXFit > SDVK_GEMM2_X_STAGES ? SDVK_GEMM2_X_STAGES : kSXFit;  // activation tiles
    static constexpr uint32_t kTmemCols = (kAcc * BNX <= 256) ? 256 : 512;
    static constexpr int kOffA = 0;
    static constexpr int kOffX = kOffA + kSA * kABytes;
    static constexpr int kOffEpi = kOffX + kSX * kXBytes;
    static constexpr int kOffBar = kOffEpi + kEpiBytes;
    static constexpr int kNumBars = 2 * kSA + 2 * kSX + 2 * kAcc + 2;
    static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;
    static constexpr int kThreads = 512;
    // dequantiser groups (stages round-robin); bf16's dequantisation goes through fp32 and needs
    // the registers of a two-group split
#ifndef SDVK_GEMM2_DQ_GROUPS
#define SDVK_GEMM2_DQ_GROUPS 4
#endif
    static constexpr int kDqGroups = std::is_same<TA, __nv_bfloat16>::value ? 2 : SDVK_GEMM2_DQ_GROUPS;
    static constexpr int kDqWarps = 8 / kDqGroups;  // warps per group
    static constexpr int kConvThreads = 32 * kDqWarps;
    static constexpr int kChunksPerRow = kBK / 16;
    static constexpr int kTasksPerThread = kBW * kChunksPerRow / kConvThreads;
    static constexpr int kRowStep = kConvThreads / kChunksPerRow;
    static_assert(kSX >= 3 && kSmemBytes <= kMaxSmem, "shared memory");
    static_assert(BNX % 32 == 0 && BNX >= 64 && BNX <= 256, "pair tile N");
    static_assert((kBW * kChunksPerRow) % kConvThreads == 0, "dequant task split");
    // Groups take stages round-robin and stage it uses dequantised slot it % kSA.  With fewer slots than
    // groups a group can reach a slot two phases ahead of the MMA, which a parity wait cannot tell
    // from one phase ahead.
    static_assert(kSA >= kDqGroups, "at least one dequantised-weight slot per dequantiser group");
};

template <class TA, int BNX, bool NN, class TC>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(512, 1)
    gemm_q8_tc2_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmC,
                       const GemmQ8Params p) {
    using Cfg = Gemm2Config<TA, BNX>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem + Cfg::kOffA;  // dequantised weight tiles
    uint8_t* sX = smem + Cfg::kOffX;  // activation tiles
    uint8_t* sEpi = smem + Cfg::kOffEpi;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* a_full = bars;
    uint64_t* a_empty = a_full + Cfg::kSA;
    uint64_t* x_full = a_empty + Cfg::kSA;
    uint64_t* x_empty = x_full + Cfg::kSX;
    uint64_t* acc_full = x_empty + Cfg::kSX;
    uint64_t* acc_empty = acc_full + Cfg::kAcc;
    uint64_t* mma_done = acc_empty + Cfg::kAcc;
    uint64_t* last_ready = mma_done + 1;  // the epilogue warps have seen the last tile's accumulator
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(last_ready + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const uint32_t cid = cluster_id_x(), ncl = nclusters_x();

    if (threadIdx.x == 0) {
        for (int i = 0; i < Cfg::kSA; ++i) {
            mbar_init(&a_full[i], 2 * Cfg::kDqWarps);  // one dequantiser group's warps of both CTAs
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < Cfg::kSX; ++i) {
            mbar_init(&x_full[i], 1);  // the even CTA producer's expect_tx (both CTAs' bytes)
            mbar_init(&x_empty[i], 1);
        }
        for (int i = 0; i < Cfg::kAcc; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 8);
        }
        mbar_init(mma_done, 1);
        mbar_init(last_ready, 4);
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmX);
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
    // Everything above overlaps the previous kernel's tail.  With static weights the dequantisers
    // and the MMA issuer go on at once (they read only the weights and scales); the activation
    // producer and the epilogue, which read and write the previous kernel's data, wait for it to
    // complete, and they alone signal the next kernel's launch.
    const bool early = p.weights_static && (warp == 1 || (warp >= 4 && warp < 12));
    if (!early) {
        grid_dependency_wait();
        grid_launch_dependents();
    }

    bool ok = true;
    auto fail = [&]() {
        atomicOr(p.err, kErrTimeout);
        ok = false;
    };
    // Pair tiles: tiles_w counts 256-row weight tiles (fastest, so the clusters working at one time
    // share activation rows in L2), tiles_x counts BNX-row activation tiles.
    auto decode = [&](uint32_t tile, uint32_t& z, uint32_t& xt, uint32_t& wt) {
        wt = tile % p.tiles_w;
        const uint32_t rest = tile / p.tiles_w;
        xt = rest % p.tiles_x;
        z = rest / p.tiles_x;
    };
    const uint32_t my_tiles = (p.num_tiles > cid) ? (p.num_tiles - cid + ncl - 1) / ncl : 0;
    const uint32_t my_iters = my_tiles * p.k_stages;

    // One 32-column chunk cc of accumulator acc, TMEM lanes 32q..32q+31 (weight rows
    // w0 .. w0 + 31, this thread's row w0 + lane with bias b): TMEM -> registers -> (GEGLU) ->
    // the staging buffer `buf` -> TMA store (or reduce-add).  `release`: hand the accumulator back
    // to the MMA as soon as this chunk's TMEM read has completed.
    auto emit_chunk = [&](uint32_t acc, int q, int cc, uint32_t z, uint32_t xt, int w0, float b, uint8_t* buf,
                          bool release) {
        const int x0 = (int)(xt * Cfg::kBNX) + cc * 32;
        uint32_t raw[32];
        tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * Cfg::kBNX + cc * 32, raw);
        tmem_wait_ld();
        if (release) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(&acc_empty[acc], 0));
        }
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]) + b;
        if (lane == 0) bulk_wait_read<Cfg::kEpiBufs - 1>();  // the store that last used `buf` has read it
        __syncwarp();
        if constexpr (!NN && sizeof(TC) == 2) {
            if (p.geglu) {
                // Lane l < 16 holds a of output column l, lane l + 16 the matching gate: 16
                // outputs a * gelu(gate) per activation row, a [32 x][16] f16 tile.  Each
                // lane computes half of the 32 rows (lanes < 16 rows 0-15, lanes >= 16 rows
                // 16-31), trading the half its partner needs in one shuffle per row pair.
                __half* t = reinterpret_cast<__half*>(buf);
                const bool lo = lane < 16;
                const int o = lane & 15;
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const float mine = lo ? v[j] : v[16 + j];  // a (lo) or gate (hi) of my row
                    const float other = __shfl_xor_sync(0xffffffffu, lo ? v[16 + j] : v[j], 16);
                    const float a = lo ? mine : other, g = lo ? other : mine;
                    t[(lo ? j : 16 + j) * 16 + o] = __float2half_rn(a * gelu_erf_as_fast(g));
                }
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_3d(&tmC, buf, w0 / 2, x0, (int)z);
                    bulk_commit();
                }
                return;
            }
        }
        if constexpr (!NN) store_epi_col<TC>(buf, lane, v);  // [32 x][32 w]
        else store_epi_row<TC>(buf, lane, v);                // [32 w][32 x]
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
    };
    // The last tile's epilogue has nothing left to overlap, so the dequantisers, idle by then, share
    // it: quadrant q's chunks go round-robin to epilogue warp 12 + q (share 0) and dequantiser warps
    // 4 + q, 8 + q (shares 1, 2), which stage through the dequantised-weight ring (free once the
    // last accumulator is complete).
    constexpr int kShares = 3;
    static_assert(Cfg::kSA * Cfg::kABytes >= 8 * Cfg::kEpiBufs * 4096, "helper staging in the weight ring");

    if (warp == 0) {
        // ------------------------------------------------------------ activation TMA producer (both CTAs)
        if (lane == 0) {
            uint32_t sx = 0, px = 0;
            for (uint32_t i = 0; ok && i < my_tiles; ++i) {
                uint32_t z, xt, wt;
                decode(cid + i * ncl, z, xt, wt);
                const int x0 = (int)(xt * Cfg::kBNX + rank * Cfg::kBXC);
                for (uint32_t ks = 0; ks < p.k_stages; ++ks) {
                    const int k0 = (int)(ks * Cfg::kBK);
                    if (!mbar_wait(&x_empty[sx], px ^ 1, p.timeout_ns)) {
                        fail();
                        break;
                    }
                    if (leader) mbar_arrive_expect_tx(&x_full[sx], 2 * Cfg::kBXC * 128);  // both CTAs' bytes
                    const uint32_t full_l = mapa_shared(&x_full[sx], 0);
                    uint8_t* x_dst = sX + sx * Cfg::kXBytes;
                    if (++sx == Cfg::kSX) sx = 0, px ^= 1;
                    if constexpr (!NN) {
                        tma_load_3d_pair(x_dst, &tmX, full_l, k0, x0, (int)z);
                    } else {  // [K][x] activations: kBXC / kBK column blocks of kBK x kBK
#pragma unroll
                        for (int j = 0; j < Cfg::kBXC / Cfg::kBK; ++j)
                            tma_load_3d_pair(x_dst + j * Cfg::kBK * 128, &tmX, full_l, x0 + j * Cfg::kBK, k0, (int)z);
                    }
                }
            }
            // The activation loads are drained by the MMA (it waits for every one it consumes).
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (even CTA)
        // The whole warp runs the loop (warp-uniform control flow and operands, no divisions on
        // the path); one elected lane issues each tcgen05 instruction.  Every cycle this warp
        // spends between MMAs can be tensor-pipe idle time.
        if (leader) {
            constexpr uint32_t idesc =
                make_idesc(OperandTraits<TA>::kFmt, OperandTraits<TA>::kFmt, 0, NN ? 1 : 0, 2 * Cfg::kBW, Cfg::kBNX);
            // Operand descriptors of slot 0; a slot adds its ring's tile size, a K step of kUmmaK elements
            // adds 32 bytes (K-major) or kUmmaK rows of 128 bytes (MN-major activations).
            const uint32_t a0 = smem_u32(sA);
            const uint64_t adesc0 = smem_desc_sw128(a0, 16, 1024);
            const uint32_t b0 = smem_u32(sX);
            uint64_t bdesc0;
            if constexpr (!NN) bdesc0 = smem_desc_sw128(b0, 16, 1024);
            else if constexpr (!OperandTraits<TA>::kTf32) bdesc0 = smem_desc_sw128(b0, Cfg::kBK * 128, 1024);
            else bdesc0 = smem_desc(b0, Cfg::kBK * 128, 512, kLayoutSw128Base32);
            constexpr uint64_t kAStageDesc = Cfg::kABytes >> 4, kXStageDesc = Cfg::kXBytes >> 4;
            constexpr uint64_t kBStep = NN ? (Cfg::kUmmaK * 128) >> 4 : 2;
            uint32_t sa = 0, pa = 0, sx = 0, px = 0;
            for (uint32_t i = 0; ok && i < my_tiles; ++i) {
                const uint32_t acc = i & (Cfg::kAcc - 1), aph = (i / Cfg::kAcc) & 1;
                if (!__all_sync(0xffffffffu, mbar_wait(&acc_empty[acc], aph ^ 1, p.timeout_ns))) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * Cfg::kBNX;
                for (uint32_t ks = 0; ks < p.k_stages; ++ks) {
                    if (!__all_sync(0xffffffffu, mbar_wait(&x_full[sx], px, p.timeout_ns) &&
                                                     mbar_wait(&a_full[sa], pa, p.timeout_ns))) {
                        fail();
                        break;
                    }
                    tc_fence_after();
                    const uint64_t ad = adesc0 + sa * kAStageDesc, bd = bdesc0 + sx * kXStageDesc;
                    if (elect_one()) {
#pragma unroll
                        for (int kk = 0; kk < Cfg::kBK / Cfg::kUmmaK; ++kk) {
                            const uint32_t accum = (ks > 0 || kk > 0) ? 1u : 0u;
                            if constexpr (OperandTraits<TA>::kTf32)
                                mma_tf32_pair(d_tmem, ad + 2 * kk, bd + kk * kBStep, idesc, accum);
                            else mma_f16_pair(d_tmem, ad + 2 * kk, bd + kk * kBStep, idesc, accum);
                        }
                        mma_commit_pair_mc(&x_empty[sx], 0x3);
                        mma_commit_pair_mc(&a_empty[sa], 0x3);
                    }
                    __syncwarp();
                    if (++sx == Cfg::kSX) sx = 0, px ^= 1;
                    if (++sa == Cfg::kSA) sa = 0, pa ^= 1;
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
        constexpr int G = Cfg::kDqGroups;
        const uint32_t grp = (uint32_t)(warp - 4) / Cfg::kDqWarps;  // this group dequantises stages grp, grp+G, ...
        const int ct = (threadIdx.x - 128) % Cfg::kConvThreads;
        const int chunk = ct % Cfg::kChunksPerRow;
        const int row0 = ct / Cfg::kChunksPerRow;
        constexpr int T = Cfg::kTasksPerThread;
        // The raw int8 chunks and their scales come from global memory (L2 hits of far-die data take
        // about a thousand cycles under load) kRing of this group's own stages ahead of use -- G *
        // kRing k-stages, several microseconds at full occupancy -- into a ring of registers
        // indexed by compile-time constants: the loop body is unrolled over the ring, so no
        // instruction (not even a register move) touches a value before its load has had kRing
        // stages to land.  Rows past wrows and chunks past K load as zeros (the TMA's fill).
        constexpr int kRing = Cfg::kRawAhead;
        WeightCursor<T> cur;
        cur.init(&p, cid, ncl, row0, Cfg::kRowStep, Cfg::kBK, chunk * 16, 2 * Cfg::kBW, rank * Cfg::kBW, Cfg::kBW);
        for (uint32_t g = 0; g < grp; ++g) cur.advance();
        auto next_own = [&]() {
#pragma unroll
            for (int g = 0; g < G; ++g) cur.advance();
        };
        float sc[kRing][T];
        uint4 rw[kRing][T];
#pragma unroll
        for (int j = 0; j < kRing; ++j) {
            cur.load<true>(sc[j], rw[j]);
            next_own();
        }
        auto stage = [&](uint32_t it, float(&scale)[T], uint4(&raw)[T]) -> bool {
            const uint32_t sa = it % Cfg::kSA, pa = (it / Cfg::kSA) & 1;
            uint8_t* adst = sA + sa * Cfg::kABytes;
            if (!__all_sync(0xffffffffu, mbar_wait(&a_empty[sa], pa ^ 1, p.timeout_ns))) return false;
#pragma unroll
            for (int t = 0; t < T; ++t) {
                const int r = row0 + t * Cfg::kRowStep;
                dequant16<TA>(raw[t], scale[t], adst + r * 128, r, chunk * Cfg::kES);
            }
            // Only this SM's tensor core reads these rows (operand A of the pair MMA): a CTA-scope
            // proxy fence orders the generic stores before its async-proxy reads.
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(mapa_shared(&a_full[sa], 0));
            cur.load<true>(scale, raw);  // this group's stage it + G * kRing
            next_own();
            return true;
        };
        for (uint32_t it = grp; ok && it < my_iters; it += G * kRing) {
#pragma unroll
            for (int j = 0; j < kRing; ++j) {
                if (it + G * j >= my_iters) break;
                if (!stage(it + G * j, sc[j], rw[j])) {
                    fail();
                    break;
                }
            }
        }
        if (ok && my_tiles > 0) {  // a share of the last tile's epilogue
            const int q = warp & 3, share = 1 + (warp - 4) / 4;
            const uint32_t i = my_tiles - 1, acc = i % Cfg::kAcc;
            uint32_t z, xt, wt;
            decode(cid + i * ncl, z, xt, wt);
            if (!__all_sync(0xffffffffu, mbar_wait(last_ready, 0, p.timeout_ns))) {
                fail();
            } else {
                tc_fence_after();
                grid_dependency_wait();  // stores into C: the previous kernel has completed (a no-op if already waited)
                uint8_t* hbuf = sA + (warp - 4) * (Cfg::kEpiBufs * 4096);
                const int w0 = (int)(wt * 2 * Cfg::kBW + rank * Cfg::kBW) + q * 32;
                const uint32_t n = (uint32_t)w0 + lane;
                const float b = (p.bias && n < p.wrows) ? __ldg(p.bias + z * p.sbias + n) : 0.0f;
                uint32_t nstore = 0;
#pragma unroll 1
                for (int cc = share; cc < Cfg::kBNX / 32; cc += kShares, ++nstore)
                    emit_chunk(acc, q, cc, z, xt, w0, b, hbuf + (nstore % Cfg::kEpiBufs) * 4096, false);
                tc_fence_before();
                if (lane == 0) bulk_wait_all();
            }
        }
    } else if (warp >= 12) {
        // ------------------------------------------------------------ epilogue (both CTAs)
        // Warp q reads TMEM lanes 32q..32q+31: weight rows w = wt*256 + rank*128 + 32q + lane; each
        // 32-column chunk is 32 activation rows.
        const int q = warp & 3;
        uint8_t* ebuf = sEpi + q * (Cfg::kEpiBufs * 4096);
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
            const bool last = i + 1 == my_tiles;
            if (last && lane == 0) mbar_arrive(last_ready);  // the helpers may read this accumulator
            const int w0 = (int)(wt * 2 * Cfg::kBW + rank * Cfg::kBW) + q * 32;  // this warp's first weight row
            const uint32_t n = (uint32_t)w0 + lane;                           // this thread's weight row
            const float b = (p.bias && n < p.wrows) ? __ldg(p.bias + z * p.sbias + n) : 0.0f;
#pragma unroll 1
            for (int cc = 0; cc < Cfg::kBNX / 32; cc += last ? kShares : 1, ++nstore)
                emit_chunk(acc, q, cc, z, xt, w0, b, ebuf + (nstore % Cfg::kEpiBufs) * 4096,
                           !last && cc + 1 == Cfg::kBNX / 32);
        }
        tc_fence_before();  // the TMEM reads before the teardown's deallocation
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
