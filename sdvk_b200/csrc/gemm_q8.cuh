// gemm_q8.cuh -- Q8_0 dequant GEMM on the sm_100a tensor cores (tcgen05 + TMA + TMEM).
//
// One kernel template serves both reference GEMM shapes:
//   NT (gemm_nt_q8_v.comp):  C[M,N]  = A[M,K] . (q[N,K]*s)^T (+bias[N])     activation is K-major
//   NN (gemm_nn_q8_v.comp):  C[M,N]  = (q[M,K]*s) . B[K,N]                  activation is N-major
// In both, the tensor-core "M" side is the activation (x rows: NT tokens M, NN tokens N) and the
// tensor-core "N" side is the weight (w rows: NT out-features N, NN out-channels M).  The TMEM
// accumulator is D[x][w]; the NN epilogue stores it transposed.
//
// Per CTA (persistent, one per SM, 16 warps):
//   warp 0      activation TMA producer (128 x 128B tiles, 128B-swizzled)
//   warp 1      TMEM allocator and the single MMA-issuing thread
//   warp 2      raw int8 weight TMA producer (its own ring, so weights stream ahead of the MMA)
//   warps 4-11  dequantisers: int8 smem tile * per-32-block scale -> f16/bf16/f32 operand tile in
//               the 128B-swizzled K-major layout the tensor core reads
//   warps 12-15 epilogue: TMEM -> registers (+bias) -> swizzled smem -> TMA store / TMA reduce-add
// Rings: 4 activation stages, 4 raw-weight stages, 2 dequantised-weight stages, 2 TMEM accumulators, so
// loads, dequantisation, MMA and the previous tile's epilogue all overlap.
//
// Every mbarrier wait is bounded (GemmQ8Params::timeout_ns): a wait that runs out records
// kErrTimeout in *err, the CTA drains its in-flight copies and MMAs, frees TMEM and returns.
#pragma once

#include "ptx.cuh"

namespace sdvk {

struct GemmQ8Params {
    const int8_t* wq;       // weight payload, element (row, k) of batch z at wq[z*sW + row*ldw + k]
    const float* ws;        // fp32 scale per 32 payload elements (flat index >> 5)
    const float* bias;      // per weight row (NT: per output column, NN: per output row), or null
    uint64_t sbias;         // bias batch stride in elements (0: one bias for all batches)
    uint32_t xrows;         // activation rows (tensor-core M extent)
    uint32_t wrows;         // weight rows (tensor-core N extent)
    uint32_t K;
    uint32_t batch;
    uint64_t ldw;           // weight row stride in elements (multiple of 32)
    uint64_t sW;            // weight batch stride in elements (0: one weight for all batches)
    uint32_t tiles_x, tiles_w, num_tiles, k_stages;
    uint32_t accumulate;    // 0: C = result, 1: C += result (TMA reduce-add)
    uint32_t* err;          // device error word
    uint64_t timeout_ns;
    void* c;                // output (direct-store epilogue): NT C[z][x][w], NN C[z][w][x]
    uint64_t ldc, sc;       // output row and batch strides (elements)
    uint32_t weights_static;  // the weights and scales are parameters no kernel writes while this GEMM
                              // may run early: the weight roles read them before griddepcontrol.wait
    uint32_t geglu;         // NT only: the weight rows are GEGLU-interleaved (see gemm_q8_geglu), and
                            // each 32-column chunk [a(16) | gate(16)] is stored as 16 a * gelu(gate)
};

// erf-GELU with the Abramowitz & Stegun 7.1.26 erf (|error| <= 1.5e-7), the reference's formula
// (unary_fwd.comp:29-35).
__device__ __forceinline__ float gelu_erf_as(float v) {
    const float xs = v * 0.70710678118654752440f;
    const float ax = fabsf(xs);
    const float t = 1.0f / (1.0f + 0.3275911f * ax);
    const float poly =
        ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
    const float e = 1.0f - poly * expf(-ax * ax);
    return 0.5f * v * (1.0f + (xs >= 0.0f ? e : -e));
}

// The same formula with the reciprocal and the exponential as single approximate hardware ops
// (rcp.approx, ex2.approx: a few ulp of fp32), for the GEMM epilogue, whose instruction count shares
// issue slots with the mainloop's warps; the result is stored in f16.
__device__ __forceinline__ float gelu_erf_as_fast(float v) {
    const float xs = v * 0.70710678118654752440f;
    const float ax = fabsf(xs);
    float t;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.3275911f, ax, 1.0f)));
    const float poly =
        ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
    float ex;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(ex) : "f"(-ax * ax * 1.4426950408889634f));
    const float e = 1.0f - poly * ex;
    return 0.5f * v * (1.0f + copysignf(e, xs));
}

template <class TA>
struct OperandTraits;
template <>
struct OperandTraits<__half> {
    static constexpr uint32_t kFmt = 0;  // f16
    static constexpr bool kTf32 = false;
};
template <>
struct OperandTraits<__nv_bfloat16> {
    static constexpr uint32_t kFmt = 1;  // bf16
    static constexpr bool kTf32 = false;
};
template <>
struct OperandTraits<float> {
    static constexpr uint32_t kFmt = 2;  // tf32
    static constexpr bool kTf32 = true;
};

template <class TA, int BN>
struct GemmQ8Config {
    static constexpr int kBM = 128;
    static constexpr int kES = sizeof(TA);
    static constexpr int kBK = 128 / kES;            // K elements per 128-byte swizzle row
    static constexpr int kUmmaK = 32 / kES;          // K per tcgen05.mma (32 bytes)
    static constexpr int kStages = 4;
    static constexpr int kBStages = 2;
    static constexpr int kAcc = 2;
    static constexpr int kABytes = kBM * 128;        // activation stage
    static constexpr int kWBytes = BN * kBK;         // raw int8 stage
    static constexpr int kBBytes = BN * 128;         // dequantised stage
    static constexpr int kEpiBytes = 4 * 2 * 32 * 32 * 4;  // 4 warps x 2 buffers x 32x32 fp32
    static constexpr uint32_t kTmemCols = (kAcc * BN <= 32) ? 32 : (kAcc * BN <= 64) ? 64 : (kAcc * BN <= 128) ? 128 : (kAcc * BN <= 256) ? 256 : 512;
    static constexpr int kOffA = 0;
    static constexpr int kOffB = kOffA + kStages * kABytes;
    static constexpr int kOffW = kOffB + kBStages * kBBytes;
    static constexpr int kOffEpi = kOffW + kStages * kWBytes;
    static constexpr int kOffBar = kOffEpi + kEpiBytes;
    static constexpr int kNumBars = 4 * kStages + 2 * kBStages + 2 * kAcc + 1;
    static constexpr int kSmemBytes = kOffBar + kNumBars * 8 + 16 + 1024;  // +1024: manual alignment
    static constexpr int kThreads = 512;
    static constexpr int kConvThreads = 256;
    static constexpr int kChunksPerRow = kBK / 16;  // 16 int8 per dequant task
    static constexpr int kTasksPerThread = BN * kChunksPerRow / kConvThreads;
    static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN");
    static_assert(kAcc * BN <= 512, "TMEM");
    static_assert(kSmemBytes <= 232448, "shared memory");
    static_assert((BN * kChunksPerRow) % kConvThreads == 0, "dequant task split");
};

// Dequantise 16 int8 (one uint4) with one scale into 16 operand elements written as 16-byte
// chunks `chunk0 .. chunk0+n-1` of a 128-byte swizzled row at `row_base` (row index r).
template <class TA>
__device__ __forceinline__ void dequant16(const uint4 raw, float scale, uint8_t* row_base, int r, int chunk0);

template <>
__device__ __forceinline__ void dequant16<__half>(const uint4 raw, float scale, uint8_t* row_base, int r, int chunk0) {
    // int8 -> fp16 exactly: byte^0x80 is v+128; placing it under exponent 0x64 gives the half
    // 1024+v+128; subtracting 1152 leaves v.  One hmul2 then rounds v*s to fp16 once.
    const __half2 s2 = __float2half2_rn(scale);
    const __half2 bias = __float2half2_rn(1152.0f);
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t x = w[i] ^ 0x80808080u;
        uint32_t lo = __byte_perm(x, 0x64646464u, 0x4140u);
        uint32_t hi = __byte_perm(x, 0x64646464u, 0x4342u);
        __half2 l2 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&lo), bias), s2);
        __half2 h2 = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&hi), bias), s2);
        o[2 * i] = *reinterpret_cast<uint32_t*>(&l2);
        o[2 * i + 1] = *reinterpret_cast<uint32_t*>(&h2);
    }
    const int sw = r & 7;
    *reinterpret_cast<uint4*>(row_base + (((chunk0 + 0) ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(row_base + (((chunk0 + 1) ^ sw) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
}

__device__ __forceinline__ void int8x4_to_f32(uint32_t w, float (&f)[4]) {
    // byte^0x80 placed in the low mantissa byte of 2^23 gives 2^23 + v + 128 exactly.
    const uint32_t x = w ^ 0x80808080u;
    f[0] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7440u)) - 8388736.0f;
    f[1] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7441u)) - 8388736.0f;
    f[2] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7442u)) - 8388736.0f;
    f[3] = __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7443u)) - 8388736.0f;
}

template <>
__device__ __forceinline__ void dequant16<__nv_bfloat16>(const uint4 raw, float scale, uint8_t* row_base, int r,
                                                         int chunk0) {
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float f[4];
        int8x4_to_f32(w[i], f);
        __nv_bfloat162 a = __floats2bfloat162_rn(f[0] * scale, f[1] * scale);
        __nv_bfloat162 b = __floats2bfloat162_rn(f[2] * scale, f[3] * scale);
        o[2 * i] = *reinterpret_cast<uint32_t*>(&a);
        o[2 * i + 1] = *reinterpret_cast<uint32_t*>(&b);
    }
    const int sw = r & 7;
    *reinterpret_cast<uint4*>(row_base + (((chunk0 + 0) ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4*>(row_base + (((chunk0 + 1) ^ sw) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
}

__device__ __forceinline__ uint32_t round_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

template <>
__device__ __forceinline__ void dequant16<float>(const uint4 raw, float scale, uint8_t* row_base, int r, int chunk0) {
    // float(int8) * scale in fp32 (the reference's own dequantisation), then rounded to tf32.
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    const int sw = r & 7;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float f[4];
        int8x4_to_f32(w[i], f);
        *reinterpret_cast<uint4*>(row_base + (((chunk0 + i) ^ sw) << 4)) =
            make_uint4(round_tf32(f[0] * scale), round_tf32(f[1] * scale), round_tf32(f[2] * scale),
                       round_tf32(f[3] * scale));
    }
}

// Walks a CTA's (tile, k-stage) sequence in order and fetches, for each stage, what a
// dequantising thread needs: for T weight rows (row0 + t*row_step of the tile's weight window),
// the scale of the 32-block holding K column k_off of the stage and, optionally, the 16 int8 at
// that column.  One tile decode per tile, no division per stage.
template <int T>
struct WeightCursor {
    const GemmQ8Params* p;
    uint32_t tile, tile_step, ks;
    uint32_t n0;          // first weight row of this thread in the current tile
    const float* ws;      // scale base of the current tile's batch
    const int8_t* wq;     // payload base of the current tile's batch
    bool valid;
    int row_step, bk, k_off, rows_per_tile;
    uint32_t tiles_x;
    uint32_t w_window;
    int row0, rows_mine;  // this thread's first row within the CTA's window, and the window size

    __device__ void set_tile() {
        valid = tile < p->num_tiles;
        if (!valid) return;
        const uint32_t wt = tile % p->tiles_w;
        const uint32_t rest = tile / p->tiles_w;
        const uint32_t z = rest / tiles_x;
        n0 = wt * rows_per_tile + w_window;
        ws = p->ws + (p->sW ? (uint64_t)z * (p->sW / 32) : 0);
        wq = p->wq + (p->sW ? (uint64_t)z * p->sW : 0);
        ks = 0;
    }
    __device__ void init(const GemmQ8Params* params, uint32_t first_tile, uint32_t step, int row0_, int rstep, int bk_,
                         int koff, int rows_tile, uint32_t window, int rows_window) {
        p = params;
        row0 = row0_;
        rows_mine = rows_window;
        tile = first_tile;
        tile_step = step;
        row_step = rstep;
        bk = bk_;
        k_off = koff;
        rows_per_tile = rows_tile;
        tiles_x = params->tiles_x;
        w_window = window + row0_;
        set_tile();
    }
    template <bool kWithRaw>
    __device__ void load(float (&sc)[T], uint4 (&raw)[T]) const {
#pragma unroll
        for (int t = 0; t < T; ++t) {
            sc[t] = 0.0f;
            if (kWithRaw) raw[t] = make_uint4(0, 0, 0, 0);
        }
        if (!valid) return;
        const uint32_t k = ks * bk + k_off;
        if (k >= p->K) return;  // K is a multiple of 32: a 16-column chunk is wholly in or out
        const uint32_t kb = k >> 5;
        const uint64_t ldb = p->ldw >> 5;
#pragma unroll
        for (int t = 0; t < T; ++t) {
            const uint32_t n = n0 + t * row_step;
            if (n < p->wrows && row0 + t * row_step < rows_mine) {
                sc[t] = __ldg(ws + (uint64_t)n * ldb + kb);
                if (kWithRaw) raw[t] = __ldg(reinterpret_cast<const uint4*>(wq + (uint64_t)n * p->ldw + k));
            }
        }
    }
    __device__ void advance() {
        if (!valid) return;
        if (++ks == p->k_stages) {
            tile += tile_step;
            set_tile();
        }
    }
};

// Direct epilogue store of one 32-column accumulator block: this thread holds activation row x
// and weight columns w0..w0+31 in v.  NT writes C[z][x][w] (128 contiguous bytes per thread, fp32);
// NN writes C[z][w][x] (consecutive lanes hold consecutive x, so every store is coalesced).
template <class TC, bool NN>
__device__ __forceinline__ void store_direct(const GemmQ8Params& p, uint32_t z, uint32_t x, uint32_t w0,
                                             const float (&v)[32]) {
    if (x >= p.xrows) return;
    TC* C = reinterpret_cast<TC*>(p.c) + (uint64_t)z * p.sc;
    if constexpr (NN) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            if (w0 + j < p.wrows) {
                TC* dst = C + (uint64_t)(w0 + j) * p.ldc + x;
                if constexpr (sizeof(TC) == 4) *dst = p.accumulate ? *dst + v[j] : v[j];
                else *dst = __float2half_rn(v[j]);
            }
        }
    } else {
        TC* row = C + (uint64_t)x * p.ldc + w0;
        if constexpr (sizeof(TC) == 4) {
#pragma unroll
            for (int c4 = 0; c4 < 8; ++c4) {
                float4 o = make_float4(v[4 * c4], v[4 * c4 + 1], v[4 * c4 + 2], v[4 * c4 + 3]);
                if (w0 + 4 * c4 + 3 < p.wrows) {
                    float4* dst = reinterpret_cast<float4*>(row + 4 * c4);
                    if (p.accumulate) {
                        const float4 old = *dst;
                        o.x += old.x, o.y += old.y, o.z += old.z, o.w += old.w;
                    }
                    *dst = o;
                } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        if (w0 + 4 * c4 + e < p.wrows) row[4 * c4 + e] = p.accumulate ? row[4 * c4 + e] + v[4 * c4 + e] : v[4 * c4 + e];
                }
            }
        } else {
#pragma unroll
            for (int c8 = 0; c8 < 4; ++c8) {
                if (w0 + 8 * c8 + 7 < p.wrows) {
                    __half2 h0 = __floats2half2_rn(v[8 * c8 + 0], v[8 * c8 + 1]);
                    __half2 h1 = __floats2half2_rn(v[8 * c8 + 2], v[8 * c8 + 3]);
                    __half2 h2 = __floats2half2_rn(v[8 * c8 + 4], v[8 * c8 + 5]);
                    __half2 h3 = __floats2half2_rn(v[8 * c8 + 6], v[8 * c8 + 7]);
                    *reinterpret_cast<uint4*>(row + 8 * c8) =
                        make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                                   *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (w0 + 8 * c8 + e < p.wrows) row[8 * c8 + e] = __float2half_rn(v[8 * c8 + e]);
                }
            }
        }
    }
}

template <class TC>
__device__ __forceinline__ void store_epi_row(uint8_t* buf, int lane, const float (&v)[32]);

template <>
__device__ __forceinline__ void store_epi_row<float>(uint8_t* buf, int lane, const float (&v)[32]) {
    // 32 fp32 = one 128-byte row, 128B-swizzled (matches the store tensor map).
    uint8_t* row = buf + lane * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c)
        *reinterpret_cast<float4*>(row + ((c ^ (lane & 7)) << 4)) =
            make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}
template <>
__device__ __forceinline__ void store_epi_row<__half>(uint8_t* buf, int lane, const float (&v)[32]) {
    // 32 fp16 = one 64-byte row, 64B-swizzled.
    uint8_t* row = buf + lane * 64;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        __half2 h0 = __floats2half2_rn(v[8 * c + 0], v[8 * c + 1]);
        __half2 h1 = __floats2half2_rn(v[8 * c + 2], v[8 * c + 3]);
        __half2 h2 = __floats2half2_rn(v[8 * c + 4], v[8 * c + 5]);
        __half2 h3 = __floats2half2_rn(v[8 * c + 6], v[8 * c + 7]);
        *reinterpret_cast<uint4*>(row + ((c ^ ((lane >> 1) & 3)) << 4)) =
            make_uint4(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1),
                       *reinterpret_cast<uint32_t*>(&h2), *reinterpret_cast<uint32_t*>(&h3));
    }
}
// Transposed tile for the NN store: element (w = j, x = lane) of a [32 w][32 x] row-major tile.
template <class TC>
__device__ __forceinline__ void store_epi_col(uint8_t* buf, int lane, const float (&v)[32]) {
    TC* t = reinterpret_cast<TC*>(buf);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        if constexpr (sizeof(TC) == 4) t[j * 32 + lane] = v[j];
        else t[j * 32 + lane] = __float2half_rn(v[j]);
    }
}

template <class TA, int BN, bool NN, class TC>
__global__ void __launch_bounds__(512, 1)
    gemm_q8_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW,
                      const __grid_constant__ CUtensorMap tmC, const GemmQ8Params p) {
    using Cfg = GemmQ8Config<TA, BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem + Cfg::kOffA;
    uint8_t* sB = smem + Cfg::kOffB;
    uint8_t* sW = smem + Cfg::kOffW;
    uint8_t* sEpi = smem + Cfg::kOffEpi;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kOffBar);
    uint64_t* a_full = bars;                                 // [kStages] activation TMA tx
    uint64_t* a_empty = a_full + Cfg::kStages;               // [kStages] MMA commit
    uint64_t* w_full = a_empty + Cfg::kStages;               // [kStages] raw weight TMA tx
    uint64_t* w_empty = w_full + Cfg::kStages;               // [kStages] 8 dequant warps
    uint64_t* b_full = w_empty + Cfg::kStages;               // [kBStages] 8 dequant warps
    uint64_t* b_empty = b_full + Cfg::kBStages;              // [kBStages] MMA commit
    uint64_t* acc_full = b_empty + Cfg::kBStages;            // [kAcc] MMA commit
    uint64_t* acc_empty = acc_full + Cfg::kAcc;              // [kAcc] 4 epilogue warps
    uint64_t* mma_done = acc_empty + Cfg::kAcc;              // final drain
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < Cfg::kStages; ++i) {
            mbar_init(&a_full[i], 1);
            mbar_init(&a_empty[i], 1);
            mbar_init(&w_full[i], 1);
            mbar_init(&w_empty[i], 8);
        }
        for (int i = 0; i < Cfg::kBStages; ++i) {
            mbar_init(&b_full[i], 8);
            mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < Cfg::kAcc; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 4);
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
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 3) return;  // spare warp takes no part in the pipeline

    bool ok = true;
    auto fail = [&]() {
        atomicOr(p.err, kErrTimeout);
        ok = false;
    };
    auto decode = [&](uint32_t tile, uint32_t& z, uint32_t& xt, uint32_t& wt) {
        wt = tile % p.tiles_w;
        const uint32_t rest = tile / p.tiles_w;
        xt = rest % p.tiles_x;
        z = rest / p.tiles_x;
    };

    if (warp == 0) {
        // ------------------------------------------------------------ activation TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            for (uint32_t tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
                uint32_t z, xt, wt;
                decode(tile, z, xt, wt);
                for (uint32_t ks = 0; ks < p.k_stages; ++ks, ++it) {
                    const uint32_t slot = it % Cfg::kStages, ph = (it / Cfg::kStages) & 1;
                    if (!mbar_wait(&a_empty[slot], ph ^ 1, p.timeout_ns)) {
                        fail();
                        break;
                    }
                    mbar_arrive_expect_tx(&a_full[slot], Cfg::kABytes);
                    const int k0 = (int)(ks * Cfg::kBK);
                    uint8_t* a_dst = sA + slot * Cfg::kABytes;
                    if constexpr (!NN) {
                        tma_load_3d(a_dst, &tmA, &a_full[slot], k0, (int)(xt * Cfg::kBM), (int)z);
                    } else {
                        // N-major activation: kBM/kBK boxes of [kBK k-rows][kBK x-elements].
#pragma unroll
                        for (int j = 0; j < Cfg::kBM / Cfg::kBK; ++j)
                            tma_load_3d(a_dst + j * Cfg::kBK * 128, &tmA, &a_full[slot],
                                        (int)(xt * Cfg::kBM) + j * Cfg::kBK, k0, (int)z);
                    }
                }
            }
            // The activation loads are drained by the MMA (it waits for every one it consumes).
        }
    } else if (warp == 2) {
        // ------------------------------------------------------------ weight TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            for (uint32_t tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x) {
                uint32_t z, xt, wt;
                decode(tile, z, xt, wt);
                const int zw = p.sW ? (int)z : 0;
                for (uint32_t ks = 0; ks < p.k_stages; ++ks, ++it) {
                    const uint32_t slot = it % Cfg::kStages, ph = (it / Cfg::kStages) & 1;
                    if (!mbar_wait(&w_empty[slot], ph ^ 1, p.timeout_ns)) {
                        fail();
                        break;
                    }
                    mbar_arrive_expect_tx(&w_full[slot], Cfg::kWBytes);
                    tma_load_3d(sW + slot * Cfg::kWBytes, &tmW, &w_full[slot], (int)(ks * Cfg::kBK), (int)(wt * BN),
                                zw);
                }
            }
            // Drain: no raw-weight load may still be landing in shared memory at exit.
            for (uint32_t i = (it > Cfg::kStages ? it - Cfg::kStages : 0); i < it; ++i)
                if (!mbar_wait(&w_full[i % Cfg::kStages], (i / Cfg::kStages) & 1, p.timeout_ns)) fail();
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = make_idesc(OperandTraits<TA>::kFmt, OperandTraits<TA>::kFmt, NN ? 1 : 0, 0,
                                                  Cfg::kBM, BN);
            uint32_t it = 0, bit = 0, tcount = 0;
            for (uint32_t tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++tcount) {
                const uint32_t acc = tcount % Cfg::kAcc, aph = (tcount / Cfg::kAcc) & 1;
                if (!mbar_wait(&acc_empty[acc], aph ^ 1, p.timeout_ns)) {
                    fail();
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (uint32_t ks = 0; ks < p.k_stages; ++ks, ++it, ++bit) {
                    const uint32_t slot = it % Cfg::kStages, ph = (it / Cfg::kStages) & 1;
                    const uint32_t bslot = bit % Cfg::kBStages, bph = (bit / Cfg::kBStages) & 1;
                    if (!mbar_wait(&a_full[slot], ph, p.timeout_ns) ||
                        !mbar_wait(&b_full[bslot], bph, p.timeout_ns)) {
                        fail();
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(sA + slot * Cfg::kABytes);
                    const uint32_t b_addr = smem_u32(sB + bslot * Cfg::kBBytes);
#pragma unroll
                    for (int kk = 0; kk < Cfg::kBK / Cfg::kUmmaK; ++kk) {
                        uint64_t adesc;
                        if constexpr (!NN)
                            adesc = smem_desc_sw128(a_addr + kk * 32, 16, 1024);
                        else if constexpr (!OperandTraits<TA>::kTf32)
                            // MN-major: k advances by kUmmaK rows of 128 B; x chunks kBK*128 B apart
                            adesc = smem_desc_sw128(a_addr + kk * Cfg::kUmmaK * 128, Cfg::kBK * 128, 1024);
                        else  // MN-major tf32 needs 32-byte swizzle atoms: 4-row K groups (512 B)
                            adesc = smem_desc(a_addr + kk * Cfg::kUmmaK * 128, Cfg::kBK * 128, 512,
                                              kLayoutSw128Base32);
                        const uint64_t bdesc = smem_desc_sw128(b_addr + kk * 32, 16, 1024);
                        const uint32_t accum = (ks > 0 || kk > 0) ? 1u : 0u;
                        if constexpr (OperandTraits<TA>::kTf32) mma_tf32(d_tmem, adesc, bdesc, idesc, accum);
                        else mma_f16(d_tmem, adesc, bdesc, idesc, accum);
                    }
                    mma_commit(&a_empty[slot]);
                    mma_commit(&b_empty[bslot]);
                }
                if (!ok) break;
                mma_commit(&acc_full[acc]);
            }
            // Drain: every MMA issued by this thread completes before TMEM is released.
            mma_commit(mma_done);
            if (!mbar_wait(mma_done, 0, p.timeout_ns)) fail();
        }
    } else if (warp >= 4 && warp < 12) {
        // ------------------------------------------------------------ dequantisers
        const int ct = threadIdx.x - 128;
        const int chunk = ct % Cfg::kChunksPerRow;
        const int row0 = ct / Cfg::kChunksPerRow;
        constexpr int kRowStep = Cfg::kConvThreads / Cfg::kChunksPerRow;
        constexpr int T = Cfg::kTasksPerThread;
        const uint32_t my_tiles = (p.num_tiles > blockIdx.x) ? (p.num_tiles - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
        const uint32_t my_iters = my_tiles * p.k_stages;
        // Scales come from L2 kRing stages ahead of use, into a ring of registers indexed by
        // compile-time constants (the loop body is unrolled over the ring), so no instruction touches
        // a scale before its load has had kRing stages to land.
        constexpr int kRing = 4;
        WeightCursor<T> cur;
        cur.init(&p, blockIdx.x, gridDim.x, row0, kRowStep, Cfg::kBK, chunk * 16, BN, 0, BN);
        float sc[kRing][T];
        uint4 unused[T];
#pragma unroll
        for (int j = 0; j < kRing; ++j) {
            cur.load<false>(sc[j], unused);
            cur.advance();
        }
        auto stage = [&](uint32_t it, float(&scale)[T]) -> bool {
            const uint32_t slot = it % Cfg::kStages, ph = (it / Cfg::kStages) & 1;
            const uint32_t bslot = it % Cfg::kBStages, bph = (it / Cfg::kBStages) & 1;
            const bool got =
                mbar_wait(&w_full[slot], ph, p.timeout_ns) && mbar_wait(&b_empty[bslot], bph ^ 1, p.timeout_ns);
            if (!__all_sync(0xffffffffu, got)) return false;  // the warp leaves the loop together
            const uint8_t* wsrc = sW + slot * Cfg::kWBytes;
            uint8_t* bdst = sB + bslot * Cfg::kBBytes;
            uint4 raw[T];
#pragma unroll
            for (int t = 0; t < T; ++t)
                raw[t] = *reinterpret_cast<const uint4*>(wsrc + (row0 + t * kRowStep) * Cfg::kBK + chunk * 16);
#pragma unroll
            for (int t = 0; t < T; ++t) {
                const int r = row0 + t * kRowStep;
                dequant16<TA>(raw[t], scale[t], bdst + r * 128, r, chunk * Cfg::kES);  // 16 elements = kES chunks
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&w_empty[slot]);
                mbar_arrive(&b_full[bslot]);
            }
            cur.load<false>(scale, unused);  // the scales of stage it + kRing
            cur.advance();
            return true;
        };
        for (uint32_t it = 0; ok && it < my_iters; it += kRing) {
#pragma unroll
            for (int j = 0; j < kRing; ++j) {
                if (it + j >= my_iters) break;
                if (!stage(it + j, sc[j])) {
                    fail();
                    break;
                }
            }
        }
    } else if (warp >= 12) {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;  // TMEM lane quarter this warp may read
        uint8_t* ebuf = sEpi + q * (2 * 4096);
        uint32_t tcount = 0, nstore = 0;
        for (uint32_t tile = blockIdx.x; ok && tile < p.num_tiles; tile += gridDim.x, ++tcount) {
            uint32_t z, xt, wt;
            decode(tile, z, xt, wt);
            const uint32_t acc = tcount % Cfg::kAcc, aph = (tcount / Cfg::kAcc) & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[acc], aph, p.timeout_ns))) {
                fail();
                break;
            }
            tc_fence_after();
            const int x0 = (int)(xt * Cfg::kBM) + q * 32;
#pragma unroll 1
            for (int cc = 0; cc < BN / 32; ++cc, ++nstore) {
                const int w0 = (int)(wt * BN) + cc * 32;
                uint32_t raw[32];
                tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN + cc * 32, raw);
                tmem_wait_ld();
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]);
                if (p.bias) {
                    const float* bz = p.bias + z * p.sbias;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const uint32_t n = (uint32_t)w0 + j;
                        v[j] += (n < p.wrows) ? __ldg(bz + n) : 0.0f;
                    }
                }
                uint8_t* buf = ebuf + (nstore & 1) * 4096;
                if (lane == 0) bulk_wait_read<1>();  // the store that last used `buf` has read it
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
            if (lane == 0) mbar_arrive(&acc_empty[acc]);
        }
        if (lane == 0) bulk_wait_all();
    }

    // ---------------------------------------------------------------- teardown
    __syncwarp();  // lanes that skipped a single-thread role wait for it here
    asm volatile("barrier.sync 1, 480;" ::: "memory");  // warps 0-2, 4-15 (3 left early)
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, Cfg::kTmemCols);
    }
}

}  // namespace sdvk
