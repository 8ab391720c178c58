// attention.cuh -- fused flash attention, O = softmax(Q K^T * scale) V per (batch, head), without
// materialising the Tq x Tk scores.  Serves both reference kernels (fused_attn_tiled.comp for
// self-attention, fused_attn.comp for the 77-token cross-attention) with one kernel.
//
// CTA = 8 warps x 16 queries = 128 queries of one (batch, head); K/V stream through shared memory
// in 64-key tiles (double-buffered cp.async).  Per warp: S = Q.K^T (m16n8k16, fp32 accumulate),
// mask, online softmax in the exp2 domain, P (f16/bf16) . V accumulated in fp32 registers,
// output normalised by 1/l (0 when a row saw no key, as the reference does).
// Head dims up to 64 are supported; smaller head dims are zero-padded to 64 in shared memory.
#pragma once

#include "ptx.cuh"

namespace sdvk {

struct AttnParams {
    const void* q;
    const void* k;
    const void* v;
    void* o;
    uint32_t batch, heads, Tq, Tk, hd;
    uint64_t ldq, ldk, ldv, ldo;  // row (token) strides, elements
    uint64_t sq, sk, sv, so;      // batch strides, elements
    uint64_t hq, hk, hv, ho;      // head strides, elements
    float scale_log2;             // softmax scale * log2(e)
    uint32_t causal;
};

constexpr int kAttnBM = 128;
constexpr int kAttnBN = 64;
constexpr int kAttnHD = 64;
constexpr int kAttnThreads = 256;
constexpr int kAttnShortThreads = 128;  // attn_short_kernel: 4 warps x 2 slabs of 16 queries
constexpr int kAttnSmem = (kAttnBM + 4 * kAttnBN) * kAttnHD * 2;  // Q + 2x(K,V), 16-bit

template <class T>
struct Half16;
template <>
struct Half16<__half> {
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};
template <>
struct Half16<__nv_bfloat16> {
    static __device__ __forceinline__ uint32_t pack(float a, float b) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
    static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
};

// Compute type: fp32 inputs are computed in f16 operands (fp32 accumulation).
template <class TIn>
struct AttnCompute {
    using T = TIn;
};
template <>
struct AttnCompute<float> {
    using T = __half;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Byte offset of 16-byte chunk c of row r in a [rows][64] 16-bit tile (128-byte rows, XOR swizzle).
__device__ __forceinline__ uint32_t tile_off(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// Stage rows [r0, r0+R) x head dims [0, 64) of one head into a swizzled tile.  16-bit inputs with
// 16-byte aligned rows use cp.async (zero-fill outside the tensor); other inputs are loaded,
// converted and stored through registers.
template <class TIn, class TC, int R, bool kAsync, int kThreads = kAttnThreads>
__device__ __forceinline__ void attn_load_tile(uint8_t* tile, const TIn* base, uint64_t ld, uint32_t r0, uint32_t T,
                                               uint32_t hd) {
    constexpr int kTasks = R * 8;
#pragma unroll
    for (int t = threadIdx.x; t < kTasks; t += kThreads) {
        const int r = t >> 3, c = t & 7;
        const uint32_t row = r0 + r;
        const bool row_ok = row < T;
        const uint32_t dst = smem_u32(tile) + tile_off(r, c);
        if constexpr (kAsync) {
            const bool ok = row_ok && (uint32_t)(c * 8) < hd;
            const TIn* src = ok ? base + (uint64_t)row * ld + c * 8 : base;
            cp_async16(dst, src, ok);
        } else {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const uint32_t d = c * 8 + e;
                f[e] = (row_ok && d < hd) ? (float)base[(uint64_t)row * ld + d] : 0.0f;
            }
            uint4 u = make_uint4(Half16<TC>::pack(f[0], f[1]), Half16<TC>::pack(f[2], f[3]),
                                 Half16<TC>::pack(f[4], f[5]), Half16<TC>::pack(f[6], f[7]));
            asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(u.x), "r"(u.y), "r"(u.z), "r"(u.w)
                         : "memory");
        }
    }
}

// One 64-key tile for one warp's 16-query slab: S = Q K^T (m16n8k16, fp32), scale and mask, online
// softmax in the exp2 domain (rows g and g+8 of the slab per lane), O += P V.  q_slab is the slab's
// first query row (for the causal mask), kv0 the tile's first key.  MMAs over 16-key groups wholly
// past the last key are skipped (their scores are masked and their P is 0, so this is exact): the
// 77-token cross-attention's second tile holds 13 keys.
template <class TC>
__device__ __forceinline__ void attn_tile(const AttnParams& p, uint32_t kbase, uint32_t vbase, uint32_t kv0,
                                          uint32_t q_slab, const uint32_t (&qf)[4][4], float (&o_acc)[8][4],
                                          float (&m_run)[2], float (&l_run)[2], int lane) {
    const int g = lane >> 2, t = lane & 3;
    const uint32_t kv_n = p.Tk > kv0 ? p.Tk - kv0 : 0;  // keys of this tile that exist (may exceed 64)
    // ---- S = Q K^T : 16 x 64 per warp
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) s[i][j] = 0.0f;
#pragma unroll
    for (int kb = 0; kb < 4; ++kb) {
#pragma unroll
        for (int np = 0; np < 4; ++np) {  // pairs of 8-key n-tiles
            if ((uint32_t)np * 16 >= kv_n) continue;
            const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
            const int c = kb * 2 + ((lane >> 3) & 1);
            uint32_t b0, b1, b2, b3;
            ldsm_x4(kbase + tile_off(key, c), b0, b1, b2, b3);
            Half16<TC>::mma(s[2 * np], qf[kb], b0, b1);
            Half16<TC>::mma(s[2 * np + 1], qf[kb], b2, b3);
        }
    }
    // ---- mask + online softmax (rows g and g+8 of the warp slab)
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const uint32_t key = kv0 + nt * 8 + 2 * t + (e & 1);
            const uint32_t qrow = q_slab + g + ((e >> 1) << 3);
            float v = s[nt][e] * p.scale_log2;
            if (key >= p.Tk || (p.causal && key > qrow)) v = -INFINITY;
            s[nt][e] = v;
            mx[e >> 1] = fmaxf(mx[e >> 1], v);
        }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
        mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        const float m_new = fmaxf(m_run[r], mx[r]);
        const float m_use = (m_new == -INFINITY) ? 0.0f : m_new;
        corr[r] = exp2f(m_run[r] - m_use);
        m_run[r] = m_new;
        l_run[r] *= corr[r];
        mx[r] = m_use;
    }
    float rs[2] = {0.0f, 0.0f};
    uint32_t pf[4][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
        const float p0 = exp2f(s[nt][0] - mx[0]), p1 = exp2f(s[nt][1] - mx[0]);
        const float p2 = exp2f(s[nt][2] - mx[1]), p3 = exp2f(s[nt][3] - mx[1]);
        rs[0] += p0 + p1;
        rs[1] += p2 + p3;
        const int kb = nt >> 1, hi = nt & 1;
        pf[kb][hi * 2 + 0] = Half16<TC>::pack(p0, p1);
        pf[kb][hi * 2 + 1] = Half16<TC>::pack(p2, p3);
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
        rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
        l_run[r] += rs[r];
    }
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
        o_acc[dt][0] *= corr[0];
        o_acc[dt][1] *= corr[0];
        o_acc[dt][2] *= corr[1];
        o_acc[dt][3] *= corr[1];
    }
    // ---- O += P V : P as A fragments (k = keys), V via transposed ldmatrix
#pragma unroll
    for (int kb = 0; kb < 4; ++kb) {
        if ((uint32_t)kb * 16 >= kv_n) continue;
        const uint32_t a[4] = {pf[kb][0], pf[kb][1], pf[kb][2], pf[kb][3]};
#pragma unroll
        for (int dp = 0; dp < 4; ++dp) {  // pairs of 8-dim n-tiles
            const int key = kb * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
            const int c = dp * 2 + (lane >> 4);
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vbase + tile_off(key, c), b0, b1, b2, b3);
            Half16<TC>::mma(o_acc[2 * dp], a, b0, b1);
            Half16<TC>::mma(o_acc[2 * dp + 1], a, b2, b3);
        }
    }
}

// Normalise one warp's 16-row slab by 1/l (0 for a row that saw no key) and store it.
template <class TOut>
__device__ __forceinline__ void attn_store_slab(const AttnParams& p, TOut* O, uint32_t q_slab,
                                                const float (&o_acc)[8][4], const float (&l_run)[2], int lane) {
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint32_t qrow = q_slab + g + r * 8;
        if (qrow >= p.Tq) continue;
        const float inv = (l_run[r] > 0.0f) ? 1.0f / l_run[r] : 0.0f;
        TOut* orow = O + (uint64_t)qrow * p.ldo;
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) {
            const uint32_t d = dt * 8 + 2 * t;
            const float v0 = o_acc[dt][2 * r] * inv, v1 = o_acc[dt][2 * r + 1] * inv;
            if constexpr (sizeof(TOut) == 4) {
                if (d < p.hd) orow[d] = v0;
                if (d + 1 < p.hd) orow[d + 1] = v1;
            } else {
                if (d + 1 < p.hd && ((reinterpret_cast<uintptr_t>(orow + d) & 3) == 0)) {
                    *reinterpret_cast<uint32_t*>(orow + d) = Half16<TOut>::pack(v0, v1);
                } else {
                    if (d < p.hd) orow[d] = TOut(v0);
                    if (d + 1 < p.hd) orow[d + 1] = TOut(v1);
                }
            }
        }
    }
}

template <class TIn, class TOut, bool kAsync>
__global__ void __launch_bounds__(kAttnThreads, 2) attn_fwd_kernel(const AttnParams p) {
    grid_dependency_wait();
    grid_launch_dependents();
    using TC = typename AttnCompute<TIn>::T;
    extern __shared__ __align__(1024) uint8_t attn_smem[];
    uint8_t* sQ = attn_smem;
    uint8_t* sK[2] = {sQ + kAttnBM * 128, sQ + kAttnBM * 128 + kAttnBN * 128};
    uint8_t* sV[2] = {sQ + kAttnBM * 128 + 2 * kAttnBN * 128, sQ + kAttnBM * 128 + 3 * kAttnBN * 128};

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t q0 = blockIdx.x * kAttnBM;
    const uint32_t h = blockIdx.y, b = blockIdx.z;
    const TIn* Q = reinterpret_cast<const TIn*>(p.q) + b * p.sq + h * p.hq;
    const TIn* K = reinterpret_cast<const TIn*>(p.k) + b * p.sk + h * p.hk;
    const TIn* V = reinterpret_cast<const TIn*>(p.v) + b * p.sv + h * p.hv;

    // Causal: keys beyond this CTA's last query never contribute.
    uint32_t kv_end = p.Tk;
    if (p.causal) kv_end = min(kv_end, q0 + kAttnBM);
    const uint32_t n_tiles = (kv_end + kAttnBN - 1) / kAttnBN;

    attn_load_tile<TIn, TC, kAttnBM, kAsync>(sQ, Q, p.ldq, q0, p.Tq, p.hd);
    if (n_tiles > 0) {
        attn_load_tile<TIn, TC, kAttnBN, kAsync>(sK[0], K, p.ldk, 0, p.Tk, p.hd);
        attn_load_tile<TIn, TC, kAttnBN, kAsync>(sV[0], V, p.ldv, 0, p.Tk, p.hd);
    }
    if constexpr (kAsync) cp_async_commit();

    const int wrow = warp * 16;  // this warp's first query row in the CTA tile
    float o_acc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) o_acc[i][j] = 0.0f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
    uint32_t qf[4][4];

    for (uint32_t it = 0; it < n_tiles; ++it) {
        const int buf = it & 1;
        if (it + 1 < n_tiles) {
            const uint32_t kn = (it + 1) * kAttnBN;
            attn_load_tile<TIn, TC, kAttnBN, kAsync>(sK[buf ^ 1], K, p.ldk, kn, p.Tk, p.hd);
            attn_load_tile<TIn, TC, kAttnBN, kAsync>(sV[buf ^ 1], V, p.ldv, kn, p.Tk, p.hd);
            if constexpr (kAsync) {
                cp_async_commit();
                cp_async_wait<1>();
            }
        } else if constexpr (kAsync) {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (it == 0) {
            // Q fragments (16 queries x 64 dims) stay in registers for the whole KV sweep.
#pragma unroll
            for (int kb = 0; kb < 4; ++kb) {
                const int r = wrow + (lane & 15), c = kb * 2 + (lane >> 4);
                ldsm_x4(smem_u32(sQ) + tile_off(r, c), qf[kb][0], qf[kb][1], qf[kb][2], qf[kb][3]);
            }
        }
        attn_tile<TC>(p, smem_u32(sK[buf]), smem_u32(sV[buf]), it * kAttnBN, q0 + wrow, qf, o_acc, m_run, l_run,
                      lane);
        __syncthreads();  // the next iteration's loads overwrite this buffer
    }
    if constexpr (kAsync) {
        if (n_tiles == 0) cp_async_wait<0>();  // Tk == 0: only the Q copy was issued
    }
    attn_store_slab<TOut>(p, reinterpret_cast<TOut*>(p.o) + b * p.so + h * p.ho, q0 + wrow, o_acc, l_run, lane);
}

// Short key sequences (Tk <= 128, the 77-token cross-attention): four warps per 128-query CTA, each
// taking two 16-query slabs, with Q and every K/V tile staged once up front.  Its 128-thread CTAs
// fit four to an SM, so the whole grid is resident at once and every CTA's loads are in flight
// together; the per-tile math is the general kernel's.
template <class TIn, class TOut, bool kAsync>
__global__ void __launch_bounds__(kAttnShortThreads, 4) attn_short_kernel(const AttnParams p) {
    grid_dependency_wait();
    grid_launch_dependents();
    using TC = typename AttnCompute<TIn>::T;
    extern __shared__ __align__(1024) uint8_t attn_smem[];
    uint8_t* sQ = attn_smem;
    uint8_t* sK[2] = {sQ + kAttnBM * 128, sQ + kAttnBM * 128 + kAttnBN * 128};
    uint8_t* sV[2] = {sQ + kAttnBM * 128 + 2 * kAttnBN * 128, sQ + kAttnBM * 128 + 3 * kAttnBN * 128};

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t q0 = blockIdx.x * kAttnBM;
    const uint32_t h = blockIdx.y, b = blockIdx.z;
    const TIn* Q = reinterpret_cast<const TIn*>(p.q) + b * p.sq + h * p.hq;
    const TIn* K = reinterpret_cast<const TIn*>(p.k) + b * p.sk + h * p.hk;
    const TIn* V = reinterpret_cast<const TIn*>(p.v) + b * p.sv + h * p.hv;

    uint32_t kv_end = p.Tk;
    if (p.causal) kv_end = min(kv_end, q0 + kAttnBM);
    const uint32_t n_tiles = (kv_end + kAttnBN - 1) / kAttnBN;  // at most 2

    attn_load_tile<TIn, TC, kAttnBM, kAsync, kAttnShortThreads>(sQ, Q, p.ldq, q0, p.Tq, p.hd);
    for (uint32_t it = 0; it < n_tiles; ++it) {
        attn_load_tile<TIn, TC, kAttnBN, kAsync, kAttnShortThreads>(sK[it], K, p.ldk, it * kAttnBN, p.Tk, p.hd);
        attn_load_tile<TIn, TC, kAttnBN, kAsync, kAttnShortThreads>(sV[it], V, p.ldv, it * kAttnBN, p.Tk, p.hd);
    }
    if constexpr (kAsync) {
        cp_async_commit();
        cp_async_wait<0>();
    }
    __syncthreads();

    TOut* O = reinterpret_cast<TOut*>(p.o) + b * p.so + h * p.ho;
#pragma unroll 1
    for (int slab = 0; slab < kAttnBM / 16 / (kAttnShortThreads / 32); ++slab) {
        const int wrow = (warp + slab * (kAttnShortThreads / 32)) * 16;
        float o_acc[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) o_acc[i][j] = 0.0f;
        float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.0f, 0.0f};
        uint32_t qf[4][4];
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
            const int r = wrow + (lane & 15), c = kb * 2 + (lane >> 4);
            ldsm_x4(smem_u32(sQ) + tile_off(r, c), qf[kb][0], qf[kb][1], qf[kb][2], qf[kb][3]);
        }
#pragma unroll 1
        for (uint32_t it = 0; it < n_tiles; ++it)
            attn_tile<TC>(p, smem_u32(sK[it]), smem_u32(sV[it]), it * kAttnBN, q0 + wrow, qf, o_acc, m_run, l_run,
                          lane);
        attn_store_slab<TOut>(p, O, q0 + wrow, o_acc, l_run, lane);
    }
}

}  // namespace sdvk
