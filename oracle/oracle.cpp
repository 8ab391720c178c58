// oracle.cpp -- TEST INFRASTRUCTURE ONLY (see oracle.h for who may load it and why).
//
// A CPU restatement, in the reference's own fp32 operation order, of the sdvk hot-path shaders,
// plus fp64 truth references and seeded input generators.  Every function names the reference
// file:line it restates.  File paths are relative to the sdvk project root.
//
// Floating-point contract: this file is compiled with -ffp-contract=off, so the only fused
// multiply-adds are the explicit fmaf() calls, placed where the GLSL accumulates `acc += a*b`
// (which Vulkan drivers contract to FMA).  Everything else rounds per operation.

#include "oracle.h"

#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

namespace {

// ------------------------------------------------------------------------ fp16 helpers
uint16_t f32_to_f16_bits(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // >= 65520 rounds to inf
    if (ax < 0x38800000u) {                                     // below 2^-14: subnormal or zero
        float a;
        std::memcpy(&a, &ax, 4);
        double v = (double)a * 16777216.0;  // exact: units of 2^-24
        double r = std::nearbyint(v);       // round half to even (default mode)
        return (uint16_t)(sign | (uint32_t)r);
    }
    uint32_t e = (ax >> 23) - 127 + 15;
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

float f16_bits_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1Fu;
    uint32_t m = h & 0x3FFu;
    float out;
    if (e == 0) {
        out = (float)m * (1.0f / 16777216.0f);  // exact: m * 2^-24
        if (sign) out = -out;
        return out;
    }
    uint32_t f = (e == 31) ? (sign | 0x7F800000u | (m << 13)) : (sign | ((e - 15 + 127) << 23) | (m << 13));
    std::memcpy(&out, &f, 4);
    return out;
}

// ------------------------------------------------------------------------ counter RNG
inline uint64_t splitmix64(uint64_t x) {
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}
inline uint64_t stream_key(uint64_t seed, uint64_t stream) {
    return splitmix64(splitmix64(seed) ^ (stream * 0xD1B54A32D192ED03ull + 0x632BE59BD9B4E019ull));
}
// One standard normal per index: Box-Muller (cosine branch) on two hashed 53-bit uniforms.
inline double normal_at(uint64_t key, uint64_t i) {
    uint64_t h1 = splitmix64(key + 2 * i);
    uint64_t h2 = splitmix64(key + 2 * i + 1);
    double u1 = ((double)(h1 >> 11) + 1.0) * (1.0 / 9007199254740992.0);  // (0, 1]
    double u2 = (double)(h2 >> 11) * (1.0 / 9007199254740992.0);          // [0, 1)
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}

const float kLog2e = (float)1.4426950408889634;  // GLSL float literal (fused_attn*.comp:19/213)

// Butterfly reduction over `lanes` values with subgroupShuffleXor offsets lanes/2 .. 1
// (fused_attn_tiled.comp:42-56 for 16 lanes, fused_attn.comp:235-242 for 32 lanes).
inline float butterfly_sum(float* x, int lanes) {
    float t[32];
    for (int off = lanes / 2; off >= 1; off >>= 1) {
        for (int l = 0; l < lanes; ++l) t[l] = x[l] + x[l ^ off];
        for (int l = 0; l < lanes; ++l) x[l] = t[l];
    }
    return x[0];
}

}  // namespace

extern "C" {

int orc_num_threads(void) { return omp_get_max_threads(); }
void orc_set_num_threads(int n) {
    if (n > 0) omp_set_num_threads(n);
}

// ======================================================================== RNG
// The reference tests draw with std::mt19937 and libstdc++'s distributions
// (tests/fused_attn_test.cpp:82-89, tests/gemm_q8_bench.cpp:230-237).
void* orc_mt19937_new(uint32_t seed) { return new std::mt19937(seed); }
void orc_mt19937_free(void* h) { delete (std::mt19937*)h; }
void orc_mt19937_uniform_f32(void* h, float lo, float hi, float* out, uint64_t n) {
    std::uniform_real_distribution<float> d(lo, hi);
    std::mt19937& r = *(std::mt19937*)h;
    for (uint64_t i = 0; i < n; ++i) out[i] = d(r);
}
void orc_mt19937_uniform_int(void* h, int32_t lo, int32_t hi, int32_t* out, uint64_t n) {
    std::uniform_int_distribution<int> d(lo, hi);
    std::mt19937& r = *(std::mt19937*)h;
    for (uint64_t i = 0; i < n; ++i) out[i] = d(r);
}

// The generation loop's noise source (src/Modules/Diffusion/sdvkgen.cpp:3732-3734, draws at :3869,
// :3946, :3996): one std::mt19937(seed) and one std::normal_distribution<float>(0, 1) kept for the
// whole run, so the initial latent and every ancestral step's draws continue one sequence (the
// distribution object carries its second polar-method value from call to call).
struct OrcGenRng {
    std::mt19937 rng;
    std::normal_distribution<float> nd{0.0f, 1.0f};
    explicit OrcGenRng(uint32_t seed) : rng(seed) {}
};
void* orc_gen_rng_new(uint32_t seed) { return new OrcGenRng(seed); }
void orc_gen_rng_free(void* h) { delete (OrcGenRng*)h; }
void orc_gen_rng_normal(void* h, float* out, uint64_t n) {
    OrcGenRng& g = *(OrcGenRng*)h;
    for (uint64_t i = 0; i < n; ++i) out[i] = g.nd(g.rng);
}

void orc_normal_f32(uint64_t seed, uint64_t stream, float std_dev, float* out, uint64_t n) {
    uint64_t key = stream_key(seed, stream);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = (float)(normal_at(key, (uint64_t)i) * std_dev);
}
void orc_normal_f16(uint64_t seed, uint64_t stream, float std_dev, uint16_t* out, uint64_t n) {
    uint64_t key = stream_key(seed, stream);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i)
        out[i] = f32_to_f16_bits((float)(normal_at(key, (uint64_t)i) * std_dev));
}

void orc_q8_weights(uint64_t seed, uint64_t stream, uint64_t rows, uint64_t cols, int8_t* q,
                    uint16_t* scale_f16, float* scale_f32) {
    uint64_t n = rows * cols, nb = n / 32;
    uint64_t kq = stream_key(seed, 2 * stream), ks = stream_key(seed, 2 * stream + 1);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) q[i] = (int8_t)((int)(splitmix64(kq + (uint64_t)i) % 255u) - 127);
#pragma omp parallel for schedule(static)
    for (int64_t b = 0; b < (int64_t)nb; ++b) {
        double d = std::fabs(normal_at(ks, (uint64_t)b) * 0.02) / 127.0;
        uint16_t h = f32_to_f16_bits((float)d);
        if (scale_f16) scale_f16[b] = h;
        if (scale_f32) scale_f32[b] = f16_bits_to_f32(h);
    }
}

void orc_f32_to_f16(const float* in, uint16_t* out, uint64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = f32_to_f16_bits(in[i]);
}
void orc_f16_to_f32(const uint16_t* in, float* out, uint64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) out[i] = f16_bits_to_f32(in[i]);
}

// ======================================================================== GGUF Q8_0 codec
// Block = little-endian fp16 d followed by 32 int8 (src/Modules/Model/Gguf.cpp:83, :514-523).
void orc_q8_0_pack_blocks(const int8_t* q, const uint16_t* d, uint64_t nblocks, uint8_t* blocks) {
    for (uint64_t b = 0; b < nblocks; ++b) {
        uint8_t* blk = blocks + b * 34;
        blk[0] = (uint8_t)(d[b] & 0xFF);
        blk[1] = (uint8_t)(d[b] >> 8);
        std::memcpy(blk + 2, q + b * 32, 32);
    }
}
// Split into the engine's device layout: int8 payload [rows*cols] + fp32 scale per block
// (Gguf.cpp:559-583 readQ8Into, uploaded by sdvkgen.cpp:561-583).
void orc_q8_0_split_blocks(const uint8_t* blocks, uint64_t nblocks, int8_t* q, float* scales) {
    for (uint64_t b = 0; b < nblocks; ++b) {
        const uint8_t* blk = blocks + b * 34;
        scales[b] = f16_bits_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
        std::memcpy(q + b * 32, blk + 2, 32);
    }
}
// Minimal GGUF v3 file with one 2-D Q8_0 tensor (ne0 = cols), laid out as Gguf.cpp:290-416 parses.
int orc_gguf_write_q8(const char* path, const char* name, uint64_t rows, uint64_t cols,
                      const uint8_t* blocks) {
    FILE* f = std::fopen(path, "wb");
    if (!f) return 1;
    auto w = [&](const void* p, size_t n) { std::fwrite(p, 1, n, f); };
    auto wstr = [&](const char* s) {
        uint64_t len = std::strlen(s);
        w(&len, 8);
        w(s, len);
    };
    uint32_t version = 3, u32 = 0;
    uint64_t nt = 1, nkv = 1;
    w("GGUF", 4);
    w(&version, 4);
    w(&nt, 8);
    w(&nkv, 8);
    wstr("general.alignment");
    u32 = 4;  // GGUF_UINT32
    w(&u32, 4);
    u32 = 32;
    w(&u32, 4);
    wstr(name);
    u32 = 2;
    w(&u32, 4);
    w(&cols, 8);
    w(&rows, 8);
    u32 = 8;  // Q8_0
    w(&u32, 4);
    uint64_t off = 0;
    w(&off, 8);
    long pos = std::ftell(f);
    long pad = (32 - pos % 32) % 32;
    for (long i = 0; i < pad; ++i) std::fputc(0, f);
    w(blocks, (size_t)(rows * cols / 32 * 34));
    std::fclose(f);
    return 0;
}

// ======================================================================== Q8_0 GEMM NT
// gemm_nt_q8_v.comp:45-127 (every BM/BN/BK variant of CMakeLists.txt:41-69 computes the same
// per-element sequence).  Per output (m,n) one shader thread accumulates acc += A*B with k
// ascending through the K tiles.  A and B are staged in groups of 4 along K, and a group is
// zero-filled unless `gc + 3 < K` (:69, :86), so only k < (K & ~3) contributes.  B is dequantised
// as float(int8) * s[(n*K + k) >> 5] in fp32 (:87-97).  The bias is added after the reduction,
// mode 0 only (:121-124); mode 1 accumulates into C without the bias (:125).
void orc_gemm_nt_q8_shader(const float* A, const int8_t* q, const float* s, const float* bias,
                           float* C, uint32_t M, uint32_t N, uint32_t K, uint32_t mode,
                           uint32_t sA, uint32_t sC, uint32_t batch, uint32_t lda, uint32_t ldc) {
    if (!lda) lda = K;
    if (!ldc) ldc = N;
    const uint32_t Keff = K & ~3u;
    const uint32_t NB = 32, MB = 4;
    const uint32_t nblk = (N + NB - 1) / NB, mblk = (M + 63) / 64;
#pragma omp parallel
    {
        std::vector<float> w((size_t)Keff * NB);
#pragma omp for collapse(3) schedule(dynamic)
        for (int64_t z = 0; z < (int64_t)batch; ++z)
            for (int64_t nb = 0; nb < (int64_t)nblk; ++nb)
                for (int64_t mb = 0; mb < (int64_t)mblk; ++mb) {
                    const uint32_t n0 = (uint32_t)nb * NB, m0 = (uint32_t)mb * 64;
                    const uint32_t nc = std::min(NB, N - n0), mEnd = std::min(M, m0 + 64);
                    // dequantised weights, transposed to [k][j]
                    for (uint32_t k = 0; k < Keff; ++k)
                        for (uint32_t j = 0; j < NB; ++j) {
                            float v = 0.0f;
                            if (j < nc) {
                                uint32_t fl = (n0 + j) * K + k;
                                v = (float)q[fl] * s[fl >> 5];
                            }
                            w[(size_t)k * NB + j] = v;
                        }
                    const float* Az = A + (size_t)z * sA;
                    float* Cz = C + (size_t)z * sC;
                    for (uint32_t m = m0; m < mEnd; m += MB) {
                        const uint32_t mr = std::min(MB, mEnd - m);
                        float acc[MB][NB];
                        for (uint32_t i = 0; i < MB; ++i)
                            for (uint32_t j = 0; j < NB; ++j) acc[i][j] = 0.0f;
                        const float* ar[MB];
                        for (uint32_t i = 0; i < MB; ++i) ar[i] = Az + (size_t)(m + std::min(i, mr - 1)) * lda;
                        for (uint32_t k = 0; k < Keff; ++k) {
                            const float* wk = &w[(size_t)k * NB];
                            for (uint32_t i = 0; i < MB; ++i) {
                                const float a = ar[i][k];
                                for (uint32_t j = 0; j < NB; ++j) acc[i][j] = fmaf(a, wk[j], acc[i][j]);
                            }
                        }
                        for (uint32_t i = 0; i < mr; ++i)
                            for (uint32_t j = 0; j < nc; ++j) {
                                float* dst = Cz + (size_t)(m + i) * ldc + n0 + j;
                                if (mode == 0) {
                                    float v = acc[i][j];
                                    if (bias) v += bias[n0 + j];
                                    *dst = v;
                                } else {
                                    *dst += acc[i][j];
                                }
                            }
                    }
                }
    }
}

// fp64 truth: dequantise to double, plain dot over all K (no group-of-4 truncation).
void orc_gemm_nt_q8_f64(const float* A, const int8_t* q, const float* s, const float* bias,
                        double* C, uint32_t M, uint32_t N, uint32_t K, uint32_t sA, uint32_t sC,
                        uint32_t batch, uint32_t lda, uint32_t ldc) {
    if (!lda) lda = K;
    if (!ldc) ldc = N;
    const uint32_t NB = 16;
    const uint32_t nblk = (N + NB - 1) / NB;
#pragma omp parallel
    {
        std::vector<double> w((size_t)K * NB);
#pragma omp for collapse(2) schedule(dynamic)
        for (int64_t z = 0; z < (int64_t)batch; ++z)
            for (int64_t nb = 0; nb < (int64_t)nblk; ++nb) {
                const uint32_t n0 = (uint32_t)nb * NB, nc = std::min(NB, N - n0);
                for (uint32_t k = 0; k < K; ++k)
                    for (uint32_t j = 0; j < NB; ++j) {
                        double v = 0.0;
                        if (j < nc) {
                            uint64_t fl = (uint64_t)(n0 + j) * K + k;
                            v = (double)q[fl] * (double)s[fl >> 5];
                        }
                        w[(size_t)k * NB + j] = v;
                    }
                for (uint32_t m = 0; m < M; ++m) {
                    const float* a = A + (size_t)z * sA + (size_t)m * lda;
                    double acc[NB] = {0};
                    for (uint32_t k = 0; k < K; ++k) {
                        const double av = a[k];
                        const double* wk = &w[(size_t)k * NB];
                        for (uint32_t j = 0; j < NB; ++j) acc[j] += av * wk[j];
                    }
                    for (uint32_t j = 0; j < nc; ++j)
                        C[(size_t)z * sC + (size_t)m * ldc + n0 + j] = acc[j] + (bias ? (double)bias[n0 + j] : 0.0);
                }
            }
    }
}

// ======================================================================== Q8_0 GEMM NN
// gemm_nn_q8_v.comp:158-237.  A = weight (int8 words + fp32 scale per 32 elements, flat index
// ao + m*lda + k, :179-200), B = fp32 [K,N] row-major with ldb, staged in groups of 4 along N and
// zero-filled unless `gc + 3 < N` (:207).  A groups need `gc + 3 < K` (:184).  Per (m,n):
// acc += A*B over k ascending; mode 0 stores, mode 1 accumulates (:233-235).  The packed word
// holding element fl is aq[fl >> 2], so an fl that is not a multiple of 4 reads the bytes of its
// word from byte 0 (restated by indexing (fl & ~3) + i).
void orc_gemm_nn_q8_shader(const int8_t* q, const float* s, const float* B, float* C, uint32_t M,
                           uint32_t N, uint32_t K, uint32_t mode, uint32_t sA, uint32_t sB,
                           uint32_t sC, uint32_t batch, uint32_t lda, uint32_t ldb, uint32_t ldc) {
    if (!lda) lda = K;
    if (!ldb) ldb = N;
    if (!ldc) ldc = N;
    const uint32_t Keff = K & ~3u;  // A groups with gc+3 >= K are zero
    const uint32_t Neff = N & ~3u;  // B groups with gc+3 >= N are zero
    const uint32_t MB = 16, NB = 64;
    const uint32_t mblk = (M + MB - 1) / MB, nblk = (N + NB - 1) / NB;
#pragma omp parallel
    {
        std::vector<float> wa((size_t)MB * (Keff ? Keff : 1));
#pragma omp for collapse(3) schedule(dynamic)
        for (int64_t z = 0; z < (int64_t)batch; ++z)
            for (int64_t mb = 0; mb < (int64_t)mblk; ++mb)
                for (int64_t nb = 0; nb < (int64_t)nblk; ++nb) {
                    const uint32_t m0 = (uint32_t)mb * MB, n0 = (uint32_t)nb * NB;
                    const uint32_t mr = std::min(MB, M - m0), nc = std::min(NB, N - n0);
                    for (uint32_t i = 0; i < mr; ++i)
                        for (uint32_t k = 0; k < Keff; k += 4) {
                            uint32_t fl = (uint32_t)z * sA + (m0 + i) * lda + k;
                            uint32_t base = fl & ~3u;
                            float sc = s[fl >> 5];
                            for (uint32_t t = 0; t < 4; ++t) wa[(size_t)i * Keff + k + t] = (float)q[base + t] * sc;
                        }
                    const float* Bz = B + (size_t)z * sB;
                    float* Cz = C + (size_t)z * sC;
                    for (uint32_t i = 0; i < mr; ++i) {
                        float acc[NB];
                        for (uint32_t j = 0; j < NB; ++j) acc[j] = 0.0f;
                        for (uint32_t k = 0; k < Keff; ++k) {
                            const float a = wa[(size_t)i * Keff + k];
                            const float* br = Bz + (size_t)k * ldb + n0;
                            for (uint32_t j = 0; j < nc; ++j) {
                                float bv = (n0 + j < Neff) ? br[j] : 0.0f;
                                acc[j] = fmaf(a, bv, acc[j]);
                            }
                        }
                        for (uint32_t j = 0; j < nc; ++j) {
                            float* dst = Cz + (size_t)(m0 + i) * ldc + n0 + j;
                            if (mode == 0) *dst = acc[j];
                            else *dst += acc[j];
                        }
                    }
                }
    }
}

void orc_gemm_nn_q8_f64(const int8_t* q, const float* s, const float* B, double* C, uint32_t M,
                        uint32_t N, uint32_t K, uint32_t sB, uint32_t sC, uint32_t batch,
                        uint32_t lda, uint32_t ldb, uint32_t ldc) {
    if (!lda) lda = K;
    if (!ldb) ldb = N;
    if (!ldc) ldc = N;
#pragma omp parallel
    {
        std::vector<double> acc(N);
        std::vector<double> wrow(K);
#pragma omp for collapse(2) schedule(dynamic)
        for (int64_t z = 0; z < (int64_t)batch; ++z)
            for (int64_t m = 0; m < (int64_t)M; ++m) {
                for (uint32_t k = 0; k < K; ++k) {
                    uint64_t fl = (uint64_t)m * lda + k;
                    wrow[k] = (double)q[fl] * (double)s[fl >> 5];
                }
                std::fill(acc.begin(), acc.end(), 0.0);
                const float* Bz = B + (size_t)z * sB;
                for (uint32_t k = 0; k < K; ++k) {
                    const double a = wrow[k];
                    const float* br = Bz + (size_t)k * ldb;
                    for (uint32_t n = 0; n < N; ++n) acc[n] += a * (double)br[n];
                }
                for (uint32_t n = 0; n < N; ++n) C[(size_t)z * sC + (size_t)m * ldc + n] = acc[n];
            }
    }
}

// ======================================================================== attention
// fused_attn_tiled.comp:58-193: one workgroup = 64 queries x one head (hd must be 64), 64-key
// tiles.  Per tile: S = Q.K^T accumulated over d ascending (:111-121), scaled after the dot
// (:132), masked to -1e30 (:133-134); row max over the 64 columns; resc = exp2((m_old-m_new)*LOG2E)
// (:140); p = s > -1e29 ? exp2((s-m_new)*LOG2E) : 0 (:149); each of the 16 lanes sums its 4
// columns in order, then a 16-lane xor butterfly (:146-154); O = O*resc + P.V over keys ascending
// (:144, :169-179); output O / l, or 0 when l == 0 (:189-192).
int orc_attn_tiled_shader(const float* Q, const float* K, const float* V, float* O, uint32_t Tq,
                          uint32_t Tk, uint32_t C, uint32_t heads, uint32_t causal, float scale) {
    if (!heads || C % heads || C / heads != 64) return 1;
    const uint32_t HD = 64, BM = 64, BN = 64;
    const uint32_t qtiles = (Tq + BM - 1) / BM;
#pragma omp parallel
    {
        std::vector<float> Qs(BM * HD), Ks(BN * HD), Vs(BN * HD), S(BM * BN), acc(BM * HD);
        std::vector<float> mRun(BM), lRun(BM);
#pragma omp for collapse(2) schedule(dynamic)
        for (int64_t h = 0; h < (int64_t)heads; ++h)
            for (int64_t qt = 0; qt < (int64_t)qtiles; ++qt) {
                const uint32_t q0 = (uint32_t)qt * BM, hOff = (uint32_t)h * HD;
                for (uint32_t r = 0; r < BM; ++r) {
                    mRun[r] = -1e30f;
                    lRun[r] = 0.0f;
                    for (uint32_t d = 0; d < HD; ++d) {
                        acc[r * HD + d] = 0.0f;
                        Qs[r * HD + d] = (q0 + r < Tq) ? Q[(size_t)(q0 + r) * C + hOff + d] : 0.0f;
                    }
                }
                for (uint32_t kv0 = 0; kv0 < Tk; kv0 += BN) {
                    for (uint32_t r = 0; r < BN; ++r)
                        for (uint32_t d = 0; d < HD; ++d) {
                            bool ok = kv0 + r < Tk;
                            Ks[r * HD + d] = ok ? K[(size_t)(kv0 + r) * C + hOff + d] : 0.0f;
                            Vs[r * HD + d] = ok ? V[(size_t)(kv0 + r) * C + hOff + d] : 0.0f;
                        }
                    for (uint32_t r = 0; r < BM; ++r) {
                        const uint32_t qr = q0 + r;
                        float mx = -1e30f;
                        for (uint32_t c = 0; c < BN; ++c) {
                            float sv = 0.0f;
                            for (uint32_t d = 0; d < HD; ++d) sv = fmaf(Qs[r * HD + d], Ks[c * HD + d], sv);
                            const uint32_t kv = kv0 + c;
                            float v = sv * scale;
                            if (qr >= Tq || kv >= Tk) v = -1e30f;
                            if (causal && kv > qr) v = -1e30f;
                            S[r * BN + c] = v;
                            mx = std::max(mx, v);
                        }
                        const float mNew = std::max(mRun[r], mx);
                        const float resc = exp2f((mRun[r] - mNew) * kLog2e);
                        mRun[r] = mNew;
                        lRun[r] *= resc;
                        for (uint32_t d = 0; d < HD; ++d) acc[r * HD + d] *= resc;
                        float lane[16];
                        for (uint32_t tx = 0; tx < 16; ++tx) {
                            float sum = 0.0f;
                            for (uint32_t j = 0; j < 4; ++j) {
                                float& sv = S[r * BN + tx * 4 + j];
                                float p = (sv > -1e29f) ? exp2f((sv - mNew) * kLog2e) : 0.0f;
                                sv = p;
                                sum += p;
                            }
                            lane[tx] = sum;
                        }
                        lRun[r] += butterfly_sum(lane, 16);
                        for (uint32_t c = 0; c < BN; ++c) {
                            const float p = S[r * BN + c];
                            for (uint32_t d = 0; d < HD; ++d) acc[r * HD + d] = fmaf(p, Vs[c * HD + d], acc[r * HD + d]);
                        }
                    }
                }
                for (uint32_t r = 0; r < BM; ++r) {
                    const uint32_t qr = q0 + r;
                    if (qr >= Tq) continue;
                    const float inv = (lRun[r] > 0.0f) ? (1.0f / lRun[r]) : 0.0f;
                    for (uint32_t d = 0; d < HD; ++d) O[(size_t)qr * C + hOff + d] = acc[r * HD + d] * inv;
                }
            }
    }
    return 0;
}

// fused_attn.comp:244-318: per query, keys one at a time (32-key smem tiles do not change the
// order).  Lane l holds dims l and l+32 (when l+32 < hd); dot = q0*k0 + q1*k1 per lane, then a
// 32-lane xor butterfly (:294-295); s = dot*scale*LOG2E (:296); causal -> -1e30 (:297); exp2-domain
// online softmax l = l*resc + p, acc = acc*resc + p*v (:298-304).  Only 32 <= hd <= 64 is
// restated: for hd < 32 the shader's lanes >= hd read neighbouring heads/keys and write into the
// next head's output columns, which races with other workgroups (result undefined).
int orc_attn_simple_shader(const float* Q, const float* K, const float* V, float* O, uint32_t Tq,
                           uint32_t Tk, uint32_t C, uint32_t heads, uint32_t causal, float scale) {
    if (!heads || C % heads) return 1;
    const uint32_t hd = C / heads;
    if (hd < 32 || hd > 64) return 1;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int64_t h = 0; h < (int64_t)heads; ++h)
        for (int64_t qr = 0; qr < (int64_t)Tq; ++qr) {
            float q0[32], q1[32], a0[32], a1[32], part[32];
            const size_t qb = (size_t)qr * C + (size_t)h * hd;
            for (uint32_t l = 0; l < 32; ++l) {
                bool has2 = l + 32 < hd;
                q0[l] = Q[qb + l];
                q1[l] = has2 ? Q[qb + l + 32] : 0.0f;
                a0[l] = a1[l] = 0.0f;
            }
            float mRun = -1e30f, lRun = 0.0f;
            for (uint32_t kv = 0; kv < Tk; ++kv) {
                const size_t kb = (size_t)kv * C + (size_t)h * hd;
                for (uint32_t l = 0; l < 32; ++l) {
                    bool has2 = l + 32 < hd;
                    float k0 = K[kb + l], k1 = has2 ? K[kb + l + 32] : 0.0f;
                    part[l] = fmaf(q1[l], k1, q0[l] * k0);
                }
                const float dot = butterfly_sum(part, 32);
                float sv = dot * scale * kLog2e;
                if (causal && kv > (uint32_t)qr) sv = -1e30f;
                const float mNew = std::max(mRun, sv);
                const float resc = exp2f(mRun - mNew);
                const float p = exp2f(sv - mNew);
                lRun = fmaf(lRun, resc, p);
                for (uint32_t l = 0; l < 32; ++l) {
                    bool has2 = l + 32 < hd;
                    float v0 = V[kb + l], v1 = has2 ? V[kb + l + 32] : 0.0f;
                    a0[l] = fmaf(p, v0, a0[l] * resc);
                    a1[l] = fmaf(p, v1, a1[l] * resc);
                }
                mRun = mNew;
            }
            const float inv = (lRun > 0.0f) ? (1.0f / lRun) : 0.0f;
            for (uint32_t l = 0; l < 32; ++l) {
                O[qb + l] = a0[l] * inv;
                if (l + 32 < hd) O[qb + l + 32] = a1[l] * inv;
            }
        }
    return 0;
}

// fusedAttention (src/Modules/GPU/fused_attn.cpp:40-61): hd = C/heads must be 1..64
// (fusedAttnSupported, :34-38); tiled kernel iff hd == 64 && Tk >= 256 && !SDVK_ATTN_SIMPLE;
// scale = 1/sqrt(hd) in fp32.
int orc_fused_attention(const float* Q, const float* K, const float* V, float* O, uint32_t Tq,
                        uint32_t Tk, uint32_t C, uint32_t heads, uint32_t causal, int force_simple) {
    if (!C || !heads || C % heads) return 1;
    const uint32_t hd = C / heads;
    if (hd == 0 || hd > 64) return 1;
    const bool tiled = (hd == 64) && Tk >= 256 && !force_simple;
    const float scale = 1.0f / std::sqrt((float)hd);
    if (tiled) return orc_attn_tiled_shader(Q, K, V, O, Tq, Tk, C, heads, causal, scale);
    return orc_attn_simple_shader(Q, K, V, O, Tq, Tk, C, heads, causal, scale);
}

// fp64 truth: the online-softmax double reference of tests/fused_attn_test.cpp:25-61, with
// explicit strides and a batch loop.  Fully masked rows produce 0.
void orc_attn_f64(const float* Q, const float* K, const float* V, double* O, uint32_t batch,
                  uint32_t Tq, uint32_t Tk, uint32_t heads, uint32_t hd, uint64_t ldq,
                  uint64_t ldk, uint64_t ldv, uint64_t ldo, uint64_t sQ, uint64_t sK, uint64_t sV,
                  uint64_t sO, uint32_t causal, double scale) {
#pragma omp parallel for collapse(3) schedule(dynamic)
    for (int64_t b = 0; b < (int64_t)batch; ++b)
        for (int64_t h = 0; h < (int64_t)heads; ++h)
            for (int64_t tq = 0; tq < (int64_t)Tq; ++tq) {
                std::vector<double> acc(hd, 0.0);
                double m = -INFINITY, l = 0.0;
                const float* q = Q + b * sQ + tq * ldq + h * hd;
                for (uint32_t tk = 0; tk < Tk; ++tk) {
                    if (causal && tk > (uint64_t)tq) continue;
                    const float* k = K + b * sK + tk * ldk + h * hd;
                    const float* v = V + b * sV + tk * ldv + h * hd;
                    double dot = 0.0;
                    for (uint32_t d = 0; d < hd; ++d) dot += (double)q[d] * (double)k[d];
                    const double s = dot * scale;
                    const double mNew = std::max(m, s);
                    const double resc = (m == -INFINITY) ? 0.0 : std::exp(m - mNew);
                    l *= resc;
                    for (uint32_t d = 0; d < hd; ++d) acc[d] *= resc;
                    const double p = std::exp(s - mNew);
                    l += p;
                    for (uint32_t d = 0; d < hd; ++d) acc[d] += p * (double)v[d];
                    m = mNew;
                }
                const double inv = l > 0.0 ? 1.0 / l : 0.0;
                double* o = O + b * sO + tq * ldo + h * hd;
                for (uint32_t d = 0; d < hd; ++d) o[d] = acc[d] * inv;
            }
}

// ======================================================================== block glue
// layernorm_fwd.comp:15-39 with 256 lanes: lane t sums x[j], j = t, t+256, ... in order; a tree
// reduction (stride 128 .. 1) combines the lanes; two-pass variance; y = (x-mean)*inv, then
// *gamma + beta when affine.
void orc_layernorm_shader(const float* x, const float* gamma, const float* beta, float* y,
                          uint32_t rows, uint32_t d, float eps, uint32_t affine) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; ++r) {
        const float* xr = x + (size_t)r * d;
        float red[256];
        for (uint32_t t = 0; t < 256; ++t) {
            float s = 0.0f;
            for (uint32_t j = t; j < d; j += 256) s += xr[j];
            red[t] = s;
        }
        for (uint32_t st = 128; st > 0; st >>= 1)
            for (uint32_t t = 0; t < st; ++t) red[t] += red[t + st];
        const float mean = red[0] / (float)d;
        for (uint32_t t = 0; t < 256; ++t) {
            float ss = 0.0f;
            for (uint32_t j = t; j < d; j += 256) {
                float dv = xr[j] - mean;
                ss = fmaf(dv, dv, ss);
            }
            red[t] = ss;
        }
        for (uint32_t st = 128; st > 0; st >>= 1)
            for (uint32_t t = 0; t < st; ++t) red[t] += red[t + st];
        const float var = red[0] / (float)d;
        const float inv = 1.0f / std::sqrt(var + eps);
        for (uint32_t j = 0; j < d; ++j) {
            float v = (xr[j] - mean) * inv;
            if (affine) v = fmaf(v, gamma[j], beta[j]);
            y[(size_t)r * d + j] = v;
        }
    }
}

// groupnorm.comp:12-39, one workgroup (256 lanes) per group: lane t sums x[base + i], i = t, t+256,
// ... in order, a tree over the 256 partials (stride 128 down to 1) gives the mean; the same for the
// squared deviations gives the population variance; then (x - mean) * r * gamma[c] + beta[c] and,
// with act == 1, v / (1 + exp(-v)).  Multiply-adds are fused as in the layernorm restatement above.
void orc_groupnorm_shader(const float* x, const float* gamma, const float* beta, float* y, uint32_t C,
                          uint32_t P, uint32_t G, float eps, uint32_t act) {
    const uint32_t Cg = C / G;
    const uint64_t cnt = (uint64_t)Cg * P;
#pragma omp parallel for schedule(static)
    for (int64_t g = 0; g < (int64_t)G; ++g) {
        const uint64_t base = (uint64_t)g * cnt;
        float red[256];
        for (uint32_t t = 0; t < 256; ++t) {
            float s = 0.0f;
            for (uint64_t i = t; i < cnt; i += 256) s += x[base + i];
            red[t] = s;
        }
        for (uint32_t st = 128; st > 0; st >>= 1)
            for (uint32_t t = 0; t < st; ++t) red[t] += red[t + st];
        const float mean = red[0] / (float)cnt;
        for (uint32_t t = 0; t < 256; ++t) {
            float ss = 0.0f;
            for (uint64_t i = t; i < cnt; i += 256) {
                const float dv = x[base + i] - mean;
                ss = fmaf(dv, dv, ss);
            }
            red[t] = ss;
        }
        for (uint32_t st = 128; st > 0; st >>= 1)
            for (uint32_t t = 0; t < st; ++t) red[t] += red[t + st];
        const float var = red[0] / (float)cnt;
        const float r = 1.0f / std::sqrt(var + eps);
        for (uint64_t i = 0; i < cnt; ++i) {
            const uint32_t ch = (uint32_t)(g * Cg + i / P);
            float v = fmaf((x[base + i] - mean) * r, gamma[ch], beta[ch]);
            if (act == 1u) v = v / (1.0f + std::exp(-v));
            y[base + i] = v;
        }
    }
}

void orc_layernorm_f64(const double* x, const float* gamma, const float* beta, double* y,
                       uint32_t rows, uint32_t d, double eps) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)rows; ++r) {
        const double* xr = x + (size_t)r * d;
        double mean = 0.0, var = 0.0;
        for (uint32_t j = 0; j < d; ++j) mean += xr[j];
        mean /= d;
        for (uint32_t j = 0; j < d; ++j) var += (xr[j] - mean) * (xr[j] - mean);
        var /= d;
        const double inv = 1.0 / std::sqrt(var + eps);
        for (uint32_t j = 0; j < d; ++j)
            y[(size_t)r * d + j] = (xr[j] - mean) * inv * (double)gamma[j] + (double)beta[j];
    }
}

// unary_fwd.comp:28-35 (mode 4, used by geluErf sdvkgen.cpp:1034): erf GELU with the
// Abramowitz & Stegun 7.1.26 polynomial in fp32.
void orc_gelu_erf_shader(const float* x, float* y, uint64_t n) {
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; ++i) {
        const float v = x[i];
        const float xs = v * 0.70710678118654752440f;
        const float ax = std::fabs(xs);
        const float t = 1.0f / (1.0f + 0.3275911f * ax);
        const float poly = (((((1.061405429f * t - 1.453152027f) * t) + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t;
        const float e = 1.0f - poly * std::exp(-ax * ax);
        const float erf = xs >= 0.0f ? e : -e;
        y[i] = 0.5f * v * (1.0f + erf);
    }
}

// evalGuided's guidance combine (src/Modules/Diffusion/sdvkgen.cpp:3825-3845), in its order:
// res = u + cfg * (c - u) in fp32; with rescale > 0, the mean and spreads in double, then
// er = (res - m) * (su / sg) + m and res = rescale * er + (1 - rescale) * res.
void orc_cfg_combine(const float* cond, const float* uncond, float* out, uint64_t n, float cfg, float rescale) {
    for (uint64_t k = 0; k < n; ++k) out[k] = uncond[k] + cfg * (cond[k] - uncond[k]);
    if (rescale > 0.0f) {
        double m = 0, s2 = 0, u2 = 0;
        for (uint64_t k = 0; k < n; ++k) m += out[k];
        m /= (double)n;
        for (uint64_t k = 0; k < n; ++k) {
            const double d = out[k] - m;
            s2 += d * d;
        }
        for (uint64_t k = 0; k < n; ++k) u2 += (double)uncond[k] * uncond[k];
        const double su = std::sqrt(u2 / (double)n);
        const double sg = std::sqrt(s2 / (double)n) + 1e-6;
        for (uint64_t k = 0; k < n; ++k) {
            const float er = (float)((out[k] - m) * (su / sg) + m);
            out[k] = (float)(rescale * er + (1.0 - rescale) * out[k]);
        }
    }
}

// ------------------------------------------------------------------ the sampler step
// ancestralSigma (sdvkgen.cpp:2809-2813)
static float orc_ancestral_sigma(float s_down, float sigma, float eta) {
    if (sigma <= 0.0f) return 0.0f;
    const float inside = s_down * s_down * (sigma * sigma - s_down * s_down) / (sigma * sigma);
    return eta * std::sqrt(std::max(0.0f, inside));
}

// One evaluation of the loop body sdvkgen.cpp:3796-4019: evalGuided (:3811-3846), x0FromEps
// (:3770-3776), finishX0 (:3779-3797), then the sampler's switch (:3859-4019).
uint64_t orc_sampler_eval(const orc_sampler_args* a) {
    const uint64_t n = a->n;
    const bool guided = a->eps_u != nullptr;
    const float sigma = a->sigma, sn = a->sigma_next, dt = sn - sigma;
    const bool last = sn <= 0.0f;
    const float eta = a->eta > 0 ? a->eta : 1.0f;
    // this evaluation's sigma and latent
    float sig = sigma;
    if (a->phase == 1) {
        if (a->kind == 2) sig = sn;
        else if (a->kind == 4) sig = sigma + 0.5f * dt;
        else {
            const float up = std::min(sn, orc_ancestral_sigma(sn, sigma, eta));
            const float down = std::sqrt(std::max(0.0f, sn * sn - up * up));
            sig = sigma + 0.5f * (down - sigma);
        }
    }
    const float* x = a->phase == 0 ? a->lat : a->x_tmp;
    uint64_t bad = 0;
    for (uint64_t k = 0; k < n; ++k)
        if (!std::isfinite(a->eps_c[k]) || (guided && !std::isfinite(a->eps_u[k]))) bad++;
    if (bad) return bad;
    std::vector<float> res(n);
    for (uint64_t k = 0; k < n; ++k) res[k] = guided ? a->eps_u[k] + a->cfg * (a->eps_c[k] - a->eps_u[k]) : a->eps_c[k];
    if (a->rescale > 0.0f && guided) {
        double m = 0, s2 = 0, u2 = 0;
        for (uint64_t k = 0; k < n; ++k) m += res[k];
        m /= (double)n;
        for (uint64_t k = 0; k < n; ++k) {
            const double d = res[k] - m;
            s2 += d * d;
        }
        for (uint64_t k = 0; k < n; ++k) u2 += (double)a->eps_u[k] * a->eps_u[k];
        const double su = std::sqrt(u2 / (double)n);
        const double sg = std::sqrt(s2 / (double)n) + 1e-6;
        for (uint64_t k = 0; k < n; ++k) {
            const float er = (float)((res[k] - m) * (su / sg) + m);
            res[k] = (float)(a->rescale * er + (1.0 - a->rescale) * res[k]);
        }
    }
    // x0FromEps
    const float s2 = sig * sig + 1.0f, root = std::sqrt(s2);
    float* x0 = a->x0;
    for (uint64_t k = 0; k < n; ++k) x0[k] = a->vpred ? res[k] * (-sig / root) + x[k] / s2 : x[k] - sig * res[k];
    // finishX0
    float thr = 1.0f;
    if (a->dynthresh) {
        std::vector<float> absv(n);
        for (uint64_t k = 0; k < n; ++k) absv[k] = std::abs(x0[k]);
        const size_t q = (size_t)((double)(n - 1) * 0.995);
        std::nth_element(absv.begin(), absv.begin() + q, absv.end());
        thr = std::max(absv[q], 1.0f);
    }
    for (uint64_t k = 0; k < n; ++k) {
        float v = x0[k];
        if (a->dynthresh) v = std::min(std::max(v, -thr), thr) / thr;
        if (a->mask) {
            const float m = a->mask[k % a->mask_cells];
            v = m * v + (1.0f - m) * a->init_lat[k];
        }
        x0[k] = v;
    }
    if (a->thr) *a->thr = thr;
    // the update
    float* lat = a->lat;
    std::vector<float> out(n);
    float next_sigma = sn;
    bool to_tmp = false;
    if (last) {
        for (uint64_t k = 0; k < n; ++k) out[k] = a->phase == 0 ? x0[k] : a->x0v[k];
    } else if (a->kind == 1) {  // Euler a
        const float up = orc_ancestral_sigma(sn, sigma, eta);
        const float down = std::sqrt(std::max(0.0f, sn * sn - up * up));
        const float ratio = down / sigma;
        for (uint64_t k = 0; k < n; ++k) out[k] = lat[k] + (lat[k] - x0[k]) * (ratio - 1.0f) + a->noise[k] * up;
    } else if (a->kind == 2) {  // Heun
        if (a->phase == 0) {
            for (uint64_t k = 0; k < n; ++k) out[k] = lat[k] + (lat[k] - x0[k]) / sigma * dt;
            to_tmp = true;
        } else {
            for (uint64_t k = 0; k < n; ++k)
                out[k] = lat[k] + 0.5f * ((lat[k] - a->x0v[k]) / sigma + (a->x_tmp[k] - x0[k]) / sn) * dt;
        }
    } else if (a->kind == 3) {  // LMS
        static const float coeff[4][4] = {
            {1.0f, 0.0f, 0.0f, 0.0f},
            {3.0f / 2.0f, -1.0f / 2.0f, 0.0f, 0.0f},
            {23.0f / 12.0f, -16.0f / 12.0f, 5.0f / 12.0f, 0.0f},
            {55.0f / 24.0f, -59.0f / 24.0f, 37.0f / 24.0f, -9.0f / 24.0f},
        };
        for (uint64_t k = 0; k < n; ++k) a->lms[0][k] = (lat[k] - x0[k]) / sigma;
        const float* cf = coeff[a->lms_count - 1];
        for (uint64_t k = 0; k < n; ++k) {
            float acc = 0.0f;
            for (int j = 0; j < a->lms_count; ++j) acc += cf[j] * a->lms[j][k];
            out[k] = lat[k] + dt * acc;
        }
    } else if (a->kind == 4 || a->kind == 5) {  // DPM2, DPM2 a
        float up = 0.0f, step = dt;
        if (a->kind == 5) {
            up = std::min(sn, orc_ancestral_sigma(sn, sigma, eta));
            step = std::sqrt(std::max(0.0f, sn * sn - up * up)) - sigma;
        }
        const float mid = sigma + 0.5f * step;
        if (a->phase == 0) {
            for (uint64_t k = 0; k < n; ++k) out[k] = lat[k] + (lat[k] - x0[k]) / sigma * (0.5f * step);
            to_tmp = true;
            next_sigma = mid;
        } else {
            for (uint64_t k = 0; k < n; ++k) {
                float v = lat[k] + (a->x_tmp[k] - x0[k]) / mid * step;
                if (a->kind == 5) v = v + a->noise[k] * up;  // (a + b) + c, left to right
                out[k] = v;
            }
        }
    } else if (a->kind == 6 || a->kind == 7) {  // DPM++ 2M, DPM++ 2S a
        float up = 0.0f, num = sn;
        if (a->kind == 7) {
            up = std::min(sn, orc_ancestral_sigma(sn, sigma, eta));
            num = std::sqrt(std::max(0.0f, sn * sn - up * up));
        }
        const double t_now = -std::log((double)sigma), t_n = -std::log((double)sn), h = t_n - t_now;
        if (!a->have_prev) {
            for (uint64_t k = 0; k < n; ++k) out[k] = (num / sigma) * lat[k] - std::expm1(-h) * x0[k];
        } else {
            const double r = (t_now - -std::log((double)a->sigma_prev)) / h;
            const float c0 = (float)(1.0 + 1.0 / (2.0 * r)), c1 = (float)(1.0 / (2.0 * r));
            for (uint64_t k = 0; k < n; ++k) {
                const float x0d = c0 * x0[k] - c1 * a->x0_prev[k];
                out[k] = (num / sigma) * lat[k] - std::expm1(-h) * x0d;
            }
        }
        if (a->kind == 7)
            for (uint64_t k = 0; k < n; ++k) out[k] += a->noise[k] * up;
        for (uint64_t k = 0; k < n; ++k) a->x0_prev[k] = x0[k];
    } else if (a->kind == 8) {  // DDIM
        for (uint64_t k = 0; k < n; ++k) out[k] = x0[k] + (sn / sigma) * (lat[k] - x0[k]);
    } else {  // Euler
        for (uint64_t k = 0; k < n; ++k) out[k] = lat[k] + (lat[k] - x0[k]) / sigma * dt;
    }
    float* dst = to_tmp ? a->x_tmp : lat;
    for (uint64_t k = 0; k < n; ++k) dst[k] = out[k];
    if (a->x_model && !last) {  // evalGuided's input scaling for the next evaluation
        const float inv = 1.0f / std::sqrt(next_sigma * next_sigma + 1.0f);
        for (uint64_t k = 0; k < n; ++k) a->x_model[k] = dst[k] * inv;
    }
    return 0;
}

}  // extern "C"
