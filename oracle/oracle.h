/*
 * oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the sdvk hot-path arithmetic (Q8_0 GEMMs, fused attention, block glue) plus
 * fp64 "truth" references and the seeded input generators.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline leg may load this library, and only as the checker / the timed CPU
 * baseline -- never as the product path.  The product (sdvk_b200/) never links or loads it.
 *
 * Parity is pinned two ways (see oracle/Makefile, target `ref`):
 *   - the reference's own test harnesses tests/fused_attn_test.cpp and tests/gemm_q8_bench.cpp are
 *     compiled from the reference sources against a host-memory stub Engine whose "device" is this
 *     restatement; their own fp64/fp32 CPU references and pass bars check it;
 *   - the reference GGUF reader src/Modules/Model/Gguf.cpp is compiled unchanged and decodes Q8_0
 *     files written by orc_gguf_write_q8(); its output must equal orc_q8_0_split_blocks() bit for bit.
 */
#pragma once
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- reference-compatible RNG (std::mt19937 + libstdc++ distributions, as the reference tests) */
void* orc_mt19937_new(uint32_t seed);
void orc_mt19937_free(void* h);
void orc_mt19937_uniform_f32(void* h, float lo, float hi, float* out, uint64_t n);
void orc_mt19937_uniform_int(void* h, int32_t lo, int32_t hi, int32_t* out, uint64_t n);

/* ---- counter-based synthetic inputs (SplitMix64 hash + Box-Muller in double) ------------------ */
void orc_normal_f32(uint64_t seed, uint64_t stream, float std_dev, float* out, uint64_t n);
void orc_normal_f16(uint64_t seed, uint64_t stream, float std_dev, uint16_t* out, uint64_t n);
/* Q8_0 weights of BASELINE config 0: int8 U[-127,127], fp16 scale = |N(0,0.02)|/127 per 32-block.
 * scale_f32 receives the exact fp32 value of each fp16 scale (what the reference loader uploads). */
void orc_q8_weights(uint64_t seed, uint64_t stream, uint64_t rows, uint64_t cols, int8_t* q,
                    uint16_t* scale_f16, float* scale_f32);

/* ---- fp16 <-> fp32 (IEEE binary16, round-to-nearest-even) ------------------------------------ */
void orc_f32_to_f16(const float* in, uint16_t* out, uint64_t n);
void orc_f16_to_f32(const uint16_t* in, float* out, uint64_t n);

/* ---- GGUF Q8_0 codec (34-byte blocks: fp16 d, 32 x int8) ------------------------------------- */
void orc_q8_0_pack_blocks(const int8_t* q, const uint16_t* d, uint64_t nblocks, uint8_t* blocks);
void orc_q8_0_split_blocks(const uint8_t* blocks, uint64_t nblocks, int8_t* q, float* scales);
int orc_gguf_write_q8(const char* path, const char* name, uint64_t rows, uint64_t cols,
                      const uint8_t* blocks);

/* ---- Q8_0 GEMMs: fp32 restatement of the shaders, and fp64 truth ------------------------------ */
/* C[M,N] (=|+=) A[M,K] . (q[N,K]*s)^T (+bias), gemm_nt_q8_v.comp semantics.  ld*=0 means packed. */
void orc_gemm_nt_q8_shader(const float* A, const int8_t* q, const float* s, const float* bias,
                           float* C, uint32_t M, uint32_t N, uint32_t K, uint32_t mode,
                           uint32_t sA, uint32_t sC, uint32_t batch, uint32_t lda, uint32_t ldc);
void orc_gemm_nt_q8_f64(const float* A, const int8_t* q, const float* s, const float* bias,
                        double* C, uint32_t M, uint32_t N, uint32_t K, uint32_t sA, uint32_t sC,
                        uint32_t batch, uint32_t lda, uint32_t ldc);
/* C[M,N] (=|+=) (q[M,K]*s) . B[K,N], gemm_nn_q8_v.comp semantics (weight is the M operand). */
void orc_gemm_nn_q8_shader(const int8_t* q, const float* s, const float* B, float* C, uint32_t M,
                           uint32_t N, uint32_t K, uint32_t mode, uint32_t sA, uint32_t sB,
                           uint32_t sC, uint32_t batch, uint32_t lda, uint32_t ldb, uint32_t ldc);
void orc_gemm_nn_q8_f64(const int8_t* q, const float* s, const float* B, double* C, uint32_t M,
                        uint32_t N, uint32_t K, uint32_t sB, uint32_t sC, uint32_t batch,
                        uint32_t lda, uint32_t ldb, uint32_t ldc);

/* ---- fused attention: [Tq,C] x [Tk,C] x [Tk,C] -> [Tq,C], head h at columns h*hd.. ---------- */
int orc_attn_tiled_shader(const float* Q, const float* K, const float* V, float* O, uint32_t Tq,
                          uint32_t Tk, uint32_t C, uint32_t heads, uint32_t causal, float scale);
int orc_attn_simple_shader(const float* Q, const float* K, const float* V, float* O, uint32_t Tq,
                           uint32_t Tk, uint32_t C, uint32_t heads, uint32_t causal, float scale);
/* fusedAttention(): kernel choice and scale exactly as the reference operator. */
int orc_fused_attention(const float* Q, const float* K, const float* V, float* O, uint32_t Tq,
                        uint32_t Tk, uint32_t C, uint32_t heads, uint32_t causal, int force_simple);
/* fp64 online-softmax truth with explicit row strides (elements) and batch strides. */
void orc_attn_f64(const float* Q, const float* K, const float* V, double* O, uint32_t batch,
                  uint32_t Tq, uint32_t Tk, uint32_t heads, uint32_t hd, uint64_t ldq,
                  uint64_t ldk, uint64_t ldv, uint64_t ldo, uint64_t sQ, uint64_t sK, uint64_t sV,
                  uint64_t sO, uint32_t causal, double scale);

/* ---- block glue ------------------------------------------------------------------------------ */
void orc_layernorm_shader(const float* x, const float* gamma, const float* beta, float* y,
                          uint32_t rows, uint32_t d, float eps, uint32_t affine);
/* groupnorm.comp:12-39 (batch 1): x[C][P], G groups; act 1 = fused SiLU. */
void orc_groupnorm_shader(const float* x, const float* gamma, const float* beta, float* y, uint32_t C,
                          uint32_t P, uint32_t G, float eps, uint32_t act);
void orc_layernorm_f64(const double* x, const float* gamma, const float* beta, double* y,
                       uint32_t rows, uint32_t d, double eps);
void orc_gelu_erf_shader(const float* x, float* y, uint64_t n);
void orc_cfg_combine(const float* cond, const float* uncond, float* out, uint64_t n, float cfg, float rescale);

/* One model evaluation of the generation loop (src/Modules/Diffusion/sdvkgen.cpp:3759-4021): the
 * guidance combine and rescale, x0FromEps, finishX0 and the sampler update, sequentially in the
 * host loop's order.  Field meanings as sdvk_sampler_step_desc (include/sdvk_cuda.h).  Returns the
 * number of non-finite model outputs (then nothing is written). */
typedef struct orc_sampler_args {
    int32_t kind, phase;
    uint64_t n;
    const float* eps_c;
    const float* eps_u;
    float cfg, rescale;
    int32_t vpred, dynthresh;
    const float* mask;
    uint64_t mask_cells;
    const float* init_lat;
    float* lat;
    float* x_tmp;
    float* x0;
    const float* x0v;
    float* x0_prev;
    float* lms[4];
    int32_t lms_count;
    const float* noise;
    float sigma, sigma_next, eta, sigma_prev;
    int32_t have_prev;
    float* x_model;
    float* thr;
} orc_sampler_args;
uint64_t orc_sampler_eval(const orc_sampler_args* a);

/* ---- the rest of the reference's kernel table (refkernels.cpp) -------------------------------- */
/* Push-constant blocks as the walker fills them (Pg, Pnd: sdvkgen.cpp:901-907; the ew2 block of mul2 :1003-1019). */
typedef struct orc_pg {
    uint32_t M, N, K, mode, sA, sB, sC, batch, lda, ldb, ldc, pad;
} orc_pg;
typedef struct orc_pnd {
    uint32_t n, d0, d1, d2, d3, os0, os1, os2, os3, ss0, ss1, ss2, ss3, mode;
    float scale;
} orc_pnd;
typedef struct orc_pew2 {
    uint32_t n, d0, d1, d2, d3, as0, as1, as2, as3, bs0, bs1, bs2, bs3, mode;
} orc_pew2;
void orc_add2_shader(float* c, const float* a, const float* b, uint32_t n);
void orc_bias_add_shader(float* x, const float* b, uint32_t C, uint32_t P);
void orc_copy_nd_shader(float* d, const float* s, const orc_pnd* p);
void orc_ew2_shader(float* c, const float* a, const float* b, const orc_pew2* p);
void orc_unary_shader(const float* x, float* y, uint32_t n, uint32_t mode);
void orc_upsample2x_shader(const float* x, float* y, uint32_t C, uint32_t H, uint32_t W);
void orc_im2col_shader(const float* x, float* col, uint32_t C, uint32_t H, uint32_t W, uint32_t row0, uint32_t rows);
void orc_im2col_s2_shader(const float* x, float* col, uint32_t C, uint32_t H, uint32_t W, uint32_t OH, uint32_t OW,
                          int32_t off);
/* nt = 1: gemm_nt.comp, nt = 0: gemm_nn.comp; batch = the dispatch's z extent. */
void orc_gemm_fp32_shader(int nt, const float* A, const float* B, float* C, const orc_pg* p, uint32_t batch);
void orc_softmax_shader(const float* x, float* y, uint32_t rows, uint32_t cols);
void orc_causal_mask_shader(float* s, uint32_t batch, uint32_t rows, uint32_t cols);

/* ---- the generation loop's host arithmetic ---------------------------------------------------- */
/* std::mt19937(seed) + one std::normal_distribution<float>(0, 1) for the whole run (the latent and
 * the ancestral draws continue one sequence). */
void* orc_gen_rng_new(uint32_t seed);
void orc_gen_rng_free(void* h);
void orc_gen_rng_normal(void* h, float* out, uint64_t n);
/* buildEuler: steps timesteps and steps + 1 sigmas; returns the initial noise sigma. */
float orc_euler_schedule(int steps, int trailing, int numTrain, int offset, int zsnr, float* timesteps, float* sigmas);

/* ---- the seeded UNet parameters of sdvk_unet_init_random, rebuilt on the host ---------------- */
void orc_unet_rand_q8(uint64_t seed, uint64_t first, uint64_t n, int8_t* out);
void orc_unet_rand_scale(uint64_t seed, uint64_t first, uint64_t n, float* out);
void orc_unet_rand_f32(uint64_t seed, uint32_t t, int init, uint64_t n, float* out);

/* ---- misc ------------------------------------------------------------------------------------ */
int orc_num_threads(void);
void orc_set_num_threads(int n);

#ifdef __cplusplus
}
#endif
