/*
 * sdvk_cuda.h -- C ABI of the sdvk-b200 CUDA back end (libsdvk_b200.so).
 *
 * It replaces sdvk's Vulkan GPU module (src/Modules/GPU/: vk_engine, fused_attn, volk) for the
 * UNet transformer-block hot path: the Q8_0 dequant GEMMs and the fused attention.  Everything is
 * extern "C", takes plain pointers and sizes, never throws, and returns an int status
 * (SDVK_OK = 0).  Device pointers are CUDA device addresses obtained from sdvk_alloc() (or any
 * cudaMalloc'd memory on the context's device); host pointers are ordinary memory (pinned memory
 * from sdvk_host_alloc() makes the *_async copies truly asynchronous).
 *
 * Threading: one context per device per process; calls on a context are not thread-safe, matching
 * the reference's single-queue Engine (src/Modules/GPU/vk_engine.hpp:90-247).  Work is queued on
 * the context's stream in call order; stream order replaces the reference's hazard barriers
 * (vk_engine.cpp:1046-1126).
 *
 * Every entry point's comment names the reference interface it replaces (paths relative to the
 * sdvk project root).
 */
#ifndef SDVK_CUDA_H
#define SDVK_CUDA_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SDVK_API __attribute__((visibility("default")))
#else
#define SDVK_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------------------------- */
#define SDVK_OK 0
#define SDVK_E_OOM 1         /* device/host allocation failed (reference: OomError, vk_engine.hpp:30-32) */
#define SDVK_E_SHAPE 2       /* unsupported shape, stride or alignment */
#define SDVK_E_CUDA 3        /* a CUDA runtime/driver call failed (reference: VK_CHECK throw, vk_engine.cpp:33-41) */
#define SDVK_E_TIMEOUT 4     /* a kernel's bounded wait or sdvk_step_wait's deadline ran out */
#define SDVK_E_ARG 5         /* invalid argument (null pointer, bad dtype, bad push size) */
#define SDVK_E_KERNEL 6      /* sdvk_dispatch: unknown kernel name (reference exits, vk_engine.cpp:1147-1150) */
#define SDVK_E_STATE 7       /* step protocol misuse (e.g. step_end without step_begin) */
#define SDVK_E_NOT_FINITE 8  /* sdvk_check_finite found a NaN/Inf */

/* ---- element types ------------------------------------------------------------------------ */
#define SDVK_F32 0
#define SDVK_F16 1
#define SDVK_BF16 2

typedef struct sdvk_ctx sdvk_ctx;

/* A non-owning view of device memory: base + offset, size bytes.
 * Replaces BufRef{VkBuffer, offset, size} (src/Modules/GPU/vk_engine.hpp:21-25). */
typedef struct sdvk_buf {
    void* ptr;
    uint64_t offset;
    uint64_t size;
} sdvk_buf;

/* ---- context ------------------------------------------------------------------------------ */
/* Engine::init + setDeviceIndex (vk_engine.hpp:97-100, vk_engine.cpp:317-436). */
SDVK_API int sdvk_ctx_create(int device, sdvk_ctx** out);
/* Engine::destroy (vk_engine.hpp:101). */
SDVK_API int sdvk_ctx_destroy(sdvk_ctx* ctx);
/* Run subsequent work on a caller-owned cudaStream_t.  NULL is CUDA's legacy default stream, as
 * cudaStream_t 0 is everywhere (e.g. torch's default stream).  A new context runs on a private
 * non-blocking stream; sdvk_ctx_reset_stream() returns to it. */
SDVK_API int sdvk_ctx_set_stream(sdvk_ctx* ctx, void* cuda_stream);
SDVK_API int sdvk_ctx_reset_stream(sdvk_ctx* ctx);
SDVK_API void* sdvk_ctx_stream(sdvk_ctx* ctx);
/* Deadline for every bounded wait inside the kernels (default 2000 ms). */
SDVK_API int sdvk_ctx_set_timeout_ms(sdvk_ctx* ctx, uint32_t ms);
/* Arithmetic for fp32 inputs.  SDVK_PRECISION_REFERENCE (the default): attention on fp32 Q/K/V is
 * computed in fp32, within the reference's own 2e-5 bar (tests/fused_attn_test.cpp:123-124).
 * SDVK_PRECISION_FAST: fp32 Q/K/V are rounded to f16 for the tensor cores (about 3e-4).  The Q8
 * GEMMs run fp32 activations in tf32 in both modes; 16-bit inputs are unaffected. */
#define SDVK_PRECISION_REFERENCE 0
#define SDVK_PRECISION_FAST 1
SDVK_API int sdvk_ctx_set_precision(sdvk_ctx* ctx, int precision);
/* Human-readable device report (Engine::deviceReport, vk_engine.hpp:169). */
SDVK_API int sdvk_device_report(sdvk_ctx* ctx, char* buf, size_t len);
/* Free and total bytes of the context's device memory (Engine::deviceLocalMb, vk_engine.hpp:166). */
SDVK_API int sdvk_device_memory(sdvk_ctx* ctx, uint64_t* free_bytes, uint64_t* total_bytes);
/* Text of the last error on this context (empty when none). */
SDVK_API const char* sdvk_last_error(sdvk_ctx* ctx);
SDVK_API const char* sdvk_status_string(int status);

/* ---- memory ------------------------------------------------------------------------------- */
/* Arena::alloc (vk_engine.hpp:38, vk_engine.cpp:251-261): 256-byte aligned device memory. */
SDVK_API int sdvk_alloc(sdvk_ctx* ctx, uint64_t bytes, void** dptr);
SDVK_API int sdvk_free(sdvk_ctx* ctx, void* dptr);
/* Pinned host memory for the asynchronous copies (the reference's staging ring, vk_engine.hpp:150-153). */
SDVK_API int sdvk_host_alloc(sdvk_ctx* ctx, uint64_t bytes, void** hptr);
SDVK_API int sdvk_host_free(sdvk_ctx* ctx, void* hptr);
/* Engine::uploadNow / downloadNow (vk_engine.hpp:135, 146): synchronous copies. */
SDVK_API int sdvk_upload(sdvk_ctx* ctx, void* dst_dev, const void* src_host, uint64_t bytes);
SDVK_API int sdvk_download(sdvk_ctx* ctx, void* dst_host, const void* src_dev, uint64_t bytes);
/* Stream-ordered copies (the staged in-step uploads/readbacks, vk_engine.hpp:136-153). */
SDVK_API int sdvk_upload_async(sdvk_ctx* ctx, void* dst_dev, const void* src_host, uint64_t bytes);
SDVK_API int sdvk_download_async(sdvk_ctx* ctx, void* dst_host, const void* src_dev, uint64_t bytes);
/* Engine::copyBuf (vk_engine.hpp:115): stream-ordered device-to-device copy. */
SDVK_API int sdvk_copy(sdvk_ctx* ctx, void* dst_dev, const void* src_dev, uint64_t bytes);
/* Engine::fill (vk_engine.hpp:114): fill with a 32-bit pattern, bytes % 4 == 0. */
SDVK_API int sdvk_fill_u32(sdvk_ctx* ctx, void* dst_dev, uint32_t value, uint64_t bytes);

/* ---- step protocol ------------------------------------------------------------------------ */
/* Engine::beginStep / endStep / waitStep (vk_engine.hpp:109-117, vk_engine.cpp:930-950,
 * 1245-1295).  begin opens a step (kernels may be queued before it too), end records the step's
 * completion, wait blocks until it completes or timeout_ms passes (SDVK_E_TIMEOUT). */
SDVK_API int sdvk_step_begin(sdvk_ctx* ctx);
SDVK_API int sdvk_step_end(sdvk_ctx* ctx);
SDVK_API int sdvk_step_wait(sdvk_ctx* ctx, uint32_t timeout_ms);
/* Block until all queued work is done and report any device-side error (timeouts). */
SDVK_API int sdvk_synchronize(sdvk_ctx* ctx);
/* Failure-path self-test, no counterpart in the reference (whose waits are host fences,
 * vk_engine.cpp:1279): queues one kernel whose bounded wait can never complete (an mbarrier that
 * nothing arrives on), so the wait runs out after the context's timeout (sdvk_ctx_set_timeout_ms),
 * the kernel records a timeout in the device error word and returns, and the next synchronisation
 * reports SDVK_E_TIMEOUT.  No fault and no trap: the context stays usable afterwards. */
SDVK_API int sdvk_selftest_wait(sdvk_ctx* ctx);

/* ---- the reference's dispatch interface --------------------------------------------------- */
/* Engine::dispatch(kernel, bufs, push, gx, gy, gz) (vk_engine.hpp:111-112, vk_engine.cpp:1143-1180)
 * for the hot-path kernels, with the reference's binding order and push-constant layouts
 * (kernel table vk_engine.cpp:51-125).  All buffers hold fp32 data, as in the reference.
 *   "gemm_nt_q8", "gemm_nt_q8_v", "gemm_nt_q8_v_bm128", "gemm_nt_q8_v_bk32",
 *   "gemm_nt_q8_v_bm128_bk32"           bufs {A, Bq, C, S}        push Pg (48 B)
 *   "gemm_nt_q8_v_b", "gemm_nt_q8_v_bm128_b"  bufs {A, Bq, C, S, bias}  push Pg
 *   "gemm_nn_q8", "gemm_nn_q8_v"        bufs {Aq, B, C, S}        push Pg
 *   "fused_attn", "fused_attn_tiled"    bufs {Q, K, V, O}         push FaPush (36 B)
 *   "layernorm_fwd"                     bufs {X, gamma, beta, Y}  push {rows, d, eps, affine} (16 B)
 *   "groupnorm"                         bufs {X, gamma, beta, Y}  push {C, P, G, eps, act} (20 B)
 * and the rest of the table that the UNet walker, the generation loop and the unfused-attention
 * fallback dispatch (sdvkgen.cpp:912-1206, 1226-1281), so that code runs unchanged on this back end:
 *   "add2"          bufs {C, A, B}        push {n} (4 B)                     add2.comp
 *   "ew2"           bufs {C, A, B}        push {n, d0..d3, as0..3, bs0..3, mode} (56 B)  ew2.comp
 *   "copy_nd"       bufs {Dst, Src}       push Pnd (60 B)                    copy_nd.comp
 *   "unary_fwd"     bufs {X, Y}           push {n, mode} (8 B)               unary_fwd.comp
 *   "bias_add"      bufs {X, B}           push {C, P} (8 B)                  bias_add.comp
 *   "upsample2x"    bufs {X, Y}           push {C, H, W} (12 B)              upsample2x.comp
 *   "im2col"        bufs {X, Col}         push {C, H, W, row0, rows} (20 B)  im2col.comp
 *   "im2col_s2"     bufs {X, Col}         push {C, H, W, OH, OW, off} (24 B) im2col_s2.comp
 *   "gemm_nt", "gemm_nn"  bufs {A, B, C}  push Pg, fp32 operands, batch = gz  gemm_nt.comp, gemm_nn.comp
 *   "softmax_fwd"   bufs {X, Y}           push {rows, cols} (8 B)            softmax_fwd.comp
 *   "causal_mask"   bufs {S}              push {batch, rows, cols} (12 B)    causal_mask.comp
 * add2, ew2, copy_nd, unary_fwd and softmax_fwd accept the in-place aliasing the walker uses.
 * Pg = {M, N, K, mode, sA, sB, sC, batch, lda, ldb, ldc, pad} (sdvkgen.cpp:901-903);
 * Pnd = {n, d0..d3, os0..3, ss0..3, mode, scale} (sdvkgen.cpp:904-907);
 * FaPush = {Tq, Tk, C, heads, hd, causal, pad0, pad1, scale} (fused_attn.cpp:15-26).
 * The grid (gx, gy, gz) the caller computed for the Vulkan tiling is accepted and ignored: each
 * kernel covers the whole shape in the push constants with its own B200 tiling; for the fp32
 * GEMMs and the Q8 GEMMs the batch count is gz, the shaders' z workgroup range.
 * Deviations: Q8 kernels require K % 32 == 0 (whole Q8_0 blocks); attention requires hd <= 64.
 * Numerics: the GEMM runs the tensor cores in tf32 on fp32 activations; attention on the fp32
 * buffers follows sdvk_ctx_set_precision (fp32 arithmetic by default). */
SDVK_API int sdvk_dispatch(sdvk_ctx* ctx, const char* kernel, const sdvk_buf* bufs, uint32_t nbufs, const void* push,
                  uint32_t push_bytes, uint32_t gx, uint32_t gy, uint32_t gz);

/* fusedAttention(Engine&, FusedAttnArgs) (src/Modules/GPU/fused_attn.hpp:13-28,
 * fused_attn.cpp:40-61): fp32 Q/K/V/out, rows of C = heads*hd, scale 1/sqrt(hd).
 * Returns SDVK_E_SHAPE where the reference's fusedAttnSupported (fused_attn.cpp:34-38) is false. */
SDVK_API int sdvk_fused_attention(sdvk_ctx* ctx, const void* q, const void* k, const void* v, void* out, uint32_t Tq,
                         uint32_t Tk, uint32_t C, uint32_t heads, int causal);
/* fusedAttnSupported (fused_attn.cpp:34-38): 1 if hd = C/heads is in 1..64. */
SDVK_API int sdvk_fused_attn_supported(uint32_t C, uint32_t heads);

/* ---- typed hot-path entry points ---------------------------------------------------------- */
/* Q8_0 NT GEMM (gemm_nt_q8_v.comp:5-128 via gemmNtQ8 / gemmNtQ8Bias, sdvkgen.cpp:917-936):
 *   C[z][m][n] (=|+=) sum_k A[z][m][k] * q[n][k] * s[(n*K + k) >> 5] (+ bias[n])
 * A: a_dtype (F16, BF16 or F32), row stride lda, batch stride sA (elements).
 * q: int8 [N][K] (row stride K), s: fp32 per 32 elements, shared by all batches.
 * C: c_dtype (F32 or F16), row stride ldc, batch stride sC.  accumulate != 0 adds into C
 * (F32 only) and, unlike the reference's mode 1, also adds the bias when one is given.
 * Requirements: K % 32 == 0; 16-byte aligned base pointers; lda, ldc (in bytes) multiples of 16. */
SDVK_API int sdvk_gemm_q8_nt(sdvk_ctx* ctx, const void* A, int a_dtype, const int8_t* q, const float* s, const float* bias,
                    void* C, int c_dtype, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldc,
                    uint32_t batch, uint64_t sA, uint64_t sC, int accumulate);

/* Q8_0 NN GEMM (gemm_nn_q8_v.comp:5-110 via gemmNnQ8, sdvkgen.cpp:944-948; used by conv1 for
 * proj_in/proj_out, sdvkgen.cpp:1180-1189):
 *   C[z][m][n] (=|+=) sum_k q[z][m][k] * s[(z*sA + m*lda + k) >> 5] * B[z][k][n] (+ bias[m])
 * q: int8 [M][lda] weight (lda % 32 == 0, batch stride sA, 0 = shared), B: b_dtype [K][ldb]. */
SDVK_API int sdvk_gemm_q8_nn(sdvk_ctx* ctx, const int8_t* q, const float* s, const void* B, int b_dtype, const float* bias,
                    void* C, int c_dtype, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb,
                    uint32_t ldc, uint32_t batch, uint64_t sA, uint64_t sB, uint64_t sC, int accumulate);

/* Fused attention with explicit layout (generalises FusedAttnArgs, fused_attn.hpp:13-23, with a
 * batch dimension, strides and a caller-chosen scale; attnCore's fused branch, sdvkgen.cpp:1226-1238).
 * Element (b, h, t, d) of Q is at q[b*sq + h*hq + t*ldq + d] (same for K, V, O).  dtype applies to
 * Q/K/V (F16, BF16 or F32); o_dtype to O (F32 or F16).  hd <= 64. */
typedef struct sdvk_attn_desc {
    const void* q;
    const void* k;
    const void* v;
    void* o;
    int dtype;
    int o_dtype;
    uint32_t batch, heads, Tq, Tk, hd;
    uint64_t ldq, ldk, ldv, ldo;
    uint64_t sq, sk, sv, so;
    uint64_t hq, hk, hv, ho;
    float scale;
    int causal;
} sdvk_attn_desc;
SDVK_API int sdvk_attention(sdvk_ctx* ctx, const sdvk_attn_desc* desc);

/* ---- the transformer block and its non-GEMM operators --------------------------------------- */
/* LayerNorm over the last dim (layernorm_fwd.comp, dispatched by layernorm(), sdvkgen.cpp:1094-1103):
 * y[r][j] = (x[r][j] - mean_r) / sqrt(var_r + eps) * gamma[j] + beta[j], two-pass mean/variance.
 * x fp32 [rows][ldx]; y F32 or F16 [rows][ldy]; gamma/beta fp32 [d] or NULL (1 / 0).
 * Requirements: d, ldx, ldy multiples of 4, d <= 3072, 16-byte aligned bases. */
SDVK_API int sdvk_layernorm(sdvk_ctx* ctx, const float* x, const float* gamma, const float* beta, void* y, int y_dtype,
                   uint32_t rows, uint32_t d, uint64_t ldx, uint64_t ldy, float eps);
/* diffusers GEGLU on the ff.net.0.proj output (geglu(), sdvkgen.cpp:1710-1720): f16 h [rows][ldh]
 * holds [a | gate] of width 2F; y[r][j] = a[r][j] * gelu_erf(gate[r][j]), f16 [rows][ldy].
 * Requirements: F, ldh, ldy multiples of 8, 16-byte aligned bases. */
SDVK_API int sdvk_geglu(sdvk_ctx* ctx, const void* h, void* y, uint32_t rows, uint32_t F, uint64_t ldh, uint64_t ldy);

/* GEGLU folded into the ff.net.0 GEMM.  sdvk_geglu_interleave repacks an ff.net.0.proj weight
 * [2F][K] (+ scales, + optional bias; rows 0..F-1 = a, F..2F-1 = gate) into row order
 * [a 0..15, gate 0..15, a 16..31, gate 16..31, ...] -- a one-time load-time repack into the caller's
 * buffers of the same sizes.  sdvk_gemm_q8_nt_geglu then computes
 * C[m][j] = a[m][j] * gelu_erf(gate[m][j]) (f16 [M][ldc]) for (a | gate) = A . W^T (+ bias) with the
 * GEGLU applied to the fp32 accumulators, in place of gemm_nt_q8 + geglu (sdvkgen.cpp:1710-1720).
 * Requirements: F % 16 == 0, K % 32 == 0, 16-byte aligned rows. */
SDVK_API int sdvk_geglu_interleave(sdvk_ctx* ctx, const int8_t* q, const float* s, const float* bias, uint32_t F,
                          uint32_t K, int8_t* q_out, float* s_out, float* bias_out);
SDVK_API int sdvk_gemm_q8_nt_geglu(sdvk_ctx* ctx, const void* A, int a_dtype, const int8_t* q_interleaved,
                          const float* s_interleaved, const float* bias_interleaved, void* C, uint32_t M, uint32_t F,
                          uint32_t K, uint32_t lda, uint32_t ldc);

/* One Q8_0 linear layer: int8 weight [N][K] (row stride K), fp32 scale per 32 weights, optional
 * fp32 bias [N] (the loader's split layout, Gguf.cpp:559-583). */
typedef struct sdvk_q8_linear {
    const int8_t* q;
    const float* s;
    const float* bias;
} sdvk_q8_linear;

/* One SDXL BasicTransformerBlock (spatialTransformer's layer body, sdvkgen.cpp:1739-1763) over
 * `batch` images at once:
 *   x += attn1(LN1(x));  x += attn2(LN2(x), ctx);  x += ff2(geglu(ff1(LN3(x))))
 * where attnN = to_out(fusedAttention(to_q, to_k, to_v)) with heads of C/heads <= 64.
 * x: fp32 [batch][T][C], updated in place.  ctx: [batch][Tctx][Cctx] in ctx_dtype (F16, BF16, F32).
 * ff1 has 2*ff_inner rows ([a | gate]); ff2 has K = ff_inner.  Q/K/V (and attn2's K/V) run as one
 * GEMM when their weights (and biases) lie back to back in memory.  eps <= 0 means 1e-5.
 * The workspace (fp16 intermediates) is the caller's: sdvk_transformer_block_workspace() bytes,
 * 256-byte aligned.  No counterpart exists as one call in the reference, which dispatches the same
 * sequence kernel by kernel. */
typedef struct sdvk_block_desc {
    float* x;
    const void* ctx;
    int ctx_dtype;
    uint32_t batch, T, C, heads, Tctx, Cctx, ff_inner;
    const float *ln1_w, *ln1_b, *ln2_w, *ln2_b, *ln3_w, *ln3_b;
    sdvk_q8_linear q, k, v, o, q2, k2, v2, o2, ff1, ff2;
    float eps;
    uint32_t ff1_geglu_interleaved;  /* ff1 was repacked by sdvk_geglu_interleave: GEGLU in its epilogue */
} sdvk_block_desc;
SDVK_API uint64_t sdvk_transformer_block_workspace(const sdvk_block_desc* desc);
SDVK_API int sdvk_transformer_block(sdvk_ctx* ctx, const sdvk_block_desc* desc, void* workspace, uint64_t workspace_bytes);

/* The same block with no workspace argument and no allocation of any kind: the intermediates live
 * in a fixed device scratch array compiled into the library, SDVK_STATIC_SCRATCH_BYTES per device.
 * A shape whose sdvk_transformer_block_workspace() exceeds it returns SDVK_E_SHAPE (one 1024-token
 * image at C = 1280 fits; the batch-2 config does not).  The array is shared by every call on a
 * device: calls that can overlap in time on one device (other streams, threads or contexts) race on
 * it, and the caller must serialise them.  The array's address is looked up on the first call on
 * each device (and again after the device's CUDA context is recreated, e.g. by cudaDeviceReset);
 * make that first call before any stream capture begins.
 * No counterpart in the reference (it dispatches the block kernel by kernel into its step arena). */
#define SDVK_STATIC_SCRATCH_BYTES (64ull << 20)
SDVK_API int sdvk_transformer_block_static(sdvk_ctx* ctx, const sdvk_block_desc* desc);

/* ---- multi-GPU: the CFG pair ----------------------------------------------------------------- */
/* Classifier-free guidance combine on the device (evalGuided, sdvkgen.cpp:3825-3845):
 *   out = uncond + cfg * (cond - uncond); with rescale > 0 the result's spread is pulled toward the
 *   unconditional output's: er = (out - mean) * std(uncond) / (std(out) + 1e-6) + mean,
 *   out = rescale * er + (1 - rescale) * out (statistics in double).  fp32 [n] each. */
SDVK_API int sdvk_cfg_combine(sdvk_ctx* ctx, const float* cond, const float* uncond, float* out, uint64_t n, float cfg,
                     float rescale);

/* ---- the sampler step on the device ------------------------------------------------------- */
/* Sampler kinds, numbered as SamplerKind (src/Modules/Diffusion/GenParams.hpp:16-26). */
#define SDVK_SAMPLER_EULER 0
#define SDVK_SAMPLER_EULER_A 1
#define SDVK_SAMPLER_HEUN 2
#define SDVK_SAMPLER_LMS 3
#define SDVK_SAMPLER_DPM2 4
#define SDVK_SAMPLER_DPM2_A 5
#define SDVK_SAMPLER_DPMPP_2M 6
#define SDVK_SAMPLER_DPMPP_2S_A 7
#define SDVK_SAMPLER_DDIM 8

/* One model evaluation's share of the generation loop (sdvkgen.cpp:3759-4021), replacing the host
 * code between downloadNow of the model output and uploadNow of the next model input:
 *   evalGuided (:3811-3846)  non-finite check, res = u + cfg * (c - u), optional spread rescale;
 *   x0FromEps (:3770-3776) and finishX0 (:3779-3797)  x0, dynamic threshold, inpaint blend;
 *   the sampler update (:3859-4019)  phase 0 after the step's first evaluation, phase 1 after the
 *   second one of Heun, DPM2 and DPM2 a (phase 0 of those writes x_tmp, the latent of the second
 *   evaluation); the last step (sigma_next <= 0) returns x0.
 * All buffers are fp32 device memory of n floats.  Results equal the host loop's bit for bit,
 * except with rescale > 0, whose double-precision sums are added in another order (a result may
 * move by one ulp).  A NaN/Inf in eps_c or eps_u leaves lat unchanged and makes the next
 * synchronising call return SDVK_E_NOT_FINITE (the reference stops the generation there). */
typedef struct sdvk_sampler_step_desc {
    int32_t kind;            /* SDVK_SAMPLER_* */
    int32_t phase;           /* 0, or 1 for the second evaluation of Heun, DPM2, DPM2 a */
    uint64_t n;              /* latent floats */
    const float* eps_c;      /* conditional model output */
    const float* eps_u;      /* unconditional model output, or NULL when guidance is off (cfg <= 1.0001) */
    float cfg, rescale;      /* guidance scale; CFG rescale ("mimic scale") factor, 0 = off */
    int32_t vpred;           /* v-prediction model */
    int32_t dynthresh;       /* dynamic thresholding at the 99.5th percentile of |x0| */
    const float* mask;       /* inpaint mask, mask_cells values indexed by k % mask_cells, or NULL */
    uint64_t mask_cells;
    const float* init_lat;   /* the encoded init latent the mask blends toward */
    float* lat;              /* the latent: read, and replaced by the step's result (phase 0 of a
                                two-evaluation sampler leaves it and writes x_tmp) */
    float* x_tmp;            /* two-evaluation samplers: the second evaluation's latent */
    float* x0;               /* out: this evaluation's finished x0 */
    const float* x0v;        /* phase 1: the step's first x0 (phase 0's x0 output) */
    float* x0_prev;          /* DPM++ samplers: the previous step's x0 (read when have_prev), then this step's */
    float* lms[4];           /* LMS: derivative history, newest first; lms[0] receives this step's */
    int32_t lms_count;       /* LMS: history entries including this step's (1..4) */
    const float* noise;      /* ancestral samplers: n standard normals for this step (the reference's
                                nd(rng) draws, in index order) */
    float sigma, sigma_next; /* the step's sigmas (sch.sigmas[i], sch.sigmas[i + 1]) */
    float eta;               /* p.eta (0 selects 1) */
    float sigma_prev;        /* DPM++ with have_prev: the previous step's sigma */
    int32_t have_prev;
    float* x_model;          /* optional: the next evaluation's model input, its latent * 1/sqrt(sigma'^2 + 1) */
    float* thr;              /* optional, device: the dynamic threshold used (1 without dynthresh) */
} sdvk_sampler_step_desc;

SDVK_API int sdvk_sampler_step(sdvk_ctx* ctx, const sdvk_sampler_step_desc* desc);

/* out = x * 1/sqrt(sigma^2 + 1): the scaled model input of a step's first evaluation
 * (sdvkgen.cpp:3808-3809). */
SDVK_API int sdvk_sampler_scale(sdvk_ctx* ctx, const float* x, float* out, uint64_t n, float sigma);

/* ---- model loading and the ResBlock's normalisation ---------------------------------------- */
/* GGUF Q8_0 ingest on the device (GgufFile::readQ8Into, src/Modules/Model/Gguf.cpp:559-583, and
 * fp16ToFp32, Gguf.cpp:11-35).  blocks: the tensor's raw data in device memory, rows x cols values
 * as rows*cols/32 blocks of 34 bytes (little-endian binary16 d, then 32 x int8), 2-byte aligned.
 * Writes q[row*ldq + k] and scales[row*(ldq/32) + k/32] (fp32, converted exactly): the layout the
 * Q8 entry points take, bit-identical to the reference loader's for ldq = cols (ldq = 0 means cols).
 * cols % 32 == 0, ldq % 32 == 0 (SDVK_E_SHAPE otherwise).  No counterpart in the reference's GPU
 * module: it replaces the host-side split when the raw blocks are uploaded as they are. */
SDVK_API int sdvk_q8_0_ingest(sdvk_ctx* ctx, const void* blocks, uint64_t rows, uint64_t cols, int8_t* q,
                              uint64_t ldq, float* scales);
/* 3x3 convolution with a Q8_0 weight (conv3RawInto / conv3s2, sdvkgen.cpp:1133-1175: im2col.comp or
 * im2col_s2.comp, then gemmNnQ8 with ldc = P, then biasAddCh).  x: x_dtype (F16, BF16 or F32)
 * [batch][cin][H][W]; q: int8 [cout][cin*9] (k = c*9 + ky*3 + kx; cin*9 % 32 == 0) with fp32 scales
 * per 32; bias fp32 [cout] or NULL; y: y_dtype (F32 or F16) [batch][cout][OH][OW].  stride 1 pads
 * 1 on every side (OH = H); stride 2 gives OH = H/2, OW = W/2 with pad_off -1 (symmetric ring, the
 * UNet downsamplers) or 0 (right/bottom only, the VAE encoder).  F32 input runs the GEMM in tf32.
 * workspace: device memory for the column matrix, 16-byte aligned; sdvk_conv3x3_workspace gives the
 * size of one whole image's (any smaller size that holds one band of output rows works, in bands). */
SDVK_API uint64_t sdvk_conv3x3_workspace(uint32_t cin, uint32_t H, uint32_t W, int stride, int x_dtype);
SDVK_API int sdvk_conv3x3_q8(sdvk_ctx* ctx, const void* x, int x_dtype, const int8_t* q, const float* s,
                             const float* bias, void* y, int y_dtype, uint32_t batch, uint32_t cin, uint32_t cout,
                             uint32_t H, uint32_t W, int stride, int pad_off, void* workspace, uint64_t workspace_bytes);
/* The same convolution as an implicit GEMM, without the column matrix: TMA im2col-mode loads read the
 * input windows from a channels-last fp16 x [batch][H][W][cin] (replacing im2col.comp + gemmNnQ8 in
 * conv3RawInto / conv3s2, sdvkgen.cpp:1133-1175).  sdvk_conv3x3_q8 takes this form by itself for an F16
 * input when sdvk_conv3x3_implicit_ok holds and its workspace holds x channels-last and the repacked
 * weights: batch*cin*H*W*2 bytes rounded up to 256, then cout*cin*9*2 (the im2col size of one image
 * holds both for the UNet's shapes).  Results agree with the im2col form up to fp32 summation order.
 * sdvk_conv3x3_implicit_ok: 1 when cin % 64 == 0, OH*OW % 128 == 0, stride is 1 or 2, the input has at
 *   least 128 KB and the environment variable SDVK_CONV_IMPLICIT is not "0"; else 0.
 * sdvk_conv3x3_weights_f16: w16, fp16 [cout][cin*9], 16-byte aligned, gets
 *   w16[o][(cb*9 + tap)*64 + j] = q[o][(cb*64 + j)*9 + tap] * scale rounded to fp16 (the value the Q8_0
 *   GEMMs' dequantiser produces; 64-channel blocks cb, tap = ky*3 + kx).  cin % 64 == 0.
 * sdvk_conv3x3_nhwc: y (y_dtype F32 or F16, [batch][cout][OH][OW] channel-major, 16-byte aligned) =
 *   conv(x, w16) + bias[b*bias_stride + o] (bias fp32 or NULL), or += with accumulate (F32 y only).
 *   SDVK_E_SHAPE when sdvk_conv3x3_implicit_ok does not hold. */
SDVK_API int sdvk_conv3x3_implicit_ok(uint32_t batch, uint32_t cin, uint32_t H, uint32_t W, int stride);
SDVK_API int sdvk_conv3x3_weights_f16(sdvk_ctx* ctx, const int8_t* q, const float* s, uint32_t cout, uint32_t cin,
                                      void* w16);
SDVK_API int sdvk_conv3x3_nhwc(sdvk_ctx* ctx, const void* x, const void* w16, const float* bias, uint64_t bias_stride,
                               int accumulate, void* y, int y_dtype, uint32_t batch, uint32_t cin, uint32_t cout,
                               uint32_t H, uint32_t W, int stride, int pad_off);
/* GroupNorm over x[batch][C][P] (channel-major, P = H*W) with G groups of C/G channels
 * (groupnorm.comp, gnInto sdvkgen.cpp:1105-1113; the reference runs batch 1): per (image, group)
 * mean and population variance, y = (x - mean)/sqrt(var + eps)*gamma[c] + beta[c], then
 * y/(1 + e^-y) when silu != 0.  fp32 in and out; y may alias x.  workspace: device memory of at
 * least sdvk_groupnorm_workspace(batch, C, P, G) bytes, 16-byte aligned.
 * sdvk_groupnorm_cl: the same values as fp16, channels-last y[batch][P][C] (C % 32 == 0; y must not
 * alias x): the layout sdvk_conv3x3_nhwc reads. */
SDVK_API uint64_t sdvk_groupnorm_workspace(uint32_t batch, uint32_t C, uint32_t P, uint32_t G);
SDVK_API int sdvk_groupnorm(sdvk_ctx* ctx, const float* x, const float* gamma, const float* beta, float* y,
                            uint32_t batch, uint32_t C, uint32_t P, uint32_t G, float eps, int silu, void* workspace,
                            uint64_t workspace_bytes);
SDVK_API int sdvk_groupnorm_cl(sdvk_ctx* ctx, const float* x, const float* gamma, const float* beta, void* y,
                               uint32_t batch, uint32_t C, uint32_t P, uint32_t G, float eps, int silu, void* workspace,
                               uint64_t workspace_bytes);

/* An NCCL communicator for the context's device.  The reference runs both CFG passes on one device
 * (runPass twice, sdvkgen.cpp:3812-3813); with a GPU pair each rank runs one pass and the halves
 * meet by all-gather.  The unique id (SDVK_COMM_ID_BYTES) is made on one rank and passed to the
 * others out of band.  Creation and every wait poll the communicator against timeout_ms: a peer
 * that never joins or stops answering aborts the communicator and returns SDVK_E_TIMEOUT.  The
 * first collective connects the peers and waits for all of them to reach it, under the same
 * creation deadline; later enqueues use the context's timeout (sdvk_ctx_set_timeout_ms).
 * NCCL itself is loaded on first use (libnccl.so.2); without it these calls return SDVK_E_CUDA. */
#define SDVK_COMM_ID_BYTES 128
typedef struct sdvk_comm sdvk_comm;
SDVK_API int sdvk_comm_unique_id(void* id);
SDVK_API int sdvk_comm_create(sdvk_ctx* ctx, int nranks, int rank, const void* id, uint32_t timeout_ms, sdvk_comm** out);
SDVK_API int sdvk_comm_destroy(sdvk_comm* comm);
SDVK_API int sdvk_comm_abort(sdvk_comm* comm);
/* recv[r * count + i] = rank r's send[i], queued on the context's stream. */
SDVK_API int sdvk_allgather(sdvk_ctx* ctx, sdvk_comm* comm, const void* send, void* recv, uint64_t count, int dtype);
/* Wait for the context's stream (the queued collectives) with the communicator's health polled. */
SDVK_API int sdvk_comm_wait(sdvk_ctx* ctx, sdvk_comm* comm, uint32_t timeout_ms);

/* NaN/Inf check of n fp32 or f16 values (the reference aborts on a non-finite UNet output,
 * sdvkgen.cpp:3819-3823): returns SDVK_E_NOT_FINITE if any value is not finite. */
SDVK_API int sdvk_check_finite(sdvk_ctx* ctx, const void* x, int dtype, uint64_t n);

/* ---- the whole SDXL UNet pass ------------------------------------------------------------- */
/* unetForward (src/Modules/Diffusion/sdvkgen.cpp:1875-1973) with resBlock (:1669-1707),
 * spatialTransformer (:1722-1777), concatCh (:1791-1796) and buildTemb (:1982-1995), over `batch`
 * images in one pass (the reference runs the CFG halves as two batch-1 passes).  The UNet owns its
 * parameters (one device arena, each tensor under the reference checkpoint's LDM name, e.g.
 * "input_blocks.4.1.transformer_blocks.0.attn1.to_q.weight"; conv weights are [cout][cin*9]) and a
 * workspace sized at creation for the given batch and latent size.
 *   x:         fp32 [batch][4][H][W] latent (the scaled model input)
 *   timesteps: fp32 [batch] (the sinusoidal embedding of timeEmbHost is computed on the device)
 *   adm:       fp32 [batch][adm_dim] (pooled text embedding + size conditioning, as buildTemb concatenates)
 *   context:   [batch][Tctx][ctx_dim] in ctx_dtype (F16, BF16 or F32)
 *   out:       fp32 [batch][4][H][W]
 * SDXL: model_ch {320, 640, 1280}, depth {0, 2, 10}, ctx_dim 2048, adm_dim 2816, temb_dim 1280,
 * head_dim 64, Tctx 77.  H and W must be multiples of 4.  The latent's 4 input channels run as 32
 * (zero-padded): "input_blocks.0.0.weight" is [ch0][32*9] and its columns past 4*9 must stay zero.
 * After parameters change, sdvk_unet_prepare redoes the load-time repacks (GEGLU interleave).
 * Every pass of one UNet uses the same workspace (fixed addresses, so a captured pass replays): passes
 * of one UNet that can overlap on the GPU race; run them on one stream, or create a UNet per stream.
 * The context must be on the device the UNet was created on (SDVK_E_ARG otherwise). */
typedef struct sdvk_unet sdvk_unet;
typedef struct sdvk_unet_desc {
    uint32_t model_ch[3];
    uint32_t depth[3];
    uint32_t ctx_dim, adm_dim, temb_dim, head_dim, Tctx;
    uint32_t batch, H, W;
} sdvk_unet_desc;
#define SDVK_UNET_Q8 0  /* int8 [rows][cols] + fp32 scale per 32 */
#define SDVK_UNET_F32 1 /* fp32 [rows] */
typedef struct sdvk_unet_tensor_info {
    const char* name; /* names in parentheses are internal groups and repacks */
    int kind;
    uint32_t rows, cols;
    int8_t* q;
    float* s;
    float* f;
} sdvk_unet_tensor_info;
SDVK_API int sdvk_unet_create(sdvk_ctx* ctx, const sdvk_unet_desc* desc, sdvk_unet** out);
/* The same UNet without device memory or a device (host only): its parameter table (null pointers),
 * FLOP, launch count and the device bytes sdvk_unet_create would allocate.  Forward, init and prepare
 * return SDVK_E_STATE on it. */
SDVK_API int sdvk_unet_plan(const sdvk_unet_desc* desc, sdvk_unet** out);
SDVK_API int sdvk_unet_destroy(sdvk_unet* unet);
/* Seeded random parameters: Q8_0 weights int8 uniform in [-127, 127] with binary16 scales
 * |N(0, 0.02)|/127, linear and conv biases uniform in [-0.02, 0.02], norm weights 1 and biases 0. */
SDVK_API int sdvk_unet_init_random(sdvk_ctx* ctx, sdvk_unet* unet, uint64_t seed);
SDVK_API int sdvk_unet_prepare(sdvk_ctx* ctx, sdvk_unet* unet);
SDVK_API uint32_t sdvk_unet_tensor_count(const sdvk_unet* unet);
SDVK_API int sdvk_unet_tensor(const sdvk_unet* unet, uint32_t index, sdvk_unet_tensor_info* out);
/* Where a tensor lives in the parameter arena (a plan has the same layout): byte offsets of its int8
 * payload and fp32 scales (Q8) or of its values (F32), and how sdvk_unet_init_random fills it.
 * The seeded values depend only on the seed and these offsets: payload byte i of the arena is
 * int8 (mix64(seed ^ i * 0xD1B54A32D192ED03) % 255) - 127; scale j (counted from the first Q8
 * tensor's scales) is binary16(|Box-Muller normal| * 0.02 / 127) from mix64((seed ^ 0x5CA1E) ^
 * j * 0x8CB92BA72F3D8DD7); F32 tensor number t (init 2) holds 0.02 * (2 u - 1) from
 * mix64((seed + 1000003 t) ^ e * 0xA24BAED4963EE407), with mix64 the SplitMix64 finaliser.  A host
 * program can therefore rebuild the same parameters (a GGUF for another engine, for instance). */
typedef struct sdvk_unet_param_layout {
    uint64_t q_off, s_off, f_off;
    int init; /* F32: 0 ones, 1 zeros, 2 uniform [-0.02, 0.02]; -1: filled through its group or a repack */
} sdvk_unet_param_layout;
SDVK_API int sdvk_unet_tensor_layout(const sdvk_unet* unet, uint32_t index, sdvk_unet_param_layout* out);
/* Algorithmic FLOP of one pass (GEMMs, convolutions at their real input channels, attention). */
SDVK_API uint64_t sdvk_unet_flops(const sdvk_unet* unet);
SDVK_API uint64_t sdvk_unet_workspace_bytes(const sdvk_unet* unet);
SDVK_API uint64_t sdvk_unet_parameter_bytes(const sdvk_unet* unet);
/* Kernel launches of one pass (this library's kernels; the concat copies are not counted). */
SDVK_API uint64_t sdvk_unet_launches(const sdvk_unet* unet);
SDVK_API int sdvk_unet_forward(sdvk_ctx* ctx, sdvk_unet* unet, const float* x, const float* timesteps, const float* adm,
                               const void* context, int ctx_dtype, float* out);

#ifdef __cplusplus
}
#endif

#endif /* SDVK_CUDA_H */
