// block.cu -- the SDXL BasicTransformerBlock on the B200 (the body of spatialTransformer's layer
// loop, src/Modules/Diffusion/sdvkgen.cpp:1739-1763) and its two non-GEMM kernels:
//   layernorm_kernel  LayerNorm over the last dim (layernorm_fwd.comp): mean, then the centred sum
//                     of squares (two-pass), y = (x - mean) / sqrt(var + eps) * gamma + beta
//   geglu_kernel      diffusers GEGLU on the ff.net.0.proj output (sdvkgen.cpp:1710-1720):
//                     y = h[:, :F] * gelu(h[:, F:]), erf-GELU by Abramowitz & Stegun 7.1.26 as
//                     unary_fwd.comp:29-35 computes it
// Both are HBM-bound: one pass over their inputs, 16-byte vector accesses, grids sized to the SMs.
//
// The block driver launches, on the context's stream (capturable in one CUDA graph):
//   n = LN1(x); [q|k|v] = n Wqkv^T; a = attn(q, k, v); x += a Wo^T + bo
//   n = LN2(x); q = n Wq2^T; [k|v] = ctx Wkv2^T; a = attn(q, k, v); x += a Wo2^T + bo2
//   n = LN3(x); g = n Wff1^T + b1; h = geglu(g); x += h Wff2^T + b2
//   (with a GEGLU-interleaved ff1 weight the middle two are one GEMM whose epilogue writes h)
// x is the fp32 residual stream [batch][T][C], updated in place by the accumulating GEMMs; every
// intermediate is fp16 in the caller's workspace.  The context's K|V projection depends on ctx
// alone and runs on the context's side stream (fork/join events), overlapping the self-attention half.  Q/K/V (and the cross K/V) run as one GEMM when
// their weights lie back to back in memory (a [3C][C] weight), else as separate GEMMs writing the
// column blocks of the same [rows][3C] buffer.
#include <cmath>

#include "backend.hpp"
#include "gemm_q8.cuh"  // gelu_erf_as
#include "ptx.cuh"

namespace sdvk {
namespace {

constexpr int kLnWarps = 8;

template <class TO>
__device__ __forceinline__ void store4(TO* dst, float a, float b, float c, float d);
template <>
__device__ __forceinline__ void store4<float>(float* dst, float a, float b, float c, float d) {
    *reinterpret_cast<float4*>(dst) = make_float4(a, b, c, d);
}
template <>
__device__ __forceinline__ void store4<__half>(__half* dst, float a, float b, float c, float d) {
    __half2 lo = __floats2half2_rn(a, b), hi = __floats2half2_rn(c, d);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&lo);
    w.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(dst) = w;
}

// One warp per row; the row is held in registers between the passes (kChunks float4 per lane,
// d <= 128 * kChunks), so x is read from HBM once.  gamma and beta are loaded once per CTA into shared
// memory, issued before x so that their latency hides under the row's loads and reductions.
template <class TO, int kChunks>
__global__ void __launch_bounds__(kLnWarps * 32) layernorm_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                                  const float* __restrict__ beta, TO* __restrict__ y,
                                                                  uint32_t rows, uint32_t d, uint64_t ldx, uint64_t ldy,
                                                                  float eps) {
    constexpr int kThreads = kLnWarps * 32, kGB = (kChunks * 32 + kThreads - 1) / kThreads;
    __shared__ float4 sg[kChunks * 32], sb[kChunks * 32];
    grid_dependency_wait();  // x is the previous kernel's output
    grid_launch_dependents();
    const uint32_t lane = threadIdx.x & 31, nq = d / 4;
    const uint32_t row = blockIdx.x * kLnWarps + (threadIdx.x >> 5);
    const bool live = row < rows;  // warp-uniform
    float4 gq[kGB], bq[kGB];
#pragma unroll
    for (int k = 0; k < kGB; ++k) {
        const uint32_t i = threadIdx.x + k * kThreads;
        if (i < nq) {
            gq[k] = gamma ? reinterpret_cast<const float4*>(gamma)[i] : make_float4(1.f, 1.f, 1.f, 1.f);
            bq[k] = beta ? reinterpret_cast<const float4*>(beta)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    const float* xr = x + (uint64_t)(live ? row : 0) * ldx;
    float4 v[kChunks];
    float s = 0.0f;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
        const uint32_t j = (c * 32 + lane) * 4;
        v[c] = (live && j < d) ? *reinterpret_cast<const float4*>(xr + j) : make_float4(0.f, 0.f, 0.f, 0.f);
        s += (v[c].x + v[c].y) + (v[c].z + v[c].w);
    }
#pragma unroll
    for (int k = 0; k < kGB; ++k) {
        const uint32_t i = threadIdx.x + k * kThreads;
        if (i < nq) sg[i] = gq[k], sb[i] = bq[k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / (float)d;
    float ss = 0.0f;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
        const uint32_t j = (c * 32 + lane) * 4;
        if (j < d) {
            const float a = v[c].x - mean, b = v[c].y - mean, e = v[c].z - mean, f = v[c].w - mean;
            ss += (a * a + b * b) + (e * e + f * f);
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.0f / sqrtf(ss / (float)d + eps);
    __syncthreads();  // sg, sb complete
    if (!live) return;
    TO* yr = y + (uint64_t)row * ldy;
#pragma unroll
    for (int c = 0; c < kChunks; ++c) {
        const uint32_t q = c * 32 + lane, j = q * 4;
        if (j < d) {
            const float4 g = sg[q], bb = sb[q];
            store4<TO>(yr + j, (v[c].x - mean) * inv * g.x + bb.x, (v[c].y - mean) * inv * g.y + bb.y,
                       (v[c].z - mean) * inv * g.z + bb.z, (v[c].w - mean) * inv * g.w + bb.w);
        }
    }
}


// y[r][j] = h[r][j] * gelu(h[r][F + j]), 8 halves per thread per step.
__global__ void geglu_kernel(const __half* __restrict__ h, __half* __restrict__ y, uint32_t rows, uint32_t F,
                             uint64_t ldh, uint64_t ldy) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint32_t per_row = F / 8;
    const uint64_t n = (uint64_t)rows * per_row;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t r = (uint32_t)(i / per_row), c = (uint32_t)(i % per_row) * 8;
        const uint4 a = *reinterpret_cast<const uint4*>(h + (uint64_t)r * ldh + c);
        const uint4 g = *reinterpret_cast<const uint4*>(h + (uint64_t)r * ldh + F + c);
        const __half2* a2 = reinterpret_cast<const __half2*>(&a);
        const __half2* g2 = reinterpret_cast<const __half2*>(&g);
        uint4 o;
        __half2* o2 = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 av = __half22float2(a2[k]), gv = __half22float2(g2[k]);
            o2[k] = __floats2half2_rn(av.x * gelu_erf_as(gv.x), av.y * gelu_erf_as(gv.y));
        }
        *reinterpret_cast<uint4*>(y + (uint64_t)r * ldy + c) = o;
    }
}

bool a16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// y[r][c] = f16(sum_z part[z][r][c] (+ bias[c])): the split-K partial planes summed in a fixed order.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, const float* __restrict__ bias,
                                     __half* __restrict__ y, uint32_t rows, uint32_t cols, uint32_t splits,
                                     uint64_t ldy) {
    grid_dependency_wait();
    grid_launch_dependents();
    const uint64_t plane = (uint64_t)rows * cols, n4 = plane / 4;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n4; i += (uint64_t)gridDim.x * blockDim.x) {
        float4 a = reinterpret_cast<const float4*>(part)[i];
        for (uint32_t z = 1; z < splits; ++z) {
            const float4 b = reinterpret_cast<const float4*>(part + z * plane)[i];
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
        }
        const uint64_t e = i * 4;
        const uint32_t r = (uint32_t)(e / cols), c = (uint32_t)(e % cols);
        if (bias) {
            a.x += bias[c];
            a.y += bias[c + 1];
            a.z += bias[c + 2];
            a.w += bias[c + 3];
        }
        store4<__half>(y + (uint64_t)r * ldy + c, a.x, a.y, a.z, a.w);
    }
}

template <class TO>
int launch_ln(const float* x, const float* g, const float* b, TO* y, uint32_t rows, uint32_t d, uint64_t ldx,
              uint64_t ldy, float eps, const LaunchEnv& env) {
    const dim3 grid((rows + kLnWarps - 1) / kLnWarps), block(kLnWarps * 32);
    auto kern = d <= 512 ? layernorm_kernel<TO, 4> : d <= 1280 ? layernorm_kernel<TO, 10> : layernorm_kernel<TO, 24>;
    return launch_pdl(kern, grid, block, 0, env, "layernorm_kernel launch", x, g, b, y, rows, d, ldx, ldy, eps);
}

}  // namespace

int layernorm(const float* x, const float* gamma, const float* beta, void* y, int y_dtype, uint32_t rows, uint32_t d,
              uint64_t ldx, uint64_t ldy, float eps, const LaunchEnv& env) {
    if (!x || !y) return fail(env, SDVK_E_ARG, "null pointer");
    if (y_dtype != SDVK_F32 && y_dtype != SDVK_F16) return fail(env, SDVK_E_ARG, "LayerNorm output must be F32 or F16");
    if (rows == 0 || d == 0) return SDVK_OK;
    if (d % 4 || d > 3072 || ldx % 4 || ldy % 4 || !a16(x) || !a16(y) || (gamma && !a16(gamma)) ||
        (beta && !a16(beta)))
        return fail(env, SDVK_E_SHAPE, "LayerNorm needs d, ldx, ldy multiples of 4, d <= 3072, 16-byte aligned bases");
    if (y_dtype == SDVK_F32)
        return launch_ln<float>(x, gamma, beta, static_cast<float*>(y), rows, d, ldx, ldy, eps, env);
    return launch_ln<__half>(x, gamma, beta, static_cast<__half*>(y), rows, d, ldx, ldy, eps, env);
}

int geglu(const void* h, void* y, uint32_t rows, uint32_t F, uint64_t ldh, uint64_t ldy, const LaunchEnv& env) {
    if (!h || !y) return fail(env, SDVK_E_ARG, "null pointer");
    if (rows == 0 || F == 0) return SDVK_OK;
    if (F % 8 || ldh % 8 || ldy % 8 || ldh < 2ull * F || ldy < F || !a16(h) || !a16(y))
        return fail(env, SDVK_E_SHAPE, "GEGLU needs F, ldh, ldy multiples of 8 and 16-byte aligned rows");
    const uint64_t n = (uint64_t)rows * (F / 8);
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((n + 255) / 256, (uint64_t)env.num_sms * 8);
    return launch_pdl(geglu_kernel, dim3(blocks), dim3(256), 0, env, "geglu_kernel launch",
                      static_cast<const __half*>(h), static_cast<__half*>(y), rows, F, ldh, ldy);
}

// ------------------------------------------------------------------------------------ the block
namespace {

struct BlockLayout {
    uint64_t n, qkv, a, g, h, part, kv, total;  // byte offsets into the workspace
};

// The context's K|V projection has few rows (batch x 77) against a long K: split K so that the GEMM
// has enough tiles to fill the GPU.
constexpr uint32_t kKvSplits = 4;
bool kv_split(uint32_t crow, uint32_t Cc) { return crow <= 512 && Cc % (kKvSplits * 64) == 0; }

uint64_t align256(uint64_t v) { return (v + 255) & ~uint64_t(255); }

BlockLayout block_layout(const sdvk_block_desc& d) {
    const uint64_t rows = (uint64_t)d.batch * d.T, C = d.C, F = d.ff_inner;
    const uint64_t crow = (uint64_t)d.batch * d.Tctx;
    BlockLayout L{};
    L.n = 0;
    L.qkv = align256(L.n + rows * C * 2);
    // [rows][3C] for self-attention, later [rows][C] (cross Q); the cross K|V has its own region, since
    // it is written on the side stream while the main stream uses this one
    L.a = align256(L.qkv + rows * 3 * C * 2);
    L.g = align256(L.a + rows * C * 2);
    L.h = align256(L.g + rows * 2 * F * 2);
    L.part = align256(L.h + rows * F * 2);
    const uint64_t part_bytes = kv_split((uint32_t)crow, d.Cctx) ? (uint64_t)kKvSplits * crow * 2 * C * 4 : 0;
    L.kv = align256(L.part + part_bytes);
    L.total = align256(L.kv + crow * 2 * C * 2);
    return L;
}

GemmQ8Desc linear_desc(const void* x, int x_dtype, uint64_t ldx, const sdvk_q8_linear& w, uint32_t N, uint32_t K,
                       void* c, int c_dtype, uint64_t ldc, uint32_t rows, bool accumulate) {
    GemmQ8Desc g{};
    g.weights_static = true;  // the block's weights are parameters
    g.x = x;
    g.x_dtype = x_dtype;
    g.ldx = ldx;
    g.wq = w.q;
    g.ws = w.s;
    g.ldw = K;
    g.bias = w.bias;
    g.c = c;
    g.c_dtype = c_dtype;
    g.ldc = ldc;
    g.xrows = rows;
    g.wrows = N;
    g.K = K;
    g.batch = 1;
    g.accumulate = accumulate;
    return g;
}

// Weights (and biases) that continue one another in memory form a single [n*N][K] weight.
bool contiguous(const sdvk_q8_linear* w, int n, uint64_t N, uint64_t K) {
    for (int i = 1; i < n; ++i) {
        if (w[i].q != w[0].q + i * N * K || w[i].s != w[0].s + i * N * K / 32) return false;
        if ((w[i].bias == nullptr) != (w[0].bias == nullptr)) return false;
        if (w[0].bias && w[i].bias != w[0].bias + i * N) return false;
    }
    return true;
}

// Y[:, i*N:(i+1)*N] = X W_i^T (+ b_i) for n weights, as one GEMM when they are contiguous.
int fused_linears(const void* x, int x_dtype, uint64_t ldx, const sdvk_q8_linear* w, int n, uint32_t N, uint32_t K,
                  __half* y, uint64_t ldy, uint32_t rows, const LaunchEnv& env) {
    if (contiguous(w, n, N, K))
        return gemm_q8(linear_desc(x, x_dtype, ldx, w[0], n * N, K, y, SDVK_F16, ldy, rows, false), env);
    for (int i = 0; i < n; ++i)
        if (int rc = gemm_q8(linear_desc(x, x_dtype, ldx, w[i], N, K, y + (uint64_t)i * N, SDVK_F16, ldy, rows, false),
                             env))
            return rc;
    return SDVK_OK;
}

// [k | v] = ctx [Wk; Wv]^T for back-to-back weights, K split into kKvSplits GEMM batches: batch z
// reads the z-th K slice of every row of ctx and of the weight (batch strides smaller than the row
// strides) and writes its own fp32 plane; splitk_reduce_kernel sums the planes into the f16 output.
int kv_linear_split(const void* ctx, int ctx_dtype, uint64_t ldctx, const sdvk_q8_linear* w, uint32_t N, uint32_t K,
                    __half* y, uint64_t ldy, uint32_t rows, float* part, const LaunchEnv& env) {
    const uint32_t Ks = K / kKvSplits;
    GemmQ8Desc g = linear_desc(ctx, ctx_dtype, ldctx, sdvk_q8_linear{w[0].q, w[0].s, nullptr}, 2 * N, Ks, part, SDVK_F32,
                               2ull * N, rows, false);
    g.ldw = K;
    g.batch = kKvSplits;
    g.sx = Ks;
    g.sw = Ks;
    g.sc = (uint64_t)rows * 2 * N;
    if (int rc = gemm_q8(g, env)) return rc;
    const uint64_t n4 = (uint64_t)rows * 2 * N / 4;
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((n4 + 255) / 256, (uint64_t)env.num_sms * 4);
    return launch_pdl(splitk_reduce_kernel, dim3(blocks), dim3(256), 0, env, "splitk_reduce_kernel launch",
                      (const float*)part, w[0].bias, y, rows, 2 * N, (uint32_t)kKvSplits, ldy);
}

sdvk_attn_desc attn_desc(const __half* q, uint64_t ldq, uint64_t sq, const __half* k, const __half* v, uint64_t ldkv,
                         uint64_t skv, __half* o, uint64_t ldo, uint64_t so, uint32_t batch, uint32_t heads,
                         uint32_t Tq, uint32_t Tk, uint32_t hd) {
    sdvk_attn_desc a{};
    a.q = q;
    a.k = k;
    a.v = v;
    a.o = o;
    a.dtype = SDVK_F16;
    a.o_dtype = SDVK_F16;
    a.batch = batch;
    a.heads = heads;
    a.Tq = Tq;
    a.Tk = Tk;
    a.hd = hd;
    a.ldq = ldq;
    a.ldk = a.ldv = ldkv;
    a.ldo = ldo;
    a.sq = sq;
    a.sk = a.sv = skv;
    a.so = so;
    a.hq = a.hk = a.hv = a.ho = hd;
    a.scale = 1.0f / std::sqrt((float)hd);
    a.causal = 0;
    return a;
}

}  // namespace

uint64_t block_workspace_bytes(const sdvk_block_desc& d) { return block_layout(d).total; }

int transformer_block(const sdvk_block_desc& d, void* ws, uint64_t ws_bytes, const LaunchEnv& env) {
    return transformer_block_ex(d, nullptr, 0, ws, ws_bytes, env);
}

int transformer_block_ex(const sdvk_block_desc& d, const __half* kv_pre, uint64_t ld_kv, void* ws, uint64_t ws_bytes,
                         const LaunchEnv& env) {
    if (!d.x || !ws) return fail(env, SDVK_E_ARG, "null pointer");
    if (d.batch == 0 || d.T == 0) return SDVK_OK;
    if (d.heads == 0 || d.C % d.heads || d.C / d.heads > 64)
        return fail(env, SDVK_E_SHAPE, "heads must divide C with head dim <= 64");
    if (d.Tctx && !d.ctx) return fail(env, SDVK_E_ARG, "null context");
    const BlockLayout L = block_layout(d);
    if (ws_bytes < L.total) return fail(env, SDVK_E_ARG, "workspace smaller than sdvk_transformer_block_workspace()");
    const uint32_t rows = d.batch * d.T, C = d.C, F = d.ff_inner, H = d.heads, hd = C / H;
    const uint32_t crow = d.batch * d.Tctx;
    uint8_t* base = static_cast<uint8_t*>(ws);
    __half* n = reinterpret_cast<__half*>(base + L.n);
    __half* qkv = reinterpret_cast<__half*>(base + L.qkv);
    __half* q2 = qkv;
    __half* kv2 = reinterpret_cast<__half*>(base + L.kv);
    __half* a = reinterpret_cast<__half*>(base + L.a);
    __half* g = reinterpret_cast<__half*>(base + L.g);
    __half* h = reinterpret_cast<__half*>(base + L.h);
    const float eps = d.eps > 0.0f ? d.eps : 1e-5f;
    int rc;
    // ---- the context's K|V projection depends on ctx alone: it runs on the side stream, forked here
    //      and joined before the cross-attention, overlapping the self-attention half
    const sdvk_q8_linear kv_w[2] = {d.k2, d.v2};
    LaunchEnv side = env;
    side.stream = env.side;
    const bool fork = crow && !kv_pre && env.side && env.fork && env.join;
    if (fork) {
        if ((rc = cuda_check(env, cudaEventRecord(env.fork, env.stream), "fork"))) return rc;
        if ((rc = cuda_check(env, cudaStreamWaitEvent(env.side, env.fork, 0), "fork"))) return rc;
    }
    const LaunchEnv& kv_env = fork ? side : env;
    if (kv_pre) {
        // K|V precomputed by the caller (the context is the same for every block): nothing to fork
    } else if (crow && kv_split(crow, d.Cctx) && contiguous(kv_w, 2, C, d.Cctx) && C % 2 == 0) {
        if ((rc = kv_linear_split(d.ctx, d.ctx_dtype, d.Cctx, kv_w, C, d.Cctx, kv2, 2ull * C, crow,
                                  reinterpret_cast<float*>(base + L.part), kv_env)))
            return rc;
    } else if (crow && (rc = fused_linears(d.ctx, d.ctx_dtype, d.Cctx, kv_w, 2, C, d.Cctx, kv2, 2ull * C, crow,
                                           kv_env))) {
        return rc;
    }
    if (fork && (rc = cuda_check(env, cudaEventRecord(env.join, env.side), "join"))) return rc;
    // ---- self-attention
    if ((rc = layernorm(d.x, d.ln1_w, d.ln1_b, n, SDVK_F16, rows, C, C, C, eps, env))) return rc;
    const sdvk_q8_linear qkv_w[3] = {d.q, d.k, d.v};
    if ((rc = fused_linears(n, SDVK_F16, C, qkv_w, 3, C, C, qkv, 3ull * C, rows, env))) return rc;
    sdvk_attn_desc at = attn_desc(qkv, 3ull * C, (uint64_t)d.T * 3 * C, qkv + C, qkv + 2 * C, 3ull * C,
                                  (uint64_t)d.T * 3 * C, a, C, (uint64_t)d.T * C, d.batch, H, d.T, d.T, hd);
    if ((rc = attention(at, env))) return rc;
    if ((rc = gemm_q8(linear_desc(a, SDVK_F16, C, d.o, C, C, d.x, SDVK_F32, C, rows, true), env))) return rc;
    // ---- cross-attention against the context
    if ((rc = layernorm(d.x, d.ln2_w, d.ln2_b, n, SDVK_F16, rows, C, C, C, eps, env))) return rc;
    if ((rc = gemm_q8(linear_desc(n, SDVK_F16, C, d.q2, C, C, q2, SDVK_F16, C, rows, false), env))) return rc;
    if (fork && (rc = cuda_check(env, cudaStreamWaitEvent(env.stream, env.join, 0), "join"))) return rc;
    if (kv_pre)
        at = attn_desc(q2, C, (uint64_t)d.T * C, kv_pre, kv_pre + C, ld_kv, (uint64_t)d.Tctx * ld_kv, a, C,
                       (uint64_t)d.T * C, d.batch, H, d.T, d.Tctx, hd);
    else
        at = attn_desc(q2, C, (uint64_t)d.T * C, kv2, kv2 + C, 2ull * C, (uint64_t)d.Tctx * 2 * C, a, C,
                       (uint64_t)d.T * C, d.batch, H, d.T, d.Tctx, hd);
    if ((rc = attention(at, env))) return rc;
    if ((rc = gemm_q8(linear_desc(a, SDVK_F16, C, d.o2, C, C, d.x, SDVK_F32, C, rows, true), env))) return rc;
    // ---- GEGLU feed-forward
    if ((rc = layernorm(d.x, d.ln3_w, d.ln3_b, n, SDVK_F16, rows, C, C, C, eps, env))) return rc;
    if (d.ff1_geglu_interleaved) {  // GEGLU in the GEMM epilogue: h straight from the accumulators
        GemmQ8Desc gd = linear_desc(n, SDVK_F16, C, d.ff1, 2 * F, C, h, SDVK_F16, F, rows, false);
        gd.geglu = true;
        if ((rc = gemm_q8(gd, env))) return rc;
    } else {
        if ((rc = gemm_q8(linear_desc(n, SDVK_F16, C, d.ff1, 2 * F, C, g, SDVK_F16, 2ull * F, rows, false), env)))
            return rc;
        if ((rc = geglu(g, h, rows, F, 2ull * F, F, env))) return rc;
    }
    return gemm_q8(linear_desc(h, SDVK_F16, F, d.ff2, C, F, d.x, SDVK_F32, C, rows, true), env);
}

}  // namespace sdvk
