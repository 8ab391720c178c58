// attention.cu -- host side of the fused attention kernel (attention.cuh) and the finite check.
#include <cmath>
#include <cstdlib>
#include <string>

#include "attention.cuh"
#include "attention_fp32.cuh"
#include "attention_tc.cuh"
#include "attention_tc_short.cuh"
#include "backend.hpp"

namespace sdvk {
namespace {

// Keys that fit two 64-key tiles go to attn_short_kernel (whole grid resident, loads in flight
// together) unless SDVK_ATTN_KERNEL=mma forces the general kernel.
bool short_eligible(const AttnParams& p) {
    const char* e = getenv("SDVK_ATTN_KERNEL");
    return p.Tk <= 2 * kAttnBN && !(e && e[0] == 'm');
}

template <class TIn, class TOut, bool kAsync>
int launch(const AttnParams& p, const LaunchEnv& env) {
    dim3 grid((p.Tq + kAttnBM - 1) / kAttnBM, p.heads, p.batch);
    if (short_eligible(p)) {
        return launch_pdl(attn_short_kernel<TIn, TOut, kAsync>, grid, dim3(kAttnShortThreads), kAttnSmem, env,
                          "attn_short_kernel launch", p);
    }
    return launch_pdl(attn_fwd_kernel<TIn, TOut, kAsync>, grid, dim3(kAttnThreads), kAttnSmem, env,
                      "attn_fwd_kernel launch", p);
}

template <class TIn, class TOut>
int launch_mode(const AttnParams& p, bool async, const LaunchEnv& env) {
    if constexpr (sizeof(TIn) == 2) {
        if (async) return launch<TIn, TOut, true>(p, env);
    }
    return launch<TIn, TOut, false>(p, env);
}

template <class TIn>
int launch_out(const AttnParams& p, int o_dtype, bool async, const LaunchEnv& env) {
    if (o_dtype == SDVK_F32) return launch_mode<TIn, float>(p, async, env);
    return launch_mode<TIn, __half>(p, async, env);
}

bool a16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// 4-D tiled map over one operand: {hd (contiguous), tokens, heads, batch}, box {64, 128, 1, 1},
// 128-byte swizzle (the UMMA K-major / MN-major SW128 operand layout).
int make_attn_map(CUtensorMap* m, int dtype, const void* base, uint32_t T, uint32_t heads, uint32_t batch,
                  uint64_t ld, uint64_t hs, uint64_t bs, const LaunchEnv& env, const char* what) {
    auto fn = tensor_map_encoder();
    if (!fn) return fail(env, SDVK_E_CUDA, "cuTensorMapEncodeTiled unavailable");
    const uint64_t es = 2;
    // a dimension of extent 1 is never stepped: give it a legal stride
    if (heads == 1) hs = ld * T;
    if (batch == 1) bs = hs * heads;
    cuuint64_t dims[4] = {64, T, heads, batch};
    cuuint64_t strides[3] = {ld * es, hs * es, bs * es};
    cuuint32_t box[4] = {64, 128, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(m, dtype == SDVK_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(env, SDVK_E_SHAPE, std::string("attention tensor map rejected: ") + what);
    return SDVK_OK;
}

// The tensor-core kernels take head dim 64, 16-bit Q/K/V, a positive scale, and TMA-legal layouts
// (16-byte aligned bases and strides) with an output that takes 16-byte vector stores.
// attn_tc_kernel serves keys beyond one 128-key tile; attn_tc_short_kernel serves at most 128
// non-causal keys (the 77-token cross-attention).  SDVK_ATTN_KERNEL=mma forces the warp-level
// kernels (attention.cuh), =tc forces attn_tc_kernel wherever the layout allows it.
enum class AttnKernel { kWarp, kTc, kTcShort };
bool tc_layout_ok(const sdvk_attn_desc& d);
AttnKernel attn_kernel_choice(const sdvk_attn_desc& d) {
    const char* e = getenv("SDVK_ATTN_KERNEL");
    if ((e && e[0] == 'm') || !tc_layout_ok(d)) return AttnKernel::kWarp;
    if (e && e[0] == 't') return AttnKernel::kTc;
    if (d.Tk > 128) return AttnKernel::kTc;
    return d.causal ? AttnKernel::kWarp : AttnKernel::kTcShort;
}
bool tc_layout_ok(const sdvk_attn_desc& d) {
    const uint64_t es = 2, eo = d.o_dtype == SDVK_F32 ? 4 : 2;
    auto s16 = [](uint64_t bytes) { return bytes % 16 == 0 && bytes < (1ull << 40); };
    return (d.dtype == SDVK_F16 || d.dtype == SDVK_BF16) && d.hd == 64 && d.scale > 0.0f && d.Tk > 0 &&
           a16(d.q) && a16(d.k) && a16(d.v) && a16(d.o) && s16(d.ldq * es) && s16(d.ldk * es) && s16(d.ldv * es) &&
           s16(d.hq * es) && s16(d.hk * es) && s16(d.hv * es) && s16(d.sq * es) && s16(d.sk * es) &&
           s16(d.sv * es) && s16(d.ldo * eo) && s16(d.ho * eo) && s16(d.so * eo) && d.heads <= 65535 &&
           d.batch <= 65535;
}

template <class T, class TO>
int launch_tc(const sdvk_attn_desc& d, const LaunchEnv& env) {
    CUtensorMap mq, mk, mv;
    if (int rc = make_attn_map(&mq, d.dtype, d.q, d.Tq, d.heads, d.batch, d.ldq, d.hq, d.sq, env, "Q")) return rc;
    if (int rc = make_attn_map(&mk, d.dtype, d.k, d.Tk, d.heads, d.batch, d.ldk, d.hk, d.sk, env, "K")) return rc;
    if (int rc = make_attn_map(&mv, d.dtype, d.v, d.Tk, d.heads, d.batch, d.ldv, d.hv, d.sv, env, "V")) return rc;
    TcAttnParams p{};
    p.o = d.o;
    p.ldo = d.ldo;
    p.so = d.so;
    p.ho = d.ho;
    p.Tq = d.Tq;
    p.Tk = d.Tk;
    p.heads = d.heads;
    p.batch = d.batch;
    p.scale_log2 = d.scale * 1.4426950408889634f;
    p.causal = d.causal ? 1u : 0u;
    p.err = env.err_dev;
    p.timeout_ns = env.timeout_ns;
    auto kern = attn_tc_kernel<T, TO>;
    if (!kernel_smem_attr(reinterpret_cast<const void*>(kern), TcAttnCfg::kSmemBytes, env.device))
        return fail(env, SDVK_E_CUDA, "attn_tc_kernel: shared memory opt-in failed");
    dim3 grid((d.Tq + TcAttnCfg::kBM - 1) / TcAttnCfg::kBM, d.heads, d.batch);
    return launch_pdl(kern, grid, dim3(TcAttnCfg::kThreads), TcAttnCfg::kSmemBytes, env, "attn_tc_kernel launch", mq,
                      mk, mv, p);
}

template <class T, class TO>
int launch_tc_short(const sdvk_attn_desc& d, const LaunchEnv& env) {
    CUtensorMap mq, mk, mv;
    if (int rc = make_attn_map(&mq, d.dtype, d.q, d.Tq, d.heads, d.batch, d.ldq, d.hq, d.sq, env, "Q")) return rc;
    if (int rc = make_attn_map(&mk, d.dtype, d.k, d.Tk, d.heads, d.batch, d.ldk, d.hk, d.sk, env, "K")) return rc;
    if (int rc = make_attn_map(&mv, d.dtype, d.v, d.Tk, d.heads, d.batch, d.ldv, d.hv, d.sv, env, "V")) return rc;
    TcAttnParams p{};
    p.o = d.o;
    p.ldo = d.ldo;
    p.so = d.so;
    p.ho = d.ho;
    p.Tq = d.Tq;
    p.Tk = d.Tk;
    p.heads = d.heads;
    p.batch = d.batch;
    p.scale_log2 = d.scale * 1.4426950408889634f;
    p.causal = 0;
    p.err = env.err_dev;
    p.timeout_ns = env.timeout_ns;
    auto kern = attn_tc_short_kernel<T, TO>;
    if (!kernel_smem_attr(reinterpret_cast<const void*>(kern), TcShortCfg::kSmemBytes, env.device))
        return fail(env, SDVK_E_CUDA, "attn_tc_short_kernel: shared memory opt-in failed");
    const uint64_t items = (uint64_t)((d.Tq + TcShortCfg::kBM - 1) / TcShortCfg::kBM) * d.heads * d.batch;
    const uint32_t grid = (uint32_t)std::min<uint64_t>(items, 2ull * env.num_sms);
    return launch_pdl(kern, dim3(grid), dim3(TcShortCfg::kThreads), TcShortCfg::kSmemBytes, env,
                      "attn_tc_short_kernel launch", mq, mk, mv, p);
}

template <class T>
int launch_tc_out(const sdvk_attn_desc& d, bool short_keys, const LaunchEnv& env) {
    if (short_keys) {
        if (d.o_dtype == SDVK_F32) return launch_tc_short<T, float>(d, env);
        return launch_tc_short<T, __half>(d, env);
    }
    if (d.o_dtype == SDVK_F32) return launch_tc<T, float>(d, env);
    return launch_tc<T, __half>(d, env);
}

template <class T>
__global__ void finite_kernel(const T* x, uint64_t n, uint32_t* flag) {
    bool bad = false;
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
        bad |= !isfinite((float)x[i]);
    if (__syncthreads_or(bad) && threadIdx.x == 0) atomicOr(flag, 1u);
}

}  // namespace

int attention(const sdvk_attn_desc& d, const LaunchEnv& env) {
    if ((d.Tq && (!d.q || !d.o)) || (d.Tk && (!d.k || !d.v))) return fail(env, SDVK_E_ARG, "null pointer");
    if (d.dtype != SDVK_F32 && d.dtype != SDVK_F16 && d.dtype != SDVK_BF16)
        return fail(env, SDVK_E_ARG, "Q/K/V dtype must be F32, F16 or BF16");
    if (d.o_dtype != SDVK_F32 && d.o_dtype != SDVK_F16) return fail(env, SDVK_E_ARG, "O dtype must be F32 or F16");
    if (d.hd == 0 || d.hd > kAttnHD) return fail(env, SDVK_E_SHAPE, "head dim must be 1..64");
    if (d.batch == 0 || d.heads == 0 || d.Tq == 0) return SDVK_OK;
    if (d.heads > 65535 || d.batch > 65535) return fail(env, SDVK_E_SHAPE, "too many heads/batches");
    AttnParams p{};
    p.q = d.q;
    p.k = d.k;
    p.v = d.v;
    p.o = d.o;
    p.batch = d.batch;
    p.heads = d.heads;
    p.Tq = d.Tq;
    p.Tk = d.Tk;
    p.hd = d.hd;
    p.ldq = d.ldq;
    p.ldk = d.ldk;
    p.ldv = d.ldv;
    p.ldo = d.ldo;
    p.sq = d.sq;
    p.sk = d.sk;
    p.sv = d.sv;
    p.so = d.so;
    p.hq = d.hq;
    p.hk = d.hk;
    p.hv = d.hv;
    p.ho = d.ho;
    p.scale_log2 = d.scale * 1.4426950408889634f;
    p.causal = d.causal ? 1u : 0u;
    const char* force = getenv("SDVK_ATTN_KERNEL");
    if (d.dtype == SDVK_F32 && env.precision == SDVK_PRECISION_REFERENCE && !(force && force[0] == 'm')) {
        const dim3 grid((d.Tq + kF32Rows - 1) / kF32Rows, d.heads, d.batch);
        if (d.o_dtype == SDVK_F32)
            return launch_pdl(attn_fp32_kernel<float>, grid, dim3(kF32Rows), 0, env, "attn_fp32_kernel launch", p);
        return launch_pdl(attn_fp32_kernel<__half>, grid, dim3(kF32Rows), 0, env, "attn_fp32_kernel launch", p);
    }
    const AttnKernel choice = attn_kernel_choice(d);
    if (choice != AttnKernel::kWarp) {
        const bool short_keys = choice == AttnKernel::kTcShort;
        if (d.dtype == SDVK_F16) return launch_tc_out<__half>(d, short_keys, env);
        return launch_tc_out<__nv_bfloat16>(d, short_keys, env);
    }
    // cp.async staging needs 16-byte aligned rows and whole 8-element chunks of the head.
    const uint64_t es = 2;
    const bool async = d.dtype != SDVK_F32 && d.hd % 8 == 0 && a16(d.q) && a16(d.k) && a16(d.v) &&
                       (d.ldq * es) % 16 == 0 && (d.ldk * es) % 16 == 0 && (d.ldv * es) % 16 == 0 &&
                       (d.sq * es) % 16 == 0 && (d.sk * es) % 16 == 0 && (d.sv * es) % 16 == 0 &&
                       (d.hq * es) % 16 == 0 && (d.hk * es) % 16 == 0 && (d.hv * es) % 16 == 0;
    switch (d.dtype) {
        case SDVK_F16: return launch_out<__half>(p, d.o_dtype, async, env);
        case SDVK_BF16: return launch_out<__nv_bfloat16>(p, d.o_dtype, async, env);
        default: return launch_out<float>(p, d.o_dtype, false, env);
    }
}

int check_finite(const void* x, int dtype, uint64_t n, uint32_t* flag_dev, const LaunchEnv& env) {
    if (!x) return fail(env, SDVK_E_ARG, "null pointer");
    if (n == 0) return SDVK_OK;
    const int blocks = env.num_sms * 4;
    if (dtype == SDVK_F32) finite_kernel<float><<<blocks, 256, 0, env.stream>>>((const float*)x, n, flag_dev);
    else if (dtype == SDVK_F16) finite_kernel<__half><<<blocks, 256, 0, env.stream>>>((const __half*)x, n, flag_dev);
    else if (dtype == SDVK_BF16)
        finite_kernel<__nv_bfloat16><<<blocks, 256, 0, env.stream>>>((const __nv_bfloat16*)x, n, flag_dev);
    else return fail(env, SDVK_E_ARG, "dtype");
    return cuda_check(env, cudaGetLastError(), "finite_kernel launch");
}

}  // namespace sdvk
