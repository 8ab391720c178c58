// attention.cu -- host side of the fused attention kernel (attention.cuh) and the finite check.
#include <cmath>

#include "attention.cuh"
#include "backend.hpp"

namespace sdvk {
namespace {

template <class TIn, class TOut, bool kAsync>
int launch(const AttnParams& p, const LaunchEnv& env) {
    dim3 grid((p.Tq + kAttnBM - 1) / kAttnBM, p.heads, p.batch);
    attn_fwd_kernel<TIn, TOut, kAsync><<<grid, kAttnThreads, kAttnSmem, env.stream>>>(p);
    return cuda_check(env, cudaGetLastError(), "attn_fwd_kernel launch");
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
