// sdvk_abi.cu -- the extern "C" boundary declared in include/sdvk_cuda.h: context, memory, step
// protocol, the reference-compatible name dispatch and the typed hot-path entry points.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <thread>

#include "backend.hpp"
#include "ptx.cuh"  // the device error codes

struct sdvk_ctx {
    int device = 0;
    int num_sms = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    uint32_t* err_dev = nullptr;   // kernels OR device error codes in here
    uint32_t* flag_dev = nullptr;  // sdvk_check_finite
    uint64_t timeout_ns = 2000000000ull;
    int precision = SDVK_PRECISION_REFERENCE;
    cudaEvent_t step_done = nullptr;
    cudaStream_t side = nullptr;  // second stream for overlapping work (forked from and joined to `stream`)
    cudaEvent_t fork = nullptr, join = nullptr;
    bool in_step = false;
    bool step_recorded = false;
    void* scratch = nullptr;  // workspace of name-dispatched kernels that need one (groupnorm)
    uint64_t scratch_bytes = 0;
    void* samp_ws = nullptr;  // the sampler step's partial sums (a few KB, sized at creation)
    uint64_t samp_ws_bytes = 0;
    std::string last_error;
    std::string device_name;
};

namespace {

// Mirrors of the reference push-constant blocks (sdvkgen.cpp:901-903, fused_attn.cpp:15-26).
struct Pg {
    uint32_t M, N, K, mode, sA, sB, sC, batch, lda, ldb, ldc, pad;
};
struct FaPush {
    uint32_t Tq, Tk, C, heads, hd, causal, pad0, pad1;
    float scale;
};
struct GnPush {  // groupnorm.comp push constants (sdvkgen.cpp:1107-1111)
    uint32_t C, P, G;
    float eps;
    uint32_t act;
};
static_assert(sizeof(GnPush) == 20, "GnPush layout");
struct LnPush {  // layernorm_fwd.comp push constants (sdvkgen.cpp:1096-1100)
    uint32_t rows, d;
    float eps;
    uint32_t affine;
};
static_assert(sizeof(Pg) == 48, "Pg layout");
static_assert(sizeof(LnPush) == 16, "LnPush layout");
static_assert(sizeof(FaPush) == 36, "FaPush layout");

int set_err(sdvk_ctx* ctx, int code, const std::string& msg) {
    if (ctx) ctx->last_error = msg;
    return code;
}

int cuda_err(sdvk_ctx* ctx, cudaError_t e, const char* what) {
    if (e == cudaSuccess) return SDVK_OK;
    return set_err(ctx, SDVK_E_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Make the context's device current for this thread (callers may switch devices in between).
int use_device(sdvk_ctx* ctx) {
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess || cur != ctx->device)
        return cuda_err(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    return SDVK_OK;
}

sdvk::LaunchEnv env_of(sdvk_ctx* ctx) {
    return sdvk::LaunchEnv{ctx->stream, ctx->err_dev,  ctx->timeout_ns, ctx->device, ctx->num_sms,
                           &ctx->last_error, ctx->precision, ctx->side,   ctx->fork,   ctx->join};
}

// After a synchronisation point: surface (and clear) any device-side error code.
int collect_device_error(sdvk_ctx* ctx) {
    uint32_t err = 0;
    cudaError_t e = cudaMemcpy(&err, ctx->err_dev, sizeof(err), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return cuda_err(ctx, e, "reading device error word");
    if (err) {
        cudaMemset(ctx->err_dev, 0, sizeof(uint32_t));
        if (err & sdvk::kErrTimeout)
            return set_err(ctx, SDVK_E_TIMEOUT, "a kernel's bounded wait timed out (device error word " +
                                                    std::to_string(err) + ")");
        return set_err(ctx, SDVK_E_NOT_FINITE, "non-finite model output in a sampler step (device error word " +
                                                   std::to_string(err) + ")");
    }
    return SDVK_OK;
}

bool buf_holds(const sdvk_buf& b, uint64_t bytes) { return b.ptr && (b.size == 0 || bytes <= b.size); }
const void* buf_ptr(const sdvk_buf& b) { return static_cast<const char*>(b.ptr) + b.offset; }
void* buf_mptr(const sdvk_buf& b) { return static_cast<char*>(b.ptr) + b.offset; }
const float* fptr(const sdvk_buf& b) { return static_cast<const float*>(buf_ptr(b)); }
float* fmptr(const sdvk_buf& b) { return static_cast<float*>(buf_mptr(b)); }

// Largest element index + 1 that a copy_nd / ew2 operand reaches for i < n, with i split over
// d0..d2 (the rest in the last coordinate); 0 for a zero dimension.
uint64_t nd_extent(uint32_t n, uint32_t d0, uint32_t d1, uint32_t d2, uint32_t s0, uint32_t s1, uint32_t s2,
                   uint32_t s3) {
    if (!n) return 0;
    if (!d0 || !d1 || !d2) return UINT64_MAX;
    const uint64_t last = n - 1ull;
    const uint64_t c0 = std::min<uint64_t>(d0 - 1ull, last), c1 = std::min<uint64_t>(d1 - 1ull, last / d0);
    const uint64_t c2 = std::min<uint64_t>(d2 - 1ull, last / ((uint64_t)d0 * d1));
    const uint64_t c3 = last / ((uint64_t)d0 * d1 * d2);
    return c0 * s0 + c1 * s1 + c2 * s2 + c3 * s3 + 1;
}

// The kernel-table entries around the hot path (table.cu): the walker's glue, in its binding orders
// and push layouts (vk_engine.cpp:51-125).  Every operand is fp32; extents are checked against the
// buffer sizes, and shapes whose indices would pass 2^32 (the shaders' uint arithmetic) are refused.
int dispatch_table(sdvk_ctx* ctx, const std::string& name, const sdvk_buf* bufs, uint32_t nbufs, const void* push,
                   uint32_t push_bytes, uint32_t batch) {
    auto need = [&](uint32_t nb, uint32_t pb) -> int {
        if (nbufs < nb || push_bytes < pb)
            return set_err(ctx, SDVK_E_ARG, name + ": needs " + std::to_string(nb) + " buffers and a " +
                                                std::to_string(pb) + "-byte push");
        return SDVK_OK;
    };
    auto small = [&](uint32_t i, uint64_t elems) {
        return elems > (1ull << 32) || !buf_holds(bufs[i], elems * 4);
    };
    auto too_small = [&]() { return set_err(ctx, SDVK_E_ARG, name + ": a buffer is smaller than the shape needs"); };
    uint32_t u[6] = {};
    std::memcpy(u, push, std::min<uint32_t>(push_bytes, sizeof u));
    if (int rc = use_device(ctx)) return rc;
    const sdvk::LaunchEnv env = env_of(ctx);
    if (name == "add2") {
        if (int rc = need(3, 4)) return rc;
        if (small(0, u[0]) || small(1, u[0]) || small(2, u[0])) return too_small();
        return sdvk::table_add2(fmptr(bufs[0]), fptr(bufs[1]), fptr(bufs[2]), u[0], env);
    }
    if (name == "copy_nd") {
        if (int rc = need(2, sizeof(sdvk::TablePnd))) return rc;
        sdvk::TablePnd p;
        std::memcpy(&p, push, sizeof p);
        if (small(0, nd_extent(p.n, p.d0, p.d1, p.d2, p.os0, p.os1, p.os2, p.os3)) ||
            small(1, nd_extent(p.n, p.d0, p.d1, p.d2, p.ss0, p.ss1, p.ss2, p.ss3)))
            return too_small();
        return sdvk::table_copy_nd(fmptr(bufs[0]), fptr(bufs[1]), p, env);
    }
    if (name == "ew2") {
        if (int rc = need(3, sizeof(sdvk::TablePew2))) return rc;
        sdvk::TablePew2 p;
        std::memcpy(&p, push, sizeof p);
        if (small(0, p.n) || small(1, nd_extent(p.n, p.d0, p.d1, p.d2, p.as0, p.as1, p.as2, p.as3)) ||
            small(2, nd_extent(p.n, p.d0, p.d1, p.d2, p.bs0, p.bs1, p.bs2, p.bs3)))
            return too_small();
        return sdvk::table_ew2(fmptr(bufs[0]), fptr(bufs[1]), fptr(bufs[2]), p, env);
    }
    if (name == "unary_fwd") {
        if (int rc = need(2, 8)) return rc;
        if (small(0, u[0]) || small(1, u[0])) return too_small();
        return sdvk::table_unary(fptr(bufs[0]), fmptr(bufs[1]), u[0], u[1], env);
    }
    if (name == "bias_add") {
        if (int rc = need(2, 8)) return rc;
        if (small(0, (uint64_t)u[0] * u[1]) || small(1, u[1] ? u[0] : 0)) return too_small();
        return sdvk::table_bias_add(fmptr(bufs[0]), fptr(bufs[1]), u[0], u[1], env);
    }
    if (name == "upsample2x") {
        if (int rc = need(2, 12)) return rc;
        const uint64_t in = (uint64_t)u[0] * u[1] * u[2];
        if (small(0, in) || small(1, in * 4)) return too_small();
        return sdvk::table_upsample2x(fptr(bufs[0]), fmptr(bufs[1]), u[0], u[1], u[2], env);
    }
    if (name == "im2col" || name == "im2col_s2") {
        const bool s2 = name == "im2col_s2";
        if (int rc = need(2, s2 ? 24 : 20)) return rc;
        const uint64_t in = (uint64_t)u[0] * u[1] * u[2];
        const uint64_t P = s2 ? (uint64_t)u[3] * u[4] : (uint64_t)u[4] * u[2];
        if (small(0, in) || small(1, (uint64_t)u[0] * 9 * P)) return too_small();
        if (!s2 && (uint64_t)u[3] + u[4] > u[1]) return set_err(ctx, SDVK_E_SHAPE, name + ": rows past the input");
        return sdvk::table_im2col(fptr(bufs[0]), fmptr(bufs[1]), u[0], u[1], u[2], u[3], u[4], s2 ? (int)u[5] : -1, s2,
                                  env);
    }
    if (name == "gemm_nt" || name == "gemm_nn") {
        const bool nt = name == "gemm_nt";
        if (int rc = need(3, sizeof(sdvk::TablePg))) return rc;
        sdvk::TablePg p;
        std::memcpy(&p, push, sizeof p);
        if (!p.M || !p.N) return SDVK_OK;
        const uint64_t lda = p.lda ? p.lda : p.K, ldb = nt ? p.K : (p.ldb ? p.ldb : p.N), ldc = p.ldc ? p.ldc : p.N;
        const uint64_t z = batch - 1ull;
        const uint64_t a_end = p.K ? z * p.sA + (p.M - 1ull) * lda + p.K : 0;
        const uint64_t b_end = !p.K ? 0 : nt ? z * p.sB + (p.N - 1ull) * ldb + p.K : z * p.sB + (p.K - 1ull) * ldb + p.N;
        const uint64_t c_end = z * p.sC + (p.M - 1ull) * ldc + p.N;
        if (small(0, a_end) || small(1, b_end) || small(2, c_end)) return too_small();
        return sdvk::table_gemm_fp32(nt, fptr(bufs[0]), fptr(bufs[1]), fmptr(bufs[2]), p, batch, env);
    }
    if (name == "softmax_fwd") {
        if (int rc = need(2, 8)) return rc;
        const uint64_t n = (uint64_t)u[0] * u[1];
        if (small(0, n) || small(1, n)) return too_small();
        return sdvk::table_softmax(fptr(bufs[0]), fmptr(bufs[1]), u[0], u[1], env);
    }
    if (name == "causal_mask") {
        if (int rc = need(1, 12)) return rc;
        if (small(0, (uint64_t)u[0] * u[1] * u[2])) return too_small();
        return sdvk::table_causal_mask(fmptr(bufs[0]), u[0], u[1], u[2], env);
    }
    return set_err(ctx, SDVK_E_KERNEL, "unknown kernel " + name);
}

// One warp waits on phase 0 of an mbarrier that nothing arrives on, through the same bounded wait
// every pipeline kernel uses (mbar_wait).  The wait runs out after timeout_ns of global time; the
// warp then records kErrTimeout in the context's error word and the kernel returns normally.
__global__ void __launch_bounds__(32) wait_selftest_kernel(uint32_t* err, uint64_t timeout_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        sdvk::mbar_init(&bar, 1);
        sdvk::fence_mbar_init();
    }
    __syncwarp();
    const bool done = sdvk::mbar_wait(&bar, 0, timeout_ns);
    if (!done && threadIdx.x == 0) atomicOr(err, sdvk::kErrTimeout);
}

}  // namespace

extern "C" {

const char* sdvk_status_string(int s) {
    switch (s) {
        case SDVK_OK: return "ok";
        case SDVK_E_OOM: return "out of memory";
        case SDVK_E_SHAPE: return "unsupported shape or layout";
        case SDVK_E_CUDA: return "CUDA error";
        case SDVK_E_TIMEOUT: return "timeout";
        case SDVK_E_ARG: return "invalid argument";
        case SDVK_E_KERNEL: return "unknown kernel";
        case SDVK_E_STATE: return "step protocol misuse";
        case SDVK_E_NOT_FINITE: return "non-finite values";
        default: return "unknown status";
    }
}

int sdvk_ctx_create(int device, sdvk_ctx** out) {
    if (!out) return SDVK_E_ARG;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return SDVK_E_ARG;
    auto* ctx = new (std::nothrow) sdvk_ctx();
    if (!ctx) return SDVK_E_OOM;
    ctx->device = device;
    int rc = cuda_err(ctx, cudaSetDevice(device), "cudaSetDevice");
    cudaDeviceProp prop{};
    if (!rc) rc = cuda_err(ctx, cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if (!rc && prop.major != 10) rc = set_err(ctx, SDVK_E_CUDA, "sdvk-b200 kernels need an sm_100 (B200) device");
    if (!rc) rc = cuda_err(ctx, cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking), "stream");
    if (!rc) rc = cuda_err(ctx, cudaMalloc(&ctx->err_dev, 256), "cudaMalloc(error word)");
    if (!rc) rc = cuda_err(ctx, cudaMemset(ctx->err_dev, 0, 256), "cudaMemset");
    if (!rc) rc = cuda_err(ctx, cudaEventCreateWithFlags(&ctx->step_done, cudaEventDisableTiming), "event");
    if (!rc) rc = cuda_err(ctx, cudaStreamCreateWithFlags(&ctx->side, cudaStreamNonBlocking), "side stream");
    if (!rc) rc = cuda_err(ctx, cudaEventCreateWithFlags(&ctx->fork, cudaEventDisableTiming), "event");
    if (!rc) rc = cuda_err(ctx, cudaEventCreateWithFlags(&ctx->join, cudaEventDisableTiming), "event");
    if (!rc) {
        ctx->samp_ws_bytes = sdvk::sampler_workspace(prop.multiProcessorCount);
        rc = cuda_err(ctx, cudaMalloc(&ctx->samp_ws, ctx->samp_ws_bytes), "cudaMalloc(sampler workspace)");
    }
    if (rc) {
        sdvk_ctx_destroy(ctx);
        return rc;
    }
    ctx->flag_dev = ctx->err_dev + 32;
    ctx->stream = ctx->own_stream;
    ctx->num_sms = prop.multiProcessorCount;
    ctx->device_name = prop.name;
    *out = ctx;
    return SDVK_OK;
}

int sdvk_ctx_destroy(sdvk_ctx* ctx) {
    if (!ctx) return SDVK_E_ARG;
    cudaSetDevice(ctx->device);
    if (ctx->own_stream) cudaStreamSynchronize(ctx->own_stream);
    if (ctx->step_done) cudaEventDestroy(ctx->step_done);
    if (ctx->side) cudaStreamSynchronize(ctx->side);
    if (ctx->fork) cudaEventDestroy(ctx->fork);
    if (ctx->join) cudaEventDestroy(ctx->join);
    if (ctx->side) cudaStreamDestroy(ctx->side);
    if (ctx->err_dev) cudaFree(ctx->err_dev);
    if (ctx->samp_ws) cudaFree(ctx->samp_ws);
    if (ctx->scratch) {
        cudaStreamSynchronize(ctx->stream);
        cudaFree(ctx->scratch);
    }
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return SDVK_OK;
}

int sdvk_ctx_set_stream(sdvk_ctx* ctx, void* s) {
    if (!ctx) return SDVK_E_ARG;
    ctx->stream = static_cast<cudaStream_t>(s);  // NULL: the legacy default stream
    return SDVK_OK;
}

int sdvk_ctx_reset_stream(sdvk_ctx* ctx) {
    if (!ctx) return SDVK_E_ARG;
    ctx->stream = ctx->own_stream;
    return SDVK_OK;
}

void* sdvk_ctx_stream(sdvk_ctx* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

int sdvk_ctx_set_timeout_ms(sdvk_ctx* ctx, uint32_t ms) {
    if (!ctx || ms == 0) return SDVK_E_ARG;
    ctx->timeout_ns = (uint64_t)ms * 1000000ull;
    return SDVK_OK;
}

int sdvk_ctx_set_precision(sdvk_ctx* ctx, int precision) {
    if (!ctx || (precision != SDVK_PRECISION_REFERENCE && precision != SDVK_PRECISION_FAST)) return SDVK_E_ARG;
    ctx->precision = precision;
    return SDVK_OK;
}

int sdvk_device_report(sdvk_ctx* ctx, char* buf, size_t len) {
    if (!ctx || !buf || !len) return SDVK_E_ARG;
    size_t free_b = 0, total_b = 0;
    use_device(ctx);
    cudaMemGetInfo(&free_b, &total_b);
    std::snprintf(buf, len, "device|%d\nname|%s\nsms|%d\nmem_total_mb|%llu\nmem_free_mb|%llu\n", ctx->device,
                  ctx->device_name.c_str(), ctx->num_sms, (unsigned long long)(total_b >> 20),
                  (unsigned long long)(free_b >> 20));
    return SDVK_OK;
}

int sdvk_selftest_wait(sdvk_ctx* ctx) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    wait_selftest_kernel<<<1, 32, 0, ctx->stream>>>(ctx->err_dev, ctx->timeout_ns);
    return cuda_err(ctx, cudaGetLastError(), "sdvk_selftest_wait");
}

int sdvk_device_memory(sdvk_ctx* ctx, uint64_t* free_bytes, uint64_t* total_bytes) {
    if (!ctx || !free_bytes || !total_bytes) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    size_t f = 0, t = 0;
    if (int rc = cuda_err(ctx, cudaMemGetInfo(&f, &t), "cudaMemGetInfo")) return rc;
    *free_bytes = f;
    *total_bytes = t;
    return SDVK_OK;
}

const char* sdvk_last_error(sdvk_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "no context"; }

// ------------------------------------------------------------------ memory
int sdvk_alloc(sdvk_ctx* ctx, uint64_t bytes, void** dptr) {
    if (!ctx || !dptr) return SDVK_E_ARG;
    *dptr = nullptr;
    if (int rc = use_device(ctx)) return rc;
    if (cudaMalloc(dptr, bytes ? bytes : 256) != cudaSuccess) {
        cudaGetLastError();
        return set_err(ctx, SDVK_E_OOM, "device allocation of " + std::to_string(bytes) + " bytes failed");
    }
    return SDVK_OK;
}

int sdvk_free(sdvk_ctx* ctx, void* dptr) {
    if (!ctx) return SDVK_E_ARG;
    if (!dptr) return SDVK_OK;
    if (int rc = use_device(ctx)) return rc;
    return cuda_err(ctx, cudaFree(dptr), "cudaFree");
}

int sdvk_host_alloc(sdvk_ctx* ctx, uint64_t bytes, void** hptr) {
    if (!ctx || !hptr) return SDVK_E_ARG;
    *hptr = nullptr;
    if (cudaMallocHost(hptr, bytes ? bytes : 256) != cudaSuccess) {
        cudaGetLastError();
        return set_err(ctx, SDVK_E_OOM, "pinned host allocation failed");
    }
    return SDVK_OK;
}

int sdvk_host_free(sdvk_ctx* ctx, void* hptr) {
    if (!ctx) return SDVK_E_ARG;
    return hptr ? cuda_err(ctx, cudaFreeHost(hptr), "cudaFreeHost") : SDVK_OK;
}

int sdvk_upload(sdvk_ctx* ctx, void* dst, const void* src, uint64_t bytes) {
    if (!ctx || (!dst && bytes) || (!src && bytes)) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    if (int rc = cuda_err(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream), "upload"))
        return rc;
    return cuda_err(ctx, cudaStreamSynchronize(ctx->stream), "upload sync");
}

int sdvk_download(sdvk_ctx* ctx, void* dst, const void* src, uint64_t bytes) {
    if (!ctx || (!dst && bytes) || (!src && bytes)) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    if (int rc = cuda_err(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream), "download"))
        return rc;
    if (int rc = cuda_err(ctx, cudaStreamSynchronize(ctx->stream), "download sync")) return rc;
    return collect_device_error(ctx);
}

int sdvk_upload_async(sdvk_ctx* ctx, void* dst, const void* src, uint64_t bytes) {
    if (!ctx || (!dst && bytes) || (!src && bytes)) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return cuda_err(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream), "upload_async");
}

int sdvk_download_async(sdvk_ctx* ctx, void* dst, const void* src, uint64_t bytes) {
    if (!ctx || (!dst && bytes) || (!src && bytes)) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return cuda_err(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream), "download_async");
}

int sdvk_copy(sdvk_ctx* ctx, void* dst, const void* src, uint64_t bytes) {
    if (!ctx || (!dst && bytes) || (!src && bytes)) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return cuda_err(ctx, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, ctx->stream), "copy");
}

int sdvk_fill_u32(sdvk_ctx* ctx, void* dst, uint32_t value, uint64_t bytes) {
    if (!ctx || !dst || bytes % 4) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    if (value == 0) return cuda_err(ctx, cudaMemsetAsync(dst, 0, bytes, ctx->stream), "fill");
    if ((value & 0xFFu) * 0x01010101u == value)
        return cuda_err(ctx, cudaMemsetAsync(dst, (int)(value & 0xFF), bytes, ctx->stream), "fill");
    return set_err(ctx, SDVK_E_ARG, "sdvk_fill_u32 supports byte-repeating patterns only");
}

// ------------------------------------------------------------------ step protocol
int sdvk_step_begin(sdvk_ctx* ctx) {
    if (!ctx) return SDVK_E_ARG;
    if (ctx->in_step) return set_err(ctx, SDVK_E_STATE, "step_begin inside an open step");
    ctx->in_step = true;
    ctx->step_recorded = false;
    return use_device(ctx);
}

int sdvk_step_end(sdvk_ctx* ctx) {
    if (!ctx) return SDVK_E_ARG;
    if (!ctx->in_step) return set_err(ctx, SDVK_E_STATE, "step_end without step_begin");
    ctx->in_step = false;
    if (int rc = use_device(ctx)) return rc;
    if (int rc = cuda_err(ctx, cudaEventRecord(ctx->step_done, ctx->stream), "step event")) return rc;
    ctx->step_recorded = true;
    return SDVK_OK;
}

int sdvk_step_wait(sdvk_ctx* ctx, uint32_t timeout_ms) {
    if (!ctx) return SDVK_E_ARG;
    if (!ctx->step_recorded) return set_err(ctx, SDVK_E_STATE, "step_wait without a finished step");
    const auto t0 = std::chrono::steady_clock::now();
    if (timeout_ms == 0) {  // no deadline: block in the driver (no polling latency)
        if (int rc = cuda_err(ctx, cudaEventSynchronize(ctx->step_done), "step wait")) return rc;
        ctx->step_recorded = false;
        return collect_device_error(ctx);
    }
    while (true) {
        cudaError_t e = cudaEventQuery(ctx->step_done);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return cuda_err(ctx, e, "step wait");
        if (timeout_ms && std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms))
            return set_err(ctx, SDVK_E_TIMEOUT, "step did not finish within the deadline");
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    ctx->step_recorded = false;
    return collect_device_error(ctx);
}

int sdvk_synchronize(sdvk_ctx* ctx) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    if (int rc = cuda_err(ctx, cudaStreamSynchronize(ctx->stream), "synchronize")) return rc;
    return collect_device_error(ctx);
}

// ------------------------------------------------------------------ typed entry points
int sdvk_gemm_q8_nt(sdvk_ctx* ctx, const void* A, int a_dtype, const int8_t* q, const float* s, const float* bias,
                    void* C, int c_dtype, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldc,
                    uint32_t batch, uint64_t sA, uint64_t sC, int accumulate) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    sdvk::GemmQ8Desc d{};
    d.x = A;
    d.x_dtype = a_dtype;
    d.ldx = lda ? lda : K;
    d.sx = sA;
    d.wq = q;
    d.ws = s;
    d.ldw = K;
    d.sw = 0;
    d.bias = bias;
    d.c = C;
    d.c_dtype = c_dtype;
    d.ldc = ldc ? ldc : N;
    d.sc = sC;
    d.xrows = M;
    d.wrows = N;
    d.K = K;
    d.batch = batch ? batch : 1;
    d.nn = false;
    d.accumulate = accumulate != 0;
    return sdvk::gemm_q8(d, env_of(ctx));
}

int sdvk_gemm_q8_nn(sdvk_ctx* ctx, const int8_t* q, const float* s, const void* B, int b_dtype, const float* bias,
                    void* C, int c_dtype, uint32_t M, uint32_t N, uint32_t K, uint32_t lda, uint32_t ldb,
                    uint32_t ldc, uint32_t batch, uint64_t sA, uint64_t sB, uint64_t sC, int accumulate) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    sdvk::GemmQ8Desc d{};
    d.x = B;
    d.x_dtype = b_dtype;
    d.ldx = ldb ? ldb : N;
    d.sx = sB;
    d.wq = q;
    d.ws = s;
    d.ldw = lda ? lda : K;
    d.sw = sA;
    d.bias = bias;
    d.c = C;
    d.c_dtype = c_dtype;
    d.ldc = ldc ? ldc : N;
    d.sc = sC;
    d.xrows = N;
    d.wrows = M;
    d.K = K;
    d.batch = batch ? batch : 1;
    d.nn = true;
    d.accumulate = accumulate != 0;
    return sdvk::gemm_q8(d, env_of(ctx));
}

int sdvk_attention(sdvk_ctx* ctx, const sdvk_attn_desc* desc) {
    if (!ctx || !desc) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::attention(*desc, env_of(ctx));
}

int sdvk_fused_attn_supported(uint32_t C, uint32_t heads) {
    if (!C || !heads || C % heads) return 0;
    const uint32_t hd = C / heads;
    return hd > 0 && hd <= 64;
}

int sdvk_fused_attention(sdvk_ctx* ctx, const void* q, const void* k, const void* v, void* out, uint32_t Tq,
                         uint32_t Tk, uint32_t C, uint32_t heads, int causal) {
    if (!ctx) return SDVK_E_ARG;
    if (!sdvk_fused_attn_supported(C, heads))
        return set_err(ctx, SDVK_E_SHAPE, "fusedAttention: unsupported C=" + std::to_string(C) +
                                              " heads=" + std::to_string(heads));
    const uint32_t hd = C / heads;
    sdvk_attn_desc d{};
    d.q = q;
    d.k = k;
    d.v = v;
    d.o = out;
    d.dtype = SDVK_F32;
    d.o_dtype = SDVK_F32;
    d.batch = 1;
    d.heads = heads;
    d.Tq = Tq;
    d.Tk = Tk;
    d.hd = hd;
    d.ldq = d.ldk = d.ldv = d.ldo = C;
    d.hq = d.hk = d.hv = d.ho = hd;
    d.scale = 1.0f / std::sqrt((float)hd);
    d.causal = causal;
    return sdvk_attention(ctx, &d);
}

int sdvk_sampler_step(sdvk_ctx* ctx, const sdvk_sampler_step_desc* desc) {
    if (!ctx || !desc) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::sampler_step(*desc, ctx->samp_ws, ctx->samp_ws_bytes, env_of(ctx));
}

int sdvk_sampler_scale(sdvk_ctx* ctx, const float* x, float* out, uint64_t n, float sigma) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::sampler_scale(x, out, n, sigma, env_of(ctx));
}

int sdvk_check_finite(sdvk_ctx* ctx, const void* x, int dtype, uint64_t n) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    auto env = env_of(ctx);
    if (int rc = cuda_err(ctx, cudaMemsetAsync(ctx->flag_dev, 0, 4, ctx->stream), "memset")) return rc;
    if (int rc = sdvk::check_finite(x, dtype, n, ctx->flag_dev, env)) return rc;
    uint32_t flag = 0;
    if (int rc = cuda_err(ctx, cudaMemcpyAsync(&flag, ctx->flag_dev, 4, cudaMemcpyDeviceToHost, ctx->stream), "copy"))
        return rc;
    if (int rc = cuda_err(ctx, cudaStreamSynchronize(ctx->stream), "sync")) return rc;
    return flag ? set_err(ctx, SDVK_E_NOT_FINITE, "non-finite value found") : SDVK_OK;
}

int sdvk_geglu_interleave(sdvk_ctx* ctx, const int8_t* q, const float* s, const float* bias, uint32_t F, uint32_t K,
                          int8_t* q_out, float* s_out, float* bias_out) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::geglu_interleave(q, s, bias, F, K, q_out, s_out, bias_out, env_of(ctx));
}

int sdvk_gemm_q8_nt_geglu(sdvk_ctx* ctx, const void* A, int a_dtype, const int8_t* q, const float* s,
                          const float* bias, void* C, uint32_t M, uint32_t F, uint32_t K, uint32_t lda, uint32_t ldc) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    sdvk::GemmQ8Desc d{};
    d.x = A;
    d.x_dtype = a_dtype;
    d.ldx = lda ? lda : K;
    d.wq = q;
    d.ws = s;
    d.ldw = K;
    d.bias = bias;
    d.c = C;
    d.c_dtype = SDVK_F16;
    d.ldc = ldc ? ldc : F;
    d.xrows = M;
    d.wrows = 2 * F;
    d.K = K;
    d.batch = 1;
    d.geglu = true;
    return sdvk::gemm_q8(d, env_of(ctx));
}

// ------------------------------------------------------------------ transformer block
int sdvk_layernorm(sdvk_ctx* ctx, const float* x, const float* gamma, const float* beta, void* y, int y_dtype,
                   uint32_t rows, uint32_t d, uint64_t ldx, uint64_t ldy, float eps) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::layernorm(x, gamma, beta, y, y_dtype, rows, d, ldx, ldy, eps, env_of(ctx));
}

int sdvk_geglu(sdvk_ctx* ctx, const void* h, void* y, uint32_t rows, uint32_t F, uint64_t ldh, uint64_t ldy) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::geglu(h, y, rows, F, ldh, ldy, env_of(ctx));
}

uint64_t sdvk_transformer_block_workspace(const sdvk_block_desc* desc) {
    return desc ? sdvk::block_workspace_bytes(*desc) : 0;
}

int sdvk_transformer_block(sdvk_ctx* ctx, const sdvk_block_desc* desc, void* workspace, uint64_t workspace_bytes) {
    if (!ctx || !desc) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::transformer_block(*desc, workspace, workspace_bytes, env_of(ctx));
}

int sdvk_transformer_block_static(sdvk_ctx* ctx, const sdvk_block_desc* desc) {
    if (!ctx || !desc) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    // the shape checks of the workspace entry point first, so a bad description gets its own error
    if (!desc->x) return set_err(ctx, SDVK_E_ARG, "null pointer");
    if (desc->batch && desc->T && (desc->heads == 0 || desc->C % desc->heads || desc->C / desc->heads > 64))
        return set_err(ctx, SDVK_E_SHAPE, "heads must divide C with head dim <= 64");
    if (desc->batch && desc->T && desc->Tctx && !desc->ctx) return set_err(ctx, SDVK_E_ARG, "null context");
    const uint64_t need = sdvk::block_workspace_bytes(*desc);
    if (need > SDVK_STATIC_SCRATCH_BYTES)
        return set_err(ctx, SDVK_E_SHAPE, "the block needs " + std::to_string(need) +
                                              " bytes of scratch, more than the static array's " +
                                              std::to_string(SDVK_STATIC_SCRATCH_BYTES));
    void* scratch = nullptr;
    const sdvk::LaunchEnv env = env_of(ctx);
    if (int rc = sdvk::static_scratch(ctx->device, &scratch, env)) return rc;
    return sdvk::transformer_block(*desc, scratch, SDVK_STATIC_SCRATCH_BYTES, env);
}

// ------------------------------------------------------------------ multi-GPU (CFG pair)
int sdvk_cfg_combine(sdvk_ctx* ctx, const float* cond, const float* uncond, float* out, uint64_t n, float cfg,
                     float rescale) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::cfg_combine(cond, uncond, out, n, cfg, rescale, env_of(ctx));
}

int sdvk_q8_0_ingest(sdvk_ctx* ctx, const void* blocks, uint64_t rows, uint64_t cols, int8_t* q, uint64_t ldq,
                     float* scales) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::q8_0_ingest(blocks, rows, cols, q, ldq ? ldq : cols, scales, env_of(ctx));
}

uint64_t sdvk_conv3x3_workspace(uint32_t cin, uint32_t H, uint32_t W, int stride, int x_dtype) {
    return sdvk::conv3x3_workspace(cin, H, W, stride > 0 ? (uint32_t)stride : 0u, x_dtype);
}

int sdvk_conv3x3_q8(sdvk_ctx* ctx, const void* x, int x_dtype, const int8_t* q, const float* s, const float* bias,
                    void* y, int y_dtype, uint32_t batch, uint32_t cin, uint32_t cout, uint32_t H, uint32_t W,
                    int stride, int pad_off, void* workspace, uint64_t workspace_bytes) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::conv3x3_q8(x, x_dtype, q, s, bias, y, y_dtype, batch, cin, cout, H, W,
                            stride > 0 ? (uint32_t)stride : 0u, pad_off, workspace, workspace_bytes, env_of(ctx));
}

int sdvk_conv3x3_implicit_ok(uint32_t batch, uint32_t cin, uint32_t H, uint32_t W, int stride) {
    return stride > 0 && sdvk::conv_implicit_ok(batch, cin, H, W, (uint32_t)stride) ? 1 : 0;
}

int sdvk_conv3x3_weights_f16(sdvk_ctx* ctx, const int8_t* q, const float* s, uint32_t cout, uint32_t cin, void* w16) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    if (w16 && (reinterpret_cast<uintptr_t>(w16) & 15u))
        return sdvk::fail(env_of(ctx), SDVK_E_SHAPE, "w16 must be 16-byte aligned");
    return sdvk::conv_weights_f16(q, s, cout, cin, static_cast<__half*>(w16), env_of(ctx));
}

int sdvk_conv3x3_nhwc(sdvk_ctx* ctx, const void* x, const void* w16, const float* bias, uint64_t bias_stride,
                      int accumulate, void* y, int y_dtype, uint32_t batch, uint32_t cin, uint32_t cout, uint32_t H,
                      uint32_t W, int stride, int pad_off) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    sdvk::ConvImplicitDesc d{static_cast<const __half*>(x), static_cast<const __half*>(w16), bias, bias_stride,
                             accumulate != 0, y, y_dtype, batch, cin, cout, H, W,
                             stride > 0 ? (uint32_t)stride : 0u, pad_off};
    return sdvk::conv3x3_implicit(d, env_of(ctx));
}

uint64_t sdvk_groupnorm_workspace(uint32_t batch, uint32_t C, uint32_t P, uint32_t G) {
    return sdvk::groupnorm_workspace(batch, C, P, G);
}

int sdvk_groupnorm(sdvk_ctx* ctx, const float* x, const float* gamma, const float* beta, float* y, uint32_t batch,
                   uint32_t C, uint32_t P, uint32_t G, float eps, int silu, void* workspace, uint64_t workspace_bytes) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::groupnorm(x, gamma, beta, y, batch, C, P, G, eps, silu ? 1u : 0u, workspace, workspace_bytes,
                           env_of(ctx));
}

int sdvk_groupnorm_cl(sdvk_ctx* ctx, const float* x, const float* gamma, const float* beta, void* y, uint32_t batch,
                      uint32_t C, uint32_t P, uint32_t G, float eps, int silu, void* workspace,
                      uint64_t workspace_bytes) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::groupnorm_ex(x, gamma, beta, y, SDVK_F16, batch, C, P, G, eps, silu ? 1u : 0u, workspace,
                              workspace_bytes, env_of(ctx), true);
}

int sdvk_comm_unique_id(void* id) { return sdvk::comm_unique_id(id); }

int sdvk_comm_create(sdvk_ctx* ctx, int nranks, int rank, const void* id, uint32_t timeout_ms, sdvk_comm** out) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::comm_create(nranks, rank, id, timeout_ms ? timeout_ms : 30000, out, env_of(ctx));
}

int sdvk_comm_destroy(sdvk_comm* comm) { return sdvk::comm_destroy(comm); }

int sdvk_comm_abort(sdvk_comm* comm) { return sdvk::comm_abort(comm); }

int sdvk_allgather(sdvk_ctx* ctx, sdvk_comm* comm, const void* send, void* recv, uint64_t count, int dtype) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::allgather(comm, send, recv, count, dtype, (uint32_t)(ctx->timeout_ns / 1000000ull), env_of(ctx));
}

int sdvk_comm_wait(sdvk_ctx* ctx, sdvk_comm* comm, uint32_t timeout_ms) {
    if (!ctx) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    if (int rc = sdvk::comm_wait(comm, timeout_ms ? timeout_ms : 30000, env_of(ctx))) return rc;
    return collect_device_error(ctx);
}

// ------------------------------------------------------------------ name dispatch
int sdvk_dispatch(sdvk_ctx* ctx, const char* kernel, const sdvk_buf* bufs, uint32_t nbufs, const void* push,
                  uint32_t push_bytes, uint32_t gx, uint32_t gy, uint32_t gz) {
    (void)gx;
    (void)gy;
    if (!ctx || !kernel || !bufs || !push) return SDVK_E_ARG;
    const std::string name(kernel);
    const uint32_t batch = gz ? gz : 1;  // the shaders batch over the z workgroup index
    auto is = [&](std::initializer_list<const char*> names) {
        for (const char* n : names)
            if (name == n) return true;
        return false;
    };
    if (is({"gemm_nt_q8", "gemm_nt_q8_v", "gemm_nt_q8_v_bm128", "gemm_nt_q8_v_bk32", "gemm_nt_q8_v_bm128_bk32",
            "gemm_nt_q8_v_b", "gemm_nt_q8_v_bm128_b"})) {
        const bool with_bias = name.size() > 2 && name.compare(name.size() - 2, 2, "_b") == 0;
        if (push_bytes < sizeof(Pg) || nbufs < (with_bias ? 5u : 4u))
            return set_err(ctx, SDVK_E_ARG, name + ": needs " + (with_bias ? "5" : "4") + " buffers and a 48-byte Pg");
        Pg pc;
        std::memcpy(&pc, push, sizeof(pc));
        const uint64_t lda = pc.lda ? pc.lda : pc.K, ldc = pc.ldc ? pc.ldc : pc.N;
        // Buffer extents the shape reads/writes (fp32 A/C/S/bias, int8 payload).
        const uint64_t a_end = ((uint64_t)(batch - 1) * pc.sA + (uint64_t)(pc.M ? pc.M - 1 : 0) * lda + pc.K) * 4;
        const uint64_t c_end = ((uint64_t)(batch - 1) * pc.sC + (uint64_t)(pc.M ? pc.M - 1 : 0) * ldc + pc.N) * 4;
        const uint64_t q_end = (uint64_t)pc.N * pc.K, s_end = (uint64_t)pc.N * pc.K / 32 * 4;
        if (!buf_holds(bufs[0], a_end) || !buf_holds(bufs[1], q_end) || !buf_holds(bufs[2], c_end) ||
            !buf_holds(bufs[3], s_end) || (with_bias && !buf_holds(bufs[4], (uint64_t)pc.N * 4)))
            return set_err(ctx, SDVK_E_ARG, name + ": a buffer is smaller than the shape needs");
        const float* bias = (with_bias && pc.mode == 0) ? static_cast<const float*>(buf_ptr(bufs[4])) : nullptr;
        return sdvk_gemm_q8_nt(ctx, buf_ptr(bufs[0]), SDVK_F32, static_cast<const int8_t*>(buf_ptr(bufs[1])),
                               static_cast<const float*>(buf_ptr(bufs[3])), bias, buf_mptr(bufs[2]), SDVK_F32, pc.M,
                               pc.N, pc.K, (uint32_t)lda, (uint32_t)ldc, batch, pc.sA, pc.sC, pc.mode != 0);
    }
    if (is({"gemm_nn_q8", "gemm_nn_q8_v"})) {
        if (push_bytes < sizeof(Pg) || nbufs < 4u)
            return set_err(ctx, SDVK_E_ARG, name + ": needs 4 buffers and a 48-byte Pg");
        Pg pc;
        std::memcpy(&pc, push, sizeof(pc));
        const uint64_t lda = pc.lda ? pc.lda : pc.K, ldb = pc.ldb ? pc.ldb : pc.N, ldc = pc.ldc ? pc.ldc : pc.N;
        const uint64_t q_end = (uint64_t)(batch - 1) * pc.sA + (uint64_t)(pc.M ? pc.M - 1 : 0) * lda + pc.K;
        const uint64_t b_end = ((uint64_t)(batch - 1) * pc.sB + (uint64_t)(pc.K ? pc.K - 1 : 0) * ldb + pc.N) * 4;
        const uint64_t c_end = ((uint64_t)(batch - 1) * pc.sC + (uint64_t)(pc.M ? pc.M - 1 : 0) * ldc + pc.N) * 4;
        if (!buf_holds(bufs[0], q_end) || !buf_holds(bufs[1], b_end) || !buf_holds(bufs[2], c_end) ||
            !buf_holds(bufs[3], (q_end + 31) / 32 * 4))
            return set_err(ctx, SDVK_E_ARG, name + ": a buffer is smaller than the shape needs");
        return sdvk_gemm_q8_nn(ctx, static_cast<const int8_t*>(buf_ptr(bufs[0])),
                               static_cast<const float*>(buf_ptr(bufs[3])), buf_ptr(bufs[1]), SDVK_F32, nullptr,
                               buf_mptr(bufs[2]), SDVK_F32, pc.M, pc.N, pc.K, (uint32_t)lda, (uint32_t)ldb,
                               (uint32_t)ldc, batch, pc.sA, pc.sB, pc.sC, pc.mode != 0);
    }
    if (is({"layernorm_fwd"})) {
        if (push_bytes < sizeof(LnPush) || nbufs < 4u)
            return set_err(ctx, SDVK_E_ARG, name + ": needs 4 buffers and a 16-byte push");
        LnPush pc;
        std::memcpy(&pc, push, sizeof(pc));
        const uint64_t xy_end = (uint64_t)pc.rows * pc.d * 4;
        if (!buf_holds(bufs[0], xy_end) || !buf_holds(bufs[3], xy_end) ||
            (pc.affine && (!buf_holds(bufs[1], (uint64_t)pc.d * 4) || !buf_holds(bufs[2], (uint64_t)pc.d * 4))))
            return set_err(ctx, SDVK_E_ARG, name + ": a buffer is smaller than the shape needs");
        return sdvk_layernorm(ctx, static_cast<const float*>(buf_ptr(bufs[0])),
                              pc.affine ? static_cast<const float*>(buf_ptr(bufs[1])) : nullptr,
                              pc.affine ? static_cast<const float*>(buf_ptr(bufs[2])) : nullptr, buf_mptr(bufs[3]),
                              SDVK_F32, pc.rows, pc.d, pc.d, pc.d, pc.eps);
    }
    if (is({"groupnorm"})) {
        if (push_bytes < sizeof(GnPush) || nbufs < 4u)
            return set_err(ctx, SDVK_E_ARG, name + ": needs 4 buffers and a 20-byte push");
        GnPush pc;
        std::memcpy(&pc, push, sizeof(pc));
        const uint64_t xy_end = (uint64_t)pc.C * pc.P * 4;
        if (!buf_holds(bufs[0], xy_end) || !buf_holds(bufs[3], xy_end) || !buf_holds(bufs[1], (uint64_t)pc.C * 4) ||
            !buf_holds(bufs[2], (uint64_t)pc.C * 4))
            return set_err(ctx, SDVK_E_ARG, name + ": a buffer is smaller than the shape needs");
        const uint64_t need = sdvk::groupnorm_workspace(1, pc.C, pc.P, pc.G);
        if (need == 0) return set_err(ctx, SDVK_E_SHAPE, name + ": C must be a multiple of G");
        if (int rc = use_device(ctx)) return rc;
        if (ctx->scratch_bytes < need) {  // grows once; stream-ordered so queued work keeps its copy valid
            if (ctx->scratch) {
                cudaStreamSynchronize(ctx->stream);
                cudaFree(ctx->scratch);
                ctx->scratch = nullptr;
                ctx->scratch_bytes = 0;
            }
            if (cudaMalloc(&ctx->scratch, need) != cudaSuccess) {
                cudaGetLastError();
                return set_err(ctx, SDVK_E_OOM, name + ": workspace allocation failed");
            }
            ctx->scratch_bytes = need;
        }
        return sdvk_groupnorm(ctx, static_cast<const float*>(buf_ptr(bufs[0])),
                              static_cast<const float*>(buf_ptr(bufs[1])), static_cast<const float*>(buf_ptr(bufs[2])),
                              static_cast<float*>(buf_mptr(bufs[3])), 1, pc.C, pc.P, pc.G, pc.eps, pc.act == 1u,
                              ctx->scratch, ctx->scratch_bytes);
    }
    if (is({"fused_attn", "fused_attn_tiled"})) {
        if (push_bytes < sizeof(FaPush) || nbufs < 4u)
            return set_err(ctx, SDVK_E_ARG, name + ": needs 4 buffers and a 36-byte FaPush");
        FaPush pc;
        std::memcpy(&pc, push, sizeof(pc));
        if (!pc.heads || !pc.hd || pc.hd > 64 || (uint64_t)pc.heads * pc.hd > pc.C)
            return set_err(ctx, SDVK_E_SHAPE, name + ": head layout not supported");
        const uint64_t q_end = (uint64_t)pc.Tq * pc.C * 4, kv_end = (uint64_t)pc.Tk * pc.C * 4;
        if (!buf_holds(bufs[0], q_end) || !buf_holds(bufs[1], kv_end) || !buf_holds(bufs[2], kv_end) ||
            !buf_holds(bufs[3], q_end))
            return set_err(ctx, SDVK_E_ARG, name + ": a buffer is smaller than the shape needs");
        sdvk_attn_desc d{};
        d.q = buf_ptr(bufs[0]);
        d.k = buf_ptr(bufs[1]);
        d.v = buf_ptr(bufs[2]);
        d.o = buf_mptr(bufs[3]);
        d.dtype = SDVK_F32;
        d.o_dtype = SDVK_F32;
        d.batch = 1;
        d.heads = pc.heads;
        d.Tq = pc.Tq;
        d.Tk = pc.Tk;
        d.hd = pc.hd;
        d.ldq = d.ldk = d.ldv = d.ldo = pc.C;
        d.hq = d.hk = d.hv = d.ho = pc.hd;
        d.scale = pc.scale;
        d.causal = (int)pc.causal;
        return sdvk_attention(ctx, &d);
    }
    return dispatch_table(ctx, name, bufs, nbufs, push, push_bytes, batch);
}

}  // extern "C"

// ------------------------------------------------------------------ the SDXL UNet pass
int sdvk_unet_create(sdvk_ctx* ctx, const sdvk_unet_desc* desc, sdvk_unet** out) {
    if (!ctx || !desc || !out) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::unet_create(*desc, out, env_of(ctx));
}

int sdvk_unet_plan(const sdvk_unet_desc* desc, sdvk_unet** out) {
    if (!desc || !out) return SDVK_E_ARG;
    const sdvk::LaunchEnv env{nullptr, nullptr, 0, -1, 148, nullptr, SDVK_PRECISION_REFERENCE, nullptr, nullptr, nullptr};
    return sdvk::unet_plan(*desc, out, env);
}

int sdvk_unet_destroy(sdvk_unet* unet) { return sdvk::unet_destroy(unet); }

int sdvk_unet_init_random(sdvk_ctx* ctx, sdvk_unet* unet, uint64_t seed) {
    if (!ctx || !unet) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::unet_init_random(unet, seed, env_of(ctx));
}

int sdvk_unet_prepare(sdvk_ctx* ctx, sdvk_unet* unet) {
    if (!ctx || !unet) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::unet_prepare(unet, env_of(ctx));
}

uint32_t sdvk_unet_tensor_count(const sdvk_unet* unet) { return sdvk::unet_tensor_count(unet); }

int sdvk_unet_tensor(const sdvk_unet* unet, uint32_t index, sdvk_unet_tensor_info* out) {
    return sdvk::unet_tensor(unet, index, out);
}

int sdvk_unet_tensor_layout(const sdvk_unet* unet, uint32_t index, sdvk_unet_param_layout* out) {
    return sdvk::unet_tensor_layout(unet, index, out);
}

uint64_t sdvk_unet_flops(const sdvk_unet* unet) { return sdvk::unet_flops(unet); }

uint64_t sdvk_unet_workspace_bytes(const sdvk_unet* unet) { return sdvk::unet_workspace_bytes(unet); }

uint64_t sdvk_unet_launches(const sdvk_unet* unet) { return sdvk::unet_launches(unet); }

uint64_t sdvk_unet_parameter_bytes(const sdvk_unet* unet) { return sdvk::unet_parameter_bytes(unet); }

int sdvk_unet_forward(sdvk_ctx* ctx, sdvk_unet* unet, const float* x, const float* timesteps, const float* adm,
                      const void* context, int ctx_dtype, float* out) {
    if (!ctx || !unet) return SDVK_E_ARG;
    if (int rc = use_device(ctx)) return rc;
    return sdvk::unet_forward(unet, x, timesteps, adm, context, ctx_dtype, out, env_of(ctx));
}
