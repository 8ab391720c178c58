// collective.cu -- the multi-GPU pieces of the sampler step, for the CFG-pair mode (one GPU runs the
// conditional pass, its partner the unconditional one):
//   cfg_combine_kernel  res = eps_u + cfg * (eps_c - eps_u), then the optional "mimic scale"
//                       rescale of the guided output's spread toward the unconditional one's, as
//                       evalGuided does on the host (src/Modules/Diffusion/sdvkgen.cpp:3825-3845);
//                       statistics in double, in the reference's order of operations
//   sdvk_comm / all-gather  an NCCL communicator per context; the all-gather of the two halves
//                       lands [cond | uncond] in every rank's memory, so both ranks combine the same
//                       bytes and keep bit-identical latents without a broadcast.
// Failure handling: the communicator is created non-blocking and every host-side wait polls
// ncclCommGetAsyncError against a deadline; a peer that never joins or stops answering turns into
// SDVK_E_TIMEOUT and the communicator is aborted (ncclCommAbort), with no device-side wait at all.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>

#include "backend.hpp"

struct sdvk_comm {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0;
    bool aborted = false;
    // NCCL connects the peers lazily, inside the first collective's enqueue, which therefore waits
    // for every rank to arrive: it gets the creation deadline, later enqueues the context's
    uint32_t setup_ms = 0;
    bool connected = false;
};

namespace sdvk {
namespace {

// One CTA: pass 1 forms res and the sums for the mean; pass 2 the spreads; pass 3 the blend.
__global__ void __launch_bounds__(1024) cfg_combine_kernel(const float* __restrict__ cond, const float* __restrict__ uncond,
                                                           float* __restrict__ out, uint64_t n, float cfg, float rescale) {
    __shared__ double red[2][32];
    const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    auto block_sum = [&](double a, double b, double& ra, double& rb) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            a += __shfl_xor_sync(0xffffffffu, a, o);
            b += __shfl_xor_sync(0xffffffffu, b, o);
        }
        if (lane == 0) {
            red[0][warp] = a;
            red[1][warp] = b;
        }
        __syncthreads();
        if (warp == 0) {
            a = lane < (blockDim.x >> 5) ? red[0][lane] : 0.0;
            b = lane < (blockDim.x >> 5) ? red[1][lane] : 0.0;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                a += __shfl_xor_sync(0xffffffffu, a, o);
                b += __shfl_xor_sync(0xffffffffu, b, o);
            }
            if (lane == 0) {
                red[0][0] = a;
                red[1][0] = b;
            }
        }
        __syncthreads();
        ra = red[0][0];
        rb = red[1][0];
        __syncthreads();
    };
    double m = 0.0, u2 = 0.0;
    for (uint64_t k = tid; k < n; k += blockDim.x) {
        // separately rounded, as the host loop computes it (no fused multiply-add)
        const float r = __fadd_rn(uncond[k], __fmul_rn(cfg, __fsub_rn(cond[k], uncond[k])));
        out[k] = r;
        m += r;
        u2 += (double)uncond[k] * uncond[k];
    }
    if (rescale <= 0.0f) return;
    block_sum(m, u2, m, u2);
    m /= (double)n;
    double s2 = 0.0;
    for (uint64_t k = tid; k < n; k += blockDim.x) {
        const double d = out[k] - m;
        s2 += d * d;
    }
    double unused;
    block_sum(s2, 0.0, s2, unused);
    const double su = sqrt(u2 / (double)n);
    const double sg = sqrt(s2 / (double)n) + 1e-6;
    for (uint64_t k = tid; k < n; k += blockDim.x) {
        const float er = (float)((out[k] - m) * (su / sg) + m);
        out[k] = (float)(rescale * er + (1.0 - rescale) * out[k]);
    }
}

// NCCL is opened on first use, not linked: a process that already loaded one (torch does) keeps
// using that copy, and a process without NCCL can still use everything else in the library.
struct NcclApi {
    decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
    decltype(&ncclCommInitRankConfig) CommInitRankConfig = nullptr;
    decltype(&ncclCommGetAsyncError) CommGetAsyncError = nullptr;
    decltype(&ncclCommAbort) CommAbort = nullptr;
    decltype(&ncclCommFinalize) CommFinalize = nullptr;
    decltype(&ncclCommDestroy) CommDestroy = nullptr;
    decltype(&ncclAllGather) AllGather = nullptr;
    decltype(&ncclGetErrorString) GetErrorString = nullptr;
    bool ok = false;
};

const NcclApi& nccl() {
    static const NcclApi api = [] {
        NcclApi a;
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!h) return a;
        a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        a.CommInitRankConfig = reinterpret_cast<decltype(a.CommInitRankConfig)>(dlsym(h, "ncclCommInitRankConfig"));
        a.CommGetAsyncError = reinterpret_cast<decltype(a.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
        a.CommAbort = reinterpret_cast<decltype(a.CommAbort)>(dlsym(h, "ncclCommAbort"));
        a.CommFinalize = reinterpret_cast<decltype(a.CommFinalize)>(dlsym(h, "ncclCommFinalize"));
        a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        a.AllGather = reinterpret_cast<decltype(a.AllGather)>(dlsym(h, "ncclAllGather"));
        a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        a.ok = a.GetUniqueId && a.CommInitRankConfig && a.CommGetAsyncError && a.CommAbort && a.CommFinalize &&
               a.CommDestroy && a.AllGather && a.GetErrorString;
        return a;
    }();
    return api;
}

ncclDataType_t nccl_type(int dt) { return dt == SDVK_F32 ? ncclFloat32 : dt == SDVK_F16 ? ncclFloat16 : ncclBfloat16; }

// Poll the communicator until its pending operation (init or enqueue) is no longer in progress.
int comm_settle(sdvk_comm* c, uint32_t timeout_ms, const LaunchEnv& env, const char* what) {
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        ncclResult_t st = ncclSuccess;
        if (nccl().CommGetAsyncError(c->comm, &st) != ncclSuccess) st = ncclSystemError;
        if (st == ncclSuccess) return SDVK_OK;
        if (st != ncclInProgress) {
            nccl().CommAbort(c->comm);
            c->aborted = true;
            return fail(env, SDVK_E_CUDA, std::string(what) + ": NCCL error " + nccl().GetErrorString(st));
        }
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
            nccl().CommAbort(c->comm);
            c->aborted = true;
            return fail(env, SDVK_E_TIMEOUT, std::string(what) + ": a peer did not answer within the deadline");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace

int cfg_combine(const float* cond, const float* uncond, float* out, uint64_t n, float cfg, float rescale,
                const LaunchEnv& env) {
    if (!cond || !uncond || !out) return fail(env, SDVK_E_ARG, "null pointer");
    if (n == 0) return SDVK_OK;
    cfg_combine_kernel<<<1, 1024, 0, env.stream>>>(cond, uncond, out, n, cfg, rescale);
    return cuda_check(env, cudaGetLastError(), "cfg_combine_kernel launch");
}

int comm_unique_id(void* id) {
    if (!id) return SDVK_E_ARG;
    if (!nccl().ok) return SDVK_E_CUDA;
    ncclUniqueId u;
    if (nccl().GetUniqueId(&u) != ncclSuccess) return SDVK_E_CUDA;
    static_assert(sizeof(u) == SDVK_COMM_ID_BYTES, "NCCL unique id size");
    std::memcpy(id, &u, sizeof(u));
    return SDVK_OK;
}

int comm_create(int nranks, int rank, const void* id, uint32_t timeout_ms, sdvk_comm** out, const LaunchEnv& env) {
    if (!out || !id || nranks < 1 || rank < 0 || rank >= nranks) return fail(env, SDVK_E_ARG, "bad rank layout");
    *out = nullptr;
    if (!nccl().ok) return fail(env, SDVK_E_CUDA, "libnccl.so.2 could not be loaded");
    auto* c = new (std::nothrow) sdvk_comm();
    if (!c) return SDVK_E_OOM;
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // every wait is ours, with a deadline
    ncclResult_t r = nccl().CommInitRankConfig(&c->comm, nranks, u, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        delete c;
        return fail(env, SDVK_E_CUDA, std::string("ncclCommInitRankConfig: ") + nccl().GetErrorString(r));
    }
    c->nranks = nranks;
    c->rank = rank;
    c->setup_ms = timeout_ms;
    if (int rc = comm_settle(c, timeout_ms, env, "communicator setup")) {
        delete c;
        return rc;
    }
    *out = c;
    return SDVK_OK;
}

int comm_destroy(sdvk_comm* c) {
    if (!c) return SDVK_E_ARG;
    if (c->comm && !c->aborted) {
        nccl().CommFinalize(c->comm);
        ncclResult_t st = ncclInProgress;
        const auto t0 = std::chrono::steady_clock::now();
        while (nccl().CommGetAsyncError(c->comm, &st) == ncclSuccess && st == ncclInProgress &&
               std::chrono::steady_clock::now() - t0 < std::chrono::seconds(10))
            std::this_thread::sleep_for(std::chrono::microseconds(50));
        if (st == ncclSuccess) nccl().CommDestroy(c->comm);
        else nccl().CommAbort(c->comm);
    }
    delete c;
    return SDVK_OK;
}

int comm_abort(sdvk_comm* c) {
    if (!c) return SDVK_E_ARG;
    if (c->comm && !c->aborted) nccl().CommAbort(c->comm);
    c->aborted = true;
    return SDVK_OK;
}

int allgather(sdvk_comm* c, const void* send, void* recv, uint64_t count, int dtype, uint32_t timeout_ms,
              const LaunchEnv& env) {
    if (!c || (!send && count) || (!recv && count)) return fail(env, SDVK_E_ARG, "null pointer");
    if (c->aborted) return fail(env, SDVK_E_STATE, "communicator was aborted");
    if (dtype != SDVK_F32 && dtype != SDVK_F16 && dtype != SDVK_BF16) return fail(env, SDVK_E_ARG, "dtype");
    ncclResult_t r = nccl().AllGather(send, recv, count, nccl_type(dtype), c->comm, env.stream);
    if (r != ncclSuccess && r != ncclInProgress)
        return fail(env, SDVK_E_CUDA, std::string("ncclAllGather: ") + nccl().GetErrorString(r));
    const uint32_t deadline = c->connected ? timeout_ms : std::max(timeout_ms, c->setup_ms);
    if (int rc = comm_settle(c, deadline, env, "all-gather enqueue")) return rc;
    c->connected = true;
    return SDVK_OK;
}

int comm_wait(sdvk_comm* c, uint32_t timeout_ms, const LaunchEnv& env) {
    if (!c) return SDVK_E_ARG;
    if (c->aborted) return fail(env, SDVK_E_STATE, "communicator was aborted");
    // the collective runs on the context's stream: wait for it with the communicator's health polled
    const auto t0 = std::chrono::steady_clock::now();
    while (true) {
        const cudaError_t e = cudaStreamQuery(env.stream);
        if (e == cudaSuccess) return SDVK_OK;
        if (e != cudaErrorNotReady) return cuda_check(env, e, "collective wait");
        ncclResult_t st = ncclSuccess;
        if (nccl().CommGetAsyncError(c->comm, &st) == ncclSuccess && st != ncclSuccess && st != ncclInProgress) {
            nccl().CommAbort(c->comm);
            c->aborted = true;
            return fail(env, SDVK_E_CUDA, std::string("collective failed: ") + nccl().GetErrorString(st));
        }
        if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms)) {
            nccl().CommAbort(c->comm);
            c->aborted = true;
            return fail(env, SDVK_E_TIMEOUT, "collective did not complete within the deadline");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

}  // namespace sdvk
