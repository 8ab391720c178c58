// no_alloc.cu -- the device scratch array behind sdvk_transformer_block_static.
//
// The array is a file-scope __device__ object of fixed size, so it exists as soon as this module is
// loaded and the entry point needs no allocation of any kind.  It lives in its own translation unit
// (its own module) so that a process that never calls the entry point does not load it under CUDA's
// lazy module loading.  Its address is looked up per device, with that device current, and cached
// together with the identity of the CUDA context it belongs to (cuCtxGetId): after a
// cudaDeviceReset the runtime makes a new primary context, the module is loaded again and the array
// moves, so a call from the new context looks the address up again instead of using the old one.
// The lookups (cudaGetSymbolAddress, cuCtxGetCurrent, cuCtxGetId) are the only calls this file makes.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "backend.hpp"

namespace sdvk {

__device__ __align__(256) uint8_t g_block_scratch[SDVK_STATIC_SCRATCH_BYTES];

namespace {
// the unique id of the context current on this thread (0 when there is none or the driver lacks
// cuCtxGetId).  The driver functions come through the runtime's entry-point query, so the library
// keeps no load-time dependency on libcuda.
unsigned long long current_context_id() {
    static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
    static PFN_cuCtxGetId_v12000 get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
    });
    CUcontext c = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&c) != CUDA_SUCCESS || !c || get_id(c, &id) != CUDA_SUCCESS) return 0;
    return id;
}
}  // namespace

int static_scratch(int device, void** ptr, const LaunchEnv& env) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static void* addr[kMaxDevices] = {};
    static unsigned long long ctx_id[kMaxDevices] = {};
    if (device < 0 || device >= kMaxDevices) return fail(env, SDVK_E_ARG, "device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    const unsigned long long id = current_context_id();
    if (!addr[device] || id == 0 || id != ctx_id[device]) {
        void* p = nullptr;
        if (int rc = cuda_check(env, cudaGetSymbolAddress(&p, g_block_scratch), "cudaGetSymbolAddress(scratch)"))
            return rc;
        addr[device] = p;
        ctx_id[device] = current_context_id();  // the lookup has bound the device's primary context
    }
    *ptr = addr[device];
    return SDVK_OK;
}

}  // namespace sdvk
