// no_alloc.cu -- the device scratch array behind sdvk_transformer_block_static.
//
// The array is a file-scope __device__ object of fixed size, so it exists as soon as this module is
// loaded and the entry point needs no allocation of any kind.  It lives in its own translation unit
// (its own module) so that a process that never calls the entry point does not load it under CUDA's
// lazy module loading.  Its address is looked up once per device (with that device current) and
// cached; the lookup is the only runtime call this file makes.
#include <mutex>

#include "backend.hpp"

namespace sdvk {

__device__ __align__(256) uint8_t g_block_scratch[SDVK_STATIC_SCRATCH_BYTES];

int static_scratch(int device, void** ptr, const LaunchEnv& env) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static void* addr[kMaxDevices] = {};
    if (device < 0 || device >= kMaxDevices) return fail(env, SDVK_E_ARG, "device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[device]) {
        void* p = nullptr;
        if (int rc = cuda_check(env, cudaGetSymbolAddress(&p, g_block_scratch), "cudaGetSymbolAddress(scratch)"))
            return rc;
        addr[device] = p;
    }
    *ptr = addr[device];
    return SDVK_OK;
}

}  // namespace sdvk
