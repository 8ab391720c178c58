// vk_engine.hpp -- CUDA-backed ofc::gpu::Engine for the sdvk hot path, over libsdvk_b200.so.
//
// It replaces src/Modules/GPU/vk_engine.hpp for the callers of the transformer-block hot path: the
// same namespace, class names, member names and argument meanings (BufRef :21-25, Arena :35-73,
// Engine :90-170), so code written against the Vulkan engine -- sdvkgen.cpp's gemm*/attnCore call
// sites and the reference's tests -- compiles against this header unchanged.  The bodies
// (engine.cpp) call only the C ABI of include/sdvk_cuda.h.
//
// What differs, and why:
//   * BufRef::buf is the base device pointer of the owning arena (a VkBuffer there).  VkBuffer,
//     VkDevice and VkPhysicalDevice are opaque pointer aliases; device()/physDevice() return the
//     sdvk context, which Arena::init takes to allocate from.
//   * Kernels are compiled into the library: loadKernels() checks the library is usable and
//     ignores the SPIR-V directory.  dispatch() accepts the hot-path kernel names (gemm_nt_q8*,
//     gemm_nn_q8*, fused_attn*) and the rest of the table the UNet walker and generation loop use
//     (layernorm_fwd, groupnorm, add2, ew2, copy_nd, unary_fwd, bias_add, upsample2x, im2col*,
//     gemm_nt, gemm_nn, softmax_fwd, causal_mask); any other name throws std::runtime_error where
//     the reference prints and exits (vk_engine.cpp:1147-1150).
//   * beginUpload / stageUpload hand out pinned staging slots that stay valid until flushUploads()
//     copies them all (the ring grows by a new pinned chunk instead of flushing under a caller that
//     still holds an earlier slot).
//   * profileDump() (OFC_KERNEL_PROFILE=1): dispatches are then synchronised one by one and their
//     host-measured times aggregated per kernel name.
//   * Work is stream-ordered on the context's CUDA stream, so barrier() has nothing to do; steps
//     map to sdvk_step_begin/end/wait.
//   * Arena::allocGrow cannot move a device allocation under live BufRefs (they hold the base
//     pointer), so it throws OomError like alloc() when the arena is full.
// Errors: OomError for allocation failures (as vk_engine.hpp:30-32), std::runtime_error with the
// back end's message for everything else.
#pragma once

#include <cstdint>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#ifndef VK_NULL_HANDLE
typedef void* VkBuffer;
typedef void* VkDevice;
typedef void* VkPhysicalDevice;
#define VK_NULL_HANDLE nullptr
#endif

struct sdvk_ctx;

namespace ofc {
namespace gpu {

struct BufRef {
    VkBuffer buf = VK_NULL_HANDLE;  // base device (or pinned host) pointer of the arena
    uint64_t offset = 0;
    uint64_t size = 0;
};

constexpr uint64_t kAlign = 256;

struct OomError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

class Arena {
public:
    // dev is Engine::device(); deviceLocal=false or hostVisible=true gives pinned host memory that
    // the device reads over PCIe and mapPtr() exposes.
    void init(VkDevice dev, VkPhysicalDevice phys, uint64_t bytes, bool deviceLocal, bool hostVisible);
    BufRef alloc(uint64_t size);
    BufRef allocGrow(uint64_t size);
    void setGrowable(bool) {}
    void reset() { used_ = 0; }
    void rewind(uint64_t used) { used_ = used; }
    void destroy();
    uint64_t used() const { return used_; }
    uint64_t cap() const { return cap_; }
    VkBuffer buffer() const { return base_; }
    void* mapPtr() const { return host_ ? base_ : nullptr; }

private:
    sdvk_ctx* ctx_ = nullptr;
    void* base_ = nullptr;
    bool host_ = false;
    uint64_t cap_ = 0, used_ = 0;
};

class Engine {
public:
    Engine() = default;
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    void init();
    void setDeviceIndex(int i) { devIndex_ = i; }
    int deviceIndex() const { return devIndex_; }
    void destroy();
    bool alive() const { return ctx_ != nullptr; }

    void loadKernels(const std::string& spvDir);
    void initArenas(uint64_t stepBytes, uint64_t scratchBytes);

    void beginStep();  // resets the step arena and opens a step
    void beginPass();  // opens a step without the reset
    void dispatch(const char* kernel, const std::vector<BufRef>& bufs, const void* push, uint32_t gx, uint32_t gy = 1,
                  uint32_t gz = 1);
    void fill(BufRef dst, uint32_t value);
    void copyBuf(BufRef dst, BufRef src);
    void endStep();
    void waitStep();

    void profileDump();

    void uploadNow(BufRef dst, const void* src, uint64_t bytes);
    void stageUpload(BufRef dst, const void* src, uint64_t bytes);
    void* beginUpload(BufRef dst, uint64_t bytes);
    void endUpload() {}
    void releaseUploadStaging();
    void flushUploads();
    void downloadNow(BufRef src, void* dst, uint64_t bytes);
    void downloadNow(BufRef src, void* dst, uint64_t bytes, uint64_t srcOff);

    void barrier() {}
    // Moves [off, off + bytes) of the step arena down to dst in stream order; the ranges may overlap.
    void compactStepArena(uint64_t dst, uint64_t off, uint64_t bytes);

    Arena& stepArena() { return stepArena_; }
    Arena& scratchArena() { return scratchArena_; }
    VkDevice device() const { return static_cast<VkDevice>(ctx_); }
    VkPhysicalDevice physDevice() const { return static_cast<VkPhysicalDevice>(ctx_); }
    const std::string& deviceName() const { return deviceName_; }
    uint64_t deviceLocalMb() const;
    uint64_t lastStepMs() const { return lastStepMs_; }
    std::string deviceReport() const;

    // The back end context, for callers that use the typed C ABI directly.
    sdvk_ctx* context() const { return ctx_; }
    // Throws the exception the reference would raise for a failed back-end call.
    void check(int status, const char* what) const;

private:
    void* stagingSlot(uint64_t bytes);
    sdvk_ctx* ctx_ = nullptr;
    int devIndex_ = 0;
    std::string deviceName_;
    Arena stepArena_, scratchArena_;
    bool inStep_ = false;
    uint64_t stepStartNs_ = 0, lastStepMs_ = 0;
    struct StagingChunk {  // pinned host memory the upload slots come from
        void* host;
        uint64_t cap, used;
    };
    struct PendingUpload {
        BufRef dst;
        const void* src;
        uint64_t bytes;
    };
    std::vector<StagingChunk> staging_;
    std::vector<PendingUpload> pending_;
    int profile_ = -1;  // OFC_KERNEL_PROFILE, read once
    std::unordered_map<std::string, std::pair<double, uint64_t>> prof_;  // kernel -> (seconds, calls)
};

}  // namespace gpu
}  // namespace ofc
