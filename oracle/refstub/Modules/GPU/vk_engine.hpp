// TEST INFRASTRUCTURE ONLY.  Host-memory stand-in for the reference's Vulkan engine header, used to
// compile reference sources unchanged (tests/fused_attn_test.cpp, tests/gemm_q8_bench.cpp, and the
// generation program src/Modules/Diffusion/main.cpp + sdvkgen.cpp) with the CPU restatement of the
// reference's shaders playing the device.  It declares the members those sources call, with the
// call shapes of src/Modules/GPU/vk_engine.hpp:21-25 (BufRef), :27-32 (kAlign, OomError), :35-73
// (Arena) and :90-247 (Engine); the bodies are in engine_stub.cpp.
//
// Buffers are host memory: BufRef::buf is the base pointer of the owning arena.  A dispatch runs the
// named kernel's restatement at once, so steps, barriers and replay have nothing to order.
#pragma once

#include <cstdint>
#include <functional>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

typedef void* VkBuffer;
typedef void* VkDevice;
typedef void* VkPhysicalDevice;
#define VK_NULL_HANDLE nullptr

namespace ofc {
namespace gpu {

struct BufRef {
    VkBuffer buf = VK_NULL_HANDLE;  // host base pointer of the owning arena
    uint64_t offset = 0;
    uint64_t size = 0;
};

constexpr uint64_t kAlign = 256;

struct OomError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

class Arena {
public:
    ~Arena() { destroy(); }
    void init(VkDevice dev, VkPhysicalDevice phys, uint64_t bytes, bool deviceLocal, bool hostVisible);
    BufRef alloc(uint64_t size);
    BufRef allocGrow(uint64_t size) { return alloc(size); }
    void setGrowable(bool) {}
    void reset() { used_ = 0; }
    void rewind(uint64_t used) { used_ = used; }
    void moveDown(uint64_t dst, uint64_t off, uint64_t bytes);
    void destroy();
    uint64_t used() const { return used_; }
    uint64_t cap() const { return cap_; }
    VkBuffer buffer() const { return mem_; }
    void* mapPtr() const { return mem_; }

private:
    unsigned char* mem_ = nullptr;
    uint64_t cap_ = 0, used_ = 0;
};

class Engine {
public:
    Engine() = default;
    ~Engine() = default;
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    void init();
    void setDeviceIndex(int i) { devIndex_ = i; }
    int deviceIndex() const { return devIndex_; }
    void destroy();
    bool alive() const { return alive_; }

    void loadKernels(const std::string& spvDir);
    void initArenas(uint64_t stepBytes, uint64_t scratchBytes);

    void beginStep();
    void beginPass() {}
    void dispatch(const char* kernel, const std::vector<BufRef>& bufs, const void* push, uint32_t gx, uint32_t gy = 1,
                  uint32_t gz = 1);
    void fill(BufRef dst, uint32_t value);
    void copyBuf(BufRef dst, BufRef src);
    void endStep() {}
    void waitStep() {}

    void enableStepReplay(bool) {}
    void invalidateReplay() {}
    bool replayActive() const { return false; }
    uint64_t lastCmdCount() const { return 0; }
    const std::unordered_map<std::string, uint64_t>& cmdHist() const { return hist_; }

    void mark(const char*) {}
    bool phaseTimes(std::vector<std::pair<std::string, double>>& out) const {
        out.clear();
        return false;
    }
    // OFC_KERNEL_PROFILE=1: host time of every restated kernel, aggregated by name.
    void profileDump();
    void profileNote(const char* kernel, double seconds);

    void uploadNow(BufRef dst, const void* src, uint64_t bytes);
    void stageUpload(BufRef dst, const void* src, uint64_t bytes);  // weight loading: not traced
    void* beginUpload(BufRef dst, uint64_t bytes);
    void endUpload() {}
    void releaseUploadStaging() {}
    void flushUploads() {}
    void downloadNow(BufRef src, void* dst, uint64_t bytes);
    void downloadNow(BufRef src, void* dst, uint64_t bytes, uint64_t srcOff);

    BufRef stagingUpload(uint64_t bytes) { return stagingArena_.alloc(bytes); }
    BufRef stagingReadback(uint64_t bytes) { return stagingArena_.alloc(bytes); }

    void barrier() {}
    void compactStepArena(uint64_t dst, uint64_t off, uint64_t bytes) { stepArena_.moveDown(dst, off, bytes); }

    Arena& stepArena() { return stepArena_; }
    Arena& scratchArena() { return scratchArena_; }
    Arena& stagingArena() { return stagingArena_; }
    VkDevice device() const { return VK_NULL_HANDLE; }
    VkPhysicalDevice physDevice() const { return VK_NULL_HANDLE; }
    const std::string& deviceName() const { return deviceName_; }
    uint64_t deviceLocalMb() const { return 0; }
    uint64_t lastStepMs() const { return 0; }
    std::string deviceReport() const;

private:
    bool alive_ = false;
    int devIndex_ = 0;
    std::string deviceName_ = "host stub (CPU restatement of the shaders)";
    std::unordered_map<std::string, uint64_t> hist_;
    std::unordered_map<std::string, std::pair<double, uint64_t>> prof_;  // name -> (seconds, calls)
    Arena stepArena_, scratchArena_, stagingArena_;
};

std::vector<std::string> vkListDevices();

}  // namespace gpu
}  // namespace ofc
