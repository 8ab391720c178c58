// TEST INFRASTRUCTURE ONLY.  Host-memory stand-in for the reference's Vulkan engine header, used to
// compile the reference's own test harnesses (tests/fused_attn_test.cpp, tests/gemm_q8_bench.cpp)
// from their sources with the CPU oracle restatement playing the device.  It declares only the
// members those two harnesses call, with the call shapes of src/Modules/GPU/vk_engine.hpp:21-25
// (BufRef), :35-73 (Arena) and :90-170 (Engine); the bodies are in engine_stub.cpp.
#pragma once

#include <cstdint>
#include <string>
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

class Arena {
public:
    void init(VkDevice dev, VkPhysicalDevice phys, uint64_t bytes, bool deviceLocal, bool hostVisible);
    BufRef alloc(uint64_t size);
    void destroy();

private:
    std::vector<unsigned char> mem_;
    uint64_t used_ = 0;
};

class Engine {
public:
    void init();
    void loadKernels(const std::string& spvDir);
    void initArenas(uint64_t stepBytes, uint64_t scratchBytes);
    void beginStep();
    void dispatch(const char* kernel, const std::vector<BufRef>& bufs, const void* push, uint32_t gx,
                  uint32_t gy = 1, uint32_t gz = 1);
    void endStep();
    void waitStep();
    void uploadNow(BufRef dst, const void* src, uint64_t bytes);
    void downloadNow(BufRef src, void* dst, uint64_t bytes);
    void destroy();
    VkDevice device() const { return VK_NULL_HANDLE; }
    VkPhysicalDevice physDevice() const { return VK_NULL_HANDLE; }
};

}  // namespace gpu
}  // namespace ofc
