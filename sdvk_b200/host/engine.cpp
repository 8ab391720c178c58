// engine.cpp -- bodies of the CUDA-backed ofc::gpu::Engine / Arena / fusedAttention declared in
// Modules/GPU/vk_engine.hpp and fused_attn.hpp.  Every call goes through the C ABI of
// include/sdvk_cuda.h (libsdvk_b200.so); nothing here touches CUDA directly.
#include <chrono>
#include <cstring>
#include <string>

#include "Modules/GPU/fused_attn.hpp"
#include "Modules/GPU/vk_engine.hpp"
#include "sdvk_cuda.h"

namespace ofc {
namespace gpu {

namespace {

uint64_t now_ns() {
    return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

[[noreturn]] void raise(sdvk_ctx* ctx, int status, const std::string& what) {
    std::string msg = what + ": " + sdvk_status_string(status);
    const char* detail = ctx ? sdvk_last_error(ctx) : nullptr;
    if (detail && *detail) msg += std::string(" (") + detail + ")";
    if (status == SDVK_E_OOM) throw OomError(msg);
    throw std::runtime_error(msg);
}

inline void* at(const BufRef& b) { return static_cast<unsigned char*>(b.buf) + b.offset; }

// Push-constant sizes of the kernels this back end runs (the reference's kernel table,
// vk_engine.cpp:51-125): Pg (48 B, sdvkgen.cpp:901-903) for the Q8 GEMMs, FaPush (36 B,
// fused_attn.cpp:15-26) for attention, 16 B for layernorm_fwd and 20 B for groupnorm
// (vk_engine.cpp:117,119).  0 = not a kernel this back end runs.
uint32_t push_size(const char* kernel) {
    if (!std::strncmp(kernel, "gemm_nt_q8", 10) || !std::strncmp(kernel, "gemm_nn_q8", 10)) return 48;
    if (!std::strncmp(kernel, "fused_attn", 10)) return 36;
    if (!std::strcmp(kernel, "layernorm_fwd")) return 16;
    if (!std::strcmp(kernel, "groupnorm")) return 20;
    return 0;
}

}  // namespace

// ---------------------------------------------------------------------------------------- Arena
void Arena::init(VkDevice dev, VkPhysicalDevice, uint64_t bytes, bool deviceLocal, bool hostVisible) {
    destroy();
    ctx_ = static_cast<sdvk_ctx*>(dev);
    if (!ctx_) throw std::runtime_error("Arena::init: engine not initialised");
    host_ = hostVisible || !deviceLocal;
    void* p = nullptr;
    const int st = host_ ? sdvk_host_alloc(ctx_, bytes, &p) : sdvk_alloc(ctx_, bytes, &p);
    if (st != SDVK_OK) raise(ctx_, st == SDVK_E_CUDA ? SDVK_E_OOM : st, "Arena::init(" + std::to_string(bytes) + " B)");
    base_ = p;
    cap_ = bytes;
    used_ = 0;
}

BufRef Arena::alloc(uint64_t size) {
    const uint64_t off = (used_ + kAlign - 1) / kAlign * kAlign;
    if (off + size > cap_)
        throw OomError("arena out of memory: need " + std::to_string(size) + " B, used " + std::to_string(used_) +
                       " of " + std::to_string(cap_) + " B");
    used_ = off + size;
    return BufRef{base_, off, size};
}

BufRef Arena::allocGrow(uint64_t size) { return alloc(size); }

void Arena::destroy() {
    if (ctx_ && base_) {
        if (host_) sdvk_host_free(ctx_, base_);
        else sdvk_free(ctx_, base_);
    }
    base_ = nullptr;
    cap_ = used_ = 0;
}

// --------------------------------------------------------------------------------------- Engine
Engine::~Engine() {
    try {
        destroy();
    } catch (...) {
    }
}

void Engine::check(int status, const char* what) const {
    if (status != SDVK_OK) raise(ctx_, status, what);
}

void Engine::init() {
    if (ctx_) return;
    sdvk_ctx* c = nullptr;
    const int st = sdvk_ctx_create(devIndex_, &c);
    if (st != SDVK_OK) raise(nullptr, st, "Engine::init(device " + std::to_string(devIndex_) + ")");
    ctx_ = c;
    char buf[512] = {0};
    if (sdvk_device_report(ctx_, buf, sizeof buf) == SDVK_OK) {
        deviceName_ = buf;
        const size_t nl = deviceName_.find('\n');
        if (nl != std::string::npos) deviceName_.resize(nl);
    }
}

void Engine::destroy() {
    if (!ctx_) return;
    releaseUploadStaging();
    stepArena_.destroy();
    scratchArena_.destroy();
    sdvk_ctx_destroy(ctx_);
    ctx_ = nullptr;
}

void Engine::loadKernels(const std::string&) {
    if (!ctx_) throw std::runtime_error("Engine::loadKernels before init");
}

void Engine::initArenas(uint64_t stepBytes, uint64_t scratchBytes) {
    stepArena_.init(device(), physDevice(), stepBytes, true, false);
    scratchArena_.init(device(), physDevice(), scratchBytes, true, false);
}

void Engine::beginStep() {
    stepArena_.reset();
    beginPass();
}

void Engine::beginPass() {
    check(sdvk_step_begin(ctx_), "Engine::beginStep");
    inStep_ = true;
    stepStartNs_ = now_ns();
}

void Engine::dispatch(const char* kernel, const std::vector<BufRef>& bufs, const void* push, uint32_t gx, uint32_t gy,
                      uint32_t gz) {
    const uint32_t pbytes = push_size(kernel);
    if (!pbytes) throw std::runtime_error(std::string("Engine::dispatch: kernel not in this back end: ") + kernel);
    std::vector<sdvk_buf> b(bufs.size());
    for (size_t i = 0; i < bufs.size(); ++i) b[i] = sdvk_buf{bufs[i].buf, bufs[i].offset, bufs[i].size};
    check(sdvk_dispatch(ctx_, kernel, b.data(), (uint32_t)b.size(), push, pbytes, gx, gy, gz), kernel);
}

void Engine::fill(BufRef dst, uint32_t value) { check(sdvk_fill_u32(ctx_, at(dst), value, dst.size), "Engine::fill"); }

void Engine::copyBuf(BufRef dst, BufRef src) {
    check(sdvk_copy(ctx_, at(dst), at(src), src.size < dst.size ? src.size : dst.size), "Engine::copyBuf");
}

void Engine::endStep() {
    check(sdvk_step_end(ctx_), "Engine::endStep");
    inStep_ = false;
}

void Engine::waitStep() {
    check(sdvk_step_wait(ctx_, 0), "Engine::waitStep");
    lastStepMs_ = (now_ns() - stepStartNs_) / 1000000ull;
}

void Engine::uploadNow(BufRef dst, const void* src, uint64_t bytes) {
    check(sdvk_upload(ctx_, at(dst), src, bytes), "Engine::uploadNow");
}

void* Engine::beginUpload(BufRef dst, uint64_t bytes) {
    if (bytes > upCap_) {
        releaseUploadStaging();
        void* p = nullptr;
        const int st = sdvk_host_alloc(ctx_, bytes, &p);
        if (st != SDVK_OK) raise(ctx_, SDVK_E_OOM, "Engine::beginUpload");
        upHost_ = p;
        upCap_ = bytes;
    }
    upDst_ = dst;
    upBytes_ = bytes;
    return upHost_;
}

void Engine::endUpload() {
    if (upBytes_) uploadNow(upDst_, upHost_, upBytes_);
    upBytes_ = 0;
}

void Engine::releaseUploadStaging() {
    if (upHost_ && ctx_) sdvk_host_free(ctx_, upHost_);
    upHost_ = nullptr;
    upCap_ = upBytes_ = 0;
}

void Engine::downloadNow(BufRef src, void* dst, uint64_t bytes) {
    check(sdvk_download(ctx_, dst, at(src), bytes), "Engine::downloadNow");
}

void Engine::downloadNow(BufRef src, void* dst, uint64_t bytes, uint64_t srcOff) {
    check(sdvk_download(ctx_, dst, static_cast<unsigned char*>(src.buf) + srcOff, bytes), "Engine::downloadNow");
}

std::string Engine::deviceReport() const {
    char buf[2048] = {0};
    check(sdvk_device_report(ctx_, buf, sizeof buf), "Engine::deviceReport");
    return buf;
}

// -------------------------------------------------------------------------------- fused attention
bool fusedAttnSupported(uint32_t C, uint32_t heads) { return sdvk_fused_attn_supported(C, heads) != 0; }

void fusedAttention(Engine& eng, const FusedAttnArgs& a) {
    if (!fusedAttnSupported(a.C, a.heads))
        throw std::runtime_error("fusedAttention: unsupported C=" + std::to_string(a.C) +
                                 " heads=" + std::to_string(a.heads));
    eng.check(sdvk_fused_attention(eng.context(), at(a.q), at(a.k), at(a.v), at(a.out), a.Tq, a.Tk, a.C, a.heads,
                                   a.causal ? 1 : 0),
              "fusedAttention");
}

}  // namespace gpu
}  // namespace ofc
