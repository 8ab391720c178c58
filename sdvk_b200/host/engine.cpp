// engine.cpp -- bodies of the CUDA-backed ofc::gpu::Engine / Arena / fusedAttention declared in
// Modules/GPU/vk_engine.hpp and fused_attn.hpp.  Every call goes through the C ABI of
// include/sdvk_cuda.h (libsdvk_b200.so); nothing here touches CUDA directly.
#include <chrono>
#include <cstring>
#include <string>

#include <algorithm>
#include <cstdio>
#include <cstdlib>

#include "Modules/GPU/fused_attn.hpp"
#include "Modules/GPU/gpu_ops.hpp"
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

// Push-constant sizes of the kernels this back end runs, from the reference's kernel table
// (vk_engine.cpp:51-125): Pg (48 B, sdvkgen.cpp:901-903) for every GEMM, FaPush (36 B,
// fused_attn.cpp:15-26) for attention, and the table's sizes for the rest.  0 = not a kernel this
// back end runs.
uint32_t push_size(const char* kernel) {
    if (!std::strncmp(kernel, "gemm_nt_q8", 10) || !std::strncmp(kernel, "gemm_nn_q8", 10)) return 48;
    if (!std::strcmp(kernel, "gemm_nt") || !std::strcmp(kernel, "gemm_nn")) return 48;
    if (!std::strncmp(kernel, "fused_attn", 10)) return 36;
    static const struct {
        const char* name;
        uint32_t bytes;
    } table[] = {{"layernorm_fwd", 16}, {"groupnorm", 20}, {"add2", 4},        {"ew2", 56},
                 {"copy_nd", 60},       {"unary_fwd", 8},  {"bias_add", 8},    {"upsample2x", 12},
                 {"im2col", 20},        {"im2col_s2", 24}, {"softmax_fwd", 8}, {"causal_mask", 12}};
    for (const auto& e : table)
        if (!std::strcmp(kernel, e.name)) return e.bytes;
    return 0;
}

constexpr uint64_t kStagingChunk = 256ull << 20;

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
    if (profile_ < 0) {
        const char* e = std::getenv("OFC_KERNEL_PROFILE");
        profile_ = (e && e[0] && e[0] != '0') ? 1 : 0;
    }
    const uint64_t t0 = profile_ ? now_ns() : 0;
    if (profile_) check(sdvk_synchronize(ctx_), "Engine::dispatch (profile)");
    const uint64_t t1 = profile_ ? now_ns() : 0;
    check(sdvk_dispatch(ctx_, kernel, b.data(), (uint32_t)b.size(), push, pbytes, gx, gy, gz), kernel);
    if (profile_) {
        check(sdvk_synchronize(ctx_), kernel);
        auto& a = prof_[kernel];
        a.first += (now_ns() - t1) * 1e-9;
        a.second++;
        (void)t0;
    }
}

void Engine::profileDump() {
    if (prof_.empty()) return;
    std::vector<std::pair<std::string, std::pair<double, uint64_t>>> v(prof_.begin(), prof_.end());
    std::sort(v.begin(), v.end(), [](const auto& a, const auto& b) { return a.second.first > b.second.first; });
    double total = 0;
    uint64_t calls = 0;
    for (const auto& e : v) {
        total += e.second.first;
        calls += e.second.second;
    }
    std::fprintf(stderr, "--- kernel profile (%zu kernels, %llu calls, %.1f ms, each dispatch synchronised) ---\n",
                 v.size(), (unsigned long long)calls, total * 1e3);
    for (const auto& e : v) {
        const double ms = e.second.first * 1e3;
        std::fprintf(stderr, "%-30s calls %6llu  total %9.2f ms  avg %7.3f ms  %5.1f%%\n", e.first.c_str(),
                     (unsigned long long)e.second.second, ms, ms / e.second.second, 100.0 * e.second.first / total);
    }
}

void Engine::compactStepArena(uint64_t dst, uint64_t off, uint64_t bytes) {
    if (bytes == 0 || dst == off) return;
    unsigned char* base = static_cast<unsigned char*>(stepArena_.buffer());
    if (dst > off) throw std::runtime_error("Engine::compactStepArena moves blocks down only");
    // Stream-ordered copies of at most (off - dst) bytes each: every piece's destination lies in
    // source bytes that the earlier pieces have already copied.
    const uint64_t gap = off - dst;
    for (uint64_t done = 0; done < bytes;) {
        const uint64_t n = std::min(gap, bytes - done);
        check(sdvk_copy(ctx_, base + dst + done, base + off + done, n), "Engine::compactStepArena");
        done += n;
    }
}

uint64_t Engine::deviceLocalMb() const {
    uint64_t free_b = 0, total_b = 0;
    if (!ctx_ || sdvk_device_memory(ctx_, &free_b, &total_b) != SDVK_OK) return 0;
    return total_b >> 20;
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

void* Engine::stagingSlot(uint64_t bytes) {
    if (staging_.empty() || staging_.back().used + bytes > staging_.back().cap) {
        const uint64_t cap = std::max(kStagingChunk, (bytes + kAlign - 1) / kAlign * kAlign);
        void* p = nullptr;
        if (sdvk_host_alloc(ctx_, cap, &p) != SDVK_OK) raise(ctx_, SDVK_E_OOM, "upload staging");
        staging_.push_back(StagingChunk{p, cap, 0});
    }
    StagingChunk& c = staging_.back();
    void* slot = static_cast<unsigned char*>(c.host) + c.used;
    c.used = (c.used + bytes + kAlign - 1) / kAlign * kAlign;
    return slot;
}

void* Engine::beginUpload(BufRef dst, uint64_t bytes) {
    if (bytes == 0) return nullptr;
    void* slot = stagingSlot(bytes);
    pending_.push_back(PendingUpload{dst, slot, bytes});
    return slot;
}

void Engine::stageUpload(BufRef dst, const void* src, uint64_t bytes) {
    void* slot = beginUpload(dst, bytes);
    if (slot) std::memcpy(slot, src, bytes);
}

void Engine::flushUploads() {
    if (pending_.empty()) return;
    for (const PendingUpload& p : pending_) check(sdvk_upload_async(ctx_, at(p.dst), p.src, p.bytes), "flushUploads");
    check(sdvk_synchronize(ctx_), "flushUploads");
    pending_.clear();
    // keep the first chunk for the next batch, give the overflow chunks back
    while (staging_.size() > 1) {
        sdvk_host_free(ctx_, staging_.back().host);
        staging_.pop_back();
    }
    if (!staging_.empty()) staging_[0].used = 0;
}

void Engine::releaseUploadStaging() {
    if (ctx_) {
        flushUploads();
        for (const StagingChunk& c : staging_) sdvk_host_free(ctx_, c.host);
    }
    staging_.clear();
    pending_.clear();
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

// ------------------------------------------------------------------------------------- gpu_ops
GContext G;

void gInit(const std::string& spvDir) {
    if (G.eng.alive()) gShutdown();
    G.eng.init();
    G.eng.loadKernels(spvDir);
    G.eng.initArenas(G.stepBytes, G.scratchBytes);
    G.paramArena.init(G.eng.device(), G.eng.physDevice(), G.paramBytes, true, false);
    if (G.allocGradArena) G.paramGradArena.init(G.eng.device(), G.eng.physDevice(), G.paramBytes, true, false);
    G.scratchArena.init(G.eng.device(), G.eng.physDevice(), G.scratchBytes, true, false);
    G.hp = G.scratchArena.alloc(64 * 4);
    G.eng.fill(G.hp, 0u);
}

void gResizeScratch(uint64_t bytes) {
    G.scratchBytes = bytes;
    G.scratchArena.init(G.eng.device(), G.eng.physDevice(), bytes, true, false);
    G.hp = G.scratchArena.alloc(64 * 4);
    G.eng.fill(G.hp, 0u);
}

void gShutdown() {
    G.paramArena.destroy();
    G.paramGradArena.destroy();
    G.scratchArena.destroy();
    G.eng.destroy();
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
