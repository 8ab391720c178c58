// TEST INFRASTRUCTURE ONLY.  Bodies of the stub engine declared in refstub/Modules/GPU/*.hpp.
//
// Buffers are host memory; a "dispatch" runs the oracle's fp32 restatement of the named shader with
// the caller's push constants and buffer bindings (the kernel table's binding orders,
// src/Modules/GPU/vk_engine.cpp:51-125), so reference code compiled against this header -- its test
// harnesses with their own CPU references and pass bars, and its generation program -- runs the
// reference's arithmetic on the host cores.
//
// The two test harnesses time large shapes on zero-filled inputs after their checks; built with
// REFSTUB_SKIP_LARGE_WORK the stub skips GEMM and attention shapes above kMaxStubWork
// multiply-adds so those loops finish in milliseconds (their outputs are never read).  The
// generation program is built without it and computes everything.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "../oracle.h"
#include "Modules/GPU/fused_attn.hpp"
#include "Modules/GPU/gpu_ops.hpp"
#include "Modules/GPU/vk_engine.hpp"

namespace {
#ifdef REFSTUB_SKIP_LARGE_WORK
const double kMaxStubWork = 5e8;
#else
const double kMaxStubWork = 1e300;
#endif
unsigned char* base(const ofc::gpu::BufRef& b) { return (unsigned char*)b.buf + b.offset; }
float* F(const ofc::gpu::BufRef& b) { return (float*)base(b); }

[[noreturn]] void die(const char* kernel, const char* what) {
    std::fprintf(stderr, "stub engine: %s: %s\n", kernel, what);
    std::exit(2);
}

// SDVK_STUB_TRACE=<file>: every uploadNow / downloadNow is appended to the file as one record
// {char op ('U' or 'D'), uint64 bytes, the bytes}: the generation loop's latents, scaled model
// inputs and model outputs in the order the loop moves them, for tests that replay the loop.
FILE* trace_file() {
    static FILE* f = nullptr;
    static bool opened = false;
    if (!opened) {
        opened = true;
        const char* path = std::getenv("SDVK_STUB_TRACE");
        if (path && *path) f = std::fopen(path, "wb");
    }
    return f;
}
void trace(char op, const void* data, uint64_t bytes) {
    FILE* f = trace_file();
    if (!f) return;
    std::fwrite(&op, 1, 1, f);
    std::fwrite(&bytes, 8, 1, f);
    std::fwrite(data, 1, bytes, f);
    std::fflush(f);
}

bool profiling() {
    static int on = -1;
    if (on < 0) {
        const char* e = std::getenv("OFC_KERNEL_PROFILE");
        on = (e && e[0] && e[0] != '0') ? 1 : 0;
    }
    return on == 1;
}
}  // namespace

namespace ofc {
namespace gpu {

GContext G;

// ------------------------------------------------------------------------------------- Arena
void Arena::init(VkDevice, VkPhysicalDevice, uint64_t bytes, bool, bool) {
    destroy();
    // calloc maps large blocks lazily zeroed, so a generous arena costs only the pages it touches
    mem_ = (unsigned char*)std::calloc(bytes ? bytes : 1, 1);
    if (!mem_) throw OomError("stub arena: host allocation of " + std::to_string(bytes) + " B failed");
    cap_ = bytes;
    used_ = 0;
}
BufRef Arena::alloc(uint64_t size) {
    const uint64_t off = (used_ + kAlign - 1) / kAlign * kAlign;
    if (!mem_ || off + size > cap_)
        throw OomError("stub arena out of memory: need " + std::to_string(size) + " B, used " + std::to_string(used_) +
                       " of " + std::to_string(cap_) + " B");
    used_ = off + size;
    return BufRef{mem_, off, size};
}
void Arena::moveDown(uint64_t dst, uint64_t off, uint64_t bytes) {
    if (bytes && dst != off) std::memmove(mem_ + dst, mem_ + off, bytes);
}
void Arena::destroy() {
    std::free(mem_);
    mem_ = nullptr;
    cap_ = used_ = 0;
}

// ------------------------------------------------------------------------------------ Engine
void Engine::init() {
    alive_ = true;
    stagingArena_.init(nullptr, nullptr, 64ull << 20, false, true);
}
void Engine::destroy() {
    stepArena_.destroy();
    scratchArena_.destroy();
    stagingArena_.destroy();
    alive_ = false;
}
void Engine::loadKernels(const std::string&) {}
void Engine::initArenas(uint64_t stepBytes, uint64_t scratchBytes) {
    stepArena_.init(nullptr, nullptr, stepBytes, true, false);
    scratchArena_.init(nullptr, nullptr, scratchBytes, true, false);
}
void Engine::beginStep() {
    stagingArena_.reset();
    stepArena_.reset();
}
void Engine::fill(BufRef dst, uint32_t value) {
    uint32_t* p = (uint32_t*)base(dst);
    for (uint64_t i = 0; i < dst.size / 4; ++i) p[i] = value;
}
void Engine::copyBuf(BufRef dst, BufRef src) { std::memmove(base(dst), base(src), dst.size); }
void Engine::uploadNow(BufRef dst, const void* src, uint64_t bytes) {
    std::memcpy(base(dst), src, bytes);
    trace('U', src, bytes);
}
void Engine::stageUpload(BufRef dst, const void* src, uint64_t bytes) { std::memcpy(base(dst), src, bytes); }
void* Engine::beginUpload(BufRef dst, uint64_t) { return base(dst); }
void Engine::downloadNow(BufRef src, void* dst, uint64_t bytes) {
    std::memcpy(dst, base(src), bytes);
    trace('D', dst, bytes);
}
void Engine::downloadNow(BufRef src, void* dst, uint64_t bytes, uint64_t srcOff) {
    std::memcpy(dst, (unsigned char*)src.buf + srcOff, bytes);
}
std::string Engine::deviceReport() const { return "device: " + deviceName_ + "\n"; }

void Engine::profileDump() {
    if (!profiling() || prof_.empty()) return;
    std::vector<std::pair<std::string, std::pair<double, uint64_t>>> v(prof_.begin(), prof_.end());
    std::sort(v.begin(), v.end(), [](const auto& a, const auto& b) { return a.second.first > b.second.first; });
    double total = 0;
    for (auto& e : v) total += e.second.first;
    std::fprintf(stderr, "--- stub kernel profile (host seconds, %zu kernels, %.2f s) ---\n", v.size(), total);
    for (auto& e : v)
        std::fprintf(stderr, "%-26s calls %7llu  total %9.3f s  %5.1f%%\n", e.first.c_str(),
                     (unsigned long long)e.second.second, e.second.first, 100.0 * e.second.first / total);
}

void Engine::dispatch(const char* kernel, const std::vector<BufRef>& bufs, const void* push, uint32_t, uint32_t,
                      uint32_t gz) {
    const auto t0 = std::chrono::steady_clock::now();
    const std::string k(kernel);
    hist_[k]++;
    const uint32_t* pu = (const uint32_t*)push;
    auto need = [&](size_t n) {
        if (bufs.size() < n) die(kernel, "too few buffers");
    };
    if (k.rfind("gemm_nt_q8", 0) == 0) {
        const orc_pg& p = *(const orc_pg*)push;
        need(4);
        if ((double)p.M * p.N * p.K * gz <= kMaxStubWork) {
            const bool hasBias = bufs.size() > 4;
            orc_gemm_nt_q8_shader(F(bufs[0]), (const int8_t*)base(bufs[1]), F(bufs[3]),
                                  hasBias ? F(bufs[4]) : nullptr, F(bufs[2]), p.M, p.N, p.K, p.mode, p.sA, p.sC,
                                  gz ? gz : 1, p.lda, p.ldc);
        }
    } else if (k.rfind("gemm_nn_q8", 0) == 0) {
        const orc_pg& p = *(const orc_pg*)push;
        need(4);
        if ((double)p.M * p.N * p.K * gz <= kMaxStubWork)
            orc_gemm_nn_q8_shader((const int8_t*)base(bufs[0]), F(bufs[3]), F(bufs[1]), F(bufs[2]), p.M, p.N, p.K,
                                  p.mode, p.sA, p.sB, p.sC, gz ? gz : 1, p.lda, p.ldb, p.ldc);
    } else if (k == "gemm_nt" || k == "gemm_nn") {
        need(3);
        orc_gemm_fp32_shader(k == "gemm_nt", F(bufs[0]), F(bufs[1]), F(bufs[2]), (const orc_pg*)push, gz ? gz : 1);
    } else if (k == "add2") {
        need(3);
        orc_add2_shader(F(bufs[0]), F(bufs[1]), F(bufs[2]), pu[0]);
    } else if (k == "copy_nd") {
        need(2);
        orc_copy_nd_shader(F(bufs[0]), F(bufs[1]), (const orc_pnd*)push);
    } else if (k == "ew2") {
        need(3);
        orc_ew2_shader(F(bufs[0]), F(bufs[1]), F(bufs[2]), (const orc_pew2*)push);
    } else if (k == "unary_fwd") {
        need(2);
        orc_unary_shader(F(bufs[0]), F(bufs[1]), pu[0], pu[1]);
    } else if (k == "bias_add") {
        need(2);
        orc_bias_add_shader(F(bufs[0]), F(bufs[1]), pu[0], pu[1]);
    } else if (k == "upsample2x") {
        need(2);
        orc_upsample2x_shader(F(bufs[0]), F(bufs[1]), pu[0], pu[1], pu[2]);
    } else if (k == "im2col") {
        need(2);
        orc_im2col_shader(F(bufs[0]), F(bufs[1]), pu[0], pu[1], pu[2], pu[3], pu[4]);
    } else if (k == "im2col_s2") {
        need(2);
        orc_im2col_s2_shader(F(bufs[0]), F(bufs[1]), pu[0], pu[1], pu[2], pu[3], pu[4], (int32_t)pu[5]);
    } else if (k == "layernorm_fwd") {
        need(4);
        float eps;
        std::memcpy(&eps, pu + 2, 4);
        orc_layernorm_shader(F(bufs[0]), F(bufs[1]), F(bufs[2]), F(bufs[3]), pu[0], pu[1], eps, pu[3]);
    } else if (k == "groupnorm") {
        need(4);
        float eps;
        std::memcpy(&eps, pu + 3, 4);
        orc_groupnorm_shader(F(bufs[0]), F(bufs[1]), F(bufs[2]), F(bufs[3]), pu[0], pu[1], pu[2], eps, pu[4]);
    } else if (k == "softmax_fwd") {
        need(2);
        orc_softmax_shader(F(bufs[0]), F(bufs[1]), pu[0], pu[1]);
    } else if (k == "causal_mask") {
        need(1);
        orc_causal_mask_shader(F(bufs[0]), pu[0], pu[1], pu[2]);
    } else {
        // the reference engine prints and exits on a kernel it does not know (vk_engine.cpp:1147-1150)
        die(kernel, "no restatement for this kernel");
    }
    if (profiling()) profileNote(kernel, std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
}

void Engine::profileNote(const char* kernel, double seconds) {
    auto& e = prof_[kernel];
    e.first += seconds;
    e.second++;
}

std::vector<std::string> vkListDevices() { return {"0|host stub|0"}; }

// ------------------------------------------------------------------------ gpu_ops set-up
void gInit(const std::string& spvDir) {
    if (G.eng.alive()) gShutdown();
    G.eng.init();
    G.eng.loadKernels(spvDir);
    G.eng.initArenas(G.stepBytes, G.scratchBytes);
    G.paramArena.init(nullptr, nullptr, G.paramBytes, true, false);
    G.scratchArena.init(nullptr, nullptr, G.scratchBytes, true, false);
    G.hp = G.scratchArena.alloc(64 * 4);
}
void gResizeScratch(uint64_t bytes) {
    G.scratchBytes = bytes;
    G.scratchArena.init(nullptr, nullptr, bytes, true, false);
    G.hp = G.scratchArena.alloc(64 * 4);
}
void gShutdown() {
    G.paramArena.destroy();
    G.paramGradArena.destroy();
    G.scratchArena.destroy();
    G.eng.destroy();
}

// --------------------------------------------------------------------- fused attention
bool fusedAttnSupported(uint32_t C, uint32_t heads) {
    if (!C || !heads || C % heads) return false;
    uint32_t hd = C / heads;
    return hd > 0 && hd <= 64;
}

void fusedAttention(Engine& eng, const FusedAttnArgs& a) {
    if ((double)a.Tq * a.Tk * a.C > kMaxStubWork) return;
    const auto t0 = std::chrono::steady_clock::now();
    const char* simple = std::getenv("SDVK_ATTN_SIMPLE");
    int rc = orc_fused_attention(F(a.q), F(a.k), F(a.v), F(a.out), a.Tq, a.Tk, a.C, a.heads, a.causal ? 1u : 0u,
                                 simple && simple[0] == '1');
    if (rc) {
        std::fprintf(stderr, "fusedAttention: unsupported C=%u heads=%u\n", a.C, a.heads);
        std::exit(1);
    }
    if (profiling())
        eng.profileNote(a.Tk >= 256 && a.C / a.heads == 64 ? "fused_attn_tiled" : "fused_attn",
                        std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count());
}

}  // namespace gpu
}  // namespace ofc
