// TEST INFRASTRUCTURE ONLY.  Bodies of the stub engine declared in refstub/Modules/GPU/*.hpp.
//
// Buffers are host memory; a "dispatch" runs the oracle's fp32 restatement of the named shader
// with the harness's push constants, so the reference's own test code (its CPU references, its
// tolerance checks and its PASS/FAIL lines) judges the restatement.  The harnesses' latency loops
// run large shapes on zero-filled inputs purely for timing; the stub skips shapes above
// kMaxStubWork multiply-adds so those loops finish in milliseconds (their outputs are not checked).
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "../oracle.h"
#include "Modules/GPU/fused_attn.hpp"
#include "Modules/GPU/vk_engine.hpp"

namespace {
const double kMaxStubWork = 5e8;
struct Pg {  // push layout of the Q8 GEMM shaders (sdvkgen.cpp:901-903)
    uint32_t M, N, K, mode, sA, sB, sC, batch, lda, ldb, ldc, pad;
};
unsigned char* base(const ofc::gpu::BufRef& b) { return (unsigned char*)b.buf + b.offset; }
}  // namespace

namespace ofc {
namespace gpu {

void Arena::init(VkDevice, VkPhysicalDevice, uint64_t bytes, bool, bool) {
    mem_.assign(bytes, 0);
    used_ = 0;
}
BufRef Arena::alloc(uint64_t size) {
    uint64_t off = (used_ + 255) / 256 * 256;
    if (off + size > mem_.size()) {
        std::fprintf(stderr, "stub arena exhausted\n");
        std::exit(2);
    }
    used_ = off + size;
    return BufRef{mem_.data(), off, size};
}
void Arena::destroy() {
    mem_.clear();
    mem_.shrink_to_fit();
}

void Engine::init() {}
void Engine::loadKernels(const std::string&) {}
void Engine::initArenas(uint64_t, uint64_t) {}
void Engine::beginStep() {}
void Engine::endStep() {}
void Engine::waitStep() {}
void Engine::destroy() {}
void Engine::uploadNow(BufRef dst, const void* src, uint64_t bytes) { std::memcpy(base(dst), src, bytes); }
void Engine::downloadNow(BufRef src, void* dst, uint64_t bytes) { std::memcpy(dst, base(src), bytes); }

void Engine::dispatch(const char* kernel, const std::vector<BufRef>& bufs, const void* push, uint32_t,
                      uint32_t, uint32_t) {
    const Pg& p = *(const Pg*)push;
    if (std::strncmp(kernel, "gemm_nt_q8", 10) == 0) {
        if ((double)p.M * p.N * p.K * p.batch > kMaxStubWork) return;
        const bool hasBias = bufs.size() > 4;
        orc_gemm_nt_q8_shader((const float*)base(bufs[0]), (const int8_t*)base(bufs[1]),
                              (const float*)base(bufs[3]), hasBias ? (const float*)base(bufs[4]) : nullptr,
                              (float*)base(bufs[2]), p.M, p.N, p.K, p.mode, p.sA, p.sC,
                              p.batch ? p.batch : 1, p.lda, p.ldc);
        return;
    }
    if (std::strncmp(kernel, "gemm_nn_q8", 10) == 0) {
        if ((double)p.M * p.N * p.K * p.batch > kMaxStubWork) return;
        orc_gemm_nn_q8_shader((const int8_t*)base(bufs[0]), (const float*)base(bufs[3]),
                              (const float*)base(bufs[1]), (float*)base(bufs[2]), p.M, p.N, p.K, p.mode,
                              p.sA, p.sB, p.sC, p.batch ? p.batch : 1, p.lda, p.ldb, p.ldc);
        return;
    }
    std::fprintf(stderr, "stub engine: no restatement for kernel %s\n", kernel);
    std::exit(2);
}

bool fusedAttnSupported(uint32_t C, uint32_t heads) {
    if (!C || !heads || C % heads) return false;
    uint32_t hd = C / heads;
    return hd > 0 && hd <= 64;
}

void fusedAttention(Engine&, const FusedAttnArgs& a) {
    if ((double)a.Tq * a.Tk * a.C > kMaxStubWork) return;
    const char* simple = std::getenv("SDVK_ATTN_SIMPLE");
    int rc = orc_fused_attention((const float*)base(a.q), (const float*)base(a.k), (const float*)base(a.v),
                                 (float*)base(a.out), a.Tq, a.Tk, a.C, a.heads, a.causal ? 1u : 0u,
                                 simple && simple[0] == '1');
    if (rc) {
        std::fprintf(stderr, "fusedAttention: unsupported C=%u heads=%u\n", a.C, a.heads);
        std::exit(1);
    }
}

}  // namespace gpu
}  // namespace ofc
