// engine_test.cpp -- the reference's operator interface (ofc::gpu::Engine / Arena / BufRef /
// fusedAttention, src/Modules/GPU/vk_engine.hpp, fused_attn.hpp) driven on the B200 through the C++
// mirror in sdvk_b200/host, in the shape of the reference's own harnesses
// (tests/fused_attn_test.cpp, tests/gemm_q8_bench.cpp): upload, beginStep, operator, endStep,
// waitStep, download, compare against an fp64 loop, print PASS/FAIL per case.
//
//   engine_test <golden dir>      exit status 0 iff every case passes
//
// Inputs are the reference harnesses' own: attention draws q, k, v per shape from
// std::mt19937(20261101) with uniform_real_distribution(-1, 1) (fused_attn_test.cpp:74-90); the
// GEMM known-answer case is 100x100x96 from std::mt19937(7), A = int8/127, scale 0.01
// (gemm_q8_bench.cpp:58-81).  The attention truth is the reference's fp64 output committed under
// tests/golden (attn_ref_<i>.f32); the GEMM truth is computed here in double.
// Bars: fp32 attention runs in fp32 at the default precision and meets the reference's own 2e-5;
// the fp32 GEMM runs in tf32 on the tensor cores, so its bar is 5e-3 (max abs / max |ref|).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <random>
#include <string>
#include <vector>

#include "Modules/GPU/fused_attn.hpp"
#include "Modules/GPU/vk_engine.hpp"

namespace {

struct Pg {  // push constants of the Q8 GEMM kernels (sdvkgen.cpp:901-903)
    uint32_t M, N, K, mode, sA, sB, sC, batch, lda, ldb, ldc, pad;
};

struct AttnCase {
    const char* name;
    uint32_t Tq, Tk, C, heads;
    bool causal;
};

int failures = 0;

void report(bool ok, const std::string& name, double maxAbs, double rel) {
    std::printf("%s %-44s maxAbs=%.3g rel=%.3g\n", ok ? "PASS" : "FAIL", name.c_str(), maxAbs, rel);
    if (!ok) ++failures;
}

double rel_err(const std::vector<float>& got, const std::vector<double>& ref, double* maxAbsOut) {
    double maxAbs = 0, maxRef = 0;
    for (size_t i = 0; i < got.size(); ++i) {
        const double d = std::fabs((double)got[i] - ref[i]);
        maxAbs = std::isfinite(d) ? std::max(maxAbs, d) : INFINITY;
        maxRef = std::max(maxRef, std::fabs(ref[i]));
    }
    *maxAbsOut = maxAbs;
    return maxAbs / std::max(1e-9, maxRef);
}

std::vector<double> read_golden(const std::string& path, size_t n) {
    std::vector<float> f(n);
    FILE* fp = std::fopen(path.c_str(), "rb");
    if (!fp || std::fread(f.data(), 4, n, fp) != n) {
        std::printf("FAIL cannot read %s\n", path.c_str());
        ++failures;
    }
    if (fp) std::fclose(fp);
    return std::vector<double>(f.begin(), f.end());
}

void attention_cases(ofc::gpu::Engine& eng, const std::string& golden) {
    const AttnCase cases[] = {
        {"self T=32 C=320 h=5 causal", 32, 32, 320, 5, true},
        {"cross Tq=32 Tk=77 C=1280 h=20", 32, 77, 1280, 20, false},
        {"self T=64 C=320 h=8 causal hd40", 64, 64, 320, 8, true},
        {"cross Tq=48 Tk=96 C=512 h=8", 48, 96, 512, 8, false},
    };
    std::mt19937 rng(20261101);
    std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
    int idx = 0;
    for (const AttnCase& s : cases) {
        std::vector<float> q((size_t)s.Tq * s.C), k((size_t)s.Tk * s.C), v((size_t)s.Tk * s.C);
        for (auto& x : q) x = dist(rng);
        for (auto& x : k) x = dist(rng);
        for (auto& x : v) x = dist(rng);
        const std::vector<double> ref = read_golden(golden + "/attn_ref_" + std::to_string(idx++) + ".f32", q.size());

        ofc::gpu::Arena arena;
        arena.init(eng.device(), eng.physDevice(), (uint64_t)(2 * s.Tq + 2 * s.Tk) * s.C * 4 + (1u << 20), true, false);
        ofc::gpu::FusedAttnArgs a{};
        a.q = arena.alloc((uint64_t)q.size() * 4);
        a.k = arena.alloc((uint64_t)k.size() * 4);
        a.v = arena.alloc((uint64_t)v.size() * 4);
        a.out = arena.alloc((uint64_t)q.size() * 4);
        a.Tq = s.Tq;
        a.Tk = s.Tk;
        a.C = s.C;
        a.heads = s.heads;
        a.causal = s.causal;
        eng.uploadNow(a.q, q.data(), (uint64_t)q.size() * 4);
        eng.uploadNow(a.k, k.data(), (uint64_t)k.size() * 4);
        eng.uploadNow(a.v, v.data(), (uint64_t)v.size() * 4);
        eng.beginStep();
        ofc::gpu::fusedAttention(eng, a);
        eng.endStep();
        eng.waitStep();
        std::vector<float> got(q.size());
        eng.downloadNow(a.out, got.data(), (uint64_t)got.size() * 4);
        double maxAbs;
        const double rel = rel_err(got, ref, &maxAbs);
        report(rel <= 2e-5, std::string("fusedAttention ") + s.name, maxAbs, rel);
        arena.destroy();
    }
}

void gemm_cases(ofc::gpu::Engine& eng) {
    const uint32_t M = 100, N = 100, K = 96;
    std::mt19937 rng(7);
    std::uniform_int_distribution<int> i8(-127, 127);
    std::vector<float> A((size_t)M * K), bias(N);
    std::vector<int8_t> B((size_t)N * K);
    std::vector<float> S((size_t)N * K / 32, 0.01f);
    for (auto& x : A) x = (float)i8(rng) / 127.0f;
    for (auto& x : B) x = (int8_t)i8(rng);
    for (uint32_t n = 0; n < N; ++n) bias[n] = 0.05f * (float)((int)n % 7 - 3);
    std::vector<double> ref((size_t)M * N), refb((size_t)M * N);
    for (uint32_t m = 0; m < M; ++m)
        for (uint32_t n = 0; n < N; ++n) {
            double acc = 0;
            for (uint32_t k = 0; k < K; ++k)
                acc += (double)A[(size_t)m * K + k] * ((double)B[(size_t)n * K + k] * (double)S[((size_t)n * K + k) >> 5]);
            ref[(size_t)m * N + n] = acc;
            refb[(size_t)m * N + n] = acc + bias[n];
        }

    ofc::gpu::Arena arena;
    arena.init(eng.device(), eng.physDevice(), 8u << 20, true, false);
    auto aB = arena.alloc((uint64_t)A.size() * 4);
    auto bB = arena.alloc((uint64_t)B.size());
    auto sB = arena.alloc((uint64_t)S.size() * 4);
    auto cB = arena.alloc((uint64_t)M * N * 4);
    auto biasB = arena.alloc((uint64_t)N * 4);
    eng.uploadNow(aB, A.data(), (uint64_t)A.size() * 4);
    eng.uploadNow(bB, B.data(), (uint64_t)B.size());
    eng.uploadNow(sB, S.data(), (uint64_t)S.size() * 4);
    eng.uploadNow(biasB, bias.data(), (uint64_t)N * 4);

    const char* names[] = {"gemm_nt_q8", "gemm_nt_q8_v", "gemm_nt_q8_v_bm128", "gemm_nt_q8_v_bk32",
                           "gemm_nt_q8_v_bm128_bk32"};
    for (const char* name : names) {
        Pg pc{M, N, K, 0, 0, 0, 0, 1, 0, 0, 0, 0};
        eng.fill(cB, 0xFFFFFFFFu);  // NaN everywhere: the kernel must write every element
        eng.beginStep();
        eng.dispatch(name, {aB, bB, cB, sB}, &pc, (N + 63) / 64, (M + 63) / 64);
        eng.endStep();
        eng.waitStep();
        std::vector<float> got((size_t)M * N);
        eng.downloadNow(cB, got.data(), (uint64_t)got.size() * 4);
        double maxAbs;
        const double rel = rel_err(got, ref, &maxAbs);
        report(rel <= 5e-3, std::string("dispatch ") + name + " 100x100x96", maxAbs, rel);
    }
    {  // bias variant, mode 0
        Pg pc{M, N, K, 0, 0, 0, 0, 1, 0, 0, 0, 0};
        eng.beginStep();
        eng.dispatch("gemm_nt_q8_v_bm128_b", {aB, bB, cB, sB, biasB}, &pc, (N + 63) / 64, (M + 127) / 128);
        eng.endStep();
        eng.waitStep();
        std::vector<float> got((size_t)M * N);
        eng.downloadNow(cB, got.data(), (uint64_t)got.size() * 4);
        double maxAbs;
        const double rel = rel_err(got, refb, &maxAbs);
        report(rel <= 5e-3, "dispatch gemm_nt_q8_v_bm128_b (bias) 100x100x96", maxAbs, rel);
    }
    arena.destroy();
}

template <class Ex, class F>
void expect_throw(const char* what, F&& f) {
    try {
        f();
    } catch (const Ex& e) {
        std::printf("PASS %-44s threw: %s\n", what, e.what());
        return;
    } catch (const std::exception& e) {
        std::printf("FAIL %-44s threw the wrong type: %s\n", what, e.what());
        ++failures;
        return;
    }
    std::printf("FAIL %-44s did not throw\n", what);
    ++failures;
}

void error_cases(ofc::gpu::Engine& eng) {
    ofc::gpu::Arena arena;
    arena.init(eng.device(), eng.physDevice(), 1u << 20, true, false);
    expect_throw<ofc::gpu::OomError>("Arena::alloc beyond capacity", [&] { arena.alloc(2u << 20); });
    auto b = arena.alloc(4096);
    expect_throw<std::runtime_error>("dispatch of a kernel outside the hot path", [&] {
        Pg pc{};
        eng.dispatch("groupnorm_fwd", {b}, &pc, 1);
    });
    expect_throw<std::runtime_error>("fusedAttention with head dim 128", [&] {
        ofc::gpu::FusedAttnArgs a{};
        a.q = a.k = a.v = a.out = b;
        a.Tq = a.Tk = 4;
        a.C = 256;
        a.heads = 2;
        ofc::gpu::fusedAttention(eng, a);
    });
    if (ofc::gpu::fusedAttnSupported(256, 2) || !ofc::gpu::fusedAttnSupported(1280, 20)) {
        std::printf("FAIL fusedAttnSupported\n");
        ++failures;
    } else {
        std::printf("PASS fusedAttnSupported(256,2)=0, (1280,20)=1\n");
    }
    arena.destroy();
}

}  // namespace

int main(int argc, char** argv) {
    std::setvbuf(stdout, nullptr, _IONBF, 0);
    const std::string golden = argc > 1 ? argv[1] : "tests/golden";
    ofc::gpu::Engine eng;
    eng.init();
    eng.loadKernels("unused");
    eng.initArenas(1u << 20, 1u << 20);
    std::printf("device: %s\n", eng.deviceName().c_str());
    attention_cases(eng, golden);
    gemm_cases(eng);
    error_cases(eng);
    eng.destroy();
    std::printf("%s (%d failure%s)\n", failures ? "FAILED" : "ALL PASS", failures, failures == 1 ? "" : "s");
    return failures ? 1 : 0;
}
