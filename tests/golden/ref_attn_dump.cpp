// Golden-vector generator (run by make_golden.py; not part of the product or of the test run).
//
// Compiles the reference's own attention test, tests/fused_attn_test.cpp, from the reference
// sources (its main() renamed away, its Engine headers satisfied by oracle/refstub), so that its
// fp64 online-softmax reference() (fused_attn_test.cpp:25-61) can be called directly.  For the
// test's four check shapes (:74-79) it regenerates the inputs exactly as the test does
// (std::mt19937(20261101), U(-1,1), q then k then v per shape, :82-89) and writes
// reference()'s output floats to <outdir>/attn_ref_<i>.f32.
#define main reference_fused_attn_test_main
#include "tests/fused_attn_test.cpp"
#undef main

#include <cstdio>
#include <string>

int main(int argc, char** argv) {
    const std::string outdir = argc > 1 ? argv[1] : ".";
    struct S { uint32_t Tq, Tk, C, heads; bool causal; };
    const S shapes[] = {{32, 32, 320, 5, true}, {32, 77, 1280, 20, false}, {64, 64, 320, 8, true}, {48, 96, 512, 8, false}};
    std::mt19937 rng(20261101);
    std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
    int i = 0;
    for (const S& s : shapes) {
        std::vector<float> q((size_t)s.Tq * s.C), k((size_t)s.Tk * s.C), v((size_t)s.Tk * s.C);
        for (auto& x : q) x = dist(rng);
        for (auto& x : k) x = dist(rng);
        for (auto& x : v) x = dist(rng);
        std::vector<float> ref = reference(q, k, v, s.Tq, s.Tk, s.C, s.heads, s.causal);
        std::string path = outdir + "/attn_ref_" + std::to_string(i++) + ".f32";
        FILE* f = std::fopen(path.c_str(), "wb");
        if (!f) return 1;
        std::fwrite(ref.data(), 4, ref.size(), f);
        std::fclose(f);
    }
    return 0;
}
