// TEST INFRASTRUCTURE ONLY.  C entry points over the reference's own GGUF reader
// (src/Modules/Model/Gguf.cpp, compiled unchanged from the reference sources by oracle/Makefile
// into oracle/_ref/libref_gguf.so).  Tests use it to pin the oracle's Q8_0 codec: a file written by
// orc_gguf_write_q8() must decode to the same int8 payload and fp32 scales through
// GgufFile::readQ8Into (Gguf.cpp:559-583) and to the same floats through readFloat (:514-523).
#include <cstdint>
#include <cstring>
#include <string>

#include "Modules/Model/Gguf.hpp"

extern "C" {

int ref_gguf_shape(const char* path, const char* name, uint64_t* rows, uint64_t* cols, uint32_t* type) {
    ofc::GgufFile f;
    std::string err;
    if (!f.open(path, &err)) return 1;
    const ofc::GgufTensor* t = f.find(name);
    if (!t) return 2;
    auto sh = t->shape();
    *rows = sh.first;
    *cols = sh.second;
    *type = (uint32_t)t->type;
    return 0;
}

int ref_gguf_read_q8(const char* path, const char* name, int8_t* q, float* scales) {
    ofc::GgufFile f;
    std::string err;
    if (!f.open(path, &err)) return 1;
    return f.readQ8Into(name, q, scales, &err) ? 0 : 3;
}

int ref_gguf_read_float(const char* path, const char* name, float* out, uint64_t n) {
    ofc::GgufFile f;
    std::string err;
    if (!f.open(path, &err)) return 1;
    std::vector<float> v = f.readFloat(name, &err);
    if (v.size() != n) return 3;
    std::memcpy(out, v.data(), n * sizeof(float));
    return 0;
}

}  // extern "C"
