// fused_attn.hpp -- the fused-attention operator of src/Modules/GPU/fused_attn.hpp:13-28 on the
// CUDA back end: the same FusedAttnArgs (fp32 token-major Q/K/V/out, head h at columns h*hd..,
// hd = C / heads, scale 1/sqrt(hd)) and the same two functions.  fusedAttention throws
// std::runtime_error for an unsupported shape where the reference prints and exits
// (fused_attn.cpp:41-44).
#pragma once

#include "vk_engine.hpp"

namespace ofc {
namespace gpu {

struct FusedAttnArgs {
    BufRef q;
    BufRef k;
    BufRef v;
    BufRef out;
    uint32_t Tq = 0;
    uint32_t Tk = 0;
    uint32_t C = 0;
    uint32_t heads = 1;
    bool causal = false;
};

bool fusedAttnSupported(uint32_t C, uint32_t heads);
void fusedAttention(Engine& eng, const FusedAttnArgs& a);

}  // namespace gpu
}  // namespace ofc
