// TEST INFRASTRUCTURE ONLY.  Stand-in for src/Modules/GPU/fused_attn.hpp:13-28 (FusedAttnArgs and
// the operator entry point) so the reference's tests/fused_attn_test.cpp compiles against the
// host-memory stub engine; fusedAttention() runs the oracle restatement (engine_stub.cpp).
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
