// TEST INFRASTRUCTURE ONLY.  Stand-in for src/Modules/GPU/gpu_ops.hpp:28-46: the global context the
// generation program reaches the engine through (GContext G with eng, paramArena, scratchArena and
// the arena sizes) and its set-up calls gInit / gResizeScratch / gShutdown.  The training-op library
// behind the rest of that header is not on the generation path and is left out.
#pragma once

#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "vk_engine.hpp"

namespace ofc {
namespace gpu {

struct GContext {
    Engine eng;
    Arena paramArena;
    Arena paramGradArena;
    Arena scratchArena;
    BufRef hp;
    bool stepPreZeroed = false;
    uint64_t paramBytes = 0;
    bool allocGradArena = true;
    uint64_t stepBytes = 2048ull << 20;
    uint64_t scratchBytes = 256ull << 20;
};
extern GContext G;

void gInit(const std::string& spvDir);
void gResizeScratch(uint64_t bytes);
void gShutdown();

}  // namespace gpu
}  // namespace ofc
