// gpu_ops.hpp -- the global context of src/Modules/GPU/gpu_ops.hpp:28-46 on the CUDA back end: GContext G
// (the engine, the parameter and scratch arenas and their sizes) and gInit / gResizeScratch /
// gShutdown (gpu_ops.cpp:181-219), which is all the generation program (sdvkgen.cpp) reaches through
// this header.  The training-op library declared next to them in the reference (tape, GTensor ops,
// optimisers) is not part of the inference path and is not provided.
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
    Arena paramArena;      // persistent weights
    Arena paramGradArena;  // kept for the reference's field list; the inference path leaves it empty
    Arena scratchArena;    // persistent small buffers
    BufRef hp;             // 64 floats of the reference's hyperparameter block, zeroed at init
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
