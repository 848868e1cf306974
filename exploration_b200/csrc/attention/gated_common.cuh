// Shared definitions of the gated-attention kernels.
#pragma once

#include "../common/util.cuh"

namespace eb {

// Keys per tile of the CUDA-core kernels: a whole number of gate blocks.
EB_HOST_DEVICE int tile_keys(int block) { return block > 32 ? block : 32; }

}  // namespace eb
