// Format-constant tables, one definition per translation unit.
#pragma once
#include <stdint.h>

#include "iq1s_grid.h"

namespace iqk {
namespace {
// IQ1_S grid codes in global memory (statically initialised, read-only);
// kernels that gather from it stage a copy in shared memory first.
__device__ const uint16_t g_iq1s_grid[2048] = {IQK_IQ1S_GRID_CODES};
}  // namespace
}  // namespace iqk
