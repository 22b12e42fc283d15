// qw6_grids.cuh -- IQ codebooks in device global memory (one copy per
// translation unit; 12 KB).  Kernels stage them into shared memory.
#pragma once

#include "qw6_iq_grids.h"

namespace qw6 {

static __device__ __align__(16) const uint8_t d_grid_iq2xxs[2048] = QW6_IQ2XXS_GRID_BYTES_INIT;
static __device__ __align__(16) const uint8_t d_grid_iq2s[8192] = QW6_IQ2S_GRID_BYTES_INIT;
static __device__ __align__(16) const uint8_t d_grid_iq3s[2048] = QW6_IQ3S_GRID_BYTES_INIT;

template <int F>
__device__ __forceinline__ const uint8_t* grid_ptr() {
    if constexpr (F == QW6F_IQ2_XXS) return d_grid_iq2xxs;
    else if constexpr (F == QW6F_IQ2_S) return d_grid_iq2s;
    else return d_grid_iq3s;
}

}  // namespace qw6
