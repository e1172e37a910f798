// Instantiations of the tiled TMA grad_x of accumulate_uz for f32 weights
// (one file per type, so the instantiations compile in parallel).
#include "accumulate_gx_tma.cuh"
NSC_GXT_INSTANTIATE(float, 1)
NSC_GXT_INSTANTIATE(float, 3)
