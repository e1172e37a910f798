// Instantiations of the tiled TMA grad_x of accumulate_uz for f16 weights
// (one file per type, so the instantiations compile in parallel).
#include "accumulate_gx_tma.cuh"
NSC_GXT_INSTANTIATE(__half, 1)
NSC_GXT_INSTANTIATE(__half, 3)
