// Instantiations of the tiled TMA grad_x of accumulate_uz for bf16 weights
// (one file per type, so the instantiations compile in parallel).
#include "accumulate_gx_tma.cuh"
NSC_GXT_INSTANTIATE(__nv_bfloat16, 1)
NSC_GXT_INSTANTIATE(__nv_bfloat16, 3)
