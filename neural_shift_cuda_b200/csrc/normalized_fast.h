// normalized_fast.h -- entry of the tiled normalized forward.
#pragma once

#include "nsc_common.cuh"

namespace nsc {

// Runs the tiled forward and returns true, or returns false without
// launching when the call is outside the tiled path's domain (the reason
// is then in norm_fast_decline_reason()).
bool norm_fwd_fast(const void* x, int xd, const void* w, int wd, int64_t Cw,
                   int64_t B, int64_t C, int64_t H, int64_t W, const ShiftTable& st,
                   int logw, void* D, void* L, int* invalid, cudaStream_t stream);
const char* norm_fast_decline_reason();

}  // namespace nsc
