// accumulate.h -- internal launchers shared by the accumulate_uz sources.
#pragma once

#include "nsc_common.cuh"

namespace nsc {

// General forward (any geometry).  Output rows [0, Hout); x rows are read
// from a buffer of x_rows rows where output row 0 sits at buffer row x_off;
// wrap != 0 means the buffer is the full image with circular rows.
nsc_status acc_fwd_generic(const void* x, int xd, const void* w, int wd,
                           int64_t Cw, int64_t B, int64_t C, int64_t Hout,
                           int64_t W, int64_t x_rows, int64_t x_off, int wrap,
                           const ShiftTable& st, void* U, void* Z,
                           cudaStream_t stream, int64_t h_begin = 0,
                           int64_t h_end = -1);

// Tiled fast forward.  Returns false (launching nothing) when the geometry
// or dtypes are outside what it handles; the caller then uses the generic
// path.  mode 0: accumulate_uz (U, Z); mode 1 / 2: normalized_accumulate_uz
// with log / positive weights (U <- D, Z <- log_C, `invalid` flag word),
// full images only (wrap != 0).  Only output rows [h_begin, h_end) are
// computed (h_end < 0: all); max_ctas > 0 caps the persistent grid (CTAs
// left free for a concurrent collective).
bool acc_fwd_fast(const void* x, int xd, const void* w, int wd, int64_t Cw,
                  int64_t B, int64_t C, int64_t Hout, int64_t W,
                  int64_t x_rows, int64_t x_off, int wrap,
                  const ShiftTable& st, void* U, void* Z, cudaStream_t stream,
                  int mode = 0, int* invalid = nullptr, int64_t h_begin = 0,
                  int64_t h_end = -1, int max_ctas = 0);

// Tiled grad_w of accumulate_uz (x, w share fp16 / bf16 / fp32 storage,
// grad_U / grad_Z fp32); false (nothing launched) when it declines.
bool acc_gw_fast(const void* x, int xd, int wd, int64_t Cw, int64_t B, int64_t C,
                 int64_t H, int64_t W, const ShiftTable& st, const void* gU,
                 const void* gZ, void* gw, cudaStream_t stream);

// Tiled grad_x of accumulate_uz (same conditions; grad_x fp32); false when
// it declines.
bool acc_gx_fast(const void* w, int xd, int wd, int64_t Cw, int64_t B, int64_t C,
                 int64_t H, int64_t W, const ShiftTable& st, const void* gU, void* gx,
                 cudaStream_t stream);

// Tiled TMA grad_x (accumulate_gx_tma.cuh) followed by its border-band
// wrap kernel: weights fp16 / bf16 / fp32, grad_U and grad_x fp32.  false
// (nothing launched) when it declines.
bool acc_gx_tma(const void* w, int wd, int64_t Cw, int64_t B, int64_t C, int64_t H,
                int64_t W, const ShiftTable& st, const void* gU, void* gx,
                cudaStream_t stream);
nsc_status acc_gx_wrap(const void* w, int wd, int64_t Cw, int64_t B, int64_t C,
                       int64_t H, int64_t W, const ShiftTable& st, const void* gU,
                       void* gx, cudaStream_t stream);

// After a tiled forward (mode 0) of a table with periodic mirror rows: add
// the wrapped mirror terms the tile kernel leaves out (border band only).
nsc_status acc_per_fix(const void* x, int xd, const void* w, int wd, int64_t Cw,
                       int64_t B, int64_t C, int64_t H, int64_t W, const ShiftTable& st,
                       void* U, void* Z, cudaStream_t stream);

// Why the last acc_fwd_fast call on this thread declined ("" if it ran).
const char* fast_decline_reason();

}  // namespace nsc
