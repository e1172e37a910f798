// nsc_common.cuh -- shared definitions for the sm_100a shift-window kernels.
//
// Geometry conventions (same as the reference op surface):
//   * images are (B, C, H, W) row-major; a weight stack is (S*B, Cw, H, W)
//     shift-major with Cw in {1, C} (Cw == 1 is a channel-broadcast weight,
//     read once per pixel and applied to every channel);
//   * a shift row is (dx, dy, has_inv); dx moves along H, dy along W;
//   * gather: out(h, w) = x((h+dx) mod H, (w+dy) mod W);
//   * the mirror term of a has_inv row at output p reads the same weight
//     plane at p - (dx, dy) and exists only when that pixel is inside the
//     image (it is never periodic).
// All flattened offsets are int64; intra-plane offsets fit int64 too.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include "../../include/nsc_b200.h"

namespace nsc {

constexpr int kMaxShifts = 1024;

// Shift table passed by value as a kernel parameter (8.3 KB, inside the
// 32 KB parameter space of sm_70+ with CUDA >= 12.1).  Reads are uniform
// across a warp, so they are served by the constant cache.
struct ShiftTable {
    int32_t S;
    int32_t R;            // max(|dx|, |dy|) over the table
    int32_t dx[kMaxShifts];
    int32_t dy[kMaxShifts];
    uint32_t inv[kMaxShifts / 32];
    uint32_t per[kMaxShifts / 32];   // mirror term periodic (column value 2)
    uint32_t nofwd[kMaxShifts / 32]; // no forward term (column value 3)
    int32_t any_per;
    int32_t any_tr;                  // some row has column value 3
    __host__ __device__ __forceinline__ bool has_inv(int s) const {
        return (inv[s >> 5] >> (s & 31)) & 1u;
    }
    // Periodic mirror: the mirror term reads the weight and x at
    // (p - d) mod (H, W) with no inside test (an extension of the
    // reference's row encoding: column value 2).
    __host__ __device__ __forceinline__ bool has_per(int s) const {
        return (per[s >> 5] >> (s & 31)) & 1u;
    }
    // Transposed row (column value 3, accumulate_uz only): the row
    // contributes w_s(p - d) x(p - d) read circularly and no forward term --
    // the transpose of the forward-only row (dx, dy, 0) with the same
    // weight plane.
    __host__ __device__ __forceinline__ bool has_fwd(int s) const {
        return !((nofwd[s >> 5] >> (s & 31)) & 1u);
    }
};

// ---- element loads/stores promoted to the accumulator type --------------
template <typename T> struct Acc { using type = float; };
template <> struct Acc<double> { using type = double; };

__device__ __forceinline__ float to_acc(float v) { return v; }
__device__ __forceinline__ double to_acc(double v) { return v; }
__device__ __forceinline__ float to_acc(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_acc(__nv_bfloat16 v) {
    return __bfloat162float(v);
}

template <typename T, typename A>
__device__ __forceinline__ A ldg_acc(const T* p) {
    return static_cast<A>(to_acc(__ldg(p)));
}

template <typename T> __device__ __forceinline__ T from_float(float v);
template <> __device__ __forceinline__ float from_float<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_float<__half>(float v) {
    return __float2half_rn(v);
}
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}

// Single-correction wrap for |d| <= n (validated on the host).
__device__ __forceinline__ int64_t wrap1(int64_t i, int64_t n) {
    return i < 0 ? i + n : (i >= n ? i - n : i);
}
__device__ __forceinline__ bool inb(int64_t i, int64_t n) {
    return i >= 0 && i < n;
}

// Pixel i of the border band of an H x W plane: the R rows at the top and
// at the bottom, then the R columns at the left and right of the rows
// between.  The band holds 2 R W + 2 R (H - 2 R) pixels (H, W > 2 R).
__device__ __forceinline__ void border_pixel(int64_t i, int64_t H, int64_t W, int64_t R,
                                             int64_t& h, int64_t& w) {
    const int64_t strip = R * W;
    if (i < strip) {
        h = i / W;
        w = i - h * W;
        return;
    }
    i -= strip;
    if (i < strip) {
        const int64_t r = i / W;
        h = H - R + r;
        w = i - r * W;
        return;
    }
    i -= strip;
    const int64_t r2 = 2 * R;
    const int64_t r = i / r2;
    const int64_t k = i - r * r2;
    h = R + r;
    w = k < R ? k : W - r2 + k;
}
inline int64_t border_count(int64_t H, int64_t W, int64_t R) {
    return 2 * R * W + 2 * R * (H - 2 * R);
}

// Grid helper: ceil-div clamped to an int grid dimension.
inline unsigned grid_1d(int64_t n, int per_block, int64_t cap = (1LL << 31) - 1) {
    if (n <= 0) return 0;
    int64_t b = 1 + (n - 1) / per_block;
    return static_cast<unsigned>(b < cap ? b : cap);
}

}  // namespace nsc
