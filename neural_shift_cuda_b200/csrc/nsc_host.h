// nsc_host.h -- host-side argument checking shared by the C entry points.
#pragma once

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <string>

#include "nsc_common.cuh"

namespace nsc {

// Thread-local message of the last failed call (nsc_last_error_string).
std::string& last_error();

inline nsc_status fail(nsc_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    last_error() = buf;
    return st;
}

inline nsc_status ok() {
    last_error().clear();
    return NSC_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline nsc_status check_launch(const char* op) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return fail(NSC_ERR_LAUNCH_FAILED, "%s: kernel launch failed: %s", op,
                    cudaGetErrorString(e));
    return ok();
}

inline bool valid_dtype(int dt) { return dt >= NSC_F16 && dt <= NSC_F64; }

inline size_t dtype_size(int dt) {
    return dt == NSC_F64 ? 8 : (dt == NSC_F32 ? 4 : 2);
}

// Validates extents and the shift table and fills `st`.  `cols` is the
// number of int64 values per row (2 or 3).  |dx| <= H and |dy| <= W keep
// the single-correction wrap of the kernels exact.
inline nsc_status build_shifts(const char* op, const int64_t* shifts,
                               int64_t S, int64_t cols, int64_t H, int64_t W,
                               ShiftTable* st) {
    if (S < 1 || S > kMaxShifts)
        return fail(NSC_ERR_S_OUT_OF_RANGE,
                    "%s: tree reduction requires 1 <= S <= 1024 (got S=%lld)", op,
                    (long long)S);
    if (cols != 2 && cols != 3)
        return fail(NSC_ERR_INVALID_ARG, "%s: shifts must have 2 or 3 columns", op);
    if (!shifts) return fail(NSC_ERR_INVALID_ARG, "%s: shifts is NULL", op);
    st->S = static_cast<int32_t>(S);
    st->R = 0;
    for (int i = 0; i < kMaxShifts / 32; ++i) st->inv[i] = st->per[i] = st->nofwd[i] = 0;
    st->any_per = 0;
    st->any_tr = 0;
    for (int64_t s = 0; s < S; ++s) {
        const int64_t dx = shifts[s * cols + 0];
        const int64_t dy = shifts[s * cols + 1];
        const int64_t iv = cols == 3 ? shifts[s * cols + 2] : 0;
        if (dx < -H || dx > H || dy < -W || dy > W)
            return fail(NSC_ERR_INVALID_ARG,
                        "%s: shift row %lld = (%lld, %lld) exceeds the image "
                        "extent (|dx| <= H=%lld, |dy| <= W=%lld required)",
                        op, (long long)s, (long long)dx, (long long)dy,
                        (long long)H, (long long)W);
        st->dx[s] = static_cast<int32_t>(dx);
        st->dy[s] = static_cast<int32_t>(dy);
        if (iv < 0 || iv > 3)
            return fail(NSC_ERR_INVALID_ARG,
                        "%s: shift row %lld has column value %lld (0..3 expected)",
                        op, (long long)s, (long long)iv);
        if (iv) st->inv[s >> 5] |= 1u << (s & 31);
        if (iv >= 2) {
            st->per[s >> 5] |= 1u << (s & 31);
            st->any_per = 1;
        }
        if (iv == 3) {
            st->nofwd[s >> 5] |= 1u << (s & 31);
            st->any_tr = 1;
        }
        const int32_t a = static_cast<int32_t>(dx < 0 ? -dx : dx);
        const int32_t b = static_cast<int32_t>(dy < 0 ? -dy : dy);
        if (a > st->R) st->R = a;
        if (b > st->R) st->R = b;
    }
    return ok();
}

inline nsc_status check_extents(const char* op, int64_t B, int64_t C,
                                int64_t H, int64_t W) {
    if (B < 0 || C < 0 || H < 0 || W < 0)
        return fail(NSC_ERR_INVALID_ARG, "%s: negative extent", op);
    if (H >= (1LL << 31) || W >= (1LL << 31))
        return fail(NSC_ERR_INVALID_ARG, "%s: H and W must be < 2^31", op);
    return ok();
}

// Accumulator dtype for a (x, w) pair, or -1 when the pair is unsupported:
// equal dtypes, or fp32 x with fp16/bf16 w; fp64 only with fp64.
inline int acc_dtype(int xd, int wd) {
    if (!valid_dtype(xd) || !valid_dtype(wd)) return -1;
    if (xd == NSC_F64 || wd == NSC_F64) return (xd == wd) ? NSC_F64 : -1;
    if (xd == wd) return NSC_F32;
    if (xd == NSC_F32) return NSC_F32;
    return -1;
}

}  // namespace nsc
