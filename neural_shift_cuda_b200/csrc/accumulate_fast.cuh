// accumulate_fast.cuh -- tiled TMA forward of accumulate_uz for sm_100a.
//
// Persistent kernel, one CTA per SM, 15 consumer warps + 1 producer warp.
// A tile is TH = 30 output rows x TW = 16*V columns (V = 16 bytes of the
// storage type: 8 fp16/bf16 or 4 fp32 pixels per thread, one row per
// thread) of one image and one weight channel (all NC image channels when
// the weight is channel-broadcast).
//
// Weights.  For every shift row s the producer TMA-loads ONE box of the
// weight plane s that covers both uses of it: the forward term reads
// w_s(p) on the tile, the mirror term reads w_s(p - d_s) on the tile
// shifted by -d_s.  The box is (TH + Rx) x (TW + slack) starting at
// (h0 - max(dx, 0), w0 - align_up(max(dy, 0))), so both reads hit shared
// memory and each weight byte leaves HBM once (the overlap with the
// neighbouring tiles is served by L2).  Out-of-image box parts are filled
// with zeros by TMA, which is exactly the mirror term's mask.  Up to four
// consecutive planes with the same box origin (dy 1..4, 5..8, ... of a
// canonical table) travel in one 4-D copy, so a full/empty mbarrier
// handshake covers four shifts; the copies stream through an NSTAGE-deep
// ring.
//
// Image.  Per tile the consumers stage a halo tile of x with circular
// rows/columns in shared memory (cp.async; one buffer, refilled at the tile
// boundary, which leaves room for a deeper weight ring).  Shifts are visited grouped
// by dx; for one dx every thread loads register windows of its forward row
// (h + dx) and mirror row (h - dx) once and serves every dy of the group with
// compile-time register indices (dy is a template-unrolled loop); on tiles
// touching the border the mirror window is zeroed outside the image in
// registers (the mirror term is never periodic).  So the
// per-shift work is one 16-byte weight load (two for the mirror) plus
// the FMAs.  fp16 / bf16 products use the mixed-precision
// fma.rn.f32.{f16,bf16} (exact products, fp32 accumulation) on the packed
// halves directly; no per-element conversion is issued.
//
// Summation order: per output, shifts in (dx, dy) order, forward before
// mirror, fp32 accumulation -- within the fp32 tolerance of the
// reference's pairwise tree (ops.py:77-92).
//
// MODE selects what is accumulated per output pixel (same tiles, copies and
// windows):
//   0  accumulate_uz: U = sum w x, Z = sum w;
//   1  normalized_accumulate_uz, log weights (logits k): D = sum a x / sum a,
//      log_C = log sum e^k, a = 2^(k log2(e) - m) with a lazy running
//      reference m (moved only when a key would give a > 2^16, the partial
//      sums rescaled by 2^(m_old - m_new)), the online normalisation of
//      Milakov & Gimelshein (2018);
//   2  normalized_accumulate_uz, positive weights: a = k 2^-e with a lazy
//      power-of-two scale, rescaled the same way (exact scaling).
// In modes 1 and 2 a mirror key outside the image contributes nothing: the
// TMA zero fill is already "no weight" for positive keys; log keys are
// masked to -inf on border tiles from the same inside test that zeroes the
// mirror x window.  A NaN / +inf key (negative positive-mode key) poisons
// the pixel: D and log_C NaN and the invalid flag set; a pixel without a
// live key gives D = 0, log_C = -inf (reference shift_ops_cuda.cu:528-653).
#pragma once

// Up to this many consecutive weight planes (same dx, consecutive plane
// index, same box origin) travel in one TMA copy.
#ifndef NSC_FAST_GROUP
#define NSC_FAST_GROUP 4
#endif

#include "nsc_common.cuh"
#include "nsc_tma.cuh"

namespace nsc {
namespace fast {

// 15 consumer warps + 1 producer warp = 16 warps: four per register-file
// sub-partition, so every thread may hold up to 128 registers.
constexpr int TH = 30;          // output rows per tile
constexpr int TPR = 16;         // threads per row
constexpr int NCONS = TH * TPR; // consumer threads
constexpr int NTHREADS = NCONS + 32;
constexpr int MAXSTAGE = 16;     // ring depth is chosen per launch (<= this)
#ifndef NSC_FAST_STRIP
#define NSC_FAST_STRIP 8
#endif
constexpr int STRIP = NSC_FAST_STRIP;   // tile columns per raster strip
constexpr int MAXR = 16;        // |dx|, |dy| <= MAXR on this path
constexpr int kInvBit = 0x800;       // row has a mirror term
constexpr int kLenShift = 12;        // bits 12-14: planes in the copy this entry
                                     // starts (1..4), 0 for a later member
constexpr int kSMask = 0x7FF;
constexpr int kGroup = NSC_FAST_GROUP;
static_assert(kGroup >= 1 && kGroup <= 4, "copies carry 1 to 4 planes");

// Box-depth 1..4 tensor maps of the weight stack.
struct WMaps {
    CUtensorMap m[4];
};

struct FastTable {
    int16_t s[2 * MAXR + 1][2 * MAXR + 1];  // [dx+MAXR][dy+MAXR] -> s | flags, or -1
    // per dx row, bit (dy + MAXR): entry present / has a mirror term /
    // position of its plane in its copy (two bits) / last plane of its copy
    uint64_t present[2 * MAXR + 1], inv[2 * MAXR + 1];
    uint64_t pos0[2 * MAXR + 1], pos1[2 * MAXR + 1], last[2 * MAXR + 1];
    uint8_t row_any[2 * MAXR + 1];
    uint8_t row_inv[2 * MAXR + 1];
    int32_t Rx;                             // max |dx|
    int32_t Rdy;                            // max dy (canonical half-plane tables)
};

struct Geo {
    int64_t B, C, H, W, Cw;     // H: output (= weight) rows
    int64_t x_rows, x_off;      // x buffer rows; buffer row of output row 0
    int32_t wrap;               // 1: x buffer is the full image, circular rows
    int32_t tiles_x, tiles_y;
    int64_t groups, ntiles;
    int32_t BH, BW;             // weight box
    uint32_t stage_tx, stage_stride;
    int32_t XH, XW;             // x halo tile
    int32_t col_border;         // W is not a multiple of the tile width
    int32_t nstage;             // weight ring depth
    uint32_t plane_bytes;       // one plane of a weight box in shared memory
};

// Tile order: planes (image, weight channel) outermost, then vertical
// strips STRIP tiles wide, row-major inside a strip.  Consecutive tiles --
// the ones the persistent CTAs work on at the same time -- form a compact
// block, so the weight rows one tile's box shares with its upper, lower and
// left neighbours are fetched by concurrently running CTAs and meet in L2.
// Launch settings kept out of Geo (a separate kernel parameter).
struct GeoExt {
    int32_t hb0, hb1;           // output rows computed: [hb0, hb1) of [0, H)
    int32_t max_ctas;           // grid cap (0: one CTA per SM)
    uint32_t wait_budget;       // hinted sleeps (~1 ms each) before a wait gives up
    int32_t skip_copy;          // test hook: this copy index is never issued (-1: none)
};

struct TileId {
    int64_t b, grp;
    int h0, w0;
};

__device__ __forceinline__ TileId decode_tile(int64_t tile, const Geo& g, int hb0, int TW,
                                              int64_t cgroups) {
    const int64_t per = static_cast<int64_t>(g.tiles_x) * g.tiles_y;
    const int64_t grp = tile / per;
    const int64_t t = tile - grp * per;
    const int64_t full = static_cast<int64_t>(STRIP) * g.tiles_y;
    const int64_t strip = t / full;
    const int64_t r = t - strip * full;
    const int64_t left = g.tiles_x - strip * STRIP;
    const int64_t sw = left < STRIP ? left : STRIP;
    const int64_t ty = r / sw;
    const int64_t tx = strip * STRIP + (r - ty * sw);
    TileId id;
    id.grp = grp;
    id.b = grp / cgroups;
    id.h0 = hb0 + static_cast<int>(ty) * TH;
    id.w0 = static_cast<int>(tx) * TW;
    return id;
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.wait_all;" ::: "memory");
}

__host__ __device__ constexpr int cmax(int a, int b) { return a > b ? a : b; }
__host__ __device__ constexpr int align_up(int a, int m) {
    return a >= 0 ? (a + m - 1) / m * m : -((-a) / m * m);
}
__host__ __device__ constexpr int align_down(int a, int m) {
    return a >= 0 ? a / m * m : -((-a + m - 1) / m * m);
}

template <typename T> struct Elem;
template <> struct Elem<__half> { static constexpr int kind = 0; };
template <> struct Elem<__nv_bfloat16> { static constexpr int kind = 1; };
template <> struct Elem<float> { static constexpr int kind = 2; };

// acc += w[WI] * x[XI] on packed 32-bit words (element indices).
template <typename T, int WI, int XI>
__device__ __forceinline__ void fma_e(float& acc, const uint32_t* w, const uint32_t* x) {
    if constexpr (Elem<T>::kind == 2) {
        acc = fmaf(__uint_as_float(w[WI]), __uint_as_float(x[XI]), acc);
    } else {
        const uint32_t ww = w[WI >> 1], xx = x[XI >> 1];
        constexpr int sel = ((WI & 1) << 1) | (XI & 1);
        if constexpr (Elem<T>::kind == 0) {
            if constexpr (sel == 0)
                asm("{.reg .b16 a0,a1,b0,b1; mov.b32 {a0,a1},%1; mov.b32 {b0,b1},%2; fma.rn.f32.f16 %0, a0, b0, %0;}" : "+f"(acc) : "r"(ww), "r"(xx));
            else if constexpr (sel == 1)
                asm("{.reg .b16 a0,a1,b0,b1; mov.b32 {a0,a1},%1; mov.b32 {b0,b1},%2; fma.rn.f32.f16 %0, a0, b1, %0;}" : "+f"(acc) : "r"(ww), "r"(xx));
            else if constexpr (sel == 2)
                asm("{.reg .b16 a0,a1,b0,b1; mov.b32 {a0,a1},%1; mov.b32 {b0,b1},%2; fma.rn.f32.f16 %0, a1, b0, %0;}" : "+f"(acc) : "r"(ww), "r"(xx));
            else
                asm("{.reg .b16 a0,a1,b0,b1; mov.b32 {a0,a1},%1; mov.b32 {b0,b1},%2; fma.rn.f32.f16 %0, a1, b1, %0;}" : "+f"(acc) : "r"(ww), "r"(xx));
        } else {
            if constexpr (sel == 0)
                asm("{.reg .b16 a0,a1,b0,b1; mov.b32 {a0,a1},%1; mov.b32 {b0,b1},%2; fma.rn.f32.bf16 %0, a0, b0, %0;}" : "+f"(acc) : "r"(ww), "r"(xx));
            else if constexpr (sel == 1)
                asm("{.reg .b16 a0,a1,b0,b1; mov.b32 {a0,a1},%1; mov.b32 {b0,b1},%2; fma.rn.f32.bf16 %0, a0, b1, %0;}" : "+f"(acc) : "r"(ww), "r"(xx));
            else if constexpr (sel == 2)
                asm("{.reg .b16 a0,a1,b0,b1; mov.b32 {a0,a1},%1; mov.b32 {b0,b1},%2; fma.rn.f32.bf16 %0, a1, b0, %0;}" : "+f"(acc) : "r"(ww), "r"(xx));
            else
                asm("{.reg .b16 a0,a1,b0,b1; mov.b32 {a0,a1},%1; mov.b32 {b0,b1},%2; fma.rn.f32.bf16 %0, a1, b1, %0;}" : "+f"(acc) : "r"(ww), "r"(xx));
        }
    }
}

// acc += w[WI]
template <typename T, int WI>
__device__ __forceinline__ void add_e(float& acc, const uint32_t* w) {
    if constexpr (Elem<T>::kind == 2) {
        acc += __uint_as_float(w[WI]);
    } else {
        const uint32_t ww = w[WI >> 1];
        if constexpr (Elem<T>::kind == 0) {
            if constexpr ((WI & 1) == 0)
                asm("{.reg .b16 a0,a1; mov.b32 {a0,a1},%1; add.f32.f16 %0, a0, %0;}" : "+f"(acc) : "r"(ww));
            else
                asm("{.reg .b16 a0,a1; mov.b32 {a0,a1},%1; add.f32.f16 %0, a1, %0;}" : "+f"(acc) : "r"(ww));
        } else {
            if constexpr ((WI & 1) == 0)
                asm("{.reg .b16 a0,a1; mov.b32 {a0,a1},%1; add.f32.bf16 %0, a0, %0;}" : "+f"(acc) : "r"(ww));
            else
                asm("{.reg .b16 a0,a1; mov.b32 {a0,a1},%1; add.f32.bf16 %0, a1, %0;}" : "+f"(acc) : "r"(ww));
        }
    }
}

// Compile-time loop helper: f(std::integral_constant<int, I>) for I in [0, N).
template <int I, int N, typename F>
__device__ __forceinline__ void static_for(F&& f) {
    if constexpr (I < N) {
        f(std::integral_constant<int, I>{});
        static_for<I + 1, N>(f);
    }
}

// Element I of packed words as fp32.
template <typename T, int I>
__device__ __forceinline__ float elem_f(const uint32_t* w) {
    if constexpr (Elem<T>::kind == 2) {
        return __uint_as_float(w[I]);
    } else if constexpr (Elem<T>::kind == 1) {
        const uint32_t v = w[I >> 1];
        return __uint_as_float((I & 1) ? (v & 0xFFFF0000u) : (v << 16));
    } else {
        const uint32_t v = w[I >> 1];
        return __half2float(__ushort_as_half(
            static_cast<unsigned short>((I & 1) ? (v >> 16) : (v & 0xFFFFu))));
    }
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kLazy = 16.0f;        // log mode: rescale when a > 2^16
constexpr float kPosLazy = 65536.0f;  // positive mode: the same bound

__device__ __forceinline__ float ex2_fast(float v) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}

// Modes 1 / 2: add V keys (key element KI + i of `kw`, image element XI + i
// of `xw[c]`) to the per-pixel online sums.  MASK: image element XI + i is
// a mirror source; bit (XI + i) of `valid` says it is inside the image.
template <typename T, int MODE, int NC, int V, int KI, int XI, bool MASK, int NX>
__device__ __forceinline__ void norm_keys(const uint32_t* kw, const uint32_t (&xw)[NC][NX],
                                          float (&u)[NC][V], float (&z)[V],
                                          float (&mr)[V], uint64_t valid) {
    float a[V];
    float amax = -INFINITY, amin = INFINITY;
    static_for<0, V>([&](auto ic) {
        constexpr int i = decltype(ic)::value;
        const float key = elem_f<T, KI + i>(kw);
        if constexpr (MODE == 1) {
            a[i] = fmaf(key, kLog2e, -mr[i]);
            if constexpr (MASK)
                a[i] = ((valid >> (XI + i)) & 1ull) ? a[i] : -INFINITY;
        } else {
            a[i] = key * mr[i];
            amin = fminf(amin, a[i]);
        }
        asm("max.NaN.f32 %0, %0, %1;" : "+f"(amax) : "f"(a[i]));
    });
    const bool need = MODE == 1 ? !(amax <= kLazy) : (!(amax <= kPosLazy) || amin < 0.f);
    if (__builtin_expect(__any_sync(0xffffffffu, need), 0)) {
        static_for<0, V>([&](auto ic) {
            constexpr int i = decltype(ic)::value;
            const float key = elem_f<T, KI + i>(kw);
            if constexpr (MODE == 1) {
                if (a[i] > kLazy) {          // false for NaN keys: they poison below
                    const float mn = key * kLog2e;
                    const float f = ex2_fast(mr[i] - mn);
                    z[i] *= f;
#pragma unroll
                    for (int c = 0; c < NC; ++c) u[c][i] *= f;
                    mr[i] = mn;
                    a[i] = fmaf(key, kLog2e, -mn);
                }
            } else {
                if (!(a[i] <= kPosLazy) || a[i] < 0.f) {
                    if (!(key >= 0.f) || key == INFINITY) {
                        z[i] = __int_as_float(0x7fffffff);   // poison: NaN
                        a[i] = 0.f;
                    } else {
                        // binary exponent of the key (subnormals clamp below)
                        int e = static_cast<int>((__float_as_uint(key) >> 23) & 0xFFu) - 127;
                        e = e < -100 ? -100 : (e > 126 ? 126 : e);
                        const float sc = __int_as_float((127 - e) << 23);
                        const float keep = mr[i] == INFINITY ? 0.f : sc / mr[i];
                        z[i] *= keep;
#pragma unroll
                        for (int c = 0; c < NC; ++c) u[c][i] *= keep;
                        mr[i] = sc;
                        a[i] = key * sc;
                    }
                }
            }
        });
    }
    static_for<0, V>([&](auto ic) {
        constexpr int i = decltype(ic)::value;
        const float ai = MODE == 1 ? ex2_fast(a[i]) : a[i];
        z[i] += ai;
#pragma unroll
        for (int c = 0; c < NC; ++c) u[c][i] = fmaf(ai, elem_f<T, XI + i>(xw[c]), u[c][i]);
    });
}

template <int N>
__device__ __forceinline__ void lds_words(uint32_t (&dst)[N], const void* src, int word0 = 0) {
    static_assert(N % 4 == 0, "16-byte granules");
#pragma unroll
    for (int k = 0; k < N / 4; ++k) {
        const uint4 v = reinterpret_cast<const uint4*>(src)[k];
        dst[word0 + 4 * k + 0] = v.x;
        dst[word0 + 4 * k + 1] = v.y;
        dst[word0 + 4 * k + 2] = v.z;
        dst[word0 + 4 * k + 3] = v.w;
    }
}

__device__ __forceinline__ int64_t pmod(int64_t a, int64_t n) {
    int64_t r = a % n;
    return r < 0 ? r + n : r;
}


// 16 / 8 / 4-byte shared-memory loads by 32-bit shared address.  volatile
// keeps them ordered after the mbarrier waits (also volatile asm).
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
// Non-volatile 16-byte shared load: free to be scheduled early.  Callers
// order it after the data became visible through a data dependency on the
// address (see `after`).
__device__ __forceinline__ uint4 lds128nv(uint32_t a) {
    uint4 v;
    asm("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
// Returns `a` through a volatile asm, so values computed from the result
// cannot be computed before the preceding volatile asm (the mbarrier wait).
__device__ __forceinline__ uint32_t after(uint32_t a) {
    uint32_t r;
    asm volatile("mov.b32 %0, %1;" : "=r"(r) : "r"(a));
    return r;
}
template <int N>
__device__ __forceinline__ void lds_words32(uint32_t* dst, uint32_t a) {
#pragma unroll
    for (int k = 0; k < N / 4; ++k) {
        const uint4 v = lds128nv(a + 16 * k);
        dst[4 * k] = v.x; dst[4 * k + 1] = v.y; dst[4 * k + 2] = v.z; dst[4 * k + 3] = v.w;
    }
}
// Load words [K, HI) of the shared-memory row at byte address `a` into
// d[K - LO ...] with the widest aligned vector (the row base is 16-byte
// aligned).
template <int K, int HI, int LO, int N>
__device__ __forceinline__ void load_win32(uint32_t (&d)[N], uint32_t a) {
    if constexpr (K < HI) {
        if constexpr (K % 4 == 0 && K + 4 <= HI) {
            const uint4 v = lds128(a + 4 * K);
            d[K - LO] = v.x; d[K - LO + 1] = v.y; d[K - LO + 2] = v.z; d[K - LO + 3] = v.w;
            load_win32<K + 4, HI, LO>(d, a);
        } else if constexpr (K % 2 == 0 && K + 2 <= HI) {
            const uint2 v = lds64(a + 4 * K);
            d[K - LO] = v.x; d[K - LO + 1] = v.y;
            load_win32<K + 2, HI, LO>(d, a);
        } else {
            d[K - LO] = lds32(a + 4 * K);
            load_win32<K + 1, HI, LO>(d, a);
        }
    }
}

// Load words [K, HI) of a shared-memory row into d[K - LO ...], using the
// widest aligned vector (the row base is 16-byte aligned).
template <int K, int HI, int LO, int N>
__device__ __forceinline__ void load_win(uint32_t (&d)[N], const uint32_t* p) {
    if constexpr (K < HI) {
        if constexpr (K % 4 == 0 && K + 4 <= HI) {
            const uint4 v = *reinterpret_cast<const uint4*>(p + K);
            d[K - LO] = v.x; d[K - LO + 1] = v.y; d[K - LO + 2] = v.z; d[K - LO + 3] = v.w;
            load_win<K + 4, HI, LO>(d, p);
        } else if constexpr (K % 2 == 0 && K + 2 <= HI) {
            const uint2 v = *reinterpret_cast<const uint2*>(p + K);
            d[K - LO] = v.x; d[K - LO + 1] = v.y;
            load_win<K + 2, HI, LO>(d, p);
        } else {
            d[K - LO] = p[K];
            load_win<K + 1, HI, LO>(d, p);
        }
    }
}

// EXACT: the table is the canonical half-plane table of radius Rdy <= DYMAX
// (for every dx: dy = 1..Rdy with mirror terms, plus (dx, 0) for dx >= 0
// with a mirror term for dx != 0; weight planes consecutive along dy), so
// which entries exist, which have a mirror term and how they group into
// copies are compile-time facts of dy and need no per-shift table tests.
template <typename T, int NC, int DYMIN, int DYMAX, bool EXACT, int MODE>
__global__ void __launch_bounds__(NTHREADS, 1)
acc_fast_kernel(const __grid_constant__ WMaps wmaps, const T* __restrict__ x,
                float* __restrict__ U, float* __restrict__ Zo, const FastTable tab,
                const Geo g, unsigned int* timeouts,
                unsigned long long* __restrict__ ticket, int* __restrict__ invalid,
                const GeoExt gx) {
    // modes 1 / 2: U receives D and Zo receives log_C
    constexpr int V = 16 / static_cast<int>(sizeof(T));
    constexpr int EPW = 4 / static_cast<int>(sizeof(T));   // elements per word
    constexpr int TW = TPR * V;
    constexpr int XC = align_up(cmax(DYMAX, -DYMIN), V);
    // register windows, in elements relative to the thread's first column
    // (tile column tc*V), then in 32-bit words
    constexpr int FLO = XC + DYMIN, FHI = XC + DYMAX + V;
    constexpr int MLO = XC - DYMAX, MHI = XC - DYMIN + V;
    constexpr int FWL = FLO / EPW, FWH = (FHI + EPW - 1) / EPW;
    constexpr int MWL = MLO / EPW, MWH = (MHI + EPW - 1) / EPW;
    constexpr int NDY = DYMAX - DYMIN + 1;

    extern __shared__ __align__(128) unsigned char smem_raw[];
    // TMA destinations must be 128-byte aligned: align the base explicitly
    // (the launcher reserves 128 extra bytes).
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int NSTAGE = g.nstage;
    unsigned char* stages = smem;
    T* xa0 = reinterpret_cast<T*>(smem + NSTAGE * g.stage_stride);
    const int xtile = NC * g.XH * g.XW;
    uint64_t* full = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(xa0 + xtile) + 15) & ~uintptr_t(15));
    uint64_t* empty = full + NSTAGE;
    // Dynamic tile order: the producer draws tickets from a global counter
    // (two tiles ahead) and publishes them in a 4-slot ring.  Tiles are then
    // processed in raster order across all CTAs, so vertically and
    // horizontally adjacent tiles -- whose weight boxes overlap -- run at the
    // same time and their shared rows are served by L2.
    uint64_t* tile_full = empty + NSTAGE;
    int64_t* tile_ring = reinterpret_cast<int64_t*>(tile_full + 4);
    int& abort_flag = *reinterpret_cast<int*>(tile_ring + 4);

    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < NSTAGE; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], NCONS / 32);
        }
        for (int i = 0; i < 4; ++i) mbar_init(&tile_full[i], 1);
        abort_flag = 0;
        (&abort_flag)[1] = static_cast<int>(gx.wait_budget);   // read by the slow waits
        fence_mbar_init();
    }
    __syncthreads();

    const int Rx = tab.Rx;
    const int64_t cgroups = (g.Cw == 1) ? 1 : g.C;

    // ------------------------------------------------------------ producer
    if (tid >= NCONS) {
        if (tid != NCONS) return;
        uint32_t it = 0;
        int stage = 0;
        uint32_t phase = 0;
        bool aborted = false;
        auto fetch = [&](uint32_t k) {
            const unsigned long long t = atomicAdd(ticket, 1ull);
            *(volatile int64_t*)&tile_ring[k & 3] =
                t < static_cast<unsigned long long>(g.ntiles) ? static_cast<int64_t>(t) : -1;
            mbar_arrive(&tile_full[k & 3]);
        };
        fetch(0);
        fetch(1);
        for (uint32_t k = 0; !aborted; ++k) {
            const int64_t tile = *(volatile int64_t*)&tile_ring[k & 3];
            if (tile < 0) break;
            fetch(k + 2);
            const TileId id = decode_tile(tile, g, gx.hb0, TW, cgroups);
            const int64_t b = id.b;
            const int64_t wc = (g.Cw == 1) ? 0 : id.grp % cgroups;
            const int h0 = id.h0, w0 = id.w0;
            for (int dx = -Rx; dx <= Rx && !aborted; ++dx) {
                if (!tab.row_any[dx + MAXR]) continue;
                for (int dy = DYMIN; dy <= DYMAX; ++dy) {
                    const int e = tab.s[dx + MAXR][dy + MAXR];
                    const int len = (e >> kLenShift) & 7;
                    if (e < 0 || len == 0) continue;
                    const int s = e & kSMask;
                    if (!mbar_wait(&empty[stage], phase ^ 1u, timeouts, gx.wait_budget) ||
                        *(volatile int*)&abort_flag) {
                        aborted = true;
                        *(volatile int*)&abort_flag = 1;
                        break;
                    }
                    if (static_cast<int32_t>(it) == gx.skip_copy) {
                        // test hook: leave this stage's copy unissued, so the
                        // consumers' bounded waits on it give up
                        ++it;
                        if (++stage == NSTAGE) { stage = 0; phase ^= 1u; }
                        continue;
                    }
                    mbar_arrive_expect_tx(&full[stage], len * g.plane_bytes);
                    const int mo = dy > 0 ? align_up(dy, V) : 0;
                    // weight plane (s, b, wc) is slice s of the (B*Cw) index
                    // b * Cw + wc; a copy of `len` planes takes s .. s+len-1.
                    const CUtensorMap* map = len == 1 ? &wmaps.m[0]
                                             : len == 2 ? &wmaps.m[1]
                                             : len == 3 ? &wmaps.m[2] : &wmaps.m[3];
                    tma_load_4d(stages + stage * g.stage_stride, map,
                                &full[stage], w0 - mo, h0 - (dx > 0 ? dx : 0),
                                static_cast<int32_t>(b * g.Cw + wc), s);
                    ++it;
                    if (++stage == NSTAGE) { stage = 0; phase ^= 1u; }
                }
            }
        }
        // Drain: the CTA must not exit with copies into its shared memory in
        // flight.  Wait (bounded) for the last NSTAGE loads to land.
        const uint32_t n = it < static_cast<uint32_t>(NSTAGE) ? it : NSTAGE;
        for (uint32_t j = it - n; j < it; ++j)
            if (static_cast<int32_t>(j) != gx.skip_copy)
                mbar_wait(&full[j % NSTAGE], (j / NSTAGE) & 1u, timeouts, gx.wait_budget);
        return;
    }

    // ------------------------------------------------------------ consumers
    const uint32_t stages32 = smem_u32(stages);
    const uint32_t full32 = smem_u32(full), empty32 = smem_u32(empty);
    const int tr = tid / TPR, tc = tid % TPR;
    const int lane = tid & 31;
    int stage = 0;
    uint32_t phase = 0;
    const int XH = g.XH, XW = g.XW, BW = g.BW;

    // A consumer whose bounded wait gave up stops waiting (`dead`) but keeps
    // executing every barrier, so no thread is left waiting for it; all
    // consumers leave together at the next tile boundary.
    bool dead = false;
    const int nv = XW / V;
    const int xtotal = NC * XH * nv;
    const int64_t xplane = g.x_rows * g.W;

    // Chunk (c, i, jv) of the x tile of a tile at (b, c0, h0, w0): 16 bytes
    // of row r = h0 - Rx + i, columns col0 .. col0 + V.  `direct` chunks are
    // inside the x buffer without wrapping and are copied asynchronously.
    auto chunk = [&](int idx, int h0, int w0, int& c, int& i, int& jv, int64_t& r,
                     int64_t& col0, int64_t& xr, bool& rv, bool& direct) {
        c = idx / (XH * nv);
        const int rem = idx - c * XH * nv;
        i = rem / nv;
        jv = rem - i * nv;
        r = static_cast<int64_t>(h0) - Rx + i;
        col0 = static_cast<int64_t>(w0) - XC + jv * V;
        xr = g.wrap ? pmod(r, g.x_rows) : r + g.x_off;
        rv = xr >= 0 && xr < g.x_rows;
        direct = rv && (g.wrap ? (r >= 0 && r < g.x_rows) : true) && col0 >= 0 &&
                 col0 + V <= g.W;
    };
    auto issue_x = [&](int64_t tile, T* dst) {
        const TileId id = decode_tile(tile, g, gx.hb0, TW, cgroups);
        const int64_t c0 = (g.Cw == 1) ? 0 : id.grp % cgroups;
        for (int idx = tid; idx < xtotal; idx += NCONS) {
            int c, i, jv;
            int64_t r, col0, xr;
            bool rv, direct;
            chunk(idx, id.h0, id.w0, c, i, jv, r, col0, xr, rv, direct);
            if (direct)
                cp_async16(dst + (c * XH + i) * XW + jv * V,
                           x + (id.b * g.C + c0 + c) * xplane + xr * g.W + col0);
        }
        cp_async_commit();
    };

    // Tile k of this CTA (ring slot k & 3), -1 when the schedule is done.
    auto tile_at = [&](uint32_t k) -> int64_t {
        if (!dead && !mbar_wait(&tile_full[k & 3], (k >> 2) & 1u, timeouts, gx.wait_budget)) {
            dead = true;
            *(volatile int*)&abort_flag = 1;
        }
        return dead ? -1 : *(volatile int64_t*)&tile_ring[k & 3];
    };
    int64_t tile = tile_at(0);
    if (tile >= 0) issue_x(tile, xa0);
    for (uint32_t k = 0; tile >= 0; ++k) {
        const TileId id = decode_tile(tile, g, gx.hb0, TW, cgroups);
        const int64_t b = id.b;
        const int64_t c0 = (g.Cw == 1) ? 0 : id.grp % cgroups;
        const int h0 = id.h0, w0 = id.w0;
        if (k > 0) {
            named_sync(1, NCONS);   // every thread is done with the previous tile
            issue_x(tile, xa0);
        }
        T* xa = xa0;
        const bool row_border = h0 - Rx < 0 || h0 + TH + Rx > g.H;
        const bool col_border = w0 - XC < 0 || w0 + TW + XC + V > g.W;

        // ---- finish the x tile: wait for this tile's async copies and fill
        // the chunks that wrap or fall outside the x buffer
        cp_async_wait_all();
        named_sync(1, NCONS);
        if (*(volatile int*)&abort_flag) break;
        if (row_border || col_border) {
            for (int idx = tid; idx < xtotal; idx += NCONS) {
                int c, i, jv;
                int64_t r, col0, xr;
                bool rv, direct;
                chunk(idx, h0, w0, c, i, jv, r, col0, xr, rv, direct);
                if (direct) continue;
                const T* xp = x + (b * g.C + c0 + c) * xplane;
                T ea[V];
#pragma unroll
                for (int k = 0; k < V; ++k)
                    ea[k] = rv ? xp[xr * g.W + pmod(col0 + k, g.W)] : T(0.0f);
                *reinterpret_cast<uint4*>(xa + (c * XH + i) * XW + jv * V) =
                    *reinterpret_cast<const uint4*>(ea);
            }
            named_sync(1, NCONS);
        }
        const int64_t next = tile_at(k + 1);

        float u[NC][V], z[V], mr[V];
#pragma unroll
        for (int i = 0; i < V; ++i) {
            z[i] = 0.f;
            // modes 1 / 2: running reference (log2 units) / scale 2^-e (inf: unset)
            mr[i] = MODE == 1 ? -3.0e38f : INFINITY;
#pragma unroll
            for (int c = 0; c < NC; ++c) u[c][i] = 0.f;
        }
        const int64_t gcol0 = static_cast<int64_t>(w0) - XC + tc * V;  // image column of window element 0

        for (int dx = -Rx; dx <= Rx; ++dx) {
            if (!tab.row_any[dx + MAXR]) continue;
            uint32_t xf[NC][FWH - FWL], xm[NC][MWH - MWL];
            uint64_t mvalid = ~0ull;   // mirror window elements inside the image
            const uint32_t xa32 = smem_u32(xa) + static_cast<uint32_t>(tc * V * sizeof(T));
            const uint32_t xrow = static_cast<uint32_t>(XH * XW * sizeof(T));
#pragma unroll
            for (int c = 0; c < NC; ++c)
                load_win32<FWL, FWH, FWL>(xf[c], xa32 + c * xrow +
                    static_cast<uint32_t>((tr + dx + Rx) * XW * sizeof(T)));
            if (tab.row_inv[dx + MAXR]) {
#pragma unroll
                for (int c = 0; c < NC; ++c)
                    load_win32<MWL, MWH, MWL>(xm[c], xa32 + c * xrow +
                        static_cast<uint32_t>((tr - dx + Rx) * XW * sizeof(T)));
                // the mirror term reads x only inside the image
                if (row_border || col_border) {
                    const int64_t grow = static_cast<int64_t>(h0) + tr - dx;
                    const bool rin = grow >= 0 && grow < g.H;
#pragma unroll
                    for (int k = 0; k < (MWH - MWL) * EPW; ++k) {
                        const int64_t gc = gcol0 + MWL * EPW + k;
                        if (!rin || gc < 0 || gc >= g.W) {
                            mvalid &= ~(1ull << k);
                            const uint32_t keep =
                                EPW == 1 ? 0u : ((k & 1) ? 0x0000FFFFu : 0xFFFF0000u);
#pragma unroll
                            for (int c = 0; c < NC; ++c) xm[c][k / EPW] &= keep;
                        }
                    }
                }
            }
            // Shared-memory byte offsets of this thread's main and mirror
            // weight rows inside a stage, hoisted out of the shift loop.
            const int mrow0 = tr + (dx > 0 ? dx : 0);
            const uint32_t off_main = static_cast<uint32_t>((mrow0 * BW + tc * V) * sizeof(T));
            const uint32_t off_mir = static_cast<uint32_t>(((mrow0 - dx) * BW + tc * V) * sizeof(T));
            const uint64_t m_pres = tab.present[dx + MAXR], m_inv = tab.inv[dx + MAXR];
            const uint64_t m_pos0 = tab.pos0[dx + MAXR], m_pos1 = tab.pos1[dx + MAXR];
            const uint64_t m_last = tab.last[dx + MAXR];
            uint32_t stp = stages32 + stage * g.stage_stride;
            // pos: plane of this entry inside its copy (the copy's first
            // entry waits for it); last: the copy is released afterwards
            auto one = [&](auto dyc, const int pos, const bool last, const bool inv) {
                constexpr int dy = decltype(dyc)::value;
                if (pos == 0)
                    mbar_wait32_ab(full32 + 8 * stage, phase, timeouts,
                                   (volatile int*)&abort_flag);
                const uint32_t sp = after(stp) + pos * g.plane_bytes;
                constexpr int mo = dy > 0 ? align_up(dy, V) : 0;
                uint32_t wv[V / EPW];
                lds_words32<V / EPW>(wv, sp + off_main + mo * sizeof(T));
                if constexpr (MODE == 0) {
                    static_for<0, V>([&](auto ic) {
                        constexpr int i = decltype(ic)::value;
#pragma unroll
                        for (int c = 0; c < NC; ++c)
                            fma_e<T, i, XC + dy + i - FWL * EPW>(u[c][i], wv, xf[c]);
                        add_e<T, i>(z[i], wv);
                    });
                } else {
                    norm_keys<T, MODE, NC, V, 0, XC + dy - FWL * EPW, false>(
                        wv, xf, u, z, mr, 0ull);
                }
                if (inv) {
                    constexpr int moff = mo - dy;               // >= 0
                    constexpr int kk = moff % V;
                    constexpr int mb = moff - kk;
                    uint32_t mw[2 * V / EPW];
                    lds_words32<V / EPW>(mw, sp + off_mir + mb * sizeof(T));
                    if constexpr (kk != 0)
                        lds_words32<V / EPW>(mw + V / EPW, sp + off_mir + (mb + V) * sizeof(T));
                    if constexpr (MODE == 0) {
                        static_for<0, V>([&](auto ic) {
                            constexpr int i = decltype(ic)::value;
#pragma unroll
                            for (int c = 0; c < NC; ++c)
                                fma_e<T, kk + i, XC - dy + i - MWL * EPW>(u[c][i], mw, xm[c]);
                            add_e<T, kk + i>(z[i], mw);
                        });
                    } else {
                        norm_keys<T, MODE, NC, V, kk, XC - dy - MWL * EPW, MODE == 1>(
                            mw, xm, u, z, mr, mvalid);
                    }
                }
                if (last) {   // copy fully used: release it
                    __syncwarp();
                    if (lane == 0) mbar_arrive32(empty32 + 8 * stage);
                    if (++stage == NSTAGE) {
                        stage = 0;
                        phase ^= 1u;
                        stp = stages32;
                    } else {
                        stp += g.stage_stride;
                    }
                }
            };
            if constexpr (EXACT) {
                // (dx, 0): a single copy, mirror term unless dx == 0
                if (dx >= 0) one(std::integral_constant<int, 0>{}, 0, true, dx != 0);
                const int R = tab.Rdy;
                // dy = 1..R: copies of kGroup planes, dy 1..kGroup,
                // kGroup+1..2 kGroup, ...; the last copy ends at dy = R.
                static_for<1, DYMAX + 1>([&](auto jc) {
                    constexpr int dy = decltype(jc)::value;
                    if (dy > R) return;
                    constexpr int p = (dy - 1) % kGroup;
                    one(jc, p, p == kGroup - 1 || dy == R, true);
                });
            } else {
                static_for<0, NDY>([&](auto jc) {
                    constexpr int dy = DYMIN + decltype(jc)::value;
                    constexpr int bit = dy + MAXR;
                    if (!((m_pres >> bit) & 1u)) return;
                    one(std::integral_constant<int, dy>{},
                        static_cast<int>(((m_pos0 >> bit) & 1u) | (((m_pos1 >> bit) & 1u) << 1)),
                        (m_last >> bit) & 1u, (m_inv >> bit) & 1u);
                });
            }
        }

        // ---- store
        const int64_t h = h0 + tr;
        const int64_t wcol = w0 + tc * V;
        if constexpr (MODE != 0) {
            // D = sum a x / sum a, log_C = reference + log(sum a); special
            // values as in the general kernel
            bool bad = false;
#pragma unroll
            for (int i = 0; i < V; ++i) {
                const float sv = z[i];
                if (sv != sv) {
                    bad = true;
                    z[i] = __int_as_float(0x7fffffff);
#pragma unroll
                    for (int c = 0; c < NC; ++c) u[c][i] = z[i];
                } else if (sv == 0.f) {
                    z[i] = -INFINITY;
#pragma unroll
                    for (int c = 0; c < NC; ++c) u[c][i] = 0.f;
                } else {
                    const float base = MODE == 1
                        ? mr[i] * kLn2
                        : -static_cast<float>(static_cast<int>((__float_as_uint(mr[i]) >> 23) & 0xFFu) - 127) * kLn2;
                    z[i] = base + logf(sv);
#pragma unroll
                    for (int c = 0; c < NC; ++c) u[c][i] = u[c][i] / sv;
                }
            }
            if (bad && invalid && h < gx.hb1 && wcol < g.W) atomicOr(invalid, 1);
        }
        if (h < gx.hb1 && wcol < g.W) {
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int64_t o = ((b * g.C + c0 + c) * g.H + h) * g.W + wcol;
#pragma unroll
                for (int q = 0; q < V / 4; ++q) {
                    *reinterpret_cast<float4*>(U + o + 4 * q) =
                        make_float4(u[c][4 * q], u[c][4 * q + 1], u[c][4 * q + 2], u[c][4 * q + 3]);
                    *reinterpret_cast<float4*>(Zo + o + 4 * q) =
                        make_float4(z[4 * q], z[4 * q + 1], z[4 * q + 2], z[4 * q + 3]);
                }
            }
        }
        tile = next;
    }
    cp_async_wait_all();
}

}  // namespace fast
}  // namespace nsc
