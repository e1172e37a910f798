// normalized_fast.cuh -- tiled forward of normalized_accumulate_uz for
// tables without mirror terms (every has_inv == 0), e.g. the full
// (2R+1)^2 attention window of the GASD / NeKDe patches.
//
// CTA = 256 threads, tile = 16 output rows x 16*V columns (V = 16 bytes of
// the storage type per thread: 8 fp16/bf16 or 4 fp32 pixels, one row per
// thread) of one image and one weight channel (all NC image channels when
// the weight is channel-broadcast).
//
// x: the tile plus its (Rx, XC) halo -- rows and columns circular, the
// forward term is periodic -- is staged once in shared memory; for every dx
// each thread loads register windows of its row h + dx and serves every dy
// of the row from them with compile-time indices (dy is a template-unrolled
// loop over [DYMIN, DYMAX], entries selected by a per-row bit mask).
//
// Keys: every thread streams its own 16-byte key vector of each shift
// through a private NST-slot ring in shared memory with cp.async (prefetch
// distance NST - 2), so no CTA barrier sits in the shift loop and each
// thread keeps NST - 2 copies in flight.
//
// Reduction per pixel: the online normalisation of Milakov & Gimelshein
// (2018) with a lazy reference.  Log mode keeps m (log2 units) and adds
// a = 2^(k*log2(e) - m); m moves only when a key would give a > 2^T, and
// then the partial sums are rescaled by 2^(m_old - m_new).  Positive mode
// keeps a power-of-two scale 2^-e and adds a = k * 2^-e (exact), rescaling
// the same way.  Sums stay below 2S * 2^T, far from overflow, and the
// result equals sum(a x) / sum(a) of the exact normalisation up to fp32
// rounding.  Semantics of the general kernel (normalized.cu): a NaN or +inf
// key (or a negative positive-mode weight) poisons the pixel's sums (D and
// log_C NaN, invalid flag set); -inf logits / zero weights contribute
// nothing; a pixel without a live key gives D = 0, log_C = -inf.
#pragma once

#include <cmath>
#include <cstdint>

#include "nsc_common.cuh"

namespace nsc {
namespace nfast {

// Key bytes per thread and shift: 16 (8 fp16/bf16 pixels) or 8 (4 pixels,
// half the unrolled code and registers, so more CTAs per SM).
#ifndef NSC_NORM_KB
#define NSC_NORM_KB 8
#endif
constexpr int KB = NSC_NORM_KB;
constexpr int TPR = 256 / KB;       // threads per row: 128 bytes of keys
constexpr int TH = 256 / TPR;       // rows per tile
constexpr int NT = TPR * TH;        // 256 threads
constexpr int NST = 8;              // key ring slots per thread
constexpr int MAXR = 16;            // |dx|, |dy| <= MAXR on this path
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kLazy = 16.0f;      // rescale when a key would give a > 2^16

struct NormTable {
    int32_t nsteps;                  // = S
    int32_t nrows;                   // dx rows with at least one entry
    int32_t row_dx[2 * MAXR + 1];
    uint32_t row_mask[2 * MAXR + 1]; // bit (dy - DYMIN): entry present
    int16_t seq[kMaxShifts];         // weight plane of each step, compute order
};

struct NormGeo {
    int32_t B, C, H, W, Cw;
    int32_t tiles_x, tiles_y;
    int32_t Rx, XH, XW;              // x halo: rows h0-Rx.., XW columns
    int64_t groups;                  // B * channel groups
    int64_t step_stride;             // elements between weight planes s, s+1
};

__device__ __forceinline__ float ex2_approx(float v) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}

__device__ __forceinline__ void cp_async16_n(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_kb(uint32_t dst, const void* src) {
    if constexpr (KB == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src)
                     : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src)
                     : "memory");
}
__device__ __forceinline__ void cp_async_commit_n() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait_n() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint4 lds128v(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
// Words [K, HI) of the shared-memory row at byte address `a` (aligned to
// 4*MAXW bytes) into d[K - LO ...], with the widest aligned vector loads.
template <int K, int HI, int LO, int MAXW, int N>
__device__ __forceinline__ void load_words(uint32_t (&d)[N], uint32_t a) {
    if constexpr (K < HI) {
        if constexpr (MAXW >= 4 && K % 4 == 0 && K + 4 <= HI) {
            const uint4 v = lds128v(a + 4 * K);
            d[K - LO] = v.x; d[K - LO + 1] = v.y; d[K - LO + 2] = v.z; d[K - LO + 3] = v.w;
            load_words<K + 4, HI, LO, MAXW>(d, a);
        } else if constexpr (K % 2 == 0 && K + 2 <= HI) {
            uint32_t p, q;
            asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(p), "=r"(q) : "r"(a + 4 * K));
            d[K - LO] = p; d[K - LO + 1] = q;
            load_words<K + 2, HI, LO, MAXW>(d, a);
        } else {
            uint32_t p;
            asm volatile("ld.shared.u32 %0, [%1];" : "=r"(p) : "r"(a + 4 * K));
            d[K - LO] = p;
            load_words<K + 1, HI, LO, MAXW>(d, a);
        }
    }
}
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Element I of a packed register array, as fp32.
template <typename T, int I, int N>
__device__ __forceinline__ float elem(const uint32_t (&w)[N]) {
    if constexpr (sizeof(T) == 4) {
        return __uint_as_float(w[I]);
    } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        const uint32_t v = w[I >> 1];
        return __uint_as_float((I & 1) ? (v & 0xFFFF0000u) : (v << 16));
    } else {
        const uint32_t v = w[I >> 1];
        return __half2float(__ushort_as_half(
            static_cast<unsigned short>((I & 1) ? (v >> 16) : (v & 0xFFFFu))));
    }
}

template <int I, int N, typename F>
__device__ __forceinline__ void sfor(F&& f) {
    if constexpr (I < N) {
        f(std::integral_constant<int, I>{});
        sfor<I + 1, N>(f);
    }
}

__device__ __forceinline__ int pmodi(int a, int n) {
    const int r = a % n;
    return r < 0 ? r + n : r;
}

template <typename T, int NC, int DYMIN, int DYMAX, bool LOGW>
__global__ void __launch_bounds__(NT, KB == 16 ? 2 : 3)
norm_fast_kernel(const T* __restrict__ x, const T* __restrict__ w,
                 float* __restrict__ D, float* __restrict__ L,
                 const NormTable tab, const NormGeo g, int* __restrict__ invalid) {
    constexpr int V = KB / static_cast<int>(sizeof(T));
    constexpr int EPW = 4 / static_cast<int>(sizeof(T));
    constexpr int TW = TPR * V;
    constexpr int VX = 16 / static_cast<int>(sizeof(T));   // staging chunk (16 bytes)
    constexpr int XC = ((DYMAX > -DYMIN ? DYMAX : -DYMIN) + VX - 1) / VX * VX;
    constexpr int FLO = XC + DYMIN, FHI = XC + DYMAX + V;   // window, elements
    constexpr int FWL = FLO / EPW, FWH = (FHI + EPW - 1) / EPW;
    constexpr int NW = FWH - FWL;
    constexpr int NDY = DYMAX - DYMIN + 1;
    static_assert(NDY <= 32, "dy mask is 32 bits");

    extern __shared__ __align__(16) unsigned char smem_n[];
    unsigned char* ring = smem_n;                             // [NST][NT][KB]
    T* xs = reinterpret_cast<T*>(smem_n + NST * NT * KB);      // [NC][XH][XW]

    const int tid = threadIdx.x;
    const int tr = tid / TPR, tc = tid % TPR;
    const int64_t HW = static_cast<int64_t>(g.H) * g.W;
    const int cgroups = (g.Cw == 1) ? (g.C + NC - 1) / NC : g.C;
    const uint32_t ring32 = smem_addr(ring) + tid * static_cast<uint32_t>(KB);

    for (int64_t grp = blockIdx.y; grp < g.groups; grp += gridDim.y) {
        const int b = static_cast<int>(grp / cgroups);
        const int cg = static_cast<int>(grp - static_cast<int64_t>(b) * cgroups);
        const int c0 = (g.Cw == 1) ? cg * NC : cg;
        const int wc = (g.Cw == 1) ? 0 : cg;
        const int nc = (g.Cw == 1) ? (g.C - c0 < NC ? g.C - c0 : NC) : 1;
        for (int64_t tile = blockIdx.x; tile < static_cast<int64_t>(g.tiles_x) * g.tiles_y;
             tile += gridDim.x) {
            const int ty = static_cast<int>(tile / g.tiles_x);
            const int tx = static_cast<int>(tile - static_cast<int64_t>(ty) * g.tiles_x);
            const int h0 = ty * TH, w0 = tx * TW;
            const int h = h0 + tr, wcol = w0 + tc * V;
            const bool active = h < g.H && wcol < g.W;

            // ---- key prefetch: steps 0 .. NST-3
            const T* wp = w + (static_cast<int64_t>(b) * g.Cw + wc) * HW +
                          static_cast<int64_t>(h) * g.W + wcol;
            auto issue = [&](int k) {
                if (active && k < tab.nsteps)
                    cp_async_kb(ring32 + (k % NST) * (NT * KB),
                                wp + static_cast<int64_t>(tab.seq[k]) * g.step_stride);
                cp_async_commit_n();
            };
            __syncthreads();   // previous tile's readers of xs are done
#pragma unroll
            for (int k = 0; k < NST - 2; ++k) issue(k);

            // ---- x halo tile, circular rows and columns
            const int nv = g.XW / VX;
            const int xtotal = NC * g.XH * nv;
            for (int idx = tid; idx < xtotal; idx += NT) {
                const int c = idx / (g.XH * nv);
                const int rem = idx - c * g.XH * nv;
                const int i = rem / nv;
                const int jv = rem - i * nv;
                T* dst = xs + (c * g.XH + i) * g.XW + jv * VX;
                if (c >= nc) {
                    *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
                    continue;
                }
                const int r = pmodi(h0 - g.Rx + i, g.H);
                const int col0 = w0 - XC + jv * VX;
                const T* src = x + (static_cast<int64_t>(b) * g.C + c0 + c) * HW +
                               static_cast<int64_t>(r) * g.W;
                if (col0 >= 0 && col0 + VX <= g.W) {
                    *reinterpret_cast<uint4*>(dst) =
                        __ldg(reinterpret_cast<const uint4*>(src + col0));
                } else {
#pragma unroll
                    for (int e = 0; e < VX; ++e) dst[e] = src[pmodi(col0 + e, g.W)];
                }
            }
            __syncthreads();

            float su[NC][V], sz[V], mr[V];
#pragma unroll
            for (int i = 0; i < V; ++i) {
                sz[i] = 0.f;
                mr[i] = LOGW ? -3.0e38f : INFINITY;   // log: m (log2); pos: scale 2^-e (inf: unset)
#pragma unroll
                for (int c = 0; c < NC; ++c) su[c][i] = 0.f;
            }
            int k = 0;
            const uint32_t xs32 = smem_addr(xs) + static_cast<uint32_t>(tc * V * sizeof(T));
            for (int ri = 0; ri < tab.nrows; ++ri) {
                const int dx = tab.row_dx[ri];
                const uint32_t pres = tab.row_mask[ri];
                uint32_t xw[NC][NW];
#pragma unroll
                for (int c = 0; c < NC; ++c)
                    load_words<FWL, FWH, FWL, KB / 4>(xw[c], xs32 + static_cast<uint32_t>(
                        ((c * g.XH + tr + dx + g.Rx) * g.XW) * sizeof(T)));
                sfor<0, NDY>([&](auto jc) {
                    constexpr int j = decltype(jc)::value;
                    constexpr int dy = DYMIN + j;
                    if (!((pres >> j) & 1u)) return;
                    issue(k + NST - 2);
                    cp_async_wait_n<NST - 2>();
                    uint32_t kw[KB / 4];
                    if constexpr (KB == 16) {
                        const uint4 kv4 = lds128v(ring32 + (k % NST) * (NT * KB));
                        kw[0] = kv4.x; kw[1] = kv4.y; kw[2] = kv4.z; kw[3] = kv4.w;
                    } else {
                        asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];"
                                     : "=r"(kw[0]), "=r"(kw[1])
                                     : "r"(ring32 + (k % NST) * (NT * KB)));
                    }
                    ++k;
                    // a_i before any rescale; one warp-uniform branch per
                    // key vector moves the reference of the lanes/pixels
                    // that need it (rare after the first keys).
                    float a[V];
                    float amax = -INFINITY, amin = INFINITY;
                    sfor<0, V>([&](auto ic) {
                        constexpr int i = decltype(ic)::value;
                        const float key = elem<T, i>(kw);
                        if constexpr (LOGW) {
                            a[i] = fmaf(key, kLog2e, -mr[i]);
                        } else {
                            a[i] = key * mr[i];
                            amin = fminf(amin, a[i]);
                        }
                        // NaN-propagating max: a NaN key takes the slow path
                        asm("max.NaN.f32 %0, %0, %1;" : "+f"(amax) : "f"(a[i]));
                    });
                    const bool need = LOGW ? !(amax <= kLazy)
                                           : (!(amax <= 65536.0f) || amin < 0.f);
                    if (__builtin_expect(__any_sync(0xffffffffu, need), 0)) {
                        sfor<0, V>([&](auto ic) {
                            constexpr int i = decltype(ic)::value;
                            const float key = elem<T, i>(kw);
                            if constexpr (LOGW) {
                                if (a[i] > kLazy) {
                                    const float mn = key * kLog2e;
                                    const float f = ex2_approx(mr[i] - mn);
                                    sz[i] *= f;
#pragma unroll
                                    for (int c = 0; c < NC; ++c) su[c][i] *= f;
                                    mr[i] = mn;
                                    a[i] = fmaf(key, kLog2e, -mn);
                                }
                            } else {
                                if (!(a[i] <= 65536.0f) || a[i] < 0.f) {
                                    if (!(key >= 0.f) || key == INFINITY) {
                                        sz[i] = __int_as_float(0x7fffffff);   // poison: NaN
                                        a[i] = 0.f;
                                    } else {
                                        // binary exponent (subnormals clamp below)
                                        int e = static_cast<int>((__float_as_uint(key) >> 23) & 0xFFu) - 127;
                                        e = e < -100 ? -100 : (e > 126 ? 126 : e);
                                        const float sc = __int_as_float((127 - e) << 23);
                                        const float keep = mr[i] == INFINITY ? 0.f : sc / mr[i];
                                        sz[i] *= keep;
#pragma unroll
                                        for (int c = 0; c < NC; ++c) su[c][i] *= keep;
                                        mr[i] = sc;
                                        a[i] = key * sc;
                                    }
                                }
                            }
                        });
                    }
                    sfor<0, V>([&](auto ic) {
                        constexpr int i = decltype(ic)::value;
                        const float ai = LOGW ? ex2_approx(a[i]) : a[i];
                        sz[i] += ai;
#pragma unroll
                        for (int c = 0; c < NC; ++c)
                            su[c][i] = fmaf(ai, elem<T, XC + dy + i - FWL * EPW>(xw[c]), su[c][i]);
                    });
                });
            }
            cp_async_wait_n<0>();

            // ---- outputs
            if (active) {
                bool bad = false;
                float d_out[NC][V], l_out[V];
#pragma unroll
                for (int i = 0; i < V; ++i) {
                    const float s = sz[i];
                    if (s != s) {
                        bad = true;
                        l_out[i] = __int_as_float(0x7fffffff);
#pragma unroll
                        for (int c = 0; c < NC; ++c) d_out[c][i] = l_out[i];
                    } else if (s == 0.f) {
                        l_out[i] = -INFINITY;
#pragma unroll
                        for (int c = 0; c < NC; ++c) d_out[c][i] = 0.f;
                    } else {
                        const float base = LOGW ? mr[i] * kLn2
                                                : -static_cast<float>(static_cast<int>((__float_as_uint(mr[i]) >> 23) & 0xFFu) - 127) * kLn2;
                        l_out[i] = base + logf(s);
#pragma unroll
                        for (int c = 0; c < NC; ++c) d_out[c][i] = su[c][i] / s;
                    }
                }
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    if (c >= nc) continue;
                    const int64_t o = (static_cast<int64_t>(b) * g.C + c0 + c) * HW +
                                      static_cast<int64_t>(h) * g.W + wcol;
                    if constexpr (V >= 4) {
#pragma unroll
                        for (int q = 0; q < V / 4; ++q) {
                            *reinterpret_cast<float4*>(D + o + 4 * q) =
                                make_float4(d_out[c][4 * q], d_out[c][4 * q + 1],
                                            d_out[c][4 * q + 2], d_out[c][4 * q + 3]);
                            *reinterpret_cast<float4*>(L + o + 4 * q) =
                                make_float4(l_out[4 * q], l_out[4 * q + 1],
                                            l_out[4 * q + 2], l_out[4 * q + 3]);
                        }
                    } else {
                        *reinterpret_cast<float2*>(D + o) = make_float2(d_out[c][0], d_out[c][1]);
                        *reinterpret_cast<float2*>(L + o) = make_float2(l_out[0], l_out[1]);
                    }
                }
                if (bad && invalid) atomicOr(invalid, 1);
            }
        }
    }
}

}  // namespace nfast
}  // namespace nsc
