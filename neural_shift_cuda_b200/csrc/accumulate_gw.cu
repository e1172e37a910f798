// accumulate_gw.cu -- tiled weight gradient of accumulate_uz.
//
//   gw_s(q) = sum_c gU_c(q) x_c(q + d) + gZ(q)
//           + inv [q + d inside] (sum_c x_c(q) gU_c(q + d) + gZ(q + d))
// (gZ summed over the channels the weight is shared by; reference
// shift_ops_cuda.cu:412-458).  The gradient never reads the weights: it is
// a correlation of grad_U with x at every shift, written once per weight
// element, so the kernel is bound by the S-fold write of grad_w (as large as
// the weight stack) and needs no weight traffic at all.
//
// CTA = 256 threads over an 8 x 128 tile of one image and one weight channel
// (all NC image channels when the weight is channel-broadcast); a thread
// owns 4 consecutive pixels of a row.  x (circular), grad_U and the channel
// sum of grad_Z (both zero outside the image: exactly the mirror term's
// inside test) are staged once per tile, with the table's row radius above
// and below and its dy range to the right, as fp32 in shared memory.  For
// every dx row of the table each thread loads register windows of x and
// grad_U at row h + dx covering all dy of the row and accumulates the
// gradients of every dy of that row in registers (dy is a compile-time
// index), channel by channel; then one 8- or 16-byte streaming store per
// (shift, thread) writes grad_w.
#include <cstdlib>
#include <cstring>
#include <initializer_list>

#include "nsc_common.cuh"
#include "nsc_host.h"
#include "accumulate.h"

namespace nsc {
namespace gwk {

constexpr int TH = 8, TPR = 32, V = 4, TW = TPR * V, NT = TH * TPR;
constexpr int MAXR = 16;

struct GwTable {
    int16_t s[2 * MAXR + 1][2 * MAXR + 1];   // [dx + MAXR][dy + MAXR] -> plane, -1 absent
    uint64_t present[2 * MAXR + 1];          // bit (dy + MAXR)
    uint64_t inv[2 * MAXR + 1];
    int32_t Rx;
};

struct GwGeo {
    int64_t B, C, H, W, Cw;
    int32_t tiles_x, tiles_y, XH, XW, CO;    // staged tile: XH rows, XW cols, col offset
};

template <typename T> __device__ __forceinline__ float to_f(T v) { return to_acc(v); }

template <typename TW> __device__ __forceinline__ void store4(TW* p, const float (&v)[V]);
template <> __device__ __forceinline__ void store4<float>(float* p, const float (&v)[V]) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(v[0], v[1], v[2], v[3]));
}
template <> __device__ __forceinline__ void store4<__half>(__half* p, const float (&v)[V]) {
    const __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    __stcs(reinterpret_cast<uint2*>(p), u);
}
template <> __device__ __forceinline__ void store4<__nv_bfloat16>(__nv_bfloat16* p,
                                                                  const float (&v)[V]) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]);
    const __nv_bfloat162 b = __floats2bfloat162_rn(v[2], v[3]);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    __stcs(reinterpret_cast<uint2*>(p), u);
}

template <int I, int N, typename F>
__device__ __forceinline__ void sfor(F&& f) {
    if constexpr (I < N) {
        f(std::integral_constant<int, I>{});
        sfor<I + 1, N>(f);
    }
}

// N floats from shared memory; ALIGNED: p is 16-byte aligned (float4 loads).
template <int N, bool ALIGNED>
__device__ __forceinline__ void load_row(float (&d)[N], const float* p) {
    if constexpr (ALIGNED) {
#pragma unroll
        for (int k = 0; k + 4 <= N; k += 4) {
            const float4 v = *reinterpret_cast<const float4*>(p + k);
            d[k] = v.x; d[k + 1] = v.y; d[k + 2] = v.z; d[k + 3] = v.w;
        }
#pragma unroll
        for (int k = N / 4 * 4; k < N; ++k) d[k] = p[k];
    } else {
#pragma unroll
        for (int k = 0; k < N; ++k) d[k] = p[k];
    }
}

// PAT (entry pattern): 0 any table (per-entry bit tests); 1 the canonical
// half-plane table of radius R = tab.Rx <= DYMAX (every dx in [-R, R] with
// dy = 1..R, all with mirror terms, plus (dx, 0) for dx >= 0 with a mirror
// term for dx > 0), so whether an entry exists and has a mirror term is a
// uniform test of the compile-time dy against R (or of dx for dy = 0);
// 2 the same table with R = DYMAX, where only the dy = 0 test is left.
template <typename T, int NC, int DYMIN, int DYMAX, int PAT>
__global__ void __launch_bounds__(NT)
acc_gw_kernel(const T* __restrict__ x, const float* __restrict__ gU,
              const float* __restrict__ gZ, T* __restrict__ gw, const GwTable tab,
              const GwGeo g) {
    constexpr int NDY = DYMAX - DYMIN + 1;
    constexpr int NWIN = NDY + V - 1;
    extern __shared__ __align__(16) float smem_f[];
    const int XH = g.XH, XW = g.XW, plane = XH * XW;
    float* sx = smem_f;                 // [NC][XH][XW] x, circular
    float* sg = sx + NC * plane;        // [NC][XH][XW] grad_U, zero outside
    float* sz = sg + NC * plane;        // [XH][XW] sum_c grad_Z, zero outside
    const int Rx = tab.Rx;
    const int64_t HW = g.H * g.W;
    const int64_t cgroups = g.Cw == 1 ? 1 : g.C;
    const int64_t grp = blockIdx.y;
    const int64_t b = grp / cgroups;
    const int64_t c0 = g.Cw == 1 ? 0 : grp % cgroups;
    const int ty = blockIdx.x / g.tiles_x, tx = blockIdx.x - ty * g.tiles_x;
    const int64_t h0 = static_cast<int64_t>(ty) * TH, w0 = static_cast<int64_t>(tx) * TW;

    // ---- stage: one warp per staged row at a time, lanes along the row
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = warp; r < XH; r += NT / 32) {
        const int64_t gh = h0 - Rx + r;
        const bool rin = gh >= 0 && gh < g.H;
        int64_t hw = gh % g.H;                       // circular row of x
        if (hw < 0) hw += g.H;
        for (int cc = lane; cc < XW; cc += 32) {
            const int e = r * XW + cc;
            const int64_t gc = w0 - g.CO + cc;
            const bool in = rin && gc >= 0 && gc < g.W;
            int64_t cw = gc;                          // circular column of x
            while (cw < 0) cw += g.W;
            while (cw >= g.W) cw -= g.W;
            const int64_t ow = hw * g.W + cw;
            const int64_t oi = in ? gh * g.W + gc : 0;
            float zs = 0.f;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int64_t pl = (b * g.C + c0 + c) * HW;
                sx[c * plane + e] = to_f(x[pl + ow]);
                sg[c * plane + e] = in ? gU[pl + oi] : 0.f;
                zs += in ? gZ[pl + oi] : 0.f;
            }
            sz[e] = zs;
        }
    }
    __syncthreads();

    const int tr = threadIdx.x / TPR, tc = threadIdx.x % TPR;
    const int64_t h = h0 + tr, wc0 = w0 + tc * V;
    if (h >= g.H || wc0 >= g.W) return;
    const int own = (tr + Rx) * XW + g.CO + tc * V;   // own pixel 0 in the staged tile
    float zo[V];
#pragma unroll
    for (int i = 0; i < V; ++i) zo[i] = sz[own + i];
    // this thread's grad_w pixels in plane 0; plane s is s * pstride further
    T* const gbase = gw + (b * g.Cw + c0) * HW + h * g.W + wc0;
    const int64_t pstride = g.B * g.Cw * HW;

    for (int dx = -Rx; dx <= Rx; ++dx) {
        // entry / mirror bits of this dx row, bit j = dy - DYMIN
        const uint32_t pres = static_cast<uint32_t>(tab.present[dx + MAXR] >> (DYMIN + MAXR));
        if (!pres) continue;
        const uint32_t invm = static_cast<uint32_t>(tab.inv[dx + MAXR] >> (DYMIN + MAXR));
        // entry j (dy = DYMIN + j) present / with a mirror term
        auto has = [&](auto jc) -> bool {
            constexpr int j = decltype(jc)::value;
            if constexpr (PAT == 2) return j > 0 || dx >= 0;
            else if constexpr (PAT == 1) return j > 0 ? j <= Rx : dx >= 0;
            else return (pres >> j) & 1u;
        };
        auto mir = [&](auto jc) -> bool {
            constexpr int j = decltype(jc)::value;
            if constexpr (PAT == 2) return j > 0 || dx > 0;
            else if constexpr (PAT == 1) return j > 0 ? j <= Rx : dx > 0;
            else return (invm >> j) & 1u;
        };
        float acc[NDY][V];
#pragma unroll
        for (int j = 0; j < NDY; ++j)
#pragma unroll
            for (int i = 0; i < V; ++i) acc[j][i] = 0.f;
        const int wrow = own + dx * XW + DYMIN;      // window element 0: q + (dx, DYMIN)
#pragma unroll 1
        for (int c = 0; c < NC; ++c) {
            float xw[NWIN], gwn[NWIN], xo[V], go[V];
            load_row<NWIN, DYMIN % 4 == 0>(xw, sx + c * plane + wrow);
            load_row<NWIN, DYMIN % 4 == 0>(gwn, sg + c * plane + wrow);
            load_row<V, true>(xo, sx + c * plane + own);
            load_row<V, true>(go, sg + c * plane + own);
            sfor<0, NDY>([&](auto jc) {
                constexpr int j = decltype(jc)::value;
                if (!has(jc)) return;
                if (mir(jc)) {
#pragma unroll
                    for (int i = 0; i < V; ++i)
                        acc[j][i] = fmaf(xo[i], gwn[j + i], fmaf(go[i], xw[j + i], acc[j][i]));
                } else {
#pragma unroll
                    for (int i = 0; i < V; ++i) acc[j][i] = fmaf(go[i], xw[j + i], acc[j][i]);
                }
            });
        }
        float zw[NWIN];
        load_row<NWIN, DYMIN % 4 == 0>(zw, sz + wrow);
        sfor<0, NDY>([&](auto jc) {
            constexpr int j = decltype(jc)::value;
            if (!has(jc)) return;
            const bool iv = mir(jc);
            float v[V];
#pragma unroll
            for (int i = 0; i < V; ++i) v[i] = acc[j][i] + zo[i] + (iv ? zw[j + i] : 0.f);
            const int s = tab.s[dx + MAXR][DYMIN + j + MAXR];
            store4<T>(gbase + s * pstride, v);
        });
    }
}

// 4 weights of plane `ws` at image row `row`, columns c0 .. c0 + 3 (c0 may
// be negative or reach past W: circular), as fp32.  OFF = c0 mod 4 is a
// compile-time fact of the caller (c0 = thread column - dy); interior
// threads use one or two aligned 8-byte loads.
template <typename T, int OFF>
__device__ __forceinline__ void load_w4(float (&d)[V], const T* ws, int64_t row,
                                        int64_t c0, int64_t W) {
    const T* r = ws + row * W;
    if (sizeof(T) == 2 && c0 >= 0 && c0 + 8 <= W) {
        const int64_t a = c0 - OFF;                 // multiple of 4
        T e[8];
        *reinterpret_cast<uint2*>(e) = __ldg(reinterpret_cast<const uint2*>(r + a));
        if constexpr (OFF != 0)
            *reinterpret_cast<uint2*>(e + 4) = __ldg(reinterpret_cast<const uint2*>(r + a + 4));
#pragma unroll
        for (int i = 0; i < V; ++i) d[i] = to_f(e[OFF + i]);
    } else if (sizeof(T) == 4 && OFF == 0 && c0 >= 0 && c0 + 4 <= W) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(r + c0));
        d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
    } else {
#pragma unroll
        for (int i = 0; i < V; ++i) {
            int64_t c = c0 + i;
            while (c < 0) c += W;
            while (c >= W) c -= W;
            d[i] = to_f(__ldg(r + c));
        }
    }
}

// grad_x of accumulate_uz (the transpose of the forward operator):
//   gx_c(q) = sum_s w_s(q - d) gU_c(q - d)                  (circular)
//           + inv [q + d inside] w_s(q) gU_c(q + d)
// Same tile and thread layout as the grad_w kernel.  grad_U is staged twice
// with its halo: circular (first term) and zero outside the image (second
// term's inside test).  Per dx row each thread holds the grad_U windows of
// its 4 pixels for every channel; per shift it reads its 4 weights at q
// and the 4 at q - d straight from global memory (neighbouring tiles read
// the same rows, so the re-reads are L2 hits) and accumulates in registers.
template <typename T, int NC, int DYMIN, int DYMAX>
__global__ void __launch_bounds__(NT)
acc_gx_kernel(const T* __restrict__ w, const float* __restrict__ gU,
              float* __restrict__ gx, const GwTable tab, const GwGeo g) {
    constexpr int NDY = DYMAX - DYMIN + 1;
    constexpr int NWIN = NDY + V - 1;
    extern __shared__ __align__(16) float smem_f[];
    const int XH = g.XH, XW = g.XW, plane = XH * XW;
    float* sc = smem_f;                 // [NC][XH][XW] grad_U, circular
    float* sm = sc + NC * plane;        // [NC][XH][XW] grad_U, zero outside
    const int Rx = tab.Rx;
    const int64_t HW = g.H * g.W;
    const int64_t cgroups = g.Cw == 1 ? 1 : g.C;
    const int64_t grp = blockIdx.y;
    const int64_t b = grp / cgroups;
    const int64_t c0 = g.Cw == 1 ? 0 : grp % cgroups;
    const int ty = blockIdx.x / g.tiles_x, tx = blockIdx.x - ty * g.tiles_x;
    const int64_t h0 = static_cast<int64_t>(ty) * TH, w0 = static_cast<int64_t>(tx) * TW;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = warp; r < XH; r += NT / 32) {
        const int64_t gh = h0 - Rx + r;
        const bool rin = gh >= 0 && gh < g.H;
        int64_t hw = gh % g.H;
        if (hw < 0) hw += g.H;
        for (int cc = lane; cc < XW; cc += 32) {
            const int e = r * XW + cc;
            const int64_t gc = w0 - g.CO + cc;
            const bool in = rin && gc >= 0 && gc < g.W;
            int64_t cw = gc;
            while (cw < 0) cw += g.W;
            while (cw >= g.W) cw -= g.W;
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                const int64_t pl = (b * g.C + c0 + c) * HW;
                const float v = gU[pl + hw * g.W + cw];
                sc[c * plane + e] = v;
                sm[c * plane + e] = in ? v : 0.f;
            }
        }
    }
    __syncthreads();

    const int tr = threadIdx.x / TPR, tc = threadIdx.x % TPR;
    const int64_t h = h0 + tr, wc0 = w0 + tc * V;
    if (h >= g.H || wc0 >= g.W) return;
    const int own = (tr + Rx) * XW + g.CO + tc * V;
    const T* const wbase = w + (b * g.Cw + (g.Cw == 1 ? 0 : c0)) * HW;
    const int64_t pstride = g.B * g.Cw * HW;
    float acc[NC][V];
#pragma unroll
    for (int c = 0; c < NC; ++c)
#pragma unroll
        for (int i = 0; i < V; ++i) acc[c][i] = 0.f;

    for (int dx = -Rx; dx <= Rx; ++dx) {
        const uint32_t pres = static_cast<uint32_t>(tab.present[dx + MAXR] >> (DYMIN + MAXR));
        if (!pres) continue;
        const uint32_t invm = static_cast<uint32_t>(tab.inv[dx + MAXR] >> (DYMIN + MAXR));
        int64_t hm = (h - dx) % g.H;            // row of q - d, circular
        if (hm < 0) hm += g.H;
        // windows: A = grad_U(q - d) over dy (circular), B = grad_U(q + d) (masked)
        float wa[NC][NWIN], wb[NC][NWIN];
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            load_row<NWIN, false>(wa[c], sc + c * plane + own - dx * XW - DYMAX);
            load_row<NWIN, DYMIN % 4 == 0>(wb[c], sm + c * plane + own + dx * XW + DYMIN);
        }
        sfor<0, NDY>([&](auto jc) {
            constexpr int j = decltype(jc)::value;
            constexpr int dy = DYMIN + j;
            if (!((pres >> j) & 1u)) return;
            const int s = tab.s[dx + MAXR][dy + MAXR];
            const T* ws = wbase + s * pstride;
            float wm[V];
            load_w4<T, ((-dy) % 4 + 4) % 4>(wm, ws, hm, wc0 - dy, g.W);
#pragma unroll
            for (int c = 0; c < NC; ++c)
#pragma unroll
                for (int i = 0; i < V; ++i)
                    acc[c][i] = fmaf(wm[i], wa[c][i - dy + DYMAX], acc[c][i]);
            if ((invm >> j) & 1u) {
                float wq[V];
                load_w4<T, 0>(wq, ws, h, wc0, g.W);
#pragma unroll
                for (int c = 0; c < NC; ++c)
#pragma unroll
                    for (int i = 0; i < V; ++i)
                        acc[c][i] = fmaf(wq[i], wb[c][j + i], acc[c][i]);
            }
        });
    }
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        float* dst = gx + (b * g.C + c0 + c) * HW + h * g.W + wc0;
        *reinterpret_cast<float4*>(dst) = make_float4(acc[c][0], acc[c][1], acc[c][2], acc[c][3]);
    }
}

template <typename T, int NC, int LO, int HI, int PAT>
bool launch(const void* x, const void* gU, const void* gZ, void* gw, const GwTable& tab,
            const GwGeo& g, size_t smem, dim3 grid, cudaStream_t stream) {
    auto k = acc_gw_kernel<T, NC, LO, HI, PAT>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    k<<<grid, NT, smem, stream>>>(static_cast<const T*>(x), static_cast<const float*>(gU),
                                  static_cast<const float*>(gZ), static_cast<T*>(gw), tab, g);
    return true;
}

template <typename T, int NC>
bool by_range(int pat, int lo, int hi, const void* x, const void* gU, const void* gZ,
              void* gw, const GwTable& tab, const GwGeo& g, size_t smem, dim3 grid,
              cudaStream_t st) {
#define NSC_GW(L, H)                                                                   \
    if (lo == L && hi == H)                                                          \
        return pat == 2 ? launch<T, NC, L, H, 2>(x, gU, gZ, gw, tab, g, smem, grid, st) \
             : pat == 1 ? launch<T, NC, L, H, 1>(x, gU, gZ, gw, tab, g, smem, grid, st) \
                        : launch<T, NC, L, H, 0>(x, gU, gZ, gw, tab, g, smem, grid, st);
    NSC_GW(0, 2) NSC_GW(0, 4) NSC_GW(0, 6) NSC_GW(0, 8) NSC_GW(0, 10) NSC_GW(0, 12)
#undef NSC_GW
    // tables reaching negative dy are never canonical half-plane tables
    if (lo == -4 && hi == 4) return launch<T, NC, -4, 4, 0>(x, gU, gZ, gw, tab, g, smem, grid, st);
    if (lo == -6 && hi == 6) return launch<T, NC, -6, 6, 0>(x, gU, gZ, gw, tab, g, smem, grid, st);
    return false;
}

template <typename T, int NC, int LO, int HI>
bool launch_gx(const void* w, const void* gU, void* gx, const GwTable& tab,
               const GwGeo& g, size_t smem, dim3 grid, cudaStream_t stream) {
    auto k = acc_gx_kernel<T, NC, LO, HI>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    k<<<grid, NT, smem, stream>>>(static_cast<const T*>(w), static_cast<const float*>(gU),
                                  static_cast<float*>(gx), tab, g);
    return true;
}

template <typename T, int NC>
bool gx_by_range(int lo, int hi, const void* w, const void* gU, void* gx,
                 const GwTable& tab, const GwGeo& g, size_t smem, dim3 grid,
                 cudaStream_t st) {
#define NSC_GX(L, H) \
    if (lo == L && hi == H) return launch_gx<T, NC, L, H>(w, gU, gx, tab, g, smem, grid, st);
    NSC_GX(0, 2) NSC_GX(0, 4) NSC_GX(0, 6) NSC_GX(0, 8) NSC_GX(0, 10) NSC_GX(0, 12)
    NSC_GX(-4, 4) NSC_GX(-6, 6)
#undef NSC_GX
    return false;
}

inline bool dispatch(int xd, int NC, int exact, int lo, int hi, const void* x,
                     const void* gU, const void* gZ, void* gw, const GwTable& tab,
                     const GwGeo& g, size_t smem, dim3 grid, cudaStream_t st) {
    if (xd == NSC_F16)
        return NC == 3 ? by_range<__half, 3>(exact, lo, hi, x, gU, gZ, gw, tab, g, smem, grid, st)
                       : by_range<__half, 1>(exact, lo, hi, x, gU, gZ, gw, tab, g, smem, grid, st);
    if (xd == NSC_BF16)
        return NC == 3 ? by_range<__nv_bfloat16, 3>(exact, lo, hi, x, gU, gZ, gw, tab, g, smem, grid, st)
                       : by_range<__nv_bfloat16, 1>(exact, lo, hi, x, gU, gZ, gw, tab, g, smem, grid, st);
    return NC == 3 ? by_range<float, 3>(exact, lo, hi, x, gU, gZ, gw, tab, g, smem, grid, st)
                   : by_range<float, 1>(exact, lo, hi, x, gU, gZ, gw, tab, g, smem, grid, st);
}

}  // namespace gwk

// Tiled grad_w; returns false (nothing launched) when the call is outside
// what it handles.
namespace {

// Table and geometry shared by the tiled grad_w and grad_x kernels; false
// when the call is outside what they handle.
bool prepare(int xd, int wd, int64_t Cw, int64_t B, int64_t C, int64_t H, int64_t W,
             const ShiftTable& st, std::initializer_list<const void*> ptrs,
             gwk::GwTable* tab, gwk::GwGeo* g, int* lo, int* hi) {
    using namespace gwk;
    if (std::getenv("NSC_DISABLE_FAST")) return false;
    if (xd != wd || xd == NSC_F64) return false;
    if (!(Cw == C || (Cw == 1 && (C == 1 || C == 3)))) return false;
    if (W % V != 0) return false;
    for (const void* p : ptrs)
        if (reinterpret_cast<uintptr_t>(p) % 16 != 0) return false;
    if (B * (Cw == 1 ? 1 : C) > 65535) return false;
    std::memset(tab, 0, sizeof(*tab));
    for (auto& r : tab->s)
        for (auto& v : r) v = -1;
    int dymin = MAXR, dymax = -MAXR, rx = 0;
    for (int s = 0; s < st.S; ++s) {
        const int dx = st.dx[s], dy = st.dy[s];
        if (dx < -MAXR || dx > MAXR || dy < -MAXR || dy > MAXR) return false;
        if (!st.has_fwd(s) || st.has_per(s)) return false;   // transposed / periodic rows
        if (tab->s[dx + MAXR][dy + MAXR] >= 0) return false; // repeated shift
        tab->s[dx + MAXR][dy + MAXR] = static_cast<int16_t>(s);
        tab->present[dx + MAXR] |= 1ull << (dy + MAXR);
        if (st.has_inv(s)) tab->inv[dx + MAXR] |= 1ull << (dy + MAXR);
        dymin = dy < dymin ? dy : dymin;
        dymax = dy > dymax ? dy : dymax;
        rx = (dx < 0 ? -dx : dx) > rx ? (dx < 0 ? -dx : dx) : rx;
    }
    tab->Rx = rx;
    if (dymin >= 0) {
        *lo = 0;
        *hi = dymax <= 2 ? 2 : dymax <= 4 ? 4 : dymax <= 6 ? 6 : dymax <= 8 ? 8
              : dymax <= 10 ? 10 : dymax <= 12 ? 12 : -1;
    } else {
        const int k = dymax > -dymin ? dymax : -dymin;
        *lo = k <= 4 ? -4 : k <= 6 ? -6 : 1;
        *hi = -*lo;
    }
    if (*hi < 0 || *lo > 0) return false;
    *g = GwGeo{};
    g->B = B; g->C = C; g->H = H; g->W = W; g->Cw = Cw;
    g->tiles_x = static_cast<int32_t>((W + TW - 1) / TW);
    g->tiles_y = static_cast<int32_t>((H + TH - 1) / TH);
    if (static_cast<int64_t>(g->tiles_x) * g->tiles_y >= (1LL << 31)) return false;
    g->XH = TH + 2 * rx;
    return true;
}

}  // namespace

bool acc_gw_fast(const void* x, int xd, int wd, int64_t Cw, int64_t B, int64_t C,
                 int64_t H, int64_t W, const ShiftTable& st, const void* gU,
                 const void* gZ, void* gw, cudaStream_t stream) {
    using namespace gwk;
    GwTable tab;
    GwGeo g;
    int lo, hi;
    if (!prepare(xd, wd, Cw, B, C, H, W, st, {x, gU, gZ, gw}, &tab, &g, &lo, &hi))
        return false;
    g.CO = (-lo + 3) / 4 * 4;                 // 16-byte aligned own pixels
    g.XW = (g.CO + TW + hi + 3) / 4 * 4;
    const int NC = Cw == 1 ? static_cast<int>(C) : 1;
    const size_t smem = static_cast<size_t>(2 * NC + 1) * g.XH * g.XW * sizeof(float);
    if (smem > 227u * 1024u) return false;
    const dim3 grid(static_cast<unsigned>(g.tiles_x * g.tiles_y),
                    static_cast<unsigned>(B * (Cw == 1 ? 1 : C)));
    // canonical half-plane table of radius R = tab.Rx <= hi (acc_gw_kernel's
    // PAT 1, or PAT 2 when R == hi): every present / mirror bit as the pattern says, nothing else
    const int R = tab.Rx;
    bool exact = lo == 0 && R >= 1 && R <= hi;
    for (int dx = -R; exact && dx <= R; ++dx) {
        uint64_t pres = 0, mir = 0;
        for (int dy = 0; dy <= R; ++dy) {
            const uint64_t bit = 1ull << (dy + MAXR);
            if (dy > 0 || dx >= 0) pres |= bit;
            if (dy > 0 || dx > 0) mir |= bit;
        }
        exact = tab.present[dx + MAXR] == pres && tab.inv[dx + MAXR] == mir;
    }
    const int pat = std::getenv("NSC_GW_GENERIC") ? 0 : !exact ? 0 : R == hi ? 2 : 1;
    return gwk::dispatch(xd, NC, pat, lo, hi, x, gU, gZ, gw, tab, g, smem, grid, stream);
}

bool acc_gx_fast(const void* w, int xd, int wd, int64_t Cw, int64_t B, int64_t C,
                 int64_t H, int64_t W, const ShiftTable& st, const void* gU, void* gx,
                 cudaStream_t stream) {
    using namespace gwk;
    // the TMA kernel first; NSC_GX_LEGACY selects the kernel below, and
    // NSC_REQUIRE_FAST (a test switch) makes a decline of the TMA kernel fail
    if (!std::getenv("NSC_GX_LEGACY")) {
        if (acc_gx_tma(w, wd, Cw, B, C, H, W, st, gU, gx, stream)) return true;
        if (std::getenv("NSC_REQUIRE_FAST")) return false;
    }
    GwTable tab;
    GwGeo g;
    int lo, hi;
    if (!prepare(xd, wd, Cw, B, C, H, W, st, {w, gU, gx}, &tab, &g, &lo, &hi))
        return false;
    const int K = hi > -lo ? hi : -lo;        // windows reach q - d and q + d
    g.CO = (K + 3) / 4 * 4;
    g.XW = (g.CO + TW + K + 3) / 4 * 4;
    const int NC = Cw == 1 ? static_cast<int>(C) : 1;
    const size_t smem = static_cast<size_t>(2 * NC) * g.XH * g.XW * sizeof(float);
    if (smem > 227u * 1024u) return false;
    const dim3 grid(static_cast<unsigned>(g.tiles_x * g.tiles_y),
                    static_cast<unsigned>(B * (Cw == 1 ? 1 : C)));
    if (xd == NSC_F16)
        return NC == 3 ? gx_by_range<__half, 3>(lo, hi, w, gU, gx, tab, g, smem, grid, stream)
                       : gx_by_range<__half, 1>(lo, hi, w, gU, gx, tab, g, smem, grid, stream);
    if (xd == NSC_BF16)
        return NC == 3 ? gx_by_range<__nv_bfloat16, 3>(lo, hi, w, gU, gx, tab, g, smem, grid, stream)
                       : gx_by_range<__nv_bfloat16, 1>(lo, hi, w, gU, gx, tab, g, smem, grid, stream);
    return NC == 3 ? gx_by_range<float, 3>(lo, hi, w, gU, gx, tab, g, smem, grid, stream)
                   : gx_by_range<float, 1>(lo, hi, w, gU, gx, tab, g, smem, grid, stream);
}

}  // namespace nsc
