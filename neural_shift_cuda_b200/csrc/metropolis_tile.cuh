// metropolis_tile.cuh -- tiled forms of the four Metropolis kernels
// (degree, aggregation, backward passes A and B) for shift tables of radius
// R <= 8.  The quantities are those of the one-pixel kernels of
// metropolis.cu (see the formulas there); what changes is where operands
// come from and how the denominators are formed.
//
// A CTA (32 x 8 threads, two pixels per thread) owns a 16 x 32 tile of one
// (image, weight channel) group.  Every per-pixel quantity an edge reads at
// a neighbour is staged once, with a circular R-pixel halo, in shared
// memory in the accumulator type; an edge reads its neighbour at the
// constant offset dx * pitch + dy.  Staged planes:
//   r(p) = 1 / max(d(p), eps)      (so 1 / den_e(p) = min(r(p), r(p + delta)):
//                                   max and round-to-nearest are monotonic,
//                                   hence exact; one division per staged
//                                   pixel instead of one per edge)
//   d(p), image channels, grad_Wx, and the per-pixel backward term
//   a(p) = sum_c gdh(p, c) - gWx(p, c) x(p, c).
// Weight planes are read straight from global memory: w_s(q) coalesced
// along the row, the mirror weight w_s(q - d) one row and column away
// (L1/L2).  Tiles whose R-halo lies inside the image take a branch-free
// form: no box masks and no wrapped addresses.  In-plane indexing is
// 32-bit.
#pragma once

#include <cstdint>
#include <type_traits>

#include "nsc_common.cuh"

namespace nsc {
namespace mtile {

#ifndef NSC_METRO_PPT
#define NSC_METRO_PPT 2
#endif
constexpr int TX = 32, TY = 8, PPT = NSC_METRO_PPT;   // pixels per thread (rows TY apart)
constexpr int TH = TY * PPT, TW = TX;
constexpr int NT = TX * TY;
constexpr int MAXR = 8;

struct Geo {
    int B, C, Cw, H, W, S, R;
    int XP, XR;                 // halo tile pitch and rows
    int tiles_x;
    int64_t ntiles, groups;
};

__device__ __forceinline__ int pmod(int a, int n) {
    const int r = a % n;
    return r < 0 ? r + n : r;
}
__device__ __forceinline__ int wrapc(int i, int n) {   // |i - [0,n)| <= n
    return i < 0 ? i + n : (i >= n ? i - n : i);
}

// Visits every element (idx, global offset) of the halo tile.
template <typename F>
__device__ __forceinline__ void for_halo(const Geo& g, int h0, int w0, F&& f) {
    const int tid = threadIdx.y * TX + threadIdx.x;
    for (int idx = tid; idx < g.XR * g.XP; idx += NT) {
        const int i = idx / g.XP;
        const int j = idx - i * g.XP;
        const int r = pmod(h0 - g.R + i, g.H);
        const int c = pmod(w0 - g.R + j, g.W);
        f(idx, static_cast<int64_t>(r) * g.W + c);
    }
}

template <typename A>
__device__ __forceinline__ A share_of(A self, A other) {
    return self > other ? A(1) : (self == other ? A(0.5) : A(0));
}
__device__ __forceinline__ float amin(float a, float b) { return fminf(a, b); }
__device__ __forceinline__ double amin(double a, double b) { return fmin(a, b); }

struct Where {
    int b, wc, c0, h0, w0;
    bool interior;   // tile + R halo inside the image
};
__device__ __forceinline__ Where where(const Geo& g, int64_t tile, int64_t grp) {
    Where o;
    o.b = static_cast<int>(grp / g.Cw);
    o.wc = static_cast<int>(grp - static_cast<int64_t>(o.b) * g.Cw);
    o.c0 = (g.Cw == 1) ? 0 : o.wc;
    const int ty = static_cast<int>(tile / g.tiles_x);
    o.h0 = ty * TH;
    o.w0 = static_cast<int>(tile - static_cast<int64_t>(ty) * g.tiles_x) * TW;
    o.interior = o.h0 - g.R >= 0 && o.h0 + TH + g.R <= g.H && o.w0 - g.R >= 0 &&
                 o.w0 + TW + g.R <= g.W;
    return o;
}

// Per-shift weight addresses of one pixel: own w_s(q) and mirror w_s(q - d)
// offsets inside the (b, s, wc) plane, and the box flags.
struct EdgeGeom {
    int64_t q, m;
    bool in_p, in_m;
};
template <bool BORDER>
__device__ __forceinline__ EdgeGeom edge_geom(const Geo& g, int h, int w, int dx, int dy) {
    EdgeGeom e;
    e.q = static_cast<int64_t>(h) * g.W + w;
    if constexpr (BORDER) {
        e.m = static_cast<int64_t>(wrapc(h - dx, g.H)) * g.W + wrapc(w - dy, g.W);
        e.in_p = static_cast<unsigned>(h + dx) < static_cast<unsigned>(g.H) &&
                 static_cast<unsigned>(w + dy) < static_cast<unsigned>(g.W);
        e.in_m = static_cast<unsigned>(h - dx) < static_cast<unsigned>(g.H) &&
                 static_cast<unsigned>(w - dy) < static_cast<unsigned>(g.W);
    } else {
        e.m = e.q - (static_cast<int64_t>(dx) * g.W + dy);
        e.in_p = e.in_m = true;
    }
    return e;
}

// Per-pixel records of the staged halo: the quantities one edge reads at a
// neighbour sit together, so a neighbour costs one address and a few
// 16-byte loads.  Records are padded to 16 bytes.
template <typename A>
__host__ __device__ constexpr int rec_len(int n) {
    return sizeof(A) == 4 ? (n + 3) / 4 * 4 : (n + 1) / 2 * 2;
}
template <typename A, int F>
struct alignas(16) Rec {
    A f[F];
};
// aggregation: r, x[NC]
template <typename A, int NC> constexpr int kAggF = rec_len<A>(1 + NC);
// backward A: d, r, a, x[NC], gWx[NC]
template <typename A, int NC> constexpr int kBwdAF = rec_len<A>(3 + 2 * NC);
// backward B: d, r, a, g_d, x[NC], gWx[NC]
template <typename A, int NC> constexpr int kBwdBF = rec_len<A>(4 + 2 * NC);

// Packed fp32 pairs: the two pixels a thread owns (rows TY apart) run as
// the two lanes of sm_100's f32x2 arithmetic, one instruction per pair.
__device__ __forceinline__ float2 f2fma(float2 a, float2 b, float2 c) {
    float2 r;
    asm("{.reg .b64 a,b,c,d; mov.b64 a,{%2,%3}; mov.b64 b,{%4,%5}; mov.b64 c,{%6,%7};"
        " fma.rn.f32x2 d,a,b,c; mov.b64 {%0,%1},d;}"
        : "=f"(r.x), "=f"(r.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return r;
}
__device__ __forceinline__ float2 f2mul(float2 a, float2 b) {
    float2 r;
    asm("{.reg .b64 a,b,d; mov.b64 a,{%2,%3}; mov.b64 b,{%4,%5};"
        " mul.rn.f32x2 d,a,b; mov.b64 {%0,%1},d;}"
        : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}
__device__ __forceinline__ float2 f2add(float2 a, float2 b) {
    float2 r;
    asm("{.reg .b64 a,b,d; mov.b64 a,{%2,%3}; mov.b64 b,{%4,%5};"
        " add.rn.f32x2 d,a,b; mov.b64 {%0,%1},d;}"
        : "=f"(r.x), "=f"(r.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return r;
}
// ---------------------------------------------------------------- degree
template <typename T>
__global__ void __launch_bounds__(NT)
degree_tile(const T* __restrict__ w, typename Acc<T>::type* __restrict__ d,
            const ShiftTable st, const Geo g, int use_box) {
    using A = typename Acc<T>::type;
    const int64_t HW = static_cast<int64_t>(g.H) * g.W;
    const int64_t sstride = static_cast<int64_t>(g.Cw) * HW;
    for (int64_t grp = blockIdx.y; grp < g.groups; grp += gridDim.y) {
        for (int64_t tile = blockIdx.x; tile < g.ntiles; tile += gridDim.x) {
            const Where o = where(g, tile, grp);
            const int wcol = o.w0 + threadIdx.x;
            if (wcol >= g.W) continue;
            int hh[PPT];
            A acc[PPT];
#pragma unroll
            for (int p = 0; p < PPT; ++p) {
                const int h = o.h0 + threadIdx.y + TY * p;
                hh[p] = h < g.H ? h : g.H - 1;   // loads stay in bounds
                acc[p] = A(0);
            }
            const T* wb = w + (static_cast<int64_t>(o.b) * g.S * g.Cw + o.wc) * HW;
            auto body = [&](auto border) {
                constexpr bool BORDER = decltype(border)::value;
#pragma unroll 4
                for (int s = 0; s < g.S; ++s) {
                    const int dx = st.dx[s], dy = st.dy[s];
                    const bool inv = st.has_inv(s);
                    const T* ws = wb + s * sstride;
                    if constexpr (std::is_same_v<A, float> && PPT == 2) {
                        // fp32: both pixels' sums as one f32x2 add per term
                        // (a masked term adds +0, which leaves every sum as is)
                        const EdgeGeom e0 = edge_geom<BORDER>(g, hh[0], wcol, dx, dy);
                        const EdgeGeom e1 = edge_geom<BORDER>(g, hh[1], wcol, dx, dy);
                        float2 wq = make_float2(ldg_acc<T, float>(ws + e0.q),
                                                ldg_acc<T, float>(ws + e1.q));
                        float2 wm = make_float2(ldg_acc<T, float>(ws + e0.m),
                                                ldg_acc<T, float>(ws + e1.m));
                        if (BORDER && use_box) {
                            if (!e0.in_p) wq.x = 0.f;
                            if (!e1.in_p) wq.y = 0.f;
                            if (!e0.in_m) wm.x = 0.f;
                            if (!e1.in_m) wm.y = 0.f;
                        }
                        float2 a2 = f2add(make_float2(acc[0], acc[1]), wq);
                        if (inv) a2 = f2add(a2, wm);
                        acc[0] = a2.x;
                        acc[1] = a2.y;
                    } else {
#pragma unroll
                        for (int p = 0; p < PPT; ++p) {
                            const EdgeGeom e = edge_geom<BORDER>(g, hh[p], wcol, dx, dy);
                            const A wq = ldg_acc<T, A>(ws + e.q);
                            const A wm = ldg_acc<T, A>(ws + e.m);
                            if (!use_box || e.in_p) acc[p] += wq;
                            if (inv && (!use_box || e.in_m)) acc[p] += wm;
                        }
                    }
                }
            };
            if (o.interior) body(std::false_type{});
            else body(std::true_type{});
#pragma unroll
            for (int p = 0; p < PPT; ++p) {
                const int h = o.h0 + threadIdx.y + TY * p;
                if (h < g.H) d[grp * HW + static_cast<int64_t>(h) * g.W + wcol] = acc[p];
            }
        }
    }
}

// ----------------------------------------------------------- aggregation
template <typename T, int NC>
__global__ void __launch_bounds__(NT)
aggregate_tile(const T* __restrict__ w, const T* __restrict__ x,
               const typename Acc<T>::type* __restrict__ d, T* __restrict__ Wx,
               T* __restrict__ dhat, const ShiftTable st, const Geo g, int use_box,
               typename Acc<T>::type eps) {
    using A = typename Acc<T>::type;
    constexpr int F = kAggF<A, NC>;
    extern __shared__ __align__(16) unsigned char smem_m[];
    Rec<A, F>* rec = reinterpret_cast<Rec<A, F>*>(smem_m);   // r, x[NC]
    const int64_t HW = static_cast<int64_t>(g.H) * g.W;
    const int64_t sstride = static_cast<int64_t>(g.Cw) * HW;
    for (int64_t grp = blockIdx.y; grp < g.groups; grp += gridDim.y) {
        for (int64_t tile = blockIdx.x; tile < g.ntiles; tile += gridDim.x) {
            const Where o = where(g, tile, grp);
            const int64_t cb = (static_cast<int64_t>(o.b) * g.C + o.c0) * HW;
            __syncthreads();
            const A* dg = d + grp * HW;
            for_halo(g, o.h0, o.w0, [&](int idx, int64_t off) {
                const A dv = dg[off];
                Rec<A, F> r;
#pragma unroll
                for (int k = 0; k < F; ++k) r.f[k] = A(0);
                r.f[0] = A(1) / (dv > eps ? dv : eps);
#pragma unroll
                for (int c = 0; c < NC; ++c)
                    r.f[1 + c] = static_cast<A>(to_acc(x[cb + c * HW + off]));
                rec[idx] = r;
            });
            __syncthreads();
            const int wcol = o.w0 + threadIdx.x;
            if (wcol >= g.W) continue;
            const T* wb = w + (static_cast<int64_t>(o.b) * g.S * g.Cw + o.wc) * HW;
            int hh[PPT], ci[PPT];
            A ri[PPT], kx[PPT][NC], dh[PPT];
#pragma unroll
            for (int p = 0; p < PPT; ++p) {
                const int h = o.h0 + threadIdx.y + TY * p;
                hh[p] = h < g.H ? h : g.H - 1;
                ci[p] = (threadIdx.y + TY * p + g.R) * g.XP + threadIdx.x + g.R;
                ri[p] = rec[ci[p]].f[0];
                dh[p] = A(0);
#pragma unroll
                for (int c = 0; c < NC; ++c) kx[p][c] = A(0);
            }
            auto body = [&](auto border) {
                constexpr bool BORDER = decltype(border)::value;
#pragma unroll 2
                for (int s = 0; s < g.S; ++s) {
                    const int dx = st.dx[s], dy = st.dy[s];
                    const bool inv = st.has_inv(s);
                    const int off = dx * g.XP + dy;
                    const T* ws = wb + s * sstride;
#pragma unroll
                    for (int p = 0; p < PPT; ++p) {
                        const EdgeGeom e = edge_geom<BORDER>(g, hh[p], wcol, dx, dy);
                        const A wq = ldg_acc<T, A>(ws + e.q);
                        const A wm = ldg_acc<T, A>(ws + e.m);
                        if (!use_box || e.in_p) {
                            const Rec<A, F> nb = rec[ci[p] + off];
                            const A wk = wq * amin(ri[p], nb.f[0]);
#pragma unroll
                            for (int c = 0; c < NC; ++c) kx[p][c] += wk * nb.f[1 + c];
                            dh[p] += wk;
                        }
                        if (inv && (!use_box || e.in_m)) {
                            const Rec<A, F> nb = rec[ci[p] - off];
                            const A wk = wm * amin(ri[p], nb.f[0]);
#pragma unroll
                            for (int c = 0; c < NC; ++c) kx[p][c] += wk * nb.f[1 + c];
                            dh[p] += wk;
                        }
                    }
                }
            };
            if (o.interior) body(std::false_type{});
            else body(std::true_type{});
#pragma unroll
            for (int p = 0; p < PPT; ++p) {
                const int h = o.h0 + threadIdx.y + TY * p;
                if (h >= g.H) continue;
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const int64_t oi = cb + c * HW + static_cast<int64_t>(h) * g.W + wcol;
                    const A xv = rec[ci[p]].f[1 + c];
                    const A dhx = dh[p] * xv;
                    Wx[oi] = static_cast<T>((xv - dhx) + kx[p][c]);
                    dhat[oi] = static_cast<T>(dh[p]);
                }
            }
        }
    }
}

// Stages one record per halo pixel: d, r = 1/max(d, eps), the per-pixel
// backward term a = sum_c gdh - gWx x (channel order), [g_d,] image
// channels, grad_Wx.  XO: offset of the image channels (3, or 4 with g_d).
template <typename T, int NC, int F, int XO, typename A>
__device__ __forceinline__ void stage_bwd(const Geo& g, const Where& o, int64_t grp,
                                          int64_t cb, int64_t HW, const A* __restrict__ d,
                                          const A* __restrict__ gd,
                                          const T* __restrict__ x, const T* __restrict__ gWx,
                                          const T* __restrict__ gdh, A eps, Rec<A, F>* rec) {
    const A* dg = d + grp * HW;
    for_halo(g, o.h0, o.w0, [&](int idx, int64_t off) {
        Rec<A, F> r;
#pragma unroll
        for (int k = 0; k < F; ++k) r.f[k] = A(0);
        const A dv = dg[off];
        r.f[0] = dv;
        r.f[1] = A(1) / (dv > eps ? dv : eps);
        A a = A(0);
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const A xv = static_cast<A>(to_acc(x[cb + c * HW + off]));
            const A gv = static_cast<A>(to_acc(gWx[cb + c * HW + off]));
            r.f[XO + c] = xv;
            r.f[XO + NC + c] = gv;
            a += static_cast<A>(to_acc(gdh[cb + c * HW + off])) - gv * xv;
        }
        r.f[2] = a;
        if constexpr (XO == 4) r.f[3] = gd[grp * HW + off];
        rec[idx] = r;
    });
}

// ------------------------------------------------------------ backward A
// grad_img and the degree gradient g_d.  Per edge touching q:
//   own edge e at q (neighbour n = q + delta):
//     G = a(q) + sum_c gWx(q) x(n);  g_d(q) -= G wt r^2 share(d(q), d(n))
//   edge of p = q - delta whose neighbour is q (weight wt_p, wk = wt_p r):
//     G = a(p) + sum_c gWx(p) x(q);  g_d(q) -= G wt_p r^2 share(d(q), d(p))
//     gx(q) += gWx(p) wk
// with r = min(r(q), r(other)); g_d terms only where max(d(q), d(other))
// >= eps (clamp_min passes no gradient below eps).  The terms come in pairs
// over one pixel pair {q, n}: same weight, denominator and tie share (the
// own forward edge of q with the mirror edge of q + d, the forward edge of
// q - d with the own mirror edge of q), so each pair is evaluated once.
template <typename T, int NC>
__global__ void __launch_bounds__(NT)
bwd_a_tile(const T* __restrict__ w, const T* __restrict__ x,
           const typename Acc<T>::type* __restrict__ d, const T* __restrict__ dhat,
           const T* __restrict__ gWx, const T* __restrict__ gdh,
           typename Acc<T>::type* __restrict__ gd, T* __restrict__ gx,
           const ShiftTable st, const Geo g, int use_box, typename Acc<T>::type eps) {
    using A = typename Acc<T>::type;
    constexpr int F = kBwdAF<A, NC>;
    constexpr int XO = 3, GO = 3 + NC;
    extern __shared__ __align__(16) unsigned char smem_m[];
    Rec<A, F>* rec = reinterpret_cast<Rec<A, F>*>(smem_m);
    const int64_t HW = static_cast<int64_t>(g.H) * g.W;
    const int64_t sstride = static_cast<int64_t>(g.Cw) * HW;
    for (int64_t grp = blockIdx.y; grp < g.groups; grp += gridDim.y) {
        for (int64_t tile = blockIdx.x; tile < g.ntiles; tile += gridDim.x) {
            const Where o = where(g, tile, grp);
            const int64_t cb = (static_cast<int64_t>(o.b) * g.C + o.c0) * HW;
            __syncthreads();
            stage_bwd<T, NC, F, XO>(g, o, grp, cb, HW, d, static_cast<const A*>(nullptr), x,
                                    gWx, gdh, eps, rec);
            __syncthreads();
            const int wcol = o.w0 + threadIdx.x;
            if (wcol >= g.W) continue;
            const T* wb = w + (static_cast<int64_t>(o.b) * g.S * g.Cw + o.wc) * HW;
            int hh[PPT], ci[PPT];
            A di[PPT], ri[PPT], aq[PPT], xq[PPT][NC], gq[PPT][NC], gxa[PPT][NC], g_d[PPT];
#pragma unroll
            for (int p = 0; p < PPT; ++p) {
                const int h = o.h0 + threadIdx.y + TY * p;
                hh[p] = h < g.H ? h : g.H - 1;
                ci[p] = (threadIdx.y + TY * p + g.R) * g.XP + threadIdx.x + g.R;
                const Rec<A, F> me = rec[ci[p]];
                di[p] = me.f[0];
                ri[p] = me.f[1];
                aq[p] = me.f[2];
                g_d[p] = A(0);
                const int64_t q = static_cast<int64_t>(hh[p]) * g.W + wcol;
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    xq[p][c] = me.f[XO + c];
                    gq[p][c] = me.f[GO + c];
                    gxa[p][c] = gq[p][c] * (A(1) - static_cast<A>(to_acc(dhat[cb + c * HW + q])));
                }
            }
            auto body = [&](auto border) {
                constexpr bool BORDER = decltype(border)::value;
#pragma unroll 1
                for (int s = 0; s < g.S; ++s) {
                    const int dx = st.dx[s], dy = st.dy[s];
                    const bool inv = st.has_inv(s);
                    const int off = dx * g.XP + dy;
                    const T* ws = wb + s * sstride;
#pragma unroll
                    for (int p = 0; p < PPT; ++p) {
                        const EdgeGeom e = edge_geom<BORDER>(g, hh[p], wcol, dx, dy);
                        const A w_q = ldg_acc<T, A>(ws + e.q);
                        const A w_m = ldg_acc<T, A>(ws + e.m);
                        const bool kp = !use_box || e.in_p, km = !use_box || e.in_m;
                        // Pair (q, q + d), weight w_s(q): own forward edge of q
                        // and (inv) the mirror edge of q + d ending at q.
                        if (kp && w_q != A(0)) {
                            const Rec<A, F> nb = rec[ci[p] + off];
                            const A dn = nb.f[0];
                            const A r = amin(ri[p], nb.f[1]);
                            A Tq = aq[p], Tn = A(0);
#pragma unroll
                            for (int c = 0; c < NC; ++c) Tq += gq[p][c] * nb.f[XO + c];
                            if (inv) {
                                const A wk = w_q * r;
                                Tn = nb.f[2];
#pragma unroll
                                for (int c = 0; c < NC; ++c) {
                                    const A gn = nb.f[GO + c];
                                    Tn += gn * xq[p][c];
                                    gxa[p][c] += gn * wk;
                                }
                            }
                            if ((di[p] > dn ? di[p] : dn) >= eps)
                                g_d[p] -= (Tq + Tn) * w_q * r * r * share_of(di[p], dn);
                        }
                        // Pair (q, q - d), weight w_s(q - d): forward edge of
                        // q - d ending at q and (inv) the own mirror edge of q.
                        if (km && w_m != A(0)) {
                            const Rec<A, F> nb = rec[ci[p] - off];
                            const A dn = nb.f[0];
                            const A r = amin(ri[p], nb.f[1]);
                            const A wk = w_m * r;
                            A Tn = nb.f[2], Tq = A(0);
#pragma unroll
                            for (int c = 0; c < NC; ++c) {
                                const A gn = nb.f[GO + c];
                                Tn += gn * xq[p][c];
                                gxa[p][c] += gn * wk;
                            }
                            if (inv) {
                                Tq = aq[p];
#pragma unroll
                                for (int c = 0; c < NC; ++c) Tq += gq[p][c] * nb.f[XO + c];
                            }
                            if ((di[p] > dn ? di[p] : dn) >= eps)
                                g_d[p] -= (Tn + Tq) * w_m * r * r * share_of(di[p], dn);
                        }
                    }
                }
            };
            if (o.interior) body(std::false_type{});
            else body(std::true_type{});
#pragma unroll
            for (int p = 0; p < PPT; ++p) {
                const int h = o.h0 + threadIdx.y + TY * p;
                if (h >= g.H) continue;
                const int64_t q = static_cast<int64_t>(h) * g.W + wcol;
                gd[grp * HW + q] = g_d[p];
#pragma unroll
                for (int c = 0; c < NC; ++c) gx[cb + c * HW + q] = static_cast<T>(gxa[p][c]);
            }
        }
    }
}

// -share(self, other) where the denominator passes gradient (max >= eps),
// else 0: the factor of a pair's degree-gradient term.
__device__ __forceinline__ float neg_share(float self, float other, float eps) {
    if (!((self > other ? self : other) >= eps)) return 0.f;
    return self > other ? -1.f : (self == other ? -0.5f : 0.f);
}

// backward A for fp32 accumulators with the thread's two pixels packed.
// Records hold pixel PAIRS: pair row i of the staged halo holds halo rows i
// and i + TY side by side (field k of both rows in one float2), so the
// neighbour records of both pixels, at the same offset (dx, dy), are one
// record.  Same terms, order and special cases as bwd_a_tile, except that a
// box-masked or zero weight contributes its (zero) products instead of
// being skipped -- identical for finite inputs.
template <int F>
struct alignas(16) PRF {
    float2 f[F];
};
template <int NC> constexpr int kBwdA2F = (3 + 2 * NC + 1) / 2 * 2;  // float2 fields
template <int NC> using PRec = PRF<kBwdA2F<NC>>;

// Stages pixel-pair records over the tile's halo: pair row i holds halo
// rows i and i + TY; fill(off, v) writes the fields of the pixel at plane
// offset off into v[0 .. F).
template <int F, typename Fill>
__device__ __forceinline__ void stage_pairs(const Geo& g, const Where& o, PRF<F>* rec,
                                            Fill&& fill) {
    const int PR = TY + 2 * g.R;
    const int tid = threadIdx.y * TX + threadIdx.x;
    for (int idx = tid; idx < PR * g.XP; idx += NT) {
        const int i = idx / g.XP;
        const int j = idx - i * g.XP;
        const int c = pmod(o.w0 - g.R + j, g.W);
        PRF<F> r;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int64_t off =
                static_cast<int64_t>(pmod(o.h0 - g.R + i + hh * TY, g.H)) * g.W + c;
            float v[F];
#pragma unroll
            for (int k = 0; k < F; ++k) v[k] = 0.f;
            fill(off, v);
#pragma unroll
            for (int k = 0; k < F; ++k) {
                if (hh == 0) r.f[k].x = v[k];
                else r.f[k].y = v[k];
            }
        }
        rec[idx] = r;
    }
}

template <typename T, int NC>
__global__ void __launch_bounds__(NT)
bwd_a_tile_x2(const T* __restrict__ w, const T* __restrict__ x,
              const float* __restrict__ d, const T* __restrict__ dhat,
              const T* __restrict__ gWx, const T* __restrict__ gdh,
              float* __restrict__ gd, T* __restrict__ gx,
              const ShiftTable st, const Geo g, int use_box, float eps) {
    static_assert(PPT == 2, "two pixels per thread");
    constexpr int F = kBwdA2F<NC>;
    constexpr int XO = 3, GO = 3 + NC;
    extern __shared__ __align__(16) unsigned char smem_m[];
    PRec<NC>* rec = reinterpret_cast<PRec<NC>*>(smem_m);
    const int64_t HW = static_cast<int64_t>(g.H) * g.W;
    const int64_t sstride = static_cast<int64_t>(g.Cw) * HW;
    for (int64_t grp = blockIdx.y; grp < g.groups; grp += gridDim.y) {
        for (int64_t tile = blockIdx.x; tile < g.ntiles; tile += gridDim.x) {
            const Where o = where(g, tile, grp);
            const int64_t cb = (static_cast<int64_t>(o.b) * g.C + o.c0) * HW;
            __syncthreads();
            const float* dg = d + grp * HW;
            stage_pairs<F>(g, o, rec, [&](int64_t off, float* v) {
                const float dv = dg[off];
                v[0] = dv;
                v[1] = 1.f / (dv > eps ? dv : eps);
                float a = 0.f;
#pragma unroll
                for (int cc = 0; cc < NC; ++cc) {
                    const float xv = to_acc(x[cb + cc * HW + off]);
                    const float gv = to_acc(gWx[cb + cc * HW + off]);
                    v[XO + cc] = xv;
                    v[GO + cc] = gv;
                    a += to_acc(gdh[cb + cc * HW + off]) - gv * xv;
                }
                v[2] = a;
            });
            __syncthreads();
            const int wcol = o.w0 + threadIdx.x;
            if (wcol >= g.W) continue;
            const T* wb = w + (static_cast<int64_t>(o.b) * g.S * g.Cw + o.wc) * HW;
            int hh[2];
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const int h = o.h0 + threadIdx.y + TY * p;
                hh[p] = h < g.H ? h : g.H - 1;
            }
            const int ci = (threadIdx.y + g.R) * g.XP + threadIdx.x + g.R;
            float2 di, ri, aq, xq[NC], gq[NC], gxa[NC];
            float2 g_d = make_float2(0.f, 0.f);
            {
                const PRec<NC> me = rec[ci];
                di = me.f[0];
                ri = me.f[1];
                aq = me.f[2];
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    xq[c] = me.f[XO + c];
                    gq[c] = me.f[GO + c];
                    const int64_t q0 = static_cast<int64_t>(hh[0]) * g.W + wcol;
                    const int64_t q1 = static_cast<int64_t>(hh[1]) * g.W + wcol;
                    gxa[c] = make_float2(
                        gq[c].x * (1.f - static_cast<float>(to_acc(dhat[cb + c * HW + q0]))),
                        gq[c].y * (1.f - static_cast<float>(to_acc(dhat[cb + c * HW + q1]))));
                }
            }
            auto body = [&](auto border) {
                constexpr bool BORDER = decltype(border)::value;
#pragma unroll 2
                for (int s = 0; s < g.S; ++s) {
                    const int dx = st.dx[s], dy = st.dy[s];
                    const bool inv = st.has_inv(s);
                    const int off = dx * g.XP + dy;
                    const T* ws = wb + s * sstride;
                    const EdgeGeom e0 = edge_geom<BORDER>(g, hh[0], wcol, dx, dy);
                    const EdgeGeom e1 = edge_geom<BORDER>(g, hh[1], wcol, dx, dy);
                    float2 wq = make_float2(ldg_acc<T, float>(ws + e0.q),
                                            ldg_acc<T, float>(ws + e1.q));
                    float2 wm = make_float2(ldg_acc<T, float>(ws + e0.m),
                                            ldg_acc<T, float>(ws + e1.m));
                    if (BORDER && use_box) {
                        if (!e0.in_p) wq.x = 0.f;
                        if (!e1.in_p) wq.y = 0.f;
                        if (!e0.in_m) wm.x = 0.f;
                        if (!e1.in_m) wm.y = 0.f;
                    }
                    // Pair (q, q + d), weight w_s(q): own forward edge of q
                    // and (inv) the mirror edge of q + d ending at q.
                    {
                        const PRec<NC> nb = rec[ci + off];
                        const float2 dn = nb.f[0];
                        const float2 r = make_float2(fminf(ri.x, nb.f[1].x),
                                                     fminf(ri.y, nb.f[1].y));
                        float2 Tq = aq, Tn = make_float2(0.f, 0.f);
#pragma unroll
                        for (int c = 0; c < NC; ++c) Tq = f2fma(gq[c], nb.f[XO + c], Tq);
                        if (inv) {
                            const float2 wk = f2mul(wq, r);
                            Tn = nb.f[2];
#pragma unroll
                            for (int c = 0; c < NC; ++c) {
                                const float2 gn = nb.f[GO + c];
                                Tn = f2fma(gn, xq[c], Tn);
                                gxa[c] = f2fma(gn, wk, gxa[c]);
                            }
                        }
                        const float2 t = f2mul(f2mul(f2mul(f2add(Tq, Tn), wq), r), r);
                        g_d = f2fma(t, make_float2(neg_share(di.x, dn.x, eps),
                                                   neg_share(di.y, dn.y, eps)), g_d);
                    }
                    // Pair (q, q - d), weight w_s(q - d): forward edge of
                    // q - d ending at q and (inv) the own mirror edge of q.
                    {
                        const PRec<NC> nb = rec[ci - off];
                        const float2 dn = nb.f[0];
                        const float2 r = make_float2(fminf(ri.x, nb.f[1].x),
                                                     fminf(ri.y, nb.f[1].y));
                        const float2 wk = f2mul(wm, r);
                        float2 Tn = nb.f[2], Tq = make_float2(0.f, 0.f);
#pragma unroll
                        for (int c = 0; c < NC; ++c) {
                            const float2 gn = nb.f[GO + c];
                            Tn = f2fma(gn, xq[c], Tn);
                            gxa[c] = f2fma(gn, wk, gxa[c]);
                        }
                        if (inv) {
                            Tq = aq;
#pragma unroll
                            for (int c = 0; c < NC; ++c) Tq = f2fma(gq[c], nb.f[XO + c], Tq);
                        }
                        const float2 t = f2mul(f2mul(f2mul(f2add(Tn, Tq), wm), r), r);
                        g_d = f2fma(t, make_float2(neg_share(di.x, dn.x, eps),
                                                   neg_share(di.y, dn.y, eps)), g_d);
                    }
                }
            };
            if (o.interior) body(std::false_type{});
            else body(std::true_type{});
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const int h = o.h0 + threadIdx.y + TY * p;
                if (h >= g.H) continue;
                const int64_t q = static_cast<int64_t>(h) * g.W + wcol;
                gd[grp * HW + q] = p == 0 ? g_d.x : g_d.y;
#pragma unroll
                for (int c = 0; c < NC; ++c)
                    gx[cb + c * HW + q] = static_cast<T>(p == 0 ? gxa[c].x : gxa[c].y);
            }
        }
    }
}

// Float2 fields per pixel-pair record holding n values: an odd number of
// 16-byte units, so the records of 8 consecutive lanes (one 128-bit shared
// load wavefront) fall in distinct 16-byte bank groups.
__host__ __device__ constexpr int pair_fields(int n) {
    return ((n + 1) / 2 * 2 / 2) % 2 == 1 ? (n + 1) / 2 * 2 : (n + 1) / 2 * 2 + 2;
}

// Aggregation for fp32 accumulators, the thread's two pixels packed as in
// bwd_a_tile_x2 (records: r, x[NC]).  A box-masked weight contributes its
// zero products instead of being skipped -- identical for finite inputs.
template <int NC> constexpr int kAgg2F = pair_fields(1 + NC);
template <typename T, int NC>
__global__ void __launch_bounds__(NT)
aggregate_tile_x2(const T* __restrict__ w, const T* __restrict__ x,
                  const float* __restrict__ d, T* __restrict__ Wx,
                  T* __restrict__ dhat, const ShiftTable st, const Geo g, int use_box,
                  float eps) {
    static_assert(PPT == 2, "two pixels per thread");
    constexpr int F = kAgg2F<NC>;
    extern __shared__ __align__(16) unsigned char smem_m[];
    PRF<F>* rec = reinterpret_cast<PRF<F>*>(smem_m);
    const int64_t HW = static_cast<int64_t>(g.H) * g.W;
    const int64_t sstride = static_cast<int64_t>(g.Cw) * HW;
    for (int64_t grp = blockIdx.y; grp < g.groups; grp += gridDim.y) {
        for (int64_t tile = blockIdx.x; tile < g.ntiles; tile += gridDim.x) {
            const Where o = where(g, tile, grp);
            const int64_t cb = (static_cast<int64_t>(o.b) * g.C + o.c0) * HW;
            __syncthreads();
            const float* dg = d + grp * HW;
            stage_pairs<F>(g, o, rec, [&](int64_t off, float* v) {
                const float dv = dg[off];
                v[0] = 1.f / (dv > eps ? dv : eps);
#pragma unroll
                for (int c = 0; c < NC; ++c) v[1 + c] = to_acc(x[cb + c * HW + off]);
            });
            __syncthreads();
            const int wcol = o.w0 + threadIdx.x;
            if (wcol >= g.W) continue;
            const T* wb = w + (static_cast<int64_t>(o.b) * g.S * g.Cw + o.wc) * HW;
            int hh[2];
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const int h = o.h0 + threadIdx.y + TY * p;
                hh[p] = h < g.H ? h : g.H - 1;
            }
            const int ci = (threadIdx.y + g.R) * g.XP + threadIdx.x + g.R;
            const float2 ri = rec[ci].f[0];
            float2 kx[NC], dh = make_float2(0.f, 0.f);
#pragma unroll
            for (int c = 0; c < NC; ++c) kx[c] = make_float2(0.f, 0.f);
            auto body = [&](auto border) {
                constexpr bool BORDER = decltype(border)::value;
#pragma unroll 2
                for (int s = 0; s < g.S; ++s) {
                    const int dx = st.dx[s], dy = st.dy[s];
                    const bool inv = st.has_inv(s);
                    const int off = dx * g.XP + dy;
                    const T* ws = wb + s * sstride;
                    const EdgeGeom e0 = edge_geom<BORDER>(g, hh[0], wcol, dx, dy);
                    const EdgeGeom e1 = edge_geom<BORDER>(g, hh[1], wcol, dx, dy);
                    float2 wq = make_float2(ldg_acc<T, float>(ws + e0.q),
                                            ldg_acc<T, float>(ws + e1.q));
                    float2 wm = make_float2(ldg_acc<T, float>(ws + e0.m),
                                            ldg_acc<T, float>(ws + e1.m));
                    if (BORDER && use_box) {
                        if (!e0.in_p) wq.x = 0.f;
                        if (!e1.in_p) wq.y = 0.f;
                        if (!e0.in_m) wm.x = 0.f;
                        if (!e1.in_m) wm.y = 0.f;
                    }
                    {
                        const PRF<F> nb = rec[ci + off];
                        const float2 wk = f2mul(wq, make_float2(fminf(ri.x, nb.f[0].x),
                                                                fminf(ri.y, nb.f[0].y)));
#pragma unroll
                        for (int c = 0; c < NC; ++c) kx[c] = f2fma(wk, nb.f[1 + c], kx[c]);
                        dh = f2add(dh, wk);
                    }
                    if (inv) {
                        const PRF<F> nb = rec[ci - off];
                        const float2 wk = f2mul(wm, make_float2(fminf(ri.x, nb.f[0].x),
                                                                fminf(ri.y, nb.f[0].y)));
#pragma unroll
                        for (int c = 0; c < NC; ++c) kx[c] = f2fma(wk, nb.f[1 + c], kx[c]);
                        dh = f2add(dh, wk);
                    }
                }
            };
            if (o.interior) body(std::false_type{});
            else body(std::true_type{});
            const PRF<F> me = rec[ci];
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const int h = o.h0 + threadIdx.y + TY * p;
                if (h >= g.H) continue;
                const float dhp = p == 0 ? dh.x : dh.y;
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const int64_t oi = cb + c * HW + static_cast<int64_t>(h) * g.W + wcol;
                    const float xv = p == 0 ? me.f[1 + c].x : me.f[1 + c].y;
                    const float dhx = dhp * xv;
                    Wx[oi] = static_cast<T>((xv - dhx) + (p == 0 ? kx[c].x : kx[c].y));
                    dhat[oi] = static_cast<T>(dhp);
                }
            }
        }
    }
}

// Backward B for fp32 accumulators, packed as in bwd_a_tile_x2 (records: d,
// r, a, g_d, x[NC], gWx[NC]).
template <int NC> constexpr int kBwdB2F = (4 + 2 * NC + 1) / 2 * 2;
template <typename T, int NC>
__global__ void __launch_bounds__(NT)
bwd_b_tile_x2(const T* __restrict__ x, const float* __restrict__ d,
              const T* __restrict__ gWx, const T* __restrict__ gdh,
              const float* __restrict__ gd, T* __restrict__ gw,
              const ShiftTable st, const Geo g, int use_box, float eps) {
    static_assert(PPT == 2, "two pixels per thread");
    constexpr int F = kBwdB2F<NC>;
    constexpr int XO = 4, GO = 4 + NC;
    extern __shared__ __align__(16) unsigned char smem_m[];
    PRF<F>* rec = reinterpret_cast<PRF<F>*>(smem_m);
    const int64_t HW = static_cast<int64_t>(g.H) * g.W;
    const int64_t sstride = static_cast<int64_t>(g.Cw) * HW;
    for (int64_t grp = blockIdx.y; grp < g.groups; grp += gridDim.y) {
        for (int64_t tile = blockIdx.x; tile < g.ntiles; tile += gridDim.x) {
            const Where o = where(g, tile, grp);
            const int64_t cb = (static_cast<int64_t>(o.b) * g.C + o.c0) * HW;
            __syncthreads();
            const float* dg = d + grp * HW;
            const float* gdg = gd + grp * HW;
            stage_pairs<F>(g, o, rec, [&](int64_t off, float* v) {
                const float dv = dg[off];
                v[0] = dv;
                v[1] = 1.f / (dv > eps ? dv : eps);
                float a = 0.f;
#pragma unroll
                for (int cc = 0; cc < NC; ++cc) {
                    const float xv = to_acc(x[cb + cc * HW + off]);
                    const float gv = to_acc(gWx[cb + cc * HW + off]);
                    v[XO + cc] = xv;
                    v[GO + cc] = gv;
                    a += to_acc(gdh[cb + cc * HW + off]) - gv * xv;
                }
                v[2] = a;
                v[3] = gdg[off];
            });
            __syncthreads();
            const int wcol = o.w0 + threadIdx.x;
            if (wcol >= g.W) continue;
            T* gwb = gw + (static_cast<int64_t>(o.b) * g.S * g.Cw + o.wc) * HW;
            int hh[2];
            bool act[2];
#pragma unroll
            for (int p = 0; p < 2; ++p) {
                const int h = o.h0 + threadIdx.y + TY * p;
                act[p] = h < g.H;
                hh[p] = act[p] ? h : g.H - 1;
            }
            const int ci = (threadIdx.y + g.R) * g.XP + threadIdx.x + g.R;
            float2 ri, gdi, aq, xq[NC], gq[NC];
            {
                const PRF<F> me = rec[ci];
                ri = me.f[1];
                aq = me.f[2];
                gdi = me.f[3];
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    xq[c] = me.f[XO + c];
                    gq[c] = me.f[GO + c];
                }
            }
            auto body = [&](auto border) {
                constexpr bool BORDER = decltype(border)::value;
#pragma unroll 2
                for (int s = 0; s < g.S; ++s) {
                    const int dx = st.dx[s], dy = st.dy[s];
                    const bool inv = st.has_inv(s);
                    const int off = dx * g.XP + dy;
                    T* gws = gwb + s * sstride;
                    const EdgeGeom e0 = edge_geom<BORDER>(g, hh[0], wcol, dx, dy);
                    const EdgeGeom e1 = edge_geom<BORDER>(g, hh[1], wcol, dx, dy);
                    const PRF<F> nb = rec[ci + off];
                    const float2 r = make_float2(fminf(ri.x, nb.f[1].x),
                                                 fminf(ri.y, nb.f[1].y));
                    float2 G = aq;
#pragma unroll
                    for (int c = 0; c < NC; ++c) G = f2fma(gq[c], nb.f[XO + c], G);
                    float2 v = f2fma(G, r, gdi);
                    if (inv) {
                        float2 Gm = nb.f[2];
#pragma unroll
                        for (int c = 0; c < NC; ++c) Gm = f2fma(nb.f[GO + c], xq[c], Gm);
                        v = f2add(v, f2fma(Gm, r, nb.f[3]));
                    }
                    if (BORDER && use_box) {
                        if (!e0.in_p) v.x = 0.f;
                        if (!e1.in_p) v.y = 0.f;
                    }
                    if (act[0]) gws[e0.q] = static_cast<T>(v.x);
                    if (act[1]) gws[e1.q] = static_cast<T>(v.y);
                }
            };
            if (o.interior) body(std::false_type{});
            else body(std::true_type{});
        }
    }
}

// ------------------------------------------------------------ backward B
// grad_w without reading w:
//   gw_s(q) = keep_f(q) (G_f r + g_d(q)) + inv keep_i(q + d) (G_m r + g_d(q + d))
//   G_f = a(q) + sum_c gWx(q) x(q + d),  G_m = a(q + d) + sum_c gWx(q + d) x(q)
// with r = min(r(q), r(q + d)); keep_i(q + d) = [q + d inside] = keep_f(q).
template <typename T, int NC>
__global__ void __launch_bounds__(NT)
bwd_b_tile(const T* __restrict__ x, const typename Acc<T>::type* __restrict__ d,
           const T* __restrict__ gWx, const T* __restrict__ gdh,
           const typename Acc<T>::type* __restrict__ gd, T* __restrict__ gw,
           const ShiftTable st, const Geo g, int use_box, typename Acc<T>::type eps) {
    using A = typename Acc<T>::type;
    constexpr int F = kBwdBF<A, NC>;
    constexpr int XO = 4, GO = 4 + NC;
    extern __shared__ __align__(16) unsigned char smem_m[];
    Rec<A, F>* rec = reinterpret_cast<Rec<A, F>*>(smem_m);
    const int64_t HW = static_cast<int64_t>(g.H) * g.W;
    const int64_t sstride = static_cast<int64_t>(g.Cw) * HW;
    for (int64_t grp = blockIdx.y; grp < g.groups; grp += gridDim.y) {
        for (int64_t tile = blockIdx.x; tile < g.ntiles; tile += gridDim.x) {
            const Where o = where(g, tile, grp);
            const int64_t cb = (static_cast<int64_t>(o.b) * g.C + o.c0) * HW;
            __syncthreads();
            stage_bwd<T, NC, F, XO>(g, o, grp, cb, HW, d, gd, x, gWx, gdh, eps, rec);
            __syncthreads();
            const int wcol = o.w0 + threadIdx.x;
            if (wcol >= g.W) continue;
            T* gwb = gw + (static_cast<int64_t>(o.b) * g.S * g.Cw + o.wc) * HW;
            int hh[PPT], ci[PPT];
            bool act[PPT];
            A ri[PPT], gdi[PPT], aq[PPT], xq[PPT][NC], gq[PPT][NC];
#pragma unroll
            for (int p = 0; p < PPT; ++p) {
                const int h = o.h0 + threadIdx.y + TY * p;
                act[p] = h < g.H;
                hh[p] = act[p] ? h : g.H - 1;
                ci[p] = (threadIdx.y + TY * p + g.R) * g.XP + threadIdx.x + g.R;
                const Rec<A, F> me = rec[ci[p]];
                ri[p] = me.f[1];
                aq[p] = me.f[2];
                gdi[p] = me.f[3];
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    xq[p][c] = me.f[XO + c];
                    gq[p][c] = me.f[GO + c];
                }
            }
            auto body = [&](auto border) {
                constexpr bool BORDER = decltype(border)::value;
#pragma unroll 2
                for (int s = 0; s < g.S; ++s) {
                    const int dx = st.dx[s], dy = st.dy[s];
                    const bool inv = st.has_inv(s);
                    const int off = dx * g.XP + dy;
                    T* gws = gwb + s * sstride;
#pragma unroll
                    for (int p = 0; p < PPT; ++p) {
                        const EdgeGeom e = edge_geom<BORDER>(g, hh[p], wcol, dx, dy);
                        const Rec<A, F> nb = rec[ci[p] + off];
                        const A r = amin(ri[p], nb.f[1]);
                        A v = A(0);
                        if (!use_box || e.in_p) {
                            A G = aq[p];
#pragma unroll
                            for (int c = 0; c < NC; ++c) G += gq[p][c] * nb.f[XO + c];
                            v += G * r + gdi[p];
                            if (inv) {
                                A Gm = nb.f[2];
#pragma unroll
                                for (int c = 0; c < NC; ++c) Gm += nb.f[GO + c] * xq[p][c];
                                v += Gm * r + nb.f[3];
                            }
                        }
                        if (act[p]) gws[e.q] = static_cast<T>(v);
                    }
                }
            };
            if (o.interior) body(std::false_type{});
            else body(std::true_type{});
        }
    }
}

}  // namespace mtile
}  // namespace nsc
