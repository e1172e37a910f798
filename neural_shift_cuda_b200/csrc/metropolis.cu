// metropolis.cu -- Metropolis-normalized symmetric aggregation, forward and
// backward (the reference has a forward kernel only: metropolis_cuda.cu).
//
// Edges of pixel p: for every half-plane row s the forward edge (delta = d_s,
// weight wt = keep_f(p) w_s(p)) and, for has_inv rows, the mirror edge
// (delta = -d_s, weight wt = keep_i(p) w_s(p - d_s), circular address).  With
// use_box, keep_f(p) = [p + d inside], keep_i(p) = [p - d inside]; without,
// both are 1 (periodic operator).
//   d(p)     = sum_e wt_e(p)                       (raw degree, K e)
//   den_e(p) = max(max(d(p), d(p + delta_e)), eps)
//   wk_e(p)  = wt_e(p) / den_e(p)
//   d_hat(p) = sum_e wk_e(p),  Khat x(p) = sum_e wk_e(p) x(p + delta_e)
//   Wx(p)    = x(p) - d_hat(p) x(p) + Khat x(p)
// (reference: metropolis.py:54-114, metropolis_cuda.cu:71-186).
//
// Forward: two launches, the degree into the caller's scratch `degree`,
// then the aggregation with the Wx epilogue fused (the reference forms Wx
// with separate ATen elementwise kernels, metropolis_cuda.cu:237).
// Backward: gradients of the same expression with torch's conventions for
// the reference's autograd path (metropolis.py:117-192): maximum() splits a
// tie equally between its arguments, clamp_min(eps) passes the gradient
// where its input >= eps.  Pass A gives grad_img and the degree gradient
// g_d (into `grad_degree`); pass B writes grad_w without reading w.

#include <cmath>

#include <cstdlib>

#include "metropolis_tile.cuh"
#include "nsc_common.cuh"
#include "nsc_host.h"

namespace nsc {
namespace {

constexpr int kBX = 32, kBY = 8;

template <typename T>
__device__ __forceinline__ T store_as(typename Acc<T>::type v) { return static_cast<T>(v); }

// w_half is (B, S, Cw, H, W); plane of (b, s, wc).
__device__ __forceinline__ int64_t wplane(int64_t b, int s, int64_t wc,
                                          int64_t S, int64_t Cw, int64_t HW) {
    return ((b * S + s) * Cw + wc) * HW;
}

template <typename T>
__global__ void __launch_bounds__(kBX * kBY)
metro_degree_kernel(const T* __restrict__ w, typename Acc<T>::type* __restrict__ d,
                    const ShiftTable st, int64_t B, int64_t Cw, int64_t H,
                    int64_t W, int use_box, int64_t groups) {
    using A = typename Acc<T>::type;
    const int64_t wcol = static_cast<int64_t>(blockIdx.x) * kBX + threadIdx.x;
    const int64_t h = static_cast<int64_t>(blockIdx.y) * kBY + threadIdx.y;
    if (wcol >= W || h >= H) return;
    const int64_t HW = H * W;
    for (int64_t g = blockIdx.z; g < groups; g += gridDim.z) {
        const int64_t b = g / Cw, wc = g % Cw;
        A acc = A(0);
        for (int s = 0; s < st.S; ++s) {
            const int64_t dx = st.dx[s], dy = st.dy[s];
            const T* ws = w + wplane(b, s, wc, st.S, Cw, HW);
            if (!use_box || (inb(h + dx, H) && inb(wcol + dy, W)))
                acc += ldg_acc<T, A>(ws + h * W + wcol);
            if (st.has_inv(s) && (!use_box || (inb(h - dx, H) && inb(wcol - dy, W))))
                acc += ldg_acc<T, A>(ws + wrap1(h - dx, H) * W + wrap1(wcol - dy, W));
        }
        d[g * HW + h * W + wcol] = acc;
    }
}

// Thread: one pixel, the NC channels that share weight channel wc.
template <typename T, int NC>
__global__ void __launch_bounds__(kBX * kBY)
metro_aggregate_kernel(const T* __restrict__ w, const T* __restrict__ x,
                       const typename Acc<T>::type* __restrict__ d,
                       T* __restrict__ Wx, T* __restrict__ dhat,
                       const ShiftTable st, int64_t B, int64_t C, int64_t Cw,
                       int64_t H, int64_t W, int use_box,
                       typename Acc<T>::type eps, int64_t groups) {
    using A = typename Acc<T>::type;
    const int64_t wcol = static_cast<int64_t>(blockIdx.x) * kBX + threadIdx.x;
    const int64_t h = static_cast<int64_t>(blockIdx.y) * kBY + threadIdx.y;
    if (wcol >= W || h >= H) return;
    const int64_t HW = H * W;
    const int64_t q = h * W + wcol;
    const int nc = (Cw == 1) ? static_cast<int>(C) : 1;
    for (int64_t g = blockIdx.z; g < groups; g += gridDim.z) {
        const int64_t b = g / Cw, wc = g % Cw;
        const int64_t c0 = (Cw == 1) ? 0 : wc;
        const T* xb = x + (b * C + c0) * HW;
        const A* dg = d + g * HW;
        const A di = dg[q];
        A kx[NC], dh = A(0);
#pragma unroll
        for (int i = 0; i < NC; ++i) kx[i] = A(0);
        for (int s = 0; s < st.S; ++s) {
            const int64_t dx = st.dx[s], dy = st.dy[s];
            const T* ws = w + wplane(b, s, wc, st.S, Cw, HW);
            if (!use_box || (inb(h + dx, H) && inb(wcol + dy, W))) {
                const int64_t n = wrap1(h + dx, H) * W + wrap1(wcol + dy, W);
                const A dj = dg[n];
                const A den = di > dj ? di : dj;
                const A wk = ldg_acc<T, A>(ws + q) / (den > eps ? den : eps);
#pragma unroll
                for (int i = 0; i < NC; ++i)
                    if (i < nc) kx[i] += wk * ldg_acc<T, A>(xb + i * HW + n);
                dh += wk;
            }
            if (st.has_inv(s) && (!use_box || (inb(h - dx, H) && inb(wcol - dy, W)))) {
                const int64_t n = wrap1(h - dx, H) * W + wrap1(wcol - dy, W);
                const A dj = dg[n];
                const A den = di > dj ? di : dj;
                const A wk = ldg_acc<T, A>(ws + n) / (den > eps ? den : eps);
#pragma unroll
                for (int i = 0; i < NC; ++i)
                    if (i < nc) kx[i] += wk * ldg_acc<T, A>(xb + i * HW + n);
                dh += wk;
            }
        }
#pragma unroll
        for (int i = 0; i < NC; ++i) {
            if (i >= nc) continue;
            const int64_t o = (b * C + c0 + i) * HW + q;
            const A xv = ldg_acc<T, A>(x + o);
            const A dhx = dh * xv;
            Wx[o] = store_as<T>((xv - dhx) + kx[i]);
            dhat[o] = store_as<T>(dh);
        }
    }
}

// Share of d(self) in maximum(d(self), d(other)): 1, 1/2 on a tie, else 0.
template <typename A>
__device__ __forceinline__ A share(A self, A other) {
    return self > other ? A(1) : (self == other ? A(0.5) : A(0));
}

// Pass A.  For pixel q: grad_img(q, c) and g_d(q) (degree gradient).
//   G_e(p) = sum_c gWx(p,c) x(p+delta_e,c) + a(p,c),  a = gdh - gWx x
//   g_den_e(p) = -G_e(p) wt_e(p) / den_e(p)^2  (0 where raw < eps)
//   g_d(q) = sum_e g_den_e(q) share(d(q), d(q+delta))
//          + sum_e g_den_e(q-delta) share(d(q), d(q-delta))
//   gx(q,c) = gWx(q,c) (1 - dh(q,c)) + sum_e gWx(q-delta,c) wk_e(q-delta)
template <typename T, int NC>
__global__ void __launch_bounds__(kBX * kBY)
metro_bwd_a_kernel(const T* __restrict__ w, const T* __restrict__ x,
                   const typename Acc<T>::type* __restrict__ d,
                   const T* __restrict__ dhat, const T* __restrict__ gWx,
                   const T* __restrict__ gdh,
                   typename Acc<T>::type* __restrict__ gd, T* __restrict__ gx,
                   const ShiftTable st, int64_t B, int64_t C, int64_t Cw,
                   int64_t H, int64_t W, int use_box,
                   typename Acc<T>::type eps, int64_t groups) {
    using A = typename Acc<T>::type;
    const int64_t wcol = static_cast<int64_t>(blockIdx.x) * kBX + threadIdx.x;
    const int64_t h = static_cast<int64_t>(blockIdx.y) * kBY + threadIdx.y;
    if (wcol >= W || h >= H) return;
    const int64_t HW = H * W;
    const int64_t q = h * W + wcol;
    const int nc = (Cw == 1) ? static_cast<int>(C) : 1;
    for (int64_t g = blockIdx.z; g < groups; g += gridDim.z) {
        const int64_t b = g / Cw, wc = g % Cw;
        const int64_t cb = (b * C + ((Cw == 1) ? 0 : wc)) * HW;
        const A* dg = d + g * HW;
        const A di = dg[q];
        A xq[NC], gq[NC], gxa[NC], Aq = A(0);
#pragma unroll
        for (int i = 0; i < NC; ++i) {
            const bool on = i < nc;
            xq[i] = on ? ldg_acc<T, A>(x + cb + i * HW + q) : A(0);
            gq[i] = on ? ldg_acc<T, A>(gWx + cb + i * HW + q) : A(0);
            const A dhq = on ? ldg_acc<T, A>(dhat + cb + i * HW + q) : A(0);
            if (on) Aq += ldg_acc<T, A>(gdh + cb + i * HW + q) - gq[i] * xq[i];
            gxa[i] = gq[i] * (A(1) - dhq);
        }
        A g_d = A(0);
        for (int s = 0; s < st.S; ++s) {
            const int64_t dx = st.dx[s], dy = st.dy[s];
            const T* ws = w + wplane(b, s, wc, st.S, Cw, HW);
            const bool inv = st.has_inv(s);
            const A w_q = ldg_acc<T, A>(ws + q);
            const int64_t qm = wrap1(h - dx, H) * W + wrap1(wcol - dy, W);  // q - d
            const int64_t qp = wrap1(h + dx, H) * W + wrap1(wcol + dy, W);  // q + d
            const bool in_m = inb(h - dx, H) && inb(wcol - dy, W);
            const bool in_p = inb(h + dx, H) && inb(wcol + dy, W);
            const A w_m = ldg_acc<T, A>(ws + qm);
            for (int e = 0; e < (inv ? 2 : 1); ++e) {
                // e == 0: forward edge (delta = d); e == 1: mirror (delta = -d)
                const int64_t nq = e == 0 ? qp : qm;          // q + delta
                const int64_t pq = e == 0 ? qm : qp;          // q - delta
                // own edge at q
                const A wt_own = e == 0 ? ((!use_box || in_p) ? w_q : A(0))
                                        : ((!use_box || in_m) ? w_m : A(0));
                if (wt_own != A(0)) {
                    const A dj = dg[nq];
                    const A raw = di > dj ? di : dj;
                    const A den = raw > eps ? raw : eps;
                    A G = Aq;
#pragma unroll
                    for (int i = 0; i < NC; ++i)
                        if (i < nc) G += gq[i] * ldg_acc<T, A>(x + cb + i * HW + nq);
                    if (raw >= eps) g_d += -G * wt_own / (den * den) * share(di, dj);
                }
                // edge of p = q - delta whose neighbour is q
                // forward: wt = keep_f(p) w_s(q - d); mirror: keep_i(p) w_s(q)
                const A wt_p = e == 0 ? ((!use_box || in_m) ? w_m : A(0))
                                      : ((!use_box || in_p) ? w_q : A(0));
                if (wt_p != A(0)) {
                    const A dp = dg[pq];
                    const A raw = dp > di ? dp : di;
                    const A den = raw > eps ? raw : eps;
                    const A wk = wt_p / den;
                    A G = A(0);
#pragma unroll
                    for (int i = 0; i < NC; ++i)
                        if (i < nc) {
                            const A gp = ldg_acc<T, A>(gWx + cb + i * HW + pq);
                            const A xp = ldg_acc<T, A>(x + cb + i * HW + pq);
                            G += gp * xq[i] + ldg_acc<T, A>(gdh + cb + i * HW + pq) - gp * xp;
                            gxa[i] += gp * wk;
                        }
                    if (raw >= eps) g_d += -G * wt_p / (den * den) * share(di, dp);
                }
            }
        }
        gd[g * HW + q] = g_d;
#pragma unroll
        for (int i = 0; i < NC; ++i)
            if (i < nc) gx[cb + i * HW + q] = store_as<T>(gxa[i]);
    }
}

// Pass B.  grad_w_s(q) = keep_f(q) (G_f(q) / den_f(q) + g_d(q))
//                      + inv keep_i(q+d) (G_m(q+d) / den_m(q+d) + g_d(q+d))
// with den_f(q) = den_m(q+d) = max(max(d(q), d(q+d)), eps).  No weight reads.
template <typename T, int NC>
__global__ void __launch_bounds__(kBX * kBY)
metro_bwd_b_kernel(const T* __restrict__ x,
                   const typename Acc<T>::type* __restrict__ d,
                   const T* __restrict__ gWx, const T* __restrict__ gdh,
                   const typename Acc<T>::type* __restrict__ gd,
                   T* __restrict__ gw, const ShiftTable st, int64_t B,
                   int64_t C, int64_t Cw, int64_t H, int64_t W, int use_box,
                   typename Acc<T>::type eps, int64_t groups) {
    using A = typename Acc<T>::type;
    const int64_t wcol = static_cast<int64_t>(blockIdx.x) * kBX + threadIdx.x;
    const int64_t h = static_cast<int64_t>(blockIdx.y) * kBY + threadIdx.y;
    if (wcol >= W || h >= H) return;
    const int64_t HW = H * W;
    const int64_t q = h * W + wcol;
    const int nc = (Cw == 1) ? static_cast<int>(C) : 1;
    for (int64_t g = blockIdx.z; g < groups; g += gridDim.z) {
        const int64_t b = g / Cw, wc = g % Cw;
        const int64_t cb = (b * C + ((Cw == 1) ? 0 : wc)) * HW;
        const A* dg = d + g * HW;
        const A* gdg = gd + g * HW;
        const A di = dg[q], gdi = gdg[q];
        A xq[NC], gq[NC], Aq = A(0);
#pragma unroll
        for (int i = 0; i < NC; ++i) {
            const bool on = i < nc;
            xq[i] = on ? ldg_acc<T, A>(x + cb + i * HW + q) : A(0);
            gq[i] = on ? ldg_acc<T, A>(gWx + cb + i * HW + q) : A(0);
            if (on) Aq += ldg_acc<T, A>(gdh + cb + i * HW + q) - gq[i] * xq[i];
        }
        for (int s = 0; s < st.S; ++s) {
            const int64_t dx = st.dx[s], dy = st.dy[s];
            const bool in_p = inb(h + dx, H) && inb(wcol + dy, W);
            const int64_t qp = wrap1(h + dx, H) * W + wrap1(wcol + dy, W);
            const A dj = dg[qp];
            const A raw = di > dj ? di : dj;
            const A den = raw > eps ? raw : eps;
            A gws = A(0);
            if (!use_box || in_p) {
                A G = Aq;
#pragma unroll
                for (int i = 0; i < NC; ++i)
                    if (i < nc) G += gq[i] * ldg_acc<T, A>(x + cb + i * HW + qp);
                gws += G / den + gdi;
            }
            if (st.has_inv(s) && (!use_box || in_p)) {
                // mirror edge at p = q + d (keep_i(p) = [q + d inside])
                A G = A(0);
#pragma unroll
                for (int i = 0; i < NC; ++i)
                    if (i < nc) {
                        const A gp = ldg_acc<T, A>(gWx + cb + i * HW + qp);
                        const A xp = ldg_acc<T, A>(x + cb + i * HW + qp);
                        G += gp * xq[i] + ldg_acc<T, A>(gdh + cb + i * HW + qp) - gp * xp;
                    }
                gws += G / den + gdg[qp];
            }
            gw[wplane(b, s, wc, st.S, Cw, HW) + q] = store_as<T>(gws);
        }
    }
}

template <int NC> struct NCTag { static constexpr int value_nc = NC; };

template <typename F>
nsc_status with_type(const char* op, int xd, int wd, F&& f) {
    if (xd != wd)
        return fail(NSC_ERR_UNSUPPORTED_DTYPE,
                    "%s: w_half and img must have the same dtype", op);
    switch (xd) {
        case NSC_F64: return f((const double*)nullptr);
        case NSC_F32: return f((const float*)nullptr);
        case NSC_F16: return f((const __half*)nullptr);
        case NSC_BF16: return f((const __nv_bfloat16*)nullptr);
        default: return fail(NSC_ERR_UNSUPPORTED_DTYPE, "%s: unsupported dtype", op);
    }
}

template <typename F>
void with_nc(int64_t C, int64_t Cw, F&& f) {
    const int64_t nc = (Cw == 1) ? C : 1;
    if (nc == 4) f(NCTag<4>{});
    else if (nc == 3) f(NCTag<3>{});
    else if (nc == 2) f(NCTag<2>{});
    else f(NCTag<1>{});
}

inline dim3 grid_for(int64_t W, int64_t H, int64_t groups) {
    return dim3(grid_1d(W, kBX), grid_1d(H, kBY),
                static_cast<unsigned>(groups < 65535 ? groups : 65535));
}

nsc_status check_metro(const char* op, int64_t Cw, int64_t B, int64_t C,
                       int64_t H, int64_t W, const int64_t* shifts, int64_t S,
                       double eps, ShiftTable* st) {
    nsc_status e = check_extents(op, B, C, H, W);
    if (e) return e;
    if (!(Cw == C || (Cw == 1 && C >= 1 && C <= 4)))
        return fail(NSC_ERR_INVALID_ARG,
                    "%s: w_half must be (B, S, C, H, W) or channel-broadcast "
                    "(B, S, 1, H, W) with C <= 4; got w_channels=%lld, C=%lld",
                    op, (long long)Cw, (long long)C);
    if (!(eps > 0.0) || !std::isfinite(eps))
        return fail(NSC_ERR_INVALID_ARG, "%s: eps must be finite and > 0", op);
    nsc_status e2 = build_shifts(op, shifts, S, 3, H, W, st);
    if (e2) return e2;
    if (st->any_tr)
        return fail(NSC_ERR_INVALID_ARG,
                    "%s: transposed rows (column value 3) are accepted by "
                    "accumulate_uz only", op);
    return ok();
}

// Geometry of the tiled kernels, or false when the call stays on the
// one-pixel kernels (radius > 8, extents >= 2^30, or NSC_METRO_GENERIC).
bool tile_geo(const ShiftTable& st, int64_t B, int64_t C, int64_t Cw, int64_t H,
              int64_t W, mtile::Geo* g) {
    if (getenv("NSC_METRO_GENERIC")) return false;
    if (st.R > mtile::MAXR || H >= (1LL << 30) || W >= (1LL << 30) ||
        B * Cw >= (1LL << 40))
        return false;
    g->B = static_cast<int>(B); g->C = static_cast<int>(C);
    g->Cw = static_cast<int>(Cw); g->H = static_cast<int>(H);
    g->W = static_cast<int>(W); g->S = st.S; g->R = st.R;
    g->XP = mtile::TW + 2 * st.R;
    g->XR = mtile::TH + 2 * st.R;
    g->tiles_x = static_cast<int>((W + mtile::TW - 1) / mtile::TW);
    g->ntiles = static_cast<int64_t>(g->tiles_x) * ((H + mtile::TH - 1) / mtile::TH);
    g->groups = B * Cw;
    return true;
}

inline dim3 tile_grid(const mtile::Geo& g) {
    return dim3(static_cast<unsigned>(g.ntiles < (1LL << 31) - 1 ? g.ntiles : (1LL << 31) - 1),
                static_cast<unsigned>(g.groups < 65535 ? g.groups : 65535));
}

// Dynamic shared memory of a tiled kernel staging `planes` values (one
// record of that many) per halo pixel.
template <typename K>
bool tile_smem(K kern, const mtile::Geo& g, int planes, size_t elem, size_t* bytes) {
    *bytes = static_cast<size_t>(planes) * g.XR * g.XP * elem;
    if (*bytes > 200 * 1024) return false;
    if (*bytes > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(*bytes)) != cudaSuccess)
        return false;
    return true;
}

// Dynamic shared memory of a packed (pixel-pair record) tiled kernel:
// TY + 2R pair rows of XP records of `rec_bytes`.
template <typename K>
bool pair_smem(K kern, const mtile::Geo& g, size_t rec_bytes, size_t* bytes) {
    *bytes = rec_bytes * static_cast<size_t>(mtile::TY + 2 * g.R) * g.XP;
    if (*bytes > 200 * 1024) return false;
    if (*bytes > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(*bytes)) != cudaSuccess)
        return false;
    return true;
}

}  // namespace
}  // namespace nsc

extern "C" {

nsc_status nsc_metropolis_fwd(const void* w_half, int w_dtype, int64_t w_channels,
                              const void* img, int x_dtype, int64_t B, int64_t C,
                              int64_t H, int64_t W, const int64_t* shifts,
                              int64_t S, int use_box, double eps, void* Wx,
                              void* d_hat, void* degree, void* stream) {
    using namespace nsc;
    const char* op = "metropolis_aggregate";
    ShiftTable st;
    nsc_status e = check_metro(op, w_channels, B, C, H, W, shifts, S, eps, &st);
    if (e) return e;
    if (B == 0 || C == 0 || H == 0 || W == 0) return ok();
    if (!w_half || !img || !Wx || !d_hat || !degree)
        return fail(NSC_ERR_INVALID_ARG, "%s: NULL tensor pointer", op);
    cudaStream_t sm = as_stream(stream);
    return with_type(op, x_dtype, w_dtype, [&](auto tp) {
        using T = std::remove_const_t<std::remove_pointer_t<decltype(tp)>>;
        using A = typename Acc<T>::type;
        const int64_t groups = B * w_channels;
        mtile::Geo tg;
        if (tile_geo(st, B, C, w_channels, H, W, &tg)) {
            bool launched = false;
            with_nc(C, w_channels, [&](auto tag) {
                constexpr int NC = decltype(tag)::value_nc;
                auto agg = mtile::aggregate_tile<T, NC>;
                size_t smem = 0;
                if (!tile_smem(agg, tg, mtile::kAggF<A, NC>, sizeof(A), &smem)) return;
                mtile::degree_tile<T><<<tile_grid(tg), dim3(mtile::TX, mtile::TY), 0, sm>>>(
                    static_cast<const T*>(w_half), static_cast<A*>(degree), st, tg,
                    use_box ? 1 : 0);
                if constexpr (std::is_same_v<A, float> && mtile::PPT == 2) {
                    // fp32: the thread's two pixels as f32x2 lanes
                    auto k2 = mtile::aggregate_tile_x2<T, NC>;
                    size_t s2 = 0;
                    if (pair_smem(k2, tg, sizeof(mtile::PRF<mtile::kAgg2F<NC>>), &s2)) {
                        k2<<<tile_grid(tg), dim3(mtile::TX, mtile::TY), s2, sm>>>(
                            static_cast<const T*>(w_half), static_cast<const T*>(img),
                            static_cast<const A*>(degree), static_cast<T*>(Wx),
                            static_cast<T*>(d_hat), st, tg, use_box ? 1 : 0,
                            static_cast<A>(eps));
                        launched = true;
                        return;
                    }
                }
                agg<<<tile_grid(tg), dim3(mtile::TX, mtile::TY), smem, sm>>>(
                    static_cast<const T*>(w_half), static_cast<const T*>(img),
                    static_cast<const A*>(degree), static_cast<T*>(Wx),
                    static_cast<T*>(d_hat), st, tg, use_box ? 1 : 0,
                    static_cast<A>(eps));
                launched = true;
            });
            if (launched) return check_launch(op);
        }
        metro_degree_kernel<T><<<grid_for(W, H, groups), dim3(kBX, kBY), 0, sm>>>(
            static_cast<const T*>(w_half), static_cast<A*>(degree), st, B,
            w_channels, H, W, use_box ? 1 : 0, groups);
        with_nc(C, w_channels, [&](auto tag) {
            constexpr int NC = decltype(tag)::value_nc;
            metro_aggregate_kernel<T, NC><<<grid_for(W, H, groups),
                                             dim3(kBX, kBY), 0, sm>>>(
                static_cast<const T*>(w_half), static_cast<const T*>(img),
                static_cast<const A*>(degree), static_cast<T*>(Wx),
                static_cast<T*>(d_hat), st, B, C, w_channels, H, W,
                use_box ? 1 : 0, static_cast<A>(eps), groups);
        });
        return check_launch(op);
    });
}

nsc_status nsc_metropolis_bwd(const void* w_half, int w_dtype, int64_t w_channels,
                              const void* img, int x_dtype, int64_t B, int64_t C,
                              int64_t H, int64_t W, const int64_t* shifts,
                              int64_t S, int use_box, double eps,
                              const void* degree, const void* d_hat,
                              const void* grad_Wx, const void* grad_d_hat,
                              void* grad_degree, void* grad_w, void* grad_img,
                              void* stream) {
    using namespace nsc;
    const char* op = "metropolis_aggregate_backward";
    ShiftTable st;
    nsc_status e = check_metro(op, w_channels, B, C, H, W, shifts, S, eps, &st);
    if (e) return e;
    if (B == 0 || C == 0 || H == 0 || W == 0) return ok();
    if (!w_half || !img || !degree || !d_hat || !grad_Wx || !grad_d_hat ||
        !grad_degree || !grad_w || !grad_img)
        return fail(NSC_ERR_INVALID_ARG, "%s: NULL tensor pointer", op);
    cudaStream_t sm = as_stream(stream);
    return with_type(op, x_dtype, w_dtype, [&](auto tp) {
        using T = std::remove_const_t<std::remove_pointer_t<decltype(tp)>>;
        using A = typename Acc<T>::type;
        const int64_t groups = B * w_channels;
        mtile::Geo tg;
        if (tile_geo(st, B, C, w_channels, H, W, &tg)) {
            bool launched = false;
            with_nc(C, w_channels, [&](auto tag) {
                constexpr int NC = decltype(tag)::value_nc;
                auto ka = mtile::bwd_a_tile<T, NC>;
                auto kb = mtile::bwd_b_tile<T, NC>;
                size_t sa = 0, sb = 0;
                if (!tile_smem(ka, tg, mtile::kBwdAF<A, NC>, sizeof(A), &sa) ||
                    !tile_smem(kb, tg, mtile::kBwdBF<A, NC>, sizeof(A), &sb))
                    return;
                bool packed = false;
                if constexpr (std::is_same_v<A, float> && mtile::PPT == 2) {
                    // fp32: the thread's two pixels as f32x2 lanes
                    auto k2 = mtile::bwd_a_tile_x2<T, NC>;
                    auto k2b = mtile::bwd_b_tile_x2<T, NC>;
                    size_t s2 = 0, s2b = 0;
                    if (pair_smem(k2, tg, sizeof(mtile::PRec<NC>), &s2) &&
                        pair_smem(k2b, tg, sizeof(mtile::PRF<mtile::kBwdB2F<NC>>), &s2b)) {
                        k2<<<tile_grid(tg), dim3(mtile::TX, mtile::TY), s2, sm>>>(
                            static_cast<const T*>(w_half), static_cast<const T*>(img),
                            static_cast<const A*>(degree), static_cast<const T*>(d_hat),
                            static_cast<const T*>(grad_Wx),
                            static_cast<const T*>(grad_d_hat),
                            static_cast<A*>(grad_degree), static_cast<T*>(grad_img), st,
                            tg, use_box ? 1 : 0, static_cast<A>(eps));
                        k2b<<<tile_grid(tg), dim3(mtile::TX, mtile::TY), s2b, sm>>>(
                            static_cast<const T*>(img), static_cast<const A*>(degree),
                            static_cast<const T*>(grad_Wx),
                            static_cast<const T*>(grad_d_hat),
                            static_cast<const A*>(grad_degree), static_cast<T*>(grad_w),
                            st, tg, use_box ? 1 : 0, static_cast<A>(eps));
                        packed = true;
                    }
                }
                if (packed) {
                    launched = true;
                    return;
                }
                ka<<<tile_grid(tg), dim3(mtile::TX, mtile::TY), sa, sm>>>(
                    static_cast<const T*>(w_half), static_cast<const T*>(img),
                    static_cast<const A*>(degree), static_cast<const T*>(d_hat),
                    static_cast<const T*>(grad_Wx), static_cast<const T*>(grad_d_hat),
                    static_cast<A*>(grad_degree), static_cast<T*>(grad_img), st, tg,
                    use_box ? 1 : 0, static_cast<A>(eps));
                kb<<<tile_grid(tg), dim3(mtile::TX, mtile::TY), sb, sm>>>(
                    static_cast<const T*>(img), static_cast<const A*>(degree),
                    static_cast<const T*>(grad_Wx), static_cast<const T*>(grad_d_hat),
                    static_cast<const A*>(grad_degree), static_cast<T*>(grad_w), st,
                    tg, use_box ? 1 : 0, static_cast<A>(eps));
                launched = true;
            });
            if (launched) return check_launch(op);
        }
        with_nc(C, w_channels, [&](auto tag) {
            constexpr int NC = decltype(tag)::value_nc;
            metro_bwd_a_kernel<T, NC><<<grid_for(W, H, groups), dim3(kBX, kBY),
                                         0, sm>>>(
                static_cast<const T*>(w_half), static_cast<const T*>(img),
                static_cast<const A*>(degree), static_cast<const T*>(d_hat),
                static_cast<const T*>(grad_Wx), static_cast<const T*>(grad_d_hat),
                static_cast<A*>(grad_degree), static_cast<T*>(grad_img), st, B,
                C, w_channels, H, W, use_box ? 1 : 0, static_cast<A>(eps), groups);
            metro_bwd_b_kernel<T, NC><<<grid_for(W, H, groups), dim3(kBX, kBY),
                                         0, sm>>>(
                static_cast<const T*>(img), static_cast<const A*>(degree),
                static_cast<const T*>(grad_Wx), static_cast<const T*>(grad_d_hat),
                static_cast<const A*>(grad_degree), static_cast<T*>(grad_w), st,
                B, C, w_channels, H, W, use_box ? 1 : 0, static_cast<A>(eps),
                groups);
        });
        return check_launch(op);
    });
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free forward (no counterpart in the reference).  For callers
// that cannot allocate device memory -- a plugin whose host framework owns
// all allocations and passes only inputs and outputs, or code that must not
// call cudaMalloc -- the degree map goes to this fixed file-scope array.
// Host code never passes `g_noalloc_scratch` itself to a kernel: on the host
// that name is only a stand-in, so its device address is looked up per
// device with cudaGetSymbolAddress and cached.  Calls that overlap on the
// GPU share the array and race; the degree pass overwrites every value the
// aggregation reads, so stale contents from an earlier call do not matter.
// ---------------------------------------------------------------------------
#include <mutex>

namespace nsc {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[NSC_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (set-up on the
// first call per device).  Returns nullptr and sets the error on failure.
void* noalloc_scratch(const char* op) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        fail(NSC_ERR_LAUNCH_FAILED, "%s: no usable current device (%s)", op,
             cudaGetErrorString(e));
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            fail(NSC_ERR_LAUNCH_FAILED,
                 "%s: cudaGetSymbolAddress of the scratch array failed: %s", op,
                 cudaGetErrorString(e));
            return nullptr;
        }
        g_noalloc_ptr[dev] = p;
    }
    return g_noalloc_ptr[dev];
}

}  // namespace
}  // namespace nsc

extern "C" nsc_status nsc_metropolis_fwd_noalloc(
    const void* w_half, int w_dtype, int64_t w_channels, const void* img,
    int x_dtype, int64_t B, int64_t C, int64_t H, int64_t W,
    const int64_t* shifts, int64_t S, int use_box, double eps, void* Wx,
    void* d_hat, void* stream) {
    using namespace nsc;
    const char* op = "metropolis_aggregate_noalloc";
    ShiftTable st;
    nsc_status e = check_metro(op, w_channels, B, C, H, W, shifts, S, eps, &st);
    if (e) return e;
    if (B == 0 || C == 0 || H == 0 || W == 0) return ok();
    if (!valid_dtype(x_dtype))
        return fail(NSC_ERR_UNSUPPORTED_DTYPE, "%s: unsupported dtype", op);
    const double need = static_cast<double>(B) * static_cast<double>(w_channels) *
                        static_cast<double>(H) * static_cast<double>(W) *
                        (x_dtype == NSC_F64 ? 8.0 : 4.0);
    if (need > static_cast<double>(NSC_NOALLOC_SCRATCH_BYTES))
        return fail(NSC_ERR_INVALID_ARG,
                    "%s: the degree map needs %.0f bytes but the built-in "
                    "scratch holds %u (B * w_channels * H * W * %d); use "
                    "nsc_metropolis_fwd with a caller-allocated degree buffer",
                    op, need, NSC_NOALLOC_SCRATCH_BYTES,
                    x_dtype == NSC_F64 ? 8 : 4);
    void* scratch = noalloc_scratch(op);
    if (!scratch) return NSC_ERR_LAUNCH_FAILED;
    return nsc_metropolis_fwd(w_half, w_dtype, w_channels, img, x_dtype, B, C,
                              H, W, shifts, S, use_box, eps, Wx, d_hat, scratch,
                              stream);
}
