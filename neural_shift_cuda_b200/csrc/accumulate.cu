// accumulate.cu -- accumulate_uz forward / backward (generic path) and the
// row-band forward used when one image is split over several GPUs.
//
//   U(p) = sum_s w_s(p) x(p + d_s) + inv_s [p - d_s inside] w_s(p - d_s) x(p - d_s)
//   Z(p) = sum_s w_s(p)            + inv_s [p - d_s inside] w_s(p - d_s)
// (reference: ops.py:157-206, shift_ops_cuda.cu:256-458).
//
// Work split: one thread owns one pixel and NC channels.  A channel-broadcast
// weight (w_channels == 1) is loaded once per (pixel, shift) and applied to
// the NC channels in registers; a per-channel weight uses NC == 1.  The
// reference gives every output pixel its own CTA with one lane per shift and
// a shared-memory tree; here shifts are a sequential fp32 (fp64) register
// accumulation and adjacent lanes own adjacent pixels, so every weight load
// of a warp is one coalesced 128-byte row segment.
//
// The tiled TMA kernel in accumulate_fast.cuh takes over the forward when the
// geometry allows it; this file is the general path (any W, any alignment).

#include <algorithm>
#include <cstdlib>

#include "nsc_common.cuh"
#include "nsc_host.h"
#include "accumulate.h"

namespace nsc {
namespace {

constexpr int kBX = 32, kBY = 8;

// Row addressing of x.  Full image: circular rows.  Row band: x_ext holds
// R halo rows above and below the band, already wrapped, so no wrap.
struct XRows {
    int64_t H;      // rows of the x buffer
    int64_t off;    // buffer row of output row 0
    int wrap;       // 1: full image, circular rows
    __device__ __forceinline__ int64_t fwd(int64_t r) const {
        return wrap ? wrap1(r, H) : r + off;
    }
    __device__ __forceinline__ int64_t own(int64_t r) const {
        return wrap ? r : r + off;
    }
};

template <typename TX, typename TW, int NC>
__global__ void __launch_bounds__(kBX * kBY)
acc_fwd_kernel(const TX* __restrict__ x, const TW* __restrict__ w,
               typename Acc<TX>::type* __restrict__ U,
               typename Acc<TX>::type* __restrict__ Z, const ShiftTable st,
               int64_t B, int64_t C, int64_t Hout, int64_t W, int64_t Cw,
               XRows xr, int64_t groups, int64_t hb0, int64_t hb1) {
    using A = typename Acc<TX>::type;
    const int64_t wcol = static_cast<int64_t>(blockIdx.x) * kBX + threadIdx.x;
    const int64_t h = hb0 + static_cast<int64_t>(blockIdx.y) * kBY + threadIdx.y;
    if (wcol >= W || h >= hb1) return;
    const int64_t plane_x = xr.H * W;
    const int64_t plane_o = Hout * W;
    const int64_t cgroups = (Cw == 1) ? (C + NC - 1) / NC : C;
    for (int64_t g = blockIdx.z; g < groups; g += gridDim.z) {
        const int64_t b = g / cgroups;
        const int64_t cg = g % cgroups;
        const int64_t c0 = (Cw == 1) ? cg * NC : cg;
        const int64_t wc = (Cw == 1) ? 0 : cg;
        const int nc = (Cw == 1) ? static_cast<int>(C - c0 < NC ? C - c0 : NC) : 1;
        const TX* xb = x + (b * C + c0) * plane_x;
        A u[NC], z = A(0);
#pragma unroll
        for (int i = 0; i < NC; ++i) u[i] = A(0);
        for (int s = 0; s < st.S; ++s) {
            const int64_t dx = st.dx[s], dy = st.dy[s];
            const TW* ws = w + ((static_cast<int64_t>(s) * B + b) * Cw + wc) * plane_o;
            if (st.has_fwd(s)) {
                const A wv = ldg_acc<TW, A>(ws + h * W + wcol);
                const int64_t xo = xr.fwd(h + dx) * W + wrap1(wcol + dy, W);
#pragma unroll
                for (int i = 0; i < NC; ++i)
                    if (i < nc) u[i] += wv * ldg_acc<TX, A>(xb + i * plane_x + xo);
                z += wv;
            }
            if (st.has_inv(s)) {
                const bool per = st.has_per(s);   // full-image calls only
                const int64_t hm = per ? wrap1(h - dx, Hout) : h - dx;
                const int64_t wm = per ? wrap1(wcol - dy, W) : wcol - dy;
                if (per || (inb(hm, Hout) && inb(wm, W))) {
                    const A mv = ldg_acc<TW, A>(ws + hm * W + wm);
                    const int64_t mo = xr.own(hm) * W + wm;
#pragma unroll
                    for (int i = 0; i < NC; ++i)
                        if (i < nc) u[i] += mv * ldg_acc<TX, A>(xb + i * plane_x + mo);
                    z += mv;
                }
            }
        }
        const int64_t ob = (b * C + c0) * plane_o + h * W + wcol;
#pragma unroll
        for (int i = 0; i < NC; ++i)
            if (i < nc) {
                U[ob + i * plane_o] = u[i];
                Z[ob + i * plane_o] = z;
            }
    }
}

// Mirror contributions of the band's own weights to the R rows outside it.
// Each strip is (2, B, C, R, W); part 0 = U, part 1 = Z; the top strip
// targets rows row0-R .. row0-1, the bottom strip the R rows below the band.
// Both strips in one launch: a block owns kEX columns of one strip row
// (blockIdx.y enumerates the 2R strip rows, top strip first) and splits the
// row's shift list over kEK thread groups, whose partial sums meet in shared
// memory in a fixed order.  The shifts that can reach each strip row (has_inv
// and a mirror source row inside the band) are listed on the host, so a
// thread visits only those: for row t above the band, rows with dx <= t;
// below, dx > t - Hb.  The block stages, per listed shift, the element
// offsets of its mirror source row (weight plane and row, x row) and dy in
// shared memory, so the shift loop is a few adds and four loads; every load
// of an unrolled group is issued unconditionally (an out-of-image column
// reads the row's column 0 and the term is dropped by a select), so eight
// shifts' loads are in flight together.
constexpr int kEX = 64, kEK = 4;
constexpr int kEdgeRows = 64;        // 2R strip rows, R <= 32
constexpr int kEdgeList = 4096;
struct EdgeLists {
    int32_t off[kEdgeRows + 1];      // row rr lists s[off[rr] .. off[rr+1])
    int16_t s[kEdgeList];
};

template <typename TX, typename TW, int NC>
__global__ void __launch_bounds__(kEX * kEK)
acc_edges_kernel(const TX* __restrict__ x, const TW* __restrict__ w,
                 typename Acc<TX>::type* __restrict__ top_out,
                 typename Acc<TX>::type* __restrict__ bot_out, const ShiftTable st,
                 const EdgeLists lists,
                 int64_t B, int64_t C, int64_t Hb, int64_t W, int64_t Cw,
                 int64_t R, int64_t row0, int64_t Hg, int64_t groups) {
    using A = typename Acc<TX>::type;
    extern __shared__ __align__(16) unsigned char edge_smem[];
    const int rr = blockIdx.y;
    const int j0 = lists.off[rr];
    const int n = lists.off[rr + 1] - j0;
    int64_t* woff = reinterpret_cast<int64_t*>(edge_smem);
    int64_t* xoff = woff + n;
    int32_t* dys = reinterpret_cast<int32_t*>(xoff + n);
    __shared__ A part[kEK][NC + 1][kEX];
    const int k = threadIdx.y;
    const int tid = k * kEX + threadIdx.x;
    const bool top = rr < R;
    const int64_t e = top ? rr : rr - R;
    const int64_t t = top ? (e - R) : (Hb + e);   // target row, band-local
    const int64_t plane_x = (Hb + 2 * R) * W;
    const int64_t plane_o = Hb * W;
    const int64_t plane_e = R * W;
    const int64_t wstride = B * Cw * plane_o;     // one shift plane
    for (int i = tid; i < n; i += kEX * kEK) {
        const int s = lists.s[j0 + i];
        const int64_t ro = (t - st.dx[s]) * W - st.dy[s];   // mirror row, column -dy
        woff[i] = s * wstride + ro;
        xoff[i] = ro;
        dys[i] = st.dy[s];
    }
    __syncthreads();
    const int64_t wcol = static_cast<int64_t>(blockIdx.x) * kEX + threadIdx.x;
    const int64_t cgroups = (Cw == 1) ? (C + NC - 1) / NC : C;
    const bool active = wcol < W && inb(row0 + t, Hg);
    A* out = top ? top_out : bot_out;
    for (int64_t g = blockIdx.z; g < groups; g += gridDim.z) {
        const int64_t b = g / cgroups;
        const int64_t cg = g % cgroups;
        const int64_t c0 = (Cw == 1) ? cg * NC : cg;
        const int64_t wc = (Cw == 1) ? 0 : cg;
        const int nc = (Cw == 1) ? static_cast<int>(C - c0 < NC ? C - c0 : NC) : 1;
        const TW* wb = w + (b * Cw + wc) * plane_o + wcol;
        const TX* xc[NC];
#pragma unroll
        for (int i = 0; i < NC; ++i)   // band row 0 of channel c0 + i (clamped)
            xc[i] = x + (b * C + c0 + (i < nc ? i : 0)) * plane_x + R * W + wcol;
        A u[NC], z = A(0);
#pragma unroll
        for (int i = 0; i < NC; ++i) u[i] = A(0);
        if (active) {
#pragma unroll 8
            for (int j = k; j < n; j += kEK) {
                const int dy = dys[j];
                const bool ok = static_cast<uint64_t>(wcol - dy) < static_cast<uint64_t>(W);
                const int64_t adj = ok ? 0 : dy - wcol;
                const A mv0 = ldg_acc<TW, A>(wb + woff[j] + adj);
                A xv[NC];
#pragma unroll
                for (int i = 0; i < NC; ++i) xv[i] = ldg_acc<TX, A>(xc[i] + xoff[j] + adj);
                const A mv = ok ? mv0 : A(0);
#pragma unroll
                for (int i = 0; i < NC; ++i) u[i] += mv * (ok ? xv[i] : A(0));
                z += mv;
            }
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < NC; ++i) part[k][i][threadIdx.x] = u[i];
        part[k][NC][threadIdx.x] = z;
        __syncthreads();
        if (k == 0 && wcol < W) {
            A su[NC + 1];
#pragma unroll
            for (int i = 0; i <= NC; ++i) {
                su[i] = A(0);
#pragma unroll
                for (int j = 0; j < kEK; ++j) su[i] += part[j][i][threadIdx.x];
            }
            const int64_t ob = (b * C + c0) * plane_e + e * W + wcol;
            const int64_t zoff = B * C * plane_e;
#pragma unroll
            for (int i = 0; i < NC; ++i)
                if (i < nc) {
                    out[ob + i * plane_e] = su[i];
                    out[zoff + ob + i * plane_e] = su[NC];
                }
        }
    }
}

// Periodic mirror rows on the tiled path: the tile kernel treats every
// mirror term as masked (its weight boxes are zero outside the image), which
// is the periodic term wherever p - d stays inside the image.  This kernel
// adds the remaining wrapped terms -- w_s((p - d) mod (H, W)) x((p - d) mod)
// for periodic rows whose p - d leaves the image -- which exist only on the
// R-pixel border band.
template <typename TX, typename TW, int NC>
__global__ void __launch_bounds__(256)
acc_per_fix_kernel(const TX* __restrict__ x, const TW* __restrict__ w,
                   typename Acc<TX>::type* __restrict__ U,
                   typename Acc<TX>::type* __restrict__ Z, const ShiftTable st,
                   int64_t B, int64_t C, int64_t H, int64_t W, int64_t Cw, int64_t R,
                   int64_t nb, int64_t groups) {
    using A = typename Acc<TX>::type;
    const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
    if (i >= nb) return;
    int64_t h, wcol;
    border_pixel(i, H, W, R, h, wcol);
    const int64_t plane = H * W;
    const int64_t cgroups = (Cw == 1) ? (C + NC - 1) / NC : C;
    for (int64_t g = blockIdx.y; g < groups; g += gridDim.y) {
        const int64_t b = g / cgroups;
        const int64_t cg = g % cgroups;
        const int64_t c0 = (Cw == 1) ? cg * NC : cg;
        const int64_t wc = (Cw == 1) ? 0 : cg;
        const int nc = (Cw == 1) ? static_cast<int>(C - c0 < NC ? C - c0 : NC) : 1;
        const TX* xb = x + (b * C + c0) * plane;
        A u[NC], z = A(0);
#pragma unroll
        for (int k = 0; k < NC; ++k) u[k] = A(0);
        for (int s = 0; s < st.S; ++s) {
            if (!st.has_per(s)) continue;
            int64_t hm = h - st.dx[s], wm = wcol - st.dy[s];
            if (inb(hm, H) && inb(wm, W)) continue;     // counted by the tile kernel
            hm = wrap1(hm, H);
            wm = wrap1(wm, W);
            const TW* ws = w + ((static_cast<int64_t>(s) * B + b) * Cw + wc) * plane;
            const A mv = ldg_acc<TW, A>(ws + hm * W + wm);
#pragma unroll
            for (int k = 0; k < NC; ++k)
                if (k < nc) u[k] += mv * ldg_acc<TX, A>(xb + k * plane + hm * W + wm);
            z += mv;
        }
        const int64_t ob = (b * C + c0) * plane + h * W + wcol;
#pragma unroll
        for (int k = 0; k < NC; ++k)
            if (k < nc) {
                U[ob + k * plane] += u[k];
                Z[ob + k * plane] += z;
            }
    }
}

// After the tiled grad_x (accumulate_gx_tma.cuh): gx += the wrapped part of
// term A, sum_s [q - d outside] w_s((q - d) mod) gU((q - d) mod), for the
// pixels within R of the image border (one thread per pixel; the tile
// kernel counted q - d inside).
template <typename TW, int NC>
__global__ void __launch_bounds__(256)
acc_gx_wrap_kernel(const float* __restrict__ gU, const TW* __restrict__ w,
                   float* __restrict__ gx, const ShiftTable st, int64_t B, int64_t C,
                   int64_t H, int64_t W, int64_t Cw, int64_t R, int64_t nb, int64_t groups) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
    if (i >= nb) return;
    int64_t h, wcol;
    border_pixel(i, H, W, R, h, wcol);
    const int64_t plane = H * W;
    const int64_t cgroups = (Cw == 1) ? (C + NC - 1) / NC : C;
    for (int64_t g = blockIdx.y; g < groups; g += gridDim.y) {
        const int64_t b = g / cgroups;
        const int64_t cg = g % cgroups;
        const int64_t c0 = (Cw == 1) ? cg * NC : cg;
        const int64_t wc = (Cw == 1) ? 0 : cg;
        const int nc = (Cw == 1) ? static_cast<int>(C - c0 < NC ? C - c0 : NC) : 1;
        const float* gb = gU + (b * C + c0) * plane;
        float u[NC];
#pragma unroll
        for (int k = 0; k < NC; ++k) u[k] = 0.f;
        for (int s = 0; s < st.S; ++s) {
            int64_t hm = h - st.dx[s], wm = wcol - st.dy[s];
            if (inb(hm, H) && inb(wm, W)) continue;     // counted by the tile kernel
            hm = wrap1(hm, H);
            wm = wrap1(wm, W);
            const TW* ws = w + ((static_cast<int64_t>(s) * B + b) * Cw + wc) * plane;
            const float mv = ldg_acc<TW, float>(ws + hm * W + wm);
#pragma unroll
            for (int k = 0; k < NC; ++k)
                if (k < nc) u[k] += mv * gb[k * plane + hm * W + wm];
        }
        const int64_t ob = (b * C + c0) * plane + h * W + wcol;
#pragma unroll
        for (int k = 0; k < NC; ++k)
            if (k < nc) gx[ob + k * plane] += u[k];
    }
}

// U/Z += neighbour strips; one thread per strip element and strip.
template <typename A>
__global__ void __launch_bounds__(256)
band_add_strips_kernel(A* __restrict__ U, A* __restrict__ Z,
                       const A* __restrict__ above, const A* __restrict__ below,
                       int64_t planes, int64_t Hb, int64_t W, int64_t R) {
    const int64_t n = planes * R * W;                 // elements per part
    const int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x;
    if (i >= n) return;
    const int64_t p = i / (R * W);
    const int64_t rw = i - p * R * W;                  // r * W + w
    const A* src = blockIdx.y == 0 ? above : below;
    if (!src) return;
    const int64_t dst = p * Hb * W + (blockIdx.y == 0 ? 0 : (Hb - R) * W) + rw;
    U[dst] += src[i];
    Z[dst] += src[n + i];
}

// Fused backward: thread owns pixel q and NC channels.
//   gx(q)   = sum_s w_s(q-d) gU(q-d) [circular] + inv [q+d inside] w_s(q) gU(q+d)
//   gw_s(q) = sum_c x(q+d) gU(q) + gZ(q) + inv [q+d inside] (x(q) gU(q+d) + gZ(q+d))
// One pass over the weight stack reads w once (plus the shifted re-read,
// served by L1/L2) and writes grad_w once.  GW == false skips grad_w: a
// channel-broadcast weight with more than NC channels needs the sum over
// every channel group, which acc_bwd_gw_bcast_kernel forms instead.
template <typename TX, typename TW, int NC, bool GW>
__global__ void __launch_bounds__(kBX * kBY)
acc_bwd_kernel(const TX* __restrict__ x, const TW* __restrict__ w,
               const typename Acc<TX>::type* __restrict__ gU,
               const typename Acc<TX>::type* __restrict__ gZ,
               typename Acc<TX>::type* __restrict__ gx, TW* __restrict__ gw,
               const ShiftTable st, int64_t B, int64_t C, int64_t H,
               int64_t W, int64_t Cw, int64_t groups) {
    using A = typename Acc<TX>::type;
    const int64_t wcol = static_cast<int64_t>(blockIdx.x) * kBX + threadIdx.x;
    const int64_t h = static_cast<int64_t>(blockIdx.y) * kBY + threadIdx.y;
    if (wcol >= W || h >= H) return;
    const int64_t plane = H * W;
    const int64_t q = h * W + wcol;
    const int64_t cgroups = (Cw == 1) ? (C + NC - 1) / NC : C;
    for (int64_t g = blockIdx.z; g < groups; g += gridDim.z) {
        const int64_t b = g / cgroups;
        const int64_t cg = g % cgroups;
        const int64_t c0 = (Cw == 1) ? cg * NC : cg;
        const int64_t wc = (Cw == 1) ? 0 : cg;
        const int nc = (Cw == 1) ? static_cast<int>(C - c0 < NC ? C - c0 : NC) : 1;
        const int64_t cb = (b * C + c0) * plane;
        A xq[NC], acc[NC];
#pragma unroll
        for (int i = 0; i < NC; ++i) {
            acc[i] = A(0);
            xq[i] = (i < nc) ? ldg_acc<TX, A>(x + cb + i * plane + q) : A(0);
        }
        A gu_q[NC], gz_q = A(0);
#pragma unroll
        for (int i = 0; i < NC; ++i) {
            gu_q[i] = (i < nc) ? gU[cb + i * plane + q] : A(0);
            if (i < nc) gz_q += gZ[cb + i * plane + q];
        }
        for (int s = 0; s < st.S; ++s) {
            const int64_t dx = st.dx[s], dy = st.dy[s];
            const int64_t wbase = ((static_cast<int64_t>(s) * B + b) * Cw + wc) * plane;
            const TW* ws = w + wbase;
            A gws = A(0);
            if (st.has_fwd(s)) {
                // forward term of output q - d (circular) reads x(q)
                const int64_t qs = wrap1(h - dx, H) * W + wrap1(wcol - dy, W);
                const A w_src = ldg_acc<TW, A>(ws + qs);
                // grad_w forward part: x(q+d) gU(q) + gZ(q)
                const int64_t qf = wrap1(h + dx, H) * W + wrap1(wcol + dy, W);
                gws = gz_q;
#pragma unroll
                for (int i = 0; i < NC; ++i)
                    if (i < nc) {
                        acc[i] += w_src * gU[cb + i * plane + qs];
                        gws += ldg_acc<TX, A>(x + cb + i * plane + qf) * gu_q[i];
                    }
            }
            if (st.has_inv(s) && (st.has_per(s) || (inb(h + dx, H) && inb(wcol + dy, W)))) {
                const A w_q = ldg_acc<TW, A>(ws + q);
                const int64_t qi = wrap1(h + dx, H) * W + wrap1(wcol + dy, W);
#pragma unroll
                for (int i = 0; i < NC; ++i)
                    if (i < nc) {
                        const A g = gU[cb + i * plane + qi];
                        acc[i] += w_q * g;
                        gws += xq[i] * g + gZ[cb + i * plane + qi];
                    }
            }
            if (GW) gw[wbase + q] = static_cast<TW>(gws);
        }
#pragma unroll
        for (int i = 0; i < NC; ++i)
            if (i < nc) gx[cb + i * plane + q] = acc[i];
    }
}

// grad_w of a channel-broadcast weight (w_channels == 1) for any C: the
// thread owns pixel q of image b and sums the C channels in a loop, so one
// thread writes each gw_s(q) exactly once.
template <typename TX, typename TW>
__global__ void __launch_bounds__(kBX * kBY)
acc_bwd_gw_bcast_kernel(const TX* __restrict__ x,
                        const typename Acc<TX>::type* __restrict__ gU,
                        const typename Acc<TX>::type* __restrict__ gZ,
                        TW* __restrict__ gw, const ShiftTable st, int64_t B,
                        int64_t C, int64_t H, int64_t W) {
    using A = typename Acc<TX>::type;
    const int64_t wcol = static_cast<int64_t>(blockIdx.x) * kBX + threadIdx.x;
    const int64_t h = static_cast<int64_t>(blockIdx.y) * kBY + threadIdx.y;
    if (wcol >= W || h >= H) return;
    const int64_t plane = H * W;
    const int64_t q = h * W + wcol;
    for (int64_t b = blockIdx.z; b < B; b += gridDim.z) {
        const int64_t cb = b * C * plane;
        for (int s = 0; s < st.S; ++s) {
            const int64_t dx = st.dx[s], dy = st.dy[s];
            const int64_t qf = wrap1(h + dx, H) * W + wrap1(wcol + dy, W);
            const bool mir = st.has_inv(s) &&
                             (st.has_per(s) || (inb(h + dx, H) && inb(wcol + dy, W)));
            const bool fwd = st.has_fwd(s);
            A gws = A(0);
            for (int64_t c = 0; c < C; ++c) {
                const int64_t co = cb + c * plane;
                if (fwd) gws += ldg_acc<TX, A>(x + co + qf) * gU[co + q] + gZ[co + q];
                if (mir)
                    gws += ldg_acc<TX, A>(x + co + q) * gU[co + qf] + gZ[co + qf];
            }
            gw[(static_cast<int64_t>(s) * B + b) * plane + q] = static_cast<TW>(gws);
        }
    }
}

template <int NC> struct NCTag { static constexpr int value_nc = NC; };

// Dispatch helpers over (TX, TW) and NC.
template <typename F>
nsc_status with_types(const char* op, int xd, int wd, F&& f) {
    if (xd == NSC_F64 && wd == NSC_F64) return f((const double*)nullptr, (const double*)nullptr);
    if (xd == NSC_F32 && wd == NSC_F32) return f((const float*)nullptr, (const float*)nullptr);
    if (xd == NSC_F16 && wd == NSC_F16) return f((const __half*)nullptr, (const __half*)nullptr);
    if (xd == NSC_BF16 && wd == NSC_BF16)
        return f((const __nv_bfloat16*)nullptr, (const __nv_bfloat16*)nullptr);
    if (xd == NSC_F32 && wd == NSC_F16) return f((const float*)nullptr, (const __half*)nullptr);
    if (xd == NSC_F32 && wd == NSC_BF16)
        return f((const float*)nullptr, (const __nv_bfloat16*)nullptr);
    return fail(NSC_ERR_UNSUPPORTED_DTYPE,
                "%s: unsupported dtype pair (x=%d, w=%d); use equal dtypes, "
                "fp32 x with fp16/bf16 weights, or fp64 for both", op, xd, wd);
}

template <typename F>
void with_nc(int64_t C, int64_t Cw, F&& f) {
    const int64_t nc = (Cw == 1) ? C : 1;
    if (nc >= 4) f(NCTag<4>{});
    else if (nc == 3) f(NCTag<3>{});
    else if (nc == 2) f(NCTag<2>{});
    else f(NCTag<1>{});
}

inline int64_t n_groups(int64_t B, int64_t C, int64_t Cw, int nc) {
    return B * ((Cw == 1) ? (C + nc - 1) / nc : C);
}

inline dim3 grid_for(int64_t W, int64_t rows, int64_t groups) {
    return dim3(grid_1d(W, kBX), grid_1d(rows, kBY),
                static_cast<unsigned>(groups < 65535 ? groups : 65535));
}

nsc_status check_common(const char* op, int xd, int wd, int64_t Cw, int64_t B,
                        int64_t C, int64_t H, int64_t W, const int64_t* shifts,
                        int64_t S, ShiftTable* st) {
    nsc_status e = check_extents(op, B, C, H, W);
    if (e) return e;
    if (acc_dtype(xd, wd) < 0)
        return fail(NSC_ERR_UNSUPPORTED_DTYPE,
                    "%s: unsupported dtype pair (x=%d, w=%d)", op, xd, wd);
    if (!(Cw == C || (Cw == 1 && C >= 1)))
        return fail(NSC_ERR_INVALID_ARG,
                    "%s: weights must be (S*B, C, H, W) or channel-broadcast "
                    "(S*B, 1, H, W); got w_channels=%lld with C=%lld",
                    op, (long long)Cw, (long long)C);
    return build_shifts(op, shifts, S, 3, H, W, st);
}

}  // namespace

// ---------------------------------------------------------------------------
nsc_status acc_fwd_generic(const void* x, int xd, const void* w, int wd,
                           int64_t Cw, int64_t B, int64_t C, int64_t Hout,
                           int64_t W, int64_t x_rows, int64_t x_off, int wrap,
                           const ShiftTable& st, void* U, void* Z,
                           cudaStream_t stream, int64_t h_begin, int64_t h_end) {
    if (h_end < 0) h_end = Hout;
    XRows xr{x_rows, x_off, wrap};
    return with_types("accumulate_uz", xd, wd, [&](auto tx, auto tw) {
        using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
        using TW = std::remove_const_t<std::remove_pointer_t<decltype(tw)>>;
        using A = typename Acc<TX>::type;
        with_nc(C, Cw, [&](auto tag) {
            constexpr int NC = decltype(tag)::value_nc;
            const int64_t groups = n_groups(B, C, Cw, NC);
            if (h_end <= h_begin) return;
            acc_fwd_kernel<TX, TW, NC><<<grid_for(W, h_end - h_begin, groups),
                                          dim3(kBX, kBY), 0, stream>>>(
                static_cast<const TX*>(x), static_cast<const TW*>(w),
                static_cast<A*>(U), static_cast<A*>(Z), st, B, C, Hout, W, Cw,
                xr, groups, h_begin, h_end);
        });
        return check_launch("accumulate_uz");
    });
}


nsc_status acc_per_fix(const void* x, int xd, const void* w, int wd, int64_t Cw,
                       int64_t B, int64_t C, int64_t H, int64_t W, const ShiftTable& st,
                       void* U, void* Z, cudaStream_t stream) {
    const int64_t R = st.R;
    const int64_t nb = border_count(H, W, R);
    return with_types("accumulate_uz", xd, wd, [&](auto tx, auto tw) {
        using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
        using TW = std::remove_const_t<std::remove_pointer_t<decltype(tw)>>;
        using A = typename Acc<TX>::type;
        with_nc(C, Cw, [&](auto tag) {
            constexpr int NC = decltype(tag)::value_nc;
            const int64_t groups = n_groups(B, C, Cw, NC);
            const dim3 grid(grid_1d(nb, 256),
                            static_cast<unsigned>(groups < 65535 ? groups : 65535));
            acc_per_fix_kernel<TX, TW, NC><<<grid, 256, 0, stream>>>(
                static_cast<const TX*>(x), static_cast<const TW*>(w), static_cast<A*>(U),
                static_cast<A*>(Z), st, B, C, H, W, Cw, R, nb, groups);
        });
        return check_launch("accumulate_uz");
    });
}

nsc_status acc_gx_wrap(const void* w, int wd, int64_t Cw, int64_t B, int64_t C,
                       int64_t H, int64_t W, const ShiftTable& st, const void* gU,
                       void* gx, cudaStream_t stream) {
    const int64_t R = st.R;
    const int64_t nb = border_count(H, W, R);
    if (nb == 0) return ok();
    return with_types("accumulate_uz_backward", NSC_F32, wd, [&](auto, auto tw) {
        using TW = std::remove_const_t<std::remove_pointer_t<decltype(tw)>>;
        with_nc(C, Cw, [&](auto tag) {
            constexpr int NC = decltype(tag)::value_nc;
            const int64_t groups = n_groups(B, C, Cw, NC);
            const dim3 grid(grid_1d(nb, 256),
                            static_cast<unsigned>(groups < 65535 ? groups : 65535));
            acc_gx_wrap_kernel<TW, NC><<<grid, 256, 0, stream>>>(
                static_cast<const float*>(gU), static_cast<const TW*>(w),
                static_cast<float*>(gx), st, B, C, H, W, Cw, R, nb, groups);
        });
        return check_launch("accumulate_uz_backward");
    });
}

nsc_status acc_edges(const void* x, int xd, const void* w, int wd, int64_t Cw,
                     int64_t B, int64_t C, int64_t Hb, int64_t W, int64_t row0,
                     int64_t Hg, const ShiftTable& st, void* top, void* bot,
                     cudaStream_t stream) {
    const int64_t R = st.R;
    if (2 * R > kEdgeRows)
        return fail(NSC_ERR_INVALID_ARG,
                    "accumulate_uz_band_edges: table radius %lld > %d", (long long)R,
                    kEdgeRows / 2);
    EdgeLists lists;
    int n = 0;
    for (int64_t rr = 0; rr < 2 * R; ++rr) {
        lists.off[rr] = n;
        const int64_t t = rr < R ? rr - R : Hb + (rr - R);   // band-local target row
        for (int s = 0; s < st.S; ++s) {
            if (!st.has_inv(s)) continue;
            const int64_t hm = t - st.dx[s];
            if (hm < 0 || hm >= Hb) continue;
            if (n >= kEdgeList)
                return fail(NSC_ERR_INVALID_ARG,
                            "accumulate_uz_band_edges: more than %d (row, shift) "
                            "pairs reach the strips", kEdgeList);
            lists.s[n++] = static_cast<int16_t>(s);
        }
    }
    lists.off[2 * R] = n;
    int maxn = 0;
    for (int64_t rr = 0; rr < 2 * R; ++rr)
        maxn = std::max(maxn, lists.off[rr + 1] - lists.off[rr]);
    const size_t smem = static_cast<size_t>(maxn) * 20;   // woff, xoff, dy
    return with_types("accumulate_uz_band_edges", xd, wd, [&](auto tx, auto tw) {
        using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
        using TW = std::remove_const_t<std::remove_pointer_t<decltype(tw)>>;
        using A = typename Acc<TX>::type;
        if (R == 0) return ok();
        with_nc(C, Cw, [&](auto tag) {
            constexpr int NC = decltype(tag)::value_nc;
            const int64_t groups = n_groups(B, C, Cw, NC);
            const dim3 grid(grid_1d(W, kEX), static_cast<unsigned>(2 * R),
                            static_cast<unsigned>(groups < 65535 ? groups : 65535));
            acc_edges_kernel<TX, TW, NC><<<grid, dim3(kEX, kEK), smem, stream>>>(
                static_cast<const TX*>(x), static_cast<const TW*>(w),
                static_cast<A*>(top), static_cast<A*>(bot), st, lists, B, C, Hb, W,
                Cw, R, row0, Hg, groups);
        });
        return check_launch("accumulate_uz_band_edges");
    });
}

nsc_status acc_bwd(const void* x, int xd, const void* w, int wd, int64_t Cw,
                   int64_t B, int64_t C, int64_t H, int64_t W,
                   const ShiftTable& st, const void* gU, const void* gZ,
                   void* gx, void* gw, cudaStream_t stream) {
    // grad_w by the tiled correlation kernel when it takes the call; the
    // general kernel then computes grad_x only
    const bool gw_done = acc_gw_fast(x, xd, wd, Cw, B, C, H, W, st, gU, gZ, gw, stream);
    if (gw_done && acc_gx_fast(w, xd, wd, Cw, B, C, H, W, st, gU, gx, stream))
        return check_launch("accumulate_uz_backward");
    if (std::getenv("NSC_REQUIRE_FAST"))
        return fail(NSC_ERR_INVALID_ARG,
                    "accumulate_uz_backward: a tiled kernel declined this call "
                    "(NSC_REQUIRE_FAST is set): %s", gw_done ? fast_decline_reason()
                                                             : "grad_w");
    return with_types("accumulate_uz_backward", xd, wd, [&](auto tx, auto tw) {
        using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
        using TW = std::remove_const_t<std::remove_pointer_t<decltype(tw)>>;
        using A = typename Acc<TX>::type;
        with_nc(C, Cw, [&](auto tag) {
            constexpr int NC = decltype(tag)::value_nc;
            const int64_t groups = n_groups(B, C, Cw, NC);
            if (gw_done) {
                acc_bwd_kernel<TX, TW, NC, false><<<grid_for(W, H, groups),
                                                     dim3(kBX, kBY), 0, stream>>>(
                    static_cast<const TX*>(x), static_cast<const TW*>(w),
                    static_cast<const A*>(gU), static_cast<const A*>(gZ),
                    static_cast<A*>(gx), static_cast<TW*>(gw), st, B, C, H, W, Cw,
                    groups);
            } else if (Cw == 1 && C > NC) {
                acc_bwd_kernel<TX, TW, NC, false><<<grid_for(W, H, groups),
                                                     dim3(kBX, kBY), 0, stream>>>(
                    static_cast<const TX*>(x), static_cast<const TW*>(w),
                    static_cast<const A*>(gU), static_cast<const A*>(gZ),
                    static_cast<A*>(gx), static_cast<TW*>(gw), st, B, C, H, W, Cw,
                    groups);
                acc_bwd_gw_bcast_kernel<TX, TW><<<grid_for(W, H, B), dim3(kBX, kBY),
                                                   0, stream>>>(
                    static_cast<const TX*>(x), static_cast<const A*>(gU),
                    static_cast<const A*>(gZ), static_cast<TW*>(gw), st, B, C, H, W);
            } else {
                acc_bwd_kernel<TX, TW, NC, true><<<grid_for(W, H, groups),
                                                    dim3(kBX, kBY), 0, stream>>>(
                    static_cast<const TX*>(x), static_cast<const TW*>(w),
                    static_cast<const A*>(gU), static_cast<const A*>(gZ),
                    static_cast<A*>(gx), static_cast<TW*>(gw), st, B, C, H, W, Cw,
                    groups);
            }
        });
        return check_launch("accumulate_uz_backward");
    });
}

}  // namespace nsc

// ---------------------------------------------------------------------------
// C entry points
// ---------------------------------------------------------------------------
extern "C" {

nsc_status nsc_accumulate_uz_fwd(const void* x, int x_dtype, const void* w,
                                 int w_dtype, int64_t w_channels, int64_t B,
                                 int64_t C, int64_t H, int64_t W,
                                 const int64_t* shifts, int64_t S, void* U,
                                 void* Z, void* stream) {
    using namespace nsc;
    ShiftTable st;
    nsc_status e = check_common("accumulate_uz", x_dtype, w_dtype, w_channels,
                                B, C, H, W, shifts, S, &st);
    if (e) return e;
    if (B == 0 || C == 0 || H == 0 || W == 0) return ok();
    if (!x || !w || !U || !Z)
        return fail(NSC_ERR_INVALID_ARG, "accumulate_uz: NULL tensor pointer");
    if (acc_fwd_fast(x, x_dtype, w, w_dtype, w_channels, B, C, H, W, H, 0, 1,
                     st, U, Z, as_stream(stream))) {
        if (st.any_per)   // wrapped periodic mirror terms of the border band
            return acc_per_fix(x, x_dtype, w, w_dtype, w_channels, B, C, H, W, st, U, Z,
                               as_stream(stream));
        return check_launch("accumulate_uz");
    }
    if (std::getenv("NSC_REQUIRE_FAST"))
        return fail(NSC_ERR_INVALID_ARG,
                    "accumulate_uz: the tiled path declined this call "
                    "(NSC_REQUIRE_FAST is set): %s", fast_decline_reason());
    return acc_fwd_generic(x, x_dtype, w, w_dtype, w_channels, B, C, H, W, H, 0,
                           1, st, U, Z, as_stream(stream));
}

nsc_status nsc_accumulate_uz_bwd(const void* x, int x_dtype, const void* w,
                                 int w_dtype, int64_t w_channels, int64_t B,
                                 int64_t C, int64_t H, int64_t W,
                                 const int64_t* shifts, int64_t S,
                                 const void* grad_U, const void* grad_Z,
                                 void* grad_x, void* grad_w, void* stream) {
    using namespace nsc;
    ShiftTable st;
    nsc_status e = check_common("accumulate_uz_backward", x_dtype, w_dtype,
                                w_channels, B, C, H, W, shifts, S, &st);
    if (e) return e;
    if (B == 0 || C == 0 || H == 0 || W == 0) return ok();
    if (!x || !w || !grad_U || !grad_Z || !grad_x || !grad_w)
        return fail(NSC_ERR_INVALID_ARG,
                    "accumulate_uz_backward: NULL tensor pointer");
    return acc_bwd(x, x_dtype, w, w_dtype, w_channels, B, C, H, W, st, grad_U,
                   grad_Z, grad_x, grad_w, as_stream(stream));
}

static nsc_status band_checks(const char* op, int64_t Hb, int64_t row0,
                              int64_t Hg, const nsc::ShiftTable& st) {
    using namespace nsc;
    if (Hg < 1 || row0 < 0 || Hb < 0 || row0 + Hb > Hg)
        return fail(NSC_ERR_INVALID_ARG,
                    "%s: band rows [%lld, %lld) outside image of %lld rows", op,
                    (long long)row0, (long long)(row0 + Hb), (long long)Hg);
    for (int s = 0; s < st.S; ++s)
        if (st.dx[s] > Hg || -st.dx[s] > Hg)
            return fail(NSC_ERR_INVALID_ARG, "%s: |dx| exceeds image rows", op);
    if (st.R > Hb)
        return fail(NSC_ERR_INVALID_ARG,
                    "%s: band of %lld rows is thinner than the radius %d", op,
                    (long long)Hb, st.R);
    if (st.any_per)
        return fail(NSC_ERR_INVALID_ARG,
                    "%s: periodic mirror rows (column value 2) are not supported "
                    "by the row-band split", op);
    return ok();
}

nsc_status nsc_accumulate_uz_band_fwd(const void* x_ext, int x_dtype,
                                      const void* w, int w_dtype,
                                      int64_t w_channels, int64_t B, int64_t C,
                                      int64_t Hb, int64_t W, int64_t row0,
                                      int64_t Hg, const int64_t* shifts,
                                      int64_t S, void* U, void* Z,
                                      void* stream) {
    using namespace nsc;
    ShiftTable st;
    // dx is checked against the global height; dy against W.
    nsc_status e = check_common("accumulate_uz_band", x_dtype, w_dtype,
                                w_channels, B, C, Hg, W, shifts, S, &st);
    if (e) return e;
    e = band_checks("accumulate_uz_band", Hb, row0, Hg, st);
    if (e) return e;
    if (B == 0 || C == 0 || Hb == 0 || W == 0) return ok();
    if (!x_ext || !w || !U || !Z)
        return fail(NSC_ERR_INVALID_ARG, "accumulate_uz_band: NULL tensor pointer");
    const int64_t R = st.R;
    if (acc_fwd_fast(x_ext, x_dtype, w, w_dtype, w_channels, B, C, Hb, W,
                     Hb + 2 * R, R, 0, st, U, Z, as_stream(stream)))
        return check_launch("accumulate_uz_band");
    return acc_fwd_generic(x_ext, x_dtype, w, w_dtype, w_channels, B, C, Hb, W,
                           Hb + 2 * R, R, 0, st, U, Z, as_stream(stream));
}

nsc_status nsc_accumulate_uz_band_rows_fwd(const void* x_ext, int x_dtype,
                                           const void* w, int w_dtype,
                                           int64_t w_channels, int64_t B, int64_t C,
                                           int64_t Hb, int64_t W, int64_t row0,
                                           int64_t Hg, int64_t r_begin, int64_t r_end,
                                           int max_ctas, const int64_t* shifts,
                                           int64_t S, void* U, void* Z,
                                           void* stream) {
    using namespace nsc;
    const char* op = "accumulate_uz_band_rows";
    ShiftTable st;
    nsc_status e = check_common(op, x_dtype, w_dtype, w_channels, B, C, Hg, W,
                                shifts, S, &st);
    if (e) return e;
    e = band_checks(op, Hb, row0, Hg, st);
    if (e) return e;
    if (r_begin < 0 || r_begin > r_end || r_end > Hb)
        return fail(NSC_ERR_INVALID_ARG, "%s: rows [%lld, %lld) outside the band of %lld",
                    op, (long long)r_begin, (long long)r_end, (long long)Hb);
    if (max_ctas < 0) return fail(NSC_ERR_INVALID_ARG, "%s: max_ctas < 0", op);
    if (B == 0 || C == 0 || W == 0 || r_begin == r_end) return ok();
    if (!x_ext || !w || !U || !Z)
        return fail(NSC_ERR_INVALID_ARG, "%s: NULL tensor pointer", op);
    const int64_t R = st.R;
    if (acc_fwd_fast(x_ext, x_dtype, w, w_dtype, w_channels, B, C, Hb, W,
                     Hb + 2 * R, R, 0, st, U, Z, as_stream(stream), 0, nullptr,
                     r_begin, r_end, max_ctas))
        return check_launch(op);
    return acc_fwd_generic(x_ext, x_dtype, w, w_dtype, w_channels, B, C, Hb, W,
                           Hb + 2 * R, R, 0, st, U, Z, as_stream(stream), r_begin, r_end);
}

nsc_status nsc_accumulate_uz_band_edges(const void* x_ext, int x_dtype,
                                        const void* w, int w_dtype,
                                        int64_t w_channels, int64_t B,
                                        int64_t C, int64_t Hb, int64_t W,
                                        int64_t row0, int64_t Hg,
                                        const int64_t* shifts, int64_t S,
                                        void* edge_top, void* edge_bot,
                                        void* stream) {
    using namespace nsc;
    ShiftTable st;
    nsc_status e = check_common("accumulate_uz_band_edges", x_dtype, w_dtype,
                                w_channels, B, C, Hg, W, shifts, S, &st);
    if (e) return e;
    e = band_checks("accumulate_uz_band_edges", Hb, row0, Hg, st);
    if (e) return e;
    if (B == 0 || C == 0 || Hb == 0 || W == 0 || st.R == 0) return ok();
    if (!x_ext || !w || !edge_top || !edge_bot)
        return fail(NSC_ERR_INVALID_ARG,
                    "accumulate_uz_band_edges: NULL tensor pointer");
    return acc_edges(x_ext, x_dtype, w, w_dtype, w_channels, B, C, Hb, W, row0,
                     Hg, st, edge_top, edge_bot, as_stream(stream));
}

}  // extern "C"

extern "C" nsc_status nsc_accumulate_uz_band_add_strips(
    void* U, void* Z, int acc_dtype, int64_t B, int64_t C, int64_t Hb, int64_t W,
    int64_t R, const void* strip_above, const void* strip_below, void* stream) {
    using namespace nsc;
    const char* op = "accumulate_uz_band_add_strips";
    if (acc_dtype != NSC_F32 && acc_dtype != NSC_F64)
        return fail(NSC_ERR_UNSUPPORTED_DTYPE, "%s: acc_dtype must be fp32 or fp64", op);
    if (B < 0 || C < 0 || Hb < 0 || W < 0 || R < 0 || R > Hb)
        return fail(NSC_ERR_INVALID_ARG, "%s: bad extents (R must be <= Hb)", op);
    if (B == 0 || C == 0 || W == 0 || R == 0 || (!strip_above && !strip_below)) return ok();
    if (!U || !Z) return fail(NSC_ERR_INVALID_ARG, "%s: NULL tensor pointer", op);
    const int64_t n = B * C * R * W;
    const dim3 grid(grid_1d(n, 256), 2);
    if (acc_dtype == NSC_F32)
        band_add_strips_kernel<float><<<grid, 256, 0, as_stream(stream)>>>(
            static_cast<float*>(U), static_cast<float*>(Z),
            static_cast<const float*>(strip_above), static_cast<const float*>(strip_below),
            B * C, Hb, W, R);
    else
        band_add_strips_kernel<double><<<grid, 256, 0, as_stream(stream)>>>(
            static_cast<double*>(U), static_cast<double*>(Z),
            static_cast<const double*>(strip_above), static_cast<const double*>(strip_below),
            B * C, Hb, W, R);
    return check_launch(op);
}
