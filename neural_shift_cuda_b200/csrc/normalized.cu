// normalized.cu -- normalized_accumulate_uz forward / backward.
//
// D(p) = sum a_i x_i / sum a_i over the keys of output p (forward term of
// every shift plus the mirror term of has_inv rows inside the image), with
// a_i = exp(l_i - m) for logits (log_weights) or w_i / m for positive
// weights, m the row maximum; log_C = (m or log m) + log(sum a_i).
// Semantics follow the reference kernels (shift_ops_cuda.cu:460-791):
// masked keys (-inf logit, zero weight) contribute nothing; a row with no
// live key gives D = 0, log_C = -inf; a NaN key, a negative positive weight
// or a +inf key make D and log_C NaN.
//
// The reference makes two block-wide tree passes per output (max, then
// sums).  Here one thread streams the S keys once with a running maximum:
// whenever a key exceeds the current maximum the partial sums are rescaled
// by exp(m_old - m_new) (w_old / w_new in positive mode), the recurrence of
// online softmax (Milakov & Gimelshein, 2018).  A channel-broadcast weight
// (w_channels == 1) shares one key sequence -- one exponential per key --
// across the NC channels a thread owns.

#include <cmath>

#include "nsc_common.cuh"
#include "normalized_fast.h"
#include "nsc_host.h"
#include "accumulate.h"

namespace nsc {
namespace {

constexpr int kBX = 32, kBY = 8;

__device__ __forceinline__ float exp_acc(float v) { return expf(v); }
__device__ __forceinline__ double exp_acc(double v) { return exp(v); }
__device__ __forceinline__ float log_acc(float v) { return logf(v); }
__device__ __forceinline__ double log_acc(double v) { return log(v); }

template <typename A>
__device__ __forceinline__ A neg_inf() { return -INFINITY; }

template <typename A, int NC>
struct Online {
    A m, sz, su[NC];
    bool bad;
    __device__ __forceinline__ void init() {
        m = neg_inf<A>();
        sz = A(0);
        bad = false;
#pragma unroll
        for (int i = 0; i < NC; ++i) su[i] = A(0);
    }
    // k: raw weight (positive mode) or logit; xv: the key's values.
    __device__ __forceinline__ void push(A k, const A (&xv)[NC], bool logw) {
        if (k != k) { bad = true; return; }
        if (logw) {
            if (k == neg_inf<A>()) return;
        } else {
            if (k < A(0)) { bad = true; return; }
            if (k == A(0)) return;
        }
        if (k > m) {
            const A f = (m == neg_inf<A>()) ? A(0)
                        : (logw ? exp_acc(m - k) : m / k);
            sz *= f;
#pragma unroll
            for (int i = 0; i < NC; ++i) su[i] *= f;
            m = k;
        }
        const A a = logw ? exp_acc(k - m) : k / m;
        sz += a;
#pragma unroll
        for (int i = 0; i < NC; ++i) su[i] += a * xv[i];
    }
};

template <typename TX, typename TW, int NC>
__global__ void __launch_bounds__(kBX * kBY)
norm_fwd_kernel(const TX* __restrict__ x, const TW* __restrict__ w,
                typename Acc<TX>::type* __restrict__ D,
                typename Acc<TX>::type* __restrict__ L, const ShiftTable st,
                int64_t B, int64_t C, int64_t H, int64_t W, int64_t Cw,
                int logw, int* __restrict__ invalid, int64_t groups) {
    using A = typename Acc<TX>::type;
    const int64_t wcol = static_cast<int64_t>(blockIdx.x) * kBX + threadIdx.x;
    const int64_t h = static_cast<int64_t>(blockIdx.y) * kBY + threadIdx.y;
    if (wcol >= W || h >= H) return;
    const int64_t plane = H * W;
    const int64_t cgroups = (Cw == 1) ? (C + NC - 1) / NC : C;
    bool seen_invalid = false;
    for (int64_t g = blockIdx.z; g < groups; g += gridDim.z) {
        const int64_t b = g / cgroups;
        const int64_t cg = g % cgroups;
        const int64_t c0 = (Cw == 1) ? cg * NC : cg;
        const int64_t wc = (Cw == 1) ? 0 : cg;
        const int nc = (Cw == 1) ? static_cast<int>(C - c0 < NC ? C - c0 : NC) : 1;
        const TX* xb = x + (b * C + c0) * plane;
        Online<A, NC> on;
        on.init();
        for (int s = 0; s < st.S; ++s) {
            const int64_t dx = st.dx[s], dy = st.dy[s];
            const TW* ws = w + ((static_cast<int64_t>(s) * B + b) * Cw + wc) * plane;
            A xv[NC];
            const int64_t xo = wrap1(h + dx, H) * W + wrap1(wcol + dy, W);
#pragma unroll
            for (int i = 0; i < NC; ++i)
                xv[i] = (i < nc) ? ldg_acc<TX, A>(xb + i * plane + xo) : A(0);
            const A kf = ldg_acc<TW, A>(ws + h * W + wcol);
            // weight contract: finite, or -inf (logits) / >= 0 (positive)
            if (kf != kf || kf == A(INFINITY) || (!logw && kf < A(0)))
                seen_invalid = true;
            on.push(kf, xv, logw);
            if (st.has_inv(s)) {
                const bool per = st.has_per(s);
                const int64_t hm = per ? wrap1(h - dx, H) : h - dx;
                const int64_t wm = per ? wrap1(wcol - dy, W) : wcol - dy;
                if (per || (inb(hm, H) && inb(wm, W))) {
                    const int64_t mo = hm * W + wm;
#pragma unroll
                    for (int i = 0; i < NC; ++i)
                        xv[i] = (i < nc) ? ldg_acc<TX, A>(xb + i * plane + mo) : A(0);
                    on.push(ldg_acc<TW, A>(ws + mo), xv, logw);
                }
            }
        }
        const int64_t ob = (b * C + c0) * plane + h * W + wcol;
        const A nan = A(NAN);
#pragma unroll
        for (int i = 0; i < NC; ++i) {
            if (i >= nc) continue;
            A d, l;
            if (on.bad) {
                d = nan; l = nan;
            } else if (on.m == neg_inf<A>()) {
                d = A(0); l = neg_inf<A>();
            } else if (isfinite(on.m) && on.sz > A(0) && isfinite(on.sz)) {
                d = on.su[i] / on.sz;
                l = (logw ? on.m : log_acc(on.m)) + log_acc(on.sz);
            } else {
                d = nan; l = nan;
            }
            D[ob + i * plane] = d;
            L[ob + i * plane] = l;
        }
    }
    if (seen_invalid && invalid) atomicOr(invalid, 1);
}

// Periodic mirror rows on the tiled path (see acc_per_fix_kernel): the
// wrapped mirror keys of the border band, normalised on their own and merged
// into the tile kernel's (D, log_C):
//   D = (D1 e^(L1 - M) + D2 e^(L2 - M)) / (e^(L1 - M) + e^(L2 - M)),
//   L = M + log(e^(L1 - M) + e^(L2 - M)),  M = max(L1, L2).
template <typename TX, typename TW, int NC>
__global__ void __launch_bounds__(256)
norm_per_fix_kernel(const TX* __restrict__ x, const TW* __restrict__ w,
                    typename Acc<TX>::type* __restrict__ D,
                    typename Acc<TX>::type* __restrict__ L, const ShiftTable st,
                    int64_t B, int64_t C, int64_t H, int64_t W, int64_t Cw, int64_t R,
                    int logw, int64_t nb, int64_t groups) {
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
        Online<A, NC> on;
        on.init();
        for (int s = 0; s < st.S; ++s) {
            if (!st.has_per(s)) continue;
            int64_t hm = h - st.dx[s], wm = wcol - st.dy[s];
            if (inb(hm, H) && inb(wm, W)) continue;     // in the tile kernel's sums
            hm = wrap1(hm, H);
            wm = wrap1(wm, W);
            const TW* ws = w + ((static_cast<int64_t>(s) * B + b) * Cw + wc) * plane;
            A xv[NC];
#pragma unroll
            for (int k = 0; k < NC; ++k)
                xv[k] = (k < nc) ? ldg_acc<TX, A>(xb + k * plane + hm * W + wm) : A(0);
            on.push(ldg_acc<TW, A>(ws + hm * W + wm), xv, logw);
        }
        if (!on.bad && on.m == neg_inf<A>()) continue;   // nothing wrapped here
        const int64_t ob = (b * C + c0) * plane + h * W + wcol;
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            if (k >= nc) continue;
            A& d = D[ob + k * plane];
            A& l = L[ob + k * plane];
            if (on.bad || !(isfinite(on.m) && on.sz > A(0) && isfinite(on.sz)) || l != l) {
                d = A(NAN);
                l = A(NAN);
                continue;
            }
            const A d2 = on.su[k] / on.sz;
            const A l2 = (logw ? on.m : log_acc(on.m)) + log_acc(on.sz);
            if (l == neg_inf<A>()) {
                d = d2;
                l = l2;
                continue;
            }
            const A M = l > l2 ? l : l2;
            const A a1 = exp_acc(l - M), a2 = exp_acc(l2 - M);
            d = (d * a1 + d2 * a2) / (a1 + a2);
            l = M + log_acc(a1 + a2);
        }
    }
}

template <typename A>
__device__ __forceinline__ A as_log(A v, int logw) {
    if (logw) return v;
    if (v > A(0)) return log_acc(v);
    if (v == A(0)) return neg_inf<A>();
    return A(NAN);
}

template <typename A>
__device__ __forceinline__ A fraction(A lw, A lc) {
    if (lw == neg_inf<A>() || lc == neg_inf<A>()) return A(0);
    return exp_acc(lw - lc);
}

// Fused backward, thread per pixel q and NC channels:
//   gx(q)   = sum_s p(w_s(q-d), logC(q-d)) gD(q-d)  [circular]
//           + inv [q+d inside] p(w_s(q), logC(q+d)) gD(q+d)
//   gw_s(q) = fac(q) (gD(q) (x(q+d) - D(q)) + gL(q))
//           + inv [q+d inside] fac'(q+d) (gD(q+d) (x(q) - D(q+d)) + gL(q+d))
// with fac = p (log mode) or exp(-logC) (positive mode); gw = 0 for masked.
// GW == false skips grad_w: a channel-broadcast weight with more than NC
// channels needs the sum over every channel group, which
// norm_bwd_gw_bcast_kernel forms instead.
template <typename TX, typename TW, int NC, bool GW>
__global__ void __launch_bounds__(kBX * kBY)
norm_bwd_kernel(const TX* __restrict__ x, const TW* __restrict__ w,
                const typename Acc<TX>::type* __restrict__ D,
                const typename Acc<TX>::type* __restrict__ L,
                const typename Acc<TX>::type* __restrict__ gD,
                const typename Acc<TX>::type* __restrict__ gL,
                typename Acc<TX>::type* __restrict__ gx, TW* __restrict__ gw,
                const ShiftTable st, int64_t B, int64_t C, int64_t H,
                int64_t W, int64_t Cw, int logw, int64_t groups) {
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
        A acc[NC], xq[NC], Lq[NC], Dq[NC], gDq[NC], gLq[NC];
#pragma unroll
        for (int i = 0; i < NC; ++i) {
            acc[i] = A(0);
            const bool on = i < nc;
            xq[i] = on ? ldg_acc<TX, A>(x + cb + i * plane + q) : A(0);
            Lq[i] = on ? L[cb + i * plane + q] : A(0);
            Dq[i] = on ? D[cb + i * plane + q] : A(0);
            gDq[i] = on ? gD[cb + i * plane + q] : A(0);
            gLq[i] = on ? gL[cb + i * plane + q] : A(0);
        }
        for (int s = 0; s < st.S; ++s) {
            const int64_t dx = st.dx[s], dy = st.dy[s];
            const int64_t wbase = ((static_cast<int64_t>(s) * B + b) * Cw + wc) * plane;
            const TW* ws = w + wbase;
            const int64_t qs = wrap1(h - dx, H) * W + wrap1(wcol - dy, W);
            const A lw_src = as_log(ldg_acc<TW, A>(ws + qs), logw);
            const A vq = ldg_acc<TW, A>(ws + q);
            const A lw_q = as_log(vq, logw);
            const int64_t qf = wrap1(h + dx, H) * W + wrap1(wcol + dy, W);
            const bool mir = st.has_inv(s) &&
                             (st.has_per(s) || (inb(h + dx, H) && inb(wcol + dy, W)));
            const int64_t qi = wrap1(h + dx, H) * W + wrap1(wcol + dy, W);
            A gws = A(0);
#pragma unroll
            for (int i = 0; i < NC; ++i) {
                if (i >= nc) continue;
                const int64_t co = cb + i * plane;
                acc[i] += fraction(lw_src, L[co + qs]) * gD[co + qs];
                const A score = gDq[i] * (ldg_acc<TX, A>(x + co + qf) - Dq[i]) + gLq[i];
                gws += (logw ? fraction(lw_q, Lq[i]) : exp_acc(-Lq[i])) * score;
                if (mir) {
                    const A Li = L[co + qi];
                    const A gDi = gD[co + qi];
                    acc[i] += fraction(lw_q, Li) * gDi;
                    const A score_i = gDi * (xq[i] - D[co + qi]) + gL[co + qi];
                    gws += (logw ? fraction(lw_q, Li) : exp_acc(-Li)) * score_i;
                }
            }
            if (lw_q == neg_inf<A>()) gws = A(0);
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
norm_bwd_gw_bcast_kernel(const TX* __restrict__ x, const TW* __restrict__ w,
                         const typename Acc<TX>::type* __restrict__ D,
                         const typename Acc<TX>::type* __restrict__ L,
                         const typename Acc<TX>::type* __restrict__ gD,
                         const typename Acc<TX>::type* __restrict__ gL,
                         TW* __restrict__ gw, const ShiftTable st, int64_t B,
                         int64_t C, int64_t H, int64_t W, int logw) {
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
            const int64_t wq = (static_cast<int64_t>(s) * B + b) * plane + q;
            const A lw_q = as_log(ldg_acc<TW, A>(w + wq), logw);
            const int64_t qf = wrap1(h + dx, H) * W + wrap1(wcol + dy, W);
            const bool mir = st.has_inv(s) &&
                             (st.has_per(s) || (inb(h + dx, H) && inb(wcol + dy, W)));
            A gws = A(0);
            for (int64_t c = 0; c < C; ++c) {
                const int64_t co = cb + c * plane;
                const A Lq = L[co + q];
                const A score = gD[co + q] * (ldg_acc<TX, A>(x + co + qf) - D[co + q]) +
                                gL[co + q];
                gws += (logw ? fraction(lw_q, Lq) : exp_acc(-Lq)) * score;
                if (mir) {
                    const A Li = L[co + qf];
                    const A score_i =
                        gD[co + qf] * (ldg_acc<TX, A>(x + co + q) - D[co + qf]) + gL[co + qf];
                    gws += (logw ? fraction(lw_q, Li) : exp_acc(-Li)) * score_i;
                }
            }
            if (lw_q == neg_inf<A>()) gws = A(0);
            gw[wq] = static_cast<TW>(gws);
        }
    }
}

// Tiled backward (the same gradients as norm_bwd_kernel), for fp16 / bf16 /
// fp32 storage and radius <= 8.  A CTA of 32 x 8 threads owns a 16 x 32
// tile of one (image, weight channel) group, two pixels per thread (rows 8
// apart).  x, D, grad_D, grad_log_C of the group's channels and log_C are
// staged once, circularly, with the R halo as fp32 in shared memory; every
// neighbour read of the shift loop is a shared-memory load at a constant
// offset, and the mirror term's inside test is a flag (interior tiles
// skip it).  log_C is the same for every channel of a channel-broadcast
// weight (the keys are shared), so it is staged and exponentiated once.
// exp(lw - lc) (0 where either is -inf) through ex2.approx: a few ulp of
// fp32, well inside the fp32 tolerance of the gradients.
__device__ __forceinline__ float ex2_fast(float v) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}
__device__ __forceinline__ float fraction_fast(float lw, float lc) {
    if (lw == -INFINITY || lc == -INFINITY) return 0.f;
    return ex2_fast((lw - lc) * 1.4426950408889634f);
}

constexpr int kTX = 32, kTY = 8, kPPT = 2, kTH = kTY * kPPT, kTW = kTX;

template <typename T, int NC>
__global__ void __launch_bounds__(kTX * kTY)
norm_bwd_tile_kernel(const T* __restrict__ x, const T* __restrict__ w,
                     const float* __restrict__ D, const float* __restrict__ L,
                     const float* __restrict__ gD, const float* __restrict__ gL,
                     float* __restrict__ gx, T* __restrict__ gw, const ShiftTable st,
                     int B, int C, int H, int W, int Cw, int R, int tiles_x, int logw) {
    extern __shared__ __align__(16) float smem_n[];
    const int XP = kTW + 2 * R, XR = kTH + 2 * R, plane = XP * XR;
    float* sx = smem_n;                 // [NC] x
    float* sD = sx + NC * plane;        // [NC] D
    float* sgD = sD + NC * plane;       // [NC] grad_D
    float* sgL = sgD + NC * plane;      // [NC] grad_log_C
    float* sL = sgL + NC * plane;       // log_C (shared by the group's channels)
    const int64_t HW = static_cast<int64_t>(H) * W;
    const int cgroups = Cw == 1 ? 1 : C;
    const int grp = blockIdx.y;
    const int b = grp / cgroups;
    const int wc = Cw == 1 ? 0 : grp % cgroups;
    const int c0 = Cw == 1 ? 0 : wc;
    const int ty = blockIdx.x / tiles_x;
    const int h0 = ty * kTH, w0 = (blockIdx.x - ty * tiles_x) * kTW;
    const int64_t cb = (static_cast<int64_t>(b) * C + c0) * HW;
    const int tid = threadIdx.y * kTX + threadIdx.x;
    for (int e = tid; e < plane; e += kTX * kTY) {
        const int i = e / XP, j = e - i * XP;
        int r = (h0 - R + i) % H;
        if (r < 0) r += H;
        int c = (w0 - R + j) % W;
        if (c < 0) c += W;
        const int64_t off = static_cast<int64_t>(r) * W + c;
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            sx[k * plane + e] = to_acc(x[cb + k * HW + off]);
            sD[k * plane + e] = D[cb + k * HW + off];
            sgD[k * plane + e] = gD[cb + k * HW + off];
            sgL[k * plane + e] = gL[cb + k * HW + off];
        }
        sL[e] = L[cb + off];
    }
    __syncthreads();
    const int wcol = w0 + threadIdx.x;
    if (wcol >= W) return;
    const bool interior = h0 - R >= 0 && h0 + kTH + R <= H && w0 - R >= 0 && w0 + kTW + R <= W;
    const T* __restrict__ wb = w + (static_cast<int64_t>(b) * Cw + wc) * HW;
    T* __restrict__ gwb = gw + (static_cast<int64_t>(b) * Cw + wc) * HW;
    const int64_t sstride = static_cast<int64_t>(B) * Cw * HW;
    int hh[kPPT], ci[kPPT];
    float Lq[kPPT], eLq[kPPT], xq[kPPT][NC], Dq[kPPT][NC], gDq[kPPT][NC], gLq[kPPT][NC];
    float acc[kPPT][NC];
#pragma unroll
    for (int p = 0; p < kPPT; ++p) {
        const int h = h0 + threadIdx.y + kTY * p;
        hh[p] = h < H ? h : H - 1;
        ci[p] = (threadIdx.y + kTY * p + R) * XP + threadIdx.x + R;
        Lq[p] = sL[ci[p]];
        eLq[p] = exp_acc(-Lq[p]);   // positive mode: exp(-log_C), once per pixel
#pragma unroll
        for (int k = 0; k < NC; ++k) {
            xq[p][k] = sx[k * plane + ci[p]];
            Dq[p][k] = sD[k * plane + ci[p]];
            gDq[p][k] = sgD[k * plane + ci[p]];
            gLq[p][k] = sgL[k * plane + ci[p]];
            acc[p][k] = 0.f;
        }
    }
    // Weights of the next LA shifts are loaded ahead of their use (a small
    // register ring), so each thread keeps 2 * kPPT * LA loads in flight.
    constexpr int LA = 6;
    float wq_r[LA][kPPT], ws_r[LA][kPPT];
    auto fetch = [&](int s, float (&wq)[kPPT], float (&wsrc)[kPPT]) {
        const int dx = st.dx[s], dy = st.dy[s];
        const T* ws = wb + s * sstride;
#pragma unroll
        for (int p = 0; p < kPPT; ++p) {
            const int h = hh[p];
            const int64_t q = static_cast<int64_t>(h) * W + wcol;
            const int64_t qsrc = static_cast<int64_t>(wrap1(h - dx, H)) * W + wrap1(wcol - dy, W);
            wq[p] = to_acc(__ldg(ws + q));
            wsrc[p] = to_acc(__ldg(ws + qsrc));
        }
    };
#pragma unroll
    for (int k = 0; k < LA; ++k)
        if (k < st.S) fetch(k, wq_r[k], ws_r[k]);
    for (int s0 = 0; s0 < st.S; s0 += LA) {
#pragma unroll
        for (int k = 0; k < LA; ++k) {
            const int s = s0 + k;
            if (s >= st.S) break;
            float wqv[kPPT], wsv[kPPT];
#pragma unroll
            for (int p = 0; p < kPPT; ++p) {
                wqv[p] = wq_r[k][p];
                wsv[p] = ws_r[k][p];
            }
            if (s + LA < st.S) fetch(s + LA, wq_r[k], ws_r[k]);
            const int dx = st.dx[s], dy = st.dy[s];
            const bool inv = st.has_inv(s), per = st.has_per(s);
            const int off = dx * XP + dy;
#pragma unroll
            for (int p = 0; p < kPPT; ++p) {
                const int h = hh[p];
                const int64_t q = static_cast<int64_t>(h) * W + wcol;
                const bool in_f = interior || (inb(h + dx, H) && inb(wcol + dy, W));
                const float lw_src = as_log(wsv[p], logw);
                const float lw_q = as_log(wqv[p], logw);
                const int qs = ci[p] - off, qf = ci[p] + off;
                const float pa = fraction_fast(lw_src, sL[qs]);
                const float fq = logw ? fraction_fast(lw_q, Lq[p]) : eLq[p];
                const bool mir = inv && (per || in_f);
                float pb = 0.f, fm = 0.f;
                if (mir) {
                    const float Lf = sL[qf];
                    pb = fraction_fast(lw_q, Lf);
                    fm = logw ? pb : ex2_fast(-Lf * 1.4426950408889634f);
                }
                float gws = 0.f;
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    acc[p][c] += pa * sgD[c * plane + qs];
                    gws += fq * (gDq[p][c] * (sx[c * plane + qf] - Dq[p][c]) + gLq[p][c]);
                    if (mir) {
                        const float gDi = sgD[c * plane + qf];
                        acc[p][c] += pb * gDi;
                        gws += fm * (gDi * (xq[p][c] - sD[c * plane + qf]) + sgL[c * plane + qf]);
                    }
                }
                if (lw_q == neg_inf<float>()) gws = 0.f;
                if (h0 + static_cast<int>(threadIdx.y) + kTY * p < H)
                    gwb[s * sstride + q] = static_cast<T>(gws);
            }
        }
    }
#pragma unroll
    for (int p = 0; p < kPPT; ++p) {
        const int h = h0 + threadIdx.y + kTY * p;
        if (h >= H) continue;
#pragma unroll
        for (int k = 0; k < NC; ++k)
            gx[cb + k * HW + static_cast<int64_t>(h) * W + wcol] = acc[p][k];
    }
}

template <int NC> struct NCTag { static constexpr int value_nc = NC; };

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
                "%s: unsupported dtype pair (x=%d, w=%d)", op, xd, wd);
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
    nsc_status e2 = build_shifts(op, shifts, S, 3, H, W, st);
    if (e2) return e2;
    if (st->any_tr)
        return fail(NSC_ERR_INVALID_ARG,
                    "%s: transposed rows (column value 3) are accepted by "
                    "accumulate_uz only", op);
    return ok();
}

}  // namespace
}  // namespace nsc

extern "C" {

nsc_status nsc_normalized_accumulate_uz_fwd(
    const void* x, int x_dtype, const void* w, int w_dtype, int64_t w_channels,
    int64_t B, int64_t C, int64_t H, int64_t W, const int64_t* shifts,
    int64_t S, int log_weights, void* D, void* log_C, int* invalid_flag,
    void* stream) {
    using namespace nsc;
    const char* op = "normalized_accumulate_uz";
    ShiftTable st;
    nsc_status e = check_common(op, x_dtype, w_dtype, w_channels, B, C, H, W,
                                shifts, S, &st);
    if (e) return e;
    if (B == 0 || C == 0 || H == 0 || W == 0) return ok();
    if (!x || !w || !D || !log_C)
        return fail(NSC_ERR_INVALID_ARG, "%s: NULL tensor pointer", op);
    cudaStream_t sm = as_stream(stream);
    if (norm_fwd_fast(x, x_dtype, w, w_dtype, w_channels, B, C, H, W, st,
                      log_weights ? 1 : 0, D, log_C, invalid_flag, sm))
        return check_launch(op);
    // tables with mirror terms: the TMA-tiled kernel in its normalized modes
    if (!getenv("NSC_NORM_GENERIC") &&
        acc_fwd_fast(x, x_dtype, w, w_dtype, w_channels, B, C, H, W, H, 0, 1, st,
                     D, log_C, sm, log_weights ? 1 : 2, invalid_flag)) {
        if (!st.any_per) return check_launch(op);
        // wrapped periodic mirror terms of the border band
        return with_types(op, x_dtype, w_dtype, [&](auto tx, auto tw) {
            using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
            using TW = std::remove_const_t<std::remove_pointer_t<decltype(tw)>>;
            using A = typename Acc<TX>::type;
            const int64_t R = st.R, nb = border_count(H, W, R);
            with_nc(C, w_channels, [&](auto tag) {
                constexpr int NC = decltype(tag)::value_nc;
                const int64_t groups = n_groups(B, C, w_channels, NC);
                const dim3 grid(grid_1d(nb, 256),
                                static_cast<unsigned>(groups < 65535 ? groups : 65535));
                norm_per_fix_kernel<TX, TW, NC><<<grid, 256, 0, sm>>>(
                    static_cast<const TX*>(x), static_cast<const TW*>(w),
                    static_cast<A*>(D), static_cast<A*>(log_C), st, B, C, H, W,
                    w_channels, R, log_weights ? 1 : 0, nb, groups);
            });
            return check_launch(op);
        });
    }
    if (getenv("NSC_REQUIRE_FAST"))
        return fail(NSC_ERR_INVALID_ARG, "%s: tiled paths declined: %s; %s", op,
                    norm_fast_decline_reason(), fast_decline_reason());
    return with_types(op, x_dtype, w_dtype, [&](auto tx, auto tw) {
        using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
        using TW = std::remove_const_t<std::remove_pointer_t<decltype(tw)>>;
        using A = typename Acc<TX>::type;
        with_nc(C, w_channels, [&](auto tag) {
            constexpr int NC = decltype(tag)::value_nc;
            const int64_t groups = n_groups(B, C, w_channels, NC);
            norm_fwd_kernel<TX, TW, NC><<<grid_for(W, H, groups),
                                           dim3(kBX, kBY), 0, sm>>>(
                static_cast<const TX*>(x), static_cast<const TW*>(w),
                static_cast<A*>(D), static_cast<A*>(log_C), st, B, C, H, W,
                w_channels, log_weights ? 1 : 0, invalid_flag, groups);
        });
        return check_launch(op);
    });
}

nsc_status nsc_normalized_accumulate_uz_bwd(
    const void* x, int x_dtype, const void* w, int w_dtype, int64_t w_channels,
    int64_t B, int64_t C, int64_t H, int64_t W, const int64_t* shifts,
    int64_t S, int log_weights, const void* D, const void* log_C,
    const void* grad_D, const void* grad_log_C, void* grad_x, void* grad_w,
    void* stream) {
    using namespace nsc;
    const char* op = "normalized_accumulate_uz_backward";
    ShiftTable st;
    nsc_status e = check_common(op, x_dtype, w_dtype, w_channels, B, C, H, W,
                                shifts, S, &st);
    if (e) return e;
    if (B == 0 || C == 0 || H == 0 || W == 0) return ok();
    if (!x || !w || !D || !log_C || !grad_D || !grad_log_C || !grad_x || !grad_w)
        return fail(NSC_ERR_INVALID_ARG, "%s: NULL tensor pointer", op);
    cudaStream_t sm = as_stream(stream);
    // tiled form: storage fp16 / bf16 / fp32 shared by x and w, radius <= 8
    const int64_t ngrp = B * (w_channels == 1 ? 1 : C);
    if (!getenv("NSC_NORM_GENERIC") && x_dtype == w_dtype && x_dtype != NSC_F64 &&
        (w_channels == C || (w_channels == 1 && (C == 1 || C == 3))) && st.R <= 8 &&
        ngrp <= 65535 && H < (1LL << 30) && W < (1LL << 30) && B * C < (1LL << 30)) {
        const int R = st.R;
        const int tiles_x = static_cast<int>((W + kTW - 1) / kTW);
        const int64_t tiles = tiles_x * ((H + kTH - 1) / kTH);
        const int NC = w_channels == 1 ? static_cast<int>(C) : 1;
        const size_t smem = static_cast<size_t>(4 * NC + 1) * (kTW + 2 * R) * (kTH + 2 * R) *
                            sizeof(float);
        if (tiles < (1LL << 31)) {
            auto go = [&](auto kern, auto tptr) {
                using T = std::remove_const_t<std::remove_pointer_t<decltype(tptr)>>;
                if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)) != cudaSuccess) {
                    cudaGetLastError();
                    return false;
                }
                kern<<<dim3(static_cast<unsigned>(tiles), static_cast<unsigned>(ngrp)),
                       dim3(kTX, kTY), smem, sm>>>(
                    static_cast<const T*>(x), static_cast<const T*>(w),
                    static_cast<const float*>(D), static_cast<const float*>(log_C),
                    static_cast<const float*>(grad_D), static_cast<const float*>(grad_log_C),
                    static_cast<float*>(grad_x), static_cast<T*>(grad_w), st,
                    static_cast<int>(B), static_cast<int>(C), static_cast<int>(H),
                    static_cast<int>(W), static_cast<int>(w_channels), R, tiles_x,
                    log_weights ? 1 : 0);
                return true;
            };
            bool ran;
            if (x_dtype == NSC_F16)
                ran = NC == 3 ? go(norm_bwd_tile_kernel<__half, 3>, (const __half*)nullptr)
                              : go(norm_bwd_tile_kernel<__half, 1>, (const __half*)nullptr);
            else if (x_dtype == NSC_BF16)
                ran = NC == 3 ? go(norm_bwd_tile_kernel<__nv_bfloat16, 3>, (const __nv_bfloat16*)nullptr)
                              : go(norm_bwd_tile_kernel<__nv_bfloat16, 1>, (const __nv_bfloat16*)nullptr);
            else
                ran = NC == 3 ? go(norm_bwd_tile_kernel<float, 3>, (const float*)nullptr)
                              : go(norm_bwd_tile_kernel<float, 1>, (const float*)nullptr);
            if (ran) return check_launch(op);
        }
    }
    return with_types(op, x_dtype, w_dtype, [&](auto tx, auto tw) {
        using TX = std::remove_const_t<std::remove_pointer_t<decltype(tx)>>;
        using TW = std::remove_const_t<std::remove_pointer_t<decltype(tw)>>;
        using A = typename Acc<TX>::type;
        with_nc(C, w_channels, [&](auto tag) {
            constexpr int NC = decltype(tag)::value_nc;
            const int64_t groups = n_groups(B, C, w_channels, NC);
            const bool split = w_channels == 1 && C > NC;
            auto launch = [&](auto kern) {
                kern<<<grid_for(W, H, groups), dim3(kBX, kBY), 0, sm>>>(
                    static_cast<const TX*>(x), static_cast<const TW*>(w),
                    static_cast<const A*>(D), static_cast<const A*>(log_C),
                    static_cast<const A*>(grad_D), static_cast<const A*>(grad_log_C),
                    static_cast<A*>(grad_x), static_cast<TW*>(grad_w), st, B, C, H,
                    W, w_channels, log_weights ? 1 : 0, groups);
            };
            if (split) {
                launch(norm_bwd_kernel<TX, TW, NC, false>);
                norm_bwd_gw_bcast_kernel<TX, TW><<<grid_for(W, H, B), dim3(kBX, kBY),
                                                    0, sm>>>(
                    static_cast<const TX*>(x), static_cast<const TW*>(w),
                    static_cast<const A*>(D), static_cast<const A*>(log_C),
                    static_cast<const A*>(grad_D), static_cast<const A*>(grad_log_C),
                    static_cast<TW*>(grad_w), st, B, C, H, W, log_weights ? 1 : 0);
            } else {
                launch(norm_bwd_kernel<TX, TW, NC, true>);
            }
        });
        return check_launch(op);
    });
}

}  // extern "C"
