// nectr_fused.cu -- the NECTR model-1 patched forward in one kernel:
// pair gather + pairwise weight head + normalized (or plain) shift-window
// accumulation, without materialising the (S*B, 2L, H, W) pair batch.
//
// The reference patch (integration/nectr_patch.py:214-234) runs
//   pair, mask = pair_gather(g, shifts)              (S*B, 2L, H, W)
//   v = out(LeakyReLU(LN(conv1x1(pair))))            (proj_depth blocks)
//   keys = v / sigma^2 (exp head, log mode) | controlled sigmoid (positive)
//          | v (raw), masked by the forward box
//   D, log_C = normalized_accumulate_uz(x, keys, shifts)   (or accumulate_uz)
// The first 1x1 convolution of [g(p); g(p+d)] splits into
// A(p) = W1[:, :L] g(p) + b1 and Bm(p+d) = W1[:, L:] g(p+d); the caller
// computes W1[:, :L] g and W1[:, L:] g once as one (B, 2 L1, H, W) map
// (a single batched matrix product) and the bias is added at staging.  Then every key is
// a small per-pixel MLP on A(p) + Bm(p+d):
//   forward term at p:  key_s(p)   = head(A(p) + Bm(p + d)),  p + d inside
//   mirror term at p:   key_s(p-d) = head(A(p - d) + Bm(p)),  p - d inside
// (the mirror of a has_inv row reads the weight plane at p - d).  A CTA
// stages A, Bm and x for a TH x TW tile plus an R halo in shared memory;
// a thread owns one pixel and all C image channels, keeps A(p), Bm(p) in
// registers and runs the per-channel online normalisation over the table.
// Image bytes read once per tile (plus the halo); the head arithmetic
// (~130 FLOP per key) is the cost, so the kernel is issue-bound, not
// HBM-bound, by design: the unfused path writes and re-reads 4+ GB.
//
// Modes: 1 = log weights (exp head, key = v / sigma^2), 2 = positive
// weights (controlled sigmoid: softplus(a) / (1 + exp(-sigmoid(b) k)) +
// 1e-8 from the three output chunks k, a, b), 0 = raw head output with the
// plain accumulate_uz sums.  Outputs: modes 1 / 2 D and log_C (B, C, H, W);
// mode 0 U and Z.  Special values follow the normalized kernels (NaN / inf
// keys poison the pixel and set the invalid flag; no live key: D = 0,
// log_C = -inf).
#include <cmath>
#include <cstring>

#include "nsc_common.cuh"
#include "nsc_host.h"

namespace nsc {
namespace nectr {

constexpr int TH = 8, TW = 32, NT = TH * TW;
constexpr int MAXC = 3;

// Pairs of accumulator values: fp32 pairs use the packed f32x2 arithmetic
// of sm_100 (one instruction per two lanes of the head's vectors); fp64
// pairs are two scalar operations.
template <typename A> struct Pair2;
template <> struct Pair2<float> { using T = float2; };
template <> struct Pair2<double> { using T = double2; };

__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ double2 add2(double2 a, double2 b) { return make_double2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ double2 mul2(double2 a, double2 b) { return make_double2(a.x * b.x, a.y * b.y); }
__device__ __forceinline__ double2 fma2(double2 a, double2 b, double2 c) {
    return make_double2(fma(a.x, b.x, c.x), fma(a.y, b.y, c.y));
}
template <typename T2> __device__ __forceinline__ T2 splat2(decltype(T2::x) v) { return T2{v, v}; }
template <typename T2> __device__ __forceinline__ decltype(T2::x) hsum2(T2 a, T2 b) {
    return (a.x + a.y) + (b.x + b.y);
}

// Head parameters in pairs along the input index of each layer.
template <typename A, int L1, int DEPTH, int COUT>
struct Head {
    using A2 = typename Pair2<A>::T;
    static constexpr int L2 = L1 / 2;
    static constexpr int LK = DEPTH == 1 ? L1 : L2;
    A bias1[L1];                           // first conv bias (added at staging)
    A2 g1[L1 / 2], b1[L1 / 2];             // LayerNorm 1 affine
    A2 w2[DEPTH == 2 ? L2 * L1 / 2 : 1];   // block 2 conv [L2][L1 / 2]
    A c2[DEPTH == 2 ? L2 : 1];
    A2 g2[DEPTH == 2 ? L2 / 2 : 1], b2[DEPTH == 2 ? L2 / 2 : 1];
    A2 wo[COUT * LK / 2];                  // output conv [COUT][LK / 2], no bias
    A eps1, eps2, slope, inv_s2;
};

template <typename A> __device__ __forceinline__ A rsqrt_a(A v);
template <> __device__ __forceinline__ float rsqrt_a<float>(float v) { return rsqrtf(v); }
template <> __device__ __forceinline__ double rsqrt_a<double>(double v) { return 1.0 / sqrt(v); }

// Sum over N2 pairs with two independent pair accumulators.
template <typename A2, int N2, typename F>
__device__ __forceinline__ decltype(A2::x) psum(F&& f) {
    A2 p0 = f(0), p1 = N2 > 1 ? f(1) : A2{0, 0};
#pragma unroll
    for (int k = 2; k < N2; ++k) {
        if (k & 1) p1 = add2(p1, f(k));
        else p0 = add2(p0, f(k));
    }
    return hsum2(p0, p1);
}
// Dot product of N2 pairs, two fused-multiply-add chains.
template <typename A2, int N2>
__device__ __forceinline__ decltype(A2::x) pdot(const A2* w, const A2* h) {
    A2 p0 = mul2(w[0], h[0]);
    A2 p1 = N2 > 1 ? mul2(w[1], h[1]) : A2{0, 0};
#pragma unroll
    for (int k = 2; k < N2; ++k) {
        if (k & 1) p1 = fma2(w[k], h[k], p1);
        else p0 = fma2(w[k], h[k], p0);
    }
    return hsum2(p0, p1);
}

// Channel LayerNorm (biased variance) and LeakyReLU of N2 pairs in place.
template <typename A, int N2>
__device__ __forceinline__ void ln_leaky(typename Pair2<A>::T (&h)[N2],
                                         const typename Pair2<A>::T* g,
                                         const typename Pair2<A>::T* b, A eps, A slope) {
    using A2 = typename Pair2<A>::T;
    constexpr A inv_n = A(1) / A(2 * N2);
    const A mean = psum<A2, N2>([&](int k) { return h[k]; }) * inv_n;
    const A2 nm = splat2<A2>(-mean);
#pragma unroll
    for (int k = 0; k < N2; ++k) h[k] = add2(h[k], nm);
    const A var = psum<A2, N2>([&](int k) { return mul2(h[k], h[k]); }) * inv_n;
    const A2 r = splat2<A2>(rsqrt_a<A>(var + eps));
    const A2 sl = splat2<A2>(slope);
#pragma unroll
    for (int k = 0; k < N2; ++k) {
        const A2 t = fma2(mul2(h[k], r), g[k], b[k]);
        const A2 u = mul2(t, sl);
        // max(t, slope t) is LeakyReLU for 0 <= slope <= 1
        h[k] = A2{t.x > u.x ? t.x : u.x, t.y > u.y ? t.y : u.y};
    }
}

// Per-channel keys of one (pixel, shift) from the first-layer input h.
template <typename A, int L1, int DEPTH, int COUT, int C, int MODE>
__device__ __forceinline__ void head_keys(typename Pair2<A>::T (&h)[L1 / 2],
                                          const Head<A, L1, DEPTH, COUT>& P,
                                          A (&key)[C]) {
    using H = Head<A, L1, DEPTH, COUT>;
    using A2 = typename Pair2<A>::T;
    ln_leaky<A, L1 / 2>(h, P.g1, P.b1, P.eps1, P.slope);
    A v[COUT];
    if constexpr (DEPTH == 1) {
#pragma unroll
        for (int o = 0; o < COUT; ++o) v[o] = pdot<A2, L1 / 2>(P.wo + o * (L1 / 2), h);
    } else {
        A2 h2[H::L2 / 2];
#pragma unroll
        for (int i = 0; i < H::L2 / 2; ++i)
            h2[i] = A2{P.c2[2 * i] + pdot<A2, L1 / 2>(P.w2 + (2 * i) * (L1 / 2), h),
                       P.c2[2 * i + 1] + pdot<A2, L1 / 2>(P.w2 + (2 * i + 1) * (L1 / 2), h)};
        ln_leaky<A, H::L2 / 2>(h2, P.g2, P.b2, P.eps2, P.slope);
#pragma unroll
        for (int o = 0; o < COUT; ++o) v[o] = pdot<A2, H::L2 / 2>(P.wo + o * (H::L2 / 2), h2);
    }
#pragma unroll
    for (int c = 0; c < C; ++c) {
        if constexpr (MODE == 1) {
            key[c] = v[c] * P.inv_s2;
        } else if constexpr (MODE == 2) {
            // softplus with torch's threshold 20, then the controlled sigmoid
            const A a = v[C + c], bb = v[2 * C + c];
            const A sp = a > A(20) ? a : log1p(exp(a));
            const A sg = A(1) / (A(1) + exp(-bb));
            key[c] = sp / (A(1) + exp(-sg * v[c])) + A(1e-8);
        } else {
            key[c] = v[c];
        }
    }
}

// Online per-channel state.  Log mode (float): m in log2 units, rescaled
// lazily when a key exceeds it by 2^16; (double): m = running max.
// Positive mode: running reference mx (lazy), sums of k / mx.
template <typename A, int MODE>
struct Acc1 {
    A u, z, m, r;   // r: 1 / mx in positive mode
    __device__ __forceinline__ void init() {
        u = z = A(0);
        m = MODE == 1 ? A(-INFINITY) : A(0);
        r = A(INFINITY);
    }
    __device__ __forceinline__ void add(A key, A xv) {
        if constexpr (MODE == 0) {
            u += key * xv;
            z += key;
        } else if constexpr (MODE == 1) {
            if constexpr (sizeof(A) == 4) {
                const float t = key * 1.4426950408889634f;
                if (t > m + 16.0f) {
                    float f;
                    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(f) : "f"(m - t));
                    u *= f;
                    z *= f;
                    m = t;
                }
                float a;
                asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(a) : "f"(t - m));
                u += a * xv;
                z += a;
            } else {
                if (key > m) {
                    const A f = exp(m - key);
                    u *= f;
                    z *= f;
                    m = key;
                }
                const A a = exp(key - m);
                u += a * xv;
                z += a;
            }
        } else {
            A a = key * r;
            if (!(a <= A(65536)) || key < A(0)) {
                if (!(key >= A(0)) || key == A(INFINITY)) {
                    z = A(NAN);
                    a = A(0);
                } else if (key == A(0)) {
                    a = A(0);
                } else {
                    const A nr = A(1) / key;
                    const A f = m * nr;     // m: current reference (0 before the first key)
                    u *= f;
                    z *= f;
                    m = key;
                    r = nr;
                    a = A(1);
                }
            }
            u += a * xv;
            z += a;
        }
    }
};

template <typename A, int L1, int DEPTH, int COUT, int C, int MODE>
__global__ void __launch_bounds__(NT)
nectr_fused_kernel(const A* __restrict__ x, const A* __restrict__ AB,
                   A* __restrict__ out0,
                   A* __restrict__ out1, const Head<A, L1, DEPTH, COUT> P,
                   const ShiftTable st, int H, int W, int R,
                   int* __restrict__ invalid) {
    using A2 = typename Pair2<A>::T;
    constexpr int N2 = L1 / 2;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int XH = TH + 2 * R, XW = TW + 2 * R;
    const int plane = XH * XW;
    A2* sA = reinterpret_cast<A2*>(smem_raw);   // [L1 / 2][XH][XW] channel pairs
    A2* sB = sA + N2 * plane;                   // [L1 / 2][XH][XW]
    A* sX = reinterpret_cast<A*>(sB + N2 * plane);   // [C][XH][XW]
    const int b = blockIdx.z;
    const int h0 = blockIdx.y * TH, w0 = blockIdx.x * TW;
    const int64_t HW = static_cast<int64_t>(H) * W;

    // ---- stage A, Bm, x with an R halo (zeros outside the image: every
    // term that would read there is masked)
    {
        // AB is (B, 2 L1, H, W): channels [0, L1) the centre term W1[:, :L] g,
        // [L1, 2 L1) the shifted term W1[:, L:] g
        const A* a0 = AB + static_cast<int64_t>(b) * 2 * L1 * HW;
        const A* b0 = a0 + static_cast<int64_t>(L1) * HW;
        const A* x0 = x + static_cast<int64_t>(b) * C * HW;
        for (int e = threadIdx.x; e < plane; e += NT) {
            const int r = e / XW, c = e - r * XW;
            const int gh = h0 - R + r, gw = w0 - R + c;
            const bool in = gh >= 0 && gh < H && gw >= 0 && gw < W;
            const int64_t o = in ? static_cast<int64_t>(gh) * W + gw : 0;
#pragma unroll
            for (int k = 0; k < N2; ++k) {
                sA[k * plane + e] = in ? A2{a0[(2 * k) * HW + o] + P.bias1[2 * k],
                                            a0[(2 * k + 1) * HW + o] + P.bias1[2 * k + 1]}
                                       : A2{A(0), A(0)};
                sB[k * plane + e] = in ? A2{b0[(2 * k) * HW + o], b0[(2 * k + 1) * HW + o]}
                                       : A2{A(0), A(0)};
            }
#pragma unroll
            for (int c2 = 0; c2 < C; ++c2) sX[c2 * plane + e] = in ? x0[c2 * HW + o] : A(0);
        }
    }
    __syncthreads();

    const int tr = threadIdx.x / TW, tc = threadIdx.x % TW;
    const int h = h0 + tr, w = w0 + tc;
    if (h >= H || w >= W) return;
    const int own = (tr + R) * XW + (tc + R);
    A2 Ap[N2], Bp[N2];
#pragma unroll
    for (int k = 0; k < N2; ++k) {
        Ap[k] = sA[k * plane + own];
        Bp[k] = sB[k * plane + own];
    }
    Acc1<A, MODE> acc[C];
#pragma unroll
    for (int c = 0; c < C; ++c) acc[c].init();

    for (int s = 0; s < st.S; ++s) {
        const int dx = st.dx[s], dy = st.dy[s];
        // Both terms are evaluated unconditionally (their halo addresses are
        // always inside the staged tile) so the two independent head
        // evaluations interleave; the inside tests select what is added.
        const bool fin = h + dx >= 0 && h + dx < H && w + dy >= 0 && w + dy < W;
        const bool min = st.has_inv(s) && h - dx >= 0 && h - dx < H &&
                         w - dy >= 0 && w - dy < W;
        const int qf = own + dx * XW + dy;
        const int qm = own - dx * XW - dy;
        A2 hf[N2], hm[N2];
#pragma unroll
        for (int k = 0; k < N2; ++k) {
            hf[k] = add2(Ap[k], sB[k * plane + qf]);
            hm[k] = add2(sA[k * plane + qm], Bp[k]);
        }
        A kf[C], km[C];
        head_keys<A, L1, DEPTH, COUT, C, MODE>(hf, P, kf);
        head_keys<A, L1, DEPTH, COUT, C, MODE>(hm, P, km);
#pragma unroll
        for (int c = 0; c < C; ++c) {
            if (fin) acc[c].add(kf[c], sX[c * plane + qf]);
            if (min) acc[c].add(km[c], sX[c * plane + qm]);
        }
    }

    bool bad = false;
    const int64_t pix = static_cast<int64_t>(h) * W + w;
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const int64_t o = (static_cast<int64_t>(b) * C + c) * HW + pix;
        const A z = acc[c].z;
        if constexpr (MODE == 0) {
            out0[o] = acc[c].u;
            out1[o] = z;
        } else if (z != z) {
            bad = true;
            out0[o] = A(NAN);
            out1[o] = A(NAN);
        } else if (z == A(0)) {
            out0[o] = A(0);
            out1[o] = A(-INFINITY);
        } else {
            out0[o] = acc[c].u / z;
            const A base = MODE == 1 ? (sizeof(A) == 4 ? acc[c].m * A(0.6931471805599453)
                                                       : acc[c].m)
                                     : log(acc[c].m);
            out1[o] = base + log(z);
        }
    }
    if (bad && invalid) atomicOr(invalid, 1);
}

template <typename A, int L1, int DEPTH, int COUT, int C, int MODE>
nsc_status launch(const void* x, const void* AB, void* o0, void* o1,
                  const double* params, int64_t n_params, const ShiftTable& st,
                  int64_t B, int64_t H, int64_t W, double eps1, double eps2,
                  double slope, double inv_s2, int* invalid, cudaStream_t stream) {
    using Hd = Head<A, L1, DEPTH, COUT>;
    constexpr int L2 = Hd::L2, LK = Hd::LK;
    const int64_t need = 3 * L1 + (DEPTH == 2 ? L2 * L1 + 3 * L2 : 0) + COUT * LK;
    if (n_params != need)
        return fail(NSC_ERR_INVALID_ARG,
                    "nectr_fused: %lld head parameters given, %lld expected",
                    (long long)n_params, (long long)need);
    Hd P;
    const double* p = params;
    auto pair = [&](typename Pair2<A>::T* dst, int n) {   // n values -> n / 2 pairs
        for (int j = 0; j < n / 2; ++j) {
            dst[j].x = static_cast<A>(p[2 * j]);
            dst[j].y = static_cast<A>(p[2 * j + 1]);
        }
        p += n;
    };
    for (int j = 0; j < L1; ++j) P.bias1[j] = static_cast<A>(*p++);
    pair(P.g1, L1);
    pair(P.b1, L1);
    if constexpr (DEPTH == 2) {
        pair(P.w2, L2 * L1);
        for (int j = 0; j < L2; ++j) P.c2[j] = static_cast<A>(*p++);
        pair(P.g2, L2);
        pair(P.b2, L2);
    }
    pair(P.wo, COUT * LK);
    P.eps1 = static_cast<A>(eps1);
    P.eps2 = static_cast<A>(eps2);
    P.slope = static_cast<A>(slope);
    P.inv_s2 = static_cast<A>(inv_s2);
    const int R = st.R;
    const size_t smem = static_cast<size_t>(2 * L1 + C) * (TH + 2 * R) * (TW + 2 * R) * sizeof(A);
    static_assert(L1 % 4 == 0, "pairs of the second block's width");
    if (smem > 227u * 1024u)
        return fail(NSC_ERR_INVALID_ARG,
                    "nectr_fused: the %zu-byte tile (L=%d, R=%d) exceeds shared memory",
                    smem, L1, R);
    auto k = nectr_fused_kernel<A, L1, DEPTH, COUT, C, MODE>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess) {
        cudaGetLastError();
        return fail(NSC_ERR_LAUNCH_FAILED, "nectr_fused: shared memory attribute");
    }
    const dim3 grid(grid_1d(W, TW), grid_1d(H, TH), static_cast<unsigned>(B));
    k<<<grid, NT, smem, stream>>>(static_cast<const A*>(x), static_cast<const A*>(AB),
                                  static_cast<A*>(o0),
                                  static_cast<A*>(o1), P, st, static_cast<int>(H),
                                  static_cast<int>(W), R, invalid);
    return check_launch("nectr_fused");
}

template <typename A, int L1, int DEPTH, int C>
nsc_status by_mode(int mode, const void* x, const void* AB, void* o0,
                   void* o1, const double* params, int64_t n_params, const ShiftTable& st,
                   int64_t B, int64_t H, int64_t W, double e1, double e2, double sl,
                   double is2, int* inv, cudaStream_t s) {
    if (mode == 1)
        return launch<A, L1, DEPTH, C, C, 1>(x, AB, o0, o1, params, n_params, st, B,
                                             H, W, e1, e2, sl, is2, inv, s);
    if (mode == 2)
        return launch<A, L1, DEPTH, 3 * C, C, 2>(x, AB, o0, o1, params, n_params, st,
                                                 B, H, W, e1, e2, sl, is2, inv, s);
    return launch<A, L1, DEPTH, C, C, 0>(x, AB, o0, o1, params, n_params, st, B, H,
                                         W, e1, e2, sl, is2, inv, s);
}

template <typename A, int L1, int DEPTH>
nsc_status by_c(int64_t C, int mode, const void* x, const void* AB,
                void* o0, void* o1, const double* params, int64_t n_params,
                const ShiftTable& st, int64_t B, int64_t H, int64_t W, double e1,
                double e2, double sl, double is2, int* inv, cudaStream_t s) {
    if (C == 1)
        return by_mode<A, L1, DEPTH, 1>(mode, x, AB, o0, o1, params, n_params, st, B,
                                        H, W, e1, e2, sl, is2, inv, s);
    return by_mode<A, L1, DEPTH, 3>(mode, x, AB, o0, o1, params, n_params, st, B, H,
                                    W, e1, e2, sl, is2, inv, s);
}

template <typename A>
nsc_status by_shape(int64_t L1, int depth, int64_t C, int mode, const void* x,
                    const void* AB, void* o0, void* o1,
                    const double* params, int64_t n_params, const ShiftTable& st,
                    int64_t B, int64_t H, int64_t W, double e1, double e2, double sl,
                    double is2, int* inv, cudaStream_t s) {
#define NSC_NF(LL, DD)                                                                 \
    if (L1 == LL && depth == DD)                                                       \
        return by_c<A, LL, DD>(C, mode, x, AB, o0, o1, params, n_params, st, B, H,  \
                               W, e1, e2, sl, is2, inv, s);
    NSC_NF(8, 1) NSC_NF(16, 1) NSC_NF(32, 1) NSC_NF(8, 2) NSC_NF(16, 2) NSC_NF(32, 2)
#undef NSC_NF
    return fail(NSC_ERR_INVALID_ARG,
                "nectr_fused: head width %lld with %d blocks is not built (widths "
                "8, 16, 32; 1 or 2 blocks)", (long long)L1, depth);
}

}  // namespace nectr
}  // namespace nsc

extern "C" nsc_status nsc_nectr_fused_fwd(
    const void* x, const void* AB_map, int dtype, int64_t B,
    int64_t C, int64_t H, int64_t W, int64_t width, int depth, const double* params,
    int64_t n_params, double ln_eps1, double ln_eps2, double slope, double inv_sigma2,
    const int64_t* shifts, int64_t S, int mode, void* out0, void* out1,
    int* invalid_flag, void* stream) {
    using namespace nsc;
    const char* op = "nectr_fused";
    nsc_status e = check_extents(op, B, C, H, W);
    if (e) return e;
    if (dtype != NSC_F32 && dtype != NSC_F64)
        return fail(NSC_ERR_UNSUPPORTED_DTYPE, "%s: dtype must be fp32 or fp64", op);
    if (C != 1 && C != 3)
        return fail(NSC_ERR_INVALID_ARG, "%s: C must be 1 or 3 (got %lld)", op, (long long)C);
    if (mode < 0 || mode > 2)
        return fail(NSC_ERR_INVALID_ARG, "%s: mode must be 0, 1 or 2", op);
    if (B > 65535 || H >= (1LL << 30) || W >= (1LL << 30))
        return fail(NSC_ERR_INVALID_ARG, "%s: extent too large", op);
    ShiftTable st;
    e = build_shifts(op, shifts, S, 3, H, W, &st);
    if (e) return e;
    if (st.any_per)
        return fail(NSC_ERR_INVALID_ARG, "%s: masked mirror rows only (column 0 or 1)", op);
    if (st.R > 16) return fail(NSC_ERR_INVALID_ARG, "%s: table radius above 16", op);
    if (B == 0 || H == 0 || W == 0) return ok();
    if (!x || !AB_map || !out0 || !out1 || !params)
        return fail(NSC_ERR_INVALID_ARG, "%s: NULL pointer", op);
    cudaStream_t s = as_stream(stream);
    if (dtype == NSC_F32)
        return nectr::by_shape<float>(width, depth, C, mode, x, AB_map, out0, out1,
                                      params, n_params, st, B, H, W, ln_eps1, ln_eps2,
                                      slope, inv_sigma2, invalid_flag, s);
    return nectr::by_shape<double>(width, depth, C, mode, x, AB_map, out0, out1,
                                   params, n_params, st, B, H, W, ln_eps1, ln_eps2, slope,
                                   inv_sigma2, invalid_flag, s);
}
