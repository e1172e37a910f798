// gather.cu -- shift_gather / pair_gather forward (+ validity mask) and
// their deterministic gather-form backward, for sm_100a.
//
// Forward: every output element is a copy, so the kernel moves storage
// words (2/4/8 bytes) and is bit-exact for every dtype.  One CTA handles a
// run of in-plane units of one output plane; a unit is VEC consecutive
// columns of one row written with a single 16-byte store when rows are
// 16-byte aligned.  The source guide (B*C planes) is small next to the
// S-fold output and stays in L1/L2, so HBM sees the output writes once.
// The mask plane of (s, b) is written by the CTAs of channel 0 in the same
// launch (the reference uses a second kernel, shift_ops_cuda.cu:134-157).
//
// Backward: gather form.  Each output element of grad_guide owns the sum of
// its S contributions (a circular shift is a bijection), accumulated in
// fp32 (fp64 for fp64) in shift order.  The reference's pair_gather
// backward scatters with atomicAdd (shift_ops_cuda.cu:206-246); this one is
// deterministic.

#include <cstdlib>

#include "nsc_common.cuh"
#include "nsc_host.h"

namespace nsc {
namespace {

constexpr int kThreads = 256;

template <int BYTES> struct Word;
template <> struct Word<2> { using type = uint16_t; };
template <> struct Word<4> { using type = uint32_t; };
template <> struct Word<8> { using type = unsigned long long; };

template <typename E, int V>
struct alignas(16) Vec { E v[V]; };

// planes: S*B*Cout output planes; Cout = C (shift) or 2C (pair).
template <typename E, int V>
__global__ void __launch_bounds__(kThreads)
gather_fwd_kernel(const E* __restrict__ guide, E* __restrict__ out,
                  E* __restrict__ mask, const ShiftTable st, int64_t B,
                  int64_t C, int64_t H, int64_t W, int pair, E one,
                  int64_t planes, int64_t units_per_plane) {
    const int64_t Cout = pair ? 2 * C : C;
    const int64_t nWv = W / V;  // V divides W on this path
    const int64_t HW = H * W;
    for (int64_t plane = blockIdx.y; plane < planes; plane += gridDim.y) {
        const int64_t cp = plane % Cout;
        const int64_t sb = plane / Cout;
        const int64_t b = sb % B;
        const int s = static_cast<int>(sb / B);
        const bool center = pair && cp < C;
        const int64_t c = pair ? (center ? cp : cp - C) : cp;
        const int64_t dx = center ? 0 : st.dx[s];
        const int64_t dy = center ? 0 : st.dy[s];
        const E* src = guide + (b * C + c) * HW;
        E* dst = out + plane * HW;
        const bool write_mask = (cp == 0);
        const int64_t mdx = st.dx[s], mdy = st.dy[s];
        E* mdst = mask + sb * HW;
        for (int64_t u = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
             u < units_per_plane; u += static_cast<int64_t>(gridDim.x) * kThreads) {
            const int64_t h = u / nWv;
            const int64_t w0 = (u - h * nWv) * V;
            const int64_t sh = wrap1(h + dx, H);
            const E* srow = src + sh * W;
            Vec<E, V> r;
#pragma unroll
            for (int i = 0; i < V; ++i) r.v[i] = __ldg(srow + wrap1(w0 + i + dy, W));
            *reinterpret_cast<Vec<E, V>*>(dst + h * W + w0) = r;
            if (write_mask) {
                const bool hv = inb(h + mdx, H);
                Vec<E, V> m;
#pragma unroll
                for (int i = 0; i < V; ++i)
                    m.v[i] = (hv && inb(w0 + i + mdy, W)) ? one : E(0);
                *reinterpret_cast<Vec<E, V>*>(mdst + h * W + w0) = m;
            }
        }
    }
}

// Tiled forward.  One CTA owns a TH x TW tile of one guide plane (b, c):
// it stages the tile plus its (Rx, Ry) halo -- rows and columns wrapped
// circularly -- in shared memory once, then writes the tile of every
// output plane that reads it: the S shifted copies, the S centre copies of
// pair_gather, and (channel 0 only) the S mask tiles.  Each thread writes
// one 16-byte vector per row with a streaming store (the S-fold output is
// written once and never re-read here, so it must not evict the guide from
// L2).  HBM sees the output once and the guide about once.
constexpr int kTileRows = 16;

__device__ __forceinline__ int pmod32(int a, int n) {
    const int r = a % n;
    return r < 0 ? r + n : r;
}

template <typename E, int V>
__global__ void __launch_bounds__(kThreads)
gather_tile_kernel(const E* __restrict__ guide, E* __restrict__ out,
                   E* __restrict__ mask, const ShiftTable st, int B, int C,
                   int H, int W, int pair, E one, int Rx, int Ry,
                   int tiles_x, int64_t ntiles, int64_t planes) {
    constexpr int TW = 32 * V;
    using Vec16 = Vec<E, V>;
    extern __shared__ __align__(16) unsigned char smem_g[];
    E* xs = reinterpret_cast<E*>(smem_g);
    const int XP = TW + 2 * Ry;          // halo row pitch (elements)
    const int XR = kTileRows + 2 * Rx;   // halo rows
    const int tid = threadIdx.x;
    const int lx = tid & 31, ly = tid >> 5;
    const int Cout = pair ? 2 * C : C;
    const int64_t HW = static_cast<int64_t>(H) * W;
    for (int64_t plane = blockIdx.y; plane < planes; plane += gridDim.y) {
        const int b = static_cast<int>(plane / C);
        const int c = static_cast<int>(plane - static_cast<int64_t>(b) * C);
        const E* src = guide + plane * HW;
        for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            const int ty = static_cast<int>(tile / tiles_x);
            const int tx = static_cast<int>(tile - static_cast<int64_t>(ty) * tiles_x);
            const int h0 = ty * kTileRows, w0 = tx * TW;
            __syncthreads();   // previous tile's readers are done
            for (int idx = tid; idx < XR * XP; idx += kThreads) {
                const int i = idx / XP;
                const int j = idx - i * XP;
                const int r = pmod32(h0 - Rx + i, H);
                const int col = pmod32(w0 - Ry + j, W);
                xs[idx] = __ldg(src + static_cast<int64_t>(r) * W + col);
            }
            __syncthreads();
            const int wc = w0 + lx * V;
            // centre vectors of this thread's rows (pair_gather)
            Vec16 ctr[kTileRows / 8];
#pragma unroll
            for (int p = 0; p < kTileRows / 8; ++p) {
                const int r = p * 8 + ly;
#pragma unroll
                for (int i = 0; i < V; ++i) ctr[p].v[i] = xs[(r + Rx) * XP + Ry + lx * V + i];
            }
            for (int s = 0; s < st.S; ++s) {
                const int dx = st.dx[s], dy = st.dy[s];
                const int64_t sb = static_cast<int64_t>(s) * B + b;
                E* dsh = out + (sb * Cout + (pair ? C + c : c)) * HW;
                E* dce = out + (sb * Cout + c) * HW;
                E* dm = mask + sb * HW;
#pragma unroll
                for (int p = 0; p < kTileRows / 8; ++p) {
                    const int r = p * 8 + ly;
                    const int h = h0 + r;
                    if (h >= H || wc >= W) continue;
                    const int64_t o = static_cast<int64_t>(h) * W + wc;
                    Vec16 v;
                    const E* row = xs + (r + dx + Rx) * XP + Ry + lx * V + dy;
#pragma unroll
                    for (int i = 0; i < V; ++i) v.v[i] = row[i];
                    __stcs(reinterpret_cast<uint4*>(dsh + o),
                           *reinterpret_cast<const uint4*>(&v));
                    if (pair)
                        __stcs(reinterpret_cast<uint4*>(dce + o),
                               *reinterpret_cast<const uint4*>(&ctr[p]));
                    if (c == 0) {
                        const bool hv = h + dx >= 0 && h + dx < H;
                        Vec16 m;
#pragma unroll
                        for (int i = 0; i < V; ++i) {
                            const int q = wc + i + dy;
                            m.v[i] = (hv && q >= 0 && q < W) ? one : E(0);
                        }
                        __stcs(reinterpret_cast<uint4*>(dm + o),
                               *reinterpret_cast<const uint4*>(&m));
                    }
                }
            }
        }
    }
}

// Backward: grad_guide(b, c, g) = sum_s go_shift(s, b, c, g - d_s) [+ the
// centre half go(s, b, c, g) for pair_gather].
template <typename T>
__global__ void __launch_bounds__(kThreads)
gather_bwd_kernel(const T* __restrict__ go, T* __restrict__ gg,
                  const ShiftTable st, int64_t B, int64_t C, int64_t H,
                  int64_t W, int pair) {
    using A = typename Acc<T>::type;
    const int64_t Cout = pair ? 2 * C : C;
    const int64_t HW = H * W;
    const int64_t planes = B * C;
    for (int64_t plane = blockIdx.y; plane < planes; plane += gridDim.y) {
        const int64_t b = plane / C;
        const int64_t c = plane % C;
        for (int64_t u = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
             u < HW; u += static_cast<int64_t>(gridDim.x) * kThreads) {
            const int64_t h = u / W;
            const int64_t w = u - h * W;
            A acc = A(0);
            for (int s = 0; s < st.S; ++s) {
                const int64_t base = ((static_cast<int64_t>(s) * B + b) * Cout) * HW;
                if (pair) acc += ldg_acc<T, A>(go + base + c * HW + u);
                const int64_t hs = wrap1(h - st.dx[s], H);
                const int64_t ws = wrap1(w - st.dy[s], W);
                const int64_t cs = pair ? C + c : c;
                acc += ldg_acc<T, A>(go + base + cs * HW + hs * W + ws);
            }
            gg[plane * HW + u] = static_cast<T>(acc);
        }
    }
}

template <typename E, int V>
void launch_fwd(const void* guide, void* out, void* mask, const ShiftTable& st,
                int64_t B, int64_t C, int64_t H, int64_t W, int pair, E one,
                cudaStream_t stream) {
    const int64_t Cout = pair ? 2 * C : C;
    const int64_t planes = static_cast<int64_t>(st.S) * B * Cout;
    const int64_t units = H * (W / V);
    unsigned gx = grid_1d(units, kThreads, 1 << 16);
    unsigned gy = static_cast<unsigned>(planes < 65535 ? planes : 65535);
    gather_fwd_kernel<E, V><<<dim3(gx, gy), kThreads, 0, stream>>>(
        static_cast<const E*>(guide), static_cast<E*>(out), static_cast<E*>(mask),
        st, B, C, H, W, pair, one, planes, units);
}

// The tiled path: 16-byte aligned rows, halo within 32 rows / 64 columns,
// per-dimension extents below 2^31 (intra-plane int32 indexing).
template <typename E>
bool launch_tile(const void* guide, void* out, void* mask, const ShiftTable& st,
                 int64_t B, int64_t C, int64_t H, int64_t W, int pair, E one,
                 cudaStream_t stream) {
    constexpr int V = 16 / sizeof(E);
    constexpr int TW = 32 * V;
    if (H >= (1LL << 30) || W >= (1LL << 30) || B * C * 2 >= (1LL << 30)) return false;
    int Rx = 0, Ry = 0;
    for (int s = 0; s < st.S; ++s) {
        Rx = st.dx[s] < 0 ? (-st.dx[s] > Rx ? -st.dx[s] : Rx) : (st.dx[s] > Rx ? st.dx[s] : Rx);
        Ry = st.dy[s] < 0 ? (-st.dy[s] > Ry ? -st.dy[s] : Ry) : (st.dy[s] > Ry ? st.dy[s] : Ry);
    }
    if (Rx > 32 || Ry > 64) return false;
    Ry = (Ry + V - 1) / V * V;   // keeps the centre vectors 16-byte aligned
    const size_t smem = static_cast<size_t>(kTileRows + 2 * Rx) * (TW + 2 * Ry) * sizeof(E);
    if (smem > 96 * 1024) return false;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(gather_tile_kernel<E, V>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return false;
    const int tiles_x = static_cast<int>((W + TW - 1) / TW);
    const int64_t ntiles = static_cast<int64_t>(tiles_x) * ((H + kTileRows - 1) / kTileRows);
    const int64_t planes = B * C;
    const unsigned gx = static_cast<unsigned>(ntiles < (1LL << 31) - 1 ? ntiles : (1LL << 31) - 1);
    const unsigned gy = static_cast<unsigned>(planes < 65535 ? planes : 65535);
    gather_tile_kernel<E, V><<<dim3(gx, gy), kThreads, smem, stream>>>(
        static_cast<const E*>(guide), static_cast<E*>(out), static_cast<E*>(mask), st,
        static_cast<int>(B), static_cast<int>(C), static_cast<int>(H),
        static_cast<int>(W), pair, one, Rx, Ry, tiles_x, ntiles, planes);
    return true;
}

template <typename E>
void dispatch_fwd(const void* guide, void* out, void* mask, const ShiftTable& st,
                  int64_t B, int64_t C, int64_t H, int64_t W, int pair, E one,
                  cudaStream_t stream) {
    constexpr int V = 16 / sizeof(E);
    const bool aligned = (W % V == 0) &&
                         (reinterpret_cast<uintptr_t>(out) % 16 == 0) &&
                         (reinterpret_cast<uintptr_t>(mask) % 16 == 0);
    if (aligned && !getenv("NSC_GATHER_GENERIC") &&
        launch_tile<E>(guide, out, mask, st, B, C, H, W, pair, one, stream))
        return;
    if (aligned)
        launch_fwd<E, V>(guide, out, mask, st, B, C, H, W, pair, one, stream);
    else
        launch_fwd<E, 1>(guide, out, mask, st, B, C, H, W, pair, one, stream);
}

nsc_status gather_fwd(const char* op, const void* guide, int dtype, int64_t B,
                      int64_t C, int64_t H, int64_t W, const int64_t* shifts,
                      int64_t S, int64_t cols, void* out, void* mask,
                      void* stream, int pair) {
    nsc_status st0 = check_extents(op, B, C, H, W);
    if (st0) return st0;
    if (!valid_dtype(dtype))
        return fail(NSC_ERR_UNSUPPORTED_DTYPE, "%s: unsupported dtype %d", op, dtype);
    ShiftTable st;
    st0 = build_shifts(op, shifts, S, cols, H, W, &st);
    if (st0) return st0;
    if (B == 0 || H == 0 || W == 0) return ok();
    if (!guide || !out || !mask)
        return fail(NSC_ERR_INVALID_ARG, "%s: NULL tensor pointer", op);
    cudaStream_t s = as_stream(stream);
    if (C == 0) return fail(NSC_ERR_INVALID_ARG, "%s: C must be >= 1", op);
    switch (dtype) {
        case NSC_F16: dispatch_fwd<uint16_t>(guide, out, mask, st, B, C, H, W, pair, 0x3C00u, s); break;
        case NSC_BF16: dispatch_fwd<uint16_t>(guide, out, mask, st, B, C, H, W, pair, 0x3F80u, s); break;
        case NSC_F32: dispatch_fwd<uint32_t>(guide, out, mask, st, B, C, H, W, pair, 0x3F800000u, s); break;
        default: dispatch_fwd<unsigned long long>(guide, out, mask, st, B, C, H, W, pair, 0x3FF0000000000000ull, s); break;
    }
    return check_launch(op);
}

template <typename T>
void launch_bwd(const void* go, void* gg, const ShiftTable& st, int64_t B,
                int64_t C, int64_t H, int64_t W, int pair, cudaStream_t stream) {
    const int64_t planes = B * C;
    unsigned gx = grid_1d(H * W, kThreads, 1 << 16);
    unsigned gy = static_cast<unsigned>(planes < 65535 ? planes : 65535);
    gather_bwd_kernel<T><<<dim3(gx, gy), kThreads, 0, stream>>>(
        static_cast<const T*>(go), static_cast<T*>(gg), st, B, C, H, W, pair);
}

nsc_status gather_bwd(const char* op, const void* go, int dtype, int64_t B,
                      int64_t C, int64_t H, int64_t W, const int64_t* shifts,
                      int64_t S, int64_t cols, void* gg, void* stream, int pair) {
    nsc_status st0 = check_extents(op, B, C, H, W);
    if (st0) return st0;
    if (!valid_dtype(dtype))
        return fail(NSC_ERR_UNSUPPORTED_DTYPE, "%s: unsupported dtype %d", op, dtype);
    ShiftTable st;
    st0 = build_shifts(op, shifts, S, cols, H, W, &st);
    if (st0) return st0;
    if (B == 0 || C == 0 || H == 0 || W == 0) return ok();
    if (!go || !gg) return fail(NSC_ERR_INVALID_ARG, "%s: NULL tensor pointer", op);
    cudaStream_t s = as_stream(stream);
    switch (dtype) {
        case NSC_F16: launch_bwd<__half>(go, gg, st, B, C, H, W, pair, s); break;
        case NSC_BF16: launch_bwd<__nv_bfloat16>(go, gg, st, B, C, H, W, pair, s); break;
        case NSC_F32: launch_bwd<float>(go, gg, st, B, C, H, W, pair, s); break;
        default: launch_bwd<double>(go, gg, st, B, C, H, W, pair, s); break;
    }
    return check_launch(op);
}

}  // namespace
}  // namespace nsc

extern "C" {

nsc_status nsc_shift_gather_fwd(const void* guide, int dtype, int64_t B, int64_t C,
                                int64_t H, int64_t W, const int64_t* shifts,
                                int64_t S, int64_t shift_cols, void* out,
                                void* mask, void* stream) {
    return nsc::gather_fwd("shift_gather", guide, dtype, B, C, H, W, shifts, S,
                           shift_cols, out, mask, stream, 0);
}

nsc_status nsc_pair_gather_fwd(const void* guide, int dtype, int64_t B, int64_t C,
                               int64_t H, int64_t W, const int64_t* shifts,
                               int64_t S, int64_t shift_cols, void* out,
                               void* mask, void* stream) {
    return nsc::gather_fwd("pair_gather", guide, dtype, B, C, H, W, shifts, S,
                           shift_cols, out, mask, stream, 1);
}

nsc_status nsc_shift_gather_bwd(const void* grad_out, int dtype, int64_t B,
                                int64_t C, int64_t H, int64_t W,
                                const int64_t* shifts, int64_t S,
                                int64_t shift_cols, void* grad_guide,
                                void* stream) {
    return nsc::gather_bwd("shift_gather_backward", grad_out, dtype, B, C, H, W,
                           shifts, S, shift_cols, grad_guide, stream, 0);
}

nsc_status nsc_pair_gather_bwd(const void* grad_out, int dtype, int64_t B,
                               int64_t C, int64_t H, int64_t W,
                               const int64_t* shifts, int64_t S,
                               int64_t shift_cols, void* grad_guide,
                               void* stream) {
    return nsc::gather_bwd("pair_gather_backward", grad_out, dtype, B, C, H, W,
                           shifts, S, shift_cols, grad_guide, stream, 1);
}

}  // extern "C"
