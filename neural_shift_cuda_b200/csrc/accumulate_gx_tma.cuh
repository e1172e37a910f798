// accumulate_gx_tma.cuh -- tiled TMA grad_x of accumulate_uz for sm_100a.
//
// grad_x is the transpose of the forward operator:
//   gx_c(q) = sum_s w_s(q - d) gU_c(q - d)                 (term A, circular)
//           + inv_s [q + d inside] w_s(q) gU_c(q + d)      (term B)
// (reference shift_ops_cuda.cu:412-458 computes the same sums per pixel).
// Both weights of a shift are the two uses the forward kernel reads from ONE
// TMA box per weight plane: w_s(q) at the tile (the forward term's
// position) and w_s(q - d) on the tile shifted by -d (the mirror term's
// position).  So this kernel runs the forward kernel's pipeline -- one
// producer warp streaming the same boxes (same table, same grouping of up to
// four consecutive planes per copy) through an mbarrier ring to 15 consumer
// warps -- with the terms exchanged: the mirror-position weight always
// contributes (term A), the forward-position weight only on mirror rows
// (term B).
//
// grad_U is staged per tile as fp32 with the halo, ZERO outside the image:
// that is term B's inside test, and on border tiles it gives term A's
// products whose q - d lies outside the value 0 (the box is zero-filled
// there as well).  Those wrapped term-A contributions are added afterwards
// by acc_gx_wrap_kernel over the R-pixel border band.
//
// A consumer thread owns V = 4 consecutive output pixels of one row (one
// 16-byte fp32 store per channel); per dx row it holds the grad_U windows
// of its pixels for every channel in registers and serves every dy of the
// row with compile-time register indices, as the forward does.
#pragma once

#include "accumulate_fast.cuh"

namespace nsc {
namespace gxt {

using fast::TH;
using fast::TPR;
using fast::NCONS;
using fast::NTHREADS;
using fast::MAXR;
using fast::FastTable;
using fast::WMaps;
using fast::Geo;
using fast::GeoExt;
using fast::kGroup;
using fast::kLenShift;
using fast::kSMask;
using fast::align_up;
using fast::cmax;

constexpr int V = 4;              // output pixels per thread
constexpr int TW = TPR * V;       // tile columns

// N = 2 or 4 words (V weights) from shared memory, non-volatile: ordered
// after the stage's mbarrier wait by the address dependency (fast::after).
template <int N>
__device__ __forceinline__ void lds_w(uint32_t* d, uint32_t a) {
    if constexpr (N == 4) {
        const uint4 v = fast::lds128nv(a);
        d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
    } else {
        uint2 v;
        asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
        d[0] = v.x; d[1] = v.y;
    }
}

template <typename T, int NC, int DYMIN, int DYMAX, bool EXACT>
__global__ void __launch_bounds__(NTHREADS, 1)
acc_gx_tma_kernel(const __grid_constant__ WMaps wmaps, const float* __restrict__ gU,
                  float* __restrict__ gx, const FastTable tab, const Geo g,
                  unsigned int* timeouts, const GeoExt ge) {
    constexpr int VA = 16 / static_cast<int>(sizeof(T));   // box column granule
    constexpr int WPV = V * static_cast<int>(sizeof(T)) / 4;   // words per V weights
    constexpr int XC = align_up(cmax(DYMAX, -DYMIN), V);   // grad_U halo columns
    // register windows in fp32 elements relative to the thread's first
    // column: term B reads gU(q + d), term A reads gU(q - d)
    constexpr int FLO = XC + DYMIN, FHI = XC + DYMAX + V;
    constexpr int MLO = XC - DYMAX, MHI = XC - DYMIN + V;
    constexpr int NDY = DYMAX - DYMIN + 1;

    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    const int NSTAGE = g.nstage;
    unsigned char* stages = smem;
    float* xa = reinterpret_cast<float*>(smem + NSTAGE * g.stage_stride);
    const int xtile = NC * g.XH * g.XW;
    uint64_t* full = reinterpret_cast<uint64_t*>(
        (reinterpret_cast<uintptr_t>(xa + xtile) + 15) & ~uintptr_t(15));
    uint64_t* empty = full + NSTAGE;
    int& abort_flag = *reinterpret_cast<int*>(empty + NSTAGE);

    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < NSTAGE; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], NCONS / 32);
        }
        abort_flag = 0;
        (&abort_flag)[1] = static_cast<int>(ge.wait_budget);   // read by the slow waits
        fence_mbar_init();
    }
    __syncthreads();

    const int Rx = tab.Rx;
    const int64_t cgroups = (g.Cw == 1) ? 1 : g.C;

    // ------------------------------------------------------------ producer
    // Tiles blockIdx.x, blockIdx.x + gridDim.x, ...: at any time the CTAs
    // work on one band of consecutive tiles, whose overlapping boxes meet in
    // L2.
    if (tid >= NCONS) {
        if (tid != NCONS) return;
        uint32_t it = 0;
        int stage = 0;
        uint32_t phase = 0;
        bool aborted = false;
        for (int64_t tile = blockIdx.x; tile < g.ntiles && !aborted; tile += gridDim.x) {
            const fast::TileId id = fast::decode_tile(tile, g, 0, TW, cgroups);
            const int64_t wc = (g.Cw == 1) ? 0 : id.grp % cgroups;
            for (int dx = -Rx; dx <= Rx && !aborted; ++dx) {
                if (!tab.row_any[dx + MAXR]) continue;
                for (int dy = DYMIN; dy <= DYMAX; ++dy) {
                    const int e = tab.s[dx + MAXR][dy + MAXR];
                    const int len = (e >> kLenShift) & 7;
                    if (e < 0 || len == 0) continue;
                    const int s = e & kSMask;
                    if (!mbar_wait(&empty[stage], phase ^ 1u, timeouts, ge.wait_budget) ||
                        *(volatile int*)&abort_flag) {
                        aborted = true;
                        *(volatile int*)&abort_flag = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(&full[stage], len * g.plane_bytes);
                    const int mo = dy > 0 ? align_up(dy, VA) : 0;
                    const CUtensorMap* map = len == 1 ? &wmaps.m[0]
                                             : len == 2 ? &wmaps.m[1]
                                             : len == 3 ? &wmaps.m[2] : &wmaps.m[3];
                    tma_load_4d(stages + stage * g.stage_stride, map, &full[stage],
                                id.w0 - mo, id.h0 - (dx > 0 ? dx : 0),
                                static_cast<int32_t>(id.b * g.Cw + wc), s);
                    ++it;
                    if (++stage == NSTAGE) { stage = 0; phase ^= 1u; }
                }
            }
        }
        // the CTA must not exit with copies into its shared memory in flight
        const uint32_t n = it < static_cast<uint32_t>(NSTAGE) ? it : NSTAGE;
        for (uint32_t j = it - n; j < it; ++j)
            mbar_wait(&full[j % NSTAGE], (j / NSTAGE) & 1u, timeouts, ge.wait_budget);
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
    const int nv = XW / V;
    const int xtotal = NC * XH * nv;
    const int64_t HW = g.H * g.W;

    for (int64_t tile = blockIdx.x; tile < g.ntiles; tile += gridDim.x) {
        const fast::TileId id = fast::decode_tile(tile, g, 0, TW, cgroups);
        const int64_t b = id.b;
        const int64_t c0 = (g.Cw == 1) ? 0 : id.grp % cgroups;
        const int h0 = id.h0, w0 = id.w0;

        // ---- stage grad_U (fp32, zero outside the image)
        named_sync(1, NCONS);   // every thread is done with the previous tile
        for (int idx = tid; idx < xtotal; idx += NCONS) {
            const int c = idx / (XH * nv);
            const int rem = idx - c * XH * nv;
            const int i = rem / nv;
            const int jv = rem - i * nv;
            const int64_t r = static_cast<int64_t>(h0) - Rx + i;
            const int64_t col0 = static_cast<int64_t>(w0) - XC + jv * V;
            float* dst = xa + (c * XH + i) * XW + jv * V;
            // W % 4 == 0 and col0 % 4 == 0: a chunk is wholly inside or outside
            if (r >= 0 && r < g.H && col0 >= 0 && col0 < g.W)
                fast::cp_async16(dst, gU + (b * g.C + c0 + c) * HW + r * g.W + col0);
            else
                *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        fast::cp_async_commit();
        fast::cp_async_wait_all();
        named_sync(1, NCONS);
        if (*(volatile int*)&abort_flag) break;

        float acc[NC][V];
#pragma unroll
        for (int c = 0; c < NC; ++c)
#pragma unroll
            for (int i = 0; i < V; ++i) acc[c][i] = 0.f;

        const uint32_t xa32 = smem_u32(xa) + static_cast<uint32_t>(tc * V * 4);
        const uint32_t xplane = static_cast<uint32_t>(XH * XW * 4);
        for (int dx = -Rx; dx <= Rx; ++dx) {
            if (!tab.row_any[dx + MAXR]) continue;
            uint32_t gfw[NC][FHI - FLO], gmw[NC][MHI - MLO];   // fp32 bit patterns
#pragma unroll
            for (int c = 0; c < NC; ++c)
                fast::load_win32<MLO, MHI, MLO>(gmw[c], xa32 + c * xplane +
                    static_cast<uint32_t>((tr - dx + Rx) * XW * 4));
            if (tab.row_inv[dx + MAXR]) {
#pragma unroll
                for (int c = 0; c < NC; ++c)
                    fast::load_win32<FLO, FHI, FLO>(gfw[c], xa32 + c * xplane +
                        static_cast<uint32_t>((tr + dx + Rx) * XW * 4));
            }
            const int mrow0 = tr + (dx > 0 ? dx : 0);
            const uint32_t off_main = static_cast<uint32_t>((mrow0 * BW + tc * V) * sizeof(T));
            const uint32_t off_mir = static_cast<uint32_t>(((mrow0 - dx) * BW + tc * V) * sizeof(T));
            const uint64_t m_pres = tab.present[dx + MAXR], m_inv = tab.inv[dx + MAXR];
            const uint64_t m_pos0 = tab.pos0[dx + MAXR], m_pos1 = tab.pos1[dx + MAXR];
            const uint64_t m_last = tab.last[dx + MAXR];
            uint32_t stp = stages32 + stage * g.stage_stride;
            auto one = [&](auto dyc, const int pos, const bool last, const bool inv) {
                constexpr int dy = decltype(dyc)::value;
                if (pos == 0)
                    mbar_wait32_ab(full32 + 8 * stage, phase, timeouts,
                                   (volatile int*)&abort_flag);
                const uint32_t sp = fast::after(stp) + pos * g.plane_bytes;
                constexpr int mo = dy > 0 ? align_up(dy, VA) : 0;
                // term A: w_s(q - d) gU(q - d)
                {
                    constexpr int moff = mo - dy;               // >= 0
                    constexpr int kk = moff % V;
                    constexpr int mb = moff - kk;
                    uint32_t mw[2 * WPV];
                    lds_w<WPV>(mw, sp + off_mir + mb * sizeof(T));
                    if constexpr (kk != 0)
                        lds_w<WPV>(mw + WPV, sp + off_mir + (mb + V) * sizeof(T));
                    fast::static_for<0, V>([&](auto ic) {
                        constexpr int i = decltype(ic)::value;
                        const float wv = fast::elem_f<T, kk + i>(mw);
#pragma unroll
                        for (int c = 0; c < NC; ++c)
                            acc[c][i] = fmaf(wv, __uint_as_float(gmw[c][XC - dy + i - MLO]),
                                             acc[c][i]);
                    });
                }
                // term B (mirror rows): w_s(q) gU(q + d)
                if (inv) {
                    uint32_t wq[WPV];
                    lds_w<WPV>(wq, sp + off_main + mo * sizeof(T));
                    fast::static_for<0, V>([&](auto ic) {
                        constexpr int i = decltype(ic)::value;
                        const float wv = fast::elem_f<T, i>(wq);
#pragma unroll
                        for (int c = 0; c < NC; ++c)
                            acc[c][i] = fmaf(wv, __uint_as_float(gfw[c][XC + dy + i - FLO]),
                                             acc[c][i]);
                    });
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
                if (dx >= 0) one(std::integral_constant<int, 0>{}, 0, true, dx != 0);
                const int R = tab.Rdy;
                fast::static_for<1, DYMAX + 1>([&](auto jc) {
                    constexpr int dy = decltype(jc)::value;
                    if (dy > R) return;
                    constexpr int p = (dy - 1) % kGroup;
                    one(jc, p, p == kGroup - 1 || dy == R, true);
                });
            } else {
                fast::static_for<0, NDY>([&](auto jc) {
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
        if (h < g.H && wcol < g.W) {
#pragma unroll
            for (int c = 0; c < NC; ++c)
                *reinterpret_cast<float4*>(gx + (b * g.C + c0 + c) * HW + h * g.W + wcol) =
                    make_float4(acc[c][0], acc[c][1], acc[c][2], acc[c][3]);
        }
    }
    fast::cp_async_wait_all();
}

}  // namespace gxt
}  // namespace nsc

// ------------------------------------------------------------------ host
namespace nsc {
int fast_sm_count();
void fast_set_decline(const char* why);

namespace gxt {

template <typename T, int NC, int DYMIN, int DYMAX, bool EXACT>
bool launch(const WMaps& maps, const void* gU, void* gx, const FastTable& tab, Geo g,
            GeoExt ge, unsigned int* timeouts, cudaStream_t stream) {
    // ring depth: as many weight stages (<= 12) as fit next to the grad_U tile
    const size_t fixed = static_cast<size_t>(NC) * g.XH * g.XW * sizeof(float) +
                         16 + 16 + 128;
    const size_t per_stage = g.stage_stride + 2 * sizeof(uint64_t);
    const size_t cap = 227u * 1024u;
    if (fixed + 3 * per_stage > cap) {
        fast_set_decline("shared memory");
        return false;
    }
    size_t ns = (cap - fixed) / per_stage;
    if (ns > 12) ns = 12;
    g.nstage = static_cast<int32_t>(ns);
    const size_t smem = fixed + ns * per_stage;
    auto k = acc_gx_tma_kernel<T, NC, DYMIN, DYMAX, EXACT>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess) {
        cudaGetLastError();
        fast_set_decline("dynamic shared memory attribute");
        return false;
    }
    const int64_t nsm = fast_sm_count();
    const unsigned grid = static_cast<unsigned>(g.ntiles < nsm ? g.ntiles : nsm);
    k<<<grid, NTHREADS, smem, stream>>>(maps, static_cast<const float*>(gU),
                                        static_cast<float*>(gx), tab, g, timeouts, ge);
    return true;
}

}  // namespace gxt
}  // namespace nsc

#define NSC_GXT_ONE(X, T, NC, A, B, E)                                               \
    X template bool nsc::gxt::launch<T, NC, A, B, E>(const nsc::fast::WMaps&,         \
        const void*, void*, const nsc::fast::FastTable&, nsc::fast::Geo,              \
        nsc::fast::GeoExt, unsigned int*, cudaStream_t);
// Every table bucket of one weight type and image-channel count (X empty:
// instantiate; X extern: declare the instantiation made elsewhere).
#define NSC_GXT_BUCKETS(X, T, NC)                                                    \
    NSC_GXT_ONE(X, T, NC, 0, 2, true) NSC_GXT_ONE(X, T, NC, 0, 4, true)              \
    NSC_GXT_ONE(X, T, NC, 0, 6, true) NSC_GXT_ONE(X, T, NC, 0, 8, true)              \
    NSC_GXT_ONE(X, T, NC, 0, 10, true) NSC_GXT_ONE(X, T, NC, 0, 12, true)            \
    NSC_GXT_ONE(X, T, NC, 0, 16, true) NSC_GXT_ONE(X, T, NC, -4, 4, false)           \
    NSC_GXT_ONE(X, T, NC, -8, 8, false) NSC_GXT_ONE(X, T, NC, -12, 12, false)
#define NSC_GXT_INSTANTIATE(T, NC) NSC_GXT_BUCKETS(, T, NC)
#define NSC_GXT_EXTERN(T, NC) NSC_GXT_BUCKETS(extern, T, NC)
