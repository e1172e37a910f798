// normalized_fast.cu -- dispatch of the tiled normalized forward
// (normalized_fast.cuh).
//
// The tiled path takes a call when: no table row has a mirror term; x and
// the keys share one storage dtype (fp16, bf16 or fp32); the keys are
// per-channel or channel-broadcast with C in {1, 3}; rows are 16-byte
// aligned; every |dx| <= 16, every |dy| <= 8 and no (dx, dy) repeats;
// H, W < 2^30.  Other calls use the general kernel (normalized.cu).
#include <cstdlib>
#include <cstring>

#include "normalized_fast.h"
#include "normalized_fast.cuh"

namespace nsc {
namespace nfast {

template <typename T, int NC, int DYMIN, int DYMAX, bool LOGW>
bool launch(const void* x, const void* w, void* D, void* L, const NormTable& tab,
            const NormGeo& g, int* invalid, cudaStream_t stream);



}  // namespace nfast

namespace {
thread_local const char* g_norm_decline = "";
#define NDECLINE(msg) do { g_norm_decline = msg; return false; } while (0)

template <typename T, int NC>
bool by_bucket(int K, bool logw, const void* x, const void* w, void* D, void* L,
               const nfast::NormTable& tab, const nfast::NormGeo& g, int* inv,
               cudaStream_t st) {
    if (K <= 4)
        return logw ? nfast::launch<T, NC, -4, 4, true>(x, w, D, L, tab, g, inv, st)
                    : nfast::launch<T, NC, -4, 4, false>(x, w, D, L, tab, g, inv, st);
    return logw ? nfast::launch<T, NC, -8, 8, true>(x, w, D, L, tab, g, inv, st)
                : nfast::launch<T, NC, -8, 8, false>(x, w, D, L, tab, g, inv, st);
}
}  // namespace

const char* norm_fast_decline_reason() { return g_norm_decline; }

bool norm_fwd_fast(const void* x, int xd, const void* w, int wd, int64_t Cw,
                   int64_t B, int64_t C, int64_t H, int64_t W, const ShiftTable& st,
                   int logw, void* D, void* L, int* invalid, cudaStream_t stream) {
    using namespace nfast;
    g_norm_decline = "";
    if (getenv("NSC_NORM_GENERIC")) NDECLINE("NSC_NORM_GENERIC set");
    if (xd != wd || xd == NSC_F64) NDECLINE("x and keys must share fp16/bf16/fp32 storage");
    for (int i = 0; i < kMaxShifts / 32; ++i)
        if (st.inv[i]) NDECLINE("table has mirror terms");
    const int NC = (Cw == 1) ? static_cast<int>(C) : 1;
    if (!(Cw == C || (Cw == 1 && (C == 1 || C == 3))))
        NDECLINE("keys must be per-channel or broadcast over C in {1, 3}");
    if (H >= (1LL << 30) || W >= (1LL << 30) || B * C >= (1LL << 30))
        NDECLINE("extent too large for the tiled path");
    const int es = xd == NSC_F32 ? 4 : 2;
    const int V = KB / es;
    const int VX = 16 / es;
    if ((W * es) % 16 || reinterpret_cast<uintptr_t>(x) % 16 ||
        reinterpret_cast<uintptr_t>(w) % 16 || reinterpret_cast<uintptr_t>(D) % 16 ||
        reinterpret_cast<uintptr_t>(L) % 16)
        NDECLINE("rows or pointers not 16-byte aligned");
    int Rx = 0, Ky = 0;
    static thread_local bool seen[2 * MAXR + 1][2 * MAXR + 1];
    std::memset(seen, 0, sizeof(seen));
    for (int s = 0; s < st.S; ++s) {
        const int dx = st.dx[s], dy = st.dy[s];
        if (dx < -MAXR || dx > MAXR || dy < -8 || dy > 8) NDECLINE("|dx| > 16 or |dy| > 8");
        if (seen[dx + MAXR][dy + MAXR]) NDECLINE("repeated (dx, dy)");
        seen[dx + MAXR][dy + MAXR] = true;
        Rx = dx < 0 ? (-dx > Rx ? -dx : Rx) : (dx > Rx ? dx : Rx);
        Ky = dy < 0 ? (-dy > Ky ? -dy : Ky) : (dy > Ky ? dy : Ky);
    }
    const int K = Ky <= 4 ? 4 : 8;
    // compute order: dx ascending, dy ascending
    NormTable tab;
    std::memset(&tab, 0, sizeof(tab));
    int idx[2 * MAXR + 1][2 * MAXR + 1];
    for (int a = 0; a < 2 * MAXR + 1; ++a)
        for (int c = 0; c < 2 * MAXR + 1; ++c) idx[a][c] = -1;
    for (int s = 0; s < st.S; ++s) idx[st.dx[s] + MAXR][st.dy[s] + MAXR] = s;
    int k = 0;
    for (int dx = -Rx; dx <= Rx; ++dx) {
        uint32_t m = 0;
        for (int dy = -K; dy <= K; ++dy) {
            const int s = idx[dx + MAXR][dy + MAXR];
            if (s < 0) continue;
            m |= 1u << (dy + K);
            tab.seq[k++] = static_cast<int16_t>(s);
        }
        if (!m) continue;
        tab.row_dx[tab.nrows] = dx;
        tab.row_mask[tab.nrows] = m;
        ++tab.nrows;
    }
    tab.nsteps = k;
    NormGeo g;
    g.B = static_cast<int>(B); g.C = static_cast<int>(C);
    g.H = static_cast<int>(H); g.W = static_cast<int>(W); g.Cw = static_cast<int>(Cw);
    const int TW = TPR * V;
    g.tiles_x = static_cast<int>((W + TW - 1) / TW);
    g.tiles_y = static_cast<int>((H + TH - 1) / TH);
    g.Rx = Rx;
    g.XH = TH + 2 * Rx;
    const int XC = (K + VX - 1) / VX * VX;
    g.XW = TW + 2 * XC;
    g.groups = B * ((Cw == 1) ? 1 : C);
    g.step_stride = B * Cw * H * W;
    bool okl;
    switch (xd) {
        case NSC_F16:
            okl = NC == 3 ? by_bucket<__half, 3>(K, logw, x, w, D, L, tab, g, invalid, stream)
                          : by_bucket<__half, 1>(K, logw, x, w, D, L, tab, g, invalid, stream);
            break;
        case NSC_BF16:
            okl = NC == 3 ? by_bucket<__nv_bfloat16, 3>(K, logw, x, w, D, L, tab, g, invalid, stream)
                          : by_bucket<__nv_bfloat16, 1>(K, logw, x, w, D, L, tab, g, invalid, stream);
            break;
        default:
            okl = NC == 3 ? by_bucket<float, 3>(K, logw, x, w, D, L, tab, g, invalid, stream)
                          : by_bucket<float, 1>(K, logw, x, w, D, L, tab, g, invalid, stream);
            break;
    }
    if (!okl) NDECLINE("launch configuration refused");
    return true;
}

}  // namespace nsc
