// accumulate_fast.cu -- dispatch of the tiled TMA forward (accumulate_fast.cuh).
//
// The tiled path takes a call when: x and weights share one storage dtype
// (fp16, bf16 or fp32); the weight is per-channel (one image channel per
// tile) or channel-broadcast with C in {1, 3}; rows are 16-byte aligned
// (W * sizeof(T) % 16 == 0, 16-byte aligned pointers); every |dx|, |dy| <=
// 16 and no (dx, dy) appears twice.  Other calls use the generic kernels.
// The dy range of the table selects a compile-time bucket: [0, K] for
// half-plane tables (every dy >= 0, K even up to 12, or 16), [-K, K]
// otherwise (K in {4, 8, 12}).
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "accumulate.h"
#include "accumulate_fast.cuh"
#include "accumulate_gx_tma.cuh"

// compiled in accumulate_gx_tma_{f16,bf16,f32}.cu
NSC_GXT_EXTERN(__half, 1) NSC_GXT_EXTERN(__half, 3)
NSC_GXT_EXTERN(__nv_bfloat16, 1) NSC_GXT_EXTERN(__nv_bfloat16, 3)
NSC_GXT_EXTERN(float, 1) NSC_GXT_EXTERN(float, 3)
#include "nsc_host.h"

namespace nsc {
namespace fast {

template <typename T, int NC, int DYMIN, int DYMAX, bool EXACT, int MODE>
bool launch(const WMaps& maps, const void* x, void* U, void* Z,
            const FastTable& tab, Geo g, GeoExt gx, unsigned int* timeouts,
            int* invalid, cudaStream_t stream);

}  // namespace fast

namespace {

thread_local const char* g_decline = "";
#define DECLINE(msg) do { g_decline = msg; return false; } while (0)

int sm_count() {
    static std::mutex mu;
    static int cache[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (!cache[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

template <typename T, int NC, int M>
bool by_bucket_m(bool exact, int K, const fast::WMaps& maps,
                 const void* x, void* U, void* Z, const fast::FastTable& tab,
                 const fast::Geo& g, const fast::GeoExt& gx, unsigned int* to, int* inv, cudaStream_t st) {
#define NSC_B(A, B, E) \
    return fast::launch<T, NC, A, B, E, M>(maps, x, U, Z, tab, g, gx, to, inv, st)
    if (exact) {
        switch (K) {
            case 2: NSC_B(0, 2, true);
            case 4: NSC_B(0, 4, true);
            case 6: NSC_B(0, 6, true);
            case 8: NSC_B(0, 8, true);
            case 10: NSC_B(0, 10, true);
            case 12: NSC_B(0, 12, true);
            default: NSC_B(0, 16, true);
        }
    }
    switch (K) {
        case 4: NSC_B(-4, 4, false);
        case 8: NSC_B(-8, 8, false);
        default: NSC_B(-12, 12, false);
    }
#undef NSC_B
}

template <typename T, int NC>
bool by_bucket(int mode, bool exact, int K, const fast::WMaps& maps,
               const void* x, void* U, void* Z, const fast::FastTable& tab,
               const fast::Geo& g, const fast::GeoExt& gx, unsigned int* to, int* inv, cudaStream_t st) {
    if (mode == 1) return by_bucket_m<T, NC, 1>(exact, K, maps, x, U, Z, tab, g, gx, to, inv, st);
    if (mode == 2) return by_bucket_m<T, NC, 2>(exact, K, maps, x, U, Z, tab, g, gx, to, inv, st);
    return by_bucket_m<T, NC, 0>(exact, K, maps, x, U, Z, tab, g, gx, to, inv, st);
}

// Shift table of the tiled kernels (forward and grad_x): entries by (dx,
// dy), their mirror flags, and the grouping of consecutive weight planes
// with one box origin into copies of up to kGroup planes (fewer when
// `smem_need(K, rx, planes per copy)` -- the kernel's shared memory with
// three stages -- exceeds 227 KB).  *exactp: the canonical half-plane
// pattern; *Kp: the dy bucket.  Returns a decline reason, or nullptr.
template <typename NeedF>
const char* build_fast_table(const ShiftTable& st, int V, NeedF&& smem_need,
                             fast::FastTable* tabp, bool* exactp, int* Kp, int* gmaxp) {
    using namespace fast;
    FastTable& tab = *tabp;
    std::memset(&tab, 0, sizeof(tab));
    for (auto& row : tab.s)
        for (auto& v : row) v = -1;
    int dymin = 0, dymax = 0, rx = 0;
    for (int s = 0; s < st.S; ++s) {
        const int dx = st.dx[s], dy = st.dy[s];
        if (dx < -MAXR || dx > MAXR || dy < -MAXR || dy > MAXR) return "radius";
        int16_t& e = tab.s[dx + MAXR][dy + MAXR];
        if (e >= 0) return "duplicate shift";
        e = static_cast<int16_t>(s | (st.has_inv(s) ? kInvBit : 0));
        tab.row_any[dx + MAXR] = 1;
        if (st.has_inv(s)) tab.row_inv[dx + MAXR] = 1;
        dymin = dy < dymin ? dy : dymin;
        dymax = dy > dymax ? dy : dymax;
        rx = (dx < 0 ? -dx : dx) > rx ? (dx < 0 ? -dx : dx) : rx;
    }
    tab.Rx = rx;
    // Copy size: up to kGroup planes, fewer when three such stages would not
    // fit next to the x tiles (the launcher needs at least three stages);
    // tables grouped below kGroup take the mask-driven (non-EXACT) kernel.
    int group_cap = kGroup;
    {
        const int span = dymax > -dymin ? dymax : -dymin;
        const int Kmax = span <= 4 ? 4 : span <= 8 ? 8 : span <= 12 ? 12 : 16;
        while (group_cap > 1 && smem_need(Kmax, rx, group_cap) > 227u * 1024u) --group_cap;
    }
    // Group consecutive entries of the visiting order ((dx, dy) ascending)
    // that are consecutive weight planes (s, s+1, ...) with the same box
    // origin, up to kGroup planes: one TMA copy then carries the group.
    int gmax = 1;
    int8_t pos[2 * MAXR + 1][2 * MAXR + 1];
    bool lastp[2 * MAXR + 1][2 * MAXR + 1];
    for (int dx = -rx; dx <= rx; ++dx) {
        int start_dy = 0, len = 0, prev_s = -2, prev_mo = -1;
        auto close = [&]() {
            if (len == 0) return;
            int16_t& e0 = tab.s[dx + MAXR][start_dy + MAXR];
            e0 = static_cast<int16_t>(e0 | (len << kLenShift));
            gmax = len > gmax ? len : gmax;
        };
        int prev_dy = 0;
        for (int dy = -MAXR; dy <= MAXR; ++dy) {
            const int16_t e = tab.s[dx + MAXR][dy + MAXR];
            if (e < 0) continue;
            const int mo = dy > 0 ? (dy + V - 1) / V * V : 0;
            const int sv = e & kSMask;
            if (len > 0 && len < group_cap && sv == prev_s + 1 && mo == prev_mo) {
                pos[dx + MAXR][dy + MAXR] = static_cast<int8_t>(len);
                lastp[dx + MAXR][prev_dy + MAXR] = false;
                ++len;
            } else {
                close();
                start_dy = dy;
                len = 1;
                pos[dx + MAXR][dy + MAXR] = 0;
            }
            lastp[dx + MAXR][dy + MAXR] = true;
            prev_s = sv;
            prev_mo = mo;
            prev_dy = dy;
        }
        close();
    }
    for (int dx = -MAXR; dx <= MAXR; ++dx)
        for (int dy = -MAXR; dy <= MAXR; ++dy) {
            const int e = tab.s[dx + MAXR][dy + MAXR];
            if (e < 0) continue;
            const uint64_t bit = 1ull << (dy + MAXR);
            tab.present[dx + MAXR] |= bit;
            if (e & kInvBit) tab.inv[dx + MAXR] |= bit;
            if (pos[dx + MAXR][dy + MAXR] & 1) tab.pos0[dx + MAXR] |= bit;
            if (pos[dx + MAXR][dy + MAXR] & 2) tab.pos1[dx + MAXR] |= bit;
            if (lastp[dx + MAXR][dy + MAXR]) tab.last[dx + MAXR] |= bit;
        }
    // Canonical half-plane table of radius R: compile-time entry pattern.
    bool exact = dymin >= 0 && dymax == rx && rx >= 1 && group_cap == kGroup;
    for (int dx = -rx; exact && dx <= rx; ++dx)
        for (int dy = 0; dy <= rx; ++dy) {
            const int e = tab.s[dx + MAXR][dy + MAXR];
            bool want = dy > 0 || dx >= 0;
            if ((e >= 0) != want) { exact = false; break; }
            if (e < 0) continue;
            const bool inv = e & kInvBit;
            const int p = pos[dx + MAXR][dy + MAXR];
            const bool l = lastp[dx + MAXR][dy + MAXR];
            const bool want_inv = dy > 0 || dx != 0;
            const int want_p = dy > 0 ? (dy - 1) % kGroup : 0;
            const bool want_l = dy == 0 || want_p == kGroup - 1 || dy == rx;
            if (inv != want_inv || p != want_p || l != want_l) {
                exact = false;
                break;
            }
        }
    tab.Rdy = dymax;
    int K;
    if (exact) {
        K = rx <= 12 ? (rx + 1) / 2 * 2 : 16;
        if (rx > 16) return "radius";
    } else {
        const int span = dymax > -dymin ? dymax : -dymin;
        K = span <= 4 ? 4 : span <= 8 ? 8 : span <= 12 ? 12 : 16;
        if (K > 12) return "dy range";
    }
    *exactp = exact;
    *Kp = K;
    *gmaxp = gmax;
    return nullptr;
}

}  // namespace

bool acc_fwd_fast(const void* x, int xd, const void* w, int wd, int64_t Cw,
                  int64_t B, int64_t C, int64_t Hout, int64_t W, int64_t x_rows,
                  int64_t x_off, int wrap, const ShiftTable& st, void* U, void* Z,
                  cudaStream_t stream, int mode, int* invalid, int64_t h_begin,
                  int64_t h_end, int max_ctas) {
    using namespace fast;
    g_decline = "";
    if (h_end < 0) h_end = Hout;
    if (h_begin < 0 || h_begin > h_end || h_end > Hout) DECLINE("row range");
    if (mode != 0 && !wrap) DECLINE("normalized modes take full images only");
    if (std::getenv("NSC_DISABLE_FAST")) DECLINE("disabled by NSC_DISABLE_FAST");
    if (st.any_tr) DECLINE("transposed rows");
    // periodic mirror rows: the tile kernel computes them as masked rows and
    // the caller adds the wrapped terms of the border band
    if (st.any_per && (!wrap || Hout <= 2 * st.R || W <= 2 * st.R))
        DECLINE("periodic mirror rows outside a full image larger than 2R");
    if (xd != wd || (xd != NSC_F16 && xd != NSC_BF16 && xd != NSC_F32)) DECLINE("dtype");
    const int es = xd == NSC_F32 ? 4 : 2;
    const int V = 16 / es;
    int NC;
    if (Cw == 1 && (C == 1 || C == 3)) NC = static_cast<int>(C);
    else if (Cw == C) NC = 1;
    else DECLINE("channels");
    if ((W * es) % 16 != 0) DECLINE("row alignment");
    for (const void* p : {x, w, static_cast<const void*>(U), static_cast<const void*>(Z)})
        if (reinterpret_cast<uintptr_t>(p) % 16 != 0) DECLINE("pointer alignment");

    FastTable tab;
    bool exact = false;
    int K = 0, gmax = 1;
    {
        const char* why = build_fast_table(st, V, [&](int Kb, int rxb, int group) {
            const int XCg = align_up(Kb, V);
            const size_t plane = static_cast<size_t>(TH + rxb) * (TPR * V + XCg) * es;
            const size_t xt = NC * (TH + 2 * rxb) *
                              (TPR * V + 2 * XCg) * es + 16 + 4 * 16 + 16 + 128;
            return xt + 3 * (((group * plane + 127) & ~size_t(127)) + 16);
        }, &tab, &exact, &K, &gmax);
        if (why) DECLINE(why);
    }
    const int rx = tab.Rx;
    if (!wrap && x_off < rx) DECLINE("band halo");

    Geo g{};
    GeoExt gx{};
    g.B = B; g.C = C; g.H = Hout; g.W = W; g.Cw = Cw;
    g.x_rows = x_rows; g.x_off = x_off; g.wrap = wrap;
    {
        int skip;
        unsigned budget;
        wait_fault_settings(&skip, &budget);
        gx.skip_copy = skip;
        gx.wait_budget = budget;
    }
    const int TW = TPR * V;
    g.tiles_x = static_cast<int32_t>((W + TW - 1) / TW);
    gx.hb0 = static_cast<int32_t>(h_begin);
    gx.hb1 = static_cast<int32_t>(h_end);
    gx.max_ctas = max_ctas;
    g.tiles_y = static_cast<int32_t>((h_end - h_begin + TH - 1) / TH);
    g.groups = B * (Cw == 1 ? 1 : C);
    g.ntiles = g.groups * g.tiles_y * g.tiles_x;
    const int XC = align_up(K, V);
    g.BH = TH + rx;
    g.BW = TW + XC;
    g.stage_tx = static_cast<uint32_t>(g.BH) * g.BW * es;
    g.stage_stride = (g.stage_tx + 127u) & ~127u;
    g.XH = TH + 2 * rx;
    g.XW = TW + 2 * XC;

    const CUtensorMapDataType dt = xd == NSC_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : xd == NSC_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    g.plane_bytes = g.stage_tx;
    g.stage_stride = (static_cast<uint32_t>(gmax) * g.stage_tx + 127u) & ~127u;
    WMaps maps;
    const char* err = nullptr;
    for (int d = 1; d <= 4; ++d)
        if (!encode_map_4d(&maps.m[d - 1], w, es, dt, W, Hout, B * Cw, st.S, g.BW, g.BH,
                           d <= st.S ? d : 1, &err))
            DECLINE("tensor map");
    unsigned int* to = wait_timeout_counter();
    if (!to) DECLINE("timeout counter");
    (void)sm_count;
    const int m = mode;
    if (xd == NSC_F16)
        return NC == 1 ? by_bucket<__half, 1>(m, exact, K, maps, x, U, Z, tab, g, gx, to, invalid, stream)
                       : by_bucket<__half, 3>(m, exact, K, maps, x, U, Z, tab, g, gx, to, invalid, stream);
    if (xd == NSC_BF16)
        return NC == 1 ? by_bucket<__nv_bfloat16, 1>(m, exact, K, maps, x, U, Z, tab, g, gx, to, invalid, stream)
                       : by_bucket<__nv_bfloat16, 3>(m, exact, K, maps, x, U, Z, tab, g, gx, to, invalid, stream);
    return NC == 1 ? by_bucket<float, 1>(m, exact, K, maps, x, U, Z, tab, g, gx, to, invalid, stream)
                   : by_bucket<float, 3>(m, exact, K, maps, x, U, Z, tab, g, gx, to, invalid, stream);
}

namespace {
template <typename T, int NC>
bool gx_bucket(bool exact, int K, const fast::WMaps& maps, const void* gU, void* gx,
               const fast::FastTable& tab, const fast::Geo& g, const fast::GeoExt& ge,
               unsigned int* to, cudaStream_t st) {
#define NSC_B(A, B, E) return gxt::launch<T, NC, A, B, E>(maps, gU, gx, tab, g, ge, to, st)
    if (exact) {
        switch (K) {
            case 2: NSC_B(0, 2, true);
            case 4: NSC_B(0, 4, true);
            case 6: NSC_B(0, 6, true);
            case 8: NSC_B(0, 8, true);
            case 10: NSC_B(0, 10, true);
            case 12: NSC_B(0, 12, true);
            default: NSC_B(0, 16, true);
        }
    }
    switch (K) {
        case 4: NSC_B(-4, 4, false);
        case 8: NSC_B(-8, 8, false);
        default: NSC_B(-12, 12, false);
    }
#undef NSC_B
}
}  // namespace

// Tiled TMA grad_x: the forward kernel's table and weight boxes (tile TH x
// 64 columns, V = 4 pixels per thread), grad_U tile fp32; then the wrapped
// term-A contributions of the border band.
bool acc_gx_tma(const void* w, int wd, int64_t Cw, int64_t B, int64_t C, int64_t H,
                int64_t W, const ShiftTable& st, const void* gU, void* gx,
                cudaStream_t stream) {
    using namespace fast;
    g_decline = "";
    if (std::getenv("NSC_DISABLE_FAST")) DECLINE("disabled by NSC_DISABLE_FAST");
    if (st.any_tr || st.any_per) DECLINE("transposed or periodic rows");
    if (wd != NSC_F16 && wd != NSC_BF16 && wd != NSC_F32) DECLINE("dtype");
    if (H <= 2 * st.R || W <= 2 * st.R) DECLINE("image not larger than 2R");
    const int es = wd == NSC_F32 ? 4 : 2;
    const int VA = 16 / es;
    constexpr int GV = gxt::V, GTW = gxt::TW;
    int NC;
    if (Cw == 1 && (C == 1 || C == 3)) NC = static_cast<int>(C);
    else if (Cw == C) NC = 1;
    else DECLINE("channels");
    if ((W * es) % 16 != 0) DECLINE("row alignment");
    for (const void* p : {w, gU, static_cast<const void*>(gx)})
        if (reinterpret_cast<uintptr_t>(p) % 16 != 0) DECLINE("pointer alignment");

    FastTable tab;
    bool exact = false;
    int K = 0, gmax = 1;
    {
        const char* why = build_fast_table(st, VA, [&](int Kb, int rxb, int group) {
            const size_t plane = static_cast<size_t>(TH + rxb) * (GTW + align_up(Kb, VA)) * es;
            const size_t xt = static_cast<size_t>(NC) * (TH + 2 * rxb) *
                              (GTW + 2 * align_up(Kb, GV)) * 4 + 16 + 16 + 128;
            return xt + 3 * (((group * plane + 127) & ~size_t(127)) + 16);
        }, &tab, &exact, &K, &gmax);
        if (why) DECLINE(why);
    }
    const int rx = tab.Rx;
    Geo g{};
    GeoExt ge{};
    g.B = B; g.C = C; g.H = H; g.W = W; g.Cw = Cw;
    g.x_rows = H; g.x_off = 0; g.wrap = 1;
    {
        int skip;
        unsigned budget;
        wait_fault_settings(&skip, &budget);
        ge.skip_copy = -1;
        ge.wait_budget = budget;
    }
    ge.hb0 = 0;
    ge.hb1 = static_cast<int32_t>(H);
    g.tiles_x = static_cast<int32_t>((W + GTW - 1) / GTW);
    g.tiles_y = static_cast<int32_t>((H + TH - 1) / TH);
    g.groups = B * (Cw == 1 ? 1 : C);
    g.ntiles = g.groups * g.tiles_y * g.tiles_x;
    g.BH = TH + rx;
    g.BW = GTW + align_up(K, VA);
    g.stage_tx = static_cast<uint32_t>(g.BH) * g.BW * es;
    g.plane_bytes = g.stage_tx;
    g.stage_stride = (static_cast<uint32_t>(gmax) * g.stage_tx + 127u) & ~127u;
    g.XH = TH + 2 * rx;
    g.XW = GTW + 2 * align_up(K, GV);

    const CUtensorMapDataType dt = wd == NSC_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : wd == NSC_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    WMaps maps;
    const char* err = nullptr;
    for (int d = 1; d <= 4; ++d)
        if (!encode_map_4d(&maps.m[d - 1], w, es, dt, W, H, B * Cw, st.S, g.BW, g.BH,
                           d <= st.S ? d : 1, &err))
            DECLINE("tensor map");
    unsigned int* to = wait_timeout_counter();
    if (!to) DECLINE("timeout counter");
    bool ok;
    if (wd == NSC_F16)
        ok = NC == 1 ? gx_bucket<__half, 1>(exact, K, maps, gU, gx, tab, g, ge, to, stream)
                     : gx_bucket<__half, 3>(exact, K, maps, gU, gx, tab, g, ge, to, stream);
    else if (wd == NSC_BF16)
        ok = NC == 1 ? gx_bucket<__nv_bfloat16, 1>(exact, K, maps, gU, gx, tab, g, ge, to, stream)
                     : gx_bucket<__nv_bfloat16, 3>(exact, K, maps, gU, gx, tab, g, ge, to, stream);
    else
        ok = NC == 1 ? gx_bucket<float, 1>(exact, K, maps, gU, gx, tab, g, ge, to, stream)
                     : gx_bucket<float, 3>(exact, K, maps, gU, gx, tab, g, ge, to, stream);
    if (!ok) return false;
    // the tile kernel ran: the wrap kernel must follow it
    return acc_gx_wrap(w, wd, Cw, B, C, H, W, st, gU, gx, stream) == NSC_OK;
}

int fast_sm_count() { return sm_count(); }

namespace {
// Tile-ticket counters of the tiled kernels: 64 slots per device, handed
// out round-robin and zeroed in-stream before each launch.  A slot is reused
// only 64 launches later, so launches on concurrent streams do not share a
// counter unless more than 64 of them are in flight at once.
constexpr int kTicketSlots = 64;
static __device__ unsigned long long g_tickets[kTicketSlots];
std::mutex g_ticket_mu;
unsigned long long* g_ticket_base[64] = {};
unsigned g_ticket_next[64] = {};
}  // namespace

unsigned long long* tile_ticket(cudaStream_t stream) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    unsigned long long* p;
    {
        std::lock_guard<std::mutex> lock(g_ticket_mu);
        if (!g_ticket_base[dev]) {
            void* a = nullptr;
            if (cudaGetSymbolAddress(&a, g_tickets) != cudaSuccess) {
                cudaGetLastError();
                return nullptr;
            }
            g_ticket_base[dev] = static_cast<unsigned long long*>(a);
        }
        p = g_ticket_base[dev] + (g_ticket_next[dev]++ % kTicketSlots);
    }
    if (cudaMemsetAsync(p, 0, sizeof(*p), stream) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    return p;
}

const char* fast_decline_reason() { return g_decline; }
void fast_set_decline(const char* why) { g_decline = why; }

}  // namespace nsc
