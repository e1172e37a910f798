// accumulate_fast_launch.cuh -- host launcher of the tiled forward; included
// by the per-dtype instantiation files so the kernels compile in parallel.
#pragma once

#include <cstdio>

#include "accumulate_fast.cuh"

namespace nsc {
int fast_sm_count();
// A zeroed tile-ticket counter for one launch on `stream` (nullptr on error).
unsigned long long* tile_ticket(cudaStream_t stream);
void fast_set_decline(const char* why);

namespace fast {

template <typename T, int NC, int DYMIN, int DYMAX, bool EXACT, int MODE>
bool launch(const WMaps& maps, const void* x, void* U, void* Z,
            const FastTable& tab, Geo g, GeoExt gx, unsigned int* timeouts,
            int* invalid, cudaStream_t stream) {
    unsigned long long* ticket = tile_ticket(stream);
    if (!ticket) {
        fast_set_decline("tile counter");
        return false;
    }
    // ring depth: as many weight stages (<= 12) as fit next to the two
    // x tiles in the 227 KB a CTA may use
    const size_t fixed = NC * g.XH * g.XW * sizeof(T) +
                         16 + 4 * 16 + 16 + 128;
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
    auto k = acc_fast_kernel<T, NC, DYMIN, DYMAX, EXACT, MODE>;
    cudaFuncAttributes attr;
    if (cudaFuncGetAttributes(&attr, k) != cudaSuccess ||
        attr.maxThreadsPerBlock < NTHREADS) {
        cudaGetLastError();
        static thread_local char why[160];
        snprintf(why, sizeof(why),
                 "CTA of %d threads exceeds the kernel's limit of %d (%d registers)",
                 NTHREADS, attr.maxThreadsPerBlock, attr.numRegs);
        fast_set_decline(why);
        return false;
    }
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess) {
        cudaGetLastError();
        fast_set_decline("dynamic shared memory attribute");
        return false;
    }
    const int64_t nsm = fast_sm_count();
    int64_t grid_cap = nsm;
    if (gx.max_ctas > 0 && gx.max_ctas < grid_cap) grid_cap = gx.max_ctas;
    const unsigned grid = static_cast<unsigned>(g.ntiles < grid_cap ? g.ntiles : grid_cap);
    k<<<grid, NTHREADS, smem, stream>>>(maps, static_cast<const T*>(x),
                                        static_cast<float*>(U),
                                        static_cast<float*>(Z), tab, g, timeouts, ticket,
                                        invalid, gx);
    return true;
}

}  // namespace fast
}  // namespace nsc

#define NSC_FAST_ONE(T, NC, A, B, E, M)                                            \
    template bool nsc::fast::launch<T, NC, A, B, E, M>(const WMaps&,                 \
        const void*, void*, void*, const FastTable&, Geo, GeoExt,                           \
        unsigned int*, int*, cudaStream_t);
// Every table bucket of one storage type, image-channel count and mode
// (0: accumulate_uz, 1: normalized log weights, 2: normalized positive).
#define NSC_FAST_INSTANTIATE_MODE(T, NC, M)                                          \
    NSC_FAST_ONE(T, NC, 0, 2, true, M) NSC_FAST_ONE(T, NC, 0, 4, true, M)            \
    NSC_FAST_ONE(T, NC, 0, 6, true, M) NSC_FAST_ONE(T, NC, 0, 8, true, M)            \
    NSC_FAST_ONE(T, NC, 0, 10, true, M) NSC_FAST_ONE(T, NC, 0, 12, true, M)          \
    NSC_FAST_ONE(T, NC, 0, 16, true, M) NSC_FAST_ONE(T, NC, -4, 4, false, M)         \
    NSC_FAST_ONE(T, NC, -8, 8, false, M) NSC_FAST_ONE(T, NC, -12, 12, false, M)
#define NSC_FAST_INSTANTIATE(T, NC) NSC_FAST_INSTANTIATE_MODE(T, NC, 0)
