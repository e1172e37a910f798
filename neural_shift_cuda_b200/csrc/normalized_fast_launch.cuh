// normalized_fast_launch.cuh -- launcher template of the tiled normalized
// forward; included only by the per-type instantiation files.
#pragma once

#include "normalized_fast.cuh"

namespace nsc {
namespace nfast {

template <typename T, int NC, int DYMIN, int DYMAX, bool LOGW>
bool launch(const void* x, const void* w, void* D, void* L, const NormTable& tab,
            const NormGeo& g, int* invalid, cudaStream_t stream) {
    const size_t smem = static_cast<size_t>(NST) * NT * KB +
                        static_cast<size_t>(NC) * g.XH * g.XW * sizeof(T);
    auto kern = norm_fast_kernel<T, NC, DYMIN, DYMAX, LOGW>;
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return false;
    const int64_t ntiles = static_cast<int64_t>(g.tiles_x) * g.tiles_y;
    const unsigned gx = static_cast<unsigned>(ntiles < (1LL << 31) - 1 ? ntiles : (1LL << 31) - 1);
    const unsigned gy = static_cast<unsigned>(g.groups < 65535 ? g.groups : 65535);
    kern<<<dim3(gx, gy), NT, smem, stream>>>(
        static_cast<const T*>(x), static_cast<const T*>(w), static_cast<float*>(D),
        static_cast<float*>(L), tab, g, invalid);
    return cudaPeekAtLastError() == cudaSuccess;
}

#define NSC_NORM_INSTANTIATE(T)                                                        \
    template bool launch<T, 1, -4, 4, true>(const void*, const void*, void*, void*,  \
        const NormTable&, const NormGeo&, int*, cudaStream_t);                        \
    template bool launch<T, 1, -4, 4, false>(const void*, const void*, void*, void*, \
        const NormTable&, const NormGeo&, int*, cudaStream_t);                        \
    template bool launch<T, 1, -8, 8, true>(const void*, const void*, void*, void*,  \
        const NormTable&, const NormGeo&, int*, cudaStream_t);                        \
    template bool launch<T, 1, -8, 8, false>(const void*, const void*, void*, void*, \
        const NormTable&, const NormGeo&, int*, cudaStream_t);                        \
    template bool launch<T, 3, -4, 4, true>(const void*, const void*, void*, void*,  \
        const NormTable&, const NormGeo&, int*, cudaStream_t);                        \
    template bool launch<T, 3, -4, 4, false>(const void*, const void*, void*, void*, \
        const NormTable&, const NormGeo&, int*, cudaStream_t);                        \
    template bool launch<T, 3, -8, 8, true>(const void*, const void*, void*, void*,  \
        const NormTable&, const NormGeo&, int*, cudaStream_t);                        \
    template bool launch<T, 3, -8, 8, false>(const void*, const void*, void*, void*, \
        const NormTable&, const NormGeo&, int*, cudaStream_t);

}  // namespace nfast
}  // namespace nsc
