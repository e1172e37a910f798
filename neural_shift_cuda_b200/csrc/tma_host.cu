// tma_host.cu -- host helpers for the TMA kernels: tensor-map encoding
// through the driver entry point (no link-time dependency on libcuda) and
// the per-device wait-timeout counter.
#include <cudaTypedefs.h>
#include <atomic>
#include <mutex>

#include "nsc_host.h"
#include "nsc_tma.cuh"

namespace nsc {
namespace {

static __device__ unsigned int g_wait_timeouts;

std::mutex g_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
constexpr int kMaxDev = 64;
unsigned int* g_counter[kMaxDev] = {};

}  // namespace

unsigned int* wait_timeout_counter() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_counter[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_wait_timeouts) != cudaSuccess) return nullptr;
        g_counter[dev] = static_cast<unsigned int*>(p);
    }
    return g_counter[dev];
}

namespace {
bool get_encoder(const char** err) {
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_encode) return true;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault,
                                &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
        *err = "cuTensorMapEncodeTiled is unavailable";
        return false;
    }
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return true;
}
}  // namespace

bool encode_map_4d(CUtensorMap* map, const void* base, int elem_bytes,
                   CUtensorMapDataType dtype, uint64_t W, uint64_t H, uint64_t P,
                   uint64_t Q, uint32_t bw, uint32_t bh, uint32_t bq,
                   const char** err) {
    if (!get_encoder(err)) return false;
    cuuint64_t dims[4] = {W, H, P, Q};
    cuuint64_t strides[3] = {W * elem_bytes, W * H * elem_bytes,
                             W * H * P * elem_bytes};
    cuuint32_t box[4] = {bw, bh, 1, bq};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = g_encode(map, dtype, 4, const_cast<void*>(base), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        *err = "cuTensorMapEncodeTiled rejected the weight layout";
        return false;
    }
    return true;
}

bool encode_map_3d(CUtensorMap* map, const void* base, int elem_bytes,
                   CUtensorMapDataType dtype, uint64_t W, uint64_t H,
                   uint64_t planes, uint32_t bw, uint32_t bh, const char** err) {
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (!g_encode) {
            void* fn = nullptr;
            cudaDriverEntryPointQueryResult q;
            if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn,
                                        cudaEnableDefault, &q) != cudaSuccess ||
                q != cudaDriverEntryPointSuccess || !fn) {
                *err = "cuTensorMapEncodeTiled is unavailable";
                return false;
            }
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        }
    }
    cuuint64_t dims[3] = {W, H, planes};
    cuuint64_t strides[2] = {W * elem_bytes, W * H * elem_bytes};
    cuuint32_t box[3] = {bw, bh, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(map, dtype, 3, const_cast<void*>(base), dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        *err = "cuTensorMapEncodeTiled rejected the weight layout";
        return false;
    }
    return true;
}

}  // namespace nsc

namespace nsc {
namespace {
unsigned int g_seen[kMaxDev] = {};
std::atomic<int> g_test_skip{-1};
std::atomic<unsigned> g_test_budget{0};
}  // namespace

void wait_fault_settings(int* skip_copy, unsigned* budget) {
    *skip_copy = g_test_skip.load();
    const unsigned b = g_test_budget.load();
    *budget = b ? b : kSleepWaits;
}
}  // namespace nsc

extern "C" NSC_API nsc_status nsc_check_waits(void* stream) {
    using namespace nsc;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev)
        return fail(NSC_ERR_LAUNCH_FAILED, "check_waits: no current device");
    cudaError_t e = cudaStreamSynchronize(as_stream(stream));
    if (e != cudaSuccess)
        return fail(NSC_ERR_LAUNCH_FAILED, "check_waits: %s", cudaGetErrorString(e));
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_wait_timeouts, sizeof(v)) != cudaSuccess)
        return fail(NSC_ERR_LAUNCH_FAILED, "check_waits: cannot read the wait counter");
    std::lock_guard<std::mutex> lock(g_mu);
    const unsigned int before = g_seen[dev];
    g_seen[dev] = v;
    if (v != before)
        return fail(NSC_ERR_TIMEOUT,
                    "%u bounded device wait(s) gave up since the last check: a "
                    "tiled kernel returned early and its outputs are undefined",
                    v - before);
    return ok();
}

extern "C" NSC_API void nsc_test_wait_fault(int skip_copy, unsigned int wait_budget) {
    nsc::g_test_skip.store(skip_copy);
    nsc::g_test_budget.store(wait_budget);
}

extern "C" NSC_API unsigned int nsc_wait_timeouts(void) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, nsc::g_wait_timeouts, sizeof(v)) != cudaSuccess)
        return 0xFFFFFFFFu;
    return v;
}
