// Instantiations of the tiled normalized forward for __nv_bfloat16.
#include "normalized_fast_launch.cuh"
namespace nsc {
namespace nfast {
NSC_NORM_INSTANTIATE(__nv_bfloat16)
}  // namespace nfast
}  // namespace nsc
