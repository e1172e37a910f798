// Instantiations of the tiled normalized forward for float.
#include "normalized_fast_launch.cuh"
namespace nsc {
namespace nfast {
NSC_NORM_INSTANTIATE(float)
}  // namespace nfast
}  // namespace nsc
