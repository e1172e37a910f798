// Instantiations of the tiled normalized forward for __half.
#include "normalized_fast_launch.cuh"
namespace nsc {
namespace nfast {
NSC_NORM_INSTANTIATE(__half)
}  // namespace nfast
}  // namespace nsc
