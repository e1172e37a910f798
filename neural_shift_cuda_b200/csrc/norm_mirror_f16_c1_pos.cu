// Instantiations of the tiled normalized_accumulate_uz forward for tables
// with mirror terms (mode 2: pos weights), __half, NC = 1.
#include "accumulate_fast_launch.cuh"
using nsc::fast::FastTable;
using nsc::fast::Geo;
using nsc::fast::WMaps;
NSC_FAST_INSTANTIATE_MODE(__half, 1, 2)
