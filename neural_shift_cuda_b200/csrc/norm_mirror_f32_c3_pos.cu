// Instantiations of the tiled normalized_accumulate_uz forward for tables
// with mirror terms (mode 2: pos weights), float, NC = 3.
#include "accumulate_fast_launch.cuh"
using nsc::fast::FastTable;
using nsc::fast::Geo;
using nsc::fast::WMaps;
NSC_FAST_INSTANTIATE_MODE(float, 3, 2)
