// Instantiations of the tiled normalized_accumulate_uz forward for tables
// with mirror terms (mode 1: log weights), float, NC = 1.
#include "accumulate_fast_launch.cuh"
using nsc::fast::FastTable;
using nsc::fast::Geo;
using nsc::fast::WMaps;
NSC_FAST_INSTANTIATE_MODE(float, 1, 1)
