// Instantiations of the tiled accumulate_uz forward for __half, NC = 1.
#include "accumulate_fast_launch.cuh"
using nsc::fast::FastTable;
using nsc::fast::Geo;
using nsc::fast::WMaps;
NSC_FAST_INSTANTIATE(__half, 1)
