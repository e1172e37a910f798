"""neural_shift_cuda_b200 -- B200-native (sm_100a) shift-window ops.

A drop-in for the hot path of `neural_shift_cuda` v0.12.0: the same op
names and installers, backed by hand-written sm_100a kernels behind the C
ABI in `include/nsc_b200.h` (library `_lib/libnsc_b200.so`, built with
`python -m neural_shift_cuda_b200.build`).
"""

from .ops import (
    accumulate_uz,
    check_validation,
    index_width_bits,
    normalized_accumulate_uz,
    pair_gather,
    shift_gather,
)
from .metropolis import metropolis_aggregate

__version__ = "0.12.0+b200.1"

__all__ = [
    "shift_gather",
    "pair_gather",
    "accumulate_uz",
    "normalized_accumulate_uz",
    "metropolis_aggregate",
    "check_validation",
    "index_width_bits",
]
