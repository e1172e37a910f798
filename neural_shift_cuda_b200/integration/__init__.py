"""Model installers: route a model's forward through the shift-window ops.

Same installer names as `neural_shift_cuda.integration` (reference
`integration/__init__.py:67-98`) for the hot-path models:

    install_cuda_shift_nectr       NECTR_denoiser (official) / legacy nekre
    install_cuda_shift_attn        NeKDeDRUNetAttn (v2 - v4)
    install_cuda_shift_gasd        GASDDRUNetAttn
    install_cuda_shift_metropolis  NeKDeMetropolisDRUNetAttn

Each patches the class in place (idempotent); `instance.use_cuda_shift =
False` or a CPU input selects the model's original forward.
"""

from .gasd_drunet_attn_patch import install_cuda_shift as install_cuda_shift_gasd
from .nectr_patch import install_cuda_shift as install_cuda_shift_nectr
from .nekde_drunet_attn_patch import install_cuda_shift as install_cuda_shift_attn
from .nkd_metropolis_attn_patch import install_cuda_shift as install_cuda_shift_metropolis

__all__ = [
    "install_cuda_shift_attn",
    "install_cuda_shift_gasd",
    "install_cuda_shift_nectr",
    "install_cuda_shift_metropolis",
]
