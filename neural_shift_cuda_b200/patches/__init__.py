"""The installer modules under their `patches/` names (the reference keeps
identical copies of `integration/*.py` in a top-level `patches/` directory
that its tests import by path, `tests/test_attn_forward_equivalence.py:116`).
Here they are the same modules: `patches.nectr_patch is
integration.nectr_patch`."""

import sys as _sys

from ..integration import (gasd_drunet_attn_patch, nectr_patch,
                           nekde_drunet_attn_patch, nkd_metropolis_attn_patch)

for _m in (gasd_drunet_attn_patch, nectr_patch, nekde_drunet_attn_patch,
           nkd_metropolis_attn_patch):
    _sys.modules[__name__ + "." + _m.__name__.rsplit(".", 1)[1]] = _m

__all__ = ["gasd_drunet_attn_patch", "nectr_patch", "nekde_drunet_attn_patch",
           "nkd_metropolis_attn_patch"]
