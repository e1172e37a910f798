"""Stub models for the attention installers (GASD / NeKDe / NKD_mp).

The real model files are not part of the reference checkout, so these small
modules implement exactly the attributes the installers call
(`pre_activation`, `_collect_shifts`, `_all_shift_weights` /
`_halfplane_weights`, `_head_mix_matrix`, `_mix_heads`, `_normalise_sigma`,
`raw_head_mix`, `comp_box`, `max_batch_shifts`, `_gather_core`,
`metropolis_eps`).  The same classes feed the reference's own installer
functions when `tests/golden/make_golden.py` records fixtures, and this
package's installers in the GPU tests.
"""

import torch
import torch.nn as nn
import torch.nn.functional as F


def roll_gather(x, dx, dy):
    """gather convention: out(h, w) = x(h+dx, w+dy) circularly"""
    return torch.roll(x, shifts=(-dx, -dy), dims=(-2, -1))


class StubBase(nn.Module):
    """The model contract the attention installers use."""

    def __init__(self, C, R, heads, comp_box, table):
        super().__init__()
        self.window_rad = R
        self.comp_box = comp_box
        self.max_batch_shifts = None
        self.output_activation = "softmax"
        self.metropolis_eps = 1e-6
        self.raw_head_mix = (nn.Parameter(torch.randn(C, heads))
                             if heads not in (1, C) else None)
        self.feat = nn.Conv2d(C, 4, 3, padding=1)
        self.score = nn.Conv2d(8, heads, 1)
        self._table = [tuple(r) for r in table]
        self._gather_core = True

    def pre_activation(self, x, sigma=None):
        return torch.tanh(self.feat(x))

    def _collect_shifts(self):
        return list(self._table)

    def _weights(self, phi, shifts):
        logits = torch.stack([self.score(torch.cat([phi, roll_gather(phi, s[0], s[1])], 1))
                              for s in shifts], 0)
        return list(F.softmax(logits, dim=0))          # (B, heads, H, W) each

    def _all_shift_weights(self, phi, padded_phi, sig, shifts):
        return self._weights(phi, shifts)

    def _halfplane_weights(self, phi, padded_phi, sig, shifts):
        return self._weights(phi, shifts)

    def _head_mix_matrix(self):
        return (F.softmax(self.raw_head_mix, dim=1)
                if self.raw_head_mix is not None else None)

    def _mix_heads(self, w, C, mat):
        if w.shape[1] == 1:
            return w.expand(-1, C, -1, -1)
        if mat is not None:
            return torch.einsum("ch,bhij->bcij", mat, w)
        return w

    def _normalise_sigma(self, x, sig):
        return sig


def _fwd_return_d(self, x, guide=None, sig=None, return_D=True):
    raise NotImplementedError("stub: the installed forward replaces this")


def _fwd_no_d(self, x, guide=None, sig=None, return_D=False):
    raise NotImplementedError("stub: the installed forward replaces this")


def full_window(R):
    return [(dx, dy) for dx in range(-R, R + 1) for dy in range(-R, R + 1)]


def halfplane(R):
    rows = [(dx, dy, True) for dx in range(-R, R + 1) for dy in range(1, R + 1)]
    rows += [(dx, 0, dx != 0) for dx in range(0, R + 1)]
    return rows


def make_class(kind, name=None):
    """A fresh subclass per installer (installers patch the class)."""
    fwd = _fwd_no_d if kind == "nkd" else _fwd_return_d
    return type(name or f"{kind.upper()}Stub", (StubBase,), {"forward": fwd})


def make_model(kind, C, R, heads, comp_box, seed, cls=None):
    """Seeded stub in fp64, eval mode (the installers' inference branch)."""
    table = full_window(R) if kind == "gasd" else halfplane(R)
    torch.manual_seed(seed)
    cls = cls or make_class(kind)
    return cls(C, R, heads, comp_box, table).double().eval()


# Cases recorded against the reference installers: (kind, B, C, H, W, R,
# heads, comp_box, seed).
INSTALLER_CASES = [
    ("gasd", 2, 3, 12, 16, 2, 1, True, 11),
    ("gasd", 2, 3, 12, 16, 2, 3, False, 12),
    ("gasd", 1, 3, 10, 9, 3, 2, True, 13),
    ("nekde", 2, 3, 11, 13, 2, 1, True, 21),
    ("nekde", 2, 3, 11, 13, 2, 3, False, 22),
    ("nekde", 1, 3, 9, 12, 3, 2, True, 23),
    ("nekde", 1, 3, 9, 12, 3, 1, False, 24),
    ("nkd", 2, 3, 10, 12, 2, 1, True, 31),
    ("nkd", 2, 3, 10, 12, 2, 1, False, 32),
    ("nkd", 1, 3, 9, 11, 3, 3, True, 33),
]


def case_name(case):
    kind, B, C, H, W, R, heads, box, seed = case
    return f"{kind}_R{R}_h{heads}_{'box' if box else 'per'}_{seed}"
