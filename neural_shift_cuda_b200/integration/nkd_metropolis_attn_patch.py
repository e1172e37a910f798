"""Installer for the Metropolis NeKDe denoiser
(`NeKDeMetropolisDRUNetAttn`).

Surface of `neural_shift_cuda/integration/nkd_metropolis_attn_patch.py`
(reference).  The forward builds the head-mixed half-plane weights
`w_half (B, S, C, H, W)` with the model's own `_halfplane_weights`,
`_head_mix_matrix` and `_mix_heads`, then calls `metropolis_aggregate`,
which forms each mirror edge by a circular shift of the post-activation
forward weight inside the kernels -- W is exactly symmetric.  Unlike the
reference, training also runs the CUDA kernels (the op has a backward).

`forward_cached(x, cache)` (cache.shifts / w_hat_fwd_list / degree_hat /
comp_box / C) reuses the cached post-Metropolis edges with one
`accumulate_uz`: Wx = x - d_hat x + K_hat x.
"""

from __future__ import annotations

import inspect

import torch
import torch.nn.functional as F

from ..metropolis import metropolis_aggregate
from ..ops import accumulate_uz
from ._common import flat, periodic_edges, shift_tensor


def _build_w_half(self, x, guide, sig):
    """(B, S, C, H, W) head-mixed forward weights and the shift rows."""
    B, C, H, W = x.shape
    R = self.window_rad
    sig = self._normalise_sigma(x, sig)
    z = x if guide is None else guide
    if z.shape != x.shape:
        raise ValueError(f"guide must have the same shape as x; got "
                         f"{tuple(z.shape)} and {tuple(x.shape)}.")
    if z.device != x.device or z.dtype != x.dtype:
        raise ValueError("guide and x must share device and dtype.")
    phi = self.pre_activation(z, sigma=sig)
    padded = F.pad(phi, (R, R, R, R), mode="circular")
    shifts = self._collect_shifts()
    w_list = self._halfplane_weights(phi, padded, sig, shifts)
    mat = self._head_mix_matrix()
    w_half = torch.stack([self._mix_heads(w_list[i], C, mat)
                          for i in range(len(shifts))], 1)
    return w_half, shifts


def _forward_cuda(self, x, guide=None, sig=None, return_D=False):
    if x.dim() != 4:
        raise ValueError(f"x must have shape (B,C,H,W), got {tuple(x.shape)}.")
    w_half, shifts = _build_w_half(self, x, guide, sig)
    eps = max(float(self.metropolis_eps), torch.finfo(x.dtype).tiny)
    Wx, d_hat = metropolis_aggregate(w_half, x, shifts,
                                     use_box=bool(getattr(self, "comp_box", True)),
                                     eps=eps)
    return (Wx, d_hat) if return_D else (Wx, None)


def _pack(self, x, cache):
    if x.dim() != 4:
        raise ValueError(f"x must have shape (B,C,H,W), got {tuple(x.shape)}.")
    if x.size(1) != cache.C:
        raise ValueError(
            f"cached weights have C={cache.C} channels but x has {x.size(1)}; "
            f"rebuild the cache for this channel count.")
    key = (tuple(x.shape), x.device, x.dtype)
    st = getattr(self, "_metropolis_parallel_weight_cache", None)
    if st is not None and st[0] is cache and st[1] == key:
        return st[2], st[3]
    w = list(cache.w_hat_fwd_list)
    if len(w) != len(cache.shifts) or not w:
        raise ValueError("cached w_hat_fwd_list must contain one tensor per cached shift.")
    for t in w:
        if tuple(t.shape) != tuple(x.shape):
            raise ValueError("cached weights and x must have identical (B,C,H,W) shapes.")
        if t.device != x.device or t.dtype != x.dtype:
            raise ValueError("cached weights and x must share device and dtype.")
    stack = torch.stack(w, 0)
    rows = [(int(dx), int(dy), int(bool(inv))) for dx, dy, inv in cache.shifts]
    if bool(cache.comp_box):
        packed = (flat(stack), shift_tensor(rows, x.device))
    else:
        packed = periodic_edges(stack, rows)
    self._metropolis_parallel_weight_cache = (cache, key, *packed)
    return packed


def _forward_cached_cuda(self, x, cache, return_D=False):
    w_all, shifts = _pack(self, x, cache)
    k_hat_x, d_red = accumulate_uz(x.contiguous(), w_all, shifts)
    d_hat = cache.degree_hat if getattr(cache, "degree_hat", None) is not None else d_red
    Wx = x - d_hat * x + k_hat_x
    return (Wx, d_hat) if return_D else (Wx, None)


def _route(self, x) -> bool:
    if not hasattr(self, "use_cuda_shift"):
        self.use_cuda_shift = True
    return bool(self.use_cuda_shift) and x.is_cuda


def install_cuda_shift(model_cls):
    """Patch `forward` (and `forward_cached` when present); idempotent.
    `DSG_NLM` and every `laplacian_*` of the model call `forward`."""
    if getattr(model_cls, "_nsc_metropolis_installed", False):
        return model_cls
    if not hasattr(model_cls, "forward"):
        raise TypeError("model_cls must provide forward(x, guide=None, sig=None).")
    orig = model_cls.forward
    p = inspect.signature(orig).parameters
    has_rd = "return_D" in p
    rd = p["return_D"].default if has_rd else False

    def forward(self, x, guide=None, sig=None, return_D=rd):
        if _route(self, x):
            return _forward_cuda(self, x, guide=guide, sig=sig, return_D=return_D)
        if has_rd:
            return orig(self, x, guide=guide, sig=sig, return_D=return_D)
        return orig(self, x, guide=guide, sig=sig)

    model_cls.forward = forward

    orig_cached = getattr(model_cls, "forward_cached", None)
    if orig_cached is not None:
        pc = inspect.signature(orig_cached).parameters
        c_has = "return_D" in pc
        c_rd = pc["return_D"].default if c_has else False

        def forward_cached(self, x, cache, return_D=c_rd):
            if _route(self, x):
                return _forward_cached_cuda(self, x, cache, return_D=return_D)
            if c_has:
                return orig_cached(self, x, cache, return_D=return_D)
            return orig_cached(self, x, cache)

        model_cls.forward_cached = forward_cached
    model_cls._nsc_metropolis_installed = True
    return model_cls
