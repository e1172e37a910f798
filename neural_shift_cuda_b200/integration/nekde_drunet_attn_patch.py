"""Installer for the NeKDe DRUNet attention denoiser (`NeKDeDRUNetAttn`,
versions 2-4).

Surface of `neural_shift_cuda/integration/nekde_drunet_attn_patch.py`
(reference).  NeKDe is the symmetric denoiser over the half-plane table:
each row (dx, dy, has_inv) has one network weight and, for has_inv rows, a
mirror edge that reuses it.

* comp_box on: the forward weights are box-masked and the table keeps its
  has_inv flags -- the kernels form the (non-periodic, masked) mirror term
  themselves.
* comp_box off (periodic): the mirror weight is the forward weight rolled
  by (dx, dy) -- the reference materialises those rolled planes as explicit
  (-dx, -dy, 0) rows; here the same table runs with periodic_mirror=True and
  the kernels read the mirror weight at (p - d) mod (H, W) directly.

Patched: `forward`, `forward_cached` (cache.shifts / w_fwd_list / comp_box
/ D / C) and `_KT_action(y, guide, sig, return_D, apply_Dinv)`.
"""

from __future__ import annotations

import inspect

import torch
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint as grad_checkpoint

from ..ops import accumulate_uz, normalized_accumulate_uz, shift_gather
from ._common import (box_stack, cached_shift_tensor, flat, head_mix_matrix,
                      mix_heads, normalise_sigma, shift_tensor)


def _rows(model):
    return [(int(dx), int(dy), int(bool(inv))) for dx, dy, inv in model._collect_shifts()]


def _get_shift_tensor(self, device):
    return cached_shift_tensor(self, "_nsc_nekde_shifts", lambda: _rows(self), device)


def _weight_stack(model, x, guide, sig):
    """(S, B, Cw, H, W) per-row forward weights (before the comp_box mask)."""
    B, C, H, W = x.shape
    R = model.window_rad
    phi = model.pre_activation(x if guide is None else guide, sigma=sig).contiguous()
    mat = head_mix_matrix(model)
    if hasattr(model, "_gather_core"):
        padded = F.pad(phi, (R, R, R, R), mode="circular")
        w = torch.stack(list(model._halfplane_weights(
            phi, padded, sig, model._collect_shifts())), 0)
        return mix_heads(w, C, mat)
    shifts = _get_shift_tensor(model, x.device)
    S = shifts.shape[0]
    chunk = model.max_batch_shifts or S
    tiles = []
    for s0 in range(0, S, chunk):
        sub = shifts[s0:s0 + chunk, :2]
        n = sub.shape[0]
        phi_s, _ = shift_gather(phi, sub)
        phi_c = phi.repeat(n, 1, 1, 1)
        sig_b = sig.repeat(n, 1, 1, 1) if sig is not None else None
        fn = (model.attn_head.logit if model.output_activation == "softmax"
              else model.attn_head.weight)
        if getattr(model, "use_grad_checkpoint", False):
            t = grad_checkpoint(fn, phi_c, phi_s, sig_b, use_reentrant=False)
        else:
            t = fn(phi_c, phi_s, sig_b)
        tiles.append(t.reshape(n, B, *t.shape[1:]))
    w = torch.cat(tiles, 0)
    if model.output_activation == "softmax":
        w = F.softmax(w - w.amax(0, keepdim=True), dim=0)
    return mix_heads(w, C, mat)


def _reduction_inputs(model, w, device, H, W, comp_box):
    """(weights, shifts, periodic_mirror) for the reduction in either
    boundary mode."""
    shifts = _get_shift_tensor(model, device)
    if comp_box:
        return flat(w * box_stack(shifts[:, :2], H, W, w.dtype, device)), shifts, False
    return flat(w), shifts, True


def _forward_cuda(self, x, guide=None, sig=None, return_D=True):
    if not self.training:
        self.max_batch_shifts = 10
    sig = normalise_sigma(x, sig)
    B, C, H, W = x.shape
    w = _weight_stack(self, x, guide, sig)
    w_all, shifts, per = _reduction_inputs(self, w, x.device, H, W,
                                           bool(getattr(self, "comp_box", True)))
    D, log_Z = normalized_accumulate_uz(x.contiguous(), w_all, shifts,
                                        return_log_degree=True, validate=False,
                                        periodic_mirror=per)
    if not self.training:
        self.max_batch_shifts = None
    return (D, log_Z.exp()) if return_D else (D, None)


def _kt_action_cuda(self, y, guide=None, sig=None, return_D=False,
                    apply_Dinv=False):
    """K^T y (or K^T D^-1 y).  The operator is symmetric by construction,
    so K^T is the same reduction as K."""
    if not self.training:
        self.max_batch_shifts = 10
    sig = normalise_sigma(y, sig)
    B, C, H, W = y.shape
    w = _weight_stack(self, y, guide, sig)
    w_all, shifts, per = _reduction_inputs(self, w, y.device, H, W,
                                           bool(getattr(self, "comp_box", True)))
    U, Z = accumulate_uz(y.contiguous(), w_all, shifts, periodic_mirror=per)
    if apply_Dinv:
        U, _ = accumulate_uz((y / Z.clamp_min(1e-6)).contiguous(), w_all, shifts,
                             periodic_mirror=per)
    if not self.training:
        self.max_batch_shifts = None
    return (U, Z) if return_D else (U, None)


def _pack(self, x, cache):
    if x.dim() != 4:
        raise ValueError(f"x must have shape (B,C,H,W), got {tuple(x.shape)}.")
    if x.size(1) != cache.C:
        raise ValueError(
            f"cached weights have C={cache.C} channels but x has {x.size(1)}; "
            f"rebuild the cache for this channel count.")
    key = (tuple(x.shape), x.device, x.dtype)
    st = getattr(self, "_nekde_parallel_weight_cache", None)
    if st is not None and st[0] is cache and st[1] == key:
        return st[2], st[3], st[4]
    w = list(cache.w_fwd_list)
    if len(w) != len(cache.shifts) or not w:
        raise ValueError("cached w_fwd_list must contain one tensor per cached shift.")
    for t in w:
        if tuple(t.shape) != tuple(x.shape):
            raise ValueError("cached weights and x must have identical (B,C,H,W) shapes.")
        if t.device != x.device or t.dtype != x.dtype:
            raise ValueError("cached weights and x must share device and dtype.")
    stack = torch.stack(w, 0)
    rows = [(int(dx), int(dy), int(bool(inv))) for dx, dy, inv in cache.shifts]
    packed = (flat(stack), shift_tensor(rows, x.device), not bool(cache.comp_box))
    self._nekde_parallel_weight_cache = (cache, key, *packed)
    return packed


def _forward_cached_cuda(self, x, cache, return_D=True):
    w_all, shifts, per = _pack(self, x, cache)
    D, log_Z = normalized_accumulate_uz(x.contiguous(), w_all, shifts,
                                        return_log_degree=True, validate=False,
                                        periodic_mirror=per)
    degree = cache.D if getattr(cache, "D", None) is not None else log_Z.exp()
    return (D, degree) if return_D else (D, None)


def _route(self, x) -> bool:
    if not hasattr(self, "use_cuda_shift"):
        self.use_cuda_shift = True
    return bool(self.use_cuda_shift) and x.is_cuda


def install_cuda_shift(model_cls):
    """Patch a NeKDeDRUNetAttn class (v2, v3, v4); idempotent."""
    if getattr(model_cls, "_nsc_nekde_installed", False):
        return model_cls
    model_cls._get_shift_tensor = _get_shift_tensor
    orig = model_cls.forward
    p = inspect.signature(orig).parameters
    has_rd = "return_D" in p
    rd = p["return_D"].default if has_rd else True

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
        c_rd = pc["return_D"].default if c_has else True

        def forward_cached(self, x, cache, return_D=c_rd):
            if _route(self, x):
                return _forward_cached_cuda(self, x, cache, return_D=return_D)
            if c_has:
                return orig_cached(self, x, cache, return_D=return_D)
            return orig_cached(self, x, cache)

        model_cls.forward_cached = forward_cached

    orig_kt = getattr(model_cls, "_KT_action", None)

    def kt_action(self, y, guide=None, sig=None, return_D=False, apply_Dinv=False):
        if _route(self, y):
            return _kt_action_cuda(self, y, guide=guide, sig=sig,
                                   return_D=return_D, apply_Dinv=apply_Dinv)
        if orig_kt is None:
            raise AttributeError(
                f"{type(self).__name__} has no reference _KT_action; add the "
                f"arch-level _KT_action/NLM_transpose before installing.")
        return orig_kt(self, y, guide=guide, sig=sig, return_D=return_D,
                       apply_Dinv=apply_Dinv)

    model_cls._KT_action = kt_action
    model_cls._nsc_nekde_installed = True
    return model_cls
