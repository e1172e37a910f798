"""Installer for the GASD DRUNet attention denoiser (`GASDDRUNetAttn`).

Surface of `neural_shift_cuda/integration/gasd_drunet_attn_patch.py`
(reference).  GASD is the row-stochastic denoiser W = Z^-1 K over the FULL
(2R+1)^2 window: every shift has its own network weight and no inverse
twin, so the shift table carries has_inv = 0 on every row.

Patched methods (CUDA inputs, `use_cuda_shift` on):

* `forward(x, guide=None, sig=None, return_D=...)`: weights from the model's
  own `_all_shift_weights` (models with `_gather_core`) or, for older files,
  from `shift_gather` + `attn_head.logit/weight` in chunks of
  `max_batch_shifts` with a joint softmax over all shifts; head mixing;
  comp_box mask when `comp_box` is on; one `normalized_accumulate_uz`.
* `forward_cached(x, cache)`, `_KT_action_cached`, `laplacian_grw_cached`
  for a fixed guide's cached edges (`cache.shifts`, `cache.w_list`,
  `cache.Z`, `cache.C`).
* `_KT_action`, `NLM_transpose`, `laplacian_grw`: K^T y(p) =
  sum_s w_s(p - d) y(p - d), one `accumulate_uz(..., transpose=True)` over
  the forward weight stack itself.  (The reference rolls every weight plane
  by its shift into a second stack and accumulates over the negated table,
  pi^-1(w * y) = pi^-1(w) * pi^-1(y); the kernel reads the planes at
  p - d instead, so no rolled copy is made.)

A single-head model's weights stay one-channel (the kernels share them
across channels) instead of being expanded and copied C times.
"""

from __future__ import annotations

import inspect
from typing import Optional

import torch
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint as grad_checkpoint

from ..ops import accumulate_uz, normalized_accumulate_uz, shift_gather
from ._common import (box_stack, cached_shift_tensor, flat, head_mix_matrix,
                      mix_heads, normalise_sigma, shift_tensor)


def _rows(model):
    return [(int(dx), int(dy), 0) for dx, dy in model._collect_shifts()]


def _get_shift_tensor(self, device):
    return cached_shift_tensor(self, "_nsc_gasd_shifts", lambda: _rows(self), device)


def _eval_chunking(model):
    if not model.training:
        model.max_batch_shifts = 10


def _restore_chunking(model):
    if not model.training:
        model.max_batch_shifts = None


def _weight_stack(model, x, guide, sig):
    """(S, B, Cw, H, W) final per-shift weights, comp_box applied."""
    B, C, H, W = x.shape
    R = model.window_rad
    phi = model.pre_activation(x if guide is None else guide, sigma=sig).contiguous()
    shifts = _get_shift_tensor(model, x.device)
    S = shifts.shape[0]
    mat = head_mix_matrix(model)
    use_box = bool(getattr(model, "comp_box", True))
    if hasattr(model, "_gather_core"):
        padded = F.pad(phi, (R, R, R, R), mode="circular")
        w = torch.stack(list(model._all_shift_weights(
            phi, padded, sig, model._collect_shifts())), 0)
        w = mix_heads(w, C, mat)
        if use_box:
            w = w * box_stack(shifts[:, :2], H, W, w.dtype, w.device)
        return w
    # older files: chunked gather + the head's logit / weight API
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
    w = torch.cat(tiles, 0)                                  # (S, B, h, H, W)
    if model.output_activation == "softmax":
        # joint softmax over every shift, then the mask (as the model does)
        w = F.softmax(w - w.amax(0, keepdim=True), dim=0)
    w = mix_heads(w, C, mat)
    if use_box:
        w = w * box_stack(shifts[:, :2], H, W, w.dtype, w.device)
    return w


def _forward_cuda(self, x, guide=None, sig=None, return_D=True):
    _eval_chunking(self)
    sig = normalise_sigma(x, sig)
    w = _weight_stack(self, x, guide, sig)
    D, log_Z = normalized_accumulate_uz(
        x.contiguous(), flat(w), _get_shift_tensor(self, x.device),
        return_log_degree=True, validate=False)
    _restore_chunking(self)
    return (D, log_Z.exp()) if return_D else (D, None)


# ----------------------------------------------------------------- cached

def _pack(self, x, cache):
    """(S*B, C, H, W) cached forward weights, packed once per cache."""
    if x.dim() != 4:
        raise ValueError(f"x must have shape (B,C,H,W), got {tuple(x.shape)}.")
    if x.size(1) != cache.C:
        raise ValueError(
            f"cached weights have C={cache.C} channels but x has {x.size(1)}; "
            f"rebuild the cache for this channel count.")
    key = (id(cache), tuple(x.shape), x.device, x.dtype)
    st = getattr(self, "_nsc_gasd_pack", None)
    if st is not None and st[0] is cache and st[1] == key:
        return st[2], st[3]
    w = list(cache.w_list)
    if len(w) != len(cache.shifts) or not w:
        raise ValueError("cached w_list must contain one tensor per cached shift.")
    for t in w:
        if tuple(t.shape) != tuple(x.shape):
            raise ValueError("cached weights and x must have identical (B,C,H,W) shapes.")
        if t.device != x.device or t.dtype != x.dtype:
            raise ValueError("cached weights and x must share device and dtype.")
    stack = torch.stack(w, 0)
    shifts = shift_tensor([(dx, dy, 0) for dx, dy in cache.shifts], x.device)
    self._nsc_gasd_pack = (cache, key, stack, shifts)
    return stack, shifts


def _forward_cached_cuda(self, x, cache, return_D=True):
    stack, shifts = _pack(self, x, cache)
    D, log_Z = normalized_accumulate_uz(x.contiguous(), flat(stack), shifts,
                                        return_log_degree=True, validate=False)
    Z = cache.Z if getattr(cache, "Z", None) is not None else log_Z.exp()
    return (D, Z) if return_D else (D, None)


def _kt_action_cached_cuda(self, y, cache):
    stack, shifts = _pack(self, y, cache)
    return accumulate_uz(y.contiguous(), flat(stack), shifts, transpose=True)[0]


def _lap_from(z, log_Z):
    floor = log_Z.new_tensor(1e-6).log()
    return z * (-torch.maximum(log_Z, floor)).exp()


def _laplacian_grw_cached_cuda(self, x, cache, eps=1e-10):
    stack, shifts = _pack(self, x, cache)
    D, log_Z = normalized_accumulate_uz(x.contiguous(), flat(stack), shifts,
                                        return_log_degree=True, validate=False)
    z = x - D
    return z - _kt_action_cached_cuda(self, _lap_from(z, log_Z), cache)


# ------------------------------------------------------------- transpose

def _kt(self, y, w_flat):
    """K^T y over the flat forward stack."""
    return accumulate_uz(y.contiguous(), w_flat, _get_shift_tensor(self, y.device),
                         transpose=True)[0]


def _kt_action_cuda(self, y, guide=None, sig=None):
    _eval_chunking(self)
    sig = normalise_sigma(y, sig)
    out = _kt(self, y, flat(_weight_stack(self, y, guide, sig)))
    _restore_chunking(self)
    return out


def _nlm_transpose_cuda(self, x, guide=None, sig=None, return_D=False):
    _eval_chunking(self)
    sig = normalise_sigma(x, sig)
    w = _weight_stack(self, x, x if guide is None else guide, sig)
    D = w.sum(0).expand(x.shape)
    out = _kt(self, x / D.clamp_min(1e-6), flat(w))
    _restore_chunking(self)
    return (out, D) if return_D else (out, None)


def _laplacian_grw_cuda(self, x, guide, sig=None, eps=1e-10):
    _eval_chunking(self)
    sig = normalise_sigma(x, sig)
    w = flat(_weight_stack(self, x, x if guide is None else guide, sig))
    D, log_Z = normalized_accumulate_uz(
        x.contiguous(), w, _get_shift_tensor(self, x.device),
        return_log_degree=True, validate=False)
    z = x - D
    out = z - _kt(self, _lap_from(z, log_Z), w)
    _restore_chunking(self)
    return out


# -------------------------------------------------------------- installer

def _route(self, x) -> bool:
    if not hasattr(self, "use_cuda_shift"):
        self.use_cuda_shift = True
    return bool(self.use_cuda_shift) and x.is_cuda


def _return_d_default(fn, fallback):
    p = inspect.signature(fn).parameters
    return ("return_D" in p, p["return_D"].default if "return_D" in p else fallback)


def install_cuda_shift(model_cls):
    """Patch a GASDDRUNetAttn class; idempotent."""
    if getattr(model_cls, "_nsc_gasd_installed", False):
        return model_cls
    model_cls._get_shift_tensor = _get_shift_tensor
    orig = model_cls.forward
    has_rd, rd_default = _return_d_default(orig, True)

    def forward(self, x, guide=None, sig=None, return_D=rd_default):
        if _route(self, x):
            return _forward_cuda(self, x, guide=guide, sig=sig, return_D=return_D)
        if has_rd:
            return orig(self, x, guide=guide, sig=sig, return_D=return_D)
        return orig(self, x, guide=guide, sig=sig)

    model_cls.forward = forward

    orig_cached = getattr(model_cls, "forward_cached", None)
    if orig_cached is not None:
        c_has_rd, c_default = _return_d_default(orig_cached, True)

        def forward_cached(self, x, cache, return_D=c_default):
            if _route(self, x):
                return _forward_cached_cuda(self, x, cache, return_D=return_D)
            if c_has_rd:
                return orig_cached(self, x, cache, return_D=return_D)
            return orig_cached(self, x, cache)

        model_cls.forward_cached = forward_cached

    orig_ktc = getattr(model_cls, "_KT_action_cached", None)
    if orig_ktc is not None:
        def kt_cached(self, y, cache):
            if _route(self, y):
                return _kt_action_cached_cuda(self, y, cache)
            return orig_ktc(self, y, cache)

        model_cls._KT_action_cached = kt_cached

    orig_lgc = getattr(model_cls, "laplacian_grw_cached", None)
    if orig_lgc is not None:
        def lap_cached(self, x, cache, eps=1e-10):
            if _route(self, x):
                return _laplacian_grw_cached_cuda(self, x, cache, eps=eps)
            return orig_lgc(self, x, cache, eps=eps)

        model_cls.laplacian_grw_cached = lap_cached

    orig_kt = getattr(model_cls, "_KT_action", None)
    orig_nt = getattr(model_cls, "NLM_transpose", None)
    orig_lg = getattr(model_cls, "laplacian_grw", None)

    def _missing(self, name):
        raise AttributeError(
            f"{type(self).__name__} has no reference {name}; add the "
            f"arch-level method before installing.")

    def kt_action(self, y, guide=None, sig=None):
        if _route(self, y):
            return _kt_action_cuda(self, y, guide=guide, sig=sig)
        if orig_kt is None:
            _missing(self, "_KT_action")
        return orig_kt(self, y, guide=guide, sig=sig)

    def nlm_transpose(self, x, guide=None, sig=None, return_D=False):
        if _route(self, x):
            return _nlm_transpose_cuda(self, x, guide=guide, sig=sig,
                                       return_D=return_D)
        if orig_nt is None:
            _missing(self, "NLM_transpose")
        return orig_nt(self, x, guide=guide, sig=sig, return_D=return_D)

    def laplacian_grw(self, x, guide, sig=None, eps=1e-10):
        if _route(self, x):
            return _laplacian_grw_cuda(self, x, guide, sig=sig, eps=eps)
        if orig_lg is None:
            _missing(self, "laplacian_grw")
        return orig_lg(self, x, guide, sig=sig, eps=eps)

    model_cls._KT_action = kt_action
    model_cls.NLM_transpose = nlm_transpose
    model_cls.laplacian_grw = laplacian_grw
    model_cls._nsc_gasd_installed = True
    return model_cls
