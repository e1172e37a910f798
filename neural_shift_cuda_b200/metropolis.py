"""Metropolis-normalized symmetric aggregation on B200
(the surface of `neural_shift_cuda.metropolis`, reference
`neural_shift_cuda/metropolis.py:195-238`).

    metropolis_aggregate(w_half, img, shifts, use_box, eps=1e-6,
                         checkpoint_train=True) -> (Wx, d_hat)

w_half: (B, S, C, H, W) forward half-plane weights (or channel-broadcast
(B, S, 1, H, W) with C <= 4, or a stride-0 expand of it); img: (B, C, H, W);
shifts: (S, 3) rows (dx, dy, has_inv) as a list or tensor.  The mirror edge
of each has_inv row is the forward weight read at p - d (circular) inside
the kernels; with use_box a neighbour reached only by wrap-around is masked.
Returns Wx = x - d_hat x + K_hat x and d_hat = K_hat e.

Unlike the reference, the CUDA path is differentiable: a fused backward
kernel pair replaces the reference's autograd through two accumulate_uz
calls, a shift_gather and a stack of rolled weights (`metropolis.py:117-192`).
`checkpoint_train` is accepted for API compatibility; nothing needs
recomputing because only the inputs and one (B, C, H, W) degree map are kept
for backward.
"""

from __future__ import annotations

from typing import List, Tuple

import torch

from . import _lib
from .ops import _require_cuda

__all__ = ["metropolis_aggregate"]


class _MetropolisFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, w_half, img, hs, use_box, eps):
        B, S, Cw, H, W = w_half.shape
        C = img.shape[1]
        acc = torch.float64 if img.dtype == torch.float64 else torch.float32
        Wx = torch.empty_like(img)
        dh = torch.empty_like(img)
        degree = torch.empty((B, Cw, H, W), dtype=acc, device=img.device)
        with torch.cuda.device(img.device):
            _lib.call("nsc_metropolis_fwd", _lib.ptr(w_half),
                      _lib.dtype_code(w_half.dtype), Cw, _lib.ptr(img),
                      _lib.dtype_code(img.dtype), B, C, H, W, hs.ptr, hs.S,
                      int(bool(use_box)), float(eps), _lib.ptr(Wx),
                      _lib.ptr(dh), _lib.ptr(degree), _lib.stream_of(img))
        ctx.save_for_backward(w_half, img, degree, dh)
        ctx.hs, ctx.use_box, ctx.eps = hs, bool(use_box), float(eps)
        return Wx, dh

    @staticmethod
    def backward(ctx, gWx, gdh):
        w_half, img, degree, dh = ctx.saved_tensors
        hs = ctx.hs
        B, S, Cw, H, W = w_half.shape
        C = img.shape[1]
        gWx = gWx.to(img.dtype).contiguous()
        gdh = gdh.to(img.dtype).contiguous()
        g_deg = torch.empty_like(degree)
        gw = torch.empty_like(w_half)
        gx = torch.empty_like(img)
        with torch.cuda.device(img.device):
            _lib.call("nsc_metropolis_bwd", _lib.ptr(w_half),
                      _lib.dtype_code(w_half.dtype), Cw, _lib.ptr(img),
                      _lib.dtype_code(img.dtype), B, C, H, W, hs.ptr, hs.S,
                      int(ctx.use_box), ctx.eps, _lib.ptr(degree),
                      _lib.ptr(dh), _lib.ptr(gWx), _lib.ptr(gdh),
                      _lib.ptr(g_deg), _lib.ptr(gw), _lib.ptr(gx),
                      _lib.stream_of(img))
        return gw, gx, None, None, None


def metropolis_aggregate(
    w_half: torch.Tensor,
    img: torch.Tensor,
    shifts,
    use_box: bool,
    eps: float = 1e-6,
    checkpoint_train: bool = True,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Fused Metropolis aggregate -> (Wx, d_hat); see the module doc."""
    del checkpoint_train  # nothing to recompute (see module docstring)
    _require_cuda("metropolis_aggregate", w_half, img)
    if w_half.dim() != 5 or img.dim() != 4:
        raise RuntimeError(
            "metropolis_aggregate: w_half must be (B, S, C, H, W) and img "
            "(B, C, H, W)")
    hs = _lib.host_shifts(shifts)
    if hs.t.dim() != 2 or hs.cols != 3:
        raise ValueError("metropolis_aggregate: shifts must be (S, 3) rows "
                         "(dx, dy, has_inv)")
    B, S, Cw, H, W = w_half.shape
    C = img.shape[1]
    if hs.S != S or img.shape[0] != B or img.shape[2:] != w_half.shape[3:]:
        raise RuntimeError(
            f"metropolis_aggregate: w_half {tuple(w_half.shape)}, img "
            f"{tuple(img.shape)} and {hs.S} shifts do not agree")
    if Cw == C and C > 1 and w_half.stride(2) == 0 and C <= 4:
        w_half = w_half[:, :, :1]
        Cw = 1
    if not (Cw == C or (Cw == 1 and C <= 4)):
        if Cw == 1:
            w_half = w_half.expand(B, S, C, H, W)
        else:
            raise RuntimeError(
                f"metropolis_aggregate: w_half has {Cw} channels, img {C}")
    dt = torch.promote_types(w_half.dtype, img.dtype)
    if dt not in _lib._DTYPES:
        raise TypeError(f"metropolis_aggregate: unsupported dtype {dt}")
    return _MetropolisFn.apply(w_half.to(dt).contiguous(),
                               img.to(dt).contiguous(), hs, bool(use_box),
                               float(eps))
