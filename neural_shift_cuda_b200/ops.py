"""Shift-window ops on B200: the public surface of `neural_shift_cuda.ops`.

    shift_gather(guide, shifts)                  -> (gs_batch, mask_batch)
    pair_gather(guide, shifts)                   -> (pair_batch, mask_batch)
    accumulate_uz(x, weights, shifts)            -> (U_num, Z)
    normalized_accumulate_uz(x, weights, shifts) -> D or (D, log_C)

Same names, argument meaning, output layouts and error types as the
reference (`neural_shift_cuda/ops.py:576-679`).  Every op is a
`torch.autograd.Function` over the sm_100a kernels of `libnsc_b200.so`
(forward and backward).  Differences, all deliberate:

* CUDA tensors only.  The reference silently runs a PyTorch fallback for
  CPU tensors; this package has none and raises instead.
* fp16 / bf16 inputs are read natively and promoted in registers (the
  reference first materialises fp32 copies, `ops.py:67-74`).  Outputs keep
  the reference's accumulator dtypes: fp32, or fp64 when an input is fp64.
* A weight stack may be channel-broadcast: `(S*B, 1, H, W)` with C > 1, or
  a stride-0 `expand` of it.  It is read once per pixel for all channels.
* `validate=True` in `normalized_accumulate_uz` is checked inside the
  reduction kernel (no extra pass over the weights) and, like the
  reference's `torch._assert_async`, without a host synchronisation: the
  kernel's flag word is copied to pinned host memory behind an event and a
  violation raises ValueError at the next normalized call or backward that
  finds the copy complete, or at `check_validation()`, which waits for it.
"""

from __future__ import annotations

import threading
from typing import List, Tuple

import torch

from . import _lib

__all__ = ["shift_gather", "pair_gather", "accumulate_uz",
           "normalized_accumulate_uz", "check_validation", "index_width_bits"]

_MAX_S = 1024


def index_width_bits() -> int:
    """ABI marker of the loaded kernel library (always 64)."""
    return _lib.index_width_bits()


# ---------------------------------------------------------------------------
# argument handling
# ---------------------------------------------------------------------------

def _require_cuda(op: str, *tensors: torch.Tensor) -> None:
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(
                f"neural_shift_cuda_b200.{op}: expects CUDA tensors (got a "
                f"{t.device} tensor); this package has no CPU path")
    lib_ok = _lib.available()
    if not lib_ok:
        _lib.load()  # raises with the loader's error
    if _lib.index_width_bits() != 64:
        raise RuntimeError(
            f"neural_shift_cuda_b200.{op}: the loaded kernel library does not "
            f"use 64-bit indices; rebuild it from the current source")


def _check_shift_shape(shifts, need3: bool, op: str):
    if isinstance(shifts, torch.Tensor):
        if shifts.dim() != 2 or shifts.size(1) not in (2, 3):
            raise ValueError(
                f"shifts must be (S, 2) or (S, 3); got {tuple(shifts.shape)}")
        if need3 and shifts.size(1) != 3:
            raise ValueError(f"{op} requires shifts of shape (S, 3)")
    hs = _lib.host_shifts(shifts)
    if hs.t.dim() != 2 or hs.cols not in (2, 3):
        raise ValueError(
            f"shifts must be (S, 2) or (S, 3); got {tuple(hs.t.shape)}")
    if need3 and hs.cols != 3:
        raise ValueError(f"{op} requires shifts of shape (S, 3)")
    return hs


def _check_nchw(t: torch.Tensor, name: str) -> None:
    if t.dim() != 4:
        raise RuntimeError(f"{name} must have 4 dims (N,C,H,W)")


def _accumulator_dtype(*tensors: torch.Tensor) -> torch.dtype:
    for t in tensors:
        if not t.is_floating_point():
            raise TypeError(
                f"accumulation inputs must be floating point; got {t.dtype}")
    return (torch.float64 if any(t.dtype == torch.float64 for t in tensors)
            else torch.float32)


def _storage_dtypes(x: torch.Tensor, w: torch.Tensor):
    """Dtypes the kernels read x and w in.  fp64 anywhere -> both fp64;
    equal dtypes pass through; otherwise x (small) is read as fp32 and w
    keeps its own half / bf16 / fp32 storage."""
    if x.device != w.device:
        raise ValueError(
            f"x and weights must share a device; got {x.device} and {w.device}")
    acc = _accumulator_dtype(x, w)
    if acc == torch.float64:
        return torch.float64, torch.float64
    if x.dtype == w.dtype:
        return x.dtype, w.dtype
    return torch.float32, w.dtype


def _weights_view(weights: torch.Tensor, S: int, B: int, C: int, H: int,
                  W: int, op: str) -> torch.Tensor:
    """Return the (S*B, Cw, H, W) tensor the kernels read, Cw in {C, 1}.

    A stride-0 channel expand is reduced to its single channel (autograd
    then sums the weight gradient over channels, the exact gradient of a
    shared weight)."""
    _check_nchw(weights, "weights")
    if (weights.size(0) != S * B or weights.size(2) != H or weights.size(3) != W
            or weights.size(1) not in (C, 1)):
        raise RuntimeError(
            f"{op}: weights must be (S*B, C, H, W) = {(S * B, C, H, W)}"
            f" (or channel-broadcast (S*B, 1, H, W)); got "
            f"{tuple(weights.shape)}")
    if C > 1 and weights.size(1) == C and weights.stride(1) == 0:
        weights = weights[:, :1]
    return weights.contiguous()


# ---------------------------------------------------------------------------
# gathers
# ---------------------------------------------------------------------------

def _gather_chunks(S: int):
    return [(s0, min(S, s0 + _MAX_S)) for s0 in range(0, S, _MAX_S)]


class _GatherFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, guide, hs, pair):
        guide = guide.contiguous()
        B, C, H, W = guide.shape
        S = hs.S
        Cout = 2 * C if pair else C
        out = torch.empty((S * B, Cout, H, W), dtype=guide.dtype,
                          device=guide.device)
        mask = torch.empty((S * B, 1, H, W), dtype=guide.dtype,
                           device=guide.device)
        name = "nsc_pair_gather_fwd" if pair else "nsc_shift_gather_fwd"
        if out.numel() or mask.numel():
            with torch.cuda.device(guide.device):
                for s0, s1 in _gather_chunks(S):
                    sub = _lib.HostShifts(hs.t[s0:s1].contiguous())
                    _lib.call(name, _lib.ptr(guide),
                              _lib.dtype_code(guide.dtype), B, C, H, W,
                              sub.ptr, s1 - s0, hs.cols,
                              _lib.ptr(out[s0 * B:s1 * B]),
                              _lib.ptr(mask[s0 * B:s1 * B]),
                              _lib.stream_of(guide))
        ctx.hs = hs
        ctx.pair = pair
        ctx.shape = (B, C, H, W)
        ctx.mark_non_differentiable(mask)
        return out, mask

    @staticmethod
    def backward(ctx, grad_out, grad_mask):
        hs, pair = ctx.hs, ctx.pair
        B, C, H, W = ctx.shape
        grad_out = grad_out.contiguous()
        name = "nsc_pair_gather_bwd" if pair else "nsc_shift_gather_bwd"
        gg = None
        if grad_out.numel():
            with torch.cuda.device(grad_out.device):
                for s0, s1 in _gather_chunks(hs.S):
                    part = torch.empty((B, C, H, W), dtype=grad_out.dtype,
                                       device=grad_out.device)
                    sub = _lib.HostShifts(hs.t[s0:s1].contiguous())
                    _lib.call(name, _lib.ptr(grad_out[s0 * B:s1 * B]),
                              _lib.dtype_code(grad_out.dtype), B, C, H, W,
                              sub.ptr, s1 - s0, hs.cols, _lib.ptr(part),
                              _lib.stream_of(grad_out))
                    gg = part if gg is None else gg + part
        if gg is None:
            gg = torch.zeros((B, C, H, W), dtype=grad_out.dtype,
                             device=grad_out.device)
        return gg, None, None


def _gather(guide, shifts, pair: bool, op: str):
    hs = _check_shift_shape(shifts, False, op)
    _require_cuda(op, guide)
    _check_nchw(guide, "guide")
    if guide.dtype not in _lib._DTYPES:
        raise TypeError(f"{op}: unsupported dtype {guide.dtype}")
    if hs.S == 0:
        raise RuntimeError(f"{op}: at least one shift is required")
    return _GatherFn.apply(guide, hs, pair)


def shift_gather(guide: torch.Tensor, shifts) -> Tuple[torch.Tensor, torch.Tensor]:
    """Circular windows of `guide` for every row of `shifts`.

        gs[s*B + b, c, h, w]   = guide[b, c, (h+dx_s) mod H, (w+dy_s) mod W]
        mask[s*B + b, 0, h, w] = 1 iff 0 <= h+dx_s < H and 0 <= w+dy_s < W

    Bit-exact copies; mask in guide's dtype (reference `ops.py:576-591`)."""
    return _gather(guide, shifts, False, "shift_gather")


def pair_gather(guide: torch.Tensor, shifts) -> Tuple[torch.Tensor, torch.Tensor]:
    """`shift_gather` with the centre guide concatenated first along
    channels: pair[s*B+b, :C] = guide[b], pair[s*B+b, C:] = shifted guide
    (reference `ops.py:594-609`)."""
    return _gather(guide, shifts, True, "pair_gather")


# ---------------------------------------------------------------------------
# accumulate_uz
# ---------------------------------------------------------------------------

class _AccumulateUZFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, hs):
        B, C, H, W = x.shape
        acc = torch.float64 if x.dtype == torch.float64 else torch.float32
        U = torch.empty((B, C, H, W), dtype=acc, device=x.device)
        Z = torch.empty_like(U)
        with torch.cuda.device(x.device):
            _lib.call("nsc_accumulate_uz_fwd", _lib.ptr(x),
                      _lib.dtype_code(x.dtype), _lib.ptr(w),
                      _lib.dtype_code(w.dtype), w.size(1), B, C, H, W,
                      hs.ptr, hs.S, _lib.ptr(U), _lib.ptr(Z),
                      _lib.stream_of(x))
        ctx.save_for_backward(x, w)
        ctx.hs = hs
        return U, Z

    @staticmethod
    def backward(ctx, grad_U, grad_Z):
        x, w = ctx.saved_tensors
        hs = ctx.hs
        B, C, H, W = x.shape
        acc = torch.float64 if x.dtype == torch.float64 else torch.float32
        gU = grad_U.to(acc).contiguous()
        gZ = grad_Z.to(acc).contiguous()
        gx = torch.empty((B, C, H, W), dtype=acc, device=x.device)
        gw = torch.empty_like(w)
        with torch.cuda.device(x.device):
            _lib.call("nsc_accumulate_uz_bwd", _lib.ptr(x),
                      _lib.dtype_code(x.dtype), _lib.ptr(w),
                      _lib.dtype_code(w.dtype), w.size(1), B, C, H, W,
                      hs.ptr, hs.S, _lib.ptr(gU), _lib.ptr(gZ),
                      _lib.ptr(gx), _lib.ptr(gw), _lib.stream_of(x))
        return gx.to(x.dtype), gw, None


def _prep_reduction(x, weights, shifts, op, periodic_mirror=False,
                    transpose=False):
    xd, wd = _storage_dtypes(x, weights)
    hs = _lib.mirror_mode(_check_shift_shape(shifts, not transpose, op),
                          periodic_mirror, transpose)
    _require_cuda(op, x, weights)
    _check_nchw(x, "x")
    B, C, H, W = x.shape
    if not (1 <= hs.S <= _MAX_S):
        raise RuntimeError(f"{op}: tree reduction requires 1 <= S <= 1024")
    w = _weights_view(weights, hs.S, B, C, H, W, op)
    return x.to(xd).contiguous(), w.to(wd), hs


def accumulate_uz(x: torch.Tensor, weights: torch.Tensor, shifts, *,
                  periodic_mirror: bool = False, transpose: bool = False):
    """(U_num, Z) over all shifts including the mirror branch of has_inv
    rows; weights are pre-multiplied by the forward box mask by the caller
    (reference `ops.py:612-631`).  U = U_num / Z is left to the caller.

    periodic_mirror=True (an extension): the mirror term of every has_inv
    row reads w and x at (p - d) mod (H, W) without the inside test -- the
    periodic (comp_box off) operator, without materialising rolled planes.

    transpose=True (an extension): the transpose of the forward-only
    operator of the same (forward-only, (S, 2) or has_inv == 0) table and
    weights, U(p) = sum_s w_s(p - d) x(p - d) circularly, Z likewise.  The
    reference forms K^T as accumulate_uz over negated shifts and weight
    planes rolled by (dx, dy) (`integration/gasd_drunet_attn_patch.py:494-549`);
    this reads the original planes instead of a rolled copy."""
    x_k, w_k, hs = _prep_reduction(x, weights, shifts, "accumulate_uz",
                                   periodic_mirror, transpose)
    return _AccumulateUZFn.apply(x_k, w_k, hs)


# ---------------------------------------------------------------------------
# normalized_accumulate_uz
# ---------------------------------------------------------------------------

_POS_MSG = "positive weights must be finite and nonnegative"
_LOG_MSG = "log_weights may be finite or -inf (mask), but not NaN or +inf"

# Validation flags of launched normalized forwards whose result the host has
# not read yet: (pinned host copy, event after the copy, log_weights).
_pending: List[Tuple[torch.Tensor, "torch.cuda.Event", bool]] = []
_pending_lock = threading.Lock()


def _defer_flag(flag: torch.Tensor, log_weights: bool) -> None:
    host = torch.empty(1, dtype=torch.int32, pin_memory=True)
    host.copy_(flag, non_blocking=True)
    ev = torch.cuda.Event()
    ev.record(torch.cuda.current_stream(flag.device))
    with _pending_lock:
        _pending.append((host, ev, bool(log_weights)))


def check_validation(block: bool = True) -> None:
    """Raise ValueError if a `validate=True` normalized forward launched so
    far saw a NaN / +inf weight (or a negative positive-mode weight).

    block=True waits for the pending flag copies (a host synchronisation on
    their streams); block=False only reads the copies that have completed.
    Each flag is reported once."""
    with _pending_lock:
        todo = list(_pending)
        _pending.clear()
    keep, bad = [], None
    for host, ev, lw in todo:
        if block:
            ev.synchronize()
        elif not ev.query():
            keep.append((host, ev, lw))
            continue
        if bad is None and int(host[0]) != 0:
            bad = lw
    if keep:
        with _pending_lock:
            _pending[:0] = keep
    if bad is not None:
        raise ValueError(_LOG_MSG if bad else _POS_MSG)


class _NormalizedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, hs, log_weights, validate):
        B, C, H, W = x.shape
        acc = torch.float64 if x.dtype == torch.float64 else torch.float32
        D = torch.empty((B, C, H, W), dtype=acc, device=x.device)
        L = torch.empty_like(D)
        flag = (torch.zeros(1, dtype=torch.int32, device=x.device)
                if validate else None)
        with torch.cuda.device(x.device):
            _lib.call("nsc_normalized_accumulate_uz_fwd", _lib.ptr(x),
                      _lib.dtype_code(x.dtype), _lib.ptr(w),
                      _lib.dtype_code(w.dtype), w.size(1), B, C, H, W,
                      hs.ptr, hs.S, int(bool(log_weights)), _lib.ptr(D),
                      _lib.ptr(L), _lib.ptr(flag), _lib.stream_of(x))
        if flag is not None:
            _defer_flag(flag, log_weights)
        ctx.save_for_backward(x, w, D, L)
        ctx.hs = hs
        ctx.log_weights = bool(log_weights)
        ctx.set_materialize_grads(False)
        return D, L

    @staticmethod
    def backward(ctx, grad_D, grad_L):
        check_validation(block=False)
        x, w, D, L = ctx.saved_tensors
        hs = ctx.hs
        B, C, H, W = x.shape
        gD = (torch.zeros_like(D) if grad_D is None
              else grad_D.to(D.dtype).contiguous())
        gL = (torch.zeros_like(L) if grad_L is None
              else grad_L.to(L.dtype).contiguous())
        gx = torch.empty_like(D)
        gw = torch.empty_like(w)
        with torch.cuda.device(x.device):
            _lib.call("nsc_normalized_accumulate_uz_bwd", _lib.ptr(x),
                      _lib.dtype_code(x.dtype), _lib.ptr(w),
                      _lib.dtype_code(w.dtype), w.size(1), B, C, H, W,
                      hs.ptr, hs.S, int(ctx.log_weights), _lib.ptr(D),
                      _lib.ptr(L), _lib.ptr(gD), _lib.ptr(gL), _lib.ptr(gx),
                      _lib.ptr(gw), _lib.stream_of(x))
        return gx.to(x.dtype), gw, None, None, None


def normalized_accumulate_uz(x: torch.Tensor, weights: torch.Tensor, shifts,
                             *, log_weights: bool = False,
                             return_log_degree: bool = False,
                             validate: bool = True,
                             periodic_mirror: bool = False):
    """Overflow-safe D = K / C over the shift window (reference
    `ops.py:634-679`).

    weights: (S*B, C, H, W) positive weights (0 masks) or, with
    log_weights=True, logits (-inf masks).  Returns D, or (D, log_C) with
    return_log_degree=True.  One pass per output with a running maximum;
    empty rows give D = 0, log_C = -inf.  validate=True flags a NaN / +inf
    weight or a negative positive-mode weight on the device; the ValueError
    is raised without a host synchronisation by a later normalized call or
    backward, or at once by `check_validation()`.  periodic_mirror=True:
    mirror terms are periodic (see accumulate_uz)."""
    check_validation(block=False)
    x_k, w_k, hs = _prep_reduction(x, weights, shifts,
                                   "normalized_accumulate_uz", periodic_mirror)
    D, L = _NormalizedFn.apply(x_k, w_k, hs, bool(log_weights), bool(validate))
    if return_log_degree:
        return D, L
    return D
