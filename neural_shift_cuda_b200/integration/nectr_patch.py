"""Installer for the NECTR denoisers (`NECTR_denoiser`, official models 1
and 2) and the legacy batched `nekre` forward.

Surface of `neural_shift_cuda/integration/nectr_patch.py` (reference):
`install_cuda_shift(cls)` patches `cls.forward` so a CUDA forward runs

    guide = pre_activation(reference or x)
    pair, mask = pair_gather(guide, half-plane shifts)      # one kernel
    values, kind = the model's own head on `pair`            # cuDNN, unchanged
    values masked by comp_box (-inf for logits, *mask otherwise)
    D, log_C = normalized_accumulate_uz(x, values, shifts)   # one kernel

instead of the serial per-shift loop of `NECTR_models1.py:154-244`.  An
exponential head is kept in log space (`value / sigma^2`) so the positive
activation can never overflow before normalisation.  The official API
returns `(U / Z, Z)`; Z is materialised in float64 from log_C.

Fused inference path (no counterpart in the reference): when autograd is
off, no weight cache is read or stored and the head is the model-1
`proj` stack (1x1 conv, channel LayerNorm, LeakyReLU; one or two blocks of
width 8 / 16 / 32) followed by the bias-free `out` conv, the whole
sequence above runs as ONE kernel (`nsc_nectr_fused_fwd`): the first conv
of [g(p); g(p+d)] is split into two per-pixel maps computed once, and the
per-shift head is evaluated in registers, so the (S*B, 2L, H, W) pair batch
(4 GB at the benchmark's shape) is never written.  `instance.use_nectr_fused
= False` selects the unfused path.

Differences from the reference installer: a CPU input runs the model's
own original forward (the reference routes CPU inputs through its ops' CPU
implementations); `instance.use_cuda_shift = False` also selects the
original forward.
"""

from __future__ import annotations

import ctypes
import functools
import inspect
from typing import List, Tuple

import torch

from .. import _lib
from ..ops import (_defer_flag, accumulate_uz, check_validation,
                   normalized_accumulate_uz, pair_gather, shift_gather)
from ._common import halfplane_rows, shift_tensor

_MISSING = object()


class NECTRWeightCache(dict):
    """Per-shift weights of one guide, tagged with their representation
    ("log", "positive" or "raw"); keys are (dx, dy)."""

    def __init__(self, *args, weight_kind: str = "positive", **kwargs):
        super().__init__(*args, **kwargs)
        self.weight_kind = weight_kind


def _rows(model) -> List[Tuple[int, int, bool]]:
    own = getattr(model, "_collect_shifts", None)
    if callable(own):
        return [(int(dx), int(dy), bool(inv)) for dx, dy, inv in own()]
    return halfplane_rows(int(model.window_rad))


def _shifts(model, device):
    rows = _rows(model)
    key = (str(device), tuple(rows))
    state = getattr(model, "_nsc_nectr_shifts", None)
    if state is None or state[0] != key:
        state = (key, shift_tensor(rows, device))
        model._nsc_nectr_shifts = state
    return rows, state[1]


def _is_model2(model) -> bool:
    return hasattr(model, "unet") and hasattr(model, "layer_norm")


def _channel_ln(layer, v):
    """LayerNorm over channels of an NCHW tensor."""
    return layer(v.permute(0, 2, 3, 1)).permute(0, 3, 1, 2)


def _head(model, pair: torch.Tensor) -> Tuple[torch.Tensor, str]:
    """The model's unchanged weight head on the gathered [centre; shifted]
    batch, returning (values, kind) with kind in {"log", "positive", "raw"}
    (`NECTR_models1.py:118-148`, `NECTR_models2.py` N_theta)."""
    act = model.output_activation
    if _is_model2(model):
        v = model.out(_channel_ln(model.layer_norm, model.unet(pair)))
        if act == "control_sigmoid":
            k, a, b = torch.chunk(v, 3, dim=1)
            return model.controlled_sigmoid(k, a, b) + 1e-8, "positive"
        return v, "raw"
    if act == "sig":
        # The released model-1 'sig' branch reads an undefined name; defer to
        # the model's own method rather than invent a behaviour.
        half = pair.shape[1] // 2
        fn = getattr(model, "N_theta", None) or model.compute_weights
        return fn(pair[:, :half], pair[:, half:]), "raw"
    v = pair
    for block in model.proj:
        for j, layer in enumerate(block):
            v = _channel_ln(layer, v) if j == 1 else layer(v)
    v = model.out(v)
    if act == "exp":
        return v / model.sigma ** 2, "log"
    if act == "control_sigmoid":
        k, a, b = torch.chunk(v, 3, dim=1)
        return model.controlled_sigmoid(k, a, b) + 1e-8, "positive"
    return v, "raw"


def _weights(model, guide: torch.Tensor, shifts: torch.Tensor):
    if getattr(model, "use_cuda_pair_gather", True):
        pair, mask = pair_gather(guide.contiguous(), shifts)
    else:
        shifted, mask = shift_gather(guide.contiguous(), shifts)
        S = shifts.shape[0]
        pair = torch.cat((guide.repeat(S, 1, 1, 1), shifted), 1)
    values, kind = _head(model, pair)
    if kind == "log":
        values = values.masked_fill(mask <= 0, float("-inf"))
    else:
        values = values * mask
    return values.contiguous(), kind


def _cache_kind(model) -> str:
    if _is_model2(model):
        return "positive" if model.output_activation == "control_sigmoid" else "raw"
    act = model.output_activation
    return {"exp": "exp-positive", "control_sigmoid": "positive"}.get(act, "raw")


def _from_cache(model, cache, rows):
    values = torch.cat([cache[(dx, dy)] for dx, dy, _ in rows], 0)
    if isinstance(cache, NECTRWeightCache):
        return values.contiguous(), cache.weight_kind
    kind = _cache_kind(model)
    if kind == "exp-positive":
        # a cache of the unpatched exp head holds exponentiated weights
        values = torch.where(values > 0, values.log(),
                             torch.full_like(values, float("-inf")))
        kind = "log"
    return values.contiguous(), kind


def _to_cache(values, rows, B, kind) -> NECTRWeightCache:
    cache = NECTRWeightCache(weight_kind=kind)
    for (dx, dy, _), v in zip(rows, values.split(B, 0)):
        cache[(dx, dy)] = v
    return cache


def _aggregate(x, values, shifts, kind):
    if kind in ("positive", "log"):
        D, log_C = normalized_accumulate_uz(
            x.contiguous(), values, shifts, log_weights=(kind == "log"),
            return_log_degree=True, validate=True)
        # the released API returns the degree itself; float64 keeps a degree
        # that overflows float32 representable
        return D, log_C.to(torch.float64).exp()
    U, Z = accumulate_uz(x.contiguous(), values, shifts)
    return U / Z, Z


def _fused_head(model, x):
    """(width, depth, params, eps1, eps2, slope, mode) of a head the fused
    kernel implements, or None."""
    if not getattr(model, "use_nectr_fused", True) or _is_model2(model):
        return None
    if getattr(model, "model_type", "concat") != "concat":
        return None
    act = model.output_activation
    mode = {"exp": 1, "control_sigmoid": 2}.get(act, 0)
    if act == "sig":
        return None
    proj, out = getattr(model, "proj", None), getattr(model, "out", None)
    if proj is None or out is None or not 1 <= len(proj) <= 2:
        return None
    C = x.shape[1]
    if C not in (1, 3) or not isinstance(out, torch.nn.Conv2d) or out.bias is not None:
        return None
    convs, norms, slopes = [], [], set()
    for blk in proj:
        if len(blk) != 3:
            return None
        cv, ln, act_l = blk
        if not (isinstance(cv, torch.nn.Conv2d) and cv.kernel_size == (1, 1)
                and cv.bias is not None and isinstance(ln, torch.nn.LayerNorm)
                and ln.elementwise_affine and isinstance(act_l, torch.nn.LeakyReLU)):
            return None
        convs.append(cv)
        norms.append(ln)
        slopes.add(float(act_l.negative_slope))
    width = convs[0].out_channels
    if width not in (8, 16, 32) or len(slopes) != 1 or not 0.0 <= min(slopes) <= 1.0:
        return None
    if len(proj) == 2 and (convs[1].in_channels != width
                           or convs[1].out_channels != width // 2):
        return None
    cout = C * (3 if mode == 2 else 1)
    if out.out_channels != cout or out.in_channels != convs[-1].out_channels:
        return None
    R = max(max(abs(dx), abs(dy)) for dx, dy, _ in _rows(model))
    es = 8 if x.dtype == torch.float64 else 4
    if R > 16 or (2 * width + C) * (8 + 2 * R) * (32 + 2 * R) * es > 227 * 1024:
        return None
    flat = [convs[0].bias, norms[0].weight, norms[0].bias]
    if len(proj) == 2:
        flat += [convs[1].weight[:, :, 0, 0], convs[1].bias, norms[1].weight,
                 norms[1].bias]
    flat.append(out.weight[:, :, 0, 0])
    # host copy of the head parameters, refreshed only when one changes
    key = tuple((t.data_ptr(), t._version) for t in flat)
    held = getattr(model, "_nsc_fused_params", None)
    if held is None or held[0] != key:
        params = torch.cat([t.detach().reshape(-1).to(torch.float64).cpu()
                            for t in flat]).contiguous()
        held = (key, params)
        model._nsc_fused_params = held
    params = held[1]
    return (width, len(proj), params, float(norms[0].eps),
            float(norms[-1].eps), slopes.pop(), mode)


def _forward_fused(model, x, guide, head, shifts):
    width, depth, params, eps1, eps2, slope, mode = head
    dt = torch.float64 if x.dtype == torch.float64 else torch.float32
    g = guide.to(dt)
    L = g.shape[1]
    W1 = model.proj[0][0].weight.detach().to(dt)[:, :, 0, 0]
    if W1.shape[1] != 2 * L:
        return None
    B, _, H, W = guide.shape
    # [W1[:, :L]; W1[:, L:]] g as one batched product: (B, 2 width, H*W)
    AB = torch.matmul(torch.cat([W1[:, :L], W1[:, L:]], 0), g.reshape(B, L, H * W))
    xk = x.to(dt).contiguous()
    C = xk.shape[1]
    o0 = torch.empty_like(xk)
    o1 = torch.empty_like(xk)
    flag = torch.zeros(1, dtype=torch.int32, device=x.device) if mode else None
    hs = _lib.host_shifts(shifts)
    with torch.cuda.device(x.device):
        _lib.call("nsc_nectr_fused_fwd", _lib.ptr(xk), _lib.ptr(AB),
                  _lib.dtype_code(dt), B, C, H, W, width, depth,
                  ctypes.cast(params.data_ptr(), ctypes.POINTER(ctypes.c_double)),
                  params.numel(), eps1, eps2, slope, 1.0 / float(model.sigma) ** 2,
                  hs.ptr, hs.S, mode, _lib.ptr(o0), _lib.ptr(o1), _lib.ptr(flag),
                  _lib.stream_of(xk))
    if mode == 0:
        return o0 / o1, o1
    _defer_flag(flag, mode == 1)
    return o0, o1.to(torch.float64).exp()


def _forward_official(model, x, reference=None, sig=None, cache=None,
                      store_cache=False):
    guide = model.pre_activation(x if reference is None else reference, sigma=sig)
    rows, shifts = _shifts(model, x.device)
    if cache is None and not store_cache and not torch.is_grad_enabled():
        head = _fused_head(model, x)
        if head is not None:
            check_validation(block=False)
            out = _forward_fused(model, x, guide, head, shifts)
            if out is not None:
                return out
    if cache is None:
        values, kind = _weights(model, guide, shifts)
        held = _to_cache(values, rows, x.shape[0], kind) if store_cache else None
    else:
        values, kind = _from_cache(model, cache, rows)
        held = {} if store_cache else None
    D, degree = _aggregate(x, values, shifts, kind)
    if store_cache:
        return D, degree, held
    return D, degree


def _forward_legacy(model, x, guide=None, sig=None):
    feats = model.pre_activation(x if guide is None else guide, sigma=sig)
    _, shifts = _shifts(model, x.device)
    values, kind = _weights(model, feats, shifts)
    return _aggregate(x, values, shifts, kind)


def _use_cuda(model, x) -> bool:
    if not hasattr(model, "use_cuda_shift"):
        model.use_cuda_shift = True
    if not hasattr(model, "use_cuda_pair_gather"):
        model.use_cuda_pair_gather = True
    return (bool(model.use_cuda_shift) and x.is_cuda
            and getattr(model, "model_type", "concat") == "concat")


def install_cuda_shift(nectr_cls):
    """Patch an official `NECTR_denoiser` (forward(x, reference=None,
    sig=None, cache=None, store_cache=False)) or a legacy batched `nekre`
    (forward(x, guide=None, sig=None, batched=...)).  Idempotent."""
    if hasattr(nectr_cls, "_nsc_original_forward"):
        return nectr_cls
    original = nectr_cls.forward
    params = inspect.signature(original).parameters
    nectr_cls._nsc_original_forward = original

    if "batched" in params:
        default = params["batched"].default
        default = False if default is inspect.Parameter.empty else default

        @functools.wraps(original)
        def forward(self, x, guide=None, sig=None, batched=_MISSING):
            b = default if batched is _MISSING else batched
            if bool(b) and _use_cuda(self, x):
                return _forward_legacy(self, x, guide=guide, sig=sig)
            return original(self, x, guide=guide, sig=sig, batched=b)
    else:
        if not {"reference", "cache", "store_cache"} <= set(params):
            raise TypeError(
                "NECTR patch expected either the legacy batched forward or "
                "the official reference/cache/store_cache forward contract")

        @functools.wraps(original)
        def forward(self, x, reference=None, sig=None, cache=None,
                    store_cache=False):
            if _use_cuda(self, x):
                return _forward_official(self, x, reference=reference, sig=sig,
                                         cache=cache, store_cache=store_cache)
            return original(self, x, reference=reference, sig=sig, cache=cache,
                            store_cache=store_cache)

    nectr_cls.forward = forward
    return nectr_cls
