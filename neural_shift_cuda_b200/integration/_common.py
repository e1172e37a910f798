"""Helpers shared by the model installers.

Everything here is tensor glue around the ops: shift tables, comp_box masks,
head mixing and the inverse-edge rolls.  Where the reference builds these
with Python loops over the S shifts (one small launch each, e.g.
`integration/gasd_drunet_attn_patch.py:344-353`), they are built here with
one vectorised expression.
"""

from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch
import torch.nn.functional as F

Shift3 = Tuple[int, int, int]


def halfplane_rows(R: int) -> List[Tuple[int, int, bool]]:
    """The half-plane enumeration of the NECTR / NeKDe models
    (`integration/nectr_patch.py:55-69`): all (dx, dy) with dy in 1..R
    (every row has an inverse), then (dx, 0) for dx in 0..R (inverse iff
    dx != 0).  S = 2R^2 + 2R + 1."""
    rows = [(dx, dy, True) for dx in range(-R, R + 1) for dy in range(1, R + 1)]
    rows += [(dx, 0, dx != 0) for dx in range(0, R + 1)]
    return rows


def shift_tensor(rows: Sequence, device) -> torch.Tensor:
    """(S, 3) int64 tensor of (dx, dy, has_inv) rows."""
    return torch.tensor([(int(r[0]), int(r[1]), int(bool(r[2])) if len(r) > 2 else 0)
                         for r in rows], dtype=torch.int64, device=device)


def cached_shift_tensor(model, attr: str, rows_fn, device) -> torch.Tensor:
    """Per-model cache of an (S, 3) shift tensor, keyed by device and rows."""
    rows = [tuple(int(v) for v in r) for r in rows_fn()]
    key = (str(device), tuple(rows))
    state = getattr(model, attr, None)
    if state is None or state[0] != key:
        state = (key, shift_tensor(rows, device))
        setattr(model, attr, state)
    return state[1]


def box_stack(shifts_xy: torch.Tensor, H: int, W: int, dtype, device) -> torch.Tensor:
    """(S, 1, 1, H, W) comp_box masks: 1 where (h+dx, w+dy) is inside the
    image.  Same values as slicing a zero-padded ones image
    (`integration/gasd_drunet_attn_patch.py:344-353`), in one expression."""
    d = shifts_xy.to(device=device, dtype=torch.int64)
    hh = torch.arange(H, device=device)
    ww = torch.arange(W, device=device)
    rh = hh[None, :] + d[:, :1]
    rw = ww[None, :] + d[:, 1:2]
    mh = (rh >= 0) & (rh < H)
    mw = (rw >= 0) & (rw < W)
    return (mh[:, :, None] & mw[:, None, :]).to(dtype)[:, None, None]


def normalise_sigma(x: torch.Tensor, sig):
    """Bring `sig` to (B, 1, 1, 1) (or leave None), as the model forwards do
    (`integration/gasd_drunet_attn_patch.py:299-305`)."""
    B = x.shape[0]
    if sig is None:
        return None
    if not torch.is_tensor(sig):
        return x.new_full((B, 1, 1, 1), float(sig))
    if sig.dim() == 0:
        return sig.view(1, 1, 1, 1).expand(B, 1, 1, 1)
    if sig.shape[0] == 1 and B > 1:
        return sig.expand(B, *sig.shape[1:])
    return sig


def head_mix_matrix(model) -> Optional[torch.Tensor]:
    """(C, n_heads) head mixing with the model's own positive activation
    (`head_mix_pos_act`: softmax (default), softplus or relu)."""
    raw = getattr(model, "raw_head_mix", None)
    if raw is None:
        return None
    act = getattr(model, "head_mix_pos_act", "softmax")
    if act == "softmax":
        return F.softmax(raw, dim=1)
    if act == "softplus":
        return F.softplus(raw)
    return F.relu(raw)


def mix_heads(w_stack: torch.Tensor, C: int,
              mat: Optional[torch.Tensor]) -> torch.Tensor:
    """(S, B, n_heads, H, W) head weights -> per-channel weights.

    Cases follow the models' `_mix_heads`: one head is shared by every
    channel -- returned with ONE channel, which the ops read once per pixel
    for all channels (the reference expands and copies it C times); a mixing
    matrix mixes heads; n_heads == C is the identity; otherwise the head mean
    is shared by every channel."""
    n_heads = w_stack.shape[2]
    if n_heads == 1:
        return w_stack
    if mat is not None:
        return torch.einsum("ch,sbhij->sbcij", mat, w_stack)
    if n_heads == C:
        return w_stack
    return w_stack.mean(dim=2, keepdim=True)


def roll_index(shifts_xy: torch.Tensor, H: int, W: int, sign: int) -> torch.Tensor:
    """Flat gather index (S, 1, 1, H*W) of out(h, w) = in((h - sign*dx) mod H,
    (w - sign*dy) mod W), i.e. torch.roll by sign*(dx, dy) per slice."""
    d = shifts_xy.to(torch.int64)
    dev = d.device
    hh = torch.arange(H, device=dev).view(1, H, 1)
    ww = torch.arange(W, device=dev).view(1, 1, W)
    src_h = (hh - sign * d[:, 0].view(-1, 1, 1)) % H
    src_w = (ww - sign * d[:, 1].view(-1, 1, 1)) % W
    return (src_h * W + src_w).reshape(-1, 1, 1, H * W)


def roll_slices(stack: torch.Tensor, shifts_xy: torch.Tensor, sign: int = 1):
    """torch.roll of slice s of (S, B, C, H, W) by sign*(dx_s, dy_s), one
    gather for the whole stack."""
    S, B, C, H, W = stack.shape
    idx = roll_index(shifts_xy.to(stack.device), H, W, sign)
    return stack.reshape(S, B, C, H * W).gather(
        3, idx.expand(S, B, C, H * W)).view(S, B, C, H, W)


def periodic_edges(w_stack: torch.Tensor, rows: Sequence) -> Tuple[torch.Tensor, torch.Tensor]:
    """Explicit edge list of the periodic (comp_box off) symmetric operator:
    every forward edge (dx, dy, 0) and, for has_inv rows, the mirror edge
    (-dx, -dy, 0) whose weight is the forward weight rolled by (dx, dy)
    (`integration/nekde_drunet_attn_patch.py:346-366`).  Returns
    ((E*B, Cw, H, W) weights, (E, 3) shifts); the rolls of all mirror rows
    are one gather."""
    dev = w_stack.device
    S = w_stack.shape[0]
    inv = [i for i, r in enumerate(rows) if bool(r[2])]
    xy = torch.tensor([(int(r[0]), int(r[1])) for r in rows], dtype=torch.int64,
                      device=dev)
    mirrored = roll_slices(w_stack[inv], xy[inv], 1) if inv else None
    order, out_rows = [], []
    k = 0
    for i, r in enumerate(rows):
        order.append(("f", i))
        out_rows.append((int(r[0]), int(r[1]), 0))
        if bool(r[2]):
            order.append(("m", k))
            out_rows.append((-int(r[0]), -int(r[1]), 0))
            k += 1
    parts = [w_stack[j] if kind == "f" else mirrored[j] for kind, j in order]
    w_all = torch.stack(parts, 0)
    E, B = w_all.shape[:2]
    return (w_all.reshape(E * B, *w_all.shape[2:]).contiguous(),
            shift_tensor(out_rows, dev))


def flat(w_stack: torch.Tensor) -> torch.Tensor:
    """(S, B, C, H, W) -> contiguous (S*B, C, H, W)."""
    S, B = w_stack.shape[:2]
    return w_stack.reshape(S * B, *w_stack.shape[2:]).contiguous()
