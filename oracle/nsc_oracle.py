"""CPU oracle for the shift-window hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in plain PyTorch on the CPU, the algorithms of the
reference project `neural_shift_cuda` (v0.12.0) for the five hot-path ops.
It is the checker used by `tests/`, by `__graft_entry__.smoke()` and by the
`cpu_baseline` / `--impl reference` legs of `bench.py`.  Nothing in the
product package (`neural_shift_cuda_b200`) imports it; the product path has
no CPU fallback.

Parity pin: `tests/golden/make_golden.py` runs the reference's own PyTorch
code on small seeded inputs and stores the results under `tests/golden/`;
`tests/test_oracle_golden.py` checks every function here against those
fixtures (see the per-function notes for the tolerance used).

Conventions (reference `neural_shift_cuda/ops.py:576-591`):
  * shifts rows are (dx, dy[, has_inv]); dx indexes H (rows), dy indexes W.
  * gather: out(h, w) = x((h + dx) mod H, (w + dy) mod W).
  * box / validity mask for (dx, dy): 1 iff 0 <= h+dx < H and 0 <= w+dy < W.
  * the synthesized inverse ("mirror") term of a row with has_inv reads the
    same weight plane at (h - dx, w - dy) and is masked by the box of
    (-dx, -dy), i.e. it is never periodic.
"""

from __future__ import annotations

from typing import List, Sequence, Tuple

import torch

__all__ = [
    "halfplane_shifts", "window_shifts", "box_mask",
    "shift_gather", "pair_gather", "shift_gather_backward",
    "pair_gather_backward", "tree_sum", "accumulate_uz",
    "accumulate_uz_backward", "normalized_accumulate_uz",
    "normalized_accumulate_uz_backward", "metropolis_aggregate",
    "metropolis_aggregate_grad", "premasked_weights",
]


# ---------------------------------------------------------------------------
# shift tables and masks
# ---------------------------------------------------------------------------

def halfplane_shifts(R: int) -> List[Tuple[int, int, int]]:
    """Half-plane enumeration, S = 2R^2 + 2R + 1.

    Follows `neural_shift_cuda/integration/nectr_patch.py:55-69` and
    `tests/test_accumulate_uz.py:12-19`: every (dx, dy) with dy in [1, R]
    (all rows have an inverse), then (dx, 0) for dx in [0, R] with an inverse
    for dx != 0.
    """
    rows = [(dx, dy, 1) for dx in range(-R, R + 1) for dy in range(1, R + 1)]
    rows += [(dx, 0, int(dx != 0)) for dx in range(0, R + 1)]
    return rows


def window_shifts(R: int) -> List[Tuple[int, int, int]]:
    """Full (2R+1)^2 window without inverse rows
    (`integration/gasd_drunet_attn_patch.py:96-103`)."""
    return [(dx, dy, 0) for dx in range(-R, R + 1) for dy in range(-R, R + 1)]


def _rows(shifts) -> List[Tuple[int, int, int]]:
    if isinstance(shifts, torch.Tensor):
        shifts = shifts.to(torch.int64).tolist()
    out = []
    for r in shifts:
        out.append((int(r[0]), int(r[1]), int(r[2]) if len(r) > 2 else 0))
    return out


def _valid(n: int, d: int) -> torch.Tensor:
    idx = torch.arange(n)
    return (idx + d >= 0) & (idx + d < n)


def box_mask(H: int, W: int, dx: int, dy: int, dtype=torch.float32):
    """(H, W) mask: 1 iff (h+dx, w+dy) lies inside the image.

    Same values as the zero-padded ones image sliced at (R+dx, R+dy) in
    `ops.py:118-130`.
    """
    return (_valid(H, dx)[:, None] & _valid(W, dy)[None, :]).to(dtype)


def _gather(x: torch.Tensor, dx: int, dy: int) -> torch.Tensor:
    """x((h+dx) mod H, (w+dy) mod W) -- a circular roll by (-dx, -dy)."""
    if dx == 0 and dy == 0:
        return x
    return torch.roll(x, shifts=(-dx, -dy), dims=(-2, -1))


# ---------------------------------------------------------------------------
# gathers (reference ops.py:95-154, shift_ops_cuda.cu:62-246)
# ---------------------------------------------------------------------------

def shift_gather(guide: torch.Tensor, shifts):
    """(S*B, C, H, W) circular windows plus the (S*B, 1, H, W) mask.

    Bit-exact copy semantics of `shift_gather_reference` (`ops.py:95-135`).
    """
    rows = _rows(shifts)
    B, C, H, W = guide.shape
    outs, masks = [], []
    for dx, dy, _ in rows:
        outs.append(_gather(guide, dx, dy))
        masks.append(box_mask(H, W, dx, dy, guide.dtype)
                     .expand(B, 1, H, W))
    return torch.cat(outs, 0).contiguous(), torch.cat(masks, 0).contiguous()


def pair_gather(guide: torch.Tensor, shifts):
    """[center; shifted] along channels (`ops.py:138-154`)."""
    gs, mask = shift_gather(guide, shifts)
    S = gs.shape[0] // guide.shape[0]
    center = guide.repeat(S, 1, 1, 1)
    return torch.cat([center, gs], 1).contiguous(), mask


def shift_gather_backward(grad_out: torch.Tensor, shifts, B, C, H, W):
    """Adjoint of the circular gather: sum over shifts of the rolled-back
    gradient planes (`shift_ops_cuda.cu:166-203`)."""
    rows = _rows(shifts)
    g = grad_out.reshape(len(rows), B, C, H, W)
    acc = torch.zeros(B, C, H, W, dtype=grad_out.dtype)
    for s, (dx, dy, _) in enumerate(rows):
        acc = acc + _gather(g[s], -dx, -dy)
    return acc


def pair_gather_backward(grad_out: torch.Tensor, shifts, B, C, H, W):
    """Adjoint of `pair_gather` (`shift_ops_cuda.cu:206-246`)."""
    rows = _rows(shifts)
    g = grad_out.reshape(len(rows), B, 2 * C, H, W)
    acc = torch.zeros(B, C, H, W, dtype=grad_out.dtype)
    for s, (dx, dy, _) in enumerate(rows):
        acc = acc + g[s, :, :C] + _gather(g[s, :, C:], -dx, -dy)
    return acc


# ---------------------------------------------------------------------------
# accumulate_uz (reference ops.py:157-206; kernels shift_ops_cuda.cu:256-458)
# ---------------------------------------------------------------------------

def tree_sum(values: torch.Tensor) -> torch.Tensor:
    """Pairwise reduction over dim 0, level by level: (0+1), (2+3), ... with
    an odd tail carried to the next level -- the summation order of
    `_tree_sum` (`ops.py:77-92`)."""
    level = values
    while level.shape[0] > 1:
        n = level.shape[0]
        nxt = level[0:n - 1:2] + level[1:n:2]
        if n % 2:
            nxt = torch.cat([nxt, level[n - 1:]], 0)
        level = nxt
    return level[0]


def _acc_dtype(*ts):
    return torch.float64 if any(t.dtype == torch.float64 for t in ts) \
        else torch.float32


def _mirror(w: torch.Tensor, dx: int, dy: int, periodic: bool = False) -> torch.Tensor:
    """w((h-dx) mod H, (w-dy) mod W) masked by the box of (-dx, -dy); with
    periodic=True unmasked -- the mirror row as the reference patches build
    it for comp_box off, a forward row over the rolled weight plane
    (`patches/nekde_drunet_attn_patch.py:346-366`).  Table column value 2
    selects the periodic form (an extension of the reference's 0/1)."""
    H, W = w.shape[-2:]
    if periodic:
        return _gather(w, -dx, -dy)
    return _gather(w, -dx, -dy) * box_mask(H, W, -dx, -dy, w.dtype)


def accumulate_uz(x: torch.Tensor, weights: torch.Tensor, shifts):
    """(U, Z) = sums over shifts of w*x_shift and w, plus mirror terms.

    Inputs are promoted first (fp16/bf16/fp32 -> fp32, fp64 stays), as in
    `ops.py:51-74`; terms are summed with `tree_sum` in the order
    [fwd_0, inv_0, fwd_1, inv_1, ...] like `ops.py:177-206`.
    """
    dt = _acc_dtype(x, weights)
    x = x.to(dt)
    B, C, H, W = x.shape
    rows = _rows(shifts)
    wv = weights.to(dt).reshape(len(rows), B, -1, H, W).expand(
        len(rows), B, C, H, W)
    u_terms, z_terms = [], []
    for s, (dx, dy, inv) in enumerate(rows):
        wf = wv[s]
        if inv != 3:       # column value 3: transposed row, no forward term
            u_terms.append(wf * _gather(x, dx, dy))
            z_terms.append(wf)
        if inv:
            wi = _mirror(wf, dx, dy, inv in (2, 3))
            u_terms.append(wi * _gather(x, -dx, -dy))
            z_terms.append(wi)
    return tree_sum(torch.stack(u_terms)), tree_sum(torch.stack(z_terms))


def accumulate_uz_backward(x, weights, grad_U, grad_Z, shifts):
    """Analytic gradients of `accumulate_uz` (`shift_ops_cuda.cu:344-458`).

    grad_x(q) = sum_s w_s(q-d) gU(q-d) [circular] +
                inv*box(q+d) w_s(q) gU(q+d)
    grad_w_s(q) = x(q+d) gU(q) + gZ(q) + inv*box(q+d) (x(q) gU(q+d) + gZ(q+d))
    Returns grad_w with the weights' own shape (a channel-broadcast weight
    gets the channel sum).
    """
    dt = _acc_dtype(x, weights)
    x, gU, gZ = x.to(dt), grad_U.to(dt), grad_Z.to(dt)
    B, C, H, W = x.shape
    rows = _rows(shifts)
    Cw = weights.shape[1]
    wv = weights.to(dt).reshape(len(rows), B, Cw, H, W).expand(
        len(rows), B, C, H, W)
    gx = torch.zeros_like(x)
    gws = []
    for s, (dx, dy, inv) in enumerate(rows):
        wf = wv[s]
        if inv != 3:
            gx = gx + _gather(wf * gU, -dx, -dy)
            gw = _gather(x, dx, dy) * gU + gZ
        else:
            gw = torch.zeros_like(x)
        if inv:
            m = box_mask(H, W, dx, dy, dt) if inv not in (2, 3) else torch.ones(H, W, dtype=dt)
            gx = gx + m * wf * _gather(gU, dx, dy)
            gw = gw + m * (x * _gather(gU, dx, dy) + _gather(gZ, dx, dy))
        if Cw == 1 and C > 1:
            gw = gw.sum(1, keepdim=True)
        gws.append(gw)
    return gx, torch.cat(gws, 0)


def premasked_weights(w: torch.Tensor, shifts, B: int) -> torch.Tensor:
    """Multiply an (S*B, Cw, H, W) tensor by each row's forward box mask
    (`tests/test_accumulate_uz.py:30-45`)."""
    rows = _rows(shifts)
    H, W = w.shape[-2:]
    m = torch.stack([box_mask(H, W, dx, dy, w.dtype) for dx, dy, _ in rows])
    m = m[:, None, None].expand(len(rows), B, 1, H, W).reshape(-1, 1, H, W)
    return w * m


# ---------------------------------------------------------------------------
# normalized_accumulate_uz (reference ops.py:209-320; kernels
# shift_ops_cuda.cu:460-791)
# ---------------------------------------------------------------------------

def _as_log(w: torch.Tensor, log_weights: bool) -> torch.Tensor:
    if log_weights:
        return w
    pos = w > 0
    return torch.where(pos, torch.where(pos, w, torch.ones_like(w)).log(),
                       torch.full_like(w, -torch.inf))


def normalized_accumulate_uz(x, weights, shifts, log_weights=False):
    """(D, log_C): row-max-shifted normalized reduction.

    Follows `normalized_accumulate_uz_reference` (`ops.py:234-320`):
    log-weights (or log of positive weights, -inf for zero), row max m,
    a = exp(l - m), D = sum(a x) / sum(a), log_C = m + log(sum(a)).  Rows with
    m == -inf give D = 0 and log_C = -inf.  No contract validation is done
    here (the public op validates before calling the kernels).
    """
    dt = _acc_dtype(x, weights)
    x = x.to(dt)
    B, C, H, W = x.shape
    rows = _rows(shifts)
    wv = weights.to(dt).reshape(len(rows), B, -1, H, W).expand(
        len(rows), B, C, H, W)
    logs, vals = [], []
    for s, (dx, dy, inv) in enumerate(rows):
        wf = wv[s]
        logs.append(_as_log(wf, log_weights))
        vals.append(_gather(x, dx, dy))
        if inv:
            wi = _gather(wf, -dx, -dy)
            keep = (box_mask(H, W, -dx, -dy, dt) > 0) if inv != 2 else \
                torch.ones(H, W, dtype=torch.bool)
            if log_weights:
                wi = torch.where(keep, wi, torch.full_like(wi, -torch.inf))
            else:
                wi = wi * keep.to(dt)
            logs.append(_as_log(wi, log_weights))
            vals.append(_gather(x, -dx, -dy))
    L = torch.stack(logs)
    V = torch.stack(vals)
    m = L.amax(0)
    empty = torch.isinf(m) & (m < 0)
    a = torch.where(empty[None], torch.full_like(L, -torch.inf),
                    L - m[None]).exp()
    num = tree_sum(a * V)
    den = tree_sum(a)
    D = torch.where(empty, torch.zeros_like(num), num / den)
    logC = torch.where(empty, torch.full_like(m, -torch.inf), m + den.log())
    return D, logC


def _fraction(lw, logC):
    """exp(lw - logC), 0 where either is -inf (`shift_ops_cuda.cu:517-525`)."""
    neg = torch.isneginf(lw) | torch.isneginf(logC)
    return torch.where(neg, torch.zeros_like(lw),
                       (torch.where(neg, torch.zeros_like(lw), lw - logC)).exp())


def normalized_accumulate_uz_backward(x, weights, D, logC, grad_D, grad_logC,
                                      shifts, log_weights=False):
    """Analytic gradients of the normalized reduction, with the reference
    kernels' conventions (`shift_ops_cuda.cu:656-791`): a masked weight
    (zero, or -inf logit) gets gradient 0; positive mode uses
    d/dw = exp(-log_C) * score, log mode p * score, where
    score = gD (x_partner - D) + g_logC.
    """
    dt = _acc_dtype(x, weights)
    x, D, logC = x.to(dt), D.to(dt), logC.to(dt)
    gD, gL = grad_D.to(dt), grad_logC.to(dt)
    B, C, H, W = x.shape
    rows = _rows(shifts)
    Cw = weights.shape[1]
    wv = weights.to(dt).reshape(len(rows), B, Cw, H, W).expand(
        len(rows), B, C, H, W)
    gx = torch.zeros_like(x)
    gws = []
    for s, (dx, dy, inv) in enumerate(rows):
        wf = wv[s]
        lw = _as_log(wf, log_weights)
        live = ~torch.isneginf(lw)
        # forward use: output q reads x(q+d)
        p_f = _fraction(lw, logC)
        gx = gx + _gather(p_f * gD, -dx, -dy)
        score_f = gD * (_gather(x, dx, dy) - D) + gL
        fac_f = p_f if log_weights else torch.exp(-logC)
        gw = fac_f * score_f
        if inv:
            m = (box_mask(H, W, dx, dy, dt) > 0) if inv != 2 else \
                torch.ones(H, W, dtype=torch.bool)
            logC_i = _gather(logC, dx, dy)
            p_i = _fraction(lw, logC_i)
            gx = gx + torch.where(m, p_i * _gather(gD, dx, dy),
                                  torch.zeros_like(x))
            score_i = _gather(gD, dx, dy) * (x - _gather(D, dx, dy)) + \
                _gather(gL, dx, dy)
            fac_i = p_i if log_weights else torch.exp(-logC_i)
            gw = gw + torch.where(m, fac_i * score_i, torch.zeros_like(x))
        gw = torch.where(live, gw, torch.zeros_like(gw))
        if Cw == 1 and C > 1:
            gw = gw.sum(1, keepdim=True)
        gws.append(gw)
    return gx, torch.cat(gws, 0)


# ---------------------------------------------------------------------------
# metropolis_aggregate (reference metropolis.py:54-192,
# metropolis_cuda.cu:71-186)
# ---------------------------------------------------------------------------

def metropolis_aggregate(w_half, img, shifts, use_box: bool, eps=1e-6):
    """(Wx, d_hat) of the Metropolis-normalized symmetric operator.

    d(p)   = sum over edges e of wt_e(p) (forward edge masked by box(+d),
             mirror edge = forward weight at p-d (circular), masked by
             box(-d) when use_box).
    wk_e(p) = wt_e(p) / max(max(d(p), d(p+delta_e)), eps)
    K_hat x = sum wk_e(p) x(p+delta_e);  d_hat = sum wk_e(p)
    Wx      = x - d_hat x + K_hat x
    Differentiable through torch autograd (used for the gradient oracle,
    like the reference's own autograd path `metropolis.py:117-192`).
    Sums run sequentially over edges like `metropolis.py:77-108`.
    """
    rows = _rows(shifts)
    B, S, Cw, H, W = w_half.shape
    C = img.shape[1]
    dt = img.dtype
    w = w_half.expand(B, S, C, H, W)
    edges = []   # (weight plane (B,C,H,W), delta)
    for s, (dx, dy, inv) in enumerate(rows):
        wf = w[:, s]
        if use_box:
            wf = wf * box_mask(H, W, dx, dy, dt)
        edges.append((wf, dx, dy))
        if inv:
            wi = _gather(wf, -dx, -dy)
            if use_box:
                wi = wi * box_mask(H, W, -dx, -dy, dt)
            edges.append((wi, -dx, -dy))
    d = torch.zeros_like(img)
    for wt, _, _ in edges:
        d = d + wt
    kx = torch.zeros_like(img)
    dh = torch.zeros_like(img)
    epsv = torch.tensor(eps, dtype=dt)
    for wt, ex, ey in edges:
        den = torch.maximum(d, _gather(d, ex, ey)).clamp_min(epsv)
        wk = wt / den
        kx = kx + wk * _gather(img, ex, ey)
        dh = dh + wk
    return img - dh * img + kx, dh


def metropolis_aggregate_grad(w_half, img, shifts, use_box, eps, gWx, gdh):
    """Gradients (grad_w_half, grad_img) via autograd of
    `metropolis_aggregate` (the reference trains through autograd of the
    same expression, `metropolis.py:117-192`; torch.maximum splits ties
    equally and clamp_min passes the gradient where its input >= eps)."""
    w = w_half.detach().clone().requires_grad_(True)
    x = img.detach().clone().requires_grad_(True)
    Wx, dh = metropolis_aggregate(w, x, shifts, use_box, eps)
    (Wx * gWx + dh * gdh).sum().backward()
    return w.grad, x.grad
