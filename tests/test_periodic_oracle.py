"""The periodic-mirror extension (table column value 2) in the oracle:
equal to the explicit edge list the reference patches build for comp_box
off -- every forward row plus, per mirror row, the row (-dx, -dy, 0) over
the forward weight rolled by (dx, dy)
(`patches/nekde_drunet_attn_patch.py:346-366`).  CPU only."""

import torch

from oracle import nsc_oracle as O


def _explicit(w, rows, B):
    """(E*B, Cw, H, W) weights and (E, 3) rows of the periodic operator."""
    S = len(rows)
    ws = w.reshape(S, B, *w.shape[1:])
    parts, out = [], []
    for s, (dx, dy, inv) in enumerate(rows):
        parts.append(ws[s])
        out.append((dx, dy, 0))
        if inv:
            parts.append(torch.roll(ws[s], shifts=(dx, dy), dims=(-2, -1)))
            out.append((-dx, -dy, 0))
    return torch.cat(parts, 0), out


def test_accumulate_periodic_equals_explicit_edges():
    torch.manual_seed(0)
    B, C, H, W, R = 2, 3, 9, 11, 2
    rows = O.halfplane_shifts(R)
    S = len(rows)
    x = torch.rand(B, C, H, W, dtype=torch.float64)
    w = torch.rand(S * B, 1, H, W, dtype=torch.float64)
    per = [(dx, dy, 2 if inv else 0) for dx, dy, inv in rows]
    U, Z = O.accumulate_uz(x, w.expand(-1, C, -1, -1), per)
    we, re = _explicit(w, rows, B)
    Ue, Ze = O.accumulate_uz(x, we.expand(-1, C, -1, -1), re)
    torch.testing.assert_close(U, Ue, rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(Z, Ze, rtol=1e-12, atol=1e-12)
    # gradients: the explicit form's weight gradient folds back onto w
    gU, gZ = torch.randn_like(U), torch.randn_like(Z)
    gx, gw = O.accumulate_uz_backward(x, w, gU, gZ, per)
    wv = w.clone().requires_grad_(True)
    xv = x.clone().requires_grad_(True)
    we2, _ = _explicit(wv, rows, B)
    U2, Z2 = O.accumulate_uz(xv, we2.expand(-1, C, -1, -1), re)
    (U2 * gU + Z2 * gZ).sum().backward()
    torch.testing.assert_close(gx, xv.grad, rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(gw, wv.grad, rtol=1e-12, atol=1e-12)


def test_normalized_periodic_equals_explicit_edges():
    torch.manual_seed(1)
    B, C, H, W, R = 1, 2, 8, 7, 2
    rows = O.halfplane_shifts(R)
    S = len(rows)
    x = torch.rand(B, C, H, W, dtype=torch.float64)
    lg = 2.0 * torch.randn(S * B, C, H, W, dtype=torch.float64)
    per = [(dx, dy, 2 if inv else 0) for dx, dy, inv in rows]
    D, L = O.normalized_accumulate_uz(x, lg, per, log_weights=True)
    we, re = _explicit(lg, rows, B)
    De, Le = O.normalized_accumulate_uz(x, we, re, log_weights=True)
    torch.testing.assert_close(D, De, rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(L, Le, rtol=1e-12, atol=1e-12)


def test_normalized_backward_periodic_equals_explicit_edges():
    torch.manual_seed(2)
    B, C, H, W, R = 1, 2, 8, 7, 2
    rows = O.halfplane_shifts(R)
    S = len(rows)
    x = torch.rand(B, C, H, W, dtype=torch.float64)
    lg = 2.0 * torch.randn(S * B, C, H, W, dtype=torch.float64)
    per = [(dx, dy, 2 if inv else 0) for dx, dy, inv in rows]
    D, L = O.normalized_accumulate_uz(x, lg, per, log_weights=True)
    gD, gL = torch.randn_like(D), torch.randn_like(L)
    gx, gw = O.normalized_accumulate_uz_backward(x, lg, D, L, gD, gL, per,
                                                 log_weights=True)
    we, re = _explicit(lg, rows, B)
    gxe, gwe = O.normalized_accumulate_uz_backward(x, we, D, L, gD, gL, re,
                                                   log_weights=True)
    torch.testing.assert_close(gx, gxe, rtol=1e-12, atol=1e-12)
    # fold the explicit rows back: a mirror row holds w rolled by (dx, dy)
    k = 0
    fold = []
    gwe = gwe.reshape(-1, B, C, H, W)
    for dx, dy, inv in rows:
        g = gwe[k].clone()
        k += 1
        if inv:
            g = g + torch.roll(gwe[k], shifts=(-dx, -dy), dims=(-2, -1))
            k += 1
        fold.append(g)
    torch.testing.assert_close(gw, torch.cat(fold, 0), rtol=1e-12, atol=1e-12)


def test_accumulate_transposed_rows_equal_rolled_kt():
    """Column value 3 (transposed row): sum_s w_s(p - d) x(p - d) equals the
    reference's K^T form -- accumulate over the negated shifts with every
    weight plane rolled by its own (dx, dy)
    (`integration/gasd_drunet_attn_patch.py:494-549`) -- values and
    gradients."""
    torch.manual_seed(1)
    B, C, H, W, R = 2, 3, 8, 10, 2
    rows = O.window_shifts(R)
    S = len(rows)
    x = torch.rand(B, C, H, W, dtype=torch.float64)
    w = torch.rand(S * B, 1, H, W, dtype=torch.float64)
    tr = [(dx, dy, 3) for dx, dy, _ in rows]
    U, Z = O.accumulate_uz(x, w.expand(-1, C, -1, -1), tr)

    def rolled(wt):
        ws = wt.reshape(S, B, *wt.shape[1:])
        return torch.cat([torch.roll(ws[s], shifts=(dx, dy), dims=(-2, -1))
                          for s, (dx, dy, _) in enumerate(rows)], 0)
    neg = [(-dx, -dy, 0) for dx, dy, _ in rows]
    Uk, Zk = O.accumulate_uz(x, rolled(w).expand(-1, C, -1, -1), neg)
    torch.testing.assert_close(U, Uk, rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(Z, Zk, rtol=1e-12, atol=1e-12)
    gU, gZ = torch.randn_like(U), torch.randn_like(Z)
    gx, gw = O.accumulate_uz_backward(x, w, gU, gZ, tr)
    wv = w.clone().requires_grad_(True)
    xv = x.clone().requires_grad_(True)
    U2, Z2 = O.accumulate_uz(xv, rolled(wv).expand(-1, C, -1, -1), neg)
    (U2 * gU + Z2 * gZ).sum().backward()
    torch.testing.assert_close(gx, xv.grad, rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(gw, wv.grad, rtol=1e-12, atol=1e-12)
