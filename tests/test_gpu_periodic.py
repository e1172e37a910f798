"""GPU parity of the periodic-mirror extension (`periodic_mirror=True`:
mirror terms read (p - d) mod (H, W) without the inside test) against the
oracle, whose periodic form is pinned to the reference patches' explicit
rolled-plane edge list (tests/test_periodic_oracle.py).  The tiled
accumulate path declines periodic rows, so these run the general kernels."""

import pytest
import torch

import neural_shift_cuda_b200 as nsc
from oracle import nsc_oracle as O

pytestmark = pytest.mark.gpu


def _per(rows):
    return [(dx, dy, 2 if inv else 0) for dx, dy, inv in rows]


def close(a, b, tol):
    torch.testing.assert_close(a.detach().cpu().to(b.dtype), b, rtol=tol, atol=tol)


@pytest.mark.parametrize("bcast", [False, True])
@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-11), (torch.float32, 1e-5)])
def test_accumulate_periodic_fwd_bwd(cuda, bcast, dtype, tol):
    torch.manual_seed(3)
    B, C, H, W, R = 2, 3, 13, 10, 3
    rows = O.halfplane_shifts(R)
    S = len(rows)
    x = torch.rand(B, C, H, W, dtype=dtype)
    w = torch.rand(S * B, 1 if bcast else C, H, W, dtype=dtype)
    xc = x.to(cuda).requires_grad_(True)
    wc = w.to(cuda).requires_grad_(True)
    U, Z = nsc.accumulate_uz(xc, wc, torch.tensor(rows), periodic_mirror=True)
    Ur, Zr = O.accumulate_uz(x, w.expand(-1, C, -1, -1), _per(rows))
    close(U, Ur, tol)
    close(Z, Zr, tol)
    gU, gZ = torch.randn_like(Ur), torch.randn_like(Zr)
    (U * gU.to(cuda) + Z * gZ.to(cuda)).sum().backward()
    gx, gw = O.accumulate_uz_backward(x, w, gU, gZ, _per(rows))
    close(xc.grad, gx, tol * 10)
    close(wc.grad, gw, tol * 10)
    # the masked form differs near the border
    U0, _ = nsc.accumulate_uz(x.to(cuda), w.to(cuda), torch.tensor(rows))
    assert not torch.allclose(U0, U)


@pytest.mark.parametrize("log_weights", [True, False])
def test_normalized_periodic_fwd_bwd(cuda, log_weights):
    torch.manual_seed(4)
    B, C, H, W, R = 1, 2, 9, 12, 2
    rows = O.halfplane_shifts(R)
    S = len(rows)
    x = torch.rand(B, C, H, W, dtype=torch.float64)
    if log_weights:
        w = 2.0 * torch.randn(S * B, C, H, W, dtype=torch.float64)
    else:
        w = torch.rand(S * B, C, H, W, dtype=torch.float64) + 0.1
    xc = x.to(cuda).requires_grad_(True)
    wc = w.to(cuda).requires_grad_(True)
    D, L = nsc.normalized_accumulate_uz(xc, wc, torch.tensor(rows), log_weights=log_weights,
                                        return_log_degree=True, periodic_mirror=True)
    Dr, Lr = O.normalized_accumulate_uz(x, w, _per(rows), log_weights)
    close(D, Dr, 1e-10)
    close(L, Lr, 1e-10)
    gD, gL = torch.randn_like(Dr), torch.randn_like(Lr)
    (D * gD.to(cuda) + L * gL.to(cuda)).sum().backward()
    gx, gw = O.normalized_accumulate_uz_backward(x, w, Dr, Lr, gD, gL, _per(rows),
                                                 log_weights)
    close(xc.grad, gx, 1e-9)
    close(wc.grad, gw, 1e-9)


def test_periodic_gradcheck(cuda):
    torch.manual_seed(5)
    rows = torch.tensor(O.halfplane_shifts(1))
    x = torch.rand(1, 1, 5, 4, dtype=torch.float64, device=cuda, requires_grad=True)
    w = torch.rand(len(rows), 1, 5, 4, dtype=torch.float64, device=cuda, requires_grad=True)
    assert torch.autograd.gradcheck(
        lambda a, b: nsc.accumulate_uz(a, b, rows, periodic_mirror=True), (x, w))


def test_value_two_without_flag_is_masked(cuda):
    """A table carrying 2 in column 2 keeps the reference's meaning (any
    nonzero = masked mirror) unless periodic_mirror=True."""
    torch.manual_seed(6)
    rows = O.halfplane_shifts(2)
    S = len(rows)
    x = torch.rand(1, 1, 8, 8, dtype=torch.float64)
    w = torch.rand(S, 1, 8, 8, dtype=torch.float64)
    twos = torch.tensor([(dx, dy, 2 * inv) for dx, dy, inv in rows])
    U, Z = nsc.accumulate_uz(x.to(cuda), w.to(cuda), twos)
    Ur, Zr = O.accumulate_uz(x, w, rows)
    close(U, Ur, 1e-12)
    close(Z, Zr, 1e-12)


@pytest.mark.parametrize("C,Cw", [(3, 1), (3, 3), (5, 1)])
@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-11), (torch.float32, 1e-5)])
def test_accumulate_transpose_fwd_bwd(cuda, C, Cw, dtype, tol):
    """accumulate_uz(..., transpose=True): U(p) = sum_s w_s(p - d) x(p - d)
    over the original planes, against the oracle's transposed rows (pinned
    to the reference's rolled-plane K^T form on the CPU)."""
    torch.manual_seed(4)
    B, H, W, R = 2, 11, 14, 2
    rows = O.window_shifts(R)
    S = len(rows)
    x = torch.rand(B, C, H, W, dtype=dtype)
    w = torch.rand(S * B, Cw, H, W, dtype=dtype)
    xc = x.to(cuda).requires_grad_(True)
    wc = w.to(cuda).requires_grad_(True)
    sh = torch.tensor([(dx, dy) for dx, dy, _ in rows])
    U, Z = nsc.accumulate_uz(xc, wc, sh, transpose=True)
    tr = [(dx, dy, 3) for dx, dy, _ in rows]
    Ur, Zr = O.accumulate_uz(x, w.expand(-1, C, -1, -1), tr)
    close(U, Ur, tol)
    close(Z, Zr, tol)
    gU, gZ = torch.randn_like(Ur), torch.randn_like(Zr)
    (U * gU.to(cuda) + Z * gZ.to(cuda)).sum().backward()
    gx, gw = O.accumulate_uz_backward(x, w, gU, gZ, tr)
    close(xc.grad, gx, tol)
    close(wc.grad, gw, tol)


def test_transpose_rejects_mirror_rows(cuda):
    x = torch.rand(1, 1, 6, 6, device=cuda)
    w = torch.rand(3, 1, 6, 6, device=cuda)
    with pytest.raises(ValueError, match="forward-only"):
        nsc.accumulate_uz(x, w, torch.tensor(O.halfplane_shifts(1))[:3], transpose=True)


@pytest.mark.parametrize("dtype,C,Cw,H,W,R", [
    (torch.float32, 3, 1, 37, 64, 3),
    (torch.float16, 3, 1, 40, 136, 5),
    (torch.bfloat16, 1, 1, 23, 48, 2),
    (torch.float32, 2, 2, 30, 36, 4),
])
def test_tiled_periodic_matches_oracle(cuda, monkeypatch, dtype, C, Cw, H, W, R):
    """Periodic mirror rows on the tiled path (masked tile kernel plus the
    wrapped terms of the border band): accumulate_uz and the normalized
    reduction in log and positive modes, against the oracle."""
    monkeypatch.setenv("NSC_REQUIRE_FAST", "1")
    torch.manual_seed(H + W)
    rows = O.halfplane_shifts(R)
    sh = torch.tensor(rows)
    S, B = len(rows), 2
    x = torch.rand(B, C, H, W).to(dtype)
    w = torch.rand(S * B, Cw, H, W).to(dtype)
    per = _per(rows)
    U, Z = nsc.accumulate_uz(x.to(cuda), w.to(cuda), sh, periodic_mirror=True)
    Ur, Zr = O.accumulate_uz(x, w.expand(-1, C, -1, -1), per)
    close(U, Ur, 1e-5)
    close(Z, Zr, 1e-5)
    for logw in (False, True):
        k = (3.0 * torch.randn(S * B, Cw, H, W)).to(dtype) if logw else w
        D, L = nsc.normalized_accumulate_uz(x.to(cuda), k.to(cuda), sh, log_weights=logw,
                                            return_log_degree=True, validate=False,
                                            periodic_mirror=True)
        Dr, Lr = O.normalized_accumulate_uz(x, k.expand(-1, C, -1, -1), per, logw)
        close(D, Dr, 1e-5)
        close(L, Lr, 1e-5)
