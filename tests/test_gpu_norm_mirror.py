"""GPU parity of the tiled normalized_accumulate_uz forward for tables
with mirror terms (the half-plane tables of NECTR and NeKDe): the TMA tile
kernel of csrc/accumulate_fast.cuh in its normalized modes, against the CPU
oracle.

NSC_REQUIRE_FAST makes the C entry point fail instead of falling back to
the general kernel, so every case here runs a tiled kernel.  Shapes cover
partial tiles, images smaller than the window, radii 2 / 5 / 10, log and
positive modes, per-channel and channel-broadcast keys, fp32 / bf16 / fp16
storage and the special key values of the reference contract (NaN / +inf
poison, -inf / zero masks, empty rows).  Tolerance: fp32 rtol/atol 1e-5.
"""

import math

import pytest
import torch

import neural_shift_cuda_b200 as nsc
from oracle import nsc_oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _require_fast(monkeypatch, cuda):
    monkeypatch.setenv("NSC_REQUIRE_FAST", "1")


def T(rows):
    return torch.tensor(rows, dtype=torch.int64)


def run(x, k, sh, logw, validate=False):
    D, L = nsc.normalized_accumulate_uz(x.cuda(), k.cuda(), sh, log_weights=logw,
                                        return_log_degree=True, validate=validate)
    if validate:
        nsc.check_validation()
    return D.cpu(), L.cpu()


def ref(x, k, sh, logw):
    C = x.shape[1]
    kk = k.expand(-1, C, -1, -1) if k.shape[1] == 1 else k
    return O.normalized_accumulate_uz(x, kk, sh, logw)


def close(a, b, tol=1e-5):
    torch.testing.assert_close(a, b.to(a.dtype), rtol=tol, atol=tol, equal_nan=True)


def keys(S, B, Cw, H, W, logw, dtype, sh=None, premask=True):
    if logw:
        k = 3.0 * torch.randn(S * B, Cw, H, W)
    else:
        k = torch.nn.functional.softplus(torch.randn(S * B, Cw, H, W))
    if premask and sh is not None:
        # forward box mask, as the installers apply it
        m = torch.stack([O.box_mask(H, W, int(dx), int(dy)) for dx, dy, _ in sh.tolist()])
        m = m.repeat_interleave(B, 0)[:, None]
        k = torch.where(m > 0, k, torch.full_like(k, -math.inf if logw else 0.0))
    return k.to(dtype)


@pytest.mark.parametrize("dtype,B,C,Cw,H,W,R,logw", [
    (torch.float32, 2, 1, 1, 40, 48, 5, True),       # NECTR shape family
    (torch.float32, 2, 1, 1, 40, 48, 5, False),
    (torch.bfloat16, 2, 1, 1, 37, 64, 5, True),      # NECTR bf16 model
    (torch.float32, 1, 1, 1, 33, 76, 2, True),
    (torch.float16, 1, 1, 1, 30, 80, 10, False),
    (torch.bfloat16, 1, 3, 1, 31, 72, 2, False),     # NeKDe, one head over C = 3
    (torch.float32, 1, 3, 1, 20, 36, 3, True),
    (torch.float32, 1, 2, 2, 22, 40, 5, False),      # per-channel keys
    (torch.float16, 1, 3, 3, 18, 24, 2, True),
    (torch.float32, 1, 1, 1, 9, 12, 5, True),        # image smaller than the window box
    (torch.bfloat16, 1, 1, 1, 64, 256, 10, True),
])
def test_norm_mirror_matches_oracle(dtype, B, C, Cw, H, W, R, logw):
    torch.manual_seed(R * 11 + H)
    sh = T(O.halfplane_shifts(R))
    x = torch.rand(B, C, H, W).to(dtype)
    k = keys(len(sh), B, Cw, H, W, logw, dtype, sh)
    D, L = run(x, k, sh, logw)
    Dr, Lr = ref(x, k, sh, logw)
    close(D, Dr)
    close(L, Lr)


def test_norm_mirror_unmasked_forward_keys():
    """Forward keys not premasked (the kernel uses them as given) and a
    large common offset (the lazy reference moves)."""
    torch.manual_seed(2)
    sh = T(O.halfplane_shifts(3))
    x = torch.randn(1, 1, 24, 32)
    k = keys(len(sh), 1, 1, 24, 32, True, torch.float32, premask=False) + 2000.0
    D, L = run(x, k, sh, True)
    Dr, Lr = ref(x, k, sh, True)
    close(D, Dr)
    close(L, Lr, 2e-4)   # |log_C| ~ 2000: relative 1e-7


def test_norm_mirror_special_values():
    torch.manual_seed(5)
    sh = T(O.halfplane_shifts(2))
    S = len(sh)
    x = torch.rand(1, 1, 16, 32)
    lw = torch.randn(S, 1, 16, 32)
    lw[:, :, 0, 0] = -math.inf           # no live forward key at (0, 0) ...
    lw[:, :, 0:3, 0:3] = -math.inf       # ... nor mirror source around it
    lw[3, 0, 5, 5] = math.nan            # NaN key poisons (5, 5) and its mirror target
    lw[7, 0, 9, 9] = math.inf
    lw[:, :, 12, 3] += 10_000.0
    D, L = run(x, lw, sh, True)
    Dr, Lr = ref(x, lw, sh, True)
    close(D, Dr)
    close(L, Lr)
    assert D[0, 0, 0, 0] == 0 and L[0, 0, 0, 0] == -math.inf
    assert math.isnan(D[0, 0, 5, 5]) and math.isnan(L[0, 0, 9, 9])
    with pytest.raises(ValueError, match=r"not NaN or \+inf"):
        run(x, lw, sh, True, validate=True)


def test_norm_mirror_positive_extremes():
    torch.manual_seed(6)
    sh = T(O.halfplane_shifts(3))
    S = len(sh)
    x = torch.rand(1, 1, 16, 32)
    w = torch.rand(S, 1, 16, 32)
    w[:, :, 1, 1] = 1e38                 # reference test: huge finite weights
    w[:, :, 8, 8] = 0.0                  # zero weights around (8, 8)
    w[::3, :, 3, 3] = 1e-42              # subnormal weights
    w[5, :, 4, 4] = 3e38
    D, L = run(x, w, sh, False)
    Dr, Lr = ref(x, w, sh, False)
    close(D, Dr)
    close(L, Lr)
    w[4, 0, 7, 7] = -1.0
    D, L = run(x, w, sh, False)
    assert math.isnan(D[0, 0, 7, 7]) and math.isnan(L[0, 0, 7, 7])
    with pytest.raises(ValueError, match="nonnegative"):
        run(x, w, sh, False, validate=True)


def test_norm_mirror_gradients_unchanged():
    """The backward (general kernel) consumes the tiled forward's D, log_C."""
    torch.manual_seed(8)
    sh = T(O.halfplane_shifts(2))
    S = len(sh)
    x = torch.randn(1, 1, 12, 16, dtype=torch.float32)
    k = torch.randn(S, 1, 12, 16)
    xc = x.cuda().requires_grad_(True)
    kc = k.cuda().requires_grad_(True)
    D, L = nsc.normalized_accumulate_uz(xc, kc, sh, log_weights=True,
                                        return_log_degree=True)
    gD, gL = torch.randn_like(x), torch.randn_like(x)
    (D * gD.cuda() + L * gL.cuda()).sum().backward()
    Dr, Lr = O.normalized_accumulate_uz(x, k, sh, True)
    gx, gw = O.normalized_accumulate_uz_backward(x, k, Dr, Lr, gD, gL, sh, True)
    close(xc.grad.cpu(), gx, 1e-4)
    close(kc.grad.cpu(), gw, 1e-4)
