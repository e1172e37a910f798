"""GPU parity of the tiled normalized_accumulate_uz forward
(csrc/normalized_fast.cuh) against the CPU oracle.

NSC_REQUIRE_FAST makes the C entry point fail instead of falling back to
the general kernel, so every case here runs the tiled kernel.  Shapes cover
partial tiles in both directions, planes smaller than the halo (wrap more
than once), both dy buckets, per-channel and channel-broadcast keys, log
and positive modes and the special key values of the reference contract.
Tolerance: fp32 rtol/atol 1e-5 (the reference's fp32 bar).
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


@pytest.mark.parametrize("dtype,B,C,Cw,H,W,R,logw", [
    (torch.bfloat16, 2, 3, 1, 37, 264, 7, True),     # configs[2] shape family
    (torch.bfloat16, 1, 3, 1, 16, 128, 7, False),
    (torch.float32, 1, 2, 2, 20, 36, 3, False),      # per-channel keys, K=4
    (torch.float32, 2, 1, 1, 33, 68, 4, True),
    (torch.float16, 1, 1, 1, 9, 40, 8, True),        # H < halo: rows wrap twice
    (torch.float16, 1, 3, 3, 18, 24, 2, True),
])
def test_norm_fast_matches_oracle(dtype, B, C, Cw, H, W, R, logw):
    torch.manual_seed(R * 7 + H)
    sh = T(O.window_shifts(R))
    S = len(sh)
    x = torch.rand(B, C, H, W).to(dtype)
    if logw:
        k = (3.0 * torch.randn(S * B, Cw, H, W)).to(dtype)
    else:
        k = torch.nn.functional.softplus(torch.randn(S * B, Cw, H, W)).to(dtype)
    D, L = run(x, k, sh, logw)
    Dr, Lr = ref(x, k, sh, logw)
    close(D, Dr)
    close(L, Lr)


def test_norm_fast_random_table_order():
    """Table rows in an arbitrary order and a sparse window: the weight
    plane of every (dx, dy) follows its row, not the compute order."""
    torch.manual_seed(3)
    rows = [(dx, dy, 0) for dx in range(-5, 6) for dy in range(-6, 7) if (dx * 3 + dy) % 4]
    perm = torch.randperm(len(rows)).tolist()
    sh = T([rows[i] for i in perm])
    S = len(sh)
    x = torch.randn(1, 3, 30, 64)
    k = 2.0 * torch.randn(S, 1, 30, 64)
    D, L = run(x, k, sh, True)
    Dr, Lr = ref(x, k, sh, True)
    close(D, Dr)
    close(L, Lr)


def test_norm_fast_special_values():
    torch.manual_seed(5)
    sh = T(O.window_shifts(2))
    S = len(sh)
    x = torch.rand(1, 1, 16, 32)
    lw = torch.randn(S, 1, 16, 32)
    lw[:, :, 0, 0] = -math.inf           # no live key
    lw[3, 0, 5, 5] = math.nan            # NaN key poisons the pixel
    lw[7, 0, 9, 9] = math.inf            # +inf key too
    lw[:, :, 12, 3] += 10_000.0          # large common offset
    lw[::2, :, 2, 20] = -math.inf        # half the keys masked
    D, L = run(x, lw, sh, True)
    Dr, Lr = ref(x, lw, sh, True)
    close(D, Dr)
    close(L, Lr)
    assert D[0, 0, 0, 0] == 0 and L[0, 0, 0, 0] == -math.inf
    assert math.isnan(D[0, 0, 5, 5]) and math.isnan(L[0, 0, 9, 9])
    with pytest.raises(ValueError, match=r"not NaN or \+inf"):
        run(x, lw, sh, True, validate=True)


def test_norm_fast_positive_extremes():
    torch.manual_seed(6)
    sh = T(O.window_shifts(3))
    S = len(sh)
    x = torch.rand(1, 1, 16, 32)
    w = torch.rand(S, 1, 16, 32)
    w[:, :, 1, 1] = 1e38                 # reference test: huge finite weights
    w[:, :, 2, 2] = 0.0                  # no live key
    w[::3, :, 3, 3] = 1e-42              # subnormal weights
    w[5, :, 4, 4] = 3e38
    D, L = run(x, w, sh, False)
    Dr, Lr = ref(x, w, sh, False)
    close(D, Dr)
    close(L, Lr)
    assert D[0, 0, 2, 2] == 0 and L[0, 0, 2, 2] == -math.inf
    w[4, 0, 7, 7] = -1.0
    D, L = run(x, w, sh, False)
    assert math.isnan(D[0, 0, 7, 7]) and math.isnan(L[0, 0, 7, 7])
    with pytest.raises(ValueError, match="nonnegative"):
        run(x, w, sh, False, validate=True)
