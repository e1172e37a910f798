"""GPU parity of the accumulate_uz backward with the tiled grad_w and
grad_x kernels (csrc/accumulate_gw.cu) against the oracle, and against the general
kernel (NSC_DISABLE_FAST=1 declines every tiled path).  Tolerance: fp32
rtol/atol 1e-4 on gradients of sums of up to 2S products; fp16 / bf16
grad_w is compared after rounding the oracle to the same storage."""

import pytest
import torch

import neural_shift_cuda_b200 as nsc
from oracle import nsc_oracle as O

pytestmark = pytest.mark.gpu


def _grads(x, w, sh, gU, gZ, dev):
    xc = x.to(dev).requires_grad_(True)
    wc = w.to(dev).requires_grad_(True)
    U, Z = nsc.accumulate_uz(xc, wc, sh)
    gx, gw = torch.autograd.grad((U, Z), (xc, wc), (gU.to(dev), gZ.to(dev)))
    return gx.cpu(), gw.cpu()


@pytest.mark.parametrize("dtype,C,Cw,H,W,table", [
    (torch.float16, 3, 1, 40, 256, ("half", 10)),     # configs[4] family
    (torch.float32, 3, 1, 23, 132, ("half", 3)),      # partial tiles
    (torch.bfloat16, 1, 1, 17, 64, ("half", 5)),
    (torch.float32, 2, 2, 20, 36, ("half", 2)),       # per-channel weights
    (torch.float16, 3, 3, 9, 40, ("window", 4)),      # full window, H < halo
    (torch.float32, 1, 1, 30, 128, ("window", 6)),
    (torch.float32, 3, 1, 12, 16, ("half", 12)),      # image narrower than a tile
    (torch.float16, 3, 1, 12, 16, ("half", 12)),      # weight rows wrap twice
    (torch.bfloat16, 3, 1, 19, 136, ("window", 6)),   # negative dy
    (torch.float16, 1, 1, 33, 200, ("half", 4)),      # partial tiles
    (torch.float16, 1, 1, 9, 12, ("half", 2)),
])
def test_tiled_grad_w_matches_oracle(cuda, monkeypatch, dtype, C, Cw, H, W, table):
    torch.manual_seed(H + W)
    kind, R = table
    rows = O.halfplane_shifts(R) if kind == "half" else O.window_shifts(R)
    sh = torch.tensor(rows)
    S = len(rows)
    B = 2
    x = torch.rand(B, C, H, W).to(dtype)
    w = torch.rand(S * B, Cw, H, W).to(dtype)
    gU, gZ = torch.randn(B, C, H, W), torch.randn(B, C, H, W)
    gx, gw = _grads(x, w, sh, gU, gZ, cuda)
    gxr, gwr = O.accumulate_uz_backward(x, w, gU, gZ, sh)
    if dtype == torch.float32:
        torch.testing.assert_close(gx, gxr, rtol=1e-4, atol=1e-4)
    else:   # grad_x is returned in x's storage dtype
        torch.testing.assert_close(gx.float(), gxr.to(dtype).float(), rtol=1e-2, atol=1e-2)
    if dtype == torch.float32:
        torch.testing.assert_close(gw, gwr, rtol=1e-4, atol=1e-4)
    else:   # one rounding to the weight storage: within one ulp of it
        torch.testing.assert_close(gw.float(), gwr.to(dtype).float(),
                                   rtol=1e-2, atol=1e-2)
    monkeypatch.setenv("NSC_DISABLE_FAST", "1")
    gx2, gw2 = _grads(x, w, sh, gU, gZ, cuda)
    tol = 1e-4 if dtype == torch.float32 else 1e-2   # fp16 / bf16: one rounding apart
    torch.testing.assert_close(gx.float(), gx2.float(), rtol=tol, atol=tol)
    torch.testing.assert_close(gw.float(), gw2.float(),
                               rtol=1e-4 if dtype == torch.float32 else 1e-2,
                               atol=1e-4 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("dtype,C,H,W,R", [
    (torch.float16, 3, 40, 256, 10),
    (torch.float32, 3, 23, 132, 3),
    (torch.bfloat16, 1, 17, 64, 5),
])
def test_grad_w_half_plane_pattern_equals_bit_tests(cuda, monkeypatch, dtype, C, H, W, R):
    """The compile-time half-plane form of the grad_w kernel and its
    per-entry bit-test form perform the same operations: equal bit for bit."""
    torch.manual_seed(R)
    sh = torch.tensor(O.halfplane_shifts(R))
    S, B = sh.shape[0], 2
    x = torch.rand(B, C, H, W).to(dtype)
    w = torch.rand(S * B, 1, H, W).to(dtype)
    gU, gZ = torch.randn(B, C, H, W), torch.randn(B, C, H, W)
    _, gw = _grads(x, w, sh, gU, gZ, cuda)
    monkeypatch.setenv("NSC_GW_GENERIC", "1")
    _, gw2 = _grads(x, w, sh, gU, gZ, cuda)
    assert torch.equal(gw, gw2)


@pytest.mark.parametrize("dtype,C,Cw,H,W,table,logw,periodic", [
    (torch.float32, 3, 1, 40, 64, ("window", 7), True, False),    # GASD family
    (torch.float32, 1, 1, 30, 48, ("half", 5), True, False),      # NECTR family
    (torch.float32, 3, 1, 23, 37, ("half", 3), False, False),     # positive, odd sizes
    (torch.float32, 2, 2, 17, 33, ("half", 2), False, True),      # per-channel, periodic
    (torch.bfloat16, 3, 1, 19, 40, ("window", 4), True, False),
    (torch.float16, 1, 1, 9, 12, ("half", 8), True, False),       # image smaller than halo
])
def test_tiled_normalized_backward_matches_oracle(cuda, monkeypatch, dtype, C, Cw, H, W,
                                                  table, logw, periodic):
    """The tiled normalized backward (csrc/normalized.cu, norm_bwd_tile_kernel)
    against the oracle's analytic gradients and the general kernel."""
    torch.manual_seed(H * W + C)
    kind, R = table
    rows = O.halfplane_shifts(R) if kind == "half" else O.window_shifts(R)
    sh = torch.tensor(rows)
    S, B = len(rows), 2
    x = torch.rand(B, C, H, W).to(dtype)
    raw = torch.randn(S * B, Cw, H, W)
    k = (2.0 * raw if logw else raw.exp()).to(dtype)
    gD, gL = torch.randn(B, C, H, W), torch.randn(B, C, H, W)

    def grads():
        xc = x.to(cuda).requires_grad_(True)
        kc = k.to(cuda).requires_grad_(True)
        D, L = nsc.normalized_accumulate_uz(xc, kc, sh, log_weights=logw,
                                            return_log_degree=True, validate=False,
                                            periodic_mirror=periodic)
        return [t.cpu() for t in torch.autograd.grad((D, L), (xc, kc),
                                                     (gD.to(cuda), gL.to(cuda)))]
    gx, gk = grads()
    rows_o = [(dx, dy, 2 if (inv and periodic) else int(inv)) for dx, dy, inv in rows]
    kk = k.expand(-1, C, -1, -1) if Cw == 1 else k
    Dr, Lr = O.normalized_accumulate_uz(x, kk, rows_o, logw)
    gxr, gkr = O.normalized_accumulate_uz_backward(x, k, Dr, Lr, gD, gL, rows_o, logw)
    tol = 2e-4 if dtype == torch.float32 else 2e-2
    torch.testing.assert_close(gx.float(), gxr.to(dtype).float(), rtol=tol, atol=tol)
    torch.testing.assert_close(gk.float(), gkr.to(dtype).float(), rtol=tol, atol=tol)
    monkeypatch.setenv("NSC_NORM_GENERIC", "1")
    gx2, gk2 = grads()
    torch.testing.assert_close(gx.float(), gx2.float(), rtol=tol, atol=tol)
    torch.testing.assert_close(gk.float(), gk2.float(), rtol=tol, atol=tol)


@pytest.mark.parametrize("dtype,C,Cw,H,W,table", [
    (torch.bfloat16, 3, 1, 70, 256, ("half", 10)),    # configs[4] family
    (torch.float16, 3, 1, 45, 136, ("half", 5)),      # partial tiles
    (torch.float32, 3, 1, 33, 72, ("half", 10)),      # fp32 weights, W % 64 != 0
    (torch.float32, 1, 1, 61, 128, ("window", 6)),    # negative dy
    (torch.bfloat16, 2, 2, 31, 80, ("window", 4)),    # per-channel weights
    (torch.float16, 1, 1, 25, 32, ("half", 12)),      # image narrower than a tile
    (torch.float32, 3, 1, 13, 16, ("half", 2)),
])
def test_tma_grad_x_matches_oracle(cuda, monkeypatch, dtype, C, Cw, H, W, table):
    """The TMA grad_x kernel (csrc/accumulate_gx_tma.cuh + the border-band
    wrap kernel) must take these calls (NSC_REQUIRE_FAST makes a decline an
    error) and match the oracle and the earlier tiled kernel (NSC_GX_LEGACY).
    grad_x is computed in fp32 and returned in x's dtype: fp32 within 1e-4,
    fp16 / bf16 within one rounding of the fp32 oracle."""
    torch.manual_seed(3 * H + W)
    kind, R = table
    rows = O.halfplane_shifts(R) if kind == "half" else O.window_shifts(R)
    sh = torch.tensor(rows)
    S = len(rows)
    B = 2
    x = torch.rand(B, C, H, W).to(dtype)
    w = torch.rand(S * B, Cw, H, W).to(dtype)
    gU, gZ = torch.randn(B, C, H, W), torch.randn(B, C, H, W)
    monkeypatch.setenv("NSC_REQUIRE_FAST", "1")
    gx, _ = _grads(x, w, sh, gU, gZ, cuda)
    monkeypatch.delenv("NSC_REQUIRE_FAST")
    gxr, _ = O.accumulate_uz_backward(x, w, gU, gZ, sh)
    if dtype == torch.float32:
        torch.testing.assert_close(gx, gxr, rtol=1e-4, atol=1e-4)
    else:
        torch.testing.assert_close(gx.float(), gxr.to(dtype).float(), rtol=1e-2, atol=1e-2)
    monkeypatch.setenv("NSC_GX_LEGACY", "1")
    gx2, _ = _grads(x, w, sh, gU, gZ, cuda)
    tol = 1e-4 if dtype == torch.float32 else 1e-2
    torch.testing.assert_close(gx.float(), gx2.float(), rtol=tol, atol=tol)
