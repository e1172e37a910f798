"""Parity at BASELINE.json's own shapes (configs[1..3]).

Full-size runs compare the tiled kernels with the general one-pixel kernels
on the GPU (each path is separately pinned to the oracle on small cases),
and one image of each batch with the CPU oracle, which is exact for a batch
crop because images are independent.  Tolerances: fp32 rtol/atol 1e-5
(the reference's fp32 bar), 1e-4 where a long fp32 sum is compared with a
differently ordered one."""

import pytest
import torch

import neural_shift_cuda_b200 as nsc
from oracle import nsc_oracle as O

pytestmark = pytest.mark.gpu


def _seeded(shape, seed, fn):
    g = torch.Generator().manual_seed(seed)
    return fn(g, shape)


def test_config3_gasd_normalized_full_size(cuda, monkeypatch):
    """x bf16 (16, 3, 512, 512), logits N(0, 9) bf16 shared by
    the 3 channels, full window R = 7 (S = 225), log weights."""
    B, C, H, W, R = 16, 3, 512, 512, 7
    rows = O.window_shifts(R)
    S = len(rows)
    sh = torch.tensor(rows)
    x = _seeded((B, C, H, W), 0, lambda g, s: torch.rand(s, generator=g)).bfloat16()
    lg = _seeded((S * B, 1, H, W), 1,
                 lambda g, s: 3.0 * torch.randn(s, generator=g)).bfloat16()
    xc, lc = x.to(cuda), lg.to(cuda)
    monkeypatch.setenv("NSC_REQUIRE_FAST", "1")
    D, L = nsc.normalized_accumulate_uz(xc, lc, sh, log_weights=True,
                                        return_log_degree=True, validate=False)
    monkeypatch.delenv("NSC_REQUIRE_FAST")
    monkeypatch.setenv("NSC_NORM_GENERIC", "1")
    Dg, Lg = nsc.normalized_accumulate_uz(xc, lc, sh, log_weights=True,
                                          return_log_degree=True, validate=False)
    torch.testing.assert_close(D, Dg, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(L, Lg, rtol=1e-5, atol=1e-5)
    # image 5 against the oracle (the shift-major stack's rows of image 5)
    b = 5
    lb = lg.reshape(S, B, 1, H, W)[:, b]
    Dr, Lr = O.normalized_accumulate_uz(x[b:b + 1], lb.expand(-1, C, -1, -1), sh, True)
    torch.testing.assert_close(D[b:b + 1].cpu(), Dr, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(L[b:b + 1].cpu(), Lr, rtol=1e-5, atol=1e-5)


def test_config4_nkd_metropolis_full_size(cuda, monkeypatch):
    """x fp32 (16, 3, 512, 512), w_half sigmoid(N(0, 1))
    (16, 61, 1, 512, 512) over C = 3, R = 5 half plane, use_box, forward and
    backward with grad N(0, 1)."""
    B, C, H, W, R = 16, 3, 512, 512, 5
    rows = O.halfplane_shifts(R)
    S = len(rows)
    x = _seeded((B, C, H, W), 2, lambda g, s: torch.rand(s, generator=g))
    wh = _seeded((B, S, 1, H, W), 3, lambda g, s: torch.sigmoid(torch.randn(s, generator=g)))
    gy = _seeded((B, C, H, W), 4, lambda g, s: torch.randn(s, generator=g))

    def run():
        w = wh.to(cuda).requires_grad_(True)
        xi = x.to(cuda).requires_grad_(True)
        Wx, dh = nsc.metropolis_aggregate(w, xi, rows, True, 1e-6)
        gw, gx = torch.autograd.grad(Wx, (w, xi), gy.to(cuda))
        return Wx.detach(), dh.detach(), gw, gx

    tiled = run()
    monkeypatch.setenv("NSC_METRO_GENERIC", "1")
    general = run()
    for a, b in zip(tiled, general):
        torch.testing.assert_close(a, b, rtol=1e-4, atol=1e-4)
    # image 9 against the oracle (values and gradients)
    b = 9
    Wr, dr = O.metropolis_aggregate(wh[b:b + 1].double(), x[b:b + 1].double(), rows,
                                    True, 1e-6)
    torch.testing.assert_close(tiled[0][b:b + 1].cpu().double(), Wr, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(tiled[1][b:b + 1].cpu().double(), dr, rtol=1e-5, atol=1e-5)
    gwr, gxr = O.metropolis_aggregate_grad(wh[b:b + 1].double(), x[b:b + 1].double(),
                                           rows, True, 1e-6, gy[b:b + 1].double(),
                                           torch.zeros(1, C, H, W, dtype=torch.float64))
    # The gradient of max(d(p), d(p + delta)) jumps where the two degrees
    # tie; fp32 and fp64 resolve near-ties differently, so a few elements
    # (< 1e-4 of them) may differ by more than the fp32 tolerance.
    for mine, ref in ((tiled[2][b:b + 1].cpu().double(), gwr),
                      (tiled[3][b:b + 1].cpu().double(), gxr)):
        bad = ~torch.isclose(mine, ref, rtol=1e-4, atol=1e-4)
        assert bad.double().mean().item() < 1e-4
        assert (mine - ref).abs().max().item() < 1e-2


def test_config2_nectr_unfused_path_full_size(cuda):
    """configs[1] through the unfused patched path (pair_gather, the head on
    the pair batch, the tiled normalized kernel with mirror terms) against
    the fused kernel at B = 8, 1 x 256 x 256, R = 5, latent 16."""
    from types import SimpleNamespace
    from neural_shift_cuda_b200 import integration as I
    from neural_shift_cuda_b200.integration.nectr_models1 import NECTR_denoiser
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        args = SimpleNamespace(model_type="concat", residual_depth=2, proj_depth=1,
                               latent_dim=16, patch_rad=1, output_activation="exp",
                               window_rad=5, in_channel=1, blind=True)
        cls = type("NECTRCfg2", (NECTR_denoiser,), {})
        I.install_cuda_shift_nectr(cls)
        torch.manual_seed(0)
        m = cls(args).to(cuda)
        x = _seeded((8, 1, 256, 256), 5,
                    lambda g, s: torch.rand(s, generator=g)
                    + (25 / 255) * torch.randn(s, generator=g)).to(cuda)
        with torch.no_grad():
            D, Z = m(x)
            m.use_nectr_fused = False
            Du, Zu = m(x)
        torch.testing.assert_close(Du, D, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(Zu, Z, rtol=1e-4, atol=1e-5)
    finally:
        torch.backends.cudnn.allow_tf32 = prev
