"""GPU parity of the tiled TMA forward of accumulate_uz (accumulate_fast.cu)
against the CPU oracle and against the generic kernel, including partial
tiles, both dy buckets, all three storage dtypes, band mode, and a
full-size (8192 x 8192, S = 221) property check.  fp32 tolerance 1e-5."""

import os

import pytest
import torch

import neural_shift_cuda_b200 as nsc
from neural_shift_cuda_b200 import _lib, bands
from oracle import nsc_oracle as O

pytestmark = pytest.mark.gpu


def T(rows):
    return torch.tensor(rows, dtype=torch.int64)


def _generic(fn, *a, **k):
    os.environ["NSC_DISABLE_FAST"] = "1"
    try:
        return fn(*a, **k)
    finally:
        del os.environ["NSC_DISABLE_FAST"]


def _w(S, B, Cw, H, W, sh, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.nn.functional.softplus(torch.randn(S * B, Cw, H, W, generator=g))
    return O.premasked_weights(w, sh, B).to(dtype)


CASES = [
    # (B, C, Cw, H, W, table, R, dtype)
    (1, 3, 1, 64, 256, "half", 10, torch.float16),
    (2, 3, 1, 37, 136, "half", 3, torch.bfloat16),
    (1, 1, 1, 50, 72, "half", 5, torch.float32),
    (2, 2, 2, 33, 20, "window", 2, torch.float32),
    (1, 3, 3, 40, 64, "window", 4, torch.float16),
    (1, 3, 1, 19, 48, "window", 7, torch.bfloat16),
    (1, 1, 1, 24, 16, "half", 12, torch.float32),
]


@pytest.mark.parametrize("case", CASES)
def test_fast_matches_oracle_and_generic(cuda, case):
    B, C, Cw, H, W, table, R, dt = case
    rows = O.halfplane_shifts(R) if table == "half" else O.window_shifts(R)
    sh = T(rows)
    g = torch.Generator().manual_seed(1)
    x = torch.rand(B, C, H, W, generator=g).to(dt)
    w = _w(len(rows), B, Cw, H, W, sh, dt, 2)
    os.environ["NSC_REQUIRE_FAST"] = "1"   # fail if the tiled path declines
    try:
        U, Z = nsc.accumulate_uz(x.to(cuda), w.to(cuda), sh)
    finally:
        del os.environ["NSC_REQUIRE_FAST"]
    Ug, Zg = _generic(nsc.accumulate_uz, x.to(cuda), w.to(cuda), sh)
    Ur, Zr = O.accumulate_uz(x, w.expand(-1, C, -1, -1) if Cw == 1 else w, sh)
    torch.testing.assert_close(U.cpu(), Ur, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(Z.cpu(), Zr, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(U, Ug, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(Z, Zg, rtol=1e-5, atol=1e-5)
    assert _lib.wait_timeouts() == 0


def test_fast_nonfinite_x_stays_out_of_masked_mirror(cuda):
    """The mirror term never reads outside the image: an inf in x must not
    leak into outputs through a masked (zero) mirror weight."""
    B, C, H, W, R = 1, 1, 32, 64, 3
    rows = O.halfplane_shifts(R)
    sh = T(rows)
    x = torch.rand(B, C, H, W)
    x[0, 0, 0, 5] = float("inf")
    w = _w(len(rows), B, C, H, W, sh, torch.float32, 3)
    U, Z = nsc.accumulate_uz(x.to(cuda), w.to(cuda), sh)
    Ug, Zg = _generic(nsc.accumulate_uz, x.to(cuda), w.to(cuda), sh)
    assert torch.equal(torch.isinf(U), torch.isinf(Ug))
    fin = torch.isfinite(Ug)
    torch.testing.assert_close(U[fin], Ug[fin], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("nb", [2, 4])
def test_fast_band_split(cuda, nb):
    B, C, H, W, R = 1, 3, 96, 128, 4
    rows = O.halfplane_shifts(R)
    sh = T(rows)
    x = torch.rand(B, C, H, W, device=cuda).half()
    w = _w(len(rows), B, 1, H, W, sh, torch.float16, 4).to(cuda)
    U, Z = nsc.accumulate_uz(x, w, sh)
    Ub, Zb = bands.accumulate_uz_banded_local(x, w, sh, nb)
    torch.testing.assert_close(Ub, U, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(Zb, Z, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("B,C,Cw,W,R,dtype,nb", [
    (2, 3, 3, 100, 3, torch.float32, 3),      # per-channel weights, general band path
    (1, 5, 1, 72, 6, torch.bfloat16, 2),      # channel-shared, C > 4, two channel groups
    (2, 2, 1, 160, 10, torch.float16, 4),     # R = 10 strips, 64-column blocks + ragged
])
def test_band_edges_shapes(cuda, B, C, Cw, W, R, dtype, nb):
    """Edge strips across images, channel groups, widths that are not a
    multiple of the kernel's 64-column block, and every storage dtype: the
    banded result equals the unsplit op."""
    H = 24 * nb
    rows = O.halfplane_shifts(R)
    sh = T(rows)
    g = torch.Generator().manual_seed(B * 100 + W)
    x = torch.rand(B, C, H, W, generator=g).to(dtype).to(cuda)
    w = _w(len(rows), B, Cw, H, W, sh, dtype, W).to(cuda)
    U, Z = nsc.accumulate_uz(x, w, sh)
    Ub, Zb = bands.accumulate_uz_banded_local(x, w, sh, nb)
    torch.testing.assert_close(Ub, U, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(Zb, Z, rtol=1e-5, atol=1e-5)


def test_fullsize_config5_properties(cuda):
    """BASELINE configs[4] at full size: x fp16 (1,3,8192,8192), R=10
    (S=221), channel-shared fp16 weights.  With x = 1 every product is the
    weight itself, so U == Z bit for bit (same order, same roundings); a
    1-strip crop checked against the oracle pins the values."""
    H = W = 8192
    R = 10
    rows = O.halfplane_shifts(R)
    S = len(rows)
    sh = T(rows)
    free, _ = torch.cuda.mem_get_info()
    if free < 40e9:
        pytest.skip("needs ~40 GB of free device memory")
    w = torch.empty(S, 1, H, W, dtype=torch.float16, device=cuda)
    gen = torch.Generator(device=cuda).manual_seed(0)
    r_idx = torch.arange(H, device=cuda)
    for s, (dx, dy, _) in enumerate(rows):
        p = torch.nn.functional.softplus(
            torch.randn(H, W, generator=gen, device=cuda))
        m = (((r_idx + dx >= 0) & (r_idx + dx < H))[:, None]
             & ((r_idx + dy >= 0) & (r_idx + dy < W))[None, :])
        w[s, 0] = (p * m).half()
        del p, m
    ones = torch.ones(1, 3, H, W, dtype=torch.float16, device=cuda)
    U, Z = nsc.accumulate_uz(ones, w, sh)
    assert torch.equal(U, Z)
    assert torch.isfinite(Z).all()
    del U, Z
    x = torch.rand(1, 3, H, W, generator=gen, device=cuda).half()
    U, Z = nsc.accumulate_uz(x, w, sh)
    # oracle on the 48 x 48 corner block (its result is exact for rows and
    # columns >= R from the crop edge; the corner also exercises the image
    # border: circular x and masked mirror terms)
    hh = 48
    xc = x[:, :, :hh, :hh].float().cpu()
    wc = w[:, :, :hh, :hh].float().cpu()
    # circular x of the full image: wrap the crop with the image's last rows
    # and columns so the oracle sees the same neighbours.
    xfull_rows = torch.cat([x[:, :, -R:, :].float().cpu(),
                            x[:, :, :hh + R, :].float().cpu()], 2)
    xwin = torch.cat([xfull_rows[..., -R:], xfull_rows[..., :hh + R]], 3)
    wpad = torch.zeros(S, 1, hh + 2 * R, hh + 2 * R)
    wpad[:, :, R:, R:] = w[:, :, :hh + R, :hh + R].float().cpu()
    Uo, Zo = O.accumulate_uz(xwin, wpad.expand(-1, 3, -1, -1), sh)
    inner = (slice(None), slice(None), slice(R, hh), slice(R, hh))
    torch.testing.assert_close(U[:, :, :hh - R, :hh - R].cpu(), Uo[inner],
                               rtol=1e-5, atol=1e-4)
    torch.testing.assert_close(Z[:, :, :hh - R, :hh - R].cpu(), Zo[inner],
                               rtol=1e-5, atol=1e-4)
    del xc, wc
    assert _lib.wait_timeouts() == 0


@pytest.mark.parametrize("overlap", [False, True])
@pytest.mark.parametrize("padded", [False, True])
def test_banded_single_rank_process_group(cuda, padded, overlap):
    """accumulate_uz_banded through a one-rank process group: the halo is
    the band's own circular wrap and no strips travel; the result equals
    the unsplit op (plain and padded x buffers)."""
    import os
    import torch.distributed as dist
    from neural_shift_cuda_b200 import bands
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29561")
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        torch.manual_seed(4)
        R = 3
        sh = T(O.halfplane_shifts(R))
        S = len(sh)
        x = torch.rand(1, 3, 40, 64, dtype=torch.float16)
        w = torch.rand(S, 1, 40, 64, dtype=torch.float16)
        U0, Z0 = nsc.accumulate_uz(x.to(cuda), w.to(cuda), sh)
        xb = x.to(cuda)
        if padded:
            xp = torch.full((1, 3, 40 + 2 * R, 64), float("nan"), dtype=x.dtype, device=cuda)
            xp[:, :, R:R + 40] = xb
            xb = xp
        U, Z = bands.accumulate_uz_banded(xb, w.to(cuda), sh, 40, padded=padded,
                                          overlap=overlap)
        torch.testing.assert_close(U, U0, rtol=1e-6, atol=1e-5)
        torch.testing.assert_close(Z, Z0, rtol=1e-6, atol=1e-5)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dtype,R,Hb", [(torch.float16, 10, 100), (torch.float32, 3, 37),
                                       (torch.bfloat16, 5, 10)])
def test_band_rows_pieces_equal_band_forward(cuda, dtype, R, Hb):
    """nsc_accumulate_uz_band_rows_fwd: interior rows with a capped grid plus
    the two border pieces reproduce the whole band forward exactly."""
    from neural_shift_cuda_b200 import bands
    torch.manual_seed(9)
    sh = T(O.halfplane_shifts(R))
    S = len(sh)
    Hg, W, row0 = 4 * Hb, 128, Hb
    x = torch.rand(1, 3, Hg, W).to(dtype).to(cuda)
    w = torch.rand(S, 1, Hg, W).to(dtype).to(cuda)
    xe = bands.x_ext_from_full(x, row0, Hb, R)
    wb = w[:, :, row0:row0 + Hb].contiguous()
    U0, Z0 = bands.band_forward_cuda(xe, wb, sh, row0, Hg)
    U = torch.full_like(U0, float("nan"))
    Z = torch.full_like(Z0, float("nan"))
    bands.band_rows_cuda(xe, wb, sh, row0, Hg, R, Hb - R, U, Z, max_ctas=100)
    bands.band_rows_cuda(xe, wb, sh, row0, Hg, 0, R, U, Z)
    bands.band_rows_cuda(xe, wb, sh, row0, Hg, Hb - R, Hb, U, Z)
    assert torch.equal(U, U0) and torch.equal(Z, Z0)
