"""GPU parity: every op of neural_shift_cuda_b200 (through the C ABI of
libnsc_b200.so) against the CPU oracle and the reference's golden fixtures.

Tolerances (the reference's own, tests/test_*.py): gathers and masks
bit-exact; fp32 rtol/atol 1e-5; fp64 1e-10 forward and 1e-9 gradients
(normalized), 1e-12-class for plain sums.
"""

import itertools
import math
import os

import pytest
import torch

import neural_shift_cuda_b200 as nsc
from oracle import nsc_oracle as O

pytestmark = pytest.mark.gpu

GOLD = torch.load(os.path.join(os.path.dirname(__file__), "golden",
                               "golden_ops.pt"), weights_only=False)


def T(rows):
    return torch.tensor(rows, dtype=torch.int64)


def close(a, b, rtol, atol):
    torch.testing.assert_close(a.detach().cpu().to(b.dtype), b, rtol=rtol,
                               atol=atol, equal_nan=True)


# ---------------------------------------------------------------------------
# gathers
# ---------------------------------------------------------------------------

GSHAPES = [(1, 8, 16, 16), (2, 16, 31, 29), (4, 32, 64, 64)]


@pytest.mark.parametrize("shape,R", list(itertools.product(GSHAPES, [1, 2, 5])))
def test_gathers_bit_exact(cuda, shape, R):
    torch.manual_seed(0)
    g = torch.randn(*shape)
    sh = T(O.halfplane_shifts(R))
    out, mask = nsc.shift_gather(g.to(cuda), sh.to(cuda))
    ro, rm = O.shift_gather(g, sh)
    assert torch.equal(out.cpu(), ro) and torch.equal(mask.cpu(), rm)
    pr, pm = nsc.pair_gather(g.to(cuda), sh)
    rp, rpm = O.pair_gather(g, sh)
    assert torch.equal(pr.cpu(), rp) and torch.equal(pm.cpu(), rpm)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16,
                                   torch.float64])
def test_gathers_other_dtypes(cuda, dtype):
    torch.manual_seed(1)
    g = torch.randn(2, 3, 13, 24).to(dtype)
    sh = T(O.window_shifts(2))[:, :2]
    out, mask = nsc.shift_gather(g.to(cuda), sh)
    ro, rm = O.shift_gather(g, sh)
    assert torch.equal(out.cpu(), ro) and torch.equal(mask.cpu(), rm)


@pytest.mark.parametrize("generic", [False, True])
@pytest.mark.parametrize("dtype,shape,rows", [
    (torch.float32, (2, 3, 37, 300), [(3, -5, 1), (-2, 7, 0), (0, 0, 1)]),
    (torch.float16, (1, 2, 5, 64), [(4, 9, 1), (-5, -3, 0), (5, 64, 1)]),
    (torch.bfloat16, (2, 1, 40, 520), [(dx, dy, 1) for dx in (-7, 0, 7) for dy in (-9, 1, 9)]),
    (torch.float64, (1, 2, 20, 18), [(1, 1, 1), (-3, 2, 0)]),
    (torch.float32, (1, 1, 64, 128), [(40, 3, 1), (0, -70, 1)]),   # halo too large: general kernel
])
def test_gathers_tiled_and_general(cuda, generic, dtype, shape, rows, monkeypatch):
    """Both forward kernels (halo-tiled and one-vector-per-thread) on ragged
    tiles, tiny planes (shifts wrapping more than a tile), every dtype."""
    if generic:
        monkeypatch.setenv("NSC_GATHER_GENERIC", "1")
    torch.manual_seed(2)
    g = torch.randn(*shape).to(dtype)
    sh = T(rows)
    for fn, ref in ((nsc.shift_gather, O.shift_gather), (nsc.pair_gather, O.pair_gather)):
        out, mask = fn(g.to(cuda), sh)
        ro, rm = ref(g, sh)
        assert torch.equal(out.cpu(), ro) and torch.equal(mask.cpu(), rm)


@pytest.mark.parametrize("pair", [False, True])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_gather_backward(cuda, pair, dtype):
    torch.manual_seed(2)
    B, C, H, W = 2, 3, 11, 13
    g = torch.randn(B, C, H, W, dtype=dtype)
    sh = T(O.halfplane_shifts(2))
    gc = g.to(cuda).requires_grad_(True)
    fn = nsc.pair_gather if pair else nsc.shift_gather
    out, _ = fn(gc, sh)
    go = torch.randn(out.shape, dtype=dtype)
    (out * go.to(cuda)).sum().backward()
    ref = (O.pair_gather_backward if pair else O.shift_gather_backward)(
        go, sh, B, C, H, W)
    tol = 1e-12 if dtype == torch.float64 else 1e-5
    close(gc.grad, ref, tol, tol)


def test_gather_gradcheck(cuda):
    torch.manual_seed(3)
    g = torch.randn(1, 2, 5, 6, dtype=torch.float64, device=cuda,
                    requires_grad=True)
    sh = T(O.halfplane_shifts(1))
    assert torch.autograd.gradcheck(lambda t: nsc.pair_gather(t, sh)[0], (g,))


@pytest.mark.parametrize("name", sorted(k for k in GOLD
                                        if k.startswith("shift_gather_")))
def test_gathers_golden(cuda, name):
    c = GOLD[name]
    out, mask = nsc.shift_gather(c["guide"].to(cuda), c["shifts"])
    assert torch.equal(out.cpu(), c["out"]) and torch.equal(mask.cpu(), c["mask"])
    pr, _ = nsc.pair_gather(c["guide"].to(cuda), c["shifts"])
    assert torch.equal(pr.cpu(), c["pair"])
    gg = c["guide"].to(cuda).requires_grad_(True)
    (nsc.pair_gather(gg, c["shifts"])[0] * c["pair_grad_out"].to(cuda)).sum().backward()
    close(gg.grad, c["pair_grad_guide"], 1e-12, 1e-12)


# ---------------------------------------------------------------------------
# accumulate_uz
# ---------------------------------------------------------------------------

def _weights(S, B, Cw, H, W, sh, dtype, gen=None):
    w = torch.nn.functional.softplus(torch.randn(S * B, Cw, H, W, generator=gen))
    return O.premasked_weights(w, sh, B).to(dtype)


ASHAPES = [(1, 3, 16, 16), (2, 3, 31, 29), (3, 6, 33, 47)]


@pytest.mark.parametrize("shape,R", list(itertools.product(ASHAPES, [1, 2, 4])))
def test_accumulate_forward_fp32(cuda, shape, R):
    B, C, H, W = shape
    torch.manual_seed(0)
    sh = T(O.halfplane_shifts(R))
    x = torch.randn(B, C, H, W)
    w = _weights(len(sh), B, C, H, W, sh, torch.float32)
    U, Z = nsc.accumulate_uz(x.to(cuda), w.to(cuda), sh.to(cuda))
    Ur, Zr = O.accumulate_uz(x, w, sh)
    assert U.dtype == torch.float32
    close(U, Ur, 1e-5, 1e-5)
    close(Z, Zr, 1e-5, 1e-5)


def test_accumulate_config1_shape(cuda):
    """Config 1 of the benchmark: x (2,1,128,128) U[0,1]+noise, R=3."""
    g = torch.Generator().manual_seed(0)
    B, C, H, W = 2, 1, 128, 128
    sh = T(O.halfplane_shifts(3))
    x = torch.rand(B, C, H, W, generator=g) + \
        (25 / 255) * torch.randn(B, C, H, W, generator=g)
    w = _weights(len(sh), B, C, H, W, sh, torch.float32, g)
    U, Z = nsc.accumulate_uz(x.to(cuda), w.to(cuda), sh)
    Ur, Zr = O.accumulate_uz(x, w, sh)
    close(U, Ur, 1e-5, 1e-5)
    close(Z, Zr, 1e-5, 1e-5)


@pytest.mark.parametrize("wdt", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("xdt", [torch.float16, torch.float32])
def test_accumulate_broadcast_and_half(cuda, wdt, xdt):
    torch.manual_seed(4)
    B, C, H, W, R = 2, 3, 24, 40, 3
    sh = T(O.halfplane_shifts(R))
    x = torch.rand(B, C, H, W).to(xdt)
    w = _weights(len(sh), B, 1, H, W, sh, wdt)
    # explicit (S*B, 1, H, W) and stride-0 expand both take the shared path
    U1, Z1 = nsc.accumulate_uz(x.to(cuda), w.to(cuda), sh)
    U2, Z2 = nsc.accumulate_uz(x.to(cuda), w.to(cuda).expand(-1, C, -1, -1), sh)
    Ur, Zr = O.accumulate_uz(x, w.expand(-1, C, -1, -1), sh)
    for U, Z in ((U1, Z1), (U2, Z2)):
        close(U, Ur, 1e-5, 1e-5)
        close(Z, Zr, 1e-5, 1e-5)


@pytest.mark.parametrize("R", [1, 3])
def test_accumulate_backward_fp64(cuda, R):
    torch.manual_seed(7)
    B, C, H, W = 2, 3, 13, 11
    sh = T(O.halfplane_shifts(R))
    x = torch.randn(B, C, H, W, dtype=torch.float64)
    w = O.premasked_weights(torch.randn(len(sh) * B, C, H, W,
                                        dtype=torch.float64), sh, B)
    xc = x.to(cuda).requires_grad_(True)
    wc = w.to(cuda).requires_grad_(True)
    U, Z = nsc.accumulate_uz(xc, wc, sh)
    gU, gZ = torch.randn_like(x), torch.randn_like(x)
    (U * gU.to(cuda) + Z * gZ.to(cuda)).sum().backward()
    gx, gw = O.accumulate_uz_backward(x, w, gU, gZ, sh)
    close(xc.grad, gx, 1e-10, 1e-10)
    close(wc.grad, gw, 1e-10, 1e-10)


def test_accumulate_backward_broadcast(cuda):
    torch.manual_seed(8)
    B, C, H, W = 1, 3, 12, 10
    sh = T(O.halfplane_shifts(2))
    x = torch.randn(B, C, H, W, dtype=torch.float64)
    w = O.premasked_weights(torch.rand(len(sh) * B, 1, H, W,
                                       dtype=torch.float64), sh, B)
    xc = x.to(cuda).requires_grad_(True)
    wc = w.to(cuda).requires_grad_(True)
    U, Z = nsc.accumulate_uz(xc, wc.expand(-1, C, -1, -1), sh)
    gU, gZ = torch.randn_like(x), torch.randn_like(x)
    (U * gU.to(cuda) + Z * gZ.to(cuda)).sum().backward()
    gx, gw = O.accumulate_uz_backward(x, w, gU, gZ, sh)
    close(xc.grad, gx, 1e-10, 1e-10)
    close(wc.grad, gw, 1e-10, 1e-10)


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-10),
                                       (torch.float32, 1e-4)])
@pytest.mark.parametrize("C", [5, 8])
@pytest.mark.parametrize("expand", [False, True])
def test_accumulate_backward_broadcast_many_channels(cuda, C, dtype, tol, expand):
    """A channel-shared weight with more channels than one thread's channel
    tile: grad_w is the sum over all C channels, written once per element."""
    torch.manual_seed(11)
    B, H, W = 2, 13, 11
    sh = T(O.halfplane_shifts(2))
    x = torch.randn(B, C, H, W, dtype=torch.float64)
    w = O.premasked_weights(torch.rand(len(sh) * B, 1, H, W,
                                       dtype=torch.float64), sh, B)
    xc = x.to(dtype).to(cuda).requires_grad_(True)
    wc = w.to(dtype).to(cuda).requires_grad_(True)
    U, Z = nsc.accumulate_uz(xc, wc.expand(-1, C, -1, -1) if expand else wc, sh)
    Ur, Zr = O.accumulate_uz(x, w, sh)
    close(U, Ur, tol, tol)
    close(Z, Zr, tol, tol)
    gU, gZ = torch.randn_like(x), torch.randn_like(x)
    (U * gU.to(dtype).to(cuda) + Z * gZ.to(dtype).to(cuda)).sum().backward()
    gx, gw = O.accumulate_uz_backward(x, w, gU, gZ, sh)
    close(xc.grad, gx, tol, tol)
    close(wc.grad, gw, tol, tol)


@pytest.mark.parametrize("R", [1, 2])
def test_accumulate_gradcheck(cuda, R):
    torch.manual_seed(0)
    B, C, H, W = 1, 2, 6, 5
    sh = T(O.halfplane_shifts(R))
    x = torch.randn(B, C, H, W, dtype=torch.float64, device=cuda,
                    requires_grad=True)
    w = O.premasked_weights(torch.randn(len(sh) * B, C, H, W,
                                        dtype=torch.float64), sh, B)
    w = w.to(cuda).requires_grad_(True)
    assert torch.autograd.gradcheck(
        lambda a, b: nsc.accumulate_uz(a, b, sh), (x, w), eps=1e-6, atol=1e-5)


@pytest.mark.parametrize("name", sorted(k for k in GOLD
                                        if k.startswith("accumulate_")))
def test_accumulate_golden(cuda, name):
    c = GOLD[name]
    xc = c["x"].to(cuda).requires_grad_(True)
    wc = c["w"].to(cuda).requires_grad_(True)
    U, Z = nsc.accumulate_uz(xc, wc, c["shifts"].to(cuda))
    tol = 1e-12 if c["x"].dtype == torch.float64 else 1e-5
    close(U, c["U"], tol, tol)
    close(Z, c["Z"], tol, tol)
    (U * c["gU"].to(cuda) + Z * c["gZ"].to(cuda)).sum().backward()
    close(xc.grad, c["gx"], tol, tol)
    close(wc.grad, c["gw"], tol, tol)


def test_accumulate_tiny_images_and_single_shift(cuda):
    """H, W smaller than the window, S = 1, R = 0 (circular wrap and mirror
    masks at every pixel)."""
    torch.manual_seed(5)
    for (B, C, H, W), rows in [((1, 1, 2, 3), O.halfplane_shifts(2)),
                               ((2, 2, 1, 1), [(0, 0, 0)]),
                               ((1, 3, 3, 2), O.window_shifts(1)),
                               ((1, 1, 5, 5), [(3, -2, 1)])]:
        sh = T(rows)
        x = torch.randn(B, C, H, W, dtype=torch.float64)
        w = torch.rand(len(rows) * B, C, H, W, dtype=torch.float64)
        U, Z = nsc.accumulate_uz(x.to(cuda), w.to(cuda), sh)
        Ur, Zr = O.accumulate_uz(x, w, sh)
        close(U, Ur, 1e-12, 1e-12)
        close(Z, Zr, 1e-12, 1e-12)


def test_accumulate_errors(cuda):
    x = torch.ones(1, 1, 4, 4, device=cuda)
    with pytest.raises(RuntimeError, match="weights must be"):
        nsc.accumulate_uz(x, torch.ones(2, 1, 4, 4, device=cuda), T([[0, 1, 1]]))
    with pytest.raises(RuntimeError, match="1 <= S <= 1024"):
        nsc.accumulate_uz(x, torch.ones(0, 1, 4, 4, device=cuda),
                          torch.zeros(0, 3, dtype=torch.int64))
    with pytest.raises(RuntimeError, match="exceeds the image extent"):
        nsc.accumulate_uz(x, torch.ones(1, 1, 4, 4, device=cuda), T([[9, 0, 0]]))


# ---------------------------------------------------------------------------
# row bands (single GPU emulation of the multi-GPU split)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("nb", [2, 3])
def test_band_split_matches_full(cuda, nb):
    from neural_shift_cuda_b200 import bands
    torch.manual_seed(6)
    B, C, H, W, R = 1, 3, 30, 20, 3
    sh = T(O.halfplane_shifts(R))
    x = torch.rand(B, C, H, W, device=cuda)
    w = _weights(len(sh), B, 1, H, W, sh, torch.float32).to(cuda)
    U, Z = nsc.accumulate_uz(x, w, sh)
    Ub, Zb = bands.accumulate_uz_banded_local(x, w, sh, nb)
    torch.testing.assert_close(Ub, U, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(Zb, Z, rtol=1e-5, atol=1e-5)


# ---------------------------------------------------------------------------
# normalized_accumulate_uz
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("log_weights", [False, True])
@pytest.mark.parametrize("table", ["window", "half"])
def test_normalized_fp64_and_grads(cuda, log_weights, table):
    torch.manual_seed(3)
    B, C, H, W = 1, 2, 8, 7
    sh = T(O.window_shifts(2) if table == "window" else O.halfplane_shifts(2))
    x = torch.randn(B, C, H, W, dtype=torch.double)
    raw = torch.randn(len(sh) * B, C, H, W, dtype=torch.double)
    w = raw if log_weights else raw.exp()
    xc = x.to(cuda).requires_grad_(True)
    wc = w.to(cuda).requires_grad_(True)
    D, L = nsc.normalized_accumulate_uz(xc, wc, sh.to(cuda),
                                        log_weights=log_weights,
                                        return_log_degree=True)
    Dr, Lr = O.normalized_accumulate_uz(x, w, sh, log_weights)
    close(D, Dr, 1e-10, 1e-10)
    close(L, Lr, 1e-10, 1e-10)
    gD, gL = torch.randn_like(x), torch.randn_like(x)
    (D * gD.to(cuda) + L * gL.to(cuda)).sum().backward()
    gx, gw = O.normalized_accumulate_uz_backward(x, w, Dr, Lr, gD, gL, sh,
                                                 log_weights)
    close(xc.grad, gx, 1e-9, 1e-9)
    close(wc.grad, gw, 1e-9, 1e-9)


@pytest.mark.parametrize("dtype,tol", [(torch.float64, 1e-9),
                                       (torch.float32, 1e-4)])
@pytest.mark.parametrize("C", [5, 8])
@pytest.mark.parametrize("log_weights", [False, True])
@pytest.mark.parametrize("expand", [False, True])
def test_normalized_backward_broadcast_many_channels(cuda, C, log_weights, dtype,
                                                     tol, expand):
    """normalized_accumulate_uz with channel-shared weights and C > 4:
    grad_w sums every channel's contribution."""
    torch.manual_seed(12)
    B, H, W = 2, 9, 10
    sh = T(O.halfplane_shifts(2))
    x = torch.randn(B, C, H, W, dtype=torch.float64)
    raw = torch.randn(len(sh) * B, 1, H, W, dtype=torch.float64)
    w = raw if log_weights else raw.exp()
    xc = x.to(dtype).to(cuda).requires_grad_(True)
    wc = w.to(dtype).to(cuda).requires_grad_(True)
    D, L = nsc.normalized_accumulate_uz(
        xc, wc.expand(-1, C, -1, -1) if expand else wc, sh,
        log_weights=log_weights, return_log_degree=True)
    Dr, Lr = O.normalized_accumulate_uz(x, w, sh, log_weights)
    close(D, Dr, tol, tol)
    close(L, Lr, tol, tol)
    gD, gL = torch.randn_like(x), torch.randn_like(x)
    (D * gD.to(dtype).to(cuda) + L * gL.to(dtype).to(cuda)).sum().backward()
    gx, gw = O.normalized_accumulate_uz_backward(x, w, Dr, Lr, gD, gL, sh,
                                                 log_weights)
    close(xc.grad, gx, tol, tol)
    close(wc.grad, gw, tol, tol)


@pytest.mark.parametrize("log_weights", [False, True])
def test_normalized_gradcheck(cuda, log_weights):
    torch.manual_seed(2)
    sh = T(O.window_shifts(1))
    x = torch.randn(1, 1, 4, 4, dtype=torch.double, device=cuda,
                    requires_grad=True)
    base = torch.randn(len(sh), 1, 4, 4, dtype=torch.double)
    w = (base if log_weights else base.exp()).to(cuda).requires_grad_(True)
    assert torch.autograd.gradcheck(
        lambda a, b: nsc.normalized_accumulate_uz(
            a, b, sh, log_weights=log_weights, return_log_degree=True),
        (x, w), eps=1e-6, atol=2e-5)


@pytest.mark.parametrize("name", sorted(k for k in GOLD if k.startswith("normalized_")))
def test_normalized_golden(cuda, name):
    c = GOLD[name]
    lw = bool(c.get("log_weights", name == "normalized_empty"))
    D, L = nsc.normalized_accumulate_uz(c["x"].to(cuda), c["w"].to(cuda),
                                        c["shifts"], log_weights=lw,
                                        return_log_degree=True)
    tol = 2e-6 if c["x"].dtype == torch.float32 else 1e-10
    close(D, c["D"], tol, tol)
    close(L, c["logC"], tol, tol)
    if "gD" in c:
        xc = c["x"].to(cuda).requires_grad_(True)
        wc = c["w_full"].to(cuda).requires_grad_(True)
        D, L = nsc.normalized_accumulate_uz(xc, wc, c["shifts"], log_weights=lw,
                                            return_log_degree=True)
        (D * c["gD"].to(cuda) + L * c["gL"].to(cuda)).sum().backward()
        for mine, gold in ((xc.grad, c["gx"]), (wc.grad, c["gw"])):
            ok = torch.isfinite(gold)
            close(mine.cpu()[ok], gold[ok], 1e-9, 1e-9)


def test_normalized_bf16_config3_like(cuda):
    """GASD-style: bf16 x and channel-shared bf16 logits, full window."""
    torch.manual_seed(9)
    B, C, H, W, R = 2, 3, 40, 36, 3
    sh = T(O.window_shifts(R))
    x = torch.rand(B, C, H, W).bfloat16()
    lg = (3.0 * torch.randn(len(sh) * B, 1, H, W)).bfloat16()
    D, L = nsc.normalized_accumulate_uz(x.to(cuda), lg.to(cuda), sh,
                                        log_weights=True,
                                        return_log_degree=True, validate=False)
    Dr, Lr = O.normalized_accumulate_uz(x, lg.expand(-1, C, -1, -1), sh, True)
    close(D, Dr, 1e-5, 1e-5)
    close(L, Lr, 1e-5, 1e-5)


def test_normalized_special_values(cuda):
    sh = T(O.halfplane_shifts(1))
    S = len(sh)
    x = torch.randn(1, 1, 4, 5, dtype=torch.float64)
    lw = torch.randn(S, 1, 4, 5, dtype=torch.float64)
    lw[:, :, 0, 0] = -math.inf          # empty row at (0, 0)
    lw[0, 0, 2, 2] = math.nan           # NaN key poisons its row
    D, L = nsc.normalized_accumulate_uz(x.cuda(), lw.cuda(), sh,
                                        log_weights=True,
                                        return_log_degree=True, validate=False)
    D, L = D.cpu(), L.cpu()
    assert D[0, 0, 0, 0] == 0 and L[0, 0, 0, 0] == -math.inf
    assert math.isnan(D[0, 0, 2, 2]) and math.isnan(L[0, 0, 2, 2])
    with pytest.raises(ValueError, match=r"not NaN or \+inf"):
        nsc.normalized_accumulate_uz(x.cuda(), lw.cuda(), sh, log_weights=True)
        nsc.check_validation()
    with pytest.raises(ValueError, match="nonnegative"):
        nsc.normalized_accumulate_uz(x.cuda(), -lw.abs().nan_to_num(1.0).cuda(),
                                     sh)
        nsc.check_validation()
    # valid weights leave nothing pending
    nsc.normalized_accumulate_uz(x.cuda(), lw.nan_to_num(0.0, posinf=0.0).cuda(),
                                 sh, log_weights=True)
    nsc.check_validation()


def test_normalized_offset_invariance(cuda):
    torch.manual_seed(1)
    sh = T(O.window_shifts(2))
    x = torch.randn(1, 2, 6, 5).cuda()
    lg = (10_000.0 + 3.0 * torch.randn(len(sh), 2, 6, 5)).cuda()
    d1, l1 = nsc.normalized_accumulate_uz(x, lg, sh, log_weights=True,
                                          return_log_degree=True)
    d2, l2 = nsc.normalized_accumulate_uz(x, lg + 5000.0, sh, log_weights=True,
                                          return_log_degree=True)
    torch.testing.assert_close(d1, d2, rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(l2 - l1, torch.full_like(l1, 5000.0), rtol=0,
                               atol=2e-3)


# ---------------------------------------------------------------------------
# metropolis_aggregate
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("name", sorted(k for k in GOLD if k.startswith("metropolis_")))
def test_metropolis_golden(cuda, name):
    c = GOLD[name]
    rows = [tuple(r) for r in c["shifts"].tolist()]
    wc = c["w_half"].to(cuda).requires_grad_(True)
    xc = c["img"].to(cuda).requires_grad_(True)
    Wx, dh = nsc.metropolis_aggregate(wc, xc, rows, c["use_box"], 1e-6)
    close(Wx, c["Wx"], 1e-12, 1e-12)
    close(dh, c["d_hat"], 1e-12, 1e-12)
    (Wx * c["gWx"].to(cuda) + dh * c["gdh"].to(cuda)).sum().backward()
    close(wc.grad, c["gw"], 1e-9, 1e-10)
    close(xc.grad, c["gx"], 1e-9, 1e-10)


@pytest.mark.parametrize("generic", [False, True])
@pytest.mark.parametrize("use_box", [True, False])
@pytest.mark.parametrize("bcast", [False, True])
def test_metropolis_vs_oracle(cuda, use_box, bcast, generic, monkeypatch):
    """Both kernel families (halo-tiled, one pixel per thread) in fp64."""
    if generic:
        monkeypatch.setenv("NSC_METRO_GENERIC", "1")
    torch.manual_seed(11)
    B, C, H, W, R = 2, 3, 17, 19, 2
    rows = O.halfplane_shifts(R)
    S = len(rows)
    w = torch.sigmoid(torch.randn(B, S, 1 if bcast else C, H, W,
                                  dtype=torch.float64))
    x = torch.rand(B, C, H, W, dtype=torch.float64)
    wc = w.to(cuda).requires_grad_(True)
    xc = x.to(cuda).requires_grad_(True)
    Wx, dh = nsc.metropolis_aggregate(wc, xc, rows, use_box)
    Wr, dr = O.metropolis_aggregate(w.expand(B, S, C, H, W), x, rows, use_box)
    close(Wx, Wr, 1e-12, 1e-12)
    close(dh, dr, 1e-12, 1e-12)
    gW, gd = torch.randn_like(x), torch.randn_like(x)
    (Wx * gW.to(cuda) + dh * gd.to(cuda)).sum().backward()
    gw, gx = O.metropolis_aggregate_grad(w, x, rows, use_box, 1e-6, gW, gd)
    close(wc.grad, gw, 1e-9, 1e-10)
    close(xc.grad, gx, 1e-9, 1e-10)


def test_metropolis_fp32(cuda):
    torch.manual_seed(12)
    B, C, H, W, R = 2, 3, 32, 24, 3
    rows = O.halfplane_shifts(R)
    w = torch.sigmoid(torch.randn(B, len(rows), 1, H, W))
    x = torch.rand(B, C, H, W)
    Wx, dh = nsc.metropolis_aggregate(w.to(cuda), x.to(cuda), rows, True)
    Wr, dr = O.metropolis_aggregate(w.double().expand(-1, -1, C, -1, -1),
                                    x.double(), rows, True)
    close(Wx, Wr.float(), 1e-5, 1e-5)
    close(dh, dr.float(), 1e-5, 1e-5)


def _metro_run(w, x, rows, use_box, gW, gd):
    wc = w.cuda().requires_grad_(True)
    xc = x.cuda().requires_grad_(True)
    Wx, dh = nsc.metropolis_aggregate(wc, xc, rows, use_box)
    (Wx * gW.cuda() + dh * gd.cuda()).sum().backward()
    return [t.detach().cpu() for t in (Wx, dh, wc.grad, xc.grad)]


@pytest.mark.parametrize("R,H,W,bcast,use_box", [
    (5, 37, 45, True, True), (5, 16, 32, False, False), (8, 20, 70, True, False),
    (1, 5, 3, True, True),
])
def test_metropolis_tiled_matches_general(cuda, R, H, W, bcast, use_box, monkeypatch):
    """fp32: the tiled kernels do the general kernels' arithmetic in the
    same order, so forward and gradients agree to rounding of contraction."""
    torch.manual_seed(R + H)
    rows = O.halfplane_shifts(R)
    B, C = 2, 3
    w = torch.sigmoid(torch.randn(B, len(rows), 1 if bcast else C, H, W))
    x = torch.rand(B, C, H, W)
    gW, gd = torch.randn_like(x), torch.randn_like(x)
    tiled = _metro_run(w, x, rows, use_box, gW, gd)
    monkeypatch.setenv("NSC_METRO_GENERIC", "1")
    general = _metro_run(w, x, rows, use_box, gW, gd)
    for a, b in zip(tiled, general):
        torch.testing.assert_close(a, b, rtol=2e-6, atol=2e-6)
