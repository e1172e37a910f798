"""GPU tests of the model installers.

* NECTR: the reference's own NECTR_models1 weights (tests/golden) through
  the installed CUDA forward, against the reference's serial and patched
  outputs (fp64).
* GASD / NeKDe / NKD_mp: the model files are not part of the reference
  checkout, so small stub models (tests/stub_models.py) implement exactly
  the attributes the installers call (`pre_activation`, `_collect_shifts`,
  the per-shift weight producers, head mixing).  The installed forwards,
  K^T actions, NLM transpose and Laplacian are checked against the
  reference's own installer functions run on the same stubs on the CPU
  (tests/golden/golden_installers.pt), and against direct CPU restatements
  of the operators they implement (the reference's own cached-path tests
  use the same approach, tests/test_cached_forward_patches.py).
"""

import os
from types import SimpleNamespace

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from neural_shift_cuda_b200 import integration as I
from oracle import nsc_oracle as O
from neural_shift_cuda_b200.integration.nectr_models1 import NECTR_denoiser
import stub_models as SM

pytestmark = pytest.mark.gpu

GOLD_NECTR = torch.load(os.path.join(os.path.dirname(__file__), "golden",
                                     "golden_nectr.pt"), weights_only=False)
GOLD_INST = torch.load(os.path.join(os.path.dirname(__file__), "golden",
                                    "golden_installers.pt"), weights_only=False)
_INSTALL = {"gasd": I.install_cuda_shift_gasd, "nekde": I.install_cuda_shift_attn,
            "nkd": I.install_cuda_shift_metropolis}


@pytest.fixture(autouse=True)
def _no_tf32():
    """fp32 convolutions in full fp32 (cuDNN defaults to TF32, ~1e-3
    relative), so fp32 results can be held to fp32 tolerances."""
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cudnn.allow_tf32 = prev


def _roll(x, dx, dy):
    """gather convention: out(h, w) = x(h+dx, w+dy) circularly"""
    return torch.roll(x, shifts=(-dx, -dy), dims=(-2, -1))


# --------------------------------------------------------------- NECTR

@pytest.mark.parametrize("act", sorted(GOLD_NECTR))
def test_nectr_installed_forward_matches_reference(cuda, act):
    c = GOLD_NECTR[act]
    cls = type("NECTRPatched", (NECTR_denoiser,), {})
    I.install_cuda_shift_nectr(cls)
    m = cls(SimpleNamespace(**c["args"])).double()
    m.load_state_dict(c["state"])
    m = m.to(cuda)
    x = c["x"].to(cuda)
    with torch.no_grad():
        U, Z = m(x)
        U2, Z2, cache = m(x, store_cache=True)
        U3, Z3 = m(x, cache=cache)
        m.use_cuda_shift = False
        Us, Zs = m(x)                  # the model's own serial forward
    for u, z in ((U, Z), (U2, Z2), (U3, Z3)):
        torch.testing.assert_close(u.cpu(), c["U_patched"], rtol=1e-9, atol=1e-10)
        torch.testing.assert_close(u.cpu(), c["U_serial"], rtol=1e-9, atol=1e-10)
        torch.testing.assert_close(z.cpu().to(c["Z_serial"].dtype), c["Z_serial"],
                                   rtol=1e-9, atol=1e-10)
    torch.testing.assert_close(Us.cpu(), c["U_serial"], rtol=1e-9, atol=1e-10)


def test_nectr_fp32_and_bf16_inputs(cuda):
    """Benchmark-shaped NECTR (latent 16, R = 5) at reduced size: fp32 vs
    the serial forward, and bf16 weights/inputs with fp32 accumulation."""
    torch.manual_seed(0)
    args = SimpleNamespace(model_type="concat", residual_depth=2, proj_depth=1,
                           latent_dim=16, patch_rad=1, output_activation="exp",
                           window_rad=5, in_channel=1, blind=True)
    cls = type("NECTRPatched2", (NECTR_denoiser,), {})
    I.install_cuda_shift_nectr(cls)
    m = cls(args).to(cuda)
    g = torch.Generator().manual_seed(0)
    x = (torch.rand(2, 1, 40, 48, generator=g)
         + (25 / 255) * torch.randn(2, 1, 40, 48, generator=g)).to(cuda)
    with torch.no_grad():
        U, Z = m(x)
        m.use_nectr_fused = False
        Uu, Zu = m(x)                  # unfused: pair batch + ops
        m.use_nectr_fused = True
        md = cls(args).to(cuda)
        md.load_state_dict(m.state_dict())
        md = md.double()
        md.use_cuda_shift = False
        Us, Zs = md(x.double())        # serial forward in fp64
        mb = m.bfloat16()
        Ub, _ = mb(x.bfloat16())
    # fp32 (fused and unfused) against the fp64 serial forward
    for u, z in ((U, Z), (Uu, Zu)):
        torch.testing.assert_close(u.double(), Us, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(z.double(), Zs.double(), rtol=1e-4, atol=1e-5)
    assert Ub.dtype == torch.float32
    assert (Ub.double() - Us).abs().max() < 0.1   # bf16 weight head


# ------------------------------------------------------------ stub models

_StubBase = SM.StubBase


def _mixed(m, x):
    C = x.shape[1]
    phi = m.pre_activation(x)
    w = torch.stack(m._weights(phi, m._collect_shifts()), 0)
    mat = m._head_mix_matrix()
    return torch.stack([m._mix_heads(w[i], C, mat) for i in range(w.shape[0])], 0)


@pytest.mark.parametrize("comp_box", [True, False])
@pytest.mark.parametrize("heads", [1, 2, 3])
def test_gasd_installed_forward(cuda, comp_box, heads):
    torch.manual_seed(1)
    B, C, H, W, R = 2, 3, 12, 16, 2
    table = [(dx, dy) for dx in range(-R, R + 1) for dy in range(-R, R + 1)]
    cls = type("GASDStub", (_StubBase,), {"forward": lambda self, x, guide=None, sig=None, return_D=True: None})
    I.install_cuda_shift_gasd(cls)
    m = cls(C, R, heads, comp_box, table).double().to(cuda)
    x = torch.rand(B, C, H, W, dtype=torch.float64, device=cuda)
    with torch.no_grad():
        D, Z = m(x)
        w = _mixed(m, x).cpu()
    sh = torch.tensor([(dx, dy, 0) for dx, dy in table])
    if comp_box:
        w = w * torch.stack([O.box_mask(H, W, dx, dy, w.dtype) for dx, dy in table])[:, None, None]
    Dr, Lr = O.normalized_accumulate_uz(x.cpu(), w.reshape(-1, C, H, W), sh, False)
    torch.testing.assert_close(D.cpu(), Dr, rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(Z.cpu(), Lr.exp(), rtol=1e-10, atol=1e-10)
    # K^T through the rolled weights and negated shifts
    y = torch.rand_like(x)
    with torch.no_grad():
        KT = m._KT_action(y, guide=x)
    ref = sum(torch.roll(w[i] * y.cpu(), shifts=(dx, dy), dims=(-2, -1))
              for i, (dx, dy) in enumerate(table))
    torch.testing.assert_close(KT.cpu(), ref, rtol=1e-10, atol=1e-10)


def _symmetric_serial(x, w, rows, use_box):
    """sum of forward and mirror terms of the symmetric operator"""
    H, W = x.shape[-2:]
    U = torch.zeros_like(x)
    Z = torch.zeros_like(x)
    for wf, (dx, dy, inv) in zip(w, rows):
        if use_box:
            wf = wf * O.box_mask(H, W, dx, dy, wf.dtype)
        U = U + wf * _roll(x, dx, dy)
        Z = Z + wf
        if inv:
            wi = torch.roll(wf, shifts=(dx, dy), dims=(-2, -1))
            if use_box:
                wi = wi * O.box_mask(H, W, -dx, -dy, wi.dtype)
            U = U + wi * _roll(x, -dx, -dy)
            Z = Z + wi
    return U, Z


@pytest.mark.parametrize("comp_box", [True, False])
@pytest.mark.parametrize("heads", [1, 3])
def test_nekde_installed_forward(cuda, comp_box, heads):
    torch.manual_seed(2)
    B, C, H, W, R = 2, 3, 11, 13, 2
    rows = O.halfplane_shifts(R)
    cls = type("NeKDeStub", (_StubBase,), {"forward": lambda self, x, guide=None, sig=None, return_D=True: None})
    I.install_cuda_shift_attn(cls)
    m = cls(C, R, heads, comp_box, rows).double().to(cuda)
    x = torch.rand(B, C, H, W, dtype=torch.float64, device=cuda)
    with torch.no_grad():
        D, Z = m(x)
        w = _mixed(m, x).cpu()
        KT, Zk = m._KT_action(x, return_D=True)
    U, Zr = _symmetric_serial(x.cpu(), w, rows, comp_box)
    torch.testing.assert_close(D.cpu(), U / Zr, rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(Z.cpu(), Zr, rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(KT.cpu(), U, rtol=1e-10, atol=1e-10)


@pytest.mark.parametrize("comp_box", [True, False])
def test_metropolis_installed_forward(cuda, comp_box):
    torch.manual_seed(3)
    B, C, H, W, R = 2, 3, 10, 12, 2
    rows = O.halfplane_shifts(R)
    cls = type("MPStub", (_StubBase,), {"forward": lambda self, x, guide=None, sig=None, return_D=False: None})
    I.install_cuda_shift_metropolis(cls)
    m = cls(C, R, 1, comp_box, rows).double().to(cuda)
    m.metropolis_eps = 1e-6
    x = torch.rand(B, C, H, W, dtype=torch.float64, device=cuda)
    with torch.no_grad():
        Wx, dh = m(x, return_D=True)
        w_half = _mixed(m, x).cpu().permute(1, 0, 2, 3, 4)
    Wr, dr = O.metropolis_aggregate(w_half, x.cpu(), rows, comp_box, 1e-6)
    torch.testing.assert_close(Wx.cpu(), Wr, rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(dh.cpu(), dr, rtol=1e-10, atol=1e-10)


@pytest.mark.parametrize("use_box", [True, False])
def test_cached_forwards(cuda, use_box):
    """Cached fixed-guide actions of the three attention installers."""
    torch.manual_seed(4)
    B, C, H, W, R = 2, 3, 7, 8, 1
    x = torch.randn(B, C, H, W, dtype=torch.float64, device=cuda)
    half = [(0, 0, False), (0, 1, True), (1, -1, True), (1, 0, True), (1, 1, True)]
    wts = []
    for dx, dy, _ in half:
        w = torch.rand_like(x) + 0.1
        if use_box:
            w = w * O.box_mask(H, W, dx, dy, w.dtype).to(cuda)
        wts.append(w)
    U, D = _symmetric_serial(x.cpu(), [w.cpu() for w in wts], half, use_box)
    from neural_shift_cuda_b200.integration import nekde_drunet_attn_patch as nk
    cache = SimpleNamespace(C=C, shifts=half, w_fwd_list=wts, comp_box=use_box, D=None)
    out, deg = nk._forward_cached_cuda(SimpleNamespace(), x, cache, True)
    torch.testing.assert_close(out.cpu(), U / D, rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(deg.cpu(), D, rtol=1e-10, atol=1e-10)

    from neural_shift_cuda_b200.integration import nkd_metropolis_attn_patch as mp
    cache = SimpleNamespace(C=C, shifts=half, w_hat_fwd_list=wts, comp_box=use_box,
                            degree_hat=None)
    Wx, dh = mp._forward_cached_cuda(SimpleNamespace(), x, cache, True)
    torch.testing.assert_close(Wx.cpu(), x.cpu() - D * x.cpu() + U, rtol=1e-10, atol=1e-10)

    from neural_shift_cuda_b200.integration import gasd_drunet_attn_patch as gp
    full = [(dx, dy) for dx in range(-R, R + 1) for dy in range(-R, R + 1)]
    gw = [torch.rand_like(x) + 0.1 for _ in full]
    Kx = sum(w.cpu() * _roll(x.cpu(), dx, dy) for w, (dx, dy) in zip(gw, full))
    Zg = sum(w.cpu() for w in gw)
    KT = sum(torch.roll(w.cpu() * x.cpu(), shifts=(dx, dy), dims=(-2, -1))
             for w, (dx, dy) in zip(gw, full))
    cache = SimpleNamespace(C=C, shifts=full, w_list=gw, Z=None)
    model = SimpleNamespace()
    out, deg = gp._forward_cached_cuda(model, x, cache, True)
    torch.testing.assert_close(out.cpu(), Kx / Zg, rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(gp._kt_action_cached_cuda(model, x, cache).cpu(), KT,
                               rtol=1e-10, atol=1e-10)


# ------------------------------------------- pinned to the reference installers

def _close(a, b):
    torch.testing.assert_close(a.detach().cpu().to(b.dtype), b, rtol=1e-10,
                               atol=1e-10)


@pytest.mark.parametrize("name", sorted(GOLD_INST))
def test_installers_match_reference_installers(cuda, name):
    """This package's installed methods on a stub model vs the reference's
    installer functions on the same stub and weights (fp64)."""
    c = GOLD_INST[name]
    kind, B, C, H, W, R, heads, box, seed = c["case"]
    cls = SM.make_class(kind, f"Pinned_{name}")
    _INSTALL[kind](cls)
    m = SM.make_model(kind, C, R, heads, box, seed, cls=cls)
    m.load_state_dict(c["state"])
    m = m.to(cuda)
    x, y, guide = (c[k].to(cuda) for k in ("x", "y", "guide"))
    with torch.no_grad():
        if kind == "gasd":
            D, Z = m(x)
            _close(D, c["D"])
            _close(Z, c["Z"])
            _close(m(x, guide=guide)[0], c["D_guided"])
            _close(m._KT_action(y, guide=guide), c["KT"])
            WT, WTD = m.NLM_transpose(x, guide=guide, return_D=True)
            _close(WT, c["WT"])
            _close(WTD, c["WT_D"])
            _close(m.laplacian_grw(x, guide), c["LAP"])
        elif kind == "nekde":
            D, Z = m(x)
            _close(D, c["D"])
            _close(Z, c["Z"])
            _close(m(x, guide=guide)[0], c["D_guided"])
            KT, KZ = m._KT_action(y, guide=guide, return_D=True)
            _close(KT, c["KT"])
            _close(KZ, c["KT_Z"])
            KTD, _ = m._KT_action(y, guide=guide, return_D=True, apply_Dinv=True)
            _close(KTD, c["KTD"])
        else:
            Wx, dh = m(x, return_D=True)
            _close(Wx, c["Wx"])
            _close(dh, c["d_hat"])
            _close(m(x, guide=guide)[0], c["Wx_guided"])


# ----------------------------------------------------- fused NECTR forward

def _nectr(args_over, cuda, seed=0):
    args = dict(model_type="concat", residual_depth=2, proj_depth=1, latent_dim=16,
                patch_rad=1, output_activation="exp", window_rad=5, in_channel=1,
                blind=True)
    args.update(args_over)
    cls = type("NECTRFused", (NECTR_denoiser,), {})
    I.install_cuda_shift_nectr(cls)
    torch.manual_seed(seed)
    return cls(SimpleNamespace(**args)).to(cuda)


@pytest.mark.parametrize("over", [
    {},                                                      # benchmark head
    {"output_activation": "control_sigmoid"},
    {"output_activation": "none"},
    {"proj_depth": 2, "latent_dim": 32, "window_rad": 3},
    {"in_channel": 3, "latent_dim": 8, "window_rad": 2},
    {"in_channel": 3, "output_activation": "control_sigmoid", "proj_depth": 2,
     "latent_dim": 16, "window_rad": 4},
])
def test_nectr_fused_matches_fp64_serial(cuda, over):
    """The fused kernel (fp32) against the model's own serial forward in
    fp64 and against the unfused patched path (fp32)."""
    m = _nectr(over, cuda)
    C = m.in_channel
    g = torch.Generator().manual_seed(1)
    x = (torch.rand(2, C, 40, 48, generator=g)
         + (25 / 255) * torch.randn(2, C, 40, 48, generator=g)).to(cuda)
    with torch.no_grad():
        D, Z = m(x)                                   # fused
        m.use_nectr_fused = False
        Du, Zu = m(x)                                 # pair batch + ops
        m.use_nectr_fused = True
        md = m.double()
        md.use_cuda_shift = False
        Ds, Zs = md(x.double())                       # serial, fp64
        md.use_cuda_shift = True
        Dd, Zd = md(x.double())                       # fused, fp64
    torch.testing.assert_close(D.double(), Ds, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(Z.double(), Zs.double(), rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(D, Du, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(Dd, Ds, rtol=1e-9, atol=1e-10)
    torch.testing.assert_close(Zd.double(), Zs.double(), rtol=1e-9, atol=1e-10)


def test_nectr_fused_benchmark_shape(cuda):
    """configs[1] shape: B = 8, 1 x 256 x 256, R = 5, latent 16, fp32 and a
    bf16 model; fused against the fp64 serial forward."""
    m = _nectr({}, cuda)
    g = torch.Generator().manual_seed(0)
    x = (torch.rand(8, 1, 256, 256, generator=g)
         + (25 / 255) * torch.randn(8, 1, 256, 256, generator=g)).to(cuda)
    with torch.no_grad():
        D, Z = m(x)
        md = _nectr({}, cuda).double()
        md.use_cuda_shift = False
        Ds, Zs = md(x.double())
        mb = _nectr({}, cuda).bfloat16()
        Db, _ = mb(x.bfloat16())
    torch.testing.assert_close(D.double(), Ds, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(Z, Zs, rtol=1e-4, atol=1e-5)
    assert Db.dtype == torch.float32
    assert (Db.double() - Ds).abs().max() < 0.1   # bf16 head weights and inputs


def test_nectr_fused_not_used_with_autograd(cuda):
    m = _nectr({"window_rad": 2, "latent_dim": 8}, cuda)
    x = torch.rand(1, 1, 16, 24, device=cuda)
    D, Z = m(x)                       # grad enabled: differentiable path
    D.sum().backward()
    assert m.out.weight.grad is not None
