"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference checkout is importable:

    PYTHONPATH=<reference checkout> python tests/golden/make_golden.py <reference checkout>

It imports the reference package `neural_shift_cuda` (v0.12.0) on the CPU,
where every op runs its own pure-PyTorch path, evaluates the ops on small
seeded inputs, and writes `tests/golden/golden_ops.pt` and
`tests/golden/golden_nectr.pt`.  Gradients are taken with torch autograd
through the reference's own functions.  Nothing here runs at test time: the
tests only read the `.pt` files.
"""

from __future__ import annotations

import os
import sys
from types import SimpleNamespace

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def halfplane(R):
    rows = [(dx, dy, 1) for dx in range(-R, R + 1) for dy in range(1, R + 1)]
    rows += [(dx, 0, int(dx != 0)) for dx in range(0, R + 1)]
    return torch.tensor(rows, dtype=torch.int64)


def window(R):
    return torch.tensor([(dx, dy, 0) for dx in range(-R, R + 1)
                         for dy in range(-R, R + 1)], dtype=torch.int64)


def box_stack(shifts, B, H, W, dtype):
    R = int(shifts[:, :2].abs().max())
    box = F.pad(torch.ones(1, 1, H, W, dtype=dtype), (R, R, R, R),
                mode="constant", value=0)
    ms = [box[:, :, R + int(dx):R + int(dx) + H, R + int(dy):R + int(dy) + W]
          for dx, dy in shifts[:, :2].tolist()]
    m = torch.cat(ms, 0)
    return m.unsqueeze(1).expand(len(ms), B, 1, H, W).reshape(-1, 1, H, W)


def main(ref_root):
    sys.path.insert(0, ref_root)
    import neural_shift_cuda as ref
    from neural_shift_cuda import metropolis as refm

    cases = {}

    # -- gathers -----------------------------------------------------------
    g = torch.Generator().manual_seed(0)
    for name, shp, R in [("g1", (2, 3, 7, 9), 2), ("g2", (1, 2, 5, 4), 3)]:
        guide = torch.randn(*shp, generator=g, dtype=torch.float64)
        sh = halfplane(R)
        gs, mask = ref.shift_gather_reference(guide, sh)
        pr, pmask = ref.pair_gather_reference(guide, sh)
        gg = guide.clone().requires_grad_(True)
        go = torch.randn(gs.shape, generator=g, dtype=torch.float64)
        (ref.shift_gather_reference(gg, sh)[0] * go).sum().backward()
        gp = guide.clone().requires_grad_(True)
        gpo = torch.randn(pr.shape, generator=g, dtype=torch.float64)
        (ref.pair_gather_reference(gp, sh)[0] * gpo).sum().backward()
        cases["shift_gather_" + name] = dict(
            guide=guide, shifts=sh, out=gs, mask=mask, pair=pr,
            pair_mask=pmask, grad_out=go, grad_guide=gg.grad,
            pair_grad_out=gpo, pair_grad_guide=gp.grad)

    # -- accumulate_uz -----------------------------------------------------
    for name, shp, R, dt, tab in [
            ("a64", (2, 3, 9, 8), 2, torch.float64, "half"),
            ("a32", (2, 1, 32, 32), 3, torch.float32, "half"),
            ("a64w", (1, 2, 6, 7), 1, torch.float64, "window")]:
        B, C, H, W = shp
        sh = halfplane(R) if tab == "half" else window(R)
        S = sh.shape[0]
        x = torch.rand(*shp, generator=g, dtype=dt) + \
            (25 / 255) * torch.randn(*shp, generator=g, dtype=dt)
        w = F.softplus(torch.randn(S * B, C, H, W, generator=g, dtype=dt))
        w = w * box_stack(sh, B, H, W, dt)
        U, Z = ref.accumulate_uz(x, w, sh)
        xg = x.clone().requires_grad_(True)
        wg = w.clone().requires_grad_(True)
        gU = torch.randn(shp, generator=g, dtype=dt)
        gZ = torch.randn(shp, generator=g, dtype=dt)
        U2, Z2 = ref.accumulate_uz_reference(xg, wg, sh)
        (U2 * gU + Z2 * gZ).sum().backward()
        cases["accumulate_" + name] = dict(
            x=x, w=w, shifts=sh, U=U, Z=Z, gU=gU, gZ=gZ,
            gx=xg.grad, gw=wg.grad)

    # -- normalized_accumulate_uz -----------------------------------------
    for name, shp, R, tab, logw in [
            ("pos_half", (2, 2, 7, 6), 2, "half", False),
            ("log_half", (1, 3, 8, 7), 2, "half", True),
            ("pos_win", (1, 2, 6, 6), 1, "window", False),
            ("log_win", (2, 1, 9, 8), 2, "window", True)]:
        B, C, H, W = shp
        sh = halfplane(R) if tab == "half" else window(R)
        S = sh.shape[0]
        x = torch.randn(*shp, generator=g, dtype=torch.float64)
        raw = 2.0 * torch.randn(S * B, C, H, W, generator=g,
                                dtype=torch.float64)
        m = box_stack(sh, B, H, W, torch.float64)
        if logw:
            w = torch.where(m > 0, raw, torch.full_like(raw, -torch.inf))
        else:
            w = raw.exp() * m
        D, L = ref.normalized_accumulate_uz(
            x, w, sh, log_weights=logw, return_log_degree=True)
        # gradients on the strictly positive / finite sub-problem only:
        # the reference's autograd is NaN at masked entries, its CUDA
        # kernels define them as 0 (documented in the oracle).
        wfull = raw if logw else raw.exp()
        xg = x.clone().requires_grad_(True)
        wg = wfull.clone().requires_grad_(True)
        Dg, Lg = ref.normalized_accumulate_uz_reference(
            xg, wg, sh, log_weights=logw, return_log_degree=True)
        gD = torch.randn(shp, generator=g, dtype=torch.float64)
        gL = torch.randn(shp, generator=g, dtype=torch.float64)
        (Dg * gD + Lg * gL).sum().backward()
        cases["normalized_" + name] = dict(
            x=x, w=w, shifts=sh, log_weights=logw, D=D, logC=L,
            w_full=wfull, D_full=Dg.detach(), logC_full=Lg.detach(),
            gD=gD, gL=gL, gx=xg.grad, gw=wg.grad)

    # overflow known-answer test (tests/test_normalized_accumulate_uz.py:43)
    sh = window(1)
    x = torch.linspace(-1, 1, 20).reshape(1, 1, 5, 4)
    w = torch.full((9, 1, 5, 4), 1.0e38, dtype=torch.float32)
    D, L = ref.normalized_accumulate_uz(x, w, sh, return_log_degree=True)
    cases["normalized_overflow"] = dict(x=x, w=w, shifts=sh, D=D, logC=L)

    # empty rows: everything masked at some pixels
    sh = halfplane(1)
    S = sh.shape[0]
    x = torch.randn(1, 1, 4, 5, generator=g, dtype=torch.float64)
    lw = torch.randn(S, 1, 4, 5, generator=g, dtype=torch.float64)
    lw[:, :, 0, 0] = -torch.inf
    lw[:, :, 1, :] = -torch.inf
    D, L = ref.normalized_accumulate_uz(
        x, lw, sh, log_weights=True, return_log_degree=True, validate=True)
    cases["normalized_empty"] = dict(x=x, w=lw, shifts=sh, D=D, logC=L)

    # -- metropolis --------------------------------------------------------
    for name, (B, S_R, C, H, W), use_box in [
            ("box", (2, 1, 2, 7, 8), True), ("circ", (1, 2, 3, 6, 9), False),
            ("box_r2", (1, 2, 1, 9, 7), True)]:
        R = S_R
        rows = [(int(a), int(b), bool(c)) for a, b, c in halfplane(R).tolist()]
        S = len(rows)
        w_half = torch.sigmoid(torch.randn(B, S, C, H, W, generator=g,
                                           dtype=torch.float64))
        img = torch.rand(B, C, H, W, generator=g, dtype=torch.float64)
        Wx_t, dh_t = refm.metropolis_aggregate_torch(w_half, img, rows,
                                                     use_box, 1e-6)
        wg = w_half.clone().requires_grad_(True)
        xg = img.clone().requires_grad_(True)
        Wx, dh = refm.metropolis_aggregate_fused(wg, xg, rows, use_box, 1e-6)
        gW = torch.randn(img.shape, generator=g, dtype=torch.float64)
        gd = torch.randn(img.shape, generator=g, dtype=torch.float64)
        (Wx * gW + dh * gd).sum().backward()
        cases["metropolis_" + name] = dict(
            w_half=w_half, img=img, shifts=torch.tensor(
                [(a, b, int(c)) for a, b, c in rows]), use_box=use_box,
            Wx=Wx_t, d_hat=dh_t, Wx_fused=Wx.detach(), d_hat_fused=dh.detach(),
            gWx=gW, gdh=gd, gw=wg.grad, gx=xg.grad)

    torch.save(cases, os.path.join(HERE, "golden_ops.pt"))

    # -- NECTR end-to-end (model file from the reference checkout) --------
    sys.path.insert(0, os.path.join(ref_root, "models"))
    import NECTR_models1 as nm
    from neural_shift_cuda.integration import nectr_patch
    nectr = {}
    for act in ["exp", "control_sigmoid", "none"]:
        torch.manual_seed(0)
        args = SimpleNamespace(
            model_type="concat", residual_depth=2, proj_depth=1,
            latent_dim=8, patch_rad=1, output_activation=act, window_rad=2,
            in_channel=1, blind=True)
        model = nm.NECTR_denoiser(args, "cpu").double()
        x = torch.rand(2, 1, 12, 11, generator=g, dtype=torch.float64)
        with torch.no_grad():
            U_ser, Z_ser = model(x)
        Patched = type("PatchedNECTR", (nm.NECTR_denoiser,), {})
        nectr_patch.install_cuda_shift(Patched)
        pm = Patched.__new__(Patched)
        pm.__dict__ = model.__dict__.copy()
        with torch.no_grad():
            U_p, Z_p = pm(x)
        nectr[act] = dict(state=model.state_dict(), x=x, U_serial=U_ser,
                          Z_serial=Z_ser, U_patched=U_p, Z_patched=Z_p,
                          args=vars(args))
    torch.save(nectr, os.path.join(HERE, "golden_nectr.pt"))
    inst = installer_cases()
    torch.save(inst, os.path.join(HERE, "golden_installers.pt"))
    print("wrote", sorted(cases), sorted(nectr), sorted(inst))


def installer_cases():
    """The reference's own GASD / NeKDe / NKD_mp installer functions on the
    stub models of tests/stub_models.py, on the CPU (where the reference
    ops run their PyTorch paths), fp64."""
    sys.path.insert(0, os.path.dirname(HERE))
    import stub_models as SM
    from neural_shift_cuda.integration import gasd_drunet_attn_patch as rg
    from neural_shift_cuda.integration import nekde_drunet_attn_patch as rn
    from neural_shift_cuda.integration import nkd_metropolis_attn_patch as rm
    mods = {"gasd": rg, "nekde": rn, "nkd": rm}
    out = {}
    for case in SM.INSTALLER_CASES:
        kind, B, C, H, W, R, heads, box, seed = case
        cls = SM.make_class(kind)
        mods[kind].install_cuda_shift(cls)
        m = SM.make_model(kind, C, R, heads, box, seed, cls=cls)
        g = torch.Generator().manual_seed(seed)
        x = torch.rand(B, C, H, W, generator=g, dtype=torch.float64)
        y = torch.randn(B, C, H, W, generator=g, dtype=torch.float64)
        guide = torch.rand(B, C, H, W, generator=g, dtype=torch.float64)
        rec = dict(case=case, state=m.state_dict(), x=x, y=y, guide=guide)
        with torch.no_grad():
            if kind == "gasd":
                rec["D"], rec["Z"] = rg._forward_cuda(m, x)
                rec["D_guided"], _ = rg._forward_cuda(m, x, guide=guide)
                rec["KT"] = rg._kt_action_cuda(m, y, guide=guide)
                rec["WT"], rec["WT_D"] = rg._nlm_transpose_cuda(
                    m, x, guide=guide, return_D=True)
                rec["LAP"] = rg._laplacian_grw_cuda(m, x, guide)
            elif kind == "nekde":
                rec["D"], rec["Z"] = rn._forward_cuda(m, x)
                rec["D_guided"], _ = rn._forward_cuda(m, x, guide=guide)
                rec["KT"], rec["KT_Z"] = rn._kt_action_cuda(
                    m, y, guide=guide, return_D=True)
                rec["KTD"], _ = rn._kt_action_cuda(
                    m, y, guide=guide, return_D=True, apply_Dinv=True)
            else:
                rec["Wx"], rec["d_hat"] = rm._forward_cuda(m, x, return_D=True)
                rec["Wx_guided"], _ = rm._forward_cuda(m, x, guide=guide)
        out[SM.case_name(case)] = rec
    return out


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ["NSC_REFERENCE"]
    if "--installers-only" in sys.argv:
        sys.path.insert(0, root)
        inst = installer_cases()
        torch.save(inst, os.path.join(HERE, "golden_installers.pt"))
        print("wrote", sorted(inst))
    else:
        main(root)
