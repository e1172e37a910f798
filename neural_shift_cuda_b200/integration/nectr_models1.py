"""The NECTR model-1 architecture (`NECTR_denoiser`), the class the NECTR
installer patches.

A restatement of `models/NECTR_models1.py` of the reference checkout
(lines 12-244): the feature network (`pre_activation`, :84-116), the
pairwise weight head (`N_theta`, :118-148) and the serial per-shift forward
(:154-244).  It is not part of the kernel path: the package ships it so the
NECTR forward can be benchmarked (random init, the benchmark's shapes) and
tested without the reference checkout.  Its serial `forward` is the
end-to-end check of the installed forward.  Parameter names follow the
reference so its state dicts load unchanged; `tests/golden/make_golden.py`
stores the reference model's own outputs for seeded inputs and
`tests/test_oracle_golden.py` pins this restatement to them.
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F


class NECTR_denoiser(nn.Module):
    def __init__(self, args, device=None):
        super().__init__()
        self.model_type = args.model_type
        self.residual_depth = args.residual_depth
        self.proj_depth = args.proj_depth
        self.latent_dim = L = args.latent_dim
        self.sigma = 1
        self.blind = args.blind
        self.patch_size = 2 * args.patch_rad + 1
        self.output_activation = args.output_activation
        self.window_rad = args.window_rad
        self.in_channel = args.in_channel
        in_dim = self.in_channel if self.blind else self.in_channel + 1
        self.in_layer = nn.Conv2d(in_dim, L, kernel_size=self.patch_size,
                                  padding=self.patch_size // 2)
        self.in_proj = nn.ModuleList(
            [nn.Sequential(nn.Conv2d(L, L, 3, padding=1), nn.LeakyReLU())
             for _ in range(self.residual_depth - 1)]
            + [nn.Conv2d(L, L, 3, padding=1)])
        self.in_residual = nn.ModuleList([
            nn.Sequential(nn.Conv2d(L, 4 * L, 1), nn.LeakyReLU(),
                          nn.Conv2d(4 * L, L, 1))
            for _ in range(self.residual_depth)])
        self.in_norm = nn.ModuleList([nn.LayerNorm(L)
                                      for _ in range(self.residual_depth)])
        if self.model_type == "rbf":
            return
        d = 2 * L if self.model_type == "concat" else L
        self.proj = nn.ModuleList([
            nn.ModuleList([nn.Conv2d(d // 2 ** i, d // 2 ** (i + 1), 1),
                           nn.LayerNorm(d // 2 ** (i + 1)), nn.LeakyReLU()])
            for i in range(self.proj_depth)])
        d = d // 2 ** self.proj_depth
        out_dim = self.in_channel * (3 if self.output_activation == "control_sigmoid" else 1)
        self.out = nn.Conv2d(d, out_dim, 1, bias=False)

    def pre_activation(self, x, sigma=None):
        if not self.blind:
            if sigma is None:
                raise ValueError("sigma is None, but blind is False")
            if not torch.is_tensor(sigma):
                sigma = torch.tensor([sigma], dtype=x.dtype, device=x.device)
            sigma = sigma.reshape(-1, 1, 1, 1)
            x = torch.cat((x, sigma.expand(x.shape[0], 1, *x.shape[2:])), 1)
        x = self.in_layer(x)
        for res, norm in zip(self.in_residual, self.in_norm):
            x = x + res(x)
            # channel LayerNorm through a (0, 3, 2, 1) permutation, as the
            # reference does
            x = norm(x.permute(0, 3, 2, 1).contiguous()).permute(0, 3, 2, 1).contiguous()
        return x

    def controlled_sigmoid(self, x, a, b):
        return F.softplus(a) / (1 + torch.exp(-torch.sigmoid(b) * x))

    def N_theta(self, x, x_s):
        v = torch.cat((x, x_s), 1) if self.model_type == "concat" else x
        for block in self.proj:
            for j, layer in enumerate(block):
                if j == 1:
                    v = layer(v.permute(0, 2, 3, 1)).permute(0, 3, 1, 2)
                else:
                    v = layer(v)
        v = self.out(v)
        if self.output_activation == "exp":
            return torch.exp(v / self.sigma ** 2)
        if self.output_activation == "control_sigmoid":
            k, a, b = torch.chunk(v, 3, dim=1)
            return self.controlled_sigmoid(k, a, b) + 1e-8
        return v

    def forward(self, x, reference=None, sig=None, cache=None, store_cache=False):
        """Serial forward: for every half-plane shift one weight-head
        evaluation, the forward term and the box-masked mirror term,
        summed in shift order; returns (U / Z, Z) (and the cache)."""
        R = self.window_rad
        H, W = x.shape[2:]
        ref = self.pre_activation(x if reference is None else reference, sigma=sig)
        pad_x = F.pad(x, (R, R, R, R), mode="circular")
        pad_r = F.pad(ref, (R, R, R, R), mode="circular")
        box = F.pad(torch.ones_like(x), (R, R, R, R), mode="constant", value=0)

        def win(t, dx, dy):
            return t[:, :, R + dx:R + dx + H, R + dy:R + dy + W]

        U = torch.zeros_like(x)
        Z = torch.zeros_like(x)
        held = {}
        rows = [(dx, dy) for dx in range(-R, R + 1) for dy in range(1, R + 1)]
        rows += [(dx, 0) for dx in range(0, R + 1)]
        for dx, dy in rows:
            if cache is None:
                w = self.N_theta(ref, win(pad_r, dx, dy)) * win(box, dx, dy)
                if store_cache:
                    held[(dx, dy)] = w
            else:
                w = cache[(dx, dy)]
            U = U + w * win(pad_x, dx, dy)
            Z = Z + w
            if dx == 0 and dy == 0:
                continue
            wi = win(F.pad(w, (R, R, R, R), mode="circular"), -dx, -dy) * win(box, -dx, -dy)
            U = U + wi * win(pad_x, -dx, -dy)
            Z = Z + wi
        U = U / Z
        return (U, Z, held) if store_cache else (U, Z)
