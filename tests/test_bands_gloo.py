"""Row-band split of accumulate_uz across ranks, on CPU `gloo` ranks.

The exchange logic of neural_shift_cuda_b200.bands (x-halo ring and
mirror-strip exchange in one grouped send/recv, plain and padded x bands)
runs unchanged; only the per-band compute is a CPU
restatement injected here, so no GPU is needed.  Every rank checks its
band against the oracle's full-image result.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from neural_shift_cuda_b200 import bands
from oracle import nsc_oracle as O


def _band_compute_cpu(x_ext, w_band, shifts, row0, Hg):
    """CPU band compute: (U, Z) of the band without cross-band mirror
    terms, and the (2, B, C, R, W) strips for the rows above / below."""
    rows = [tuple(int(v) for v in r) for r in torch.as_tensor(shifts).tolist()]
    R = max(max(abs(r[0]), abs(r[1])) for r in rows)
    B, C, He, W = x_ext.shape
    Hb = He - 2 * R
    x = x_ext.double()
    w = w_band.double().reshape(len(rows), B, -1, Hb, W).expand(len(rows), B, C, Hb, W)
    U = torch.zeros(B, C, Hb, W, dtype=torch.float64)
    Z = torch.zeros_like(U)
    top = torch.zeros(2, B, C, R, W, dtype=torch.float64)
    bot = torch.zeros_like(top)
    cols = torch.arange(W)
    for s, (dx, dy, inv) in enumerate(rows):
        for h in range(Hb):
            U[:, :, h] += w[s, :, :, h] * x[:, :, h + dx + R, (cols + dy) % W]
            Z[:, :, h] += w[s, :, :, h]
        if not inv:
            continue
        src_c = cols - dy
        okc = (src_c >= 0) & (src_c < W)
        sc = src_c.clamp(0, W - 1)
        for t in list(range(-R, 0)) + list(range(Hb)) + list(range(Hb, Hb + R)):
            hs = t - dx
            if not (0 <= hs < Hb) or not (0 <= row0 + t < Hg):
                continue
            contrib_u = (w[s, :, :, hs, sc] * x[:, :, hs + R, sc]) * okc
            contrib_z = w[s, :, :, hs, sc] * okc
            if t < 0:
                top[0, :, :, t + R] += contrib_u
                top[1, :, :, t + R] += contrib_z
            elif t >= Hb:
                bot[0, :, :, t - Hb] += contrib_u
                bot[1, :, :, t - Hb] += contrib_z
            else:
                U[:, :, t] += contrib_u
                Z[:, :, t] += contrib_z
    return U, Z, top, bot


def _worker(rank, world, port, Hg, W, R, padded, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        B, C = 1, 2
        rows = O.halfplane_shifts(R)
        sh = torch.tensor(rows)
        x = torch.rand(B, C, Hg, W, generator=g, dtype=torch.float64)
        w = O.premasked_weights(torch.rand(len(rows) * B, 1, Hg, W, generator=g,
                                           dtype=torch.float64), sh, B)
        U_ref, Z_ref = O.accumulate_uz(x, w.expand(-1, C, -1, -1), sh)
        row0, Hb = bands.band_rows(Hg, world, rank)
        xb = x[:, :, row0:row0 + Hb].contiguous()
        if padded:   # spare halo rows hold NaN: the exchange must overwrite them
            if padded == "strided":   # a non-contiguous buffer: staged halo copies
                xp = torch.full((B, Hb + 2 * R, W, C), float("nan"),
                                dtype=x.dtype).permute(0, 3, 1, 2)
            else:                     # contiguous: halo rows received in place
                xp = torch.full((B, C, Hb + 2 * R, W), float("nan"), dtype=x.dtype)
            xp[:, :, R:R + Hb] = xb
            xb = xp
        U, Z = bands.accumulate_uz_banded(
            xb, w[:, :, row0:row0 + Hb].contiguous(), sh, Hg,
            compute=_band_compute_cpu, padded=bool(padded))
        ok = (torch.allclose(U, U_ref[:, :, row0:row0 + Hb], rtol=1e-10, atol=1e-10)
              and torch.allclose(Z, Z_ref[:, :, row0:row0 + Hb], rtol=1e-10, atol=1e-10))
        out[rank] = 1 if ok else 0
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world,Hg,W,R,padded", [(2, 12, 9, 2, False), (3, 17, 7, 3, False),
                                                 (2, 8, 6, 1, False), (3, 17, 7, 3, True),
                                                 (2, 12, 9, 2, True),
                                                 (3, 17, 7, 3, "strided")])
def test_banded_accumulate_gloo(world, Hg, W, R, padded):
    ctx = mp.get_context("spawn")
    out = ctx.Array("i", [0] * world)
    mp.start_processes(_worker, args=(world, _free_port(), Hg, W, R, padded, out),
                       nprocs=world, join=True, start_method="spawn")
    assert list(out) == [1] * world


def test_band_rows_cover_image():
    for Hg, world in [(8192, 8), (10, 3), (7, 7)]:
        spans = [bands.band_rows(Hg, world, r) for r in range(world)]
        assert spans[0][0] == 0
        for (a, n), (b, _) in zip(spans, spans[1:]):
            assert a + n == b
        assert spans[-1][0] + spans[-1][1] == Hg


def _leaver_worker(rank, world, port, out):
    """Step 1 on every rank; then rank world-1 leaves (exits without
    shutting its process group down) and the others run step 2, which must
    fail on the host with BandExchangeError within the deadline."""
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=20))
    Hg, W, R = 15, 6, 2
    g = torch.Generator().manual_seed(0)
    rows = O.halfplane_shifts(R)
    sh = torch.tensor(rows)
    x = torch.rand(1, 1, Hg, W, generator=g, dtype=torch.float64)
    w = torch.rand(len(rows), 1, Hg, W, generator=g, dtype=torch.float64)
    row0, Hb = bands.band_rows(Hg, world, rank)
    args = (x[:, :, row0:row0 + Hb].contiguous(), w[:, :, row0:row0 + Hb].contiguous(),
            sh, Hg)
    bands.accumulate_uz_banded(*args, compute=_band_compute_cpu, deadline=5.0)
    dist.barrier()
    if rank == world - 1:
        out[rank] = 1
        os._exit(0)                      # leaves between steps
    t0 = time.monotonic()
    try:
        bands.accumulate_uz_banded(*args, compute=_band_compute_cpu, deadline=5.0)
        out[rank] = 0                    # should not complete
    except bands.BandExchangeError:
        out[rank] = 1 if time.monotonic() - t0 < 15.0 else 2
    os._exit(0)


def test_banded_rank_leaves_between_steps():
    world = 3
    ctx = mp.get_context("spawn")
    out = ctx.Array("i", [0] * world)
    mp.start_processes(_leaver_worker, args=(world, _free_port(), out),
                       nprocs=world, join=True, start_method="spawn")
    assert list(out) == [1] * world
