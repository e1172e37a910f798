"""Row-band split of one image across GPUs for `accumulate_uz`.

A single large image (e.g. 8192 x 8192 with S = 221 weight planes, ~30 GB
of fp16 weights) is cut into horizontal bands, one per rank.  Each rank
holds the weight rows of its own band only.  Two exchanges make the result
identical to the unsplit op:

1. x halo: the forward term at row h reads x at h + dx (circular), so each
   band needs R rows of x above and below it.  Rank r sends its first R rows
   to rank r-1 and its last R rows to rank r+1, around a ring (circular
   wrap).
2. mirror strips: the mirror term at output p reads the weight AND x at
   p - d, i.e. a product owned by the rank holding row p - dx.  Instead of
   shipping R rows of every weight plane (36 MB per boundary at S = 221),
   each rank computes the mirror contributions of its own weights to the R
   rows just outside its band (nsc_accumulate_uz_band_edges, a
   (2, B, C, R, W) fp32 strip, ~1 MB) and sends them to the neighbour that
   owns those rows, which adds them.  The mirror term is never periodic, so
   the strips of the first and last band are not exchanged.

Both exchanges are one grouped send/recv step each (`batch_isend_irecv`,
NCCL over NVLink for CUDA tensors).  The compute is injectable so the
exchange logic runs on CPU `gloo` ranks in the tests.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch

from . import _lib
from .ops import _require_cuda, _storage_dtypes

__all__ = ["band_rows", "x_ext_from_full", "band_compute_cuda",
           "accumulate_uz_banded_local", "accumulate_uz_banded",
           "radius_of"]


def band_rows(Hg: int, world: int, rank: int) -> Tuple[int, int]:
    """(row0, Hb) of `rank`'s band: an even split, the first Hg % world
    bands one row taller."""
    base, extra = divmod(Hg, world)
    row0 = rank * base + min(rank, extra)
    return row0, base + (1 if rank < extra else 0)


def radius_of(shifts) -> int:
    hs = _lib.host_shifts(shifts)
    return int(hs.t[:, :2].abs().max()) if hs.S else 0


def x_ext_from_full(x: torch.Tensor, row0: int, Hb: int, R: int) -> torch.Tensor:
    """Rows row0-R .. row0+Hb+R-1 of x, wrapped circularly (single-process
    construction of the halo-extended band)."""
    Hg = x.shape[2]
    idx = torch.arange(row0 - R, row0 + Hb + R, device=x.device) % Hg
    return x.index_select(2, idx).contiguous()


def band_compute_cuda(x_ext, w_band, shifts, row0: int, Hg: int):
    """(U, Z, top, bot) of one band on its GPU via the C ABI.

    x_ext: (B, C, Hb + 2R, W); w_band: (S*B, Cw, Hb, W).  U, Z: (B, C, Hb,
    W) without the cross-band mirror terms; top / bot: (2, B, C, R, W)
    mirror strips for the rows above / below the band."""
    _require_cuda("accumulate_uz_band", x_ext, w_band)
    hs = _lib.host_shifts(shifts)
    R = int(hs.t[:, :2].abs().max())
    B, C, He, W = x_ext.shape
    Hb = He - 2 * R
    xd, wd = _storage_dtypes(x_ext, w_band)
    x_k = x_ext.to(xd).contiguous()
    w_k = w_band.to(wd).contiguous()
    acc = torch.float64 if xd == torch.float64 else torch.float32
    U = torch.empty((B, C, Hb, W), dtype=acc, device=x_ext.device)
    Z = torch.empty_like(U)
    top = torch.empty((2, B, C, R, W), dtype=acc, device=x_ext.device)
    bot = torch.empty_like(top)
    with torch.cuda.device(x_ext.device):
        st = _lib.stream_of(x_ext)
        args = (_lib.ptr(x_k), _lib.dtype_code(xd), _lib.ptr(w_k),
                _lib.dtype_code(wd), w_k.size(1), B, C, Hb, W, row0, Hg,
                hs.ptr, hs.S)
        _lib.call("nsc_accumulate_uz_band_fwd", *args, _lib.ptr(U),
                  _lib.ptr(Z), st)
        if R > 0:
            _lib.call("nsc_accumulate_uz_band_edges", *args, _lib.ptr(top),
                      _lib.ptr(bot), st)
    return U, Z, top, bot


def _add_strips(U, Z, from_below: Optional[torch.Tensor],
                from_above: Optional[torch.Tensor]):
    """Add a neighbour's mirror strips: `from_below` (the lower band's top
    strip) lands on this band's last R rows, `from_above` (the upper band's
    bottom strip) on its first R rows."""
    if from_below is not None:
        R = from_below.shape[3]
        U[:, :, -R:] += from_below[0]
        Z[:, :, -R:] += from_below[1]
    if from_above is not None:
        R = from_above.shape[3]
        U[:, :, :R] += from_above[0]
        Z[:, :, :R] += from_above[1]
    return U, Z


def accumulate_uz_banded_local(x, w, shifts, nbands: int,
                               compute: Callable = band_compute_cuda):
    """Single-process emulation of the split (all bands on one device):
    equal to `accumulate_uz(x, w, shifts)`.  Used to test the band path."""
    R = radius_of(shifts)
    B, C, Hg, W = x.shape
    S = _lib.host_shifts(shifts).S
    outs = []
    for r in range(nbands):
        row0, Hb = band_rows(Hg, nbands, r)
        x_ext = x_ext_from_full(x, row0, Hb, R)
        wb = w.reshape(S * B, w.shape[1], Hg, W)[:, :, row0:row0 + Hb]
        outs.append(compute(x_ext, wb.contiguous(), shifts, row0, Hg))
    res = []
    for r, (U, Z, top, bot) in enumerate(outs):
        below = outs[r + 1][2] if r + 1 < nbands else None
        above = outs[r - 1][3] if r > 0 else None
        res.append(_add_strips(U.clone(), Z.clone(), below, above))
    return (torch.cat([u for u, _ in res], 2), torch.cat([z for _, z in res], 2))


def exchange_x_halo(x_band: torch.Tensor, R: int, group=None) -> torch.Tensor:
    """Build this rank's (B, C, Hb + 2R, W) halo-extended band from its own
    rows and its ring neighbours' edge rows (one grouped send/recv)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if R == 0:
        return x_band.contiguous()
    if world == 1:
        Hb = x_band.shape[2]
        idx = torch.arange(-R, Hb + R, device=x_band.device) % Hb
        return x_band.index_select(2, idx).contiguous()
    up, down = (rank - 1) % world, (rank + 1) % world
    first = x_band[:, :, :R].contiguous()
    last = x_band[:, :, -R:].contiguous()
    from_up = torch.empty_like(last)     # the upper band's last R rows
    from_down = torch.empty_like(first)  # the lower band's first R rows
    # With two ranks `up` and `down` are the same peer and messages between
    # a pair match in issue order, so every rank sends its last rows before
    # its first rows and receives from_up before from_down.
    ops = [dist.P2POp(dist.isend, last, _g(down, group), group),
           dist.P2POp(dist.isend, first, _g(up, group), group),
           dist.P2POp(dist.irecv, from_up, _g(up, group), group),
           dist.P2POp(dist.irecv, from_down, _g(down, group), group)]
    for req in dist.batch_isend_irecv(ops):
        req.wait()
    return torch.cat([from_up, x_band, from_down], 2).contiguous()


def _g(r, group):
    import torch.distributed as dist
    return r if group is None else dist.get_global_rank(group, r)


def exchange_strips(top: torch.Tensor, bot: torch.Tensor, group=None):
    """Send this band's mirror strips to the bands that own those rows and
    receive theirs: returns (from_below, from_above), None at the image
    edges (the mirror term is not periodic)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    ops: List = []
    from_below = from_above = None
    if rank > 0:
        ops.append(dist.P2POp(dist.isend, top.contiguous(), _g(rank - 1, group), group))
        from_above = torch.empty_like(bot)
        ops.append(dist.P2POp(dist.irecv, from_above, _g(rank - 1, group), group))
    if rank + 1 < world:
        ops.append(dist.P2POp(dist.isend, bot.contiguous(), _g(rank + 1, group), group))
        from_below = torch.empty_like(top)
        ops.append(dist.P2POp(dist.irecv, from_below, _g(rank + 1, group), group))
    if ops:
        for req in dist.batch_isend_irecv(ops):
            req.wait()
    return from_below, from_above


def accumulate_uz_banded(x_band, w_band, shifts, Hg: int, group=None,
                         compute: Callable = band_compute_cuda):
    """accumulate_uz of this rank's band of a row-split image.

    x_band: (B, C, Hb, W) this rank's rows of x; w_band: (S*B, Cw, Hb, W)
    this rank's rows of every weight plane; Hg: rows of the whole image.
    Bands follow `band_rows(Hg, world, rank)` and must be at least R rows
    tall.  Returns this band's (U, Z) rows."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    row0, Hb = band_rows(Hg, world, rank)
    if x_band.shape[2] != Hb:
        raise RuntimeError(f"rank {rank}: band has {x_band.shape[2]} rows, "
                           f"expected {Hb}")
    R = radius_of(shifts)
    x_ext = exchange_x_halo(x_band, R, group)
    U, Z, top, bot = compute(x_ext, w_band, shifts, row0, Hg)
    if R == 0 or world == 1:
        return U, Z
    from_below, from_above = exchange_strips(top, bot, group)
    return _add_strips(U, Z, from_below, from_above)
