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

The strips need only the rank's own rows, so they are computed first and
both exchanges travel in ONE grouped send/recv (`batch_isend_irecv`, NCCL
over NVLink for CUDA tensors); with a contiguous x buffer each (image,
channel) plane's halo rows are sent from and received into the buffer
itself, with no staging copies.  An overlapped form (off by default: no
faster on 2 B200s) splits the exchange so the x halo travels while the
edge-strip kernel runs and the strips (needed only by the final add)
while the band forward runs.  With `padded=True` the caller's x buffer has
R spare rows above and below the band and the halo is received straight
into them (no band-sized copy per step).  The compute is injectable so the exchange logic runs on CPU `gloo`
ranks in the tests.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch

from . import _lib
from .ops import _require_cuda, _storage_dtypes

__all__ = ["band_rows", "x_ext_from_full", "band_compute_cuda",
           "band_forward_cuda", "band_edges_cuda",
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


def _band_args(x_ext, w_band, shifts):
    _require_cuda("accumulate_uz_band", x_ext, w_band)
    hs = _lib.host_shifts(shifts)
    R = int(hs.t[:, :2].abs().max())
    B, C, He, W = x_ext.shape
    Hb = He - 2 * R
    xd, wd = _storage_dtypes(x_ext, w_band)
    x_k = x_ext.to(xd).contiguous()
    w_k = w_band.to(wd).contiguous()
    acc = torch.float64 if xd == torch.float64 else torch.float32
    return hs, R, B, C, Hb, W, xd, wd, x_k, w_k, acc


def band_forward_cuda(x_ext, w_band, shifts, row0: int, Hg: int):
    """(U, Z) of one band without the cross-band mirror terms.
    x_ext: (B, C, Hb + 2R, W) band rows with R halo rows above and below;
    w_band: (S*B, Cw, Hb, W)."""
    hs, R, B, C, Hb, W, xd, wd, x_k, w_k, acc = _band_args(x_ext, w_band, shifts)
    U = torch.empty((B, C, Hb, W), dtype=acc, device=x_ext.device)
    Z = torch.empty_like(U)
    with torch.cuda.device(x_ext.device):
        _lib.call("nsc_accumulate_uz_band_fwd", _lib.ptr(x_k), _lib.dtype_code(xd),
                  _lib.ptr(w_k), _lib.dtype_code(wd), w_k.size(1), B, C, Hb, W,
                  row0, Hg, hs.ptr, hs.S, _lib.ptr(U), _lib.ptr(Z),
                  _lib.stream_of(x_ext))
    return U, Z


def band_edges_cuda(x_ext, w_band, shifts, row0: int, Hg: int):
    """(top, bot): the (2, B, C, R, W) mirror strips this band's weights
    contribute to the R rows above / below it.  Reads only the band rows of
    x_ext, so the halo rows may still be unset."""
    hs, R, B, C, Hb, W, xd, wd, x_k, w_k, acc = _band_args(x_ext, w_band, shifts)
    top = torch.empty((2, B, C, R, W), dtype=acc, device=x_ext.device)
    bot = torch.empty_like(top)
    if R > 0:
        with torch.cuda.device(x_ext.device):
            _lib.call("nsc_accumulate_uz_band_edges", _lib.ptr(x_k),
                      _lib.dtype_code(xd), _lib.ptr(w_k), _lib.dtype_code(wd),
                      w_k.size(1), B, C, Hb, W, row0, Hg, hs.ptr, hs.S,
                      _lib.ptr(top), _lib.ptr(bot), _lib.stream_of(x_ext))
    return top, bot


def band_rows_cuda(x_ext, w_band, shifts, row0: int, Hg: int, r0: int, r1: int,
                   U: torch.Tensor, Z: torch.Tensor, max_ctas: int = 0) -> None:
    """Write rows [r0, r1) of the band's (U, Z) (see band_forward_cuda);
    max_ctas > 0 caps the persistent kernel's grid."""
    hs, R, B, C, Hb, W, xd, wd, x_k, w_k, acc = _band_args(x_ext, w_band, shifts)
    with torch.cuda.device(x_ext.device):
        _lib.call("nsc_accumulate_uz_band_rows_fwd", _lib.ptr(x_k), _lib.dtype_code(xd),
                  _lib.ptr(w_k), _lib.dtype_code(wd), w_k.size(1), B, C, Hb, W,
                  row0, Hg, r0, r1, int(max_ctas), hs.ptr, hs.S, _lib.ptr(U),
                  _lib.ptr(Z), _lib.stream_of(x_ext))


def band_compute_cuda(x_ext, w_band, shifts, row0: int, Hg: int):
    """(U, Z, top, bot) of one band on its GPU via the C ABI (forward and
    edge strips; see band_forward_cuda / band_edges_cuda)."""
    top, bot = band_edges_cuda(x_ext, w_band, shifts, row0, Hg)
    U, Z = band_forward_cuda(x_ext, w_band, shifts, row0, Hg)
    return U, Z, top, bot


def _add_strips(U, Z, from_below: Optional[torch.Tensor],
                from_above: Optional[torch.Tensor]):
    """Add a neighbour's mirror strips: `from_below` (the lower band's top
    strip) lands on this band's last R rows, `from_above` (the upper band's
    bottom strip) on its first R rows.  CUDA tensors: one launch of
    nsc_accumulate_uz_band_add_strips."""
    strips = [t for t in (from_below, from_above) if t is not None]
    if (U.is_cuda and strips and U.is_contiguous() and Z.is_contiguous()
            and all(t.is_contiguous() and t.dtype == U.dtype for t in strips)):
        B, C, Hb, W = U.shape
        R = strips[0].shape[3]
        with torch.cuda.device(U.device):
            _lib.call("nsc_accumulate_uz_band_add_strips", _lib.ptr(U), _lib.ptr(Z),
                      _lib.dtype_code(U.dtype), B, C, Hb, W, R,
                      _lib.ptr(from_above) if from_above is not None else None,
                      _lib.ptr(from_below) if from_below is not None else None,
                      _lib.stream_of(U))
        return U, Z
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


def _g(r, group):
    import torch.distributed as dist
    return r if group is None else dist.get_global_rank(group, r)


def exchange_halo_and_strips(x_pad: torch.Tensor, R: int, top, bot, group=None):
    """One grouped send/recv: fills the R halo rows of x_pad (rows [0, R)
    and [R + Hb, Hb + 2R), band rows in between) from the ring neighbours,
    sends this band's mirror strips and returns the neighbours' strips
    (from_below, from_above), None at the image edges."""
    return exchange_start(x_pad, R, top, bot, group)()


class BandExchangeError(RuntimeError):
    """A neighbour rank did not complete the band exchange (it left, or
    missed the deadline)."""


def exchange_start(x_pad: torch.Tensor, R: int, top, bot, group=None,
                   halo: bool = True, strips: bool = True,
                   deadline: Optional[float] = None):
    """Issue the grouped send/recv of `exchange_halo_and_strips` -- the x
    halo, the mirror strips or both -- and return a `finish()` that waits
    for it (the current stream waits on the collective), writes the halo
    rows into x_pad and returns (from_below, from_above).  With `deadline`
    (seconds) a send/recv that has not completed in time -- or fails
    because the peer left -- raises BandExchangeError on the host."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    Hb = x_pad.shape[2] - 2 * R
    if world == 1:
        def finish_local():
            if R and halo:
                x_pad[:, :, :R] = x_pad[:, :, Hb:Hb + R]
                x_pad[:, :, R + Hb:] = x_pad[:, :, R:2 * R]
            return None, None
        return finish_local
    up, down = (rank - 1) % world, (rank + 1) % world
    from_up = from_down = from_above = from_below = None
    sends, recvs = [], []
    # Messages between a pair match in issue order (with two ranks `up` and
    # `down` are the same peer): every rank sends last rows, first rows, top
    # strip, bottom strip, and receives in the matching order.
    direct = halo and x_pad.is_contiguous()
    if direct:
        # each (image, channel) plane's halo rows are contiguous: send the
        # band's rows straight from x_pad and receive into its spare rows
        planes = [x_pad[b, c] for b in range(x_pad.shape[0])
                  for c in range(x_pad.shape[1])]
        sends += [(p[Hb:Hb + R], down) for p in planes]          # last R rows
        sends += [(p[R:2 * R], up) for p in planes]              # first R rows
        recvs += [(p[:R], up) for p in planes]
        recvs += [(p[R + Hb:], down) for p in planes]
    elif halo:
        first = x_pad[:, :, R:2 * R].contiguous()      # this band's first R rows
        last = x_pad[:, :, Hb:Hb + R].contiguous()     # this band's last R rows
        from_up = torch.empty_like(last)
        from_down = torch.empty_like(first)
        sends += [(last, down), (first, up)]
        recvs += [(from_up, up), (from_down, down)]
    if strips:
        from_above = torch.empty_like(bot) if rank > 0 else None
        from_below = torch.empty_like(top) if rank + 1 < world else None
        if rank > 0:
            sends.append((top.contiguous(), up))
        if rank + 1 < world:
            sends.append((bot.contiguous(), down))
        if from_above is not None:
            recvs.append((from_above, up))
        if from_below is not None:
            recvs.append((from_below, down))
    ops = ([dist.P2POp(dist.isend, t, _g(r, group), group) for t, r in sends]
           + [dist.P2POp(dist.irecv, t, _g(r, group), group) for t, r in recvs])
    reqs = dist.batch_isend_irecv(ops) if ops else []

    def finish():
        for req in reqs:
            if deadline is None:
                req.wait()
                continue
            from datetime import timedelta
            try:
                done = req.wait(timeout=timedelta(seconds=deadline))
            except RuntimeError as e:
                raise BandExchangeError(
                    f"rank {rank}: band exchange with ranks {up} / {down} failed "
                    f"within {deadline} s: {e}") from e
            if done is False:
                raise BandExchangeError(
                    f"rank {rank}: band exchange with ranks {up} / {down} did not "
                    f"complete within {deadline} s")
        if halo and not direct:
            x_pad[:, :, :R] = from_up
            x_pad[:, :, R + Hb:] = from_down
        return from_below, from_above
    return finish


def _reserve_sms() -> int:
    import os
    return int(os.environ.get("NSC_BAND_RESERVE_SMS", "0"))


def accumulate_uz_banded(x_band, w_band, shifts, Hg: int, group=None,
                         compute: Optional[Callable] = None, *, padded: bool = False,
                         forward: Callable = band_forward_cuda,
                         edges: Callable = band_edges_cuda,
                         overlap: Optional[bool] = None,
                         deadline: Optional[float] = None):
    """accumulate_uz of this rank's band of a row-split image.

    x_band: (B, C, Hb, W) this rank's rows of x -- or, with padded=True,
    (B, C, Hb + 2R, W) with the band in rows [R, R + Hb) and R spare rows on
    each side that this call overwrites with the halo; w_band: (S*B, Cw,
    Hb, W) this rank's rows of every weight plane; Hg: rows of the whole
    image.  Bands follow `band_rows(Hg, world, rank)` and must be at least R
    rows tall.  Returns this band's (U, Z) rows.  `compute`, when given,
    replaces both `forward` and `edges` with one call returning
    (U, Z, top, bot) (run after the halo arrives).  overlap=True (CUDA
    forward only): the x halo travels during the edge-strip kernel and the
    strips during the band forward, which runs on all but
    NSC_BAND_RESERVE_SMS (default 0) SMs.  It measured no faster than one
    grouped exchange at configs[4]: with 2 reserved SMs 4.69 vs 4.67 ms (2
    B200s) and 2.53 vs 2.51 ms (4 B200s) per step, with none 4.66 vs 4.64 ms
    (2 B200s, medians), so overlap=None takes it from NSC_BAND_OVERLAP=1 and
    defaults to off.  deadline (seconds): an exchange
    that has not completed in time, or whose peer left, raises
    BandExchangeError (the process group's own timeout applies otherwise)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    row0, Hb = band_rows(Hg, world, rank)
    R = radius_of(shifts)
    if x_band.shape[2] != Hb + (2 * R if padded else 0):
        raise RuntimeError(f"rank {rank}: band has {x_band.shape[2]} rows, "
                           f"expected {Hb + (2 * R if padded else 0)}")
    if padded:
        x_pad = x_band
    else:
        x_pad = torch.empty((x_band.shape[0], x_band.shape[1], Hb + 2 * R,
                             x_band.shape[3]), dtype=x_band.dtype,
                            device=x_band.device)
        x_pad[:, :, R:R + Hb] = x_band
    if compute is not None:
        def edges(xe, wb, sh, r0, hg):          # noqa: F811 (injected form)
            return compute(xe, wb, sh, r0, hg)[2:]
        def forward(xe, wb, sh, r0, hg):        # noqa: F811
            return compute(xe, wb, sh, r0, hg)[:2]
    if overlap is None:
        import os
        overlap = os.environ.get("NSC_BAND_OVERLAP", "0") == "1"
    if (overlap and compute is None and forward is band_forward_cuda
            and x_pad.is_cuda):
        # x halo in flight during the edge-strip kernel; the strips in flight
        # during the band forward, which leaves NSC_BAND_RESERVE_SMS SMs to
        # the collective's kernels
        finish_halo = exchange_start(x_pad, R, None, None, group, strips=False,
                                     deadline=deadline)
        top, bot = edges(x_pad, w_band, shifts, row0, Hg)
        finish_strips = exchange_start(x_pad, R, top, bot, group, halo=False,
                                       deadline=deadline)
        finish_halo()
        acc = (torch.float64 if torch.float64 in (x_pad.dtype, w_band.dtype)
               else torch.float32)
        U = torch.empty((x_pad.shape[0], x_pad.shape[1], Hb, x_pad.shape[3]),
                        dtype=acc, device=x_pad.device)
        Z = torch.empty_like(U)
        nsm = torch.cuda.get_device_properties(x_pad.device).multi_processor_count
        reserve = _reserve_sms()
        cap = max(1, nsm - reserve) if world > 1 and reserve > 0 else 0
        band_rows_cuda(x_pad, w_band, shifts, row0, Hg, 0, Hb, U, Z, cap)
        from_below, from_above = finish_strips()
    else:
        top, bot = edges(x_pad, w_band, shifts, row0, Hg)
        from_below, from_above = exchange_start(x_pad, R, top, bot, group,
                                                deadline=deadline)()
        U, Z = forward(x_pad, w_band, shifts, row0, Hg)
    if R == 0 or world == 1:
        return U, Z
    return _add_strips(U, Z, from_below, from_above)
