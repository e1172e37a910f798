"""The allocation-free metropolis forward, `nsc_metropolis_fwd_noalloc`.

Some callers cannot allocate device memory: a plugin whose host framework
owns every allocation and passes it only the input and output buffers, or
code that must not call cudaMalloc because that can synchronize the device
or fail in the middle of a run.  For them the library keeps the degree map
of the metropolis forward in a fixed built-in scratch array.  These tests
call it through the C ABI and check it against `nsc_metropolis_fwd` (which
takes a caller-allocated degree buffer) on two calls in a row, with the
tolerance the other fp32 parity tests use.  The file is named so that
pytest collects it last.
"""

import ctypes

import pytest
import torch

from neural_shift_cuda_b200 import _lib
from oracle import nsc_oracle as O

pytestmark = pytest.mark.gpu


def _run(name, w, x, rows, use_box, eps, degree=None):
    hs = _lib.host_shifts(rows)
    B, S, Cw, H, W = w.shape
    C = x.shape[1]
    Wx = torch.empty_like(x)
    dh = torch.empty_like(x)
    args = [_lib.ptr(w), _lib.dtype_code(w.dtype), Cw, _lib.ptr(x),
            _lib.dtype_code(x.dtype), B, C, H, W, hs.ptr, hs.S,
            int(use_box), ctypes.c_double(eps), _lib.ptr(Wx), _lib.ptr(dh)]
    if degree is not None:
        args.append(_lib.ptr(degree))
    args.append(_lib.stream_of(x))
    with torch.cuda.device(x.device):
        _lib.call(name, *args)
    return Wx, dh


def _case(seed, B, C, Cw, H, W, R, dev):
    g = torch.Generator().manual_seed(seed)
    rows = O.halfplane_shifts(R)
    w = torch.sigmoid(torch.randn(B, len(rows), Cw, H, W, generator=g))
    x = torch.rand(B, C, H, W, generator=g)
    return w.to(dev), x.to(dev), rows


def test_noalloc_matches_allocating_entry_point(cuda):
    # second call: a smaller problem, so stale scratch contents from the
    # first call would show up if the degree pass did not overwrite them
    for seed, (B, C, Cw, H, W, R), use_box in [
            (0, (4, 3, 1, 64, 96, 3), True),
            (1, (2, 2, 2, 33, 40, 2), False)]:
        w, x, rows = _case(seed, B, C, Cw, H, W, R, cuda)
        degree = torch.empty((B, Cw, H, W), dtype=torch.float32, device=cuda)
        Wx_a, dh_a = _run("nsc_metropolis_fwd", w, x, rows, use_box, 1e-6,
                          degree)
        Wx_n, dh_n = _run("nsc_metropolis_fwd_noalloc", w, x, rows, use_box,
                          1e-6)
        torch.cuda.synchronize()
        torch.testing.assert_close(Wx_n, Wx_a, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(dh_n, dh_a, rtol=1e-5, atol=1e-5)


def test_noalloc_rejects_oversized_problem(cuda):
    # 17 * 512 * 512 fp32 values exceed the 16 MiB scratch
    w = torch.zeros(17, 1, 1, 512, 512, device=cuda)
    x = torch.zeros(17, 1, 512, 512, device=cuda)
    with pytest.raises(RuntimeError, match="built-in scratch"):
        _run("nsc_metropolis_fwd_noalloc", w, x, [(0, 0, 0)], True, 1e-6)


def test_noalloc_fp64_at_the_limit_and_one_pixel_kernels(cuda, monkeypatch):
    """fp64 degree values are 8 bytes: B * Cw * H * W = 2^21 fills the
    16 MiB array exactly and one more column is rejected.  With
    NSC_METRO_GENERIC=1 the one-pixel degree and aggregation kernels run
    instead of the tiled ones; both forms must overwrite every scratch value
    they read (two calls in a row, the second smaller)."""
    w, x, rows = _case(5, 2, 3, 1, 1024, 1024, 2, cuda)
    w, x = w.double(), x.double()
    degree = torch.empty((2, 1, 1024, 1024), dtype=torch.float64, device=cuda)
    Wx_a, dh_a = _run("nsc_metropolis_fwd", w, x, rows, True, 1e-6, degree)
    Wx_n, dh_n = _run("nsc_metropolis_fwd_noalloc", w, x, rows, True, 1e-6)
    torch.testing.assert_close(Wx_n, Wx_a, rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(dh_n, dh_a, rtol=1e-12, atol=1e-12)
    wbig = torch.zeros(2, 1, 1, 1024, 1025, dtype=torch.float64, device=cuda)
    xbig = torch.zeros(2, 1, 1024, 1025, dtype=torch.float64, device=cuda)
    with pytest.raises(RuntimeError, match="built-in scratch"):
        _run("nsc_metropolis_fwd_noalloc", wbig, xbig, [(0, 0, 0)], True, 1e-6)
    monkeypatch.setenv("NSC_METRO_GENERIC", "1")
    for seed, (B, C, Cw, H, W, R) in [(6, (2, 3, 1, 40, 48, 3)), (7, (1, 3, 3, 17, 23, 2))]:
        w, x, rows = _case(seed, B, C, Cw, H, W, R, cuda)
        degree = torch.empty((B, Cw, H, W), dtype=torch.float32, device=cuda)
        Wx_a, dh_a = _run("nsc_metropolis_fwd", w, x, rows, True, 1e-6, degree)
        Wx_n, dh_n = _run("nsc_metropolis_fwd_noalloc", w, x, rows, True, 1e-6)
        torch.cuda.synchronize()
        torch.testing.assert_close(Wx_n, Wx_a, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(dh_n, dh_a, rtol=1e-5, atol=1e-5)
