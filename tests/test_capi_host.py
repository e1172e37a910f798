"""CPU-only checks of the C ABI and the host-side logic: the library loads,
exports every symbol the header declares, and rejects bad arguments before
touching a device (no compute call is made here)."""

import ctypes
import os
import re

import pytest
import torch

import neural_shift_cuda_b200 as nsc
from neural_shift_cuda_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "nsc_b200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"NSC_API\s+[\w\s\*]*?\b(nsc_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    assert "nsc_accumulate_uz_fwd" in names and len(names) >= 15


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    for name in _declared():
        assert hasattr(lib, name), name
    # and the Python binding knows each of them
    assert set(_declared()) <= set(_lib.EXPORTED)


def test_index_width_marker():
    assert nsc.index_width_bits() == 64
    assert _lib.version().startswith("0.12.0")


def _shift_arr(rows):
    t = torch.tensor(rows, dtype=torch.int64)
    return t, ctypes.cast(t.data_ptr(), ctypes.POINTER(ctypes.c_int64))


def _status(name, *args):
    lib = _lib.load()
    st = getattr(lib, name)(*args)
    return st, lib.nsc_last_error_string().decode()


def test_rejects_s_out_of_range():
    t, p = _shift_arr([[0, 0, 0]])
    st, msg = _status("nsc_accumulate_uz_fwd", None, 2, None, 2, 1, 1, 1, 4, 4,
                      p, 0, None, None, None)
    assert st == 3 and "1 <= S <= 1024" in msg
    big = torch.zeros(1025, 3, dtype=torch.int64)
    st, msg = _status("nsc_accumulate_uz_fwd", None, 2, None, 2, 1, 1, 1, 4, 4,
                      ctypes.cast(big.data_ptr(), ctypes.POINTER(ctypes.c_int64)),
                      1025, None, None, None)
    assert st == 3


def test_rejects_shift_beyond_extent():
    t, p = _shift_arr([[5, 0, 1]])
    st, msg = _status("nsc_accumulate_uz_fwd", None, 2, None, 2, 1, 1, 1, 4, 4,
                      p, 1, None, None, None)
    assert st == 1 and "exceeds the image extent" in msg


def test_rejects_dtype_pairs_and_channels():
    t, p = _shift_arr([[0, 1, 1]])
    st, _ = _status("nsc_accumulate_uz_fwd", None, 0, None, 2, 1, 1, 1, 4, 4,
                    p, 1, None, None, None)
    assert st == 2  # fp16 x with fp32 w
    st, _ = _status("nsc_accumulate_uz_fwd", None, 3, None, 2, 1, 1, 1, 4, 4,
                    p, 1, None, None, None)
    assert st == 2  # fp64 mixed
    st, msg = _status("nsc_accumulate_uz_fwd", None, 2, None, 2, 2, 1, 3, 4, 4,
                      p, 1, None, None, None)
    assert st == 1 and "channel-broadcast" in msg


def test_empty_extents_are_noops():
    t, p = _shift_arr([[0, 1, 1]])
    st, _ = _status("nsc_accumulate_uz_fwd", None, 2, None, 2, 1, 0, 1, 4, 4,
                    p, 1, None, None, None)
    assert st == 0


def test_null_pointers_rejected():
    t, p = _shift_arr([[0, 1, 1]])
    st, msg = _status("nsc_accumulate_uz_fwd", None, 2, None, 2, 1, 1, 1, 4, 4,
                      p, 1, None, None, None)
    assert st == 1 and "NULL" in msg


def test_metropolis_checks():
    t, p = _shift_arr([[0, 1, 1]])
    st, msg = _status("nsc_metropolis_fwd", None, 2, 1, None, 2, 1, 8, 4, 4,
                      p, 1, 1, ctypes.c_double(1e-6), None, None, None, None)
    assert st == 1 and "C <= 4" in msg
    st, msg = _status("nsc_metropolis_fwd", None, 2, 1, None, 2, 1, 3, 4, 4,
                      p, 1, 1, ctypes.c_double(0.0), None, None, None, None)
    assert st == 1 and "eps" in msg


def test_band_checks():
    t, p = _shift_arr([[3, 1, 1]])
    st, msg = _status("nsc_accumulate_uz_band_fwd", None, 2, None, 2, 1, 1, 1,
                      2, 8, 0, 16, p, 1, None, None, None)
    assert st == 1 and "thinner" in msg
    st, msg = _status("nsc_accumulate_uz_band_fwd", None, 2, None, 2, 1, 1, 1,
                      8, 8, 12, 16, p, 1, None, None, None)
    assert st == 1 and "outside image" in msg


def test_ops_refuse_cpu_tensors():
    x = torch.ones(1, 1, 4, 4)
    with pytest.raises(RuntimeError, match="no CPU path"):
        nsc.accumulate_uz(x, torch.ones(1, 1, 4, 4), torch.tensor([[0, 0, 0]]))
    with pytest.raises(RuntimeError, match="no CPU path"):
        nsc.shift_gather(x, torch.tensor([[0, 1]]))


def test_shift_shape_errors_match_reference():
    x = torch.ones(1, 1, 4, 4)
    with pytest.raises(ValueError, match=r"shifts must be \(S, 2\) or \(S, 3\)"):
        nsc.shift_gather(x, torch.zeros(3, dtype=torch.int64))
    with pytest.raises(ValueError, match=r"requires shifts of shape \(S, 3\)"):
        nsc.accumulate_uz(x, x, torch.zeros(1, 2, dtype=torch.int64))
    with pytest.raises(TypeError, match="floating point"):
        nsc.accumulate_uz(x.long(), x, torch.zeros(1, 3, dtype=torch.int64))


def test_host_shift_cache_roundtrip():
    large = 2 ** 31 + 17
    t = torch.tensor([[large, -large, 0]], dtype=torch.int32 if False else torch.int64)
    hs = _lib.host_shifts(t)
    assert hs.t.dtype == torch.int64 and hs.rows() == [(large, -large, 0)]
    hs2 = _lib.host_shifts([(1, -2, True), (0, 0, False)])
    assert hs2.rows() == [(1, -2, 1), (0, 0, 0)]
    assert _lib.host_shifts(torch.tensor([[1, -2, 1]], dtype=torch.int32)).t.dtype \
        == torch.int64


def test_transposed_rows_only_for_accumulate():
    """Column value 3 (transposed row) is an accumulate_uz table value; the
    normalized entry point rejects it before any launch, and values outside
    0..3 are rejected everywhere."""
    t, p = _shift_arr([[0, 1, 3], [1, 0, 3]])
    st, msg = _status("nsc_normalized_accumulate_uz_fwd", None, 2, None, 2, 1, 1,
                      1, 4, 4, p, 2, 1, None, None, None, None)
    assert st != 0 and "accumulate_uz only" in msg
    t, p = _shift_arr([[0, 1, 5]])
    st, msg = _status("nsc_accumulate_uz_fwd", None, 2, None, 2, 1, 1, 1, 4, 4,
                      p, 1, None, None, None)
    assert st != 0 and "0..3 expected" in msg
