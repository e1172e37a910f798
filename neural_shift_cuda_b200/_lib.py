"""ctypes binding of `libnsc_b200.so` (the C ABI in include/nsc_b200.h).

The library is loaded once, from this package's `_lib/` directory (built by
`python -m neural_shift_cuda_b200.build`).  If it is missing or stale the
ops raise at their first CUDA call with the underlying loader error, like
the reference's `_require_cuda_ext` (`neural_shift_cuda/ops.py:510-546`).
There is no CPU path.
"""

from __future__ import annotations

import ctypes
import os
import threading
import weakref
from typing import Optional

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("NSC_LIB_PATH") or os.path.join(
    _HERE, "_lib", "libnsc_b200.so")

NSC_F16, NSC_BF16, NSC_F32, NSC_F64 = 0, 1, 2, 3
_DTYPES = {torch.float16: NSC_F16, torch.bfloat16: NSC_BF16,
           torch.float32: NSC_F32, torch.float64: NSC_F64}

_STATUS = {0: "NSC_OK", 1: "NSC_ERR_INVALID_ARG",
           2: "NSC_ERR_UNSUPPORTED_DTYPE", 3: "NSC_ERR_S_OUT_OF_RANGE",
           4: "NSC_ERR_LAUNCH_FAILED", 5: "NSC_ERR_TIMEOUT"}

_lib: Optional[ctypes.CDLL] = None
_load_error: Optional[BaseException] = None
_lock = threading.Lock()

_P = ctypes.c_void_p
_I = ctypes.c_int
_L = ctypes.c_int64
_D = ctypes.c_double
_LP = ctypes.POINTER(ctypes.c_int64)

# argument lists, in header order
_SIGS = {
    "nsc_shift_gather_fwd": [_P, _I, _L, _L, _L, _L, _LP, _L, _L, _P, _P, _P],
    "nsc_pair_gather_fwd": [_P, _I, _L, _L, _L, _L, _LP, _L, _L, _P, _P, _P],
    "nsc_shift_gather_bwd": [_P, _I, _L, _L, _L, _L, _LP, _L, _L, _P, _P],
    "nsc_pair_gather_bwd": [_P, _I, _L, _L, _L, _L, _LP, _L, _L, _P, _P],
    "nsc_accumulate_uz_fwd": [_P, _I, _P, _I, _L, _L, _L, _L, _L, _LP, _L,
                              _P, _P, _P],
    "nsc_accumulate_uz_bwd": [_P, _I, _P, _I, _L, _L, _L, _L, _L, _LP, _L,
                              _P, _P, _P, _P, _P],
    "nsc_accumulate_uz_band_fwd": [_P, _I, _P, _I, _L, _L, _L, _L, _L, _L,
                                   _L, _LP, _L, _P, _P, _P],
    "nsc_accumulate_uz_band_rows_fwd": [_P, _I, _P, _I, _L, _L, _L, _L, _L, _L,
                                        _L, _L, _L, _I, _LP, _L, _P, _P, _P],
    "nsc_accumulate_uz_band_edges": [_P, _I, _P, _I, _L, _L, _L, _L, _L, _L,
                                     _L, _LP, _L, _P, _P, _P],
    "nsc_accumulate_uz_band_add_strips": [_P, _P, _I, _L, _L, _L, _L, _L, _P,
                                          _P, _P],
    "nsc_normalized_accumulate_uz_fwd": [_P, _I, _P, _I, _L, _L, _L, _L, _L,
                                         _LP, _L, _I, _P, _P, _P, _P],
    "nsc_normalized_accumulate_uz_bwd": [_P, _I, _P, _I, _L, _L, _L, _L, _L,
                                         _LP, _L, _I, _P, _P, _P, _P, _P, _P,
                                         _P],
    "nsc_metropolis_fwd": [_P, _I, _L, _P, _I, _L, _L, _L, _L, _LP, _L, _I,
                           _D, _P, _P, _P, _P],
    "nsc_metropolis_fwd_noalloc": [_P, _I, _L, _P, _I, _L, _L, _L, _L, _LP,
                                   _L, _I, _D, _P, _P, _P],
    "nsc_metropolis_bwd": [_P, _I, _L, _P, _I, _L, _L, _L, _L, _LP, _L, _I,
                           _D, _P, _P, _P, _P, _P, _P, _P, _P],
    "nsc_check_waits": [_P],
    "nsc_nectr_fused_fwd": [_P, _P, _I, _L, _L, _L, _L, _L, _I,
                            ctypes.POINTER(ctypes.c_double), _L, _D, _D, _D, _D,
                            _LP, _L, _I, _P, _P, _P, _P],
}

EXPORTED = ["nsc_index_width_bits", "nsc_version", "nsc_last_error_string",
            "nsc_wait_timeouts", "nsc_test_wait_fault", *_SIGS]


def load() -> ctypes.CDLL:
    """Load the library (once); raise RuntimeError with the cause if absent."""
    global _lib, _load_error
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        try:
            lib = ctypes.CDLL(LIB_PATH)
            lib.nsc_index_width_bits.restype = ctypes.c_int
            lib.nsc_version.restype = ctypes.c_char_p
            lib.nsc_last_error_string.restype = ctypes.c_char_p
            lib.nsc_wait_timeouts.restype = ctypes.c_uint
            lib.nsc_test_wait_fault.argtypes = [ctypes.c_int, ctypes.c_uint]
            lib.nsc_test_wait_fault.restype = None
            for name, args in _SIGS.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = ctypes.c_int
        except (OSError, AttributeError) as e:
            _load_error = e
            raise RuntimeError(
                f"neural_shift_cuda_b200: cannot load the kernel library "
                f"{LIB_PATH}: {type(e).__name__}: {e}. Build it with "
                f"`python -m neural_shift_cuda_b200.build`.") from e
        _lib = lib
        return lib


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def index_width_bits() -> int:
    return int(load().nsc_index_width_bits())


def wait_timeouts() -> int:
    """Bounded device waits that gave up on the current device (synchronizes)."""
    return int(load().nsc_wait_timeouts())


def check_device_waits(device=None) -> None:
    """Synchronize the current stream of `device` and raise RuntimeError
    ([NSC_ERR_TIMEOUT]) if a bounded device wait gave up since the previous
    check: a tiled kernel then returned early with undefined outputs."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    with torch.cuda.device(dev):
        call("nsc_check_waits", ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))


def test_wait_fault(skip_copy: int = -1, wait_budget: int = 0) -> None:
    """Test hook (nsc_test_wait_fault): leave copy `skip_copy` of every CTA
    of later tiled launches unissued, with `wait_budget` ~1 ms sleeps per
    bounded wait; (-1, 0) restores normal operation."""
    load().nsc_test_wait_fault(int(skip_copy), int(wait_budget))


def version() -> str:
    return load().nsc_version().decode()


def call(name: str, *args) -> None:
    """Call a library entry point and map a non-zero status to an error.

    Argument errors raise RuntimeError with the library's message, which
    mirrors the reference's TORCH_CHECK messages (csrc/shift_ops.cpp)."""
    lib = load()
    st = getattr(lib, name)(*args)
    if st != 0:
        msg = lib.nsc_last_error_string().decode()
        raise RuntimeError(f"{msg} [{_STATUS.get(st, st)}]")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPES[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


def ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


# ---------------------------------------------------------------------------
# host copies of shift tables
# ---------------------------------------------------------------------------

class HostShifts:
    """A contiguous int64 host copy of a shift table, kept alive while the
    ctypes pointer is in use."""

    __slots__ = ("t", "S", "cols", "modes")

    def __init__(self, t: torch.Tensor):
        self.t = t
        self.S = int(t.shape[0])
        self.cols = int(t.shape[1])
        self.modes = {}

    @property
    def ptr(self):
        return ctypes.cast(self.t.data_ptr(), _LP)

    def rows(self):
        return [tuple(int(v) for v in r) for r in self.t.tolist()]


def mirror_mode(hs: HostShifts, periodic: bool, transpose: bool = False) -> HostShifts:
    """The table as the library reads it: column 2 becomes 0 (no mirror),
    1 (masked mirror, the reference's meaning of any nonzero value) or, with
    periodic=True, 2 (periodic mirror) for every row with a mirror term.
    transpose=True turns every (forward-only) row into 3: the row then adds
    w_s(p - d) x(p - d), read circularly, and no forward term."""
    if transpose:
        if hs.cols == 3 and bool((hs.t[:, 2] != 0).any()):
            raise ValueError("transpose=True needs forward-only rows "
                             "(has_inv == 0 on every row)")
        key = "T"
        hit = hs.modes.get(key)
        if hit is None:
            t = torch.zeros((hs.S, 3), dtype=torch.int64)
            t[:, :2] = hs.t[:, :2]
            t[:, 2] = 3
            hit = HostShifts(t.contiguous())
            hs.modes[key] = hit
        return hit
    if hs.cols != 3:
        return hs
    key = bool(periodic)
    hit = hs.modes.get(key)
    if hit is not None:
        return hit
    col = hs.t[:, 2]
    if not periodic and bool(((col == 0) | (col == 1)).all()):
        res = hs
    else:
        t = hs.t.clone()
        t[:, 2] = (col != 0).to(torch.int64) * (2 if periodic else 1)
        res = HostShifts(t.contiguous())
    hs.modes[key] = res
    return res


_shift_cache: dict = {}


def _drop(key):
    _shift_cache.pop(key, None)


def host_shifts(shifts) -> HostShifts:
    """Int64 host copy of `shifts` ((S, 2|3) tensor, or a list of rows).

    A device tensor is copied to the host once and cached per tensor object
    and version, so a model that keeps its shift tensor on the GPU (as the
    reference's installers do) pays one device-to-host copy, not one per
    call."""
    if not isinstance(shifts, torch.Tensor):
        rows = [[int(v) for v in r] for r in shifts]
        t = torch.tensor(rows, dtype=torch.int64).reshape(len(rows), -1)
        return HostShifts(t.contiguous())
    if shifts.device.type == "cpu":
        return HostShifts(shifts.detach().to(torch.int64).contiguous())
    key = id(shifts)
    hit = _shift_cache.get(key)
    ver = shifts._version
    if hit is not None and hit[0]() is shifts and hit[1] == ver:
        return hit[2]
    hs = HostShifts(shifts.detach().to("cpu", torch.int64).contiguous())
    _shift_cache[key] = (weakref.ref(shifts), ver, hs)
    weakref.finalize(shifts, _drop, key)
    return hs
