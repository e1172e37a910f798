"""Failure handling of the tiled kernels' bounded waits, without a GPU
fault: the test hook nsc_test_wait_fault leaves one weight copy per CTA
unissued, so the consumers' waits on it run out (a barrier that nothing
completes).  The kernel must return, the host must see NSC_ERR_TIMEOUT from
nsc_check_waits, and the context must stay usable: a clean run afterwards
matches the oracle and reports no timeout."""

import pytest
import torch

import neural_shift_cuda_b200 as nsc
from neural_shift_cuda_b200 import _lib
from oracle import nsc_oracle as O

pytestmark = pytest.mark.gpu


def _case():
    torch.manual_seed(3)
    sh = torch.tensor(O.halfplane_shifts(3))
    x = torch.rand(1, 3, 64, 256, dtype=torch.float16)
    w = torch.rand(len(sh), 1, 64, 256, dtype=torch.float16)
    return x, w, sh


@pytest.mark.parametrize("op", ["accumulate", "normalized"])
def test_skipped_copy_times_out_and_context_survives(cuda, monkeypatch, op):
    monkeypatch.setenv("NSC_REQUIRE_FAST", "1")
    x, w, sh = _case()
    xc, wc = x.to(cuda), w.to(cuda)

    def run():
        if op == "accumulate":
            return nsc.accumulate_uz(xc, wc, sh)
        return nsc.normalized_accumulate_uz(xc, wc, sh, return_log_degree=True,
                                            validate=False)
    run()
    _lib.check_device_waits()               # clean baseline
    before = _lib.wait_timeouts()
    _lib.test_wait_fault(skip_copy=2, wait_budget=4)
    try:
        run()                                # returns early, outputs undefined
        with pytest.raises(RuntimeError, match="NSC_ERR_TIMEOUT"):
            _lib.check_device_waits()
    finally:
        _lib.test_wait_fault(-1, 0)
    assert _lib.wait_timeouts() > before
    # the context is intact: a clean run is correct and reports nothing
    out = run()
    _lib.check_device_waits()
    if op == "accumulate":
        Ur, Zr = O.accumulate_uz(x, w.expand(-1, 3, -1, -1), sh)
        torch.testing.assert_close(out[0].cpu(), Ur, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(out[1].cpu(), Zr, rtol=1e-5, atol=1e-5)
    else:
        Dr, Lr = O.normalized_accumulate_uz(x, w.expand(-1, 3, -1, -1), sh, False)
        torch.testing.assert_close(out[0].cpu(), Dr, rtol=1e-5, atol=1e-5)
        torch.testing.assert_close(out[1].cpu(), Lr, rtol=1e-5, atol=1e-5)
