"""Failure detection without a GPU fault: every on-chip wait of the library is
bounded, and a wait that gives up records a code (lsb_device_error) and
returns instead of hanging. The self-test kernel waits on an mbarrier that
nothing arrives on; the test checks the status it writes, the recorded code,
the time it took, and that the context still runs kernels afterwards."""
import time

import pytest
import torch

from oracle.rmsnorm import rmsnorm_residual
from lightserve_b200 import _lib
from lightserve_b200.kernels import fused_add_rmsnorm

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_context_stays_usable():
    lib = _lib.load()
    torch.cuda.synchronize()
    lib.lsb_device_error_reset()
    assert lib.lsb_device_error() == 0
    status = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    t0 = time.perf_counter()
    assert lib.lsb_selftest_bounded_wait(status.data_ptr(), _lib.stream_ptr(status.device)) == 0
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(status.item()) == 0          # the wait reported that it gave up
    assert lib.lsb_device_error() == 0xE01  # ... and recorded which wait it was
    assert 0.05 < elapsed < 60.0
    # The context is intact: a kernel runs and matches the oracle.
    x, r = (torch.randn(8, 512, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    w = torch.ones(512, device="cuda", dtype=torch.bfloat16)
    out, h = fused_add_rmsnorm(x, r, w, 1e-6)
    eo, eh = rmsnorm_residual(x, r, w, 1e-6)
    torch.testing.assert_close(out.cpu(), eo, atol=2e-2, rtol=2e-2)
    assert lib.lsb_device_error_reset() == 0xE01
    assert lib.lsb_device_error() == 0


def test_operator_after_timed_out_wait_raises_through_check():
    """A bounded wait that gave up is reported by check_device_errors() (and
    by ServingEngine / bench.py, which call it), once, then cleared."""
    from lightserve_b200 import check_device_errors
    from lightserve_b200._lib import DeviceWaitError

    lib = _lib.load()
    check_device_errors()
    status = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    assert lib.lsb_selftest_bounded_wait(status.data_ptr(), _lib.stream_ptr(status.device)) == 0
    x, r = (torch.randn(8, 512, device="cuda", dtype=torch.bfloat16) for _ in range(2))
    fused_add_rmsnorm(x, r, torch.ones(512, device="cuda", dtype=torch.bfloat16), 1e-6)
    with pytest.raises(DeviceWaitError) as ei:
        check_device_errors()
    assert ei.value.code == 0xE01
    check_device_errors()  # cleared by the read above
