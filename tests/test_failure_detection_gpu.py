"""Failure detection on the GPU without a fault: the bounded wait every kernel uses gives up,
records KF_ERR_DEVICE_TIMEOUT in a device error word, and returns, so the host reads status 6
through kf_query_device_error and the CUDA context keeps working (kf_selftest_bounded_wait waits
on an mbarrier that nothing ever arrives on)."""

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA is required")
    from kernelforge_b200 import _lib

    return _lib


def test_bounded_wait_reports_timeout_and_context_survives(lib):
    dev = torch.device("cuda", torch.cuda.current_device())
    assert lib.query_device_error(dev) == 0  # clears any earlier word
    t0 = time.perf_counter()
    with torch.cuda.device(dev):
        lib.check(lib.lib.kf_selftest_bounded_wait(lib.stream_handle(dev)), "kf_selftest_bounded_wait")
    assert lib.query_device_error(dev) == 6  # KF_ERR_DEVICE_TIMEOUT
    elapsed = time.perf_counter() - t0
    assert 3.5 < elapsed < 60, elapsed  # the library's 4 s bound
    assert lib.query_device_error(dev) == 0  # reading clears the word
    assert lib.status_string(6) == "a kernel's bounded wait expired"
    # The context still runs kernels correctly.
    from kernelforge_b200.rmsnorm import rmsnorm_forward
    from oracle import rmsnorm as oracle
    from tests.tolerances import assert_rmsnorm_close

    x = torch.randn(64, 1024, device=dev).to(torch.bfloat16)
    w = torch.ones(1024, device=dev, dtype=torch.bfloat16)
    assert_rmsnorm_close(rmsnorm_forward(x, w, 1e-6), oracle.rmsnorm_forward(x.cpu(), w.cpu(), 1e-6))
