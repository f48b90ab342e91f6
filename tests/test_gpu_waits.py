"""The bounded device waits report a timeout instead of hanging.

Every mbarrier wait in the library's pipelines (GEMM, attention) goes
through mbar_wait_bounded: after a limited number of probes it records a
bit in the device error word and returns, and the host reads the bit as
CHELIS_CUDA_ERR_TIMEOUT from chelis_cuda_device_status.  Here the limit is
lowered to about a millisecond and a one-CTA probe runs the same wait with
its producer told to skip the arrival (a barrier that nothing completes):
the status must be TIMEOUT, the context must stay usable, and with the
arrival made the same probe must pass.  No GPU fault or hang is involved.
"""
import pytest

from chelis_b200 import lib as L

pytestmark = pytest.mark.gpu


def test_bounded_wait_times_out_and_reports(cuda):
    import torch
    x = torch.zeros(4, device="cuda")
    cuda._prepare(x)
    lib = L.load()
    default = lib.chelis_cuda_get_wait_limit()
    assert default == 1 << 22
    try:
        L.call("chelis_cuda_set_wait_limit", 1000)
        assert lib.chelis_cuda_get_wait_limit() == 1000
        cuda.device_status()  # clean slate
        L.call("chelis_cuda_selftest_bounded_wait", 1)  # producer skips its arrival
        status = lib.chelis_cuda_device_status()
        assert status == 5, (status, L.last_error())  # CHELIS_CUDA_ERR_TIMEOUT
        assert "bounded device wait" in L.last_error()
        # the word was read and cleared; the context is still usable
        assert lib.chelis_cuda_device_status() == 0
        L.call("chelis_cuda_selftest_bounded_wait", 0)  # producer arrives
        assert lib.chelis_cuda_device_status() == 0
        y = (x + 1).sum().item()
        assert y == 4.0
    finally:
        L.call("chelis_cuda_set_wait_limit", 0)
    assert lib.chelis_cuda_get_wait_limit() == default
