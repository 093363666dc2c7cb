"""Failure detection on the GPU without a fault: a bounded wait that runs out.

Every mbarrier wait in the kernels gives up after a time limit, records
SN_ERR_TIMEOUT in a device status word and unwinds.  sn_diag_bounded_wait
launches one thread that waits, with that same wait, on a barrier nothing
arrives on, with a 1 ms limit: the kernel must return, sn_device_status must
report SN_ERR_TIMEOUT (and clear it on request), and the context must stay
usable for the next kernel.
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

SN_ERR_TIMEOUT = -6


def test_bounded_wait_runs_out_and_reports(cuda_lib):
    assert cuda_lib.sn_device_status(1, None) == 0
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    assert cuda_lib.sn_diag_bounded_wait(1_000_000, None) == 0
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert waited >= 1e-3 and waited < 5.0, waited
    assert cuda_lib.sn_device_status(0, None) == SN_ERR_TIMEOUT
    assert cuda_lib.sn_device_status(1, None) == SN_ERR_TIMEOUT  # read, then cleared
    assert cuda_lib.sn_device_status(0, None) == 0
    # the context is still usable: a GEMV runs and is right
    from sonata_b200.kernels import gemv as G
    W = torch.randn(256, 512, device="cuda").to(torch.bfloat16)
    x = torch.randn(1, 512, device="cuda").to(torch.bfloat16)
    y = G.candidate_cute_splitk(x, W).float()
    ref = x.float() @ W.float().t()
    assert (y - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()
    assert cuda_lib.sn_device_status(1, None) == 0


def test_bounded_wait_limits_are_checked(cuda_lib):
    assert cuda_lib.sn_diag_bounded_wait(10, None) == -1  # below 1 us
    assert cuda_lib.sn_diag_bounded_wait(2_000_000_000, None) == -1  # above 1 s
