"""Failure detection without a GPU fault: the bounded wait every GEMM
pipeline role uses gives up after its limit, records an error code in the
device error word and returns, and the device keeps working."""
import ctypes

import pytest
import torch

import cabi

pytestmark = pytest.mark.gpu


def _selftest(ns):
    f = cabi.lib().cmpx_selftest_bounded_wait
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_ulonglong, ctypes.c_void_p]
    return f(ns, torch.cuda.current_stream().cuda_stream)


def test_bounded_wait_expires_and_reports(cuda):
    assert cabi.device_error() == 0
    assert _selftest(50_000_000) == cabi.ERR_DEVICE  # 50 ms limit, nothing completes the barrier
    assert cabi.device_error() == 6                   # recorded by the kernel...
    assert cabi.device_error() == 0                   # ...and cleared by reading it
    # the context is intact: a GEMM afterwards runs and is correct
    A = torch.randn(256, 128, device="cuda", dtype=torch.float16)
    B = torch.randn(128, 256, device="cuda", dtype=torch.float16)
    C = torch.empty(256, 256, device="cuda", dtype=torch.float16)
    assert cabi.gemm(cabi.gemm_args(A, B, C)) == cabi.OK
    torch.cuda.synchronize()
    assert (C.float() - A.float() @ B.float()).abs().max().item() < 0.1
    assert cabi.device_error() == 0
