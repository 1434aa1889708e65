"""cmpx_matmul_skinny_noalloc: the decode-shape matmul for callers that may
not allocate device memory (fixed memory budgets, allocator hooks, processes
that set the device up once).  It runs the same skinny kernel as cmpx_gemm,
with its scratch in a fixed array inside libcmpx.so instead of cudaMalloc'd
memory.

This file is collected last on purpose: it is checked both after every other
GPU test (the library's workspaces and the fixed array already used) and on
its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

import cabi
from oracle import oracle as o

pytestmark = pytest.mark.gpu


def _fn():
    f = cabi.lib().cmpx_matmul_skinny_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
    return f


def _noalloc(A, B, C, bias, M, N, K, layout):
    return _fn()(cabi.dtype_code(A.dtype), A.data_ptr(), B.data_ptr(), C.data_ptr(),
                 bias.data_ptr() if bias is not None else None, M, N, K, layout,
                 torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("dtype,M,N,K,layout,bias", [
    (torch.float16, 16, 28672, 8192, cabi.B_KN, False),   # config 4, the decode shape
    (torch.bfloat16, 7, 1000, 520, cabi.B_NK, True),
    (torch.float16, 64, 4096, 2048, cabi.B_NK, False),
])
def test_noalloc_matches_gemm_twice(cuda, dtype, M, N, K, layout, bias):
    g = torch.Generator(device="cuda").manual_seed(3)
    A = torch.randn(M, K, generator=g, device="cuda").to(dtype)
    Bshape = (K, N) if layout == cabi.B_KN else (N, K)
    B = (torch.randn(Bshape, generator=g, device="cuda") * 0.02).to(dtype)
    bvec = torch.randn(N, generator=g, device="cuda").to(dtype) if bias else None
    # fp64 ground truth of the same product (exact inputs, fp64 accumulation)
    Bkn = B if layout == cabi.B_KN else B.t()
    C64 = (A.double() @ Bkn.double() + (bvec.double()[None, :] if bias else 0)).cpu().numpy()
    # the reference's arithmetic (CPU oracle: 16-bit accumulation, then its
    # separate bias add, rounded once) on a few rows
    rows = list(range(min(M, 4)))
    kind = "f16" if dtype == torch.float16 else "bf16"
    bits = lambda t: t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    refc = o.bits_to_f64(kind, o.oracle_matmul(kind, bits(A[rows]), bits(Bkn.contiguous())))
    if bias:
        refc = (torch.from_numpy(refc).float() + bvec.float().cpu()[None, :]).to(dtype).double().numpy()
    ref_err = o.normwise_err(refc, C64[rows])
    ref = torch.empty((M, N), dtype=dtype, device="cuda")
    args = cabi.gemm_args(A, B, ref, bias=bvec, b_layout=layout, path=cabi.PATH_SKINNY)
    assert cabi.gemm(args, torch.cuda.current_stream().cuda_stream) == cabi.OK
    for _ in range(2):  # the fixed scratch keeps the previous call's contents
        C = torch.full((M, N), float("nan"), dtype=dtype, device="cuda")
        st = _noalloc(A, B, C, bvec, M, N, K, layout)
        assert st == cabi.OK, cabi.lib().cmpx_status_string(st)
        torch.cuda.synchronize()
        assert not torch.isnan(C.float()).any()
        # the path's contract against fp64 on the sampled rows:
        # err <= err(reference kernel's arithmetic, the CPU oracle) + 1e-3
        err64 = o.normwise_err(C[rows].double().cpu().numpy(), C64[rows])
        assert err64 <= ref_err + 1e-3, (err64, ref_err)
        # and the same numbers as cmpx_gemm's skinny path (same kernel, its
        # scratch from the library workspace instead of the fixed array)
        err = o.normwise_err(C.double().cpu().numpy(), ref.double().cpu().numpy())
        assert err <= 1e-3, err
    assert cabi.device_error() == 0


def test_noalloc_rejects_out_of_range_sizes(cuda):
    A = torch.zeros((65, 64), dtype=torch.float16, device="cuda")
    B = torch.zeros((64, 128), dtype=torch.float16, device="cuda")
    C = torch.zeros((65, 128), dtype=torch.float16, device="cuda")
    assert _noalloc(A, B, C, None, 65, 128, 64, cabi.B_KN) == cabi.ERR_TOO_LARGE    # M > 64
    huge_n = 16384 * 128 + 8                                                       # > 16384 slabs
    assert _noalloc(A, B, C, None, 16, huge_n, 64, cabi.B_KN) == cabi.ERR_TOO_LARGE
    assert _noalloc(A, B, C, None, 16, 128, 64, 7) == cabi.ERR_INVALID_ARG
    assert b"fixed scratch" in cabi.lib().cmpx_status_string(cabi.ERR_TOO_LARGE)
