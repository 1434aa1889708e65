"""The six reference-named C++ launchers that libcmpx.so exports, called on a
B200 exactly as a binary linked against the reference would call them: by
their mangled C++ names, with device pointers and packed row-major strides,
on the legacy default stream (reference src/main.cpp:12-19).

  launch_matmul_{fp16,bf16,fp32}  vs the CPU oracle's error (the reference
      kernel's arithmetic) + the path tolerance, on odd shapes and config 1
      (fp16_matmul.cu:301-340, bf16_matmul.cu:232-254, fp32_matmul.cu:236-265);
  launch_add_bias_{fp16,bf16,fp32} on the column counts the reference gets
      wrong: odd N for fp16 (skipped there, fp16_matmul.cu:357-366) and
      N % 4 != 0 for fp32 (fp32_matmul.cu:186-227, 272-287).  The result must
      be C + bias computed in fp32 and rounded once, and within half an output
      ulp of the fp64 sum.
"""
import ctypes

import numpy as np
import pytest
import torch

import cabi
from oracle import oracle as o

pytestmark = pytest.mark.gpu

MATMUL = {
    torch.float16: "_Z18launch_matmul_fp16PKvS0_Pviii",
    torch.bfloat16: "_Z18launch_matmul_bf16PKvS0_Pviii",
    torch.float32: "_Z18launch_matmul_fp32PKfS0_Pfiii",
}
ADD_BIAS = {
    torch.float16: "_Z20launch_add_bias_fp16PvPKvii",
    torch.bfloat16: "_Z20launch_add_bias_bf16PvPKvii",
    torch.float32: "_Z20launch_add_bias_fp32PfPKfii",
}
KIND = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}
TOL = {torch.float16: 1e-3, torch.bfloat16: 1e-3, torch.float32: 1e-5}


def _sym(name):
    f = getattr(cabi.lib(), name)
    f.restype = None
    if "matmul" in name:
        f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
    else:
        f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
    return f


def _bits(t):
    t = t.cpu()
    return t.numpy() if t.dtype == torch.float32 else t.view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("dtype,M,N,K", [
    (torch.float32, 257, 383, 511),   # config 1, the odd shape
    (torch.float32, 300, 264, 136),   # 3xTF32 tensor-core path
    (torch.float16, 130, 200, 72),
    (torch.float16, 16, 1000, 520),   # decode-shaped: skinny path
    (torch.bfloat16, 77, 136, 520),
    (torch.bfloat16, 384, 512, 320),  # CTA-pair tile kernel
    (torch.bfloat16, 33, 17, 45),     # unaligned rows: CUDA-core fallback
])
def test_launch_matmul_symbols(cuda, dtype, M, N, K):
    g = torch.Generator().manual_seed(11)
    A = torch.randn(M, K, generator=g).to(dtype)
    B = (torch.randn(K, N, generator=g) * (0.02 if dtype == torch.bfloat16 else 1.0)).to(dtype)
    dA, dB = A.cuda(), B.cuda()
    dC = torch.full((M, N), float("nan"), dtype=dtype, device="cuda")
    torch.cuda.synchronize()
    _sym(MATMUL[dtype])(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), M, N, K)
    torch.cuda.synchronize()
    assert not torch.isnan(dC.float()).any()
    C64 = o.fp64_matmul(KIND[dtype], _bits(A), _bits(B))
    ref = o.bits_to_f64(KIND[dtype], o.oracle_matmul(KIND[dtype], _bits(A), _bits(B)))
    err = o.normwise_err(dC.double().cpu().numpy(), C64)
    ref_err = o.normwise_err(ref, C64)
    assert err <= ref_err + TOL[dtype], (err, ref_err)
    assert cabi.device_error() == 0


@pytest.mark.parametrize("dtype,rows,cols", [
    (torch.float16, 37, 255),     # odd N: the reference's fp16 launcher adds nothing
    (torch.float16, 5, 1),
    (torch.bfloat16, 129, 333),
    (torch.float32, 64, 383),     # N % 4 == 3: the reference's float4 loop misplaces columns
    (torch.float32, 7, 6),
    (torch.float32, 1000, 1030),
    (torch.bfloat16, 70000, 3),   # more rows than one grid row of blocks
])
def test_launch_add_bias_symbols(cuda, dtype, rows, cols):
    g = torch.Generator().manual_seed(12)
    C = torch.randn(rows, cols, generator=g).to(dtype)
    bias = torch.randn(cols, generator=g).to(dtype)
    dC, db = C.cuda(), bias.cuda()
    torch.cuda.synchronize()
    _sym(ADD_BIAS[dtype])(dC.data_ptr(), db.data_ptr(), rows, cols)
    torch.cuda.synchronize()
    got = dC.cpu()
    want = (C.float() + bias.float()[None, :]).to(dtype)   # fp32 add, one rounding
    assert np.array_equal(_bits(got), _bits(want)), "not C + bias rounded once"
    exact = C.double() + bias.double()[None, :]
    ulp = {torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7, torch.float32: 2.0 ** -23}[dtype]
    floor = {torch.float16: 2.0 ** -25, torch.bfloat16: 2.0 ** -134, torch.float32: 2.0 ** -150}[dtype]
    bound = 0.5 * ulp * exact.abs() + floor  # relative half ulp; half the smallest subnormal
    # fp32 for the sum of two 16-bit values is exact, so one rounding is within
    # half an ulp; fp32 inputs: the fp32 add itself is the one rounding.
    assert ((got.double() - exact).abs() <= bound * (1 + 1e-12)).all()


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_cmpx_add_bias_on_stream(cuda, dtype):
    """The extern "C" form of the same kernel on a non-default stream."""
    g = torch.Generator().manual_seed(13)
    rows, cols = 300, 129
    C = torch.randn(rows, cols, generator=g).to(dtype)
    bias = torch.randn(cols, generator=g).to(dtype)
    dC, db = C.cuda(), bias.cuda()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    st = cabi.lib().cmpx_add_bias(cabi.dtype_code(dtype), dC.data_ptr(), db.data_ptr(), rows, cols, s.cuda_stream)
    assert st == cabi.OK
    s.synchronize()
    want = (C.float() + bias.float()[None, :]).to(dtype)
    assert np.array_equal(_bits(dC), _bits(want))
