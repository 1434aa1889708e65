"""Scaled dot-product attention on the GPU (cmpext3.attention, the C ABI
cmpx_attention and the reference-named launch_attention_* symbols) against
the fp64 definition softmax(scale * Q K^T) V and against the reference's own
attention kernels (compiled from its sources into oracle/_ref) run on the
same inputs:

    err(build) <= err(reference kernel) + TOL,  err = max|O - O64| / max|O64|

with TOL = 1e-3 (fp16 / bf16) and 1e-5 (fp32), on the shapes the reference's
kernels handle (fp16: D = 128).  Every case also has a fixed bound against
fp64 (the tensor-core kernel rounds P to 16 bits once; the output once).
"""
import ctypes
import math

import numpy as np
import pytest
import torch

import cabi
import cmp_ext_b200 as cx
from oracle import oracle as o

pytestmark = pytest.mark.gpu

KIND = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}
TOL = {torch.float16: 1e-3, torch.bfloat16: 1e-3, torch.float32: 1e-5}
# bound against fp64: P and O each rounded once to the 16-bit type
BOUND = {torch.float16: 4e-3, torch.bfloat16: 3e-2, torch.float32: 2e-5}


def _fn():
    f = cabi.lib().cmpx_attention
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                  ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    return f


def _inputs(B, H, S, D, dtype, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (torch.randn(B, H, S, D, generator=g, device="cuda").to(dtype) for _ in range(3))
    return q, k, v


def _err(out, q, k, v, scale):
    want = o.fp64_attention(q.double().cpu().numpy(), k.double().cpu().numpy(), v.double().cpu().numpy(), scale)
    return o.normwise_err(out.double().cpu().numpy(), want), want


def _run(q, k, v, scale, path):
    out = torch.full_like(q, float("nan"))
    B, H, S, D = q.shape
    st = _fn()(cabi.dtype_code(q.dtype), q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, S, D,
               scale, path, torch.cuda.current_stream().cuda_stream)
    assert st == cabi.OK, cabi.lib().cmpx_status_string(st)
    torch.cuda.synchronize()
    assert not torch.isnan(out.float()).any(), "output not fully written"
    return out


def _ref_err(q, k, v, scale, want):
    B, H, S, D = q.shape
    kind = KIND[q.dtype]
    if not (o.ref_gpu_available() and o.ref_attention_supported(kind, S, D)):
        return None
    ref = torch.zeros_like(q)
    o.ref_gpu_attention(kind, q.data_ptr(), k.data_ptr(), v.data_ptr(), ref.data_ptr(), B, H, S, D, scale)
    return o.normwise_err(ref.double().cpu().numpy(), want)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("B,H,S", [(1, 1, 128), (2, 3, 200), (1, 2, 77), (1, 2, 1024), (2, 1, 389), (1, 1, 1),
                                   (2, 2, 300), (1, 1, 640)],
                         ids=lambda x: str(x))
def test_tc_attention(cuda, dtype, D, B, H, S):
    q, k, v = _inputs(B, H, S, D, dtype, seed=S + D)
    scale = 1.0 / math.sqrt(D)
    assert cabi.lib().cmpx_attention_select_path(cabi.dtype_code(dtype), q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                  q.data_ptr(), D, cabi.PATH_AUTO) == cabi.PATH_TC
    out = _run(q, k, v, scale, cabi.PATH_TC)
    err, want = _err(out, q, k, v, scale)
    assert err <= BOUND[dtype], err
    ref_err = _ref_err(q, k, v, scale, want)
    if ref_err is not None:
        assert err <= ref_err + TOL[dtype], (err, ref_err)
    # and the same result through the torch operator (AUTO path)
    assert torch.equal(cx.attention(q, k, v, scale=scale), out)
    assert cabi.device_error() == 0


@pytest.mark.parametrize("dtype,D", [(torch.float32, 64), (torch.float32, 128), (torch.float32, 72),
                                     (torch.float16, 80), (torch.bfloat16, 96), (torch.float16, 128),
                                     (torch.float32, 300)])
@pytest.mark.parametrize("S", [1, 130])
def test_simt_attention(cuda, dtype, D, S):
    q, k, v = _inputs(2, 2, S, D, dtype, seed=D)
    scale = 0.3
    out = _run(q, k, v, scale, cabi.PATH_SIMT)
    err, want = _err(out, q, k, v, scale)
    assert err <= BOUND[dtype], err
    ref_err = _ref_err(q, k, v, scale, want)
    if ref_err is not None:
        assert err <= ref_err + TOL[dtype], (err, ref_err)


@pytest.mark.parametrize("dtype,D,top,scale", [
    (torch.float16, 128, 8.0, 1.0),     # the maximum moves by hundreds between blocks
    (torch.bfloat16, 64, 8.0, -1.0),    # negative scale: the row minimum leads
    (torch.float16, 64, 1.5, 1.0),      # the maximum creeps up by less than the rescale step
    (torch.bfloat16, 128, 1.5, 0.5),
])
def test_attention_large_logits(cuda, dtype, D, top, scale):
    """Scores far from zero whose running maximum grows block after block:
    the online softmax must rescale (or keep P within range while it does
    not), never overflow."""
    q, k, v = _inputs(1, 2, 640, D, dtype, seed=5)
    k = k * torch.linspace(0.1, top, 640, device="cuda", dtype=dtype)[None, None, :, None]
    out = _run(q, k, v, scale, cabi.PATH_TC)
    err, _ = _err(out, q, k, v, scale)
    assert err <= BOUND[dtype], err


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_launch_attention_symbols(cuda, dtype):
    """The reference-named C++ launchers (src/main.cpp:48-50) on the legacy
    default stream."""
    name = {torch.float32: "_Z21launch_attention_fp32PKfS0_S0_Pfiiiif",
            torch.float16: "_Z21launch_attention_fp16PKvS0_S0_Pviiiif",
            torch.bfloat16: "_Z21launch_attention_bf16PKvS0_S0_Pviiiif"}[dtype]
    f = getattr(cabi.lib(), name)
    f.restype = None
    f.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 4 + [ctypes.c_float]
    B, H, S, D = 2, 2, 300, 128
    q, k, v = _inputs(B, H, S, D, dtype, seed=9)
    out = torch.full_like(q, float("nan"))
    torch.cuda.synchronize()
    f(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, S, D, 1.0 / math.sqrt(D))
    torch.cuda.synchronize()
    err, want = _err(out, q, k, v, 1.0 / math.sqrt(D))
    assert err <= BOUND[dtype], err
    ref_err = _ref_err(q, k, v, 1.0 / math.sqrt(D), want)
    if ref_err is not None:
        assert err <= ref_err + TOL[dtype], (err, ref_err)


def test_attention_operator_defaults_and_errors(cuda):
    q, k, v = _inputs(1, 2, 64, 64, torch.bfloat16, seed=3)
    out = cx.attention(q, k, v)  # default scale 1/sqrt(D)
    err, _ = _err(out, q, k, v, 1.0 / 8.0)
    assert err <= BOUND[torch.bfloat16]
    with pytest.raises(RuntimeError, match="Dtype mismatch"):
        cx.attention(q, k.half(), v)
    with pytest.raises(RuntimeError, match="Unsupported dtype for attention"):
        cx.attention(q.double(), k.double(), v.double())
    # non-contiguous inputs are made contiguous, as the reference does
    qt = q.transpose(1, 2).contiguous().transpose(1, 2)
    assert torch.equal(cx.attention(qt, k, v), out)
