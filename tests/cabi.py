"""ctypes binding of libcmpx.so's C ABI (include/cmpx.h) for the tests.

The GPU parity tests call the kernels through exactly this boundary: plain
device pointers, sizes, a stream handle and an int status.
"""
from __future__ import annotations

import ctypes
import os
import re

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(REPO, "cmp_ext_b200", "libcmpx.so")
HEADER = os.path.join(REPO, "include", "cmpx.h")

F16, BF16, F32 = 0, 1, 2
B_KN, B_NK = 0, 1
PATH_AUTO, PATH_TC, PATH_SKINNY, PATH_SIMT, PATH_BF16X3 = 0, 1, 2, 3, 4
OK, ERR_INVALID_ARG, ERR_UNSUPPORTED, ERR_CUDA, ERR_NO_MEMORY, ERR_DEVICE, ERR_WORKSPACE, ERR_TOO_LARGE = range(8)


class GemmArgs(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int),
        ("A", ctypes.c_void_p),
        ("B", ctypes.c_void_p),
        ("C", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("batch", ctypes.c_int64),
        ("M", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("K", ctypes.c_int64),
        ("lda", ctypes.c_int64),
        ("ldb", ctypes.c_int64),
        ("ldc", ctypes.c_int64),
        ("stride_a", ctypes.c_int64),
        ("stride_b", ctypes.c_int64),
        ("stride_c", ctypes.c_int64),
        ("b_layout", ctypes.c_int),
        ("path", ctypes.c_int),
        ("workspace", ctypes.c_void_p),
        ("workspace_bytes", ctypes.c_size_t),
        ("bias_along_m", ctypes.c_int),
        ("peer_C", ctypes.POINTER(ctypes.c_void_p)),
        ("n_peer_C", ctypes.c_int),
        ("mc_C", ctypes.c_void_p),
    ]


_lib = None


def lib():
    global _lib
    if _lib is None:
        L = ctypes.CDLL(LIB_PATH)
        for name in ("cmpx_matmul_f16", "cmpx_matmul_bf16", "cmpx_matmul_f32"):
            f = getattr(L, name)
            f.restype = ctypes.c_int
            f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                          ctypes.c_int64, ctypes.c_void_p]
        L.cmpx_gemm.restype = ctypes.c_int
        L.cmpx_gemm.argtypes = [ctypes.POINTER(GemmArgs), ctypes.c_void_p]
        L.cmpx_gemm_workspace_size.restype = ctypes.c_size_t
        L.cmpx_gemm_workspace_size.argtypes = [ctypes.POINTER(GemmArgs)]
        L.cmpx_gemm_select_path.restype = ctypes.c_int
        L.cmpx_gemm_select_path.argtypes = [ctypes.POINTER(GemmArgs)]
        L.cmpx_add_bias.restype = ctypes.c_int
        L.cmpx_add_bias.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                    ctypes.c_void_p]
        L.cmpx_device_error.restype = ctypes.c_int
        L.cmpx_device_error.argtypes = [ctypes.POINTER(ctypes.c_int)]
        L.cmpx_status_string.restype = ctypes.c_char_p
        L.cmpx_status_string.argtypes = [ctypes.c_int]
        L.cmpx_version.restype = ctypes.c_char_p
        L.cmpx_gemm_gather_ce.restype = ctypes.c_int
        L.cmpx_gemm_gather_ce.argtypes = [ctypes.POINTER(GemmArgs), ctypes.POINTER(ctypes.c_void_p), ctypes.c_int,
                                          ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_uint, ctypes.c_void_p,
                                          ctypes.POINTER(ctypes.c_void_p), ctypes.c_int]
        _lib = L
    return _lib


def declared_symbols() -> list[str]:
    """Every CMPX_API function declared in include/cmpx.h."""
    text = open(HEADER).read()
    return re.findall(r"CMPX_API\s+[\w\s\*]+?\b(cmpx_\w+)\s*\(", text)


def dtype_code(t) -> int:
    import torch

    return {torch.float16: F16, torch.bfloat16: BF16, torch.float32: F32}[t]


def gemm_args(A, B, C, *, bias=None, b_layout=B_KN, path=PATH_AUTO, batch=1, M=None, N=None, K=None,
              lda=None, ldb=None, ldc=None, sa=0, sb=0, sc=0, workspace=None, workspace_bytes=0) -> GemmArgs:
    """Builds args from torch tensors (2-D or 3-D, row-major, possibly strided)."""
    a = GemmArgs()
    a.dtype = dtype_code(A.dtype)
    a.A, a.B, a.C = A.data_ptr(), B.data_ptr(), C.data_ptr()
    a.bias = bias.data_ptr() if bias is not None else None
    a.batch = batch
    a.M = M if M is not None else A.shape[-2]
    a.K = K if K is not None else A.shape[-1]
    a.N = N if N is not None else (B.shape[-1] if b_layout == B_KN else B.shape[-2])
    a.lda = lda if lda is not None else A.stride(-2)
    a.ldb = ldb if ldb is not None else B.stride(-2)
    a.ldc = ldc if ldc is not None else C.stride(-2)
    a.stride_a, a.stride_b, a.stride_c = sa, sb, sc
    a.b_layout = b_layout
    a.path = path
    a.workspace = workspace
    a.workspace_bytes = workspace_bytes
    return a


def gemm(args: GemmArgs, stream: int = 0) -> int:
    return lib().cmpx_gemm(ctypes.byref(args), stream)


def device_error() -> int:
    code = ctypes.c_int(0)
    st = lib().cmpx_device_error(ctypes.byref(code))
    assert st == OK, f"cmpx_device_error failed: {st}"
    return code.value
