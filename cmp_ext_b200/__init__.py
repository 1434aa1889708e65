"""cmp_ext_b200 -- B200 (sm_100a) dense matmul path of cmpext3.

Public operators (same names, arguments, checks and output layout as the
reference's pybind module, src/main.cpp:1594-1602, plus the 2-D forms):

    linear(input, weight, bias=None)   y = input @ weight.T + bias
    bmm(input, mat2)                   (B,M,K) x (B,K,N) -> (B,M,N)
    conv2d(input, weight, bias=None, stride=1, padding=0, dilation=1, groups=1)
                                       the 1x1 / stride 1 / padding 0 case, as one
                                       batched GEMM on NCHW (no layout copies)
    attention(query, key, value, scale=None)
                                       softmax(scale * Q K^T) V on [B, H, S, D]
    fp16_matmul(a, b) / bf16_matmul(a, b) / fp32_matmul(a, b)
                                       a[M,K] @ b[K,N] -> [M,N]

All of them run the hand-written sm_100a kernels of libcmpx.so through the
torch shim _cmpext3.  There is no CPU or library fallback: if the native
extension is missing, importing this package raises ImportError.
"""
from __future__ import annotations

import os

import torch  # noqa: F401  (loads libtorch / c10 before the shim)

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcmpx.so")

_OPS = ("linear", "bmm", "conv2d", "attention", "fp16_matmul", "bf16_matmul", "fp32_matmul", "_set_path", "_matmul_into", "_matmul_gather_ce", "version")


def _load_ext():
    try:
        from . import _cmpext3  # type: ignore[attr-defined]
    except ImportError as e:
        raise ImportError(
            "cmp_ext_b200 native extension is not built; run `python -m cmp_ext_b200.build` "
            f"(or __graft_entry__.build()) first: {e}"
        ) from e
    return _cmpext3


def __getattr__(name):
    # The operators resolve on first use so that `cmp_ext_b200.build` can be
    # imported (and run) before the extension exists.  A missing extension is
    # an ImportError, never a fallback.
    if name in _OPS:
        ext = _load_ext()
        value = getattr(ext, "_version" if name == "version" else name)
        globals()[name] = value
        return value
    raise AttributeError(f"module 'cmp_ext_b200' has no attribute {name!r}")


__all__ = ["linear", "bmm", "conv2d", "attention", "fp16_matmul", "bf16_matmul", "fp32_matmul", "LIB_PATH", "version"]
