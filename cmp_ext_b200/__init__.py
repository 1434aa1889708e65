"""cmp_ext_b200 -- B200 (sm_100a) dense matmul path of cmpext3.

Public operators (same names, arguments, checks and output layout as the
reference's pybind module, src/main.cpp:1594-1602, plus the 2-D forms):

    linear(input, weight, bias=None)   y = input @ weight.T + bias
    bmm(input, mat2)                   (B,M,K) x (B,K,N) -> (B,M,N)
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

try:
    from . import _cmpext3 as _ext  # type: ignore[attr-defined]
except ImportError as e:  # pragma: no cover - exercised only on unbuilt trees
    raise ImportError(
        "cmp_ext_b200 native extension is not built; run `python -m cmp_ext_b200.build` "
        f"(or __graft_entry__.build()) first: {e}"
    ) from e

linear = _ext.linear
bmm = _ext.bmm
fp16_matmul = _ext.fp16_matmul
bf16_matmul = _ext.bf16_matmul
fp32_matmul = _ext.fp32_matmul
_set_path = _ext._set_path
version = _ext._version

__all__ = ["linear", "bmm", "fp16_matmul", "bf16_matmul", "fp32_matmul", "LIB_PATH", "version"]
