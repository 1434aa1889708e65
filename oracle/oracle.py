"""Python side of the parity oracles (test infrastructure only).

* ``oracle_matmul``   -- the CPU restatement of the reference kernels'
  arithmetic (oracle/ref_matmul.c, bit-faithful to
  src/cuda/{fp16,bf16,fp32}_matmul.cu), via ctypes.
* ``ref_gpu_matmul``  -- the reference's own kernels compiled from its sources
  into oracle/_ref/libref_matmul.so (GPU only).
* ``fp64_matmul`` and ``normwise_err`` -- the ground truth and the error
  metric both sides are measured with: max|C - C64| / max|C64|.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module; the product never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libref_matmul.so")

DTYPE_CODE = {"f16": 0, "bf16": 1, "f32": 2}

_lib = None
_ref = None


def reference_dir() -> str | None:
    """The reference checkout: $CMPX_REFERENCE_DIR, else BASELINE.json's
    `reference_path` at the repository root; None when neither names an
    existing directory (e.g. on a GPU box, which uses the prebuilt _ref)."""
    d = os.environ.get("CMPX_REFERENCE_DIR")
    if not d:
        try:
            import json

            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                d = json.load(f).get("reference_path")
        except (OSError, ValueError):
            d = None
    return d if d and os.path.isdir(d) else None


def build(force: bool = False) -> None:
    """Compiles liboracle.so (and oracle/_ref when the reference sources exist)."""
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(os.path.join(HERE, "ref_matmul.c")):
        subprocess.run(["make", "-s", "-f", os.path.join(HERE, "Makefile"), LIB], check=True)
    ref = reference_dir()
    if ref is not None:
        subprocess.run(["make", "-s", "-f", os.path.join(HERE, "Makefile"), f"REF={ref}", "ref"], check=True,
                       stdout=subprocess.DEVNULL)


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        lib = ctypes.CDLL(LIB)
        lib.oracle_matmul.restype = ctypes.c_int
        lib.oracle_matmul.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_int]
        lib.oracle_round_f16.restype = ctypes.c_uint16
        lib.oracle_round_f16.argtypes = [ctypes.c_double]
        lib.oracle_round_bf16.restype = ctypes.c_uint16
        lib.oracle_round_bf16.argtypes = [ctypes.c_double]
        _lib = lib
    return _lib


def round_f16_bits(x: float) -> int:
    return int(_load().oracle_round_f16(float(x)))


def round_bf16_bits(x: float) -> int:
    return int(_load().oracle_round_bf16(float(x)))


def oracle_matmul(dtype: str, A: np.ndarray, B: np.ndarray, rows: tuple[int, int] | None = None,
                  nthreads: int | None = None) -> np.ndarray:
    """C = A @ B with the reference kernel's arithmetic, on the CPU.

    dtype "f16"/"bf16": A, B are uint16 arrays of raw bits; returns uint16 bits.
    dtype "f32": float32 arrays; returns float32.  ``rows`` restricts the
    computation to C[r0:r1] (other rows are returned as zeros).
    """
    lib = _load()
    code = DTYPE_CODE[dtype]
    want = np.float32 if dtype == "f32" else np.uint16
    A = np.ascontiguousarray(A, dtype=want)
    B = np.ascontiguousarray(B, dtype=want)
    M, K = A.shape
    K2, N = B.shape
    assert K == K2, "inner dimensions differ"
    C = np.zeros((M, N), dtype=want)
    r0, r1 = rows if rows is not None else (0, M)
    nt = nthreads or (os.cpu_count() or 1)
    rc = lib.oracle_matmul(code, A.ctypes.data, B.ctypes.data, C.ctypes.data, M, N, K, r0, r1, nt)
    if rc != 0:
        raise ValueError("oracle_matmul rejected its arguments")
    return C


def _load_ref():
    global _ref
    if _ref is None:
        if not os.path.exists(REF_LIB):
            raise FileNotFoundError(f"{REF_LIB} is not built (make -f oracle/Makefile ref)")
        lib = ctypes.CDLL(REF_LIB)
        lib.ref_matmul.restype = ctypes.c_int
        lib.ref_matmul.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                   ctypes.c_int, ctypes.c_int, ctypes.c_int]
        _ref = lib
    return _ref


def ref_attention_supported(dtype: str, S: int, D: int) -> bool:
    """Shapes the reference's attention kernels handle without reading out
    of bounds (read from their sources): the fp16 flash kernel indexes D as
    exactly 128 (src/cuda/fp16_attention.cu:133-160); the fp32 kernel keeps
    D <= 128 registers and loads float4s (src/cuda/fp32_attention.cu:66-110);
    the bf16 kernel keeps S fp32 logits in the default 48 KB of shared
    memory (src/cuda/bf16_attention.cu:97-103)."""
    if dtype == "f16":
        return D == 128
    if dtype == "f32":
        return D % 4 == 0 and D <= 128
    return S * 4 <= 48 * 1024


def ref_gpu_attention(dtype: str, q_ptr: int, k_ptr: int, v_ptr: int, o_ptr: int, B: int, H: int, S: int, D: int,
                      scale: float) -> None:
    """Runs the reference's own attention kernel on device pointers."""
    if not ref_attention_supported(dtype, S, D):
        raise ValueError(f"the reference's {dtype} attention kernel does not handle S={S}, D={D}")
    lib = _load_ref()
    lib.ref_attention.restype = ctypes.c_int
    lib.ref_attention.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float]
    rc = lib.ref_attention(DTYPE_CODE[dtype], q_ptr, k_ptr, v_ptr, o_ptr, B, H, S, D, scale)
    if rc != 0:
        raise RuntimeError(f"reference attention kernel failed with cudaError {rc}")


def fp64_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float) -> np.ndarray:
    """softmax(scale * q k^T) v in fp64 for [..., S, D] arrays (the
    mathematical definition the reference's kernels approximate,
    src/main.cpp:1027-1098): the ground truth for both sides."""
    q, k, v = (np.asarray(x, dtype=np.float64) for x in (q, k, v))
    s = np.einsum("...qd,...kd->...qk", q, k) * float(scale)
    s -= s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("...qk,...kd->...qd", p, v)


def ref_gpu_available() -> bool:
    return os.path.exists(REF_LIB)


def ref_gpu_matmul(dtype: str, A_dev_ptr: int, B_dev_ptr: int, C_dev_ptr: int, M: int, N: int, K: int) -> None:
    """Runs the reference's own kernel (compiled from its sources) on device
    pointers; synchronises; raises on a CUDA error."""
    rc = _load_ref().ref_matmul(DTYPE_CODE[dtype], A_dev_ptr, B_dev_ptr, C_dev_ptr, M, N, K)
    if rc != 0:
        raise RuntimeError(f"reference kernel failed with cudaError {rc}")


# ------------------------------------------------------------------ metrics
def bits_to_f64(dtype: str, X: np.ndarray) -> np.ndarray:
    if dtype == "f32":
        return X.astype(np.float64)
    if dtype == "f16":
        return X.view(np.float16).astype(np.float64)
    return (X.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def fp64_matmul(dtype: str, A: np.ndarray, B: np.ndarray) -> np.ndarray:
    return bits_to_f64(dtype, A) @ bits_to_f64(dtype, B)


def normwise_err(C: np.ndarray, C64: np.ndarray) -> float:
    """max|C - C64| / max|C64| (the error metric for both reference and build)."""
    C = np.asarray(C, dtype=np.float64)
    denom = float(np.max(np.abs(C64))) if C64.size else 0.0
    if denom == 0.0:
        return float(np.max(np.abs(C - C64))) if C.size else 0.0
    return float(np.max(np.abs(C - C64)) / denom)
