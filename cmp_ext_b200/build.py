"""In-tree build of the native parts of cmp_ext_b200.

Outputs (next to this file, git-ignored, shipped with the source tree):
  libcmpx.so     C-ABI kernel library (nvcc, sm_100a only, static cudart)
  _cmpext3*.so   torch extension shim over the C ABI (g++, links libcmpx.so)

Replaces the reference's setup.py (CUDAExtension over 56 sources, no arch
flags, --fmad=false --use_fast_math; setup.py:10-93): here only the matmul
path is built, for sm_100a alone, with no fast-math and normal FMA contraction.

Usage: python -m cmp_ext_b200.build [--force] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
INCLUDE = os.path.join(REPO, "include")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

CU_SOURCES = ["cmpx_api.cu", "gemm_tc.cu", "gemm_tc2.cu", "gemm_skinny.cu", "gemm_simt.cu", "cmpx_selftest.cu", "gather_ce.cu",
              "attention.cu"]
HEADERS = ["ptx.cuh", "internal.h"]
LIB = os.path.join(HERE, "libcmpx.so")
SHIM_SRC = os.path.join(CSRC, "torch_shim.cpp")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I", INCLUDE,
]


def _shim_target() -> str:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return os.path.join(HERE, "_cmpext3" + suffix)


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed ({r.returncode}):\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def build_lib(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(INCLUDE, "cmpx.h")]
    objs, jobs = [], []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or not _newer(o, [s] + hdrs):
            flags = NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else [])
            jobs.append([NVCC] + flags + ["-c", s, "-o", o])
    logs = []
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        for out in ex.map(lambda c: _run(c, verbose), jobs):
            logs.append(out)
    if ptxas_verbose:
        print("\n".join(logs))
    if force or jobs or not _newer(LIB, objs):
        _run([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", LIB] + objs
             + ["-Xlinker", "-soname=libcmpx.so"], verbose)
    return LIB


def build_shim(force: bool = False, verbose: bool = False) -> str:
    import torch  # noqa: F401  (only for include/library paths)
    from torch.utils import cpp_extension as ce

    target = _shim_target()
    if not force and _newer(target, [SHIM_SRC, LIB, os.path.join(INCLUDE, "cmpx.h")]):
        return target
    import torch as _t
    abi = int(_t._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-shared", "-fPIC", "-std=c++17", SHIM_SRC, "-o", target,
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_cmpext3", "-DTORCH_API_INCLUDE_EXTENSION_H",
           "-I", INCLUDE, "-I", sysconfig.get_paths()["include"], "-I", os.path.join(CUDA_HOME, "include")]
    for p in ce.include_paths():
        cmd += ["-isystem", p]
    for p in ce.library_paths():
        cmd += ["-L", p, f"-Wl,-rpath,{p}"]
    cmd += ["-L", HERE, "-lcmpx", "-Wl,-rpath,$ORIGIN", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
            "-ltorch_python"]
    _run(cmd, verbose)
    return target


def build(force: bool = False, verbose: bool = False) -> None:
    build_lib(force, verbose)
    build_shim(force, verbose)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v register/smem usage")
    ap.add_argument("--lib-only", action="store_true")
    a = ap.parse_args(argv)
    build_lib(a.force or a.ptxas, a.verbose, a.ptxas)
    if not a.lib_only:
        build_shim(a.force, a.verbose)
    return 0


if __name__ == "__main__":
    sys.exit(main())
