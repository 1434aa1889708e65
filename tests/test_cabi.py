"""The C ABI boundary without a GPU: the library loads, exports every symbol
include/cmpx.h declares (plus the reference's six C++ launcher symbols), and
rejects bad arguments before touching a device; path selection is pure host
logic."""
import ctypes
import subprocess

import pytest

import cabi

REF_LAUNCHERS = [  # reference src/main.cpp:12-19, C++ linkage
    "_Z18launch_matmul_fp16PKvS0_Pviii",
    "_Z18launch_matmul_fp32PKfS0_Pfiii",
    "_Z18launch_matmul_bf16PKvS0_Pviii",
    "_Z20launch_add_bias_fp16PvPKvii",
    "_Z20launch_add_bias_fp32PfPKfii",
    "_Z20launch_add_bias_bf16PvPKvii",
    "_Z21launch_attention_fp32PKfS0_S0_Pfiiiif",  # src/main.cpp:48-50
    "_Z21launch_attention_fp16PKvS0_S0_Pviiiif",
    "_Z21launch_attention_bf16PKvS0_S0_Pviiiif",
]


def test_header_declares_entry_points():
    names = cabi.declared_symbols()
    for want in ("cmpx_matmul_f16", "cmpx_matmul_bf16", "cmpx_matmul_f32", "cmpx_gemm", "cmpx_add_bias",
                 "cmpx_device_error", "cmpx_gemm_workspace_size", "cmpx_gemm_select_path"):
        assert want in names


def test_library_exports_every_declared_symbol():
    lib = cabi.lib()
    for name in cabi.declared_symbols():
        assert hasattr(lib, name), name


def test_reference_launcher_symbols_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", cabi.LIB_PATH], capture_output=True, text=True).stdout
    for sym in REF_LAUNCHERS:
        assert sym in out, sym


def test_status_strings_and_version():
    lib = cabi.lib()
    assert lib.cmpx_status_string(0) == b"ok"
    assert lib.cmpx_status_string(cabi.ERR_WORKSPACE) == b"workspace too small"
    assert lib.cmpx_status_string(99) == b"unknown status"
    assert b"sm_100a" in lib.cmpx_version()


def _args(**kw):
    a = cabi.GemmArgs()
    a.dtype, a.batch, a.M, a.N, a.K = cabi.F16, 1, 128, 256, 64
    a.A, a.B, a.C = 0x100000, 0x200000, 0x300000  # fake, 16-byte aligned; never dereferenced
    a.lda, a.ldb, a.ldc = 64, 256, 256
    a.b_layout, a.path = cabi.B_KN, cabi.PATH_AUTO
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw", [dict(dtype=7), dict(M=-1), dict(K=-3), dict(b_layout=5), dict(path=9),
                                dict(ldc=100), dict(lda=10), dict(ldb=100), dict(C=None), dict(A=None),
                                dict(stride_a=-1)])
def test_invalid_args_rejected_before_device(kw):
    assert cabi.gemm(_args(**kw)) == cabi.ERR_INVALID_ARG


def test_null_args_and_empty_problems():
    assert cabi.lib().cmpx_gemm(None, None) == cabi.ERR_INVALID_ARG
    assert cabi.gemm(_args(M=0)) == cabi.OK
    assert cabi.gemm(_args(N=0, C=None)) == cabi.OK
    assert cabi.gemm(_args(batch=0)) == cabi.OK
    assert cabi.lib().cmpx_add_bias(0, None, None, 0, 5, None) == cabi.OK
    assert cabi.lib().cmpx_add_bias(9, None, None, 1, 1, None) == cabi.ERR_INVALID_ARG


def sel(**kw):
    return cabi.lib().cmpx_gemm_select_path(ctypes.byref(_args(**kw)))


def test_path_selection():
    assert sel(M=129) == cabi.PATH_TC
    assert sel(M=16) == cabi.PATH_SKINNY                   # one tile, K 64
    kw = lambda M, N, K: dict(M=M, N=N, K=K, lda=K, ldb=N, ldc=N)
    # M <= 32: skinny unless ~96+ tiles of 256 columns with K < 128 * tiles
    assert sel(**kw(16, 28672, 8192)) == cabi.PATH_TC       # config 4: 112 tiles
    assert sel(**kw(16, 14336, 4096)) == cabi.PATH_SKINNY   # 56 tiles
    assert sel(**kw(32, 16384, 16384)) == cabi.PATH_SKINNY  # 64 tiles
    assert sel(**kw(4, 28672, 8192)) == cabi.PATH_SKINNY    # M < 8: always skinny
    # 32 < M <= 128: skinny when K >= 128 * tiles and the tiles leave SMs idle
    assert sel(M=64) == cabi.PATH_TC                       # N 256, K 64: one shallow tile
    assert sel(**kw(65, 4096, 4096)) == cabi.PATH_SKINNY
    assert sel(**kw(100, 4096, 14336)) == cabi.PATH_SKINNY
    assert sel(**kw(128, 8192, 8192)) == cabi.PATH_SKINNY
    assert sel(**kw(100, 8192, 2048)) == cabi.PATH_TC
    assert sel(**kw(48, 14336, 4096)) == cabi.PATH_TC
    assert sel(**kw(64, 28672, 4096)) == cabi.PATH_TC
    assert sel(**kw(128, 1024, 8192)) == cabi.PATH_SKINNY
    wide = 256 * 160
    assert sel(**kw(128, wide, wide * 2)) == cabi.PATH_TC
    assert sel(A=0x100002) == cabi.PATH_SIMT           # misaligned base
    assert sel(N=250, ldb=250, ldc=250) == cabi.PATH_SIMT  # row stride not 16-byte multiple
    assert sel(b_layout=cabi.B_NK, ldb=64) == cabi.PATH_TC
    assert sel(K=0) == cabi.PATH_SIMT                  # fill kernel
    # fp32: 3xTF32 when the packed rows are 16-byte multiples and the problem is not tiny
    assert sel(dtype=cabi.F32, M=4096, N=4096, K=4096, lda=4096, ldb=4096, ldc=4096) == cabi.PATH_TC
    assert sel(dtype=cabi.F32, M=257, N=383, K=511, lda=511, ldb=383, ldc=383) == cabi.PATH_SIMT
    assert sel(dtype=cabi.F32, M=8, N=8, K=8, lda=8, ldb=8, ldc=8) == cabi.PATH_SIMT
    # forced paths
    assert sel(path=cabi.PATH_SIMT) == cabi.PATH_SIMT
    assert sel(path=cabi.PATH_SKINNY) == cabi.PATH_SKINNY
    assert sel(path=cabi.PATH_SKINNY, M=129) == -1      # M > 128
    assert sel(path=cabi.PATH_TC, N=250, ldb=250, ldc=250) == -1
    assert sel(dtype=cabi.F32, path=cabi.PATH_SKINNY, lda=64, ldb=256, ldc=256) == -1
    # bf16x3 (fp32 only, opt-in): packed bf16 rows need K % 8 == 0
    f32 = dict(dtype=cabi.F32, M=512, N=512, K=512, lda=512, ldb=512, ldc=512)
    assert sel(path=cabi.PATH_BF16X3, **f32) == cabi.PATH_BF16X3
    assert sel(path=cabi.PATH_BF16X3, **{**f32, "K": 516, "lda": 516}) == -1
    assert sel(path=cabi.PATH_BF16X3) == -1             # fp16 operands
    assert sel(path=5) == -1
    assert sel(dtype=9) == -1


def test_selftest_rejects_bad_limits_without_device():
    f = cabi.lib().cmpx_selftest_bounded_wait
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_ulonglong, ctypes.c_void_p]
    assert f(0, None) == cabi.ERR_INVALID_ARG
    assert f(20_000_000_000, None) == cabi.ERR_INVALID_ARG


def _attn_fn():
    f = cabi.lib().cmpx_attention
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                  ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    return f


def test_attention_argument_checks_before_device():
    f = _attn_fn()
    p = 0x100000  # fake, 16-byte aligned; never dereferenced
    assert f(7, p, p, p, p, 1, 1, 8, 64, 1.0, 0, None) == cabi.ERR_INVALID_ARG     # dtype
    assert f(0, p, p, p, p, -1, 1, 8, 64, 1.0, 0, None) == cabi.ERR_INVALID_ARG    # negative size
    assert f(0, None, p, p, p, 1, 1, 8, 64, 1.0, 0, None) == cabi.ERR_INVALID_ARG  # null pointer
    assert f(0, None, None, None, None, 0, 1, 8, 64, 1.0, 0, None) == cabi.OK      # empty: nothing to do
    assert f(0, None, None, None, None, 1, 1, 0, 64, 1.0, 0, None) == cabi.OK


def test_attention_path_selection_is_host_logic():
    sel = cabi.lib().cmpx_attention_select_path
    sel.restype = ctypes.c_int
    sel.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                    ctypes.c_int]
    p, odd = 0x100000, 0x100008
    assert sel(cabi.F16, p, p, p, p, 128, cabi.PATH_AUTO) == cabi.PATH_TC
    assert sel(cabi.BF16, p, p, p, p, 64, cabi.PATH_AUTO) == cabi.PATH_TC
    assert sel(cabi.F16, p, p, p, p, 80, cabi.PATH_AUTO) == cabi.PATH_SIMT     # D not 64/128
    assert sel(cabi.F32, p, p, p, p, 128, cabi.PATH_AUTO) == cabi.PATH_SIMT    # fp32: CUDA cores
    assert sel(cabi.F16, odd, p, p, p, 128, cabi.PATH_AUTO) == cabi.PATH_SIMT  # unaligned: no TMA
    assert sel(cabi.F32, p, p, p, p, 128, cabi.PATH_TC) == -1
    assert sel(cabi.F16, p, p, p, p, 1024, cabi.PATH_AUTO) == -1               # beyond the CUDA-core limit
    assert sel(cabi.F16, p, p, p, p, 128, cabi.PATH_SKINNY) == -1


def test_gather_ce_argument_checks_before_device():
    f = cabi.lib().cmpx_gemm_gather_ce
    args = _args(M=512)
    flags = ctypes.c_void_p(0x200000)
    peers = (ctypes.c_void_p * 1)(0x300000)
    streams = (ctypes.c_void_p * 1)(None)
    assert f(None, peers, 1, flags, 4, 4, 1, None, streams, 1) == cabi.ERR_INVALID_ARG       # no args
    assert f(ctypes.byref(args), peers, 8, flags, 4, 4, 1, None, streams, 1) == cabi.ERR_INVALID_ARG  # > 7 peers
    assert f(ctypes.byref(args), peers, 1, None, 4, 4, 1, None, streams, 1) == cabi.ERR_INVALID_ARG   # no flags
    assert f(ctypes.byref(args), peers, 1, flags, 4, 4, 0, None, streams, 1) == cabi.ERR_INVALID_ARG  # epoch 0
    assert f(ctypes.byref(args), peers, 1, flags, 4, 4, 1, None, None, 0) == cabi.ERR_INVALID_ARG    # no streams
    a32 = _args(M=512, dtype=cabi.F32)
    assert f(ctypes.byref(a32), peers, 1, flags, 4, 4, 1, None, streams, 1) == cabi.ERR_UNSUPPORTED  # fp32
    small = _args(M=64)
    assert f(ctypes.byref(small), peers, 1, flags, 4, 4, 1, None, streams, 1) == cabi.ERR_UNSUPPORTED  # M <= 128


def test_multicast_output_rejected_with_peer_outputs():
    peers = (ctypes.c_void_p * 1)(0x300000)
    a = _args(M=512, mc_C=0x400000, n_peer_C=1)
    a.peer_C = ctypes.cast(peers, ctypes.POINTER(ctypes.c_void_p))
    assert cabi.gemm(a) == cabi.ERR_INVALID_ARG
