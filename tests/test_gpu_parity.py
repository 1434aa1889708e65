"""GPU parity tests: the sm_100a kernels, called through the C ABI of
libcmpx.so, against the CPU oracle (the reference's arithmetic), the
reference's own kernels (oracle/_ref), fp64 ground truth and a torch fp32
reference.

Pass criterion (the path's contract): for every case,
    err(build) <= err(reference kernel) + TOL
with err = max|C - C64| / max|C64| and TOL = 1e-3 (fp16/bf16), 1e-5 (fp32).
"""
import ctypes

import numpy as np
import pytest
import torch

import cabi
from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 1e-3, torch.bfloat16: 1e-3, torch.float32: 1e-5}
# fp32-accumulating kernels land near output rounding; these are generous
# bounds on the distance to a torch fp32 reference of the same product.
# (torch's CPU fp32 matmul carries its own rounding error at large K, hence
# the looser fp32 figure; the fp64 bound below is the real check).
VS_TORCH = {torch.float16: 2e-3, torch.bfloat16: 1.6e-2, torch.float32: 1e-4}
KIND = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.float32:
        return t.numpy()
    return t.view(torch.int16).numpy().view(np.uint16)


def _rand(shape, dtype, gen, std=1.0, uniform=False):
    if uniform:
        x = torch.rand(shape, generator=gen) * 2 - 1
    else:
        x = torch.randn(shape, generator=gen) * std
    return x.to(dtype)


def run_cabi(A, B, *, b_layout=cabi.B_KN, path=cabi.PATH_AUTO, bias=None, expect=cabi.OK):
    M, K = A.shape
    N = B.shape[1] if b_layout == cabi.B_KN else B.shape[0]
    C = torch.full((M, N), float("nan"), dtype=A.dtype, device=A.device)
    args = cabi.gemm_args(A, B, C, bias=bias, b_layout=b_layout, path=path)
    st = cabi.gemm(args, torch.cuda.current_stream().cuda_stream)
    assert st == expect, f"cmpx_gemm returned {st} ({cabi.lib().cmpx_status_string(st).decode()})"
    torch.cuda.synchronize()
    return C


def check_case(M, N, K, dtype, *, b_layout=cabi.B_KN, path=cabi.PATH_AUTO, seed=0, bias=False, oracle=True):
    g = torch.Generator().manual_seed(seed)
    uniform = dtype == torch.float16
    std = 0.02 if dtype == torch.bfloat16 else 1.0
    A = _rand((M, K), dtype, g, uniform=uniform)
    Bkn = _rand((K, N), dtype, g, std=std, uniform=uniform)
    bvec = _rand((N,), dtype, g) if bias else None
    Bdev = (Bkn if b_layout == cabi.B_KN else Bkn.t().contiguous()).cuda()
    C = run_cabi(A.cuda(), Bdev, b_layout=b_layout, path=path, bias=bvec.cuda() if bias else None)
    assert not torch.isnan(C.float()).any(), "output not fully written"
    C64 = o.fp64_matmul(KIND[dtype], _bits(A), _bits(Bkn))
    if bias:
        C64 = C64 + o.bits_to_f64(KIND[dtype], _bits(bvec))[None, :]
    err = o.normwise_err(C.double().cpu().numpy(), C64)
    # torch fp32 reference of the same op
    tref = A.float() @ Bkn.float() + (bvec.float()[None, :] if bias else 0)
    assert o.normwise_err(C.double().cpu().numpy(), tref.double().numpy()) <= VS_TORCH[dtype] + 1e-7
    if oracle and not bias:
        ref = o.oracle_matmul(KIND[dtype], _bits(A), _bits(Bkn))
        ref_err = o.normwise_err(o.bits_to_f64(KIND[dtype], ref), C64)
        assert err <= ref_err + TOL[dtype], (err, ref_err)
    return err


# ------------------------------------------------------------ tensor-core path
TC_SHAPES = [(128, 256, 64), (256, 512, 1024), (300, 264, 200), (129, 8, 8), (1000, 1000, 72), (384, 768, 4096)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("b_layout", [cabi.B_KN, cabi.B_NK])
@pytest.mark.parametrize("shape", TC_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_tc_path(cuda, dtype, b_layout, shape):
    M, N, K = shape
    check_case(M, N, K, dtype, b_layout=b_layout, path=cabi.PATH_TC)


@pytest.mark.parametrize("b_layout", [cabi.B_KN, cabi.B_NK])
def test_tc_path_bias(cuda, b_layout):
    check_case(300, 264, 200, torch.bfloat16, b_layout=b_layout, path=cabi.PATH_TC, bias=True)
    check_case(130, 520, 96, torch.float16, b_layout=b_layout, path=cabi.PATH_TC, bias=True)


# ------------------------------------------------------------ skinny path
# large-N cases: (16, 28672, 512), (16, 8192, 8192), (40, 4096, 16384)
SK_SHAPES = [(1, 128, 64), (7, 1000, 200), (16, 4096, 1024), (17, 256, 8192), (32, 520, 640), (33, 384, 256),
             (64, 2048, 2048), (16, 28672, 512), (16, 8192, 8192), (40, 4096, 16384), (65, 640, 384),
             (100, 4096, 2048), (128, 8192, 4096), (127, 1000, 1000)]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("b_layout", [cabi.B_KN, cabi.B_NK])
@pytest.mark.parametrize("shape", SK_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_skinny_path(cuda, dtype, b_layout, shape):
    M, N, K = shape
    check_case(M, N, K, dtype, b_layout=b_layout, path=cabi.PATH_SKINNY)


def test_skinny_bias_and_determinism(cuda):
    check_case(16, 1000, 4096, torch.float16, path=cabi.PATH_SKINNY, bias=True)
    g = torch.Generator().manual_seed(5)
    A = _rand((16, 8192), torch.float16, g).cuda()
    B = _rand((8192, 4096), torch.float16, g, std=0.02).cuda()
    c1 = run_cabi(A, B, path=cabi.PATH_SKINNY)
    c2 = run_cabi(A, B, path=cabi.PATH_SKINNY)
    assert torch.equal(c1, c2), "stream-K reduction must be deterministic"


# ------------------------------------------------------------ fp32 paths
@pytest.mark.parametrize("b_layout", [cabi.B_KN, cabi.B_NK])
@pytest.mark.parametrize("shape", [(256, 256, 256), (300, 260, 132), (128, 128, 4096)],
                         ids=lambda s: "x".join(map(str, s)))
def test_tf32x3_path(cuda, b_layout, shape):
    M, N, K = shape
    err = check_case(M, N, K, torch.float32, b_layout=b_layout, path=cabi.PATH_TC)
    assert err < 5e-6


@pytest.mark.parametrize("b_layout", [cabi.B_KN, cabi.B_NK])
@pytest.mark.parametrize("shape", [(256, 256, 256), (300, 260, 136), (128, 128, 4096), (257, 384, 512),
                                   (1000, 136, 72)],
                         ids=lambda s: "x".join(map(str, s)))
def test_bf16x3_path(cuda, b_layout, shape):
    """fp32 through bf16 hi/lo splits: truncation leaves ~2^-17 per
    product, so the normwise error sits near 5e-6, inside the fp32 contract
    (reference kernel error + 1e-5, checked by check_case)."""
    M, N, K = shape
    err = check_case(M, N, K, torch.float32, b_layout=b_layout, path=cabi.PATH_BF16X3)
    assert err < 1e-5


@pytest.mark.parametrize("n", [136, 260])  # N-major splits of B / transposed splits (N % 8 != 0)
def test_bf16x3_batched(cuda, n):
    g = torch.Generator().manual_seed(12)
    Bt, M, K = 3, 200, 328
    A = _rand((Bt, M, K), torch.float32, g).cuda()
    B = _rand((Bt, K, n), torch.float32, g).cuda()
    C = torch.empty((Bt, M, n), device="cuda")
    args = cabi.gemm_args(A[0], B[0], C[0], batch=Bt, sa=M * K, sb=K * n, sc=M * n, path=cabi.PATH_BF16X3)
    assert cabi.gemm(args) == cabi.OK
    torch.cuda.synchronize()
    want = torch.bmm(A.double(), B.double())
    assert o.normwise_err(C.double().cpu().numpy(), want.cpu().numpy()) < 1e-5


def test_bf16x3_workspace_and_odd_k(cuda):
    g = torch.Generator().manual_seed(11)
    A = _rand((256, 520), torch.float32, g).cuda()
    B = _rand((520, 384), torch.float32, g).cuda()
    C = torch.empty((256, 384), device="cuda")
    args = cabi.gemm_args(A, B, C, path=cabi.PATH_BF16X3)
    need = cabi.lib().cmpx_gemm_workspace_size(ctypes.byref(args))
    assert need == 2 * (256 * 520 * 2) + 2 * (520 * 384 * 2)  # bf16 hi + lo of A and B (256-byte rounded)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    args = cabi.gemm_args(A, B, C, path=cabi.PATH_BF16X3, workspace=ws.data_ptr(), workspace_bytes=need)
    assert cabi.gemm(args) == cabi.OK
    torch.cuda.synchronize()
    want = A.double() @ B.double()
    assert o.normwise_err(C.double().cpu().numpy(), want.cpu().numpy()) < 1e-5
    # K % 8 != 0: packed bf16 rows would not be 16-byte multiples
    A2 = _rand((128, 132), torch.float32, g).cuda()
    B2 = _rand((132, 128), torch.float32, g).cuda()
    run_cabi(A2, B2, path=cabi.PATH_BF16X3, expect=cabi.ERR_UNSUPPORTED)


@pytest.mark.parametrize("path", [cabi.PATH_TC, cabi.PATH_BF16X3])
@pytest.mark.parametrize("b_layout", [cabi.B_KN, cabi.B_NK])
def test_f32_split_near_flt_max(cuda, path, b_layout):
    """fp32 inputs within half an ulp (of tf32 / bf16) of FLT_MAX: rounding
    the hi part to nearest would give inf and lo = -inf, so the product would
    be NaN where the reference's fp32 arithmetic is finite.  hi is clamped to
    the format's largest finite value; the result must match the oracle's
    error bound like any other input."""
    M, N, K = 256, 264, 136
    g = torch.Generator().manual_seed(21)
    fmax = torch.finfo(torch.float32).max
    A = (torch.rand(M, K, generator=g) * 0.02 + 0.98) * fmax
    A = torch.where(torch.rand(M, K, generator=g) < 0.5, A, -A)
    A[0, :] = fmax
    A[1, :] = -fmax
    A[2, ::2] = torch.tensor(0x7F7FF000, dtype=torch.int32).view(torch.float32)  # rounds up in tf32 and bf16
    B = torch.randn(K, N, generator=g) * 2.0 ** -100  # products ~2^28: no overflow in any partial sum
    Bdev = (B if b_layout == cabi.B_KN else B.t().contiguous()).cuda()
    C = run_cabi(A.cuda(), Bdev, b_layout=b_layout, path=path)
    assert torch.isfinite(C).all()
    C64 = o.fp64_matmul("f32", A.numpy(), B.numpy())
    ref = o.oracle_matmul("f32", A.numpy(), B.numpy())
    err = o.normwise_err(C.double().cpu().numpy(), C64)
    ref_err = o.normwise_err(ref.astype(np.float64), C64)
    assert err <= ref_err + TOL[torch.float32], (err, ref_err)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(257, 383, 511), (5, 7, 3), (70, 130, 33), (1, 1, 1)],
                         ids=lambda s: "x".join(map(str, s)))
def test_simt_path(cuda, dtype, shape):
    M, N, K = shape
    check_case(M, N, K, dtype, path=cabi.PATH_SIMT)


def test_config1_odd_fp32_auto(cuda):
    """Config 1: fp32 257x383x511 N(0,1) seed 0 through the automatic path."""
    from cmp_ext_b200.workloads import CONFIGS, make_inputs

    A, B = make_inputs(CONFIGS[1], "cpu", seed=0)
    C = run_cabi(A.cuda(), B.cuda())
    C64 = A.double().numpy() @ B.double().numpy()
    ref = o.oracle_matmul("f32", A.numpy(), B.numpy())
    err, ref_err = o.normwise_err(C.double().cpu().numpy(), C64), o.normwise_err(ref, C64)
    assert err <= ref_err + 1e-5


# ------------------------------------------------------------ edge cases
def test_k_zero_and_empty(cuda):
    A = torch.empty((4, 0), dtype=torch.float16, device="cuda")
    B = torch.empty((0, 8), dtype=torch.float16, device="cuda")
    C = run_cabi(A, B)
    assert torch.equal(C, torch.zeros_like(C))
    bias = torch.arange(8, dtype=torch.float16, device="cuda")
    C = run_cabi(A, B, bias=bias)
    assert torch.equal(C, bias.expand(4, 8))
    A = torch.empty((0, 16), dtype=torch.bfloat16, device="cuda")
    B = torch.ones((16, 8), dtype=torch.bfloat16, device="cuda")
    run_cabi(A, B)


def test_forced_path_rejections(cuda):
    A = torch.ones((128, 72), dtype=torch.float16, device="cuda")
    B = torch.ones((72, 13), dtype=torch.float16, device="cuda")  # ldb*2 not a multiple of 16
    run_cabi(A, B, path=cabi.PATH_TC, expect=cabi.ERR_UNSUPPORTED)
    C = run_cabi(A, B)  # auto -> SIMT
    assert torch.equal(C, torch.full_like(C, 72.0))
    A = torch.ones((129, 64), dtype=torch.float16, device="cuda")
    B = torch.ones((64, 64), dtype=torch.float16, device="cuda")
    run_cabi(A, B, path=cabi.PATH_SKINNY, expect=cabi.ERR_UNSUPPORTED)  # M > 128


def test_batched_and_strided(cuda):
    """3-D TMA batching and non-packed leading dimensions."""
    g = torch.Generator().manual_seed(9)
    Bt, M, N, K = 3, 200, 136, 328
    A = _rand((Bt, M, K), torch.bfloat16, g).cuda()
    B = _rand((Bt, K, N), torch.bfloat16, g, std=0.02).cuda()
    C = torch.empty((Bt, M, N), dtype=torch.bfloat16, device="cuda")
    args = cabi.gemm_args(A[0], B[0], C[0], batch=Bt, sa=M * K, sb=K * N, sc=M * N, path=cabi.PATH_TC)
    assert cabi.gemm(args) == cabi.OK
    torch.cuda.synchronize()
    want = torch.bmm(A.float(), B.float())
    assert o.normwise_err(C.double().cpu().numpy(), want.double().cpu().numpy()) < 1.6e-2
    # padded leading dimensions (row strides larger than the logical width)
    Abig = _rand((M, K + 24), torch.float16, g).cuda()
    Bbig = _rand((K, N + 8), torch.float16, g).cuda()
    Cbig = torch.zeros((M, N + 16), dtype=torch.float16, device="cuda")
    a, b = Abig[:, :K], Bbig[:, :N]
    args = cabi.gemm_args(a, b, Cbig, M=M, N=N, K=K, lda=K + 24, ldb=N + 8, ldc=N + 16, path=cabi.PATH_TC)
    assert cabi.gemm(args) == cabi.OK
    torch.cuda.synchronize()
    want = a.float() @ b.float()
    assert o.normwise_err(Cbig[:, :N].double().cpu().numpy(), want.double().cpu().numpy()) < 2e-3
    assert not Cbig[:, N:].any(), "wrote outside the logical C"


def test_caller_workspace(cuda):
    g = torch.Generator().manual_seed(11)
    A = _rand((16, 4096), torch.float16, g).cuda()
    B = _rand((4096, 2048), torch.float16, g, std=0.02).cuda()
    C = torch.empty((16, 2048), dtype=torch.float16, device="cuda")
    args = cabi.gemm_args(A, B, C)
    need = cabi.lib().cmpx_gemm_workspace_size(args)
    assert need > 0
    args.workspace_bytes = need - 1
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    args.workspace = ws.data_ptr()
    assert cabi.gemm(args) == cabi.ERR_WORKSPACE
    args.workspace_bytes = need
    assert cabi.gemm(args) == cabi.OK
    torch.cuda.synchronize()
    ref = run_cabi(A, B)
    assert torch.equal(C, ref)


def test_no_device_error_recorded(cuda):
    assert cabi.device_error() == 0


# ------------------------------------------------------------ reference kernels
@pytest.mark.skipif(not o.ref_gpu_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("dtype,shape", [(torch.float16, (64, 64, 64)), (torch.float16, (96, 136, 200)),
                                         (torch.bfloat16, (130, 136, 264)), (torch.float32, (33, 17, 45))])
def test_reference_kernel_matches_oracle(cuda, dtype, shape):
    """Pins the CPU oracle against the reference's own kernel on this GPU."""
    M, N, K = shape
    g = torch.Generator().manual_seed(21)
    A = _rand((M, K), dtype, g)
    B = _rand((K, N), dtype, g, std=0.02 if dtype == torch.bfloat16 else 1.0)
    C = torch.empty((M, N), dtype=dtype, device="cuda")
    Ad, Bd = A.cuda(), B.cuda()
    o.ref_gpu_matmul(KIND[dtype], Ad.data_ptr(), Bd.data_ptr(), C.data_ptr(), M, N, K)
    want = o.oracle_matmul(KIND[dtype], _bits(A), _bits(B))
    assert np.array_equal(_bits(C).view(np.uint8), want.view(np.uint8))


@pytest.mark.parametrize("path,shape", [(cabi.PATH_TC, (512, 264, 136)), (cabi.PATH_TC, (100, 264, 136)),
                                        (cabi.PATH_SIMT, (70, 130, 33))], ids=["pair-tma", "single-cta", "simt"])
def test_peer_outputs(cuda, path, shape):
    """n_peer_C extra outputs receive exactly C (here two buffers on the same
    GPU stand in for peers' memory): the CTA-pair kernel's staged TMA-store
    epilogue, the single-CTA kernel's and the fallback's direct stores."""
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(13)
    A = torch.randn(M, K, generator=g, device="cuda").half()
    B = (torch.randn(K, N, generator=g, device="cuda") * 0.1).half()
    bias = torch.randn(N, generator=g, device="cuda").half()
    C = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    p1 = torch.full_like(C, float("nan"))
    p2 = torch.full_like(C, float("nan"))
    arr = (ctypes.c_void_p * 2)(p1.data_ptr(), p2.data_ptr())
    args = cabi.gemm_args(A, B, C, bias=bias, path=path)
    args.peer_C = ctypes.cast(arr, ctypes.POINTER(ctypes.c_void_p))
    args.n_peer_C = 2
    assert cabi.gemm(args) == cabi.OK
    torch.cuda.synchronize()
    assert not torch.isnan(C.float()).any()
    assert torch.equal(C, p1) and torch.equal(C, p2)
    assert o.normwise_err(C.double().cpu().numpy(), (A.float() @ B.float() + bias.float()).double().cpu().numpy()) < 2e-3


@pytest.mark.parametrize("shape", [(16, 28672, 8192), (8, 1024, 8192), (100, 4096, 14336)],
                         ids=lambda s: "x".join(map(str, s)))
def test_skinny_caller_workspace(cuda, shape):
    """Skinny path with a caller-provided (zero-filled) workspace: same bits
    as the library-managed one, and reusable call after call."""
    M, N, K = shape
    g = torch.Generator().manual_seed(11)
    A = _rand((M, K), torch.float16, g).cuda()
    B = _rand((K, N), torch.float16, g, std=0.02).cuda()
    ref = run_cabi(A, B, path=cabi.PATH_SKINNY)
    C = torch.empty((M, N), dtype=torch.float16, device="cuda")
    args = cabi.gemm_args(A, B, C, path=cabi.PATH_SKINNY)
    need = cabi.lib().cmpx_gemm_workspace_size(ctypes.byref(args))
    assert need > 0
    ws = torch.zeros(need // 4 + 64, dtype=torch.int32, device="cuda")
    small = cabi.gemm_args(A, B, C, path=cabi.PATH_SKINNY, workspace=ws.data_ptr(), workspace_bytes=need - 1)
    assert cabi.gemm(small, torch.cuda.current_stream().cuda_stream) == cabi.ERR_WORKSPACE
    for _ in range(3):
        C.fill_(float("nan"))
        a = cabi.gemm_args(A, B, C, path=cabi.PATH_SKINNY, workspace=ws.data_ptr(), workspace_bytes=need)
        assert cabi.gemm(a, torch.cuda.current_stream().cuda_stream) == cabi.OK
        torch.cuda.synchronize()
        assert torch.equal(C, ref)


@pytest.mark.parametrize("shape,groups,nstreams", [((512, 2048, 384), 4, 2), ((300, 1000, 136), 3, 1),
                                                   ((256, 256, 64), 8, 3), ((2304, 1024, 128), 2, 3)],
                         ids=["even", "ragged", "one-column", "two-m-groups"])
def test_gather_ce_local_peers(cuda, shape, groups, nstreams):
    """cmpx_gemm_gather_ce on one GPU, with local buffers standing in for the
    peers' outputs: every "peer" gets the GEMM's rows through the copy
    streams' flag waits and 2-D copies, on three calls in a row (epochs 1-3;
    the flags are never cleared).  Flags count per (M group of 2048 rows,
    column group)."""
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(31)
    A = torch.randn(M, K, generator=g, device="cuda").bfloat16()
    B = (torch.randn(K, N, generator=g, device="cuda") * 0.05).bfloat16()
    want = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
    assert cabi.gemm(cabi.gemm_args(A, B, want)) == cabi.OK
    tiles_m, tiles_n = (M + 255) // 256, (N + 255) // 256
    mgroups = (tiles_m + 7) // 8
    flags = torch.zeros(mgroups * groups, dtype=torch.int32, device="cuda")
    streams = [torch.cuda.Stream() for _ in range(nstreams)]
    cs = (ctypes.c_void_p * nstreams)(*[s.cuda_stream for s in streams])
    for epoch in (1, 2, 3):
        C = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        peers = [torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda") for _ in range(3)]
        pp = (ctypes.c_void_p * 3)(*[p.data_ptr() for p in peers])
        torch.cuda.synchronize()
        st = cabi.lib().cmpx_gemm_gather_ce(ctypes.byref(cabi.gemm_args(A, B, C)), pp, 3, flags.data_ptr(),
                                            flags.numel(), groups, epoch, torch.cuda.current_stream().cuda_stream,
                                            cs, nstreams)
        assert st == cabi.OK, cabi.lib().cmpx_status_string(st)
        torch.cuda.current_stream().synchronize()  # the call made this stream wait for the copies
        assert torch.equal(C, want)
        for p in peers:
            assert torch.equal(p, want)
    ft = (tiles_n + groups - 1) // groups
    ncol = [min(ft, tiles_n - j * ft) for j in range((tiles_n + ft - 1) // ft)]
    nrow = [min(8, tiles_m - i * 8) for i in range(mgroups)]
    want_flags = [3 * mt * nt * 8 for mt in nrow for nt in ncol]
    got_flags = flags.view(mgroups, groups)[:, :len(ncol)].flatten().tolist()
    assert got_flags == want_flags
    assert cabi.device_error() == 0
    # a flags array too small for the blocks is refused
    st = cabi.lib().cmpx_gemm_gather_ce(ctypes.byref(cabi.gemm_args(A, B, C)), pp, 3, flags.data_ptr(),
                                        mgroups * len(ncol) - 1, groups, 4, torch.cuda.current_stream().cuda_stream,
                                        cs, nstreams)
    assert st == cabi.ERR_WORKSPACE
    # shapes that would not run the CTA-pair kernel are refused
    small = torch.empty((64, N), dtype=torch.bfloat16, device="cuda")
    st = cabi.lib().cmpx_gemm_gather_ce(ctypes.byref(cabi.gemm_args(A[:64], B, small)), pp, 3, flags.data_ptr(),
                                        flags.numel(), groups, 4, torch.cuda.current_stream().cuda_stream, cs,
                                        nstreams)
    assert st == cabi.ERR_UNSUPPORTED
