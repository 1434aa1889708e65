"""The cmpext3-compatible operators on the GPU: linear (weight read in place,
fused bias, N-D input), bmm (one batched launch), conv2d's 1x1 case (batched
GEMM with a shared weight and a per-channel bias), against torch fp32
references of the same op and against the path's contract:

    err(build) <= err(reference operator) + TOL,  err = max|C - C64| / max|C64|

where the reference operator's output is the CPU oracle's product (the
reference kernel's arithmetic, src/cuda/*_matmul.cu) followed by the
reference's bias add (C + bias rounded once, src/main.cpp:240-246), on a
sample of output rows, and C64 is the fp64 result of the same rows.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import cmp_ext_b200 as cx
import cabi
from oracle import oracle as o

pytestmark = pytest.mark.gpu

TOL = {torch.float16: 2e-3, torch.bfloat16: 1.6e-2, torch.float32: 1e-4}


CONTRACT = {torch.float16: 1e-3, torch.bfloat16: 1e-3, torch.float32: 1e-5}
KIND = {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}


def _err(got, want):
    return o.normwise_err(got.double().cpu().numpy(), want.double().cpu().numpy())


def _bits(t):
    t = t.detach().cpu().contiguous()
    return t.numpy() if t.dtype == torch.float32 else t.view(torch.int16).numpy().view(np.uint16)


def _contract(got_rows, a_rows, b_kn, bias=None, max_rows=48):
    """err(got) <= err(reference operator) + TOL on (a sample of) the rows of
    a_rows @ b_kn (+ bias); got_rows holds the build's output for those rows."""
    dtype = a_rows.dtype
    sel = torch.linspace(0, a_rows.shape[0] - 1, min(max_rows, a_rows.shape[0])).long()
    a, got = a_rows[sel].cpu(), got_rows[sel].cpu()
    b = b_kn.cpu()
    kind = KIND[dtype]
    c64 = o.fp64_matmul(kind, _bits(a), _bits(b))
    ref = torch.from_numpy(o.bits_to_f64(kind, o.oracle_matmul(kind, _bits(a), _bits(b))))
    if bias is not None:
        bb = bias.cpu()
        c64 = c64 + bb.double().numpy()[None, :]
        ref = (ref.float() + bb.float()[None, :]).to(dtype).double()  # the reference's separate bias add
    err = o.normwise_err(got.double().numpy(), c64)
    ref_err = o.normwise_err(ref.numpy(), c64)
    assert err <= ref_err + CONTRACT[dtype], (err, ref_err)
    return err, ref_err


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(2, 64, 96, 16, 16), (3, 128, 32, 8, 8), (2, 32, 200, 7, 7), (1, 256, 512, 32, 32)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("bias", [False, True])
def test_conv2d_1x1(cuda, dtype, shape, bias):
    B, Cin, Cout, H, W = shape
    g = torch.Generator(device="cuda").manual_seed(7)
    x = torch.randn(B, Cin, H, W, generator=g, device="cuda").to(dtype)
    w = (torch.randn(Cout, Cin, 1, 1, generator=g, device="cuda") * 0.1).to(dtype)
    b = torch.randn(Cout, generator=g, device="cuda").to(dtype) if bias else None
    y = cx.conv2d(x, w, b)
    assert y.shape == (B, Cout, H, W) and y.dtype == dtype and y.is_contiguous()
    want = F.conv2d(x.float().cpu(), w.float().cpu(), b.float().cpu() if bias else None)
    assert _err(y, want) <= TOL[dtype]
    # contract, in the reference's orientation (NHWC rows x W^T, src/main.cpp:402-424)
    x_rows = x.permute(0, 2, 3, 1).reshape(-1, Cin)
    y_rows = y.permute(0, 2, 3, 1).reshape(-1, Cout)
    _contract(y_rows, x_rows, w.reshape(Cout, Cin).t(), b)


def test_conv2d_tuple_params(cuda):
    x = torch.randn(2, 16, 4, 4, device="cuda", dtype=torch.float16)
    w = torch.randn(8, 16, 1, 1, device="cuda", dtype=torch.float16)
    y = cx.conv2d(x, w, None, (1, 1), (0, 0), (1, 1), 1)
    assert _err(y, F.conv2d(x.float(), w.float())) <= TOL[torch.float16]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_linear_nd_bias(cuda, dtype):
    g = torch.Generator(device="cuda").manual_seed(8)
    x = torch.randn(2, 3, 40, 320, generator=g, device="cuda").to(dtype)
    w = (torch.randn(200, 320, generator=g, device="cuda") * 0.05).to(dtype)
    b = torch.randn(200, generator=g, device="cuda").to(dtype)
    y = cx.linear(x, w, b)
    assert y.shape == (2, 3, 40, 200)
    assert _err(y, x.float() @ w.float().t() + b.float()) <= TOL[dtype]
    _contract(y.reshape(-1, 200), x.reshape(-1, 320), w.t(), b)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(16, 4096, 1024), (300, 520, 264), (1024, 1024, 2048)],
                         ids=lambda s: "x".join(map(str, s)))
def test_linear_contract(cuda, dtype, shape):
    """linear on the decode, ragged and pair-tile shapes: W read as [N,K] in
    place, bias fused; contract against the reference's linear (transposed
    weight, matmul, separate bias add)."""
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(18)
    x = torch.randn(M, K, generator=g, device="cuda").to(dtype)
    w = (torch.randn(N, K, generator=g, device="cuda") * 0.05).to(dtype)
    b = torch.randn(N, generator=g, device="cuda").to(dtype)
    y = cx.linear(x, w, b)
    _contract(y, x, w.t(), b)
    y0 = cx.linear(x, w)
    _contract(y0, x, w.t())


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_bmm(cuda, dtype):
    g = torch.Generator(device="cuda").manual_seed(9)
    a = torch.randn(5, 300, 136, generator=g, device="cuda").to(dtype)
    b = (torch.randn(5, 136, 264, generator=g, device="cuda") * 0.1).to(dtype)
    c = cx.bmm(a, b)
    assert c.shape == (5, 300, 264)
    assert _err(c, torch.bmm(a.float(), b.float())) <= TOL[dtype]
    for i in range(5):
        _contract(c[i], a[i], b[i], max_rows=16)


@pytest.mark.parametrize("path", [cabi.PATH_TC, cabi.PATH_SKINNY, cabi.PATH_SIMT])
def test_shared_a_and_row_bias_cabi(cuda, path):
    """stride_a = 0 (one A for every batch entry) and bias_along_m through the
    C ABI on each path."""
    Bt, M, N, K = 3, 48 if path == cabi.PATH_SKINNY else 200, 264, 136
    g = torch.Generator(device="cuda").manual_seed(10)
    A = torch.randn(M, K, generator=g, device="cuda").half()
    Bm = (torch.randn(Bt, K, N, generator=g, device="cuda") * 0.1).half()
    bias = torch.randn(M, generator=g, device="cuda").half()
    C = torch.full((Bt, M, N), float("nan"), device="cuda", dtype=torch.float16)
    args = cabi.gemm_args(A, Bm[0], C[0], bias=bias, batch=Bt, sa=0, sb=K * N, sc=M * N, path=path)
    args.bias_along_m = 1
    assert cabi.gemm(args) == cabi.OK
    torch.cuda.synchronize()
    want = torch.matmul(A.float(), Bm.float()) + bias.float()[None, :, None]
    assert _err(C, want) <= TOL[torch.float16]


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("chunks", [1, 3, 8])
def test_host_matmul(cuda, dtype, chunks):
    from cmp_ext_b200.host import host_matmul

    g = torch.Generator().manual_seed(12)
    a = torch.randn(1000, 264, generator=g).to(dtype).pin_memory()
    b = (torch.randn(264, 520, generator=g) * 0.1).to(dtype).pin_memory()
    c = host_matmul(a, b, chunks=chunks)
    torch.cuda.synchronize()
    assert not c.is_cuda and c.shape == (1000, 520)
    assert _err(c, a.float() @ b.float()) <= TOL[dtype]
    c2 = torch.zeros_like(c).pin_memory()
    host_matmul(a, b, out=c2, chunks=chunks)
    torch.cuda.synchronize()
    assert torch.equal(c, c2)


def test_bmm_batch_beyond_grid_limit(cuda):
    """More batch entries than a grid dimension holds (65535): processed in
    slices, as the reference's per-batch loop would."""
    a = torch.randn(70000, 2, 8, device="cuda", dtype=torch.float16)
    b = torch.randn(70000, 8, 4, device="cuda", dtype=torch.float16)
    c = cx.bmm(a, b)
    assert _err(c, torch.bmm(a.float(), b.float())) <= TOL[torch.float16]


@pytest.mark.parametrize("shape", [(16, 4096, 8192), (16, 28672, 8192), (8, 1024, 8192)],
                         ids=lambda s: "x".join(map(str, s)))
def test_skinny_in_cuda_graph(cuda, shape):
    """The decode path (stream-K with split-K hand-offs through a
    library workspace) captured in a CUDA graph and replayed on new inputs."""
    M, N, K = shape
    g = torch.Generator(device="cuda").manual_seed(3)
    A = torch.randn(M, K, generator=g, device="cuda").half()
    B = (torch.randn(K, N, generator=g, device="cuda") * 0.02).half()
    first = cx.fp16_matmul(A, B)  # eager call first: workspace and kernel attributes
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        C = cx.fp16_matmul(A, B)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(C, first)
    A.copy_(torch.randn(M, K, generator=g, device="cuda").half())
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(C, cx.fp16_matmul(A, B))
    assert _err(C, A.float() @ B.float()) <= TOL[torch.float16]
