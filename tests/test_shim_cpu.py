"""The cmpext3-compatible operators' argument checks (reference messages,
src/main.cpp:161-170, 196-200, 275-302) -- all raised before any device work,
so they run on CPU tensors."""
import pytest
import torch

import cmp_ext_b200 as cx
import cmpext3


def raises(msg, fn, *a):
    with pytest.raises(RuntimeError, match=msg):
        fn(*a)


def test_drop_in_module_names():
    for name in ("linear", "bmm", "conv2d", "attention", "fp16_matmul", "bf16_matmul", "fp32_matmul"):
        assert getattr(cmpext3, name) is getattr(cx, name)


def test_linear_checks():
    w = torch.zeros(4, 8)
    raises("Input dim >= 2", cx.linear, torch.zeros(8), w)
    raises("Weight dim == 2", cx.linear, torch.zeros(2, 8), torch.zeros(1, 4, 8))
    raises("Input shape mismatch with Weight", cx.linear, torch.zeros(2, 7), w)
    raises("expects CUDA tensors", cx.linear, torch.zeros(2, 8), w)


def test_bmm_checks():
    raises(r"Input must be 3D \(B, M, K\)", cx.bmm, torch.zeros(2, 3), torch.zeros(1, 3, 4))
    raises(r"Mat2 must be 3D \(B, K, N\)", cx.bmm, torch.zeros(1, 2, 3), torch.zeros(3, 4))
    raises("Dtype mismatch", cx.bmm, torch.zeros(1, 2, 3), torch.zeros(1, 3, 4, dtype=torch.float16))
    raises("Batch size mismatch", cx.bmm, torch.zeros(1, 2, 3), torch.zeros(2, 3, 4))
    raises(r"Contracting dimension \(K\) mismatch", cx.bmm, torch.zeros(1, 2, 3), torch.zeros(1, 5, 4))
    raises("expects CUDA tensors", cx.bmm, torch.zeros(1, 2, 3), torch.zeros(1, 3, 4))


def test_matmul_2d_checks():
    h = torch.float16
    raises(r"Input must be 2D \(M, K\)", cx.fp16_matmul, torch.zeros(1, 2, 3, dtype=h), torch.zeros(3, 4, dtype=h))
    raises(r"Mat2 must be 2D \(K, N\)", cx.fp16_matmul, torch.zeros(2, 3, dtype=h), torch.zeros(3, dtype=h))
    raises("Dtype mismatch", cx.fp16_matmul, torch.zeros(2, 3, dtype=h), torch.zeros(3, 4))
    raises("fp16_matmul expects Half tensors", cx.fp16_matmul, torch.zeros(2, 3), torch.zeros(3, 4))
    raises("bf16_matmul expects BFloat16", cx.bf16_matmul, torch.zeros(2, 3), torch.zeros(3, 4))
    raises("fp32_matmul expects Float", cx.fp32_matmul, torch.zeros(2, 3, dtype=h), torch.zeros(3, 4, dtype=h))
    raises(r"Contracting dimension \(K\) mismatch", cx.fp32_matmul, torch.zeros(2, 3), torch.zeros(4, 4))
    raises("expects CUDA tensors", cx.fp32_matmul, torch.zeros(2, 3), torch.zeros(3, 4))


def test_set_path_validation():
    cx._set_path("auto")
    with pytest.raises(RuntimeError, match="unknown path"):
        cx._set_path("fast")


def test_conv2d_checks():
    x = torch.zeros(1, 4, 3, 3)
    w = torch.zeros(6, 4, 1, 1)
    raises(r"Input must be 4D \(NCHW\)", cx.conv2d, torch.zeros(4, 3, 3), w)
    raises(r"Weight must be 4D", cx.conv2d, x, torch.zeros(6, 4))
    raises("groups=1", lambda: cx.conv2d(x, w, None, 1, 0, 1, 2))
    raises("Input channels mismatch weight channels", cx.conv2d, x, torch.zeros(6, 5, 1, 1))
    raises("1x1, stride 1, padding 0", cx.conv2d, x, torch.zeros(6, 4, 3, 3))
    raises("1x1, stride 1, padding 0", lambda: cx.conv2d(x, w, None, 2))
    raises("1x1, stride 1, padding 0", lambda: cx.conv2d(x, w, None, (1, 1), (0, 1)))
    raises("expects CUDA tensors", cx.conv2d, x, w)


def test_host_matmul_argument_checks():
    from cmp_ext_b200.host import host_matmul

    with pytest.raises(ValueError, match="2-D"):
        host_matmul(torch.zeros(2, 3, 4), torch.zeros(4, 5))
    with pytest.raises(ValueError, match="Dtype mismatch"):
        host_matmul(torch.zeros(2, 3), torch.zeros(3, 4, dtype=torch.float16))
    with pytest.raises(ValueError, match="Contracting"):
        host_matmul(torch.zeros(2, 3), torch.zeros(4, 4))


def test_attention_checks():
    """Reference messages of custom_attention_forward (src/main.cpp:1034-1045)."""
    q = torch.zeros(1, 2, 8, 4)
    raises(r"Query must be 4D \(Batch, Head, Seq, Dim\)", cx.attention, torch.zeros(2, 8, 4), q, q)
    raises("Key must be 4D", cx.attention, q, torch.zeros(2, 8, 4), q)
    raises("Value must be 4D", cx.attention, q, q, torch.zeros(2, 8, 4))
    raises("Key shape mismatch", cx.attention, q, torch.zeros(1, 2, 9, 4), q)
    raises("Value shape mismatch", cx.attention, q, q, torch.zeros(1, 2, 8, 5))
    raises("expects CUDA tensors", cx.attention, q, q, q)
    raises("expects CUDA tensors", lambda: cx.attention(q, q, q, scale=0.5))
