"""Drop-in module name for the reference's matmul-path operators.

`import cmpext3` then `cmpext3.linear(...)`, `cmpext3.bmm(...)`,
`cmpext3.attention(...)`, `cmpext3.fp16_matmul(...)` etc. resolve to the
sm_100a implementations in cmp_ext_b200.  Provided: the dense matmul path,
conv2d's 1x1 case (which the reference routes through its matmul) and
scaled dot-product attention (its QK^T and PV products); the reference's
other operators (general conv, norms, activations) are not part of this
build.
"""
from cmp_ext_b200 import attention, bf16_matmul, bmm, conv2d, fp16_matmul, fp32_matmul, linear  # noqa: F401

__all__ = ["linear", "bmm", "conv2d", "attention", "fp16_matmul", "bf16_matmul", "fp32_matmul"]
