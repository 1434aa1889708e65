"""Drop-in module name for the reference's matmul operators.

`import cmpext3` then `cmpext3.linear(...)`, `cmpext3.bmm(...)`,
`cmpext3.fp16_matmul(...)` etc. resolve to the sm_100a implementations in
cmp_ext_b200.  Only the dense matmul path is provided, plus conv2d's 1x1
case (which the reference routes through its matmul); the reference's other
operators (general conv, attention, norms, activations) are not part of this
build.
"""
from cmp_ext_b200 import bf16_matmul, bmm, conv2d, fp16_matmul, fp32_matmul, linear  # noqa: F401

__all__ = ["linear", "bmm", "conv2d", "fp16_matmul", "bf16_matmul", "fp32_matmul"]
