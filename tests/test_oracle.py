"""The CPU oracle (oracle/ref_matmul.c) against independent restatements and
the golden vectors produced by the reference's own kernels on a B200."""
import glob
import os

import numpy as np
import pytest

from oracle import oracle as o

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _bf16_round_ref(x: float) -> int:
    """Nearest bf16 to double x (ties to even), by bracketing with float32 bit patterns."""
    if x == 0.0:
        return 0x8000 if np.signbit(x) else 0
    f = np.float32(x)  # may round; bracket around it
    u = int(np.array(f, dtype=np.float32).view(np.uint32)) >> 16
    best = None
    for c in (u - 1, u, u + 1):
        c &= 0xFFFF
        v = float(np.array(c << 16, dtype=np.uint32).view(np.float32))
        d = abs(v - x)
        key = (d, c & 1)
        if best is None or key < best[0]:
            best = (key, c)
    return best[1]


def test_round_f16_matches_numpy():
    rng = np.random.default_rng(1)
    xs = np.concatenate([
        rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 5, 20000),
        np.array([1.0, 1 + 2 ** -11, 1 + 3 * 2 ** -11, 65504.0, 65519.0, 65520.0, 2 ** -24, 2 ** -25,
                  3 * 2 ** -26, -2 ** -25, 6.1e-5, -0.0]),
    ])
    for x in xs:
        want = int(np.array(np.float16(x)).view(np.uint16))
        assert o.round_f16_bits(float(x)) == want, x


def test_round_bf16_matches_bracketing():
    rng = np.random.default_rng(2)
    xs = rng.standard_normal(5000) * 10.0 ** rng.integers(-30, 30, 5000)
    for x in list(xs) + [1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 1.0 + 2 ** -8 + 2 ** -40]:
        assert o.round_bf16_bits(float(x)) == _bf16_round_ref(float(x)), x


def _emulate_half(A16, B16, kind):
    """Independent numpy restatement: acc = round(a*b + acc) per k, in float64."""
    Ad, Bd = o.bits_to_f64(kind, A16), o.bits_to_f64(kind, B16)
    acc = np.zeros((A16.shape[0], B16.shape[1]))
    for k in range(A16.shape[1]):
        s = Ad[:, k:k + 1] * Bd[k:k + 1, :] + acc
        if kind == "f16":
            acc = s.astype(np.float16).astype(np.float64)
        else:
            acc = np.vectorize(lambda v: o.bits_to_f64("bf16", np.array([_bf16_round_ref(v)], np.uint16))[0])(s)
    return acc


@pytest.mark.parametrize("shape", [(8, 16, 24), (17, 9, 40), (64, 40, 128)])
def test_oracle_f16_bit_exact_vs_numpy(shape):
    M, N, K = shape
    rng = np.random.default_rng(3)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float16).view(np.uint16)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float16).view(np.uint16)
    C = o.oracle_matmul("f16", A, B)
    want = _emulate_half(A, B, "f16").astype(np.float16).view(np.uint16)
    assert np.array_equal(C, want)


def test_oracle_bf16_bit_exact_vs_numpy():
    M, N, K = 6, 5, 24
    rng = np.random.default_rng(4)
    A = np.array([_bf16_round_ref(v) for v in rng.standard_normal(M * K)], np.uint16).reshape(M, K)
    B = np.array([_bf16_round_ref(v * 0.02) for v in rng.standard_normal(K * N)], np.uint16).reshape(K, N)
    C = o.oracle_matmul("bf16", A, B)
    want = _emulate_half(A, B, "bf16")
    assert np.array_equal(o.bits_to_f64("bf16", C), want)


def test_oracle_f32_mul_then_add_ftz():
    rng = np.random.default_rng(5)
    M, N, K = 7, 11, 33
    A = rng.standard_normal((M, K)).astype(np.float32)
    B = rng.standard_normal((K, N)).astype(np.float32)
    A[0, 0] = np.float32(1e-39)  # subnormal input: flushed by the reference (--use_fast_math)
    C = o.oracle_matmul("f32", A, B)
    Af = np.where(np.abs(A) < np.finfo(np.float32).tiny, np.float32(0), A)
    acc = np.zeros((M, N), np.float32)
    for k in range(K):
        acc = (acc + (Af[:, k:k + 1] * B[k:k + 1, :]).astype(np.float32)).astype(np.float32)
    assert np.array_equal(C, acc)


def test_oracle_rows_and_threads():
    rng = np.random.default_rng(6)
    A = rng.uniform(-1, 1, (50, 64)).astype(np.float16).view(np.uint16)
    B = rng.uniform(-1, 1, (64, 24)).astype(np.float16).view(np.uint16)
    full = o.oracle_matmul("f16", A, B, nthreads=1)
    part = o.oracle_matmul("f16", A, B, rows=(10, 37), nthreads=5)
    assert np.array_equal(part[10:37], full[10:37])
    assert not part[:10].any() and not part[37:].any()


def test_oracle_error_is_half_precision_accumulation():
    """The reference accumulates in fp16: its error grows with K far beyond
    the output rounding of an fp32-accumulating kernel."""
    rng = np.random.default_rng(7)
    A = rng.uniform(-1, 1, (32, 1024)).astype(np.float16).view(np.uint16)
    B = rng.uniform(-1, 1, (1024, 32)).astype(np.float16).view(np.uint16)
    C64 = o.fp64_matmul("f16", A, B)
    err = o.normwise_err(o.bits_to_f64("f16", o.oracle_matmul("f16", A, B)), C64)
    fp32acc = o.normwise_err(C64.astype(np.float16).astype(np.float64), C64)
    assert err > 4 * fp32acc


def _golden_files():
    return sorted(glob.glob(os.path.join(GOLDEN, "ref_*.npz")) + glob.glob(os.path.join(GOLDEN, "cfg1_*.npz")))


def test_golden_vectors_present():
    assert _golden_files(), "tests/golden/ref_*.npz missing (generate with tests/golden/make_golden.py on a B200)"


@pytest.mark.parametrize("path", _golden_files(), ids=lambda p: os.path.basename(p))
def test_oracle_matches_reference_kernel_outputs(path):
    """Pins the oracle: the reference's own kernel, run on a B200, produced C;
    the CPU restatement must reproduce it bit for bit."""
    z = np.load(path)
    kind = str(z["dtype"])
    if "A" in z:
        A, B = z["A"], z["B"]
    else:  # config 1: inputs regenerated from the seeded generator, checked by hash
        import hashlib

        from cmp_ext_b200.workloads import CONFIGS, make_inputs

        At, Bt = make_inputs(CONFIGS[1], "cpu", seed=0)
        A, B = At.numpy(), Bt.numpy()
        assert hashlib.sha256(A.tobytes() + B.tobytes()).hexdigest() == str(z["sha256"])
    C = o.oracle_matmul(kind, A, B)
    ref = z["C"]
    if kind == "f32":
        assert np.array_equal(C.view(np.uint32), ref.view(np.uint32))
    else:
        assert np.array_equal(C, ref)
