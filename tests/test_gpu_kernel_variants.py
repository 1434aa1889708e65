"""The tile-kernel parity tests again, under each fp16/bf16 tile-kernel
variant the dispatcher can pick: single-CTA 128x256 tiles (chosen for M <= 128), and CTA-pair
(cta_group::2) 256x128 and 256x256 tiles, each CTA-pair size also with the
opt-in stream-K split of the last wave.  The variant is fixed per process
(CMPX_TC_PAIR, CMPX_TC_STREAMK), so each runs in a child pytest."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("pair,streamk", [("0", "0"), ("128", "0"), ("256", "0"), ("256", "1"), ("128", "1")])
def test_tile_kernel_variant(cuda, pair, streamk):
    env = dict(os.environ, CMPX_TC_PAIR=pair, CMPX_TC_STREAMK=streamk)
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.join(HERE, "test_gpu_parity.py"), "-k", "tc_path or batched or bias"],
                       env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


@pytest.mark.parametrize("ns", ["2", "4"])
def test_skinny_unit_width_variant(cuda, ns):
    """The skinny kernel with wider work units (2 / 4 sub-slabs), which the
    dispatcher does not pick by default but CMPX_SKINNY_NS can select."""
    env = dict(os.environ, CMPX_SKINNY_NS=ns)
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.join(HERE, "test_gpu_parity.py"), "-k", "skinny"],
                       env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


def test_bf16x3_three_mma_variant(cuda):
    """The fp32 bf16x3 kernel in its three-MMA form (lo*hi, hi*lo, hi*hi at
    width 128); the default form issues hi*[hi | lo] at width 256 plus lo*hi."""
    env = dict(os.environ, CMPX_BF16X3_NCAT="0")
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.join(HERE, "test_gpu_parity.py"), "-k", "bf16x3"],
                       env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]


_ATTN_CHILD = r"""
import sys, torch
import cmp_ext_b200 as cx
outs = []
for dt in (torch.float16, torch.bfloat16):
    for (B, H, S, D, scale) in ((2, 3, 1024, 128, None), (1, 2, 333, 64, None), (1, 1, 257, 128, -0.2),
                                (1, 1, 640, 64, 3.0)):
        g = torch.Generator(device="cuda").manual_seed(S + D)
        q, k, v = (torch.randn(B, H, S, D, generator=g, device="cuda").to(dt) for _ in range(3))
        outs.append(cx.attention(q, k, v, scale=scale).cpu())
torch.save(outs, sys.argv[1])
"""


def test_attention_packed_softmax_bit_identical(cuda, tmp_path):
    """The one-tile tensor-core attention kernel's softmax in paired fp32 /
    three-input max instructions (default) gives the same bits as its scalar form
    (CMPX_ATTN_PACKED=0): fp16 and bf16, D 64 and 128, ragged S, negative
    and large scales."""
    import torch
    res = {}
    for pk in ("1", "0"):
        f = tmp_path / f"attn{pk}.pt"
        env = dict(os.environ, CMPX_ATTN_PACKED=pk, CMPX_ATTN_KERNEL="one", PYTHONPATH=os.path.dirname(HERE))
        r = subprocess.run([sys.executable, "-c", _ATTN_CHILD, str(f)], env=env, capture_output=True, text=True,
                           timeout=600)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
        res[pk] = torch.load(f)
    for a, b in zip(res["1"], res["0"]):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


@pytest.mark.parametrize("kernel", ["pp", "one"])
def test_attention_kernel_variant(cuda, kernel):
    """The attention tests under each tensor-core attention kernel: two
    128-row query tiles per CTA ("pp") and one tile per CTA ("one")."""
    env = dict(os.environ, CMPX_ATTN_KERNEL=kernel)
    r = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                        os.path.join(HERE, "test_gpu_attention.py")],
                       env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
