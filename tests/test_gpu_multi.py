"""M-sharded matmul with one process per GPU, launched as child processes:
on two GPUs (skipped on a one-GPU box) and as a one-rank job (runs on any
box, so the collective plumbing runs on every GPU test pass).  Checks that
every rank ends up with the full product -- NCCL in-place gather, NCCL
chunked gather, and the fused NVLink epilogue stores into symmetric memory --
equal to the product one GPU computes, and that the host-to-host sharded
matmul (B uploaded in slices and all-gathered) gives each rank its rows."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)

WORKER = r"""
import os, sys, torch, torch.distributed as dist
sys.path.insert(0, os.environ["REPO"])
from cmp_ext_b200.distributed import shard_rows, sharded_matmul
import cmp_ext_b200 as cx
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
import datetime
dist.init_process_group("nccl", device_id=torch.device("cuda", rank), timeout=datetime.timedelta(seconds=60))
g = torch.Generator(device="cuda").manual_seed(0)
M, K, N = 2048, 1024, 768
A = torch.randn(M, K, generator=g, device="cuda").bfloat16()
B = (torch.randn(K, N, generator=g, device="cuda") * 0.05).bfloat16()
full = cx.bf16_matmul(A, B)
r0, r1 = shard_rows(M, world, rank)
for chunks in (1, 4):
    C = sharded_matmul(A[r0:r1].contiguous(), B, M=M, gather=True, chunks=chunks)
    torch.cuda.synchronize()
    err = ((C.float() - full.float()).abs().max() / full.float().abs().max()).item()
    assert err <= 2 ** -7, (chunks, err)
from cmp_ext_b200.distributed import gather_output
out = gather_output(M, N, torch.bfloat16, "cuda")
for rep in range(2):
    out.fill_(float("nan"))
    dist.barrier()
    C = sharded_matmul(A[r0:r1].contiguous(), B, M=M, gather=True, transport="nvlink", out=out)
    torch.cuda.synchronize()
    assert not torch.isnan(C.float()).any(), "nvlink gather left rows unwritten"
    err = ((C.float() - full.float()).abs().max() / full.float().abs().max()).item()
    assert err <= 2 ** -7, ("nvlink", err)
out2 = gather_output(M, N, torch.bfloat16, "cuda")
for rep in range(3):  # copy-engine transport: flags are never reset, so repeat calls matter
    out2.fill_(float("nan"))
    dist.barrier()
    C = sharded_matmul(A[r0:r1].contiguous(), B, M=M, gather=True, transport="ce", out=out2)
    torch.cuda.synchronize()
    assert not torch.isnan(C.float()).any(), "ce gather left rows unwritten"
    err = ((C.float() - full.float()).abs().max() / full.float().abs().max()).item()
    assert err <= 2 ** -7, ("ce", err)
out3 = gather_output(M, N, torch.bfloat16, "cuda")
from cmp_ext_b200.distributed import _SYMM
h3 = _SYMM[out3.data_ptr()]
if world > 1 and h3.has_multicast_support and int(h3.multicast_ptr) != 0:
    for rep in range(3):  # epilogue stores through the NVLink multicast address
        out3.fill_(float("nan"))
        dist.barrier()
        C = sharded_matmul(A[r0:r1].contiguous(), B, M=M, gather=True, transport="nvls", out=out3)
        torch.cuda.synchronize()
        assert not torch.isnan(C.float()).any(), "nvls gather left rows unwritten"
        err = ((C.float() - full.float()).abs().max() / full.float().abs().max()).item()
        assert err <= 2 ** -7, ("nvls", err)
    print("rank", rank, "nvls checked")
from cmp_ext_b200.distributed import sharded_host_matmul
hA = A[r0:r1].cpu().pin_memory()
hB = B.cpu().pin_memory()
for K_cut in (K, K - 1):  # K % world == 0 (slices gathered) and, at 2 ranks, ragged K (full upload)
    hC = sharded_host_matmul(hA[:, :K_cut].contiguous(), hB[:K_cut].contiguous(), chunks=3)
    torch.cuda.synchronize()
    want = cx.bf16_matmul(A[r0:r1, :K_cut].contiguous(), B[:K_cut].contiguous()).cpu()
    err = ((hC.float() - want.float()).abs().max() / want.float().abs().max()).item()
    assert err <= 2 ** -7, ("host", K_cut, err)
mine = sharded_matmul(A[r0:r1].contiguous(), B)
assert torch.equal(mine, full[r0:r1]) or ((mine.float() - full[r0:r1].float()).abs().max() / full.float().abs().max()).item() <= 2 ** -7
dist.barrier()
dist.destroy_process_group()
print("rank", rank, "ok")
"""


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("world", [1, 2])
def test_sharded_gather(cuda, tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    script = tmp_path / "worker.py"
    script.write_text(WORKER)
    env = dict(os.environ, REPO=REPO, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
                        "--master-addr=127.0.0.1", f"--master-port={_port()}", str(script)],
                       env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    assert r.stdout.count(" ok") == world
    if world > 1:  # which transports ran is visible with -rP
        print("multicast transport checked on", r.stdout.count("nvls checked"), "of", world, "ranks")
