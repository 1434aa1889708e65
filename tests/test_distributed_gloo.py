"""Host-side logic of the M-sharded multi-GPU path, on CPU with gloo ranks.

The per-shard GEMM is replaced by torch.matmul (op=...): what is tested here
is the partitioning, the (chunked, overlapped) all-gather and the reassembly,
plus failure handling of a rank that raises before the collective."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cmp_ext_b200.distributed import shard_rows, sharded_matmul


def test_shard_rows_cover_exactly():
    for M in (1, 7, 16, 100, 16384):
        for world in (1, 2, 3, 4, 8):
            got = [shard_rows(M, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == M
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            sizes = [b - a for a, b in got]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, M, chunks, q, fail_rank):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=__import__("datetime").timedelta(seconds=20))
        g = torch.Generator().manual_seed(0)
        A = torch.randn(M, 24, generator=g)
        B = torch.randn(24, 16, generator=g)
        r0, r1 = shard_rows(M, world, rank)
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        local = sharded_matmul(A[r0:r1], B, op=torch.matmul)
        full = sharded_matmul(A[r0:r1].contiguous(), B, M=M, gather=True, chunks=chunks, op=torch.matmul)
        ok = torch.allclose(local, A[r0:r1] @ B, atol=1e-5) and torch.allclose(full, A @ B, atol=1e-5)
        q.put((rank, "ok" if ok else "mismatch"))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, f"error: {e}"))


def _run(world, M, chunks, fail_rank=-1, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, M, chunks, q, fail_rank)) for r in range(world)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(timeout)
    for p in ps:
        if p.is_alive():
            p.kill()
    out = {}
    while not q.empty():
        r, s = q.get()
        out[r] = s
    return out


@pytest.mark.parametrize("M,chunks", [(32, 1), (32, 3), (31, 1)])
def test_sharded_gather_world2(M, chunks):
    out = _run(2, M, chunks)
    assert out == {0: "ok", 1: "ok"}, out


def test_rank_failure_is_reported_not_hung():
    """Rank 1 raises before the collective; rank 0's gather must end with an
    error (process-group timeout) instead of hanging."""
    out = _run(2, 32, 1, fail_rank=1, timeout=90)
    assert out.get(1, "").startswith("error: injected"), out
    assert out.get(0, "").startswith("error"), out
