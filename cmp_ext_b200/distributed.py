"""M-sharded GEMM across the GPUs of one node (one process per GPU).

The reference has no multi-GPU code; this is the partitioning the path admits:
C = A @ B splits into independent row blocks, so rank r owns rows
[r0, r1) of A and C while B is replicated.  No data-path collective is needed
unless the caller wants the full C on every rank, in which case the row
blocks are all-gathered over NCCL (NVLink / NVSwitch).  Chunked gathering
(``chunks > 1``) overlaps the all-gather of finished row chunks with the
GEMM of the next chunk on a second stream.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

# Symmetric-memory outputs registered by gather_output(): data_ptr -> handle.
_SYMM = {}
# transport="ce" state per output: column-progress flags, call count, copy streams.
_CE = {}


def shard_rows(M: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced row range [r0, r1) of rank `rank` out of `world`."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} for world size {world}")
    base, extra = divmod(M, world)
    r0 = rank * base + min(rank, extra)
    return r0, r0 + base + (1 if rank < extra else 0)


def gather_output(M: int, N: int, dtype: torch.dtype, device, group=None) -> torch.Tensor:
    """Allocates the full [M, N] output for ``sharded_matmul(..., gather=True,
    transport="nvlink" | "ce" | "nvls")``: a symmetric-memory tensor mapped
    into every rank of `group` (a collective call; every rank passes the
    same shape), bound to an NVLink multicast object where the system
    supports one ("nvls").  The buffer is reused by every call given it."""
    import torch.distributed._symmetric_memory as symm_mem

    t = symm_mem.empty((M, N), dtype=dtype, device=device)
    h = symm_mem.rendezvous(t, group if group is not None else dist.group.WORLD)
    _SYMM[t.data_ptr()] = h
    return t


def default_op(dtype: torch.dtype) -> Callable[[torch.Tensor, torch.Tensor], torch.Tensor]:
    import cmp_ext_b200 as cx

    return {torch.float16: cx.fp16_matmul, torch.bfloat16: cx.bf16_matmul, torch.float32: cx.fp32_matmul}[dtype]


def sharded_matmul(a_shard: torch.Tensor, b: torch.Tensor, *, M: int | None = None, gather: bool = False,
                   chunks: int = 1, group=None, op=None, out: torch.Tensor | None = None,
                   transport: str = "nccl", ce_groups: int = 4) -> torch.Tensor:
    """This rank's rows of A @ B, or (gather=True) the full product on every rank.

    a_shard: this rank's rows of A, as given by ``shard_rows(M, world, rank)``.
    M: total rows (needed when gathering; defaults to a_shard rows x world,
       which is right when M divides evenly).
    gather: each rank computes straight into its row block of the full
       output and the blocks are all-gathered in place over NCCL -- no
       staging buffer and no extra copy.
    chunks: with gather=True (NCCL transport), split the shard into this
       many row chunks; chunk i's rows are sent to every peer (point-to-point,
       received in place) while chunk i+1 is multiplied.
    op: the per-shard GEMM (defaults to cmp_ext_b200's *_matmul for the dtype;
       tests on CPU pass torch.matmul).
    transport: "nvls": the GEMM's epilogue writes each output element once
       through the buffer's NVLink multicast address and the switch delivers
       it to every rank's output, so each GPU sends its rows once instead of
       once per peer.  Otherwise "nccl" (all-gather after the GEMM), "nvlink" (the GEMM's
       epilogue stores every output tile to its own rows and, over NVLink, to
       the same rows of every peer's output, overlapping the exchange with the
       remaining tiles) or "ce" (the GEMM counts finished tile columns in
       device flags; one copy stream per peer waits on each group of columns
       and copies it to the peer's output with the copy engines, so the
       exchange overlaps the GEMM without taking SM time).  "nvlink" and
       "ce" need `out` from gather_output() and evenly divided rows; a
       device-side barrier before and after the call orders the reuse of
       every rank's output.
    """
    op_is_default = op is None
    op = op or default_op(a_shard.dtype)
    if not gather:
        return op(a_shard, b)
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    M = a_shard.shape[0] * world if M is None else M
    N = b.shape[1]
    sizes = [shard_rows(M, world, r)[1] - shard_rows(M, world, r)[0] for r in range(world)]
    if sizes[rank] != a_shard.shape[0]:
        raise ValueError(f"rank {rank} holds {a_shard.shape[0]} rows, expected {sizes[rank]}")
    if out is None:
        out = torch.empty((M, N), dtype=a_shard.dtype, device=a_shard.device)
    even = all(s == sizes[0] for s in sizes)
    if not even:
        # Ragged shards: gather padded blocks, then compact.
        rows = max(sizes)
        local = torch.zeros((rows, N), dtype=a_shard.dtype, device=a_shard.device)
        local[: sizes[rank]] = op(a_shard, b)
        buf = torch.empty((world * rows, N), dtype=a_shard.dtype, device=a_shard.device)
        dist.all_gather_into_tensor(buf, local, group=group)
        for r in range(world):
            r0, r1 = shard_rows(M, world, r)
            out[r0:r1] = buf[r * rows: r * rows + sizes[r]]
        return out
    S = sizes[0]
    if transport == "nvlink":
        h = _SYMM.get(out.data_ptr())
        if h is None or out.shape != (M, N) or not out.is_contiguous():
            raise ValueError("transport='nvlink' needs the output from gather_output(M, N, ...)")
        if not op_is_default:
            raise ValueError("transport='nvlink' runs the library's own GEMM (op must be None)")
        import cmp_ext_b200 as cx

        row_bytes = N * out.element_size()
        offset = rank * S * row_bytes
        peers = [int(h.buffer_ptrs[p]) + offset for p in range(world) if p != rank]
        h.barrier(channel=0)  # every rank is done with the previous contents of its output
        cx._matmul_into(a_shard, b, out[rank * S:(rank + 1) * S], peers)
        h.barrier(channel=0)  # every rank's stores into every output are done
        return out
    elif transport == "nvls":
        h = _SYMM.get(out.data_ptr())
        if h is None or out.shape != (M, N) or not out.is_contiguous():
            raise ValueError("transport='nvls' needs the output from gather_output(M, N, ...)")
        if not op_is_default:
            raise ValueError("transport='nvls' runs the library's own GEMM (op must be None)")
        mc = int(h.multicast_ptr) if h.has_multicast_support else 0
        if mc == 0:
            raise RuntimeError("transport='nvls': no NVLink multicast support for this buffer")
        import cmp_ext_b200 as cx

        offset = rank * S * N * out.element_size()
        h.barrier(channel=0)  # every rank is done with the previous contents of its output
        cx._matmul_into(a_shard, b, out[rank * S:(rank + 1) * S], [], mc + offset)
        h.barrier(channel=0)  # every rank's multicast stores have landed everywhere
        return out
    elif transport == "ce":
        h = _SYMM.get(out.data_ptr())
        if h is None or out.shape != (M, N) or not out.is_contiguous():
            raise ValueError("transport='ce' needs the output from gather_output(M, N, ...)")
        if not op_is_default:
            raise ValueError("transport='ce' runs the library's own GEMM (op must be None)")
        import cmp_ext_b200 as cx

        st = _CE.get(out.data_ptr())
        if st is None:
            # one flag per (M group, column group); an M group is at least one
            # 256-row pair tile, whatever the raster's group height
            nflags = ((S + 255) // 256) * ce_groups
            st = {"flags": torch.zeros(nflags, dtype=torch.int32, device=out.device), "epoch": 0,
                  "streams": [torch.cuda.Stream(out.device) for _ in range(max(1, world - 1))]}
            _CE[out.data_ptr()] = st
        st["epoch"] += 1
        row_bytes = N * out.element_size()
        offset = rank * S * row_bytes
        peers = [int(h.buffer_ptrs[p]) + offset for p in range(world) if p != rank]
        h.barrier(channel=0)  # every rank is done with the previous contents of its output
        cx._matmul_gather_ce(a_shard, b, out[rank * S:(rank + 1) * S], peers, st["flags"], ce_groups, st["epoch"],
                             [s.cuda_stream for s in st["streams"]])
        h.barrier(channel=0)  # every rank's copies into every output have landed
        return out
    elif transport != "nccl":
        raise ValueError(f"unknown transport {transport!r}")
    chunks = max(1, min(chunks, S))
    if chunks == 1:
        mine = out[rank * S:(rank + 1) * S]
        if op_is_default and a_shard.is_cuda:
            import cmp_ext_b200 as cx

            cx._matmul_into(a_shard, b, mine)
        else:
            mine.copy_(op(a_shard, b))
        dist.all_gather_into_tensor(out, mine, group=group)  # in place: input is this rank's block of out
        return out
    # Chunked: the GEMM runs in row chunks, and as soon as chunk i is queued
    # its rows go to every peer with point-to-point sends, received straight
    # into the peers' row blocks of `out` (one NCCL group of sends and
    # receives per chunk: an all-gather with in-place destinations, no
    # staging buffer and no reorder copy).  NCCL's stream waits for the
    # chunk's GEMM; the next chunk's GEMM runs on the compute stream while
    # the previous chunk is on the wire.
    bounds = [(S * i // chunks, S * (i + 1) // chunks) for i in range(chunks)]
    mine = out[rank * S:(rank + 1) * S]
    works = []
    for c0, c1 in bounds:
        if c1 == c0:
            continue
        if op_is_default and a_shard.is_cuda:
            import cmp_ext_b200 as cx

            cx._matmul_into(a_shard[c0:c1], b, mine[c0:c1])
        else:
            mine[c0:c1].copy_(op(a_shard[c0:c1], b))
        ops = []
        for q in range(world):
            if q == rank:
                continue
            peer = dist.get_global_rank(group, q) if group is not None else q
            ops.append(dist.P2POp(dist.isend, mine[c0:c1], peer, group))
            ops.append(dist.P2POp(dist.irecv, out[q * S + c0:q * S + c1], peer, group))
        if ops:
            works.extend(dist.batch_isend_irecv(ops))
    for w in works:
        w.wait()
    return out


def sharded_host_matmul(a_host: torch.Tensor, b_host: torch.Tensor, *, out: torch.Tensor | None = None,
                        chunks: int = 8, group=None, device=None) -> torch.Tensor:
    """This rank's rows of A @ B from (pinned) host memory, with B crossing
    PCIe once per job instead of once per rank.

    a_host: this rank's rows of A [m, K]; b_host: the full B [K, N] (the same
    on every rank).  Rank r copies only its slice of B's rows
    ``shard_rows(K, world, r)`` to its GPU, and the slices are all-gathered
    in place over NCCL (NVLink) into the full device copy of B, while this
    rank's A row chunks stream in on a copy stream.  Each A chunk is
    multiplied as soon as it and B are on the device, and each C chunk is
    copied back to `out` (pinned host [m, N]) on a third stream, as in
    ``host_matmul``.  At 8 ranks this moves B's 134 MB (config 3) over PCIe
    once per job instead of eight times.

    The work is queued on the current stream of `device` and two helper
    streams; the result is in `out` once the current stream reaches the end
    of this call.  Every rank of `group` must call it with the same B shape.
    """
    import cmp_ext_b200 as cx

    if a_host.dim() != 2 or b_host.dim() != 2:
        raise ValueError("sharded_host_matmul expects 2-D tensors")
    if a_host.is_cuda or b_host.is_cuda:
        raise ValueError("sharded_host_matmul takes host tensors")
    if a_host.dtype != b_host.dtype:
        raise ValueError("Dtype mismatch")
    if a_host.shape[1] != b_host.shape[0]:
        raise ValueError("Contracting dimension (K) mismatch")
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    m, K = a_host.shape
    N = b_host.shape[1]
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if out is None:
        out = torch.empty((m, N), dtype=a_host.dtype, pin_memory=True)
    elif out.shape != (m, N) or out.dtype != a_host.dtype or out.is_cuda or not out.is_contiguous():
        raise ValueError("out must be a contiguous host tensor of shape [m, N] and the inputs' dtype")
    with torch.cuda.device(dev):
        compute = torch.cuda.current_stream(dev)
        s_in = torch.cuda.Stream(dev)
        s_out = torch.cuda.Stream(dev)
        s_in.wait_stream(compute)
        s_out.wait_stream(compute)
        dB = torch.empty((K, N), dtype=b_host.dtype, device=dev)
        even = K % world == 0
        with torch.cuda.stream(s_in):
            if even:
                k0, k1 = rank * (K // world), (rank + 1) * (K // world)
                dB[k0:k1].copy_(b_host[k0:k1], non_blocking=True)
                # in place: this rank's slice of dB is the input (NCCL waits for s_in's upload)
                work = dist.all_gather_into_tensor(dB, dB[k0:k1], group=group, async_op=True)
            else:
                dB.copy_(b_host, non_blocking=True)  # ragged K: every rank uploads all of B
                work = None
        if work is not None:
            work.wait()  # the compute stream waits for the gathered B (the host does not)
        else:
            compute.wait_stream(s_in)
        dA = torch.empty((m, K), dtype=a_host.dtype, device=dev)
        dC = torch.empty((m, N), dtype=a_host.dtype, device=dev)
        chunks = max(1, min(chunks, m)) if m > 0 else 1
        bounds = [(m * i // chunks, m * (i + 1) // chunks) for i in range(chunks)]
        for r0, r1 in bounds:
            if r1 == r0:
                continue
            with torch.cuda.stream(s_in):
                dA[r0:r1].copy_(a_host[r0:r1], non_blocking=True)
            compute.wait_event(s_in.record_event())
            cx._matmul_into(dA[r0:r1], dB, dC[r0:r1])
            s_out.wait_event(compute.record_event())
            with torch.cuda.stream(s_out):
                out[r0:r1].copy_(dC[r0:r1], non_blocking=True)
        compute.wait_stream(s_out)
        for t in (dA, dB, dC):
            t.record_stream(s_in)
            t.record_stream(s_out)
    return out
