"""Host-to-host matmul with the PCIe transfers overlapped.

For callers whose operands live in (pinned) host memory, the copies dominate
a large GEMM on a B200: for bf16 16384 x 8192 x 8192, moving A and B in
(402 MB) and C out (268 MB) one after the other takes ~13 ms against ~1.5 ms
of compute.  `host_matmul` moves B first (every row block of C needs all of
it), then streams A in row chunks on one stream, multiplies each chunk as it
lands on the compute stream, and copies each finished C chunk back on a third
stream, so host-to-device copies, GEMMs and device-to-host copies run
concurrently on the GPU's separate copy engines and SMs.
"""
from __future__ import annotations

import torch


def host_matmul(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None, chunks: int = 8,
                device: torch.device | int | None = None) -> torch.Tensor:
    """out = a @ b for 2-D host tensors a [M,K], b [K,N] (fp16 / bf16 / fp32).

    a, b (and out, if given) should be pinned for the copies to be
    asynchronous.  Returns `out` (a new pinned tensor when not given).  The
    work is queued on the current CUDA stream of `device` and its two helper
    streams; the result is ready when the current stream reaches the end of
    this call (e.g. after torch.cuda.synchronize()).
    """
    import cmp_ext_b200 as cx

    if a.dim() != 2 or b.dim() != 2:
        raise ValueError("host_matmul expects 2-D tensors")
    if a.is_cuda or b.is_cuda:
        raise ValueError("host_matmul takes host tensors; use fp16_matmul & co. for device tensors")
    if a.dtype != b.dtype:
        raise ValueError("Dtype mismatch")
    if a.shape[1] != b.shape[0]:
        raise ValueError("Contracting dimension (K) mismatch")
    M, K = a.shape
    N = b.shape[1]
    if device is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    elif isinstance(device, int):
        dev = torch.device("cuda", device)
    else:
        dev = torch.device(device)
    a = a.contiguous()
    b = b.contiguous()
    if out is None:
        out = torch.empty((M, N), dtype=a.dtype, pin_memory=True)
    elif out.shape != (M, N) or out.dtype != a.dtype or out.is_cuda or not out.is_contiguous():
        raise ValueError("out must be a contiguous host tensor of shape [M, N] and the inputs' dtype")
    if M == 0 or N == 0:
        return out

    with torch.cuda.device(dev):
        compute = torch.cuda.current_stream(dev)
        s_in = torch.cuda.Stream(dev)
        s_out = torch.cuda.Stream(dev)
        s_in.wait_stream(compute)   # the copies follow everything queued before this call
        s_out.wait_stream(compute)
        dA = torch.empty((M, K), dtype=a.dtype, device=dev)
        dB = torch.empty((K, N), dtype=a.dtype, device=dev)
        dC = torch.empty((M, N), dtype=a.dtype, device=dev)
        chunks = max(1, min(chunks, M))
        bounds = [(M * i // chunks, M * (i + 1) // chunks) for i in range(chunks)]
        with torch.cuda.stream(s_in):
            dB.copy_(b, non_blocking=True)
        ev_b = s_in.record_event()
        compute.wait_event(ev_b)
        for r0, r1 in bounds:
            if r1 == r0:
                continue
            with torch.cuda.stream(s_in):
                dA[r0:r1].copy_(a[r0:r1], non_blocking=True)
            compute.wait_event(s_in.record_event())
            cx._matmul_into(dA[r0:r1], dB, dC[r0:r1])  # on the compute (current) stream
            s_out.wait_event(compute.record_event())
            with torch.cuda.stream(s_out):
                out[r0:r1].copy_(dC[r0:r1], non_blocking=True)
        compute.wait_stream(s_out)
        # keep the device buffers alive until the streams are done with them
        for t in (dA, dB, dC):
            t.record_stream(s_in)
            t.record_stream(s_out)
    return out
