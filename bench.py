"""Benchmark of the dense matmul path (one JSON line on rank 0).

Default workload: BASELINE config 3 -- bf16_matmul, A [16384, 8192] ~ N(0,1),
B [8192, 8192] ~ N(0,0.02), bf16 out -- M-sharded over the ranks (rank r owns
rows shard_rows(16384, N, r); B replicated; no collective unless --gather).
Total work is fixed as N grows (strong scaling).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config {2,3,4,5,6,7}]
                    [--impl ours|reference] [--gather] [--no-e2e] [--no-cpu]

One step = one pass of the hot path over the resident inputs: one GEMM launch
per rank.  `value` is whole-job TFLOP/s (algorithmic 2*M*N*K over the max over
ranks of the CUDA-event time of K steps).  `e2e` is the same metric through
the public operator (cmp_ext_b200.bf16_matmul) with pinned host inputs copied
in and the result copied out inside the timed region.  `roofline` is the GEMM
kernel's achieved TFLOP/s (or GB/s for the HBM-bound decode config) over the
measured peak in MEASURED_PEAKS.json.  `cpu_baseline` times the CPU
restatement of the reference kernel's arithmetic (oracle/, kind "port") on a
bounded row sample, rank 0 at N=1 only.

--impl reference times the reference's implementation of this path on the
host cores: the reference's kernels are CUDA-only, so its arithmetic is run
through the CPU restatement (oracle/ref_matmul.c, all host threads) on a
bounded row sample per step, reported in the same metric and unit.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from cmp_ext_b200.distributed import shard_rows  # noqa: E402
from cmp_ext_b200.workloads import CONFIGS, make_inputs  # noqa: E402

PEAKS_FILE = os.path.join(REPO, "MEASURED_PEAKS.json")
FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
TRAFFIC_FILE = os.path.join(REPO, "profiles", "dram_traffic.txt")


def peaks():
    try:
        with open(PEAKS_FILE) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return FALLBACK, "fallback"


def traffic_per_launch(key: str):
    """dram__bytes_read.sum + dram__bytes_write.sum per launch, from the
    committed ncu summary (lines `key: <bytes>`), or None."""
    try:
        with open(TRAFFIC_FILE) as f:
            for line in f:
                if line.startswith(key + ":"):
                    return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.path = tempfile.mktemp(prefix="clocks_", suffix=".csv")
        self.proc = None

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-i", str(self.idx), "-lms", "100"], stdout=self.f,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 10:
                    continue
                try:
                    rows.append((float(parts[2]), float(parts[3]), float(parts[4]) if parts[4] not in ("[N/A]", "N/A") else 0.0, parts[6:10]))
                except ValueError:
                    continue
        os.unlink(self.path)
        if not rows:
            return None
        loaded = [r for r in rows if r[2] > 200.0] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in loaded for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in loaded), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(loaded)}


# ------------------------------------------------------------------ helpers
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        if args.impl == "ours":
            torch.cuda.set_device(local)
            import datetime

            dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                    timeout=datetime.timedelta(seconds=180))
        else:
            dist.init_process_group("gloo")
    return world, rank, local


def max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        dist.barrier()


def op_for(dtype):
    import cmp_ext_b200 as cx

    return {torch.float16: cx.fp16_matmul, torch.bfloat16: cx.bf16_matmul, torch.float32: cx.fp32_matmul}[dtype]


def launches_per_step(cfg, rows=None) -> int:
    """Kernels of this library one step launches (per rank): the GEMM, plus
    the two split pre-passes (tf32 or bf16 hi/lo) on the fp32 tensor-core
    paths (fp32 with K % 4 == 0 and more than 2^22 multiply-adds, as all fp32
    configs here)."""
    return 3 if cfg.dtype == torch.float32 else 1


def kernel_name(cfg, m=None) -> str:
    """The dominant kernel of a step, from the library's own path choice."""
    from cmp_ext_b200 import _cmpext3 as ext

    m = cfg.M if m is None else m
    path = ext._matmul_path(m, cfg.N, cfg.K, cfg.dtype_name)
    if path == "skinny":
        return "gemm_skinny_kernel"
    if path == "simt":
        return "gemm_simt_kernel"
    if path == "bf16x3":
        return "gemm_tc_kernel(bf16x3)"
    if cfg.dtype == torch.float32:
        return "gemm_tc_kernel(3xTF32)"
    return "gemm_tc2_kernel (CTA pairs, 256x256)" if m > 128 else "gemm_tc_kernel"


# ------------------------------------------------------------------ CPU legs
def cpu_port_sample(cfg, rows: int, seed: int = 0, reps: int = 1):
    """Times the CPU restatement of the reference kernel (oracle, all host
    threads) on `rows` rows of the workload; returns (TFLOP/s, seconds, threads)."""
    import numpy as np

    from oracle import oracle as o

    kind = cfg.dtype_name
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(rows, cfg.K, generator=g).to(cfg.dtype)
    B = (torch.randn(cfg.K, cfg.N, generator=g) * cfg.b_std).to(cfg.dtype)

    def bits(t):
        return t.numpy() if t.dtype == torch.float32 else t.view(torch.int16).numpy().view(np.uint16)

    a, b = bits(A), bits(B)
    threads = os.cpu_count() or 1
    best = None
    for _ in range(reps):
        t0 = time.perf_counter()
        o.oracle_matmul(kind, a, b, nthreads=threads)
        dt = time.perf_counter() - t0
        best = dt if best is None else min(best, dt)
    return 2.0 * rows * cfg.N * cfg.K / best / 1e12, best, threads


def torch_cpu_sample(cfg, rows: int):
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    A = torch.randn(rows, cfg.K).to(cfg.dtype)
    B = (torch.randn(cfg.K, cfg.N) * cfg.b_std).to(cfg.dtype)
    torch.matmul(A[:8], B)
    t0 = time.perf_counter()
    torch.matmul(A, B)
    dt = time.perf_counter() - t0
    return 2.0 * rows * cfg.N * cfg.K / dt / 1e12, dt, threads


def config_block(cfg, world, gather, transport="nccl"):
    return {"workload": f"config{cfg.cid}: {cfg.name}", "M": cfg.M, "N": cfg.N, "K": cfg.K,
            "a": "N(0,1)" if cfg.a_dist == "normal" else "U(-1,1)",
            "b": f"N(0,{cfg.b_std})" if cfg.a_dist == "normal" else "U(-1,1)",
            "parallelism": f"M-shard x{world}" + ((" + all-gather (" + transport + ")") if gather else ""),
            "l2": "inputs larger than L2 (126 MB) per GPU" if cfg.bytes(cfg.M // world) > 126e6
            else "L2 flushed between steps"}


def metric_of(cfg):
    if cfg.bound == "hbm":
        return "matmul GB/s (algorithmic bytes, HBM roofline)", "GB/s"
    return "matmul TFLOP/s (2*M*N*K, tensor roofline)", "TFLOP/s"


def run_reference(args):
    world, rank, _ = dist_setup(args)
    cfg = CONFIGS[args.config]
    if rank != 0:
        return 0
    metric, unit = metric_of(cfg)
    rows = 16 if args.steps + args.warmup <= 30 else 4
    if cfg.K * cfg.N > 1e8:
        rows = max(1, rows // 2)
    for _ in range(args.warmup):
        cpu_port_sample(cfg, rows)
    times = []
    tflops = []
    for _ in range(args.steps):
        tf, dt, threads = cpu_port_sample(cfg, rows)
        times.append(dt)
        tflops.append(tf)
    total = sum(times)
    flops = 2.0 * rows * cfg.N * cfg.K * args.steps
    value = flops / total / 1e12
    if unit == "GB/s":
        e = torch.empty((), dtype=cfg.dtype).element_size()
        value = args.steps * (rows * cfg.K + cfg.K * cfg.N + rows * cfg.N) * e / total / 1e9
    sample = f"{rows} rows x N={cfg.N} x K={cfg.K} per step of config{cfg.cid}"
    line = {"impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": cfg.dtype_name, "data": "synthetic (seeded N(0,1)/N(0,0.02))",
            "config": config_block(cfg, world, False),
            "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port", "sample": sample,
                             "what": "CPU restatement of the reference kernel arithmetic (oracle/ref_matmul.c); "
                                     "the reference's own kernels are CUDA-only"},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    world, rank, local = dist_setup(args)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    cfg = CONFIGS[args.config]
    metric, unit = metric_of(cfg)
    r0, r1 = shard_rows(cfg.M, world, rank)
    m = r1 - r0 if args.rows is None else args.rows
    if args.quick:
        args.no_e2e = args.no_cpu = True
    op = op_for(cfg.dtype)
    if cfg.dtype == torch.float32 and args.f32_path == "bf16x3":
        from cmp_ext_b200 import _cmpext3 as ext

        ext._set_path("bf16x3")  # every fp32 call of this process, e2e included

    # Inputs resident in HBM (drawn on the device, seeded per config).
    A, B = make_inputs(cfg, device, seed=0, m=m)
    A = A.contiguous()
    flush = None
    if cfg.bytes(m) <= 126e6 * 1.5:
        flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)  # 256 MB > L2

    gather = args.gather and world > 1
    if gather:
        from cmp_ext_b200.distributed import gather_output, sharded_matmul
        if args.transport == "nvlink":
            Cfull = gather_output(cfg.M, cfg.N, cfg.dtype, device)
        else:
            Cfull = torch.empty((cfg.M, cfg.N), dtype=cfg.dtype, device=device)

    def step():
        if flush is not None:
            flush.fill_(1)
        if gather:
            sharded_matmul(A, B, M=cfg.M, gather=True, chunks=args.chunks, out=Cfull, transport=args.transport)
        else:
            op(A, B)

    stream = torch.cuda.current_stream()
    clock = ClockSampler(local)
    if not args.quick:
        clock.start()
    t_start = time.perf_counter()
    for _ in range(args.warmup if args.quick else max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    # keep warming until the clock sampler has produced samples (~0.5 s)
    while not args.quick and time.perf_counter() - t_start < 0.6:
        step()
        torch.cuda.synchronize()

    # kernel-only timing: events bracket exactly the K launches on this stream
    barrier(world)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    flush_ms = 0.0
    if flush is not None:
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(args.steps):
            flush.fill_(1)
        f1.record(stream)
        torch.cuda.synchronize()
        flush_ms = f0.elapsed_time(f1)
    barrier(world)
    torch.cuda.synchronize()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    ms_total = ev0.elapsed_time(ev1)
    barrier(world)
    clocks = clock.stop()
    ms_gemm_total = max(ms_total - flush_ms, 1e-6)
    ms_total = max_over_ranks(ms_total, world, device)
    ms_gemm = max_over_ranks(ms_gemm_total, world, device)

    # Dominant kernel alone (average launch duration, events on its stream).
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kreps = 1 if args.quick else max(5, min(args.steps, 50))
    launch_ms = []
    for _ in range(kreps):
        if flush is not None:
            flush.fill_(1)
        k0.record(stream)
        op(A, B)
        k1.record(stream)
        torch.cuda.synchronize()
        launch_ms.append(k0.elapsed_time(k1))
    launch_ms = statistics.median(launch_ms)

    M_job = cfg.M if args.rows is None else args.rows * world
    step_flops = 2.0 * M_job * cfg.N * cfg.K  # whole job (all ranks)
    e = torch.empty((), dtype=cfg.dtype).element_size()
    step_bytes_job = (M_job * cfg.K + world * cfg.K * cfg.N + M_job * cfg.N) * e
    if unit == "GB/s":
        value = step_bytes_job * args.steps / (ms_gemm / 1e3) / 1e9
    else:
        value = step_flops * args.steps / (ms_gemm / 1e3) / 1e12
    ms_per_step = ms_gemm / args.steps

    P, peak_src = peaks()
    # Average launch duration of the dominant kernel over the timed region:
    # when a step is that one launch and nothing runs between steps, it is
    # the timed region divided by K; otherwise the isolated launch above.
    one_launch = launches_per_step(cfg, args.rows) == 1 and flush is None and not gather
    avg_launch_ms = ms_gemm / args.steps if one_launch else launch_ms
    timing = ("timed region / K (back-to-back launches)" if one_launch
              else "median of isolated launches (events around each)")
    scale = 1e9 if cfg.bound == "hbm" else 1e12
    if cfg.bound == "hbm":
        per_launch = cfg.bytes(m)
        peak = peak_isolated = P["hbm_gbs"]
        peak_kind = "copy"
        runit, rbound = "GB/s", "hbm"
    else:
        # a kernel timed back to back for the whole timed region runs under
        # the power cap: the sustained GEMM figure; an isolated launch: burst
        per_launch = 2.0 * m * cfg.N * cfg.K
        div = 2.0 if cfg.dtype == torch.float32 else 1.0  # tf32 rate = bf16 / 2
        burst = P["bf16_tflops"] / div
        sustained = P.get("bf16_tflops_sustained", P["bf16_tflops"]) / div
        peak, peak_kind = (sustained, "sustained") if one_launch else (burst, "burst")
        peak_isolated = burst
        runit, rbound = "TFLOP/s", "tensor"
    achieved = per_launch / (avg_launch_ms / 1e3) / scale
    achieved_isolated = per_launch / (launch_ms / 1e3) / scale
    traffic = traffic_per_launch(f"config{cfg.cid}_m{m}")

    # End-to-end through the public operator with pinned host buffers.
    e2e = None
    if not args.no_e2e:
        hA = A.cpu().pin_memory()
        hB = B.cpu().pin_memory()
        hC = torch.empty((m, cfg.N), dtype=cfg.dtype).pin_memory()
        e_steps = max(3, min(args.steps, 10))

        from cmp_ext_b200.host import host_matmul

        def e2e_step():
            # host in, host out; uploads, GEMMs and downloads overlapped in row chunks
            host_matmul(hA, hB, out=hC, chunks=8, device=device)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        x0.record(stream)
        for _ in range(e_steps):
            e2e_step()
        x1.record(stream)
        torch.cuda.synchronize()
        e_ms = max_over_ranks(x0.elapsed_time(x1), world, device) / e_steps
        h2d = (hA.numel() + hB.numel()) * e
        d2h = hC.numel() * e
        ev = (step_bytes_job / (e_ms / 1e3) / 1e9) if unit == "GB/s" else (step_flops / (e_ms / 1e3) / 1e12)
        e2e = {"value": ev, "unit": unit, "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
               "ms_per_step": e_ms, "api": "cmp_ext_b200.host.host_matmul (pinned host in/out, 8 row chunks)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        rows = 32 if cfg.K * cfg.N <= 1e8 else 16
        tf, dt, threads = cpu_port_sample(cfg, rows)
        cpu = {"value": tf if unit == "TFLOP/s" else (rows * cfg.K + cfg.K * cfg.N + rows * cfg.N) * e / dt / 1e9,
               "unit": unit, "cores": threads, "kind": "port",
               "sample": f"{rows} rows of config{cfg.cid} ({rows}x{cfg.N}x{cfg.K}), {dt:.2f} s",
               "what": "CPU restatement of the reference kernel arithmetic (oracle/ref_matmul.c)"}
        try:
            ttf, tdt, _ = torch_cpu_sample(cfg, 256 if cfg.M >= 256 else cfg.M)
            cpu["torch_cpu"] = {"value": ttf if unit == "TFLOP/s" else None, "unit": "TFLOP/s",
                                "sample": f"torch.matmul {256 if cfg.M >= 256 else cfg.M} rows, {tdt:.2f} s"}
        except Exception as ex:  # pragma: no cover
            cpu["torch_cpu"] = {"error": str(ex)}

    if rank == 0:
        line = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": cfg.dtype_name, "data": "synthetic (seeded, drawn on device)",
                "config": {**config_block(cfg, world, gather, args.transport),
                           **({"f32_path": args.f32_path} if cfg.dtype == torch.float32 else {})},
                "roofline": {"bound": rbound, "kernel": kernel_name(cfg, m), "achieved": achieved, "peak": peak,
                             "peak_source": peak_src, "unit": runit, "frac": achieved / peak,
                             "traffic": traffic, "launch_ms": avg_launch_ms, "timing": timing,
                             "peak_kind": peak_kind,
                             "isolated_launch": {"ms": launch_ms, "achieved": achieved_isolated,
                                                 "peak": peak_isolated, "frac": achieved_isolated / peak_isolated},
                             "per_launch": per_launch},
                "e2e": e2e, "gpu_launches": args.steps * launches_per_step(cfg, args.rows),
                "clocks": clocks, "cpu_baseline": cpu,
                "step_ms_including_flush": ms_total / args.steps}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=3, choices=[2, 3, 4, 5, 6, 7])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--gather", action="store_true", help="all-gather C to every rank (N>1)")
    ap.add_argument("--chunks", type=int, default=1, help="row chunks for the overlapped gather (1 = in place)")
    ap.add_argument("--transport", default="nccl", choices=["nccl", "nvlink"],
                    help="gather: NCCL all-gather, or epilogue stores into peers' outputs over NVLink")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--quick", action="store_true",
                    help="profiling mode: only W warm-up + K timed steps (no clock sampling, e2e or CPU legs)")
    ap.add_argument("--rows", type=int, default=None, help="override this rank's M rows (profiling small cases)")
    ap.add_argument("--f32-path", default="tf32x3", choices=["tf32x3", "bf16x3"],
                    help="fp32 configs: 3xTF32 (default) or the opt-in bf16x3 split")
    args = ap.parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
