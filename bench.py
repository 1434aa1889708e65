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
REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}


class ClockSampler:
    """SM clock, power and throttle reasons of one GPU, sampled every ~5 ms
    by a thread (NVML) between start() and stop(): only the timed region is
    sampled, so even a 30 ms region yields a handful of samples.  Falls back
    to `nvidia-smi -lms 100` when NVML is unavailable."""

    def __init__(self, device: torch.device):
        self.device = device
        self.samples = []
        self._stop = None
        self._thread = None
        self._smi = None
        self.handle = None
        try:
            import pynvml

            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByUUID("GPU-" + uuid if not uuid.startswith("GPU-") else uuid)
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(device.index or 0)
            self.nvml = pynvml
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM))
        except Exception:
            self.handle = None

    def _poll(self):
        import threading  # noqa: F401

        nv = self.nvml
        while not self._stop.is_set():
            try:
                mhz = float(nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM))
                pw = nv.nvmlDeviceGetPowerUsage(self.handle) / 1000.0
                rs = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                self.samples.append((mhz, pw, rs))
            except Exception:
                pass
            self._stop.wait(0.005)

    def start(self):
        self.samples = []
        if self.handle is not None:
            import threading

            self._stop = threading.Event()
            self._thread = threading.Thread(target=self._poll, daemon=True)
            self._thread.start()
        else:
            try:
                self._path = tempfile.mktemp(prefix="clocks_", suffix=".csv")
                self._f = open(self._path, "w")
                self._smi = subprocess.Popen(
                    ["nvidia-smi", "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active",
                     "--format=csv,noheader,nounits", "-i", str(self.device.index or 0), "-lms", "100"],
                    stdout=self._f, stderr=subprocess.DEVNULL)
            except OSError:
                self._smi = None

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=2)
            self._thread = None
            rows = self.samples
            max_mhz = self.max_mhz
            src = "nvml, ~5 ms"
        elif self._smi is not None:
            self._smi.terminate()
            try:
                self._smi.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self._smi.kill()
            self._f.close()
            rows, max_mhz = [], 0.0
            with open(self._path) as f:
                for line in f:
                    parts = [p.strip() for p in line.split(",")]
                    try:
                        rows.append((float(parts[0]), float(parts[2]), int(parts[3], 16)))
                        max_mhz = max(max_mhz, float(parts[1]))
                    except (ValueError, IndexError):
                        continue
            os.unlink(self._path)
            self._smi = None
            src = "nvidia-smi, 100 ms"
        else:
            return None
        if not rows:
            return None
        reasons = sorted({n for r in rows for n, bit in REASON_BITS.items() if r[2] & bit})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max_mhz,
                "sm_mhz_min": min(r[0] for r in rows), "power_w_max": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows), "sampler": src, "window": "timed region only"}


def pick_peak(P, clocks, div=1.0):
    """Burst or sustained GEMM peak, chosen from the state the run was
    measured in: sustained when the power cap was active or the SM clock sat
    well below its maximum, burst otherwise."""
    burst = P["bf16_tflops"] / div
    sustained = P.get("bf16_tflops_sustained", P["bf16_tflops"]) / div
    if clocks is None:
        return sustained, "sustained (no clock record)"
    capped = "sw_power_cap" in clocks["reasons"] or clocks["sm_mhz"] < 0.85 * max(clocks["sm_max_mhz"], 1.0)
    return (sustained, "sustained (power-capped clocks seen)") if capped else (burst, "burst (clocks at max)")


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


class Timer:
    """Times K back-to-back steps on this rank's stream, max over ranks,
    after holding the GPU busy for `hold_s` seconds (so every run, whatever
    N, is measured in the same power state), with the clocks sampled inside
    the timed region only."""

    def __init__(self, world, device, quick, hold_s):
        self.world, self.device, self.quick, self.hold_s = world, device, quick, hold_s
        self.stream = torch.cuda.current_stream(device)
        self.clock = None if quick else ClockSampler(device)

    def hold(self, step, warmup):
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        if self.quick:
            return
        t0 = time.perf_counter()
        n = 1
        while time.perf_counter() - t0 < self.hold_s:
            for _ in range(n):
                step()
            torch.cuda.synchronize()
            n = min(n * 2, 64)

    def run(self, step, steps, warmup):
        """(ms of the K back-to-back steps, max over ranks; clocks)."""
        self.hold(step, warmup)
        barrier(self.world)
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        if self.clock is not None:
            self.clock.start()
        ev0.record(self.stream)
        for _ in range(steps):
            step()
        ev1.record(self.stream)
        torch.cuda.synchronize()
        clocks = self.clock.stop() if self.clock is not None else None
        barrier(self.world)
        ms = ev0.elapsed_time(ev1)
        return max_over_ranks(ms, self.world, self.device), clocks

    def isolated(self, fn, reps):
        """Median event time of single launches, each after a device sync."""
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        out = []
        for _ in range(reps):
            torch.cuda.synchronize()
            k0.record(self.stream)
            fn()
            k1.record(self.stream)
            torch.cuda.synchronize()
            out.append(k0.elapsed_time(k1))
        return statistics.median(out)


L2_BYTES = 126e6


def input_sets(cfg, device, m, rank):
    """Resident input sets for one workload: enough of them that the sets a
    step cycles through exceed three times the L2 (126 MB), so consecutive
    steps never find their operands in L2 and no flush is needed."""
    n = max(1, min(16, int(-(-3 * L2_BYTES // cfg.bytes(m))))) if cfg.bytes(m) < 3 * L2_BYTES else 1
    sets = [make_inputs(cfg, device, seed=0 if i == 0 else 7 + i, m=m, a_seed=1000 + rank + 64 * i)
            for i in range(n)]
    desc = ("inputs larger than L2 (126 MB) per GPU" if n == 1 else
            f"{n} resident input sets rotated per step ({n * cfg.bytes(m) / 1e6:.0f} MB > 3 x L2); no flush")
    return sets, desc


def rows_err(C, A, B, rows=64):
    """Normwise error max|C - C64| / max|C64| of a spread sample of C's rows
    against the fp64 product of the same rows (computed on the GPU)."""
    M = A.shape[0]
    idx = torch.linspace(0, M - 1, min(rows, M), device=A.device).long()
    ref = A[idx].double() @ B.double()
    return float((C[idx].double() - ref).abs().max() / ref.abs().max())


def tensor_record(cfg, m, ms_step, clocks, P, kernel, launch_ms=None, extra=None):
    """One measured workload: TFLOP/s (or GB/s) and its roofline fraction."""
    e = torch.empty((), dtype=cfg.dtype).element_size()
    rec = {"workload": f"config{cfg.cid}: {cfg.name}" + ("" if m == cfg.M else f" ({m} rows)"), "kernel": kernel,
           "ms_per_step": ms_step, "clocks": clocks}
    if cfg.bound == "hbm":
        byt = (m * cfg.K + cfg.K * cfg.N + m * cfg.N) * e
        ach = byt / (ms_step / 1e3) / 1e9
        rec.update({"value": ach, "unit": "GB/s", "roofline": {"bound": "hbm", "achieved": ach, "peak": P["hbm_gbs"],
                    "peak_kind": "measured copy", "frac": ach / P["hbm_gbs"], "unit": "GB/s"}})
        if launch_ms:
            rec["isolated_launch"] = {"ms": launch_ms, "achieved": byt / (launch_ms / 1e3) / 1e9,
                                      "frac": byt / (launch_ms / 1e3) / 1e9 / P["hbm_gbs"]}
    else:
        fl = 2.0 * m * cfg.N * cfg.K
        ach = fl / (ms_step / 1e3) / 1e12
        div = 2.0 if cfg.dtype == torch.float32 else 1.0  # tf32 tensor rate = bf16 / 2
        peak, kind = pick_peak(P, clocks, div)
        rec.update({"value": ach, "unit": "TFLOP/s",
                    "roofline": {"bound": "tensor", "achieved": ach, "peak": peak, "peak_kind": kind,
                                 "frac": ach / peak, "unit": "TFLOP/s",
                                 "tflops_per_mhz": (ach / clocks["sm_mhz"]) if clocks else None}})
        if cfg.dtype == torch.float32:
            rec["roofline"]["note"] = ("peak = bf16 figure / 2 (tf32 rate); the tensor pipe does 3 MMAs per "
                                       "product, so frac <= 1/3 at best for 3xTF32")
        if launch_ms:
            rec["isolated_launch"] = {"ms": launch_ms, "achieved": fl / (launch_ms / 1e3) / 1e12,
                                      "peak": P["bf16_tflops"] / div,
                                      "frac": fl / (launch_ms / 1e3) / 1e12 / (P["bf16_tflops"] / div)}
    if extra:
        rec.update(extra)
    return rec


def sub_workload(cid, timer, P, args, device, world, rank, path=None, steps=None, sharded=False):
    """Measures one more config in the same run (resident inputs, same timing
    rules) and returns its record."""
    from cmp_ext_b200 import _cmpext3 as ext

    cfg = CONFIGS[cid]
    r0, r1 = shard_rows(cfg.M, world, rank) if sharded else (0, cfg.M)
    m = r1 - r0
    sets, l2 = input_sets(cfg, device, m, rank)
    op = op_for(cfg.dtype)
    prev = None
    if path is not None:
        ext._set_path(path)
    try:
        out = {"i": 0}

        def step():
            A, B = sets[out["i"] % len(sets)]
            out["i"] += 1
            out["C"], out["AB"] = op(A, B), (A, B)

        K = steps or max(3, min(args.steps, 20))
        ms, clocks = timer.run(step, K, 3)
        launch_ms = timer.isolated(step, 5 if K >= 5 else 2)
        err = rows_err(out["C"], *out["AB"])
        kern = kernel_name(cfg, m) if path is None else {"simt": "gemm_simt_kernel", "tc": kernel_name(cfg, m),
                                                         "bf16x3": "gemm_tc_kernel(bf16x3)"}[path]
        rec = tensor_record(cfg, m, ms / K, clocks, P, kern, launch_ms,
                            {"err_vs_fp64_rows": err, "steps": K, "l2": l2})
        if sharded:
            job = 2.0 * cfg.M * cfg.N * cfg.K
            rec["job_value"] = job / (ms / K / 1e3) / 1e12
            rec["parallelism"] = f"M-shard x{world}, no gather"
        if path == "simt":
            # CUDA-core fp32: 2 FLOP per FMA, 128 FMA lanes per SM per clock
            sm = clocks["sm_mhz"] if clocks else 1965.0
            pk = 2.0 * 128 * torch.cuda.get_device_properties(device).multi_processor_count * sm * 1e6 / 1e12
            rec["roofline"] = {"bound": "fp32 CUDA cores", "achieved": rec["value"], "peak": pk,
                               "peak_kind": f"nominal FFMA rate at the observed {sm:.0f} MHz",
                               "frac": rec["value"] / pk, "unit": "TFLOP/s"}
        return rec
    finally:
        if path is not None:
            ext._set_path(prev or "auto")
        sets.clear()
        out.clear()
        torch.cuda.empty_cache()


def attention_record(timer, P, args, device, dtype=torch.float16):
    """cmpext3.attention on the reference's own benchmark shape
    (tools/bench.py:276-287: B=8, H=8, L=1024, D=128, scale 1/sqrt(D)),
    4 rotating input sets (402 MB > 3 x L2): FLOPs 4*B*H*L^2*D (QK^T and PV)."""
    import cmp_ext_b200 as cx

    B, H, L, D = 8, 8, 1024, 128
    g = torch.Generator(device=device).manual_seed(0)
    sets = [tuple(torch.randn(B, H, L, D, generator=g, device=device).to(dtype) for _ in range(3)) for _ in range(4)]
    st = {"i": 0}
    scale = 1.0 / D ** 0.5

    def step():
        q, k, v = sets[st["i"] % len(sets)]
        st["i"] += 1
        st["out"], st["qkv"] = cx.attention(q, k, v, scale=scale), (q, k, v)

    K = max(3, min(args.steps, 20))
    ms, clocks = timer.run(step, K, 3)
    launch_ms = timer.isolated(step, 5)
    q, k, v = st["qkv"]
    # fp64 check of 64 query rows of one (batch, head)
    idx = torch.linspace(0, L - 1, 64, device=device).long()
    s64 = (q[1, 3, idx].double() @ k[1, 3].double().t()) * scale
    want = torch.softmax(s64, dim=-1) @ v[1, 3].double()
    err = float((st["out"][1, 3, idx].double() - want).abs().max() / want.abs().max())
    fl = 4.0 * B * H * L * L * D
    ach = fl / (ms / K / 1e3) / 1e12
    peak, kind = pick_peak(P, clocks)
    rec = {"workload": f"attention {B}x{H}x{L}x{D} {KIND_NAMES[dtype]} (reference tools/bench.py shape)",
           "kernel": ("attention_tc_kernel" if os.environ.get("CMPX_ATTN_KERNEL", "").startswith("o")
                      else "attention_pp_kernel"), "value": ach, "unit": "TFLOP/s", "ms_per_step": ms / K, "steps": K,
           "clocks": clocks, "err_vs_fp64_rows": err, "l2": "4 resident input sets rotated per step",
           "roofline": {"bound": "tensor", "achieved": ach, "peak": peak, "peak_kind": kind, "frac": ach / peak,
                        "unit": "TFLOP/s", "flops_per_step": fl},
           "isolated_launch": {"ms": launch_ms, "achieved": fl / (launch_ms / 1e3) / 1e12,
                               "frac": fl / (launch_ms / 1e3) / 1e12 / P["bf16_tflops"]}}
    sets.clear()
    st.clear()
    torch.cuda.empty_cache()
    return rec


KIND_NAMES = {torch.float16: "fp16", torch.bfloat16: "bf16", torch.float32: "fp32"}


def library_context(timer, P, args, device):
    """Context only, not this library: the same config-3 GEMM through
    torch.matmul (cuBLAS) and the attention shape through torch's
    scaled_dot_product_attention, timed with the same rules, so the kernels
    here can be read against the vendor libraries on the same GPU and in the
    same power state."""
    import torch.nn.functional as F

    out = {}
    cfg = CONFIGS[3]
    A, B = make_inputs(cfg, device, seed=0, a_seed=1000)
    K = max(3, min(args.steps, 20))
    ms, clocks = timer.run(lambda: torch.matmul(A, B), K, 3)
    v = cfg.flops / (ms / K / 1e3) / 1e12
    out["config3_torch_matmul"] = {"value": v, "unit": "TFLOP/s", "ms_per_step": ms / K, "clocks": clocks,
                                   "tflops_per_mhz": v / clocks["sm_mhz"] if clocks else None}
    del A, B
    Bh, H, L, D = 8, 8, 1024, 128
    g = torch.Generator(device=device).manual_seed(0)
    sets = [tuple(torch.randn(Bh, H, L, D, generator=g, device=device).half() for _ in range(3)) for _ in range(4)]
    st = {"i": 0}

    def sdpa():
        q, k, v_ = sets[st["i"] % 4]
        st["i"] += 1
        F.scaled_dot_product_attention(q, k, v_, scale=1.0 / D ** 0.5)

    ms, clocks = timer.run(sdpa, K, 3)
    v = 4.0 * Bh * H * L * L * D / (ms / K / 1e3) / 1e12
    out["attention_fp16_torch_sdpa"] = {"value": v, "unit": "TFLOP/s", "ms_per_step": ms / K, "clocks": clocks}
    sets.clear()
    torch.cuda.empty_cache()
    return out


def gathered_record(cfg, transport, timer, P, args, device, world, rank, chunks=1):
    """Config 3 M-sharded with the all-gather of C (every rank ends with the
    whole C), and a check of the gathered C: sampled rows of every rank's
    block against the fp64 product of that rank's A rows, which this rank
    regenerates from the rank's seed."""
    from cmp_ext_b200.distributed import gather_output, sharded_matmul

    S = cfg.M // world
    A, B = make_inputs(cfg, device, seed=0, m=S, a_seed=1000 + rank)
    if transport in ("nvlink", "ce", "nvls"):
        Cfull = gather_output(cfg.M, cfg.N, cfg.dtype, device)
    else:
        Cfull = torch.empty((cfg.M, cfg.N), dtype=cfg.dtype, device=device)

    def step():
        sharded_matmul(A, B, M=cfg.M, gather=True, out=Cfull, transport=transport, chunks=chunks)

    K = max(3, min(args.steps, 20))
    ms, clocks = timer.run(step, K, 3)
    torch.cuda.synchronize()
    errs = []
    for q in range(world):
        Aq, _ = make_inputs(cfg, device, seed=0, m=S, a_seed=1000 + q)
        idx = torch.linspace(0, S - 1, 8, device=device).long()
        ref = Aq[idx].double() @ B.double()
        got = Cfull[q * S + idx].double()
        errs.append(float((got - ref).abs().max() / ref.abs().max()))
        del Aq
    ok = max(errs) <= 1e-2  # the build's bf16 error is ~3e-3; a missing or stale block gives ~1
    okt = torch.tensor([1.0 if ok else 0.0], device=device)
    if world > 1:
        dist.all_reduce(okt, op=dist.ReduceOp.MIN)
    how = f"{transport} all-gather" if chunks == 1 else f"{transport} point-to-point in {chunks} row chunks"
    rec = tensor_record(cfg, S, ms / K, clocks, P, kernel_name(cfg, S) + f" + {how}")
    job = 2.0 * cfg.M * cfg.N * cfg.K / (ms / K / 1e3) / 1e12
    rec.update({"job_value": job, "unit": "TFLOP/s", "transport": transport, "chunks": chunks,
                "check": {"all_ranks_ok": bool(okt.item() == 1.0), "max_err_vs_fp64_rows": max(errs),
                          "what": "8 rows of every rank's block of the gathered C on this rank vs fp64"},
                "bytes_in_per_rank": (world - 1) * S * cfg.N * torch.empty((), dtype=cfg.dtype).element_size()})
    del A, B, Cfull
    torch.cuda.empty_cache()
    return rec


def run_ours(args):
    sys.setswitchinterval(0.0005)  # let the clock-sampling thread run while this one launches
    world, rank, local = dist_setup(args)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.attention is not None:
        # profiling / spot runs of the attention workload alone (one GPU)
        dt = {"fp16": torch.float16, "bf16": torch.bfloat16}[args.attention]
        rec = attention_record(Timer(1, device, args.quick, args.hold), peaks()[0], args, device, dt)
        print(json.dumps(rec), flush=True)
        return 0
    cfg = CONFIGS[args.config]
    metric, unit = metric_of(cfg)
    r0, r1 = shard_rows(cfg.M, world, rank)
    m = r1 - r0 if args.rows is None else args.rows
    if args.quick:
        args.no_e2e = args.no_cpu = True
        args.sub = "none"
    op = op_for(cfg.dtype)
    if cfg.dtype == torch.float32 and args.f32_path == "bf16x3":
        from cmp_ext_b200 import _cmpext3 as ext

        ext._set_path("bf16x3")  # every fp32 call of this process, e2e included
    P, peak_src = peaks()
    timer = Timer(world, device, args.quick, args.hold)

    # Inputs resident in HBM (drawn on the device; the same B on every rank,
    # a different A shard per rank; small configs rotate several sets so the
    # operands of a step are never in L2).
    sets, l2_desc = input_sets(cfg, device, m, rank)
    A, B = sets[0]

    gather = args.gather and world > 1
    if gather:
        from cmp_ext_b200.distributed import gather_output, sharded_matmul
        if args.transport in ("nvlink", "ce", "nvls"):
            Cfull = gather_output(cfg.M, cfg.N, cfg.dtype, device)
        else:
            Cfull = torch.empty((cfg.M, cfg.N), dtype=cfg.dtype, device=device)

    last = {"i": 0}

    def step():
        if gather:
            sharded_matmul(A, B, M=cfg.M, gather=True, chunks=args.chunks, out=Cfull, transport=args.transport)
        else:
            a, b = sets[last["i"] % len(sets)]
            last["i"] += 1
            last["C"], last["AB"] = op(a, b), (a, b)

    ms_gemm, clocks = timer.run(step, args.steps, args.warmup if args.quick else max(3, args.warmup))
    launch_ms = timer.isolated(step if not gather else (lambda: op(A, B)),
                               1 if args.quick else max(5, min(args.steps, 20)))
    err = None if gather or args.quick else rows_err(last["C"], *last["AB"])

    M_job = cfg.M if args.rows is None else args.rows * world
    step_flops = 2.0 * M_job * cfg.N * cfg.K  # whole job (all ranks)
    e = torch.empty((), dtype=cfg.dtype).element_size()
    step_bytes_job = (M_job * cfg.K + world * cfg.K * cfg.N + M_job * cfg.N) * e
    if unit == "GB/s":
        value = step_bytes_job * args.steps / (ms_gemm / 1e3) / 1e9
    else:
        value = step_flops * args.steps / (ms_gemm / 1e3) / 1e12
    ms_per_step = ms_gemm / args.steps

    # Average launch duration of the dominant kernel over the timed region:
    # when a step is that one launch, it is the timed region divided by K;
    # otherwise the isolated launch.
    one_launch = launches_per_step(cfg, args.rows) == 1 and not gather
    avg_launch_ms = ms_per_step if one_launch else launch_ms
    timing = ("timed region / K (back-to-back launches)" if one_launch
              else "median of isolated launches (events around each)")
    scale = 1e9 if cfg.bound == "hbm" else 1e12
    if cfg.bound == "hbm":
        per_launch = cfg.bytes(m)
        peak = peak_isolated = P["hbm_gbs"]
        peak_kind = "measured copy"
        runit, rbound = "GB/s", "hbm"
    else:
        per_launch = 2.0 * m * cfg.N * cfg.K
        div = 2.0 if cfg.dtype == torch.float32 else 1.0  # tf32 rate = bf16 / 2
        peak, peak_kind = pick_peak(P, clocks if one_launch else None, div)
        if not one_launch:
            peak, peak_kind = P["bf16_tflops"] / div, "burst (isolated launch)"
        peak_isolated = P["bf16_tflops"] / div
        runit, rbound = "TFLOP/s", "tensor"
    achieved = per_launch / (avg_launch_ms / 1e3) / scale
    achieved_isolated = per_launch / (launch_ms / 1e3) / scale
    traffic = traffic_per_launch(f"config{cfg.cid}_m{m}")

    # Other configs, measured in this same run (N=1: configs 2, 4, 5 on both
    # fp32 paths, 6, 7; N>1: config 3 with the all-gather over both
    # transports, and config 5 M-sharded).
    sub = {}
    if args.sub != "none" and args.rows is None:
        if world == 1:
            for cid in (2, 4, 6, 7):
                sub[f"config{cid}"] = sub_workload(cid, timer, P, args, device, world, rank)
            sub["config5_tf32x3"] = sub_workload(5, timer, P, args, device, world, rank, path="tc")
            sub["config5_simt"] = sub_workload(5, timer, P, args, device, world, rank, path="simt", steps=3)
            for dt in (torch.float16, torch.bfloat16):
                try:
                    sub[f"attention_{KIND_NAMES[dt]}"] = attention_record(timer, P, args, device, dt)
                except Exception as ex:  # reported, never hidden
                    sub[f"attention_{KIND_NAMES[dt]}"] = {"error": repr(ex)[:300]}
            try:
                sub["context_vendor_libraries"] = library_context(timer, P, args, device)
            except Exception as ex:  # context only
                sub["context_vendor_libraries"] = {"error": repr(ex)[:300]}
        else:
            c3 = CONFIGS[3]
            if c3.M % world == 0:
                for tr, ch in (("nccl", 1), ("nccl", 4), ("nvlink", 1), ("ce", 1), ("nvls", 1)):
                    key = f"gathered_{tr}" + (f"_chunks{ch}" if ch > 1 else "")
                    try:
                        sub[key] = gathered_record(c3, tr, timer, P, args, device, world, rank, chunks=ch)
                    except Exception as ex:  # reported, never hidden
                        sub[key] = {"error": repr(ex)[:300]}
            sub["config5_sharded_tf32x3"] = sub_workload(5, timer, P, args, device, world, rank, path="tc",
                                                         sharded=True)

    # End-to-end through the public API with pinned host buffers: host_matmul
    # at N=1; at N>1 sharded_host_matmul (B uploaded once per job in 1/N
    # slices and all-gathered over NVLink, each rank's A rows in, its C rows out).
    e2e = None
    if not args.no_e2e:
        hA = A.cpu().pin_memory()
        hB = B.cpu().pin_memory()
        hC = torch.empty((m, cfg.N), dtype=cfg.dtype).pin_memory()
        e_steps = max(3, min(args.steps, 10))
        if world == 1:
            from cmp_ext_b200.host import host_matmul

            def e2e_step():
                host_matmul(hA, hB, out=hC, chunks=8, device=device)
            api = "cmp_ext_b200.host.host_matmul (pinned host in/out, 8 row chunks)"
            h2d = (hA.numel() + hB.numel()) * e
        else:
            from cmp_ext_b200.distributed import sharded_host_matmul

            def e2e_step():
                sharded_host_matmul(hA, hB, out=hC, chunks=8, device=device)
            api = ("cmp_ext_b200.distributed.sharded_host_matmul (pinned host in/out; each rank uploads its A rows "
                   "and 1/N of B, B all-gathered over NVLink)")
            h2d = (hA.numel() + (hB.numel() // world if cfg.K % world == 0 else hB.numel())) * e
        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        stream = torch.cuda.current_stream()
        x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        x0.record(stream)
        for _ in range(e_steps):
            e2e_step()
        x1.record(stream)
        torch.cuda.synchronize()
        e_ms = max_over_ranks(x0.elapsed_time(x1), world, device) / e_steps
        d2h = hC.numel() * e
        ev = (step_bytes_job / (e_ms / 1e3) / 1e9) if unit == "GB/s" else (step_flops / (e_ms / 1e3) / 1e12)
        e2e = {"value": ev, "unit": unit, "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
               "ms_per_step": e_ms, "api": api}

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
        n_launch = args.steps * launches_per_step(cfg, args.rows)
        line = {"metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": cfg.dtype_name, "data": "synthetic (seeded, drawn on device)",
                "config": {**config_block(cfg, world, gather, args.transport), "l2": l2_desc,
                           "power_state": f"{args.hold:.0f} s of back-to-back steps before every timed region",
                           **({"f32_path": args.f32_path} if cfg.dtype == torch.float32 else {})},
                "roofline": {"bound": rbound, "kernel": kernel_name(cfg, m), "achieved": achieved, "peak": peak,
                             "peak_source": peak_src, "unit": runit, "frac": achieved / peak,
                             "traffic": traffic, "launch_ms": avg_launch_ms, "timing": timing,
                             "peak_kind": peak_kind,
                             "tflops_per_mhz": (achieved / clocks["sm_mhz"]) if (clocks and runit == "TFLOP/s")
                             else None,
                             "isolated_launch": {"ms": launch_ms, "achieved": achieved_isolated,
                                                 "peak": peak_isolated, "frac": achieved_isolated / peak_isolated},
                             "per_launch": per_launch},
                "err_vs_fp64_rows": err,
                "e2e": e2e, "gpu_launches": n_launch,
                "clocks": clocks, "cpu_baseline": cpu,
                "sub": sub or None}
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
    ap.add_argument("--transport", default="nccl", choices=["nccl", "nvlink", "ce", "nvls"],
                    help="gather: NCCL all-gather, epilogue stores into peers' outputs over NVLink, or copy-engine "
                         "copies of finished tile columns")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--quick", action="store_true",
                    help="profiling mode: only W warm-up + K timed steps (no clock sampling, e2e or CPU legs)")
    ap.add_argument("--attention", default=None, choices=["fp16", "bf16"],
                    help="measure only cmpext3.attention on the reference's benchmark shape (8x8x1024x128)")
    ap.add_argument("--rows", type=int, default=None, help="override this rank's M rows (profiling small cases)")
    ap.add_argument("--f32-path", default="tf32x3", choices=["tf32x3", "bf16x3"],
                    help="fp32 configs: 3xTF32 (default) or the opt-in bf16x3 split")
    ap.add_argument("--hold", type=float, default=3.0,
                    help="seconds of back-to-back steps before each timed region (same power state at every N)")
    ap.add_argument("--sub", default="all", choices=["all", "none"],
                    help="also measure the other configs in this run (N=1) / the gathered and fp32 lines (N>1)")
    args = ap.parse_args(argv)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
