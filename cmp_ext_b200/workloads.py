"""The five benchmark/parity configurations of the matmul path, with seeded
synthetic inputs (no dataset is involved: the reference benchmarks random
matrices, tools/bench.py:156-193).

Config ids follow the order of the benchmark configs of the matmul path:
  1  fp32 257 x 383 x 511,  A,B ~ N(0,1)                     (odd shape)
  2  fp16 4096^3,           A,B ~ U(-1,1)                     (tensor-bound)
  3  bf16 M=16384 K=8192 N=8192, A ~ N(0,1), B ~ N(0,0.02)    (prefill, M-sharded)
  4  fp16 M=16 K=8192 N=28672,   A ~ N(0,1), B ~ N(0,0.02)    (decode, HBM-bound)
  5  fp32 8192^3,           A,B ~ N(0,1)                      (3xTF32)

Two extra workloads carry the path's stated 1-GPU tensor target (fp16/bf16
8192^3, >= 70% of dense peak); they are bench lines, not parity configs:
  6  fp16 8192^3,           A,B ~ U(-1,1)
  7  bf16 8192^3,           A ~ N(0,1), B ~ N(0,0.02)
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Config:
    cid: int
    name: str
    dtype: torch.dtype
    M: int
    N: int
    K: int
    a_dist: str  # "normal" | "uniform"
    b_std: float
    bound: str   # "tensor" | "hbm" | "correctness"

    @property
    def flops(self) -> float:
        return 2.0 * self.M * self.N * self.K

    def bytes(self, m: int | None = None) -> int:
        m = self.M if m is None else m
        e = torch.empty((), dtype=self.dtype).element_size()
        return (m * self.K + self.K * self.N + m * self.N) * e

    @property
    def dtype_name(self) -> str:
        return {torch.float16: "f16", torch.bfloat16: "bf16", torch.float32: "f32"}[self.dtype]


CONFIGS = {
    1: Config(1, "fp32_matmul odd 257x383x511", torch.float32, 257, 383, 511, "normal", 1.0, "correctness"),
    2: Config(2, "fp16_matmul 4096^3", torch.float16, 4096, 4096, 4096, "uniform", 1.0, "tensor"),
    3: Config(3, "bf16_matmul prefill 16384x8192x8192", torch.bfloat16, 16384, 8192, 8192, "normal", 0.02, "tensor"),
    4: Config(4, "fp16_matmul decode 16x28672x8192", torch.float16, 16, 28672, 8192, "normal", 0.02, "hbm"),
    5: Config(5, "fp32_matmul 8192^3", torch.float32, 8192, 8192, 8192, "normal", 1.0, "tensor"),
    6: Config(6, "fp16_matmul 8192^3", torch.float16, 8192, 8192, 8192, "uniform", 1.0, "tensor"),
    7: Config(7, "bf16_matmul 8192^3", torch.bfloat16, 8192, 8192, 8192, "normal", 0.02, "tensor"),
}


def _draw(shape, dist: str, std: float, gen: torch.Generator, device) -> torch.Tensor:
    if dist == "uniform":
        return torch.rand(shape, generator=gen, device=device, dtype=torch.float32).mul_(2.0).sub_(1.0)
    return torch.randn(shape, generator=gen, device=device, dtype=torch.float32).mul_(std)


def make_inputs(cfg: Config, device="cpu", seed: int = 0, rows: tuple[int, int] | None = None,
                m: int | None = None, a_seed: int | None = None):
    """Seeded A [M,K] and B [K,N] of cfg.dtype on `device`.

    The draw happens on `device` with a generator seeded by `seed` (so a CPU
    draw and a CUDA draw differ, but each is reproducible).  `rows` returns
    only A[r0:r1] (the rows an M-shard owns) with the same values the full
    draw would have; `m` overrides cfg.M.  With `a_seed`, B is drawn from
    `seed` alone and A from its own generator seeded `a_seed` (M-sharded
    runs: the same B on every rank, a different A shard per rank).
    """
    M = cfg.M if m is None else m
    gen = torch.Generator(device=device).manual_seed(seed)
    b_dist = cfg.a_dist if cfg.a_dist == "uniform" else "normal"
    if a_seed is not None:
        B = _draw((cfg.K, cfg.N), b_dist, cfg.b_std, gen, device)
        A = _draw((M, cfg.K), cfg.a_dist, 1.0, torch.Generator(device=device).manual_seed(a_seed), device)
        return A.to(cfg.dtype), B.to(cfg.dtype)
    A = _draw((M, cfg.K), cfg.a_dist, 1.0, gen, device)
    B = _draw((cfg.K, cfg.N), b_dist, cfg.b_std, gen, device)
    if rows is not None:
        A = A[rows[0]:rows[1]].contiguous()
    return A.to(cfg.dtype), B.to(cfg.dtype)
