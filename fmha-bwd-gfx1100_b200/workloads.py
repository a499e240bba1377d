"""Workload definitions of the attention-backward path and a seeded,
on-device input generator.

Each workload is (M query rows, N key rows, d head dim, total heads, dtype,
dO standard deviation). Inputs: Q, K, V, dO ~ N(0, 1) (dO ~ N(0, std)), and
P = row-softmax(Q K^T / sqrt(d)) computed in fp32 from the 16-bit Q and K and
then stored in the 16-bit type. Batch is folded into heads. All data is
synthetic; no dataset is involved.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Workload:
    name: str
    M: int
    N: int
    d: int
    heads: int
    dtype: str  # "bf16" | "fp16"
    do_std: float = 1.0
    description: str = ""

    @property
    def torch_dtype(self) -> torch.dtype:
        return torch.bfloat16 if self.dtype == "bf16" else torch.float16

    def flops(self, heads: int | None = None) -> float:
        """Counted FLOPs: 4 matmuls of 2*M*N*d per head (8*M*N*d*H)."""
        return 8.0 * self.M * self.N * self.d * (self.heads if heads is None else heads)

    def algorithmic_bytes(self, heads: int | None = None) -> float:
        """P, Q, K, V, dO read once and dQ, dK, dV written once (16-bit)."""
        h = self.heads if heads is None else heads
        return 2.0 * h * (self.M * self.N + 3 * self.M * self.d + 4 * self.N * self.d)


WORKLOADS = {
    "cpu_case": Workload("cpu_case", 128, 128, 64, 2, "bf16",
                         description="CPU-runnable correctness case M=N=128 d=64 H=2 bf16"),
    "flux": Workload("flux", 4608, 4608, 128, 24, "bf16",
                     description="FLUX-like joint self-attention M=N=4608 d=128 H=24 bf16"),
    "cross": Workload("cross", 4096, 512, 128, 48, "bf16", do_std=0.1,
                      description="cross-attention M=4096 N=512 d=128 H=48 (2x24) bf16, dO~N(0,0.1)"),
    "fp16": Workload("fp16", 2048, 2048, 64, 128, "fp16",
                     description="fp16 path M=N=2048 d=64 H=128 (4x32) fp16"),
    "video": Workload("video", 16384, 16384, 128, 40, "bf16",
                      description="long video self-attention M=N=16384 d=128 H=40 bf16"),
}


def make_inputs(w: Workload, seed: int = 42, device: str | torch.device = "cuda",
                heads: int | None = None, head_offset: int = 0):
    """Seeded inputs for heads [head_offset, head_offset + heads) of ``w`` on
    ``device``: returns (Q, K, V, P, dO) as contiguous [h, rows, cols] tensors.

    Each head is drawn from its own generator seeded with (seed, head index),
    so any head range can be rebuilt independently (used for head-sharded
    multi-GPU runs and for sampled-head oracle checks)."""
    h = w.heads if heads is None else heads
    dt = w.torch_dtype
    dev = torch.device(device)
    Q = torch.empty(h, w.M, w.d, dtype=dt, device=dev)
    K = torch.empty(h, w.N, w.d, dtype=dt, device=dev)
    V = torch.empty(h, w.N, w.d, dtype=dt, device=dev)
    dO = torch.empty(h, w.M, w.d, dtype=dt, device=dev)
    P = torch.empty(h, w.M, w.N, dtype=dt, device=dev)
    scale = 1.0 / math.sqrt(w.d)
    for i in range(h):
        g = torch.Generator(device=dev)
        g.manual_seed(seed * 1_000_003 + head_offset + i)
        Q[i] = torch.randn(w.M, w.d, generator=g, device=dev, dtype=torch.float32).to(dt)
        K[i] = torch.randn(w.N, w.d, generator=g, device=dev, dtype=torch.float32).to(dt)
        V[i] = torch.randn(w.N, w.d, generator=g, device=dev, dtype=torch.float32).to(dt)
        dO[i] = (torch.randn(w.M, w.d, generator=g, device=dev, dtype=torch.float32)
                 * w.do_std).to(dt)
        # softmax in fp32 over row chunks to bound the temporary size
        rows = max(1, (1 << 26) // max(w.N, 1))
        Kf = K[i].float()
        for r0 in range(0, w.M, rows):
            s = (Q[i, r0:r0 + rows].float() @ Kf.T) * scale
            P[i, r0:r0 + rows] = torch.softmax(s, dim=-1).to(dt)
    return Q, K, V, P, dO


def head_range(total_heads: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous head range [h0, h1) of ``rank`` when ``total_heads`` are
    split over ``world`` GPUs: ceil-sized blocks, the last one possibly
    shorter or empty."""
    per = -(-total_heads // world)
    h0 = min(total_heads, rank * per)
    h1 = min(total_heads, h0 + per)
    return h0, h1


def gather_rank_stats(dist, values, device) -> torch.Tensor:
    """All-gather one row of float64 statistics per rank (timings, checksums)
    after the timed region; returns a [world, len(values)] CPU tensor. Every
    rank must call it with the same number of values. With the NCCL backend
    ``device`` is the rank's GPU; with gloo it is the CPU."""
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    parts = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t)
    return torch.stack(parts).cpu()
