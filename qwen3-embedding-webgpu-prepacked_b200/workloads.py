"""Seeded synthetic workloads for the attention hot path.

The reference benchmarks on text fixtures whose only carried-over property is
the token count (scripts/workloads.ts: 15, 50, 150, 500, 1500, 5000). Here
every layer's ``qkvRaw`` activation is f16 ~N(0,1) from a seed, and the
per-layer q_norm / k_norm weights are 1 + N(0, 0.02), as the benchmark
configurations specify. No checkpoint or dataset is involved.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

import numpy as np

QKV_WIDTH = 4096  # q 2048 | k 1024 | v 1024 (src/webgpu/model.ts:69)
LAYERS = 28  # src/webgpu/model.ts:21


@dataclass(frozen=True)
class Workload:
    name: str
    lengths: tuple
    layers: int
    mode: int  # 0 AUTO (reference rule), 1 FULL, 2 SPARSE

    @property
    def tokens(self) -> int:
        return int(sum(self.lengths))

    def cu_seqlens(self) -> List[int]:
        return [0] + list(np.cumsum(self.lengths).astype(int).tolist())


def ragged_lengths(n: int, lo: int, hi: int, seed: int) -> tuple:
    rng = np.random.default_rng(seed)
    return tuple(int(x) for x in rng.integers(lo, hi + 1, size=n))


# The five benchmark configurations (BASELINE configs[0..4]).
WORKLOADS = {
    "c1_single_50": Workload("c1_single_50", (50,), 1, 0),
    "c2_ragged16": Workload("c2_ragged16", ragged_lengths(16, 15, 150, 2024), LAYERS, 0),
    "c3_16x500": Workload("c3_16x500", (500,) * 16, LAYERS, 0),
    "c4_4x1500_sparse": Workload("c4_4x1500_sparse", (1500,) * 4, LAYERS, 0),
    "c5_16x5000_sparse": Workload("c5_16x5000_sparse", (5000,) * 16, LAYERS, 0),
    "c5_16x5000_full": Workload("c5_16x5000_full", (5000,) * 16, LAYERS, 1),
}


def host_layer_inputs(tokens: int, seed: int):
    """qkv f16 [tokens, 4096] ~N(0,1), q/k norm weights f32 [128] ~1+N(0,0.02)."""
    rng = np.random.default_rng(seed)
    qkv = rng.standard_normal((tokens, QKV_WIDTH), dtype=np.float32).astype(np.float16)
    qw = (1.0 + 0.02 * rng.standard_normal(128)).astype(np.float32)
    kw = (1.0 + 0.02 * rng.standard_normal(128)).astype(np.float32)
    return qkv, qw, kw


def device_layer_inputs(tokens: int, seed: int, device):
    """Same distributions generated directly on the device (bench inputs)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    qkv = torch.randn(tokens, QKV_WIDTH, generator=g, device=device, dtype=torch.float32).half()
    w = 1.0 + 0.02 * torch.randn(2, 128, generator=g, device=device, dtype=torch.float32)
    return qkv, w[0].contiguous(), w[1].contiguous()
