"""Seeded synthetic workloads with the shapes of the benchmark configurations.

No public dataset is used: lengths come from ``torch.Generator().manual_seed(0)`` and
q/k/v ~ N(0, 1) bf16 from a second seed, as the benchmark plan prescribes. Totals for seed 0:
config 1 T=9,371; config 2 T=147,509; config 3 T=450,079; config 4 T=250,189; config 5
T=543,071.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

GLOBAL = ((-1, -1), False)
LOCAL64 = ((64, 64), False)
CAUSAL = ((-1, -1), True)


@dataclass(frozen=True)
class Workload:
    name: str
    lengths: tuple[int, ...]
    heads: int
    kv_heads: int
    head_dim: int
    scale: float
    layers: tuple[tuple[tuple[int, int], bool], ...]  # ((window_left, window_right), causal) per layer
    note: str = ""
    extra: dict = field(default_factory=dict)

    @property
    def tokens(self) -> int:
        return sum(self.lengths)

    def cu_seqlens(self) -> torch.Tensor:
        cu = torch.zeros(len(self.lengths) + 1, dtype=torch.int32)
        cu[1:] = torch.tensor(self.lengths, dtype=torch.int64).cumsum(0).to(torch.int32)
        return cu


def config1(layer: str = "both") -> Workload:
    g = torch.Generator().manual_seed(0)
    lengths = tuple(int(x) for x in torch.randint(8, 513, (32,), generator=g))
    layers = {"global": (GLOBAL,), "local": (LOCAL64,), "both": (GLOBAL, LOCAL64)}[layer]
    return Workload(f"config1-modernbert-base-op-{layer}", lengths, 12, 12, 64, 0.125, layers,
                    "32 x U[8,512], 12x64, scale 1/8")


def config2() -> Workload:
    g = torch.Generator().manual_seed(0)
    lengths = tuple(int(x) for x in torch.randint(8, 65, (4096,), generator=g))
    return Workload("config2-query-batch", lengths, 12, 12, 64, 0.125, (GLOBAL,), "4096 x U[8,64], 12x64, global")


def config3_lengths(n: int = 512, seed: int = 0) -> tuple[int, ...]:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, generator=g) * 0.8 + math.log(600.0)
    return tuple(int(v) for v in x.exp().round().clamp(64, 8192).long())


def config3(pattern: str = "mix", n: int = 512, seed: int = 0) -> Workload:
    lengths = config3_lengths(n, seed)
    layers = {"global": (GLOBAL,), "local": (LOCAL64,),
              "mix": tuple(GLOBAL if i % 3 == 0 else LOCAL64 for i in range(28))}[pattern]
    return Workload(f"config3-document-batch-{pattern}", lengths, 16, 16, 64, 0.125, layers,
                    "512 x lognormal(median 600, sigma 0.8) clipped [64,8192], 16x64; 28 layers, global every 3rd")


def config5(n: int = 256, seed: int = 0) -> Workload:
    g = torch.Generator().manual_seed(seed)
    lengths = tuple(int(x) for x in torch.randint(128, 4097, (n,), generator=g))
    return Workload("config5-qwen35-gqa-causal", lengths, 8, 2, 256, 1.0 / 16, (CAUSAL,),
                    "256 x U[128,4096], GQA 8/2, head_dim 256, causal, scale 1/16")


def make_qkv(lengths, heads: int, kv_heads: int, dim: int, *, seed: int = 1, device="cuda"):
    """q [T,H,D], k/v [T,KV,D] bf16 ~ N(0,1), generated on ``device`` from a seeded generator."""
    total = int(sum(lengths))
    gen = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(total, heads, dim, device=device, generator=gen, dtype=torch.float32).to(torch.bfloat16)
    k = torch.randn(total, kv_heads, dim, device=device, generator=gen, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn(total, kv_heads, dim, device=device, generator=gen, dtype=torch.float32).to(torch.bfloat16)
    return q, k, v


def useful_flops(lengths, heads: int, dim: int, window=(-1, -1), causal: bool = False) -> int:
    """4 * pairs * H * D (QK^T and PV, 2 flops per MAC); masked / skipped work is not counted."""
    from packed_encoders_b200.shard import band_pairs

    pairs = sum(band_pairs(n, tuple(window), causal) for n in lengths)
    return 4 * pairs * heads * dim


def algorithmic_bytes(total_q: int, total_k: int, heads: int, kv_heads: int, dim: int, lse: bool = False) -> int:
    """Read q, k, v once and write out once (bf16); plus the fp32 LSE when written."""
    return 2 * dim * (2 * heads * total_q + 2 * kv_heads * total_k) + (4 * heads * total_q if lse else 0)
