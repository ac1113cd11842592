"""Shared fixtures: golden vectors, seeded packed inputs, and the ``gpu`` marker."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) and the built extension")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this process")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden_names() -> list[str]:
    """Plain attention fixtures (the ``rope_*`` ones take un-rotated q/k plus tables)."""
    return sorted(p.stem for p in GOLDEN.glob("*.npz") if not p.stem.startswith("rope_"))


def rope_golden_names() -> list[str]:
    return sorted(p.stem for p in GOLDEN.glob("rope_*.npz"))


def load_rope_golden(name: str) -> dict:
    """A ``rope_*`` fixture: un-rotated q/k/v, bf16 per-token tables, the reference's rotated q/k
    (fp32) and its attention output over them."""
    g = load_golden(name)
    data = np.load(GOLDEN / f"{name}.npz")
    for key in ("cos", "sin"):
        g[key] = torch.from_numpy(data[key].view(np.int16).copy()).view(torch.bfloat16)
    g["rq"] = torch.from_numpy(data["rq"].copy())
    g["rk"] = torch.from_numpy(data["rk"].copy())
    return g


def load_golden(name: str) -> dict:
    data = np.load(GOLDEN / f"{name}.npz")

    def bf16(key):
        return torch.from_numpy(data[key].view(np.int16).copy()).view(torch.bfloat16)

    return {
        "q": bf16("q"), "k": bf16("k"), "v": bf16("v"),
        "cu_q": torch.from_numpy(data["cu_q"].copy()), "cu_k": torch.from_numpy(data["cu_k"].copy()),
        "out": torch.from_numpy(data["out"].copy()), "scale": float(data["scale"]),
        "window": tuple(int(w) for w in data["window"]), "causal": bool(int(data["causal"])),
        "note": str(data["note"]),
    }


def packed_inputs(lengths, heads, dim, *, kv_heads=None, seed=0, device="cpu", logit_scale=1.0):
    """Seeded bf16 q [T,H,D], k/v [T,KV,D] ~ N(0,1) and int32 cu_seqlens."""
    kv_heads = heads if kv_heads is None else kv_heads
    gen = torch.Generator().manual_seed(seed)
    total = int(sum(lengths))
    q = (torch.randn(total, heads, dim, generator=gen) * logit_scale).to(torch.bfloat16)
    k = (torch.randn(total, kv_heads, dim, generator=gen) * logit_scale).to(torch.bfloat16)
    v = torch.randn(total, kv_heads, dim, generator=gen).to(torch.bfloat16)
    cu = torch.zeros(len(lengths) + 1, dtype=torch.int32)
    if len(lengths):
        cu[1:] = torch.tensor(list(lengths), dtype=torch.int64).cumsum(0).to(torch.int32)
    return q.to(device), k.to(device), v.to(device), cu.to(device)


def rope_tables(lengths, theta=10000.0, dim=64, device="cpu"):
    """Per-token gathered RoPE tables [T, dim] bf16 (positions restart in every sequence), the
    rotary embedding of ModernBERT (inverse frequencies theta^(-2i/dim), emb = [freqs, freqs])."""
    inv = 1.0 / theta ** (torch.arange(0, dim, 2, dtype=torch.float32) / dim)
    pos = torch.cat([torch.arange(int(n), dtype=torch.float32) for n in lengths])
    freqs = pos[:, None] * inv[None, :]
    emb = torch.cat((freqs, freqs), -1)
    return emb.cos().to(torch.bfloat16).to(device), emb.sin().to(torch.bfloat16).to(device)

