"""Seeded synthetic workloads for the CDQ-LRR decode path.

The reference publishes no weights that are usable offline, so every
measurement and parity case runs on seeded random weights with the shapes and
value distributions the workloads name:

* a projection weight drawn from N(0, std^2), with ``outlier_frac`` of its
  entries (positions from a seeded permutation) multiplied by a factor drawn
  uniformly from [lo, hi], then rounded to bf16;
* activations drawn from N(0, 1) in bf16.

The same generator runs on CPU (small parity cases, golden fixtures) and on a
CUDA device (full-size workloads, where CPU generation would take minutes).
Torch's CPU generator is deterministic across machines; the CUDA generator is
deterministic for a given device type and torch build.
"""
from __future__ import annotations

import torch

# Qwen2.5-0.5B projection shapes as nn.Linear weights [out_features, in_features].
QWEN05 = dict(hidden=896, inter=4864, layers=24, heads=14, kv_heads=2, head_dim=64,
              vocab=151936)
QWEN7B = dict(hidden=3584, inter=18944, layers=28, heads=28, kv_heads=4, head_dim=128,
              vocab=152064)
LLAMA70B_SHAPES = ((28672, 8192), (8192, 28672))

PROJ_NAMES = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


def layer_shapes(cfg: dict) -> list[tuple[str, int, int]]:
    """The seven projection weight shapes of one decoder layer, in module order."""
    h, i = cfg["hidden"], cfg["inter"]
    q = cfg["heads"] * cfg["head_dim"]
    kv = cfg["kv_heads"] * cfg["head_dim"]
    return [("q_proj", q, h), ("k_proj", kv, h), ("v_proj", kv, h), ("o_proj", h, q),
            ("gate_proj", i, h), ("up_proj", i, h), ("down_proj", h, i)]


def synth_weight(rows: int, cols: int, std: float = 0.02, seed: int = 0,
                 outlier_frac: float = 0.015, lo: float = 8.0, hi: float = 20.0,
                 device: str | torch.device = "cpu") -> torch.Tensor:
    """bf16 [rows, cols]: N(0, std^2) with a seeded fraction of heavy-tailed outliers."""
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    w = torch.randn(rows, cols, generator=g, device=dev, dtype=torch.float32) * std
    n = rows * cols
    k = int(round(n * outlier_frac))
    if k > 0:
        pos = torch.randperm(n, generator=g, device=dev)[:k]
        fac = torch.empty(k, device=dev, dtype=torch.float32).uniform_(lo, hi, generator=g)
        w.view(-1)[pos] *= fac
    return w.to(torch.bfloat16)


def synth_activation(m: int, k: int, seed: int = 1,
                     device: str | torch.device = "cpu") -> torch.Tensor:
    """bf16 [m, k] drawn from N(0, 1)."""
    dev = torch.device(device)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    return torch.randn(m, k, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
