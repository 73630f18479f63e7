"""CPU port of the reference's decode forward, for the timed CPU baseline.

TEST / BASELINE INFRASTRUCTURE ONLY (imported by tests/ and by bench.py's
cpu_baseline and ``--impl reference`` legs). It restates CDQLinear.forward,
code/cdq_lrr_qwen05.py:188-198 (the loader's twin is code/cdq_loader.py:53-58),
with the same torch CPU operations the reference runs: gather the lattice
by index, multiply by the bf16 scale, overwrite the residual positions,
F.linear. Timing it on the host's cores is the CPU baseline.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import cdq_oracle as O


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


class OracleCDQLinear:
    """Reference-format buffers + the reference forward, on the CPU."""

    def __init__(self, pack: dict, bias_bits: np.ndarray | None = None):
        self.quant_indices = torch.from_numpy(np.ascontiguousarray(pack["quant_indices"]))
        self.scales_bf16 = _bf16(pack["scales_bf16"]).view(-1, 1)
        self.residual_indices = torch.from_numpy(np.asarray(pack["residual_indices"], np.int64))
        self.residual_values = _bf16(pack["residual_values"])
        self.lattice = _bf16(pack["lattice"])
        self.orig_shape = tuple(pack["orig_shape"])
        self.bias = _bf16(bias_bits) if bias_bits is not None else None

    def dequant_weight(self) -> torch.Tensor:
        w = self.lattice[self.quant_indices.long()].to(torch.bfloat16) * self.scales_bf16
        if int(self.residual_indices.numel()) > 0:
            w.view(-1)[self.residual_indices.long()] = self.residual_values
        return w.view(self.orig_shape)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        w = self.dequant_weight().to(x.dtype)
        return F.linear(x, w, self.bias.to(x.dtype) if self.bias is not None else None)

    __call__ = forward

    def reference_bytes(self) -> int:
        """Bytes of this weight's .cdq tile records (the algorithmic bytes)."""
        n_states = 26 if self.lattice.numel() == 26 else 16
        n_tiles = self.quant_indices.shape[0]
        tc = np.bincount(self.residual_indices.numpy() // 32, minlength=n_tiles)
        return int(n_tiles * (2 + (20 if n_states == 26 else 16)) + ((tc * 21 + 7) // 8).sum())


def quantize_to_oracle_linear(w_bits: np.ndarray, n_states: int = 26,
                              stc_frac: float = O.STC_FRAC) -> OracleCDQLinear:
    return OracleCDQLinear(O.quantize(w_bits, n_states=n_states, stc_frac=stc_frac))
