"""Quality report of a quantized model on the GPU, the reference's step 3-4
report (code/run_any_model.py:80-110): per quantized linear, MSE and cosine
between the original bf16 weight and w_hat; for the model, MSE and cosine
between baseline and quantized logits. The sums come from one deterministic
float64 reduction kernel (cdq_compare_stats); nothing is copied to the host
but the four sums."""
from __future__ import annotations

import math
import time

import torch
import torch.nn as nn

from . import _lib as L
from . import ops

_WS_BYTES = 32 * 1024


def compare(a: torch.Tensor, b: torch.Tensor) -> dict:
    """MSE and cosine of two same-size CUDA tensors (bf16 or float32), float64 sums."""
    if a.numel() != b.numel() or a.dtype != b.dtype or not a.is_cuda or a.device != b.device:
        raise ValueError("compare: two CUDA tensors of one dtype and size expected")
    dt = {torch.bfloat16: 0, torch.float32: 1}.get(a.dtype)
    if dt is None:
        raise ValueError("compare: bf16 or float32")
    a, b = a.contiguous(), b.contiguous()
    out = torch.empty(4, dtype=torch.float64, device=a.device)
    ws = torch.empty(_WS_BYTES // 8, dtype=torch.float64, device=a.device)
    L.check(L.lib().cdq_compare_stats(a.data_ptr(), b.data_ptr(), a.numel(), dt, out.data_ptr(), ws.data_ptr(),
                                      _WS_BYTES, torch.cuda.current_stream(a.device).cuda_stream),
            "cdq_compare_stats")
    sd, sab, saa, sbb = out.tolist()
    return {"mse": sd / a.numel(), "cos": sab / max(math.sqrt(saa * sbb), 1e-8), "n": a.numel()}


@torch.no_grad()
def quantize_with_report(model: nn.Module, subs=("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj",
                                                  "up_proj", "down_proj"), lattice=None) -> dict:
    """The reference's quantize-and-measure loop (code/run_any_model.py:80-102):
    every nn.Linear whose name contains one of `subs` is quantized on the GPU,
    compared with its w_hat, and replaced by the fused CDQLinear."""
    from .quant import CDQLinear
    t0 = time.time()
    mses, coss, per = [], [], {}
    tot_w = tot_res = 0
    targets = [(n, m) for n, m in model.named_modules()
               if isinstance(m, nn.Linear) and m.weight.dim() == 2 and any(s in n for s in subs)]
    for name, mod in targets:
        ow = mod.weight.data.to(torch.bfloat16)
        cdq, _ = CDQLinear.from_linear(mod, lattice=lattice)
        rw = ops.dequant(cdq.device_pack)
        r = compare(ow.reshape(-1), rw.reshape(-1))
        mses.append(r["mse"])
        coss.append(r["cos"])
        per[name] = r
        tot_w += ow.numel()
        tot_res += int(cdq.device_pack.n_res)
        parent, _, attr = name.rpartition(".")
        setattr(model.get_submodule(parent) if parent else model, attr, cdq)
    return {"linears": len(targets), "params": tot_w, "residuals": tot_res,
            "residual_pct": 100.0 * tot_res / max(1, tot_w), "seconds": time.time() - t0,
            "weight_mse": sum(mses) / max(1, len(mses)), "weight_cos": sum(coss) / max(1, len(coss)),
            "per_linear": per}


def logit_report(base_logits: torch.Tensor, q_logits: torch.Tensor) -> dict:
    """code/run_any_model.py:105-110: MSE and cosine over all logits (float32)."""
    r = compare(base_logits.float().reshape(-1), q_logits.float().reshape(-1))
    return {"logits_mse": r["mse"], "logits_cos": r["cos"]}
