"""Drop-in mirror of the reference loader, code/cdq_loader.py.

``load_cdq(model, path)`` parses a .cdq file (the C codec), builds each
packed weight in the device layout on the GPU and swaps the matching
submodule for a loader ``CDQLinear`` whose forward is the fused
dequant-GEMV (code/cdq_loader.py:61-110). The loader ``CDQLinear(q, s,
offs, vals, shape, bias)`` keeps the reference's constructor
(code/cdq_loader.py:43-58); its q / s / offs / vals are read-only views
rebuilt from the device pack. Unlike the reference loader, which accepts
version 1 files only, 16-state (version 2) files load as well.
"""
from __future__ import annotations

import struct

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops
from .pack_file import decode_tensor_device, scan_cdq
from .quant import CAMKII_LATTICE

MAGIC, VER = b"CDQ1", 1
TILE = 32
LATTICE = CAMKII_LATTICE


def _fp8_codes_of(s: torch.Tensor) -> np.ndarray:
    """The loader keeps decoded scales (bf16 of the fp8 value); the fp8 code
    is recovered exactly by re-encoding (every fp8 value is a bf16 value)."""
    return s.detach().cpu().reshape(-1).to(torch.float8_e4m3fn).view(torch.uint8).numpy()


class CDQLinear(nn.Module):
    """Loader CDQLinear (code/cdq_loader.py:43-58) on the fused GPU kernel."""

    def __init__(self, q=None, s=None, offs=None, vals=None, shape=None, bias=None,
                 device_pack: ops.DevicePack | None = None):
        super().__init__()
        if device_pack is None:
            rows, cols = shape
            n_states = 26
            device_pack = ops.DevicePack.from_reference(
                q, _fp8_codes_of(s), offs, vals, rows, cols, n_states,
                device=torch.device("cuda", torch.cuda.current_device()))
        self.shape = (device_pack.rows, device_pack.cols)
        self.n_states = device_pack.n_states
        self._n_res = device_pack.n_res
        for k, v in device_pack.tensors().items():
            self.register_buffer(k, v)
        self.bias = (nn.Parameter(bias.detach().to(device_pack.device), requires_grad=False)
                     if bias is not None else None)
        self._ws: dict = {}

    @property
    def device_pack(self) -> ops.DevicePack:
        return ops.DevicePack(self.shape[0], self.shape[1], self.n_states, self._n_res,
                              self.units, self.res_ptr, self.res_ent, self.res_q,
                              _ws=self._ws)

    def _ref(self):
        return self.device_pack.to_reference()

    @property
    def q(self):
        return torch.from_numpy(self._ref()["quant_indices"])

    @property
    def s(self):
        return torch.from_numpy(self._ref()["scales_f8"]).view(torch.float8_e4m3fn) \
            .to(torch.bfloat16).view(-1, 1)

    @property
    def offs(self):
        return torch.from_numpy(self._ref()["residual_indices"])

    @property
    def vals(self):
        return torch.from_numpy(self._ref()["residual_values"]).view(torch.bfloat16)

    def forward(self, x):
        if x.dtype == torch.bfloat16:
            b = self.bias.to(x.dtype) if self.bias is not None else None
            return ops.linear(self.device_pack, x, b)
        w = ops.dequant(self.device_pack).view(self.shape).to(x.dtype)
        return F.linear(x, w, self.bias.to(x.dtype) if self.bias is not None else None)


def load_cdq(model, path="qwen05.cdq"):
    raw = open(path, "rb").read()
    assert raw[:4] == MAGIC
    (ver,) = struct.unpack_from("<H", raw, 4)
    assert ver in (1, 2), f"unsupported version {ver}"
    n_states, tabs = scan_cdq(raw)
    dev = torch.device("cuda", torch.cuda.current_device())
    got = 0
    for t in tabs:
        name = t.name.decode()
        modname = name.replace(".weight", "")
        try:
            mod = model.get_submodule(modname)
        except AttributeError:
            continue
        d = decode_tensor_device(raw, n_states, t, dev)  # records unpacked and converted on the GPU
        pack = ops.DevicePack.from_reference_device(d["quant_indices"], d["scales_f8"],
                                                    d["residual_indices"], d["residual_values"],
                                                    int(t.rows), int(t.cols), n_states)
        bias = mod.bias.data if getattr(mod, "bias", None) is not None else None
        cdq = CDQLinear(bias=bias, device_pack=pack)
        parent, _, attr = modname.rpartition(".")
        setattr(model.get_submodule(parent) if parent else model, attr, cdq)
        got += 1
    print(f"patched {got} CDQLinear modules from {path}")
    return model
