"""Drop-in mirror of the reference quantizer module, code/cdq_lrr_qwen05.py.

Same names, arguments and return values as the reference:

* ``CAMKII_LATTICE`` / ``CAMKII_LATTICE_16`` / ``TILE`` / ``STC_FRAC``
  (code/cdq_lrr_qwen05.py:24-44);
* ``fp8_quantize_scale`` (:49-60);
* ``quantize_cdq_lrr(weight, chunk_tiles=8192, lattice=None, stc_frac=None)``
  (:63-133) -> dict with the reference's keys, CPU tensors;
* ``dequantize(pack, device=None, dtype=torch.bfloat16)`` (:141-152);
* ``CDQLinear(pack, in_features, out_features, bias=None)`` with
  ``from_linear``, ``dequant_weight`` and ``forward`` (:155-204);
* ``effective_bpw`` (:207-215).

The work runs on the GPU: quantisation in cdq_quantize, dequantisation in
cdq_dequant, and ``CDQLinear.forward`` in the fused dequant-GEMV, which never
materialises w_hat. Differences from the reference, all deliberate:

* only the two built-in lattices are accepted (the kernels carry their bf16
  tables); any other ``lattice`` raises ValueError;
* the returned dict has exactly the reference's keys; the packed weight in
  the device layout it was built from is remembered alongside (keyed by the
  dict's quant_indices tensor), so CDQLinear does not repack it;
* CDQLinear stores the device pack as its buffers (``units``,
  ``res_ptr``, ``res_ent``, ``res_q``); the reference buffer names
  (``quant_indices``, ``scales_f8``, ``scales_bf16``, ``residual_indices``,
  ``residual_values``, ``lattice``) are read-only properties rebuilt from it,
  and ``load_state_dict`` accepts a reference CDQLinear state dict;
* inputs that are not bf16 go through the bit-exact dequant kernel and
  ``F.linear`` in the input's dtype (the reference's ``w.to(x.dtype)``).
"""
from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops

TARGET_SUBSTRINGS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
TILE = 32
STC_FRAC = 0.0156

CAMKII_LATTICE = torch.tensor([
    -1.0000, -0.7321, -0.5284, -0.3752, -0.2612, -0.1774, -0.1167, -0.0734,
    -0.0432, -0.0229, -0.0101, -0.0031, -0.0005, 0.0005, 0.0031, 0.0101,
    0.0229, 0.0432, 0.0734, 0.1167, 0.1774, 0.2612, 0.3752, 0.5284,
    0.7321, 1.0000,
], dtype=torch.bfloat16)

CAMKII_LATTICE_16 = torch.tensor([
    -0.9685, -0.7525, -0.5834, -0.4414, -0.3174, -0.2048, -0.0998,
    0.0000,
    0.0998, 0.2048, 0.3174, 0.4414, 0.5834, 0.7525, 0.9685,
    0.9685,
], dtype=torch.bfloat16)

FP8_DTYPE = torch.float8_e4m3fn


def _n_states_of(lattice) -> int:
    if lattice is None:
        return 26
    lat = torch.as_tensor(lattice).to(torch.bfloat16).cpu()
    for ref, n in ((CAMKII_LATTICE, 26), (CAMKII_LATTICE_16, 16)):
        if lat.numel() == ref.numel() and torch.equal(lat.view(torch.int16), ref.view(torch.int16)):
            return n
    raise ValueError("only the built-in 26-state and 16-state CaMKII lattices are supported")


def _lattice_of(n_states: int) -> torch.Tensor:
    return CAMKII_LATTICE if n_states == 26 else CAMKII_LATTICE_16


def _device_for(t: torch.Tensor) -> torch.device:
    if t.is_cuda:
        return t.device
    if not torch.cuda.is_available():
        raise RuntimeError("the CDQ kernels need a CUDA device; none is available")
    return torch.device("cuda", torch.cuda.current_device())


def fp8_quantize_scale(sigma_bf16: torch.Tensor) -> torch.Tensor:
    """Per-tile scale to float8 e4m3fn and back to bf16 (code/cdq_lrr_qwen05.py:49-52)."""
    return sigma_bf16.to(FP8_DTYPE).to(torch.bfloat16)


def quantize_cdq_lrr(weight: torch.Tensor, chunk_tiles: int = 8192, lattice=None,
                     stc_frac: float | None = None) -> dict:
    """Full CDQ-LRR quantisation of a 2-D weight on the GPU.

    Returns the reference's dict (CPU tensors, code/cdq_lrr_qwen05.py:121-133:
    the same keys, types, dtypes and shapes). ``chunk_tiles`` is accepted for
    signature compatibility; the GPU quantizer needs no chunking.
    """
    assert weight.dim() == 2, f"expected 2D, got {weight.shape}"
    n_states = _n_states_of(lattice)
    if stc_frac is None:
        stc_frac = STC_FRAC
    orig_shape = tuple(weight.shape)
    dev = _device_for(weight)
    w = weight.detach().to(device=dev, dtype=torch.bfloat16).contiguous()
    pack, info = ops.quantize(w, n_states=n_states, stc_frac=stc_frac)
    ref = pack.to_reference()
    n_tiles = pack.n_tiles
    scales_u8 = torch.from_numpy(ref["scales_f8"]).view(n_tiles, 1)
    scales_f8 = scales_u8.view(FP8_DTYPE)
    out = {
        "quant_indices": torch.from_numpy(ref["quant_indices"]),
        "scales_f8": scales_f8,
        "scales_bf16": scales_f8.to(torch.bfloat16),
        "residual_indices": torch.from_numpy(ref["residual_indices"]),
        "residual_values": torch.from_numpy(ref["residual_values"]).view(torch.bfloat16),
        "orig_shape": orig_shape,
        "outlier_count": int(info["n_res"]),
        "numel": int(w.numel()),
        "n_tiles": int(n_tiles),
        "lattice": _lattice_of(n_states).clone(),
        "n_states": n_states,
    }
    _remember(out["quant_indices"], pack)
    return out


# The device pack a quantize_cdq_lrr dict was built from, keyed by the dict's
# quant_indices tensor (held weakly), so that CDQLinear(pack, ...) and
# dequantize(pack) reuse it instead of uploading the arrays again. The dict
# itself keeps exactly the reference's keys.
_PACKS: dict[int, tuple] = {}


def _remember(key: torch.Tensor, dp: ops.DevicePack) -> None:
    import weakref
    k = id(key)
    _PACKS[k] = (weakref.ref(key), dp)
    weakref.finalize(key, _PACKS.pop, k, None)


def _device_pack_of(pack: dict, device=None) -> ops.DevicePack:
    entry = _PACKS.get(id(pack["quant_indices"]))
    dp = entry[1] if entry is not None and entry[0]() is pack["quant_indices"] else None
    if dp is None:
        rows, cols = pack["orig_shape"]
        n_states = _n_states_of(pack.get("lattice"))
        dp = ops.DevicePack.from_reference(
            pack["quant_indices"], pack["scales_f8"], pack["residual_indices"],
            pack["residual_values"], rows, cols, n_states)
    if device is not None:
        dp = dp.to(device)
    elif dp.device.type != "cuda":
        dp = dp.to(torch.device("cuda", torch.cuda.current_device()))
    return dp


def dequantize(pack: dict, device=None, dtype=torch.bfloat16) -> torch.Tensor:
    """w_hat = sigma * Lattice[q] + residuals, bit-exact, by the GPU dequant kernel.

    With ``device=None`` the result is returned on the CPU like the
    reference's (whose pack lives on the CPU)."""
    target = torch.device(device) if device is not None else None
    run_on = target if (target is not None and target.type == "cuda") else None
    dp = _device_pack_of(pack, run_on)
    w = ops.dequant(dp)
    if target is None:
        w = w.cpu()
    elif w.device != target:
        w = w.to(target)
    return w.view(pack["orig_shape"]).to(dtype)


class CDQLinear(nn.Module):
    """Linear with the fused CDQ-LRR dequant-GEMV (code/cdq_lrr_qwen05.py:155-204)."""

    def __init__(self, pack, in_features: int, out_features: int, bias=None):
        super().__init__()
        dp = _device_pack_of(pack)
        self.orig_shape = tuple(pack["orig_shape"])
        self.in_features = in_features
        self.out_features = out_features
        self.n_states = dp.n_states
        self._n_res = dp.n_res
        for k, v in dp.tensors().items():
            self.register_buffer(k, v)
        if bias is not None:
            self.bias = nn.Parameter(bias.detach().to(device=dp.device, dtype=torch.bfloat16),
                                     requires_grad=False)
        else:
            self.bias = None
        self._pack_meta = {
            "outlier_count": int(pack.get("outlier_count", dp.n_res)),
            "numel": int(pack.get("numel", self.orig_shape[0] * self.orig_shape[1])),
            "n_tiles": int(pack.get("n_tiles", dp.n_tiles)),
        }
        self._ws: dict = {}

    @property
    def device_pack(self) -> ops.DevicePack:
        dp = ops.DevicePack(self.orig_shape[0], self.orig_shape[1], self.n_states, self._n_res,
                            self.units, self.res_ptr, self.res_ent, self.res_q,
                            _ws=self._ws)
        return dp

    @classmethod
    def from_linear(cls, lin: nn.Linear, lattice=None):
        with torch.no_grad():
            pack = quantize_cdq_lrr(lin.weight.data, lattice=lattice)
        obj = cls(pack, lin.in_features, lin.out_features,
                  bias=lin.bias.data if lin.bias is not None else None)
        return obj, pack

    # reference buffer names, rebuilt from the device pack
    def _reference(self) -> dict:
        return self.device_pack.to_reference()

    @property
    def quant_indices(self) -> torch.Tensor:
        return torch.from_numpy(self._reference()["quant_indices"])

    @property
    def scales_f8(self) -> torch.Tensor:
        r = self._reference()["scales_f8"]
        return torch.from_numpy(r).view(-1, 1).view(FP8_DTYPE)

    @property
    def scales_bf16(self) -> torch.Tensor:
        return self.scales_f8.to(torch.bfloat16)

    @property
    def residual_indices(self) -> torch.Tensor:
        return torch.from_numpy(self._reference()["residual_indices"])

    @property
    def residual_values(self) -> torch.Tensor:
        return torch.from_numpy(self._reference()["residual_values"]).view(torch.bfloat16)

    @property
    def lattice(self) -> torch.Tensor:
        return _lattice_of(self.n_states).clone()

    def dequant_weight(self) -> torch.Tensor:
        return ops.dequant(self.device_pack).view(self.orig_shape)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dtype == torch.bfloat16:
            return ops.linear(self.device_pack, x, self.bias)
        w = self.dequant_weight().to(x.dtype)
        return F.linear(x, w, self.bias.to(x.dtype) if self.bias is not None else None)

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys,
                              unexpected_keys, error_msgs):
        # a reference CDQLinear state dict: repack it into the device layout
        ref_keys = ("quant_indices", "scales_f8", "residual_indices", "residual_values")
        if all(prefix + k in state_dict for k in ref_keys):
            lat = state_dict.get(prefix + "lattice")
            n_states = _n_states_of(lat)
            rows, cols = self.orig_shape
            dp = ops.DevicePack.from_reference(
                state_dict[prefix + "quant_indices"], state_dict[prefix + "scales_f8"],
                state_dict[prefix + "residual_indices"], state_dict[prefix + "residual_values"],
                rows, cols, n_states, device=self.units.device)
            self.n_states = n_states
            self._n_res = dp.n_res
            self._ws.clear()
            for k, v in dp.tensors().items():
                setattr(self, k, v)
            for k in ref_keys + ("scales_bf16", "lattice"):
                state_dict.pop(prefix + k, None)
            if prefix + "bias" in state_dict and self.bias is not None:
                with torch.no_grad():
                    self.bias.copy_(state_dict.pop(prefix + "bias"))
            return
        # own format: buffers may change length (residual count); they did not
        # come through the validating converters, so they are checked before
        # any kernel reads them
        own = {k: state_dict[prefix + k].to(self.units.device)
               for k in ("units", "res_ptr", "res_ent", "res_q") if prefix + k in state_dict}
        if own and self.units.is_cuda:
            rows, cols = self.orig_shape
            t = {k: own.get(k, getattr(self, k)) for k in ("units", "res_ptr", "res_ent", "res_q")}
            ops.DevicePack(rows, cols, self.n_states, int(t["res_ent"].numel()), **t).validate()
        for k, v in own.items():
            setattr(self, k, v)
        self._n_res = int(self.res_ent.numel())
        self._ws.clear()
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys,
                                      unexpected_keys, error_msgs)

    def extra_repr(self):
        m = self._pack_meta
        return (f"shape={self.orig_shape}, states={self.n_states}, "
                f"outliers={m['outlier_count']}/{m['numel']} "
                f"({100 * m['outlier_count'] / max(1, m['numel']):.2f}%)")


def effective_bpw(total_numel, total_tiles, total_residuals, index_bits=5,
                  header_bytes_per_tile=0):
    """Bits per weight of the prototype accounting (code/cdq_lrr_qwen05.py:207-215)."""
    bits = (total_numel * index_bits + total_tiles * 8
            + total_residuals * (16 + 32)
            + total_tiles * header_bytes_per_tile * 8)
    return bits / max(1, total_numel)
