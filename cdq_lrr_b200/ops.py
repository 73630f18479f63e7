"""Torch-facing calls into the C ABI: device packs, fused linear, dequant, quantize.

PyTorch provides device memory and the current CUDA stream; every piece of
arithmetic runs in libcdq_b200.so. CPU tensors are rejected: there is no CPU
path in the product.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib as L

TILE = 32


def _vp(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{what}: expected a CUDA tensor (the CDQ kernels have no CPU path)")


@dataclass
class DevicePack:
    """One packed weight in the device layout of include/cdq.h.

    The units are a uint8 tensor; uint32 buffers are held as int32 tensors
    (bit patterns)."""
    rows: int
    cols: int
    n_states: int
    n_res: int
    units: torch.Tensor
    res_ptr: torch.Tensor
    res_ent: torch.Tensor
    res_q: torch.Tensor
    _ws: dict = field(default_factory=dict, repr=False)

    @property
    def device(self) -> torch.device:
        return self.units.device

    @property
    def n_tiles(self) -> int:
        return self.rows * self.cols // TILE

    def struct(self) -> L.cdq_packed:
        p = L.cdq_packed()
        p.rows, p.cols, p.n_states, p.reserved0 = self.rows, self.cols, self.n_states, 0
        p.n_res = self.n_res
        p.units = self.units.data_ptr()
        p.res_ptr = self.res_ptr.data_ptr()
        p.res_ent = self.res_ent.data_ptr() if self.res_ent.numel() else None
        p.res_q = self.res_q.data_ptr() if self.res_q.numel() else None
        return p

    def validate(self) -> "DevicePack":
        """Checks a pack that did not come from this library's converters or
        quantizer (for example buffers loaded from a state dict) before any
        kernel reads it: buffer sizes and dtypes on the host, then the pair
        codes and the residual CSR on the GPU (cdq_check_device_pack). Raises
        CdqError (status 5, CDQ_ERR_FORMAT) on a malformed pack; returns self."""
        _require_cuda(self.units, "DevicePack.validate")
        s = L.sizes(self.rows, self.cols, self.n_states)
        ok = (self.units.dtype == torch.uint8 and self.units.numel() == s.units_bytes
              and self.res_ptr.dtype == torch.int32 and self.res_ptr.numel() == s.res_ptr_count
              and self.res_ent.dtype == torch.int32 and self.res_ent.numel() >= self.n_res >= 0
              and all(t.is_contiguous() and t.device == self.units.device
                      for t in (self.units, self.res_ptr, self.res_ent)))
        if not ok:
            raise L.CdqError(5, "DevicePack.validate (buffer sizes)")
        bad = torch.zeros(1, dtype=torch.int32, device=self.device)
        st = self.struct()
        L.check(L.lib().cdq_check_device_pack(C.byref(st), _vp(bad), _stream(self.device)),
                "cdq_check_device_pack")
        if int(bad.item()):
            raise L.CdqError(5, f"DevicePack.validate ({int(bad.item())} malformed parts)")
        return self

    def tensors(self) -> dict[str, torch.Tensor]:
        return {"units": self.units, "res_ptr": self.res_ptr,
                "res_ent": self.res_ent, "res_q": self.res_q}

    @classmethod
    def empty(cls, rows: int, cols: int, n_states: int, res_capacity: int,
              device) -> "DevicePack":
        s = L.sizes(rows, cols, n_states)
        dev = torch.device(device)
        return cls(rows, cols, n_states, 0,
                   torch.empty(s.units_bytes, dtype=torch.uint8, device=dev),
                   torch.empty(s.res_ptr_count, dtype=torch.int32, device=dev),
                   torch.empty(max(res_capacity, 0), dtype=torch.int32, device=dev),
                   torch.empty(max(res_capacity, 0), dtype=torch.uint8, device=dev))

    def to(self, device) -> "DevicePack":
        t = {k: v.to(device) for k, v in self.tensors().items()}
        return DevicePack(self.rows, self.cols, self.n_states, self.n_res, **t)

    # ---- reference-format conversion (host C code) ----
    @classmethod
    def from_reference(cls, quant_indices, scales_f8, residual_indices, residual_values,
                       rows: int, cols: int, n_states: int, device="cpu") -> "DevicePack":
        """Reference pack tensors (code/cdq_lrr_qwen05.py:121-133) -> device layout.
        For a CUDA device the arrays are copied there as they are and converted
        by the device ingest (byte-identical to the host converter used for
        device="cpu")."""
        if torch.device(device).type == "cuda":
            def up(a, dt):
                t = a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(_np(a, dt)))
                return t.to(device)
            rv = residual_values
            if not isinstance(rv, torch.Tensor):
                rv = torch.from_numpy(np.ascontiguousarray(_np(rv, np.uint16)).view(np.int16))
            try:
                return cls.from_reference_device(up(quant_indices, np.uint8), up(scales_f8, np.uint8),
                                                 up(residual_indices, np.int64), rv.to(device), rows, cols, n_states)
            except ValueError as e:
                if "malformed" not in str(e):
                    raise
                raise L.CdqError(3, "cdq_pack_from_reference_device") from e
        q = np.ascontiguousarray(_np(quant_indices, np.uint8).reshape(-1))
        sc = np.ascontiguousarray(_np(scales_f8, np.uint8).reshape(-1))
        ri = np.ascontiguousarray(_np(residual_indices, np.int64).reshape(-1))
        rv = np.ascontiguousarray(_np(residual_values, np.uint16).reshape(-1))
        if q.size != rows * cols or sc.size != rows * cols // TILE or ri.size != rv.size:
            raise ValueError("reference pack tensors do not match the weight shape")
        host = cls.empty(rows, cols, n_states, ri.size, "cpu")
        st = host.struct()
        L.check(L.lib().cdq_host_from_reference(
            rows, cols, n_states, q.ctypes.data_as(C.c_void_p), sc.ctypes.data_as(C.c_void_p),
            ri.ctypes.data_as(C.c_void_p) if ri.size else None,
            rv.ctypes.data_as(C.c_void_p) if rv.size else None, ri.size, C.byref(st)),
            "cdq_host_from_reference")
        host.n_res = int(ri.size)
        return host if torch.device(device).type == "cpu" else host.to(device)

    @classmethod
    def from_reference_device(cls, quant_indices: torch.Tensor, scales_f8: torch.Tensor,
                              residual_indices: torch.Tensor, residual_values: torch.Tensor,
                              rows: int, cols: int, n_states: int) -> "DevicePack":
        """Reference pack tensors already on a CUDA device -> device layout, on the
        GPU (cdq_pack_from_reference_device; byte-identical to from_reference)."""
        dev = quant_indices.device
        for t in (scales_f8, residual_indices, residual_values):
            if t.device != dev:
                raise ValueError("reference pack tensors must be on one CUDA device")
        q = quant_indices.reshape(-1).contiguous().view(torch.uint8)
        sc = scales_f8.reshape(-1).contiguous().view(torch.uint8)
        ri = residual_indices.reshape(-1).to(torch.int64).contiguous()
        rv = residual_values.reshape(-1).contiguous().view(torch.int16)
        if q.numel() != rows * cols or sc.numel() != rows * cols // TILE or ri.numel() != rv.numel():
            raise ValueError("reference pack tensors do not match the weight shape")
        pack = cls.empty(rows, cols, n_states, ri.numel(), dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        st = pack.struct()
        with torch.cuda.device(dev):
            L.check(L.lib().cdq_pack_from_reference_device(
                rows, cols, n_states, q.data_ptr(), sc.data_ptr(), ri.data_ptr() if ri.numel() else None,
                rv.data_ptr() if rv.numel() else None, ri.numel(), C.byref(st), err.data_ptr(),
                torch.cuda.current_stream(dev).cuda_stream), "cdq_pack_from_reference_device")
        if int(err.item()) != 0:
            raise ValueError("malformed reference pack (lattice index or residual positions)")
        pack.n_res = int(ri.numel())
        return pack

    def to_reference(self) -> dict[str, np.ndarray]:
        """Device layout -> reference pack arrays (numpy, host)."""
        host = self.to("cpu")
        n_tiles = self.n_tiles
        q = np.empty((n_tiles, TILE), dtype=np.uint8)
        sc = np.empty(n_tiles, dtype=np.uint8)
        ri = np.empty(self.n_res, dtype=np.int64)
        rv = np.empty(self.n_res, dtype=np.uint16)
        st = host.struct()
        L.check(L.lib().cdq_host_to_reference(
            C.byref(st), q.ctypes.data_as(C.c_void_p), sc.ctypes.data_as(C.c_void_p),
            ri.ctypes.data_as(C.c_void_p) if ri.size else None,
            rv.ctypes.data_as(C.c_void_p) if rv.size else None), "cdq_host_to_reference")
        return {"quant_indices": q, "scales_f8": sc, "residual_indices": ri, "residual_values": rv}

    # ---- byte accounting ----
    def device_bytes(self) -> int:
        return sum(int(t.numel() * t.element_size()) for t in self.tensors().values()
                   if t is not self.res_q)

    def reference_bytes(self) -> int:
        """Bytes of the reference .cdq tile records of this weight:
        sum over tiles of 2 + index bytes + ceil(21 * residuals / 8)."""
        ib = 20 if self.n_states == 26 else 16
        kt = self.cols // TILE
        rp = self.res_ptr.to("cpu", torch.int64)
        ent = self.res_ent[: self.n_res].to("cpu", torch.int64)
        counts = (rp[1:] - rp[:-1])
        kg = (kt + 31) // 32
        b = torch.arange(counts.numel())
        rows = b // kg  # buckets are (row, group), row major
        row_of = torch.repeat_interleave(rows, counts)
        col = (ent >> 16) & 0xFFFF
        tile = row_of * kt + col // TILE
        tc = torch.bincount(tile, minlength=self.n_tiles)
        return int(self.n_tiles * (2 + ib) + ((tc * 21 + 7) // 8).sum().item())

    # ---- workspace of cdq_linear, kept by the pack: row-block arrival counters
    # (zero before the first call; every call leaves them zero), then float32
    # group sums or the tile path's prepared activations ----
    def linear_workspace(self, m: int) -> torch.Tensor:
        dev = self.device
        key = (dev, m)
        ws = self._ws.get(key)
        if ws is None:
            s = L.sizes(self.rows, self.cols, self.n_states, max_batch=m)
            ws = torch.zeros(max(s.linear_workspace_bytes, 256), dtype=torch.uint8, device=dev)
            self._ws[key] = ws
        return ws


def _np(t, dtype) -> np.ndarray:
    if isinstance(t, torch.Tensor):
        t = t.detach().cpu()
        if t.dtype in (torch.bfloat16, torch.float16):
            t = t.view(torch.int16)
        elif t.dtype == torch.float8_e4m3fn:
            t = t.view(torch.uint8)
        return t.numpy().view(dtype) if t.numpy().dtype.itemsize == np.dtype(dtype).itemsize \
            else t.numpy().astype(dtype)
    a = np.asarray(t)
    return a.view(dtype) if a.dtype.itemsize == np.dtype(dtype).itemsize else a.astype(dtype)


# ------------------------------------------------------------------ kernels


def linear(pack: DevicePack, x: torch.Tensor, bias: torch.Tensor | None = None,
           out_f32: bool = False, out: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ w_hat^T (+ bias) with the fused kernel; x bf16 [..., cols] on CUDA."""
    _require_cuda(x, "cdq linear")
    if x.dtype != torch.bfloat16:
        raise TypeError("cdq linear: x must be bf16")
    if x.shape[-1] != pack.cols:
        raise ValueError(f"cdq linear: x has {x.shape[-1]} features, weight has {pack.cols}")
    if x.device != pack.device:
        raise ValueError("cdq linear: x and the packed weight are on different devices")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, pack.cols)
    if x2.data_ptr() % 16 or not x2.is_contiguous():
        x2 = x2.contiguous().clone()
    m_total = x2.shape[0]
    ydt = torch.float32 if out_f32 else torch.bfloat16
    y = out if out is not None else torch.empty(m_total, pack.rows, dtype=ydt, device=x.device)
    if bias is not None:
        _require_cuda(bias, "cdq linear bias")
        bias = bias.to(torch.bfloat16).contiguous()
    fn = L.lib().cdq_linear_f32 if out_f32 else L.lib().cdq_linear
    st = pack.struct()
    stream = _stream(x.device)
    for m0 in range(0, m_total, L.MAX_BATCH):
        m = min(L.MAX_BATCH, m_total - m0)
        ws = pack.linear_workspace(m)
        L.check(fn(C.byref(st), _vp(x2[m0:m0 + m]), m, _vp(y[m0:m0 + m]), _vp(bias),
                   _vp(ws), ws.numel(), stream), "cdq_linear")
    return y.reshape(*lead, pack.rows)


def _job_workspace(pack: DevicePack, m: int, seen: set, keep: list) -> torch.Tensor:
    """The pack's own workspace for its first job of a launch; further jobs of
    the same launch on the same pack get a workspace each (the jobs run
    concurrently), held in `keep` by the caller for as long as it launches."""
    if id(pack) not in seen:
        seen.add(id(pack))
        return pack.linear_workspace(m)
    s = L.sizes(pack.rows, pack.cols, pack.n_states, max_batch=m)
    ws = torch.zeros(max(s.linear_workspace_bytes, 256), dtype=torch.uint8, device=pack.device)
    keep.append(ws)
    return ws


@dataclass
class GemvTask:
    pack: DevicePack
    x: torch.Tensor
    y: torch.Tensor
    bias: torch.Tensor | None = None


def linear_grouped(tasks: list[GemvTask], m: int) -> None:
    """Independent GEMVs with the same batch m in one launch (per lattice size)."""
    if not tasks:
        return
    jobs = (L.cdq_gemv_job * len(tasks))()
    seen: set[int] = set()
    extra: list[torch.Tensor] = []  # freed after the launch: the allocator is stream-ordered
    for j, t in zip(jobs, tasks):
        _require_cuda(t.x, "cdq grouped linear")
        ws = _job_workspace(t.pack, m, seen, extra)
        j.w = t.pack.struct()
        j.x = t.x.data_ptr()
        j.y = t.y.data_ptr()
        j.bias = t.bias.data_ptr() if t.bias is not None else None
        j.workspace = ws.data_ptr()
        j.workspace_bytes = ws.numel()
        j.out_f32 = 1 if t.y.dtype == torch.float32 else 0
    L.check(L.lib().cdq_linear_grouped(jobs, len(tasks), m, _stream(tasks[0].x.device)),
            "cdq_linear_grouped")


class GroupedLinear:
    """A prepared grouped GEMV: the job table is built once, each call is one
    C-ABI call (one launch per lattice size). The tensors given here must stay
    alive and keep their storage between calls (the decode-step pattern)."""

    def __init__(self, tasks: list[GemvTask], m: int):
        self.tasks = list(tasks)
        self.m = m
        self.jobs = (L.cdq_gemv_job * len(self.tasks))()
        seen: set[int] = set()
        self._extra_ws: list[torch.Tensor] = []
        for j, t in zip(self.jobs, self.tasks):
            _require_cuda(t.x, "cdq grouped linear")
            ws = _job_workspace(t.pack, m, seen, self._extra_ws)
            j.w = t.pack.struct()
            j.x = t.x.data_ptr()
            j.y = t.y.data_ptr()
            j.bias = t.bias.data_ptr() if t.bias is not None else None
            j.workspace = ws.data_ptr()
            j.workspace_bytes = ws.numel()
            j.out_f32 = 1 if t.y.dtype == torch.float32 else 0
        self.device = self.tasks[0].x.device if self.tasks else None
        # per lattice size, per batch of at most L.MAX_JOBS jobs: the residual
        # pre-pass and the streaming kernel for m <= 8; above, the pre-pass,
        # the wide streaming kernel and its fix-up (or, on the tcgen05 tile
        # path, the activation layout and the tile kernel)
        per_ns = {}
        for t in self.tasks:
            per_ns[t.pack.n_states] = per_ns.get(t.pack.n_states, 0) + 1
        per = 2 if m <= 8 else 3
        self.launches = sum(per * -(-n // L.MAX_JOBS) for n in per_ns.values())

    def __call__(self) -> None:
        if self.tasks:
            L.check(L.lib().cdq_linear_grouped(self.jobs, len(self.tasks), self.m,
                                               _stream(self.device)), "cdq_linear_grouped")


def dequant(pack: DevicePack) -> torch.Tensor:
    """Bit-exact w_hat [rows, cols] bf16 on the pack's device."""
    if pack.device.type != "cuda":
        raise RuntimeError("cdq dequant: the pack must be on a CUDA device")
    out = torch.empty(pack.rows, pack.cols, dtype=torch.bfloat16, device=pack.device)
    st = pack.struct()
    L.check(L.lib().cdq_dequant(C.byref(st), _vp(out), _stream(pack.device)), "cdq_dequant")
    return out


def quantize(w: torch.Tensor, n_states: int = 26, stc_frac: float = 0.0156,
             topk_guard: bool = True) -> tuple[DevicePack, dict]:
    """GPU tile quantizer: bf16 [rows, cols] CUDA tensor -> (device pack, info).

    topk_guard=False quantizes as the reference packer CLI does
    (code/cdq_pack.py:279-291, no top-k tie guard): up to every weight can
    become a residual, so the residual buffers are sized for rows * cols."""
    _require_cuda(w, "cdq quantize")
    if w.dim() != 2:
        raise ValueError(f"expected 2D, got {tuple(w.shape)}")
    rows, cols = w.shape
    w = w.detach().to(torch.bfloat16).contiguous()
    s = L.sizes(rows, cols, n_states, stc_frac)
    cap = s.max_res if topk_guard else rows * cols
    pack = DevicePack.empty(rows, cols, n_states, cap, w.device)
    ws = torch.empty(s.quantize_workspace_bytes, dtype=torch.uint8, device=w.device)
    info_t = torch.zeros(C.sizeof(L.cdq_quant_info), dtype=torch.uint8, device=w.device)
    st = pack.struct()
    flags = 0 if topk_guard else L.QUANT_NO_TOPK_GUARD
    L.check(L.lib().cdq_quantize_ex(_vp(w), rows, cols, n_states, stc_frac, flags, cap, C.byref(st),
                                    _vp(info_t), _vp(ws), ws.numel(), _stream(w.device)), "cdq_quantize_ex")
    raw = bytes(info_t.cpu().numpy().tobytes())
    info = L.cdq_quant_info.from_buffer_copy(raw)
    pack.n_res = int(info.n_res)
    if pack.n_res > cap:
        raise L.CdqError(6, "cdq_quantize_ex: residual buffers too small")
    # release the unused residual capacity
    pack.res_ent = pack.res_ent[: pack.n_res].clone()
    pack.res_q = pack.res_q[: pack.n_res].clone()
    return pack, {"n_res": int(info.n_res), "k": int(info.k), "threshold": float(info.threshold),
                  "topk_fallback": bool(info.topk_fallback), "mask_count": int(info.mask_count)}
