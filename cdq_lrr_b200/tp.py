"""Tensor-parallel execution of CDQ projections (one process per GPU).

Column-parallel projections (q/k/v/gate/up: split the output rows) need no
collective; row-parallel projections (o/down: split K on tile boundaries)
produce float32 partial outputs that are summed by an all-reduce, after which
the bias is added once and the result is rounded to bf16. Shards are cut from
the reference-format pack (code/cdq_lrr_qwen05.py:121-133), whose tiles are
row-local 32-weight runs, so a sharded weight is bit-identical to the
corresponding part of the unsharded one.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops

TILE = 32
UNIT_TILES = 2  # a device unit spans two tile columns: K splits prefer unit boundaries


def _bounds(n: int, world: int, rank: int, align: int) -> tuple[int, int]:
    """Contiguous balanced split of n into world parts on `align` boundaries."""
    units = -(-n // align)
    lo = (units * rank) // world
    hi = (units * (rank + 1)) // world
    return min(lo * align, n), min(hi * align, n)


def row_bounds(rows: int, world: int, rank: int) -> tuple[int, int]:
    return _bounds(rows, world, rank, 16)


def k_bounds(cols: int, world: int, rank: int) -> tuple[int, int]:
    """Column range [c0, c1) of rank's K slice, on tile (preferably unit) boundaries."""
    kt = cols // TILE
    align = UNIT_TILES if kt >= world * UNIT_TILES else 1
    t0, t1 = _bounds(kt, world, rank, align)
    return t0 * TILE, t1 * TILE


def shard_reference(ref: dict, rows: int, cols: int, kind: str, world: int, rank: int) -> tuple[dict, int, int, int]:
    """Cut rank's shard out of a reference-format pack.

    kind "col": rows split (column-parallel layer); kind "row": K split
    (row-parallel layer). Returns (shard pack, shard rows, shard cols, offset)
    where offset is the first output row ("col") or input column ("row")."""
    q = np.asarray(ref["quant_indices"]).reshape(rows, cols // TILE, TILE)
    sc = np.asarray(ref["scales_f8"]).reshape(rows, cols // TILE)
    ri = np.asarray(ref["residual_indices"], dtype=np.int64).reshape(-1)
    rv = np.asarray(ref["residual_values"]).reshape(-1)
    sb = np.asarray(ref["scales_bf16"]).reshape(rows, cols // TILE) if "scales_bf16" in ref else None
    r_of, c_of = ri // cols, ri % cols
    if kind == "col":
        r0, r1 = row_bounds(rows, world, rank)
        keep = (r_of >= r0) & (r_of < r1)
        out = {"quant_indices": q[r0:r1].reshape(-1, TILE), "scales_f8": sc[r0:r1].reshape(-1),
               "residual_indices": (r_of[keep] - r0) * cols + c_of[keep], "residual_values": rv[keep]}
        if sb is not None:
            out["scales_bf16"] = sb[r0:r1].reshape(-1)
        return out, r1 - r0, cols, r0
    if kind == "row":
        c0, c1 = k_bounds(cols, world, rank)
        t0, t1 = c0 // TILE, c1 // TILE
        keep = (c_of >= c0) & (c_of < c1)
        w = c1 - c0
        out = {"quant_indices": q[:, t0:t1].reshape(-1, TILE), "scales_f8": sc[:, t0:t1].reshape(-1),
               "residual_indices": r_of[keep] * w + (c_of[keep] - c0), "residual_values": rv[keep]}
        if sb is not None:
            out["scales_bf16"] = sb[:, t0:t1].reshape(-1)
        return out, rows, w, c0
    raise ValueError(f"unknown shard kind {kind!r}")


class OneShotAllReduce:
    """In-place float32 sum across the ranks of a process group by one kernel
    over NVLink peer memory (cdq_allreduce_f32): every rank's region is
    exported once with a CUDA IPC handle and mapped by every other rank, so a
    call costs one launch, one flag exchange and W peer reads per element, and
    every rank gets bit-identical sums (rank-order addition). Every rank must
    make the same calls in the same order; capturable in a CUDA graph.
    close() releases the mappings (after a barrier, so no peer still reads)."""

    def __init__(self, cap: int, group=None, device=None):
        import ctypes as C
        import torch.distributed as dist
        from . import _lib as L
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if self.world > L.AR_MAX_RANKS:
            raise ValueError(f"one-shot all-reduce serves at most {L.AR_MAX_RANKS} ranks")
        self.cap = int(cap)
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        with torch.cuda.device(self.device):
            own = C.c_void_p()
            h = L.cdq_ipc_handle()
            L.check(L.lib().cdq_ar_create(self.cap, C.byref(own), C.byref(h)), "cdq_ar_create")
            handles = [bytes(h.bytes)]
            if self.world > 1:
                handles = [None] * self.world
                dist.all_gather_object(handles, bytes(h.bytes), group=group)
            ptrs = []
            for q in range(self.world):
                if q == self.rank:
                    ptrs.append(own.value)
                    continue
                hq = L.cdq_ipc_handle()
                C.memmove(hq.bytes, handles[q], 64)
                p = C.c_void_p()
                L.check(L.lib().cdq_ar_open(C.byref(hq), C.byref(p)), "cdq_ar_open")
                ptrs.append(p.value)
        self._own = own.value
        self._regions = (C.c_void_p * L.AR_MAX_RANKS)(*ptrs)

    def __call__(self, y: torch.Tensor) -> torch.Tensor:
        from . import _lib as L
        if y.dtype != torch.float32 or not y.is_cuda or not y.is_contiguous():
            raise ValueError("one-shot all-reduce: contiguous float32 CUDA tensor expected")
        L.check(L.lib().cdq_allreduce_f32(self._regions, self.world, self.rank, self.cap, y.data_ptr(),
                                          y.numel(), torch.cuda.current_stream(y.device).cuda_stream),
                "cdq_allreduce_f32")
        return y

    def close(self) -> None:
        import torch.distributed as dist
        from . import _lib as L
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for q in range(self.world):
                if q != self.rank:
                    L.lib().cdq_ar_close(self._regions[q])
            L.lib().cdq_ar_destroy(self._own)
        self._own = None


class TPLinear:
    """One projection's shard on this rank.

    kind "col": y_local = x @ w_shard^T (+ bias slice), bf16 [M, rows_shard].
    kind "row": y = all_reduce_sum(x[:, K slice] @ w_shard^T) (+ bias), bf16
    [M, rows]; the partial sums are float32 and the reduction runs on the
    current stream, through the given OneShotAllReduce or else
    torch.distributed (NCCL between GPUs)."""

    def __init__(self, pack: ops.DevicePack, kind: str, offset: int, full_rows: int,
                 bias: torch.Tensor | None = None, group=None, allreduce: OneShotAllReduce | None = None):
        self.pack, self.kind, self.offset, self.full_rows = pack, kind, offset, full_rows
        self.bias = bias
        self.group = group
        self.allreduce = allreduce

    @classmethod
    def from_reference(cls, ref: dict, rows: int, cols: int, n_states: int, kind: str, world: int,
                       rank: int, bias: torch.Tensor | None = None, device="cuda", group=None):
        shard, rs, cs, off = shard_reference(ref, rows, cols, kind, world, rank)
        pack = ops.DevicePack.from_reference(shard["quant_indices"], shard["scales_f8"],
                                             shard["residual_indices"], shard["residual_values"],
                                             rs, cs, n_states, device=device)
        b = None
        if bias is not None:
            b = bias[off:off + rs] if kind == "col" else bias
            b = b.to(device)
        return cls(pack, kind, off, rows, b, group)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.kind == "col":
            return ops.linear(self.pack, x, self.bias)
        xs = x[..., self.offset:self.offset + self.pack.cols].contiguous()
        y = ops.linear(self.pack, xs, None, out_f32=True)
        if self.allreduce is not None:
            self.allreduce(y)
        elif torch.distributed.is_available() and torch.distributed.is_initialized():
            torch.distributed.all_reduce(y, group=self.group)
        if self.bias is not None:
            y = y + self.bias.float()
        return y.to(torch.bfloat16)
