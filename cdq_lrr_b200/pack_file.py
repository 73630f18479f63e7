""".cdq file codec and packer, mirroring code/cdq_pack.py.

Same names and formats as the reference module: the bit packers
(``pack_5bit_row``, ``unpack_5bit_row``, ``pack_indices_nibble``,
``unpack_nibble_row``, ``pack_residuals``, ``unpack_residuals``,
code/cdq_pack.py:50-119), ``write_cdq(path, tensors, n_states=26)`` and
``read_cdq(path)`` (:162-234), ``dequant_tile`` (:237-248) and the packer
CLI (:251-318). Encoding and decoding of whole tensors run in the C library
(cdq_file_*), byte-exact with the reference writer. ``write_cdq`` also
accepts tensors given as flat residual lists (``residual_indices`` /
``residual_values``) instead of per-tile blobs, which avoids the per-tile
Python loop, and ``read_device_packs`` returns device packs directly.

The CLI quantises on the GPU with the top-k tie guard of
quantize_cdq_lrr by default; ``--no-topk-guard`` quantises exactly as the
reference CLI's inline quantiser (:279-291), which has no guard (the two
differ only on tensors where the guard fires).
"""
from __future__ import annotations

import ctypes as C
import struct

import numpy as np
import torch

from . import _lib as L
from .ops import DevicePack

MAGIC = b"CDQ1"
VERSION = 1
VERSION2 = 2
TILE = 32
IDX_BYTES_PER_TILE = 20
NIBBLE_BYTES_PER_TILE = 16


def _c_u8(a) -> np.ndarray:
    if isinstance(a, torch.Tensor):
        a = a.detach().cpu().numpy()
    return np.ascontiguousarray(np.asarray(a)).astype(np.uint8, copy=False).reshape(-1)


def _tile_indices(q32, n_states: int) -> bytes:
    q = _c_u8(q32)
    assert q.size == 32
    out = np.empty(20 if n_states == 26 else 16, dtype=np.uint8)
    L.check(L.lib().cdq_pack_tile_indices(q.ctypes.data_as(C.c_void_p), 1, n_states,
                                          out.ctypes.data_as(C.c_void_p)), "cdq_pack_tile_indices")
    return out.tobytes()


def _tile_unpack(buf: bytes, n_states: int) -> torch.Tensor:
    assert len(buf) == (20 if n_states == 26 else 16)
    src = np.frombuffer(bytes(buf), dtype=np.uint8)
    q = np.empty(32, dtype=np.uint8)
    L.check(L.lib().cdq_unpack_tile_indices(src.ctypes.data_as(C.c_void_p), 1, n_states,
                                            q.ctypes.data_as(C.c_void_p)), "cdq_unpack_tile_indices")
    return torch.from_numpy(q)


def pack_5bit_row(q32) -> bytes:
    """32 indices (0..25) -> 20 bytes, 5 bits each, LSB first (code/cdq_pack.py:50-56)."""
    return _tile_indices(q32, 26)


def unpack_5bit_row(buf: bytes) -> torch.Tensor:
    """20 bytes -> 32 indices (code/cdq_pack.py:59-64)."""
    return _tile_unpack(buf, 26)


def pack_indices_nibble(indices_32) -> bytes:
    """32 indices (0..15) -> 16 bytes, even index in the low nibble (code/cdq_pack.py:67-78)."""
    return _tile_indices(indices_32, 16)


def unpack_nibble_row(buf: bytes) -> torch.Tensor:
    """16 bytes -> 32 indices (code/cdq_pack.py:81-88)."""
    return _tile_unpack(buf, 16)


def _bf16_bits(values) -> np.ndarray:
    if isinstance(values, torch.Tensor):
        v = values.detach().cpu()
        if v.dtype != torch.bfloat16:
            v = v.to(torch.bfloat16)
        return np.ascontiguousarray(v.view(torch.int16).numpy().view(np.uint16)).reshape(-1)
    return np.ascontiguousarray(np.asarray(values, dtype=np.uint16)).reshape(-1)


def pack_residuals(offsets, values_bf16) -> bytes:
    """Residuals of one tile -> ceil(21 R / 8) bytes: per residual a 5-bit
    offset then the 16 bf16 bits, LSB first (code/cdq_pack.py:91-105)."""
    offs = _c_u8(offsets)
    vals = _bf16_bits(values_bf16)
    assert offs.size == vals.size
    if offs.size == 0:
        return b""
    out = np.empty((21 * offs.size + 7) // 8, dtype=np.uint8)
    L.check(L.lib().cdq_pack_residual_stream(offs.ctypes.data_as(C.c_void_p), vals.ctypes.data_as(C.c_void_p),
                                             offs.size, out.ctypes.data_as(C.c_void_p)), "cdq_pack_residual_stream")
    return out.tobytes()


def unpack_residuals(buf: bytes, tag_count: int):
    """(offsets uint8 [R], values bf16 [R]) of one tile's residual stream
    (code/cdq_pack.py:108-119)."""
    if tag_count == 0:
        return torch.empty(0, dtype=torch.uint8), torch.empty(0, dtype=torch.bfloat16)
    src = np.frombuffer(bytes(buf), dtype=np.uint8)
    assert src.size >= (21 * tag_count + 7) // 8
    offs = np.empty(tag_count, dtype=np.uint8)
    vals = np.empty(tag_count, dtype=np.uint16)
    L.check(L.lib().cdq_unpack_residual_stream(src.ctypes.data_as(C.c_void_p), tag_count,
                                               offs.ctypes.data_as(C.c_void_p), vals.ctypes.data_as(C.c_void_p)),
            "cdq_unpack_residual_stream")
    return torch.from_numpy(offs), torch.from_numpy(vals.view(np.int16)).view(torch.bfloat16)


def _u8(a) -> np.ndarray:
    if isinstance(a, torch.Tensor):
        a = a.detach().cpu()
        if a.dtype == torch.float8_e4m3fn:
            a = a.view(torch.uint8)
        a = a.numpy()
    return np.ascontiguousarray(np.asarray(a).astype(np.uint8, copy=False)).reshape(-1)


def _flat_residuals(t: dict) -> tuple[np.ndarray, np.ndarray]:
    if "residual_indices" in t:
        ri = t["residual_indices"]
        rv = t["residual_values"]
        ri = np.ascontiguousarray(np.asarray(ri.cpu() if isinstance(ri, torch.Tensor) else ri,
                                             dtype=np.int64)).reshape(-1)
        if isinstance(rv, torch.Tensor):
            rv = rv.detach().cpu()
            rv = (rv.view(torch.int16) if rv.dtype == torch.bfloat16 else rv).numpy()
        rv = np.ascontiguousarray(np.asarray(rv).view(np.uint16) if np.asarray(rv).dtype.itemsize == 2
                                  else np.asarray(rv).astype(np.uint16)).reshape(-1)
        return ri, rv
    tags = _u8(t["tag_counts"])
    ri, rv = [], []
    for ti, (tc, blob) in enumerate(zip(tags.tolist(), t["res_blobs"])):
        if tc:
            o, v = unpack_residuals(blob, tc)
            ri.append(ti * TILE + o.numpy().astype(np.int64))
            rv.append(v.view(torch.int16).numpy().view(np.uint16))
    if not ri:
        return np.empty(0, dtype=np.int64), np.empty(0, dtype=np.uint16)
    ri_a, rv_a = np.concatenate(ri), np.concatenate(rv)
    order = np.argsort(ri_a, kind="stable")
    return ri_a[order], rv_a[order]


def encode_cdq(tensors: dict, n_states: int = 26) -> bytes:
    """The .cdq bytes of ``tensors`` (see write_cdq)."""
    assert n_states in (26, 16)
    lib = L.lib()
    n = C.c_int64()
    L.check(lib.cdq_file_encode_header(n_states, len(tensors), None, 0, C.byref(n)), "encode header")
    hdr = np.empty(n.value, dtype=np.uint8)
    L.check(lib.cdq_file_encode_header(n_states, len(tensors), hdr.ctypes.data_as(C.c_void_p),
                                       hdr.size, C.byref(n)), "encode header")
    parts = [hdr.tobytes()]
    for name, t in tensors.items():
        rows, cols = int(t["rows"]), int(t["cols"])
        q = _u8(t["q"] if "q" in t else t["quant_indices"])
        sc = _u8(t["scales_f8_u8"] if "scales_f8_u8" in t else t["scales_f8"])
        ri, rv = _flat_residuals(t)
        args = (name.encode(), rows, cols, n_states, q.ctypes.data_as(C.c_void_p),
                sc.ctypes.data_as(C.c_void_p),
                ri.ctypes.data_as(C.c_void_p) if ri.size else None,
                rv.ctypes.data_as(C.c_void_p) if rv.size else None, ri.size)
        L.check(lib.cdq_file_encode_tensor(*args, None, 0, C.byref(n)), f"encode {name}")
        buf = np.empty(n.value, dtype=np.uint8)
        L.check(lib.cdq_file_encode_tensor(*args, buf.ctypes.data_as(C.c_void_p), buf.size,
                                           C.byref(n)), f"encode {name}")
        parts.append(buf.tobytes())
    return b"".join(parts)


def write_cdq(path, tensors: dict, n_states: int = 26) -> None:
    """tensors: {name: dict(rows, cols, scales_f8_u8[N,1], q[N,32] u8,
    tag_counts[N] u8, res_blobs[list])} as in code/cdq_pack.py:162-190, or
    with residual_indices / residual_values in place of the per-tile blobs."""
    data = encode_cdq(tensors, n_states)
    with open(path, "wb") as f:
        f.write(data)


def scan_cdq(data: bytes) -> tuple[int, list]:
    lib = L.lib()
    buf = np.frombuffer(data, dtype=np.uint8)
    ns, cnt = C.c_int32(), C.c_int32()
    L.check(lib.cdq_file_scan(buf.ctypes.data_as(C.c_void_p), buf.size, C.byref(ns), None, 0,
                              C.byref(cnt)), "cdq_file_scan")
    tabs = (L.cdq_file_tensor * max(cnt.value, 1))()
    L.check(lib.cdq_file_scan(buf.ctypes.data_as(C.c_void_p), buf.size, C.byref(ns), tabs,
                              cnt.value, C.byref(cnt)), "cdq_file_scan")
    return ns.value, [tabs[i] for i in range(cnt.value)]


def decode_tensor(data: bytes, n_states: int, t) -> dict:
    """One scanned tensor -> reference pack arrays (numpy)."""
    buf = np.frombuffer(data, dtype=np.uint8)
    q = np.empty((t.n_tiles, TILE), dtype=np.uint8)
    sc = np.empty(t.n_tiles, dtype=np.uint8)
    ri = np.empty(t.n_res, dtype=np.int64)
    rv = np.empty(t.n_res, dtype=np.uint16)
    L.check(L.lib().cdq_file_decode(
        buf.ctypes.data_as(C.c_void_p), buf.size, n_states, C.byref(t),
        q.ctypes.data_as(C.c_void_p), sc.ctypes.data_as(C.c_void_p),
        ri.ctypes.data_as(C.c_void_p) if ri.size else None,
        rv.ctypes.data_as(C.c_void_p) if rv.size else None), f"decode {t.name.decode()}")
    return {"quant_indices": q, "scales_f8": sc, "residual_indices": ri, "residual_values": rv}


SPAN_TILES = 256  # tiles per device decode thread


def decode_tensor_device(data: bytes, n_states: int, t, device="cuda") -> dict:
    """One scanned tensor -> reference pack arrays on a CUDA device: a host pass
    over the records' count bytes finds where every 256-tile span starts
    (cdq_file_checkpoints), the records go to the device once, and one thread
    per span unpacks it (cdq_file_decode_device). Same arrays as decode_tensor."""
    buf = np.frombuffer(data, dtype=np.uint8)
    spans = -(-int(t.n_tiles) // SPAN_TILES)
    boff = np.empty(spans, dtype=np.int64)
    roff = np.empty(spans, dtype=np.int64)
    L.check(L.lib().cdq_file_checkpoints(buf.ctypes.data_as(C.c_void_p), buf.size, n_states, C.byref(t),
                                         SPAN_TILES, boff.ctypes.data_as(C.c_void_p),
                                         roff.ctypes.data_as(C.c_void_p)), f"checkpoints {t.name.decode()}")
    dev = torch.device(device)
    rec = torch.from_numpy(buf[t.record_offset:t.record_offset + t.record_bytes].copy()).to(dev)
    boff_d, roff_d = torch.from_numpy(boff).to(dev), torch.from_numpy(roff).to(dev)
    q = torch.empty((t.n_tiles, TILE), dtype=torch.uint8, device=dev)
    sc = torch.empty(t.n_tiles, dtype=torch.uint8, device=dev)
    ri = torch.empty(t.n_res, dtype=torch.int64, device=dev)
    rv = torch.empty(t.n_res, dtype=torch.int16, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        L.check(L.lib().cdq_file_decode_device(
            rec.data_ptr(), t.record_bytes, n_states, t.n_tiles, t.n_res, SPAN_TILES, boff_d.data_ptr(),
            roff_d.data_ptr(), q.data_ptr(), sc.data_ptr(), ri.data_ptr() if t.n_res else None,
            rv.data_ptr() if t.n_res else None, err.data_ptr(), torch.cuda.current_stream(dev).cuda_stream),
            f"device decode {t.name.decode()}")
    if int(err.item()):
        raise L.CdqError(5, f"device decode {t.name.decode()}")
    return {"quant_indices": q, "scales_f8": sc, "residual_indices": ri, "residual_values": rv}


def read_cdq(path) -> dict:
    """code/cdq_pack.py:193-234: {name: {rows, cols, n_tiles, scales_f8_u8, q,
    tag_counts, res_blobs, n_states}}."""
    with open(path, "rb") as f:
        data = f.read()
    assert data[:4] == MAGIC, "bad magic"
    (ver,) = struct.unpack_from("<H", data, 4)
    assert ver in (VERSION, VERSION2), f"unsupported version {ver}"
    n_states, tabs = scan_cdq(data)
    ib = IDX_BYTES_PER_TILE if n_states == 26 else NIBBLE_BYTES_PER_TILE
    out = {}
    raw = np.frombuffer(data, dtype=np.uint8)
    for t in tabs:
        d = decode_tensor(data, n_states, t)
        nt = int(t.n_tiles)
        base = int(t.record_offset)
        tags = raw[base + 1: base + 1 + 1]  # placeholder, rebuilt below
        # walk the records once with numpy: record length = 2 + ib + blob
        tc = np.bincount(d["residual_indices"] // TILE, minlength=nt).astype(np.int64)
        blen = (tc * 21 + 7) // 8
        roff = base + np.concatenate([[0], np.cumsum(2 + ib + blen)[:-1]])
        boff = roff + 2 + ib
        blobs = [bytes(data[o:o + n]) for o, n in zip(boff.tolist(), blen.tolist())]
        tags = tc.astype(np.uint8)
        out[t.name.decode()] = {
            "rows": int(t.rows), "cols": int(t.cols), "n_tiles": nt,
            "scales_f8_u8": torch.from_numpy(d["scales_f8"].reshape(nt, 1).copy()),
            "q": torch.from_numpy(d["quant_indices"]),
            "tag_counts": torch.from_numpy(tags),
            "res_blobs": blobs,
            "n_states": n_states,
        }
    return out


def read_device_packs(path, device="cuda") -> dict[str, DevicePack]:
    """Each tensor of a .cdq file straight to a device pack."""
    with open(path, "rb") as f:
        data = f.read()
    n_states, tabs = scan_cdq(data)
    out = {}
    for t in tabs:
        if torch.device(device).type == "cuda":  # the records are unpacked and converted on the GPU
            d = decode_tensor_device(data, n_states, t, device)
            out[t.name.decode()] = DevicePack.from_reference_device(
                d["quant_indices"], d["scales_f8"], d["residual_indices"], d["residual_values"],
                int(t.rows), int(t.cols), n_states)
            continue
        d = decode_tensor(data, n_states, t)
        out[t.name.decode()] = DevicePack.from_reference(
            d["quant_indices"], d["scales_f8"], d["residual_indices"], d["residual_values"],
            int(t.rows), int(t.cols), n_states, device=device)
    return out


def dequant_tile(q32, scale_bf16, res_blob, tag_count, lattice=None):
    """One tile -> 32 bf16 values (code/cdq_pack.py:237-248)."""
    from .quant import CAMKII_LATTICE
    lat = CAMKII_LATTICE if lattice is None else lattice
    w = lat[torch.as_tensor(q32).long()].to(torch.bfloat16) * scale_bf16
    if tag_count:
        offs, vals = unpack_residuals(res_blob, int(tag_count))
        w[offs.long()] = vals.to(torch.bfloat16)
    return w


def main(argv=None):
    import argparse
    import os
    import time
    from .ops import quantize
    ap = argparse.ArgumentParser(description="quantise a safetensors checkpoint to .cdq on the GPU")
    ap.add_argument("--model", default=os.environ.get("CDQ_MODEL", "models/qwen-local"))
    ap.add_argument("--out", default="qwen05.cdq")
    ap.add_argument("--max-tensors", type=int, default=-1, help="-1 = all")
    ap.add_argument("--states", type=int, choices=(26, 16), default=16)
    ap.add_argument("--stc-frac", type=float, default=0.0156)
    ap.add_argument("--no-topk-guard", action="store_true",
                    help="quantize exactly as the reference packer CLI (no top-k tie guard, "
                         "code/cdq_pack.py:279-291); by default the guard of quantize_cdq_lrr applies")
    args = ap.parse_args(argv)
    from safetensors import safe_open
    f = safe_open(os.path.join(args.model, "model.safetensors"), framework="pt")
    keys = [k for k in f.keys() if k.endswith(".weight") and any(
        s in k for s in ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj"))]
    if args.max_tensors > 0:
        keys = keys[:args.max_tensors]
    print(f"lattice: {args.states}-state ({5 if args.states == 26 else 4}-bit indices)")
    print(f"packing {len(keys)} tensors ...")
    t0 = time.time()
    tensors, tot_w, tot_res = {}, 0, 0
    for k in keys:
        w = f.get_tensor(k).to(torch.bfloat16).cuda()
        pack, info = quantize(w, n_states=args.states, stc_frac=args.stc_frac,
                              topk_guard=not args.no_topk_guard)
        ref = pack.to_reference()
        rows, cols = w.shape
        tensors[k] = {"rows": rows, "cols": cols, "q": ref["quant_indices"],
                      "scales_f8_u8": ref["scales_f8"], "residual_indices": ref["residual_indices"],
                      "residual_values": ref["residual_values"]}
        tot_w += w.numel()
        tot_res += info["n_res"]
    write_cdq(args.out, tensors, n_states=args.states)
    size = os.path.getsize(args.out)
    print(f"wrote {args.out} ({size / 1e6:.1f} MB) in {time.time() - t0:.1f}s")
    print(f"params={tot_w} residuals={tot_res} ({100 * tot_res / max(1, tot_w):.2f}%)")
    print(f"on-disk = {size * 8 / max(1, tot_w):.3f} bpw")


if __name__ == "__main__":
    main()
