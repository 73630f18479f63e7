"""CPU oracle for the CDQ-LRR decode path.

TEST INFRASTRUCTURE ONLY. This module restates, in numpy, the reference's
algorithm for the quantize -> pack -> dequantize -> linear path so that the
CUDA implementation can be checked against it. Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it, and only as the checker or the timed CPU
baseline. The product (``cdq_lrr_b200``) never calls it.

Pinning: every function here is checked against golden vectors produced by
running the reference Python itself (``tests/golden/make_golden.py`` imports
``code/cdq_lrr_qwen05.py``, ``code/cdq_pack.py`` and ``code/cdq_loader.py``
and records their outputs; ``tests/test_oracle_golden.py`` compares). The
reference has no tests or fixtures of its own, so those recorded outputs are
the pin.

Arithmetic follows the reference's torch 2.x CPU semantics, established by
probing torch 2.11 and then pinned by the fixtures:

* per-tile variance: unbiased, accumulated by a sequential Welford recurrence
  in float64 and rounded once to float32 (torch's CPU ``var`` reduction);
* ``torch.quantile(..., interpolation='linear')``: float32 rank
  ``q_f32 * (n - 1)`` rounded to float32, then a fused-multiply-add lerp
  between the two neighbouring order statistics;
* float32 division, subtraction and absolute value with IEEE round to
  nearest even, no contraction;
* ``argmin``: first index of the minimum, NaN counts as the minimum;
* float8 e4m3fn conversion: round to nearest even; magnitudes that round to
  480 or more, and NaN, become the NaN code 0x7F (sign kept);
* bf16 products: the exact float32 product rounded to nearest even.
"""
from __future__ import annotations

import math
import struct

import numpy as np

TILE = 32

# Decimal lattice literals, code/cdq_lrr_qwen05.py:27-32 (26 states) and
# :39-44 (16 states, zero-clamped, code 15 duplicates code 14). The reference
# builds them with torch.tensor(..., dtype=bfloat16); the bf16 bits used here
# are those decimals rounded to float32 and then to bf16 (pinned by fixture).
LATTICE26_DEC = (
    -1.0000, -0.7321, -0.5284, -0.3752, -0.2612, -0.1774, -0.1167, -0.0734,
    -0.0432, -0.0229, -0.0101, -0.0031, -0.0005, 0.0005, 0.0031, 0.0101,
    0.0229, 0.0432, 0.0734, 0.1167, 0.1774, 0.2612, 0.3752, 0.5284,
    0.7321, 1.0000,
)
LATTICE16_DEC = (
    -0.9685, -0.7525, -0.5834, -0.4414, -0.3174, -0.2048, -0.0998,
    0.0000,
    0.0998, 0.2048, 0.3174, 0.4414, 0.5834, 0.7525, 0.9685,
    0.9685,
)
STC_FRAC = 0.0156  # code/cdq_lrr_qwen05.py:25

# ---------------------------------------------------------------- bf16 helpers


def f32_to_bf16_bits(x) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even; NaN -> 0x7FC0."""
    f = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = f.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    r = r.astype(np.uint16)
    r[np.isnan(f)] = 0x7FC0
    return r


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def lattice_bits(n_states: int) -> np.ndarray:
    if n_states == 26:
        dec = LATTICE26_DEC
    elif n_states == 16:
        dec = LATTICE16_DEC
    else:
        raise ValueError(f"unsupported lattice size {n_states}")
    return f32_to_bf16_bits(np.array(dec, dtype=np.float32))


# ------------------------------------------------------------ float8 e4m3fn


def fp8_e4m3fn_encode(x) -> np.ndarray:
    """float32 values -> e4m3fn codes (uint8), round to nearest even.

    Grid: subnormals m*2^-9 (m = 0..7), normals (1 + m/8)*2^(e-7) for
    e = 1..15; code 0x7F / 0xFF is NaN, so 448 is the largest finite value
    and anything that rounds to 480 or beyond saturates to NaN.
    Used by code/cdq_lrr_qwen05.py:52 (``.to(torch.float8_e4m3fn)``).
    """
    f = np.asarray(x, dtype=np.float32).astype(np.float64)
    sign = np.signbit(f)
    a = np.abs(f)
    code = np.zeros(a.shape, dtype=np.int64)
    nan = np.isnan(a) | np.isinf(a)
    a_ = np.where(nan, 0.0, a)
    small = a_ < 2.0 ** -6
    # subnormal range: quantum 2^-9 (rounds up into the first normal cleanly)
    q_sub = np.round(a_ / 2.0 ** -9)  # numpy rounds half to even
    # normal range
    m, e = np.frexp(np.where(small, 1.0, a_))  # a = m * 2^e, m in [0.5, 1)
    e = e - 1  # a = (2m) * 2^(e)
    frac = (2.0 * m - 1.0) * 8.0
    q = np.round(frac)
    carry = q >= 8
    q = np.where(carry, 0, q)
    e = np.where(carry, e + 1, e)
    code_n = ((e + 7) << 3) | q.astype(np.int64)
    code = np.where(small, q_sub.astype(np.int64), code_n)
    over = (~small) & ((e + 7 > 15) | (code_n >= 0x7F))
    code = np.where(over | nan, 0x7F, code)
    code = code | np.where(sign, 0x80, 0)
    return code.astype(np.uint8)


def fp8_e4m3fn_decode(c) -> np.ndarray:
    """e4m3fn codes -> float32 (exact); 0x7F/0xFF -> NaN."""
    c = np.asarray(c, dtype=np.uint8).astype(np.int64)
    s = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 7
    v = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    v = np.where((c & 0x7F) == 0x7F, np.nan, v)
    return (s * v).astype(np.float32)


# -------------------------------------------------------------- statistics


def tile_var_f32(x: np.ndarray) -> np.ndarray:
    """Unbiased variance of each row of ``x`` [N, 32] (float32 values).

    Restates ``torch.var(flat.float(), dim=1)`` (code/cdq_lrr_qwen05.py:87;
    code/cdq_pack.py:286): a sequential Welford recurrence in float64,
    m2 / (n - 1), rounded to float32.
    """
    xd = np.asarray(x, dtype=np.float32).astype(np.float64)
    n_t, t = xd.shape
    mean = np.zeros(n_t)
    m2 = np.zeros(n_t)
    for i in range(t):
        d = xd[:, i] - mean
        mean = mean + d / float(i + 1)
        m2 = m2 + d * (xd[:, i] - mean)
    return (m2 / float(t - 1)).astype(np.float32)


def _fma_f32(a: float, b: float, c: float) -> np.float32:
    """Single-rounded float32 a*b + c, exact via rationals."""
    from fractions import Fraction
    a32, b32, c32 = (np.float32(v) for v in (a, b, c))
    if not all(np.isfinite(v) for v in (a32, b32, c32)):
        return np.float32(a32 * b32 + c32)
    ex = Fraction(float(a32)) * Fraction(float(b32)) + Fraction(float(c32))
    r = np.float32(float(ex))
    best = r
    for cand in (np.nextafter(r, np.float32(np.inf)), np.nextafter(r, np.float32(-np.inf))):
        da, db = abs(Fraction(float(cand)) - ex), abs(Fraction(float(best)) - ex)
        if da < db or (da == db and (int(cand.view(np.uint32)) & 1) == 0):
            best = cand
    return np.float32(best)


def quantile_rank(n: int, q: float) -> tuple[int, int, np.float32]:
    """(lower index, upper index, lerp weight) of torch.quantile's linear rule."""
    qf = np.float32(q)
    r = np.float32(qf * np.float32(n - 1))
    lo = int(math.floor(float(r)))
    hi = int(math.ceil(float(r)))
    w = np.float32(r - np.float32(lo))
    return lo, hi, w


def lerp_f32(a: np.float32, b: np.float32, w: np.float32) -> np.float32:
    """torch's lerp: w < 0.5 ? fma(w, b-a, a) : fma(w-1, b-a, b)."""
    diff = np.float32(np.float32(b) - np.float32(a))
    if abs(float(w)) < 0.5:
        return _fma_f32(w, diff, a)
    return _fma_f32(np.float32(w - np.float32(1.0)), diff, b)


def quantile_linear(values: np.ndarray, q: float) -> np.float32:
    """Restates torch.quantile(values, q) (linear interpolation, float32).

    Used at code/cdq_lrr_qwen05.py:90 and code/cdq_pack.py:288. torch refuses
    inputs above 2**24 elements; beyond that size this restatement keeps the
    same float32 rank rule, which is this implementation's convention. Any
    NaN input makes the result NaN, as in torch (then no weight reaches the
    threshold and the tensor keeps no residuals).
    """
    v = np.sort(np.asarray(values, dtype=np.float32).ravel())
    if np.isnan(v[-1]):
        return np.float32(np.nan)  # torch propagates NaN through quantile
    lo, hi, w = quantile_rank(v.size, q)
    return lerp_f32(v[lo], v[hi], w)


# --------------------------------------------------------------- quantizer


def quantize(w_bits: np.ndarray, n_states: int = 26, stc_frac: float | None = None,
             chunk_tiles: int = 16384, topk_guard: bool = True) -> dict:
    """Restates quantize_cdq_lrr (code/cdq_lrr_qwen05.py:63-133).

    ``topk_guard=False`` restates the packer CLI's inline quantizer instead
    (code/cdq_pack.py:279-291): the same steps without the top-k tie guard,
    so every weight whose saliency reaches the threshold is a residual.

    ``w_bits``: uint16 bf16 bits [rows, cols], cols % 32 == 0. Returns numpy
    arrays with the reference pack's keys (bf16 tensors as uint16 bits, fp8 as
    uint8 codes) plus ``topk_fallback`` (True when the tie guard at :93-96
    replaced the quantile mask).
    """
    if stc_frac is None:
        stc_frac = STC_FRAC
    w_bits = np.ascontiguousarray(np.asarray(w_bits, dtype=np.uint16))
    assert w_bits.ndim == 2, "expected 2D"
    rows, cols = w_bits.shape
    assert (rows * cols) % TILE == 0
    flat_b = w_bits.reshape(-1, TILE)
    n_tiles = flat_b.shape[0]
    x = bf16_bits_to_f32(flat_b)  # exact

    # sigma = max|w| in bf16, clamp(min=1e-8): the clamp only ever lifts an
    # all-zero tile to bf16(1e-8), which encodes to fp8 0 like zero itself.
    absx = np.abs(x)
    with np.errstate(invalid="ignore"):
        sigma = absx.max(axis=1)
    sigma = np.where(np.isnan(sigma) | (sigma >= np.float32(1e-8)), sigma,
                     bf16_bits_to_f32(f32_to_bf16_bits(np.float32(1e-8))))
    scales_f8 = fp8_e4m3fn_encode(sigma)
    sigma_q = fp8_e4m3fn_decode(scales_f8)  # exact in bf16
    scales_bf16 = f32_to_bf16_bits(sigma_q)

    var = tile_var_f32(x)
    with np.errstate(invalid="ignore"):
        sal = absx * (var + np.float32(1e-6))[:, None]
    sal = sal.astype(np.float32)
    numel = sal.size
    k = max(1, int(round(numel * stc_frac)))
    thr = quantile_linear(sal, 1.0 - stc_frac)
    mask = sal >= thr
    topk_fallback = False
    if topk_guard and int(mask.sum()) > 2 * k:
        # torch.topk's choice among equal values is implementation defined;
        # torch 2.11 on CPU takes the lowest flat indices, restated here.
        topk_fallback = True
        fl = sal.ravel()
        order = np.lexsort((np.arange(fl.size), -fl.astype(np.float64)))
        mask = np.zeros(fl.size, dtype=bool)
        mask[order[:k]] = True
        mask = mask.reshape(sal.shape)

    res_idx = np.flatnonzero(mask.ravel()).astype(np.int64)
    res_val = flat_b.ravel()[res_idx].copy()

    lat = bf16_bits_to_f32(lattice_bits(n_states))
    q_out = np.empty((n_tiles, TILE), dtype=np.uint8)
    for s in range(0, n_tiles, chunk_tiles):
        e = min(s + chunk_tiles, n_tiles)
        with np.errstate(invalid="ignore", divide="ignore"):
            norm = (x[s:e] / sigma_q[s:e, None]).astype(np.float32)
            d = np.abs(norm[:, :, None] - lat[None, None, :]).astype(np.float32)
        q_out[s:e] = np.argmin(d, axis=-1).astype(np.uint8)  # first index; NaN first

    return {
        "quant_indices": q_out,
        "scales_f8": scales_f8,
        "scales_bf16": scales_bf16,
        "residual_indices": res_idx,
        "residual_values": res_val,
        "orig_shape": (rows, cols),
        "outlier_count": int(res_idx.size),
        "numel": int(numel),
        "n_tiles": int(n_tiles),
        "lattice": lattice_bits(n_states),
        "n_states": int(n_states),
        "topk_fallback": topk_fallback,
        "threshold": np.float32(thr),
    }


def dequantize(pack: dict) -> np.ndarray:
    """Restates dequantize (code/cdq_lrr_qwen05.py:141-152) -> bf16 bits [rows, cols].

    w_hat = bf16(LUT[q] * sigma_bf16) (exact float32 product rounded to
    nearest even), then residual positions take their stored bf16 values.
    NaN products are returned as 0x7FC0; the reference's own NaN bits vary
    with the position inside its vectorised loop, so tests compare NaN-ness.
    """
    lat = bf16_bits_to_f32(pack["lattice"])
    q = np.asarray(pack["quant_indices"]).astype(np.int64)
    s = bf16_bits_to_f32(pack["scales_bf16"]).reshape(-1, 1)
    with np.errstate(invalid="ignore"):
        w = f32_to_bf16_bits(lat[q] * s).ravel()
    ri = np.asarray(pack["residual_indices"], dtype=np.int64)
    if ri.size:
        w[ri] = np.asarray(pack["residual_values"], dtype=np.uint16)
    return w.reshape(pack["orig_shape"])


def linear_f64(w_hat_bits: np.ndarray, x_bits: np.ndarray, bias_bits=None) -> np.ndarray:
    """y = x @ w_hat^T (+ bias) in float64 from bf16 bits: the GEMV check value."""
    w = bf16_bits_to_f32(w_hat_bits).astype(np.float64)
    x = bf16_bits_to_f32(x_bits).astype(np.float64)
    y = x @ w.T
    if bias_bits is not None:
        y = y + bf16_bits_to_f32(bias_bits).astype(np.float64)
    return y


# ------------------------------------------------------------ .cdq codec


def pack_5bit(q: np.ndarray) -> np.ndarray:
    """[N, 32] codes 0..31 -> [N, 20] bytes, LSB-first (code/cdq_pack.py:50-56)."""
    q = np.asarray(q, dtype=np.uint8)
    bits = ((q[:, :, None] >> np.arange(5, dtype=np.uint8)) & 1).astype(np.uint8)
    return np.packbits(bits.reshape(q.shape[0], 160), axis=1, bitorder="little")


def unpack_5bit(b: np.ndarray) -> np.ndarray:
    """Inverse of pack_5bit (code/cdq_pack.py:59-65)."""
    b = np.asarray(b, dtype=np.uint8)
    bits = np.unpackbits(b, axis=1, bitorder="little").reshape(b.shape[0], 32, 5)
    return (bits * (1 << np.arange(5, dtype=np.uint8))).sum(axis=2).astype(np.uint8)


def pack_nibble(q: np.ndarray) -> np.ndarray:
    """[N, 32] codes 0..15 -> [N, 16] bytes, even lane in the low nibble (code/cdq_pack.py:68-78)."""
    q = np.asarray(q, dtype=np.uint8)
    return ((q[:, 0::2] & 0xF) | ((q[:, 1::2] & 0xF) << 4)).astype(np.uint8)


def unpack_nibble(b: np.ndarray) -> np.ndarray:
    """Inverse of pack_nibble (code/cdq_pack.py:81-88)."""
    b = np.asarray(b, dtype=np.uint8)
    out = np.empty((b.shape[0], 32), dtype=np.uint8)
    out[:, 0::2] = b & 0xF
    out[:, 1::2] = b >> 4
    return out


def residual_blob_len(tag_count) -> np.ndarray:
    """Bytes of a tile's residual stream: ceil(21 * tc / 8) (code/cdq_pack.py:104, cdq_loader.py:84)."""
    return (np.asarray(tag_count, dtype=np.int64) * 21 + 7) // 8


def tile_residuals(pack: dict):
    """Per-tile residual lists from a pack: (tag_counts [N], offsets [R], values [R], tile_of [R]).

    Mirrors the packer CLI's per-tile split (code/cdq_pack.py:293-299): the
    flat residual index ri gives tile ri // 32 and offset ri % 32.
    """
    ri = np.asarray(pack["residual_indices"], dtype=np.int64)
    tile_of = ri // TILE
    offs = (ri % TILE).astype(np.uint8)
    tags = np.bincount(tile_of, minlength=pack["n_tiles"]).astype(np.int64)
    return tags, offs, np.asarray(pack["residual_values"], dtype=np.uint16), tile_of


def pack_residual_blobs(tags: np.ndarray, offs: np.ndarray, vals: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """All tiles' residual streams back to back (code/cdq_pack.py:91-104).

    Returns (bytes uint8 [sum of blob lengths], byte offset of each tile's blob).
    Per entry: 5-bit offset then 16-bit bf16 bits, LSB-first, entries packed
    without padding, the tile's stream padded to a whole byte.
    """
    tags = np.asarray(tags, dtype=np.int64)
    blen = residual_blob_len(tags)
    boff = np.zeros(tags.size + 1, dtype=np.int64)
    np.cumsum(blen, out=boff[1:])
    total_bits = int(boff[-1]) * 8
    bits = np.zeros(total_bits, dtype=np.uint8)
    if offs.size:
        tile_of = np.repeat(np.arange(tags.size), tags)
        first = np.zeros(tags.size, dtype=np.int64)
        np.cumsum(tags[:-1], out=first[1:])
        j = np.arange(offs.size) - first[tile_of]
        base = boff[tile_of] * 8 + 21 * j
        ob = ((np.asarray(offs, dtype=np.uint32)[:, None] >> np.arange(5)) & 1).astype(np.uint8)
        vb = ((np.asarray(vals, dtype=np.uint32)[:, None] >> np.arange(16)) & 1).astype(np.uint8)
        bits[(base[:, None] + np.arange(5)).ravel()] = ob.ravel()
        bits[(base[:, None] + 5 + np.arange(16)).ravel()] = vb.ravel()
    return np.packbits(bits, bitorder="little"), boff


def unpack_residual_blob(blob: bytes, tag_count: int) -> tuple[list[int], list[int]]:
    """One tile's stream -> (offsets, bf16 bits) (code/cdq_pack.py:107-119)."""
    acc = int.from_bytes(bytes(blob), "little")
    offs, vals, pos = [], [], 0
    for _ in range(tag_count):
        offs.append((acc >> pos) & 0x1F)
        pos += 5
        vals.append((acc >> pos) & 0xFFFF)
        pos += 16
    return offs, vals


MAGIC = b"CDQ1"


def write_cdq(tensors: list[tuple[str, dict]], n_states: int) -> bytes:
    """Restates write_cdq (code/cdq_pack.py:162-190) -> file bytes.

    ``tensors``: (name, pack) pairs in file order; each pack carries
    orig_shape, n_tiles, scales_f8 (codes), quant_indices and the residual
    lists. Header: magic, u16 version (1 = 26 states, 2 = 16 states), u16
    tensor count, bf16 lattice. Per tensor: u16 name length, name, u32 rows,
    u32 cols, u32 n_tiles. Per tile: u8 fp8 scale, u8 tag count, 20 (v1) or
    16 (v2) index bytes, residual stream.
    """
    assert n_states in (26, 16)
    ver = 1 if n_states == 26 else 2
    out = bytearray(MAGIC)
    out += struct.pack("<HH", ver, len(tensors))
    out += lattice_bits(n_states).astype("<u2").tobytes()
    for name, p in tensors:
        rows, cols = p["orig_shape"]
        nb = name.encode()
        out += struct.pack("<H", len(nb)) + nb
        out += struct.pack("<III", rows, cols, p["n_tiles"])
        out += tile_records(p, n_states).tobytes()
    return bytes(out)


def tile_records(p: dict, n_states: int) -> np.ndarray:
    """The per-tile record stream of one tensor (scale, tag, indices, residuals)."""
    q = np.asarray(p["quant_indices"], dtype=np.uint8)
    idx = pack_5bit(q) if n_states == 26 else pack_nibble(q)
    ib = idx.shape[1]
    tags, offs, vals, _ = tile_residuals(p)
    blob, boff = pack_residual_blobs(tags, offs, vals)
    blen = np.diff(boff)
    rlen = 2 + ib + blen
    roff = np.zeros(tags.size + 1, dtype=np.int64)
    np.cumsum(rlen, out=roff[1:])
    buf = np.zeros(int(roff[-1]), dtype=np.uint8)
    buf[roff[:-1]] = np.asarray(p["scales_f8"], dtype=np.uint8).ravel()
    buf[roff[:-1] + 1] = tags.astype(np.uint8)
    buf[(roff[:-1, None] + 2 + np.arange(ib)).ravel()] = idx.ravel()
    if blob.size:
        t = np.repeat(np.arange(tags.size), blen)
        pos = np.arange(blob.size) - boff[t]
        buf[roff[t] + 2 + ib + pos] = blob
    return buf


def read_cdq(data: bytes) -> dict:
    """Restates read_cdq (code/cdq_pack.py:193-234): name -> dict of arrays."""
    p = 0
    assert data[0:4] == MAGIC, "bad magic"
    ver, n = struct.unpack_from("<HH", data, 4)
    assert ver in (1, 2), f"unsupported version {ver}"
    n_states = 26 if ver == 1 else 16
    p = 8 + (52 if ver == 1 else 32)
    ib = 20 if ver == 1 else 16
    out = {}
    for _ in range(n):
        (nl,) = struct.unpack_from("<H", data, p)
        p += 2
        name = bytes(data[p:p + nl]).decode()
        p += nl
        rows, cols, nt = struct.unpack_from("<III", data, p)
        p += 12
        scales = np.empty(nt, dtype=np.uint8)
        tags = np.empty(nt, dtype=np.uint8)
        idx = np.empty((nt, ib), dtype=np.uint8)
        blobs = []
        mv = memoryview(data)
        for i in range(nt):
            scales[i] = data[p]
            tc = data[p + 1]
            tags[i] = tc
            idx[i] = np.frombuffer(mv[p + 2:p + 2 + ib], dtype=np.uint8)
            p += 2 + ib
            nb_ = (tc * 21 + 7) // 8
            blobs.append(bytes(mv[p:p + nb_]))
            p += nb_
        q = unpack_5bit(idx) if ver == 1 else unpack_nibble(idx)
        out[name] = {"rows": rows, "cols": cols, "n_tiles": nt, "scales_f8_u8": scales,
                     "q": q, "tag_counts": tags, "res_blobs": blobs, "n_states": n_states}
    return out


def pack_from_records(rec: dict) -> dict:
    """A read_cdq tensor record -> pack dict (flat residual indices as in the
    loader, code/cdq_loader.py:94-100: index = tile * 32 + offset)."""
    offs_all, vals_all = [], []
    for ti, (tc, blob) in enumerate(zip(rec["tag_counts"], rec["res_blobs"])):
        if tc:
            o, v = unpack_residual_blob(blob, int(tc))
            offs_all += [ti * TILE + oo for oo in o]
            vals_all += v
    n_states = rec["n_states"]
    return {
        "quant_indices": rec["q"],
        "scales_f8": np.asarray(rec["scales_f8_u8"], dtype=np.uint8).ravel(),
        "scales_bf16": f32_to_bf16_bits(fp8_e4m3fn_decode(rec["scales_f8_u8"])).ravel(),
        "residual_indices": np.array(offs_all, dtype=np.int64),
        "residual_values": np.array(vals_all, dtype=np.uint16),
        "orig_shape": (rec["rows"], rec["cols"]),
        "n_tiles": rec["n_tiles"],
        "numel": rec["rows"] * rec["cols"],
        "outlier_count": len(offs_all),
        "lattice": lattice_bits(n_states),
        "n_states": n_states,
    }
