"""The C-ABI library on the host: it loads, exports every declared symbol, and
its host-side conversions and .cdq codec agree with the oracle and with the
reference CLI's files byte for byte. No GPU needed."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import cdq_oracle as O

ROOT = Path(__file__).resolve().parent.parent
GOLD = ROOT / "tests" / "golden"


@pytest.fixture(scope="module")
def L():
    from cdq_lrr_b200 import _lib
    _lib.lib()
    return _lib


def test_library_exports_every_declared_symbol(L):
    header = (ROOT / "include" / "cdq.h").read_text()
    declared = set(re.findall(r"CDQ_API\s+(?:const\s+)?\w+\*?\s+\**(cdq_\w+)\s*\(", header))
    assert declared, "no declarations found"
    lib = L.lib()
    for name in sorted(declared):
        assert hasattr(lib, name), name
    assert declared == set(L.exported_symbols())


def test_version(L):
    assert b"sm_100a" in L.lib().cdq_version()


def test_sizes_and_errors(L):
    s = L.sizes(4864, 896, 26)
    assert s.row_blocks == 304 and s.tile_pairs == 14 and s.res_groups == 1
    assert s.units_bytes == 304 * 14 * 672
    assert L.sizes(896, 4864, 16).units_bytes == 56 * 76 * 544
    assert s.max_res == 2 * round(4864 * 896 * 0.0156)
    out = L.cdq_sizes()
    lib = L.lib()
    assert lib.cdq_get_sizes(4864, 900, 26, 0.0156, 1, C.byref(out)) == 1   # cols % 32
    assert lib.cdq_get_sizes(4864, 896, 25, 0.0156, 1, C.byref(out)) == 2   # states
    assert lib.cdq_get_sizes(4864, 896, 26, 0.0156, 65, C.byref(out)) == 3  # batch
    assert lib.cdq_get_sizes(16, 65568, 26, 0.0156, 1, C.byref(out)) == 1   # > 65536 cols


CASES = ["small26", "small16", "rect26", "frac03125", "frac50", "onetile", "zeros",
         "constant", "zerotiles", "tiny", "huge", "wide16", "mid26"]


@pytest.mark.parametrize("name", CASES)
def test_host_layout_round_trip(L, golden, golden_meta, name):
    """reference pack -> device layout (host) -> reference pack is the identity."""
    from cdq_lrr_b200.ops import DevicePack
    meta = golden_meta["cases"][name]
    w = golden[f"{name}.weight"]
    rows, cols = w.shape
    q = golden[f"{name}.quant_indices"]
    sc = golden[f"{name}.scales_f8"]
    ri = golden[f"{name}.residual_indices"]
    rv = golden[f"{name}.residual_values"]
    dp = DevicePack.from_reference(q, sc, ri, rv, rows, cols, meta["n_states"])
    back = dp.to_reference()
    assert np.array_equal(back["quant_indices"], q)
    assert np.array_equal(back["scales_f8"], sc)
    assert np.array_equal(back["residual_indices"], ri)
    assert np.array_equal(back["residual_values"], rv)
    # the reference .cdq byte count from the device pack equals the file's records
    p = O.quantize(w, n_states=meta["n_states"], stc_frac=meta["stc_frac"])
    assert dp.reference_bytes() == O.tile_records(p, meta["n_states"]).size


def test_ragged_rows_layout(L):
    """rows not a multiple of 32: the padding rows of the last row block."""
    from cdq_lrr_b200.ops import DevicePack
    from cdq_lrr_b200.synth import synth_weight
    w = synth_weight(45, 96, seed=3).view(torch.int16).numpy().view(np.uint16)
    p = O.quantize(w)
    dp = DevicePack.from_reference(p["quant_indices"], p["scales_f8"], p["residual_indices"],
                                   p["residual_values"], 45, 96, 26)
    back = dp.to_reference()
    assert np.array_equal(back["quant_indices"], p["quant_indices"])
    assert np.array_equal(back["residual_indices"], p["residual_indices"])


def test_bad_reference_input_rejected(L):
    from cdq_lrr_b200.ops import DevicePack
    from cdq_lrr_b200 import CdqError
    q = np.zeros((2, 32), dtype=np.uint8)
    sc = np.zeros(2, dtype=np.uint8)
    with pytest.raises(CdqError):   # index beyond the lattice
        DevicePack.from_reference(np.full((2, 32), 26, np.uint8), sc, [], [], 1, 64, 26)
    with pytest.raises(CdqError):   # residual indices not ascending
        DevicePack.from_reference(q, sc, np.array([5, 3]), np.array([1, 2], np.uint16), 1, 64, 26)
    with pytest.raises(CdqError):   # residual index out of range
        DevicePack.from_reference(q, sc, np.array([64]), np.array([1], np.uint16), 1, 64, 26)


@pytest.mark.parametrize("states", [26, 16])
def test_file_codec_matches_reference_cli(L, golden_meta, states):
    """Decode the reference CLI's file with the C codec and re-encode it byte for byte."""
    from cdq_lrr_b200 import pack_file as PF
    data = (GOLD / f"cli_{states}.cdq").read_bytes()
    rd = O.read_cdq(data)
    ns, tabs = PF.scan_cdq(data)
    assert ns == states and len(tabs) == len(rd)
    tensors = {}
    for t in tabs:
        name = t.name.decode()
        d = PF.decode_tensor(data, ns, t)
        ref = O.pack_from_records(rd[name])
        assert np.array_equal(d["quant_indices"], ref["quant_indices"])
        assert np.array_equal(d["scales_f8"], ref["scales_f8"])
        assert np.array_equal(d["residual_indices"], ref["residual_indices"])
        assert np.array_equal(d["residual_values"], ref["residual_values"])
        tensors[name] = {"rows": t.rows, "cols": t.cols, "q": d["quant_indices"],
                         "scales_f8_u8": d["scales_f8"], "residual_indices": d["residual_indices"],
                         "residual_values": d["residual_values"]}
    assert PF.encode_cdq(tensors, states) == data


def test_read_write_cdq_reference_dicts(L, tmp_path):
    """read_cdq / write_cdq with the reference's per-tile blob dicts."""
    from cdq_lrr_b200 import pack_file as PF
    src = GOLD / "cli_26.cdq"
    rd = PF.read_cdq(src)
    dst = tmp_path / "x.cdq"
    PF.write_cdq(dst, rd, n_states=26)
    assert dst.read_bytes() == src.read_bytes()
    ref = O.read_cdq(src.read_bytes())
    for name, t in rd.items():
        assert np.array_equal(t["q"].numpy(), ref[name]["q"])
        assert np.array_equal(t["tag_counts"].numpy(), ref[name]["tag_counts"])
        assert t["res_blobs"] == ref[name]["res_blobs"]


@pytest.mark.parametrize("cut", [3, 9, 70, -1, -7])
def test_truncated_or_corrupt_file_rejected(L, cut):
    from cdq_lrr_b200 import pack_file as PF
    from cdq_lrr_b200 import CdqError
    data = (GOLD / "cli_26.cdq").read_bytes()
    bad = data[:cut] if cut > 0 else data[:len(data) + cut]
    with pytest.raises((CdqError, AssertionError)):
        ns, tabs = PF.scan_cdq(bad)
        for t in tabs:
            PF.decode_tensor(bad, ns, t)


def test_corrupt_header_rejected(L):
    from cdq_lrr_b200 import pack_file as PF
    from cdq_lrr_b200 import CdqError
    data = bytearray((GOLD / "cli_26.cdq").read_bytes())
    data[4] = 7  # version
    with pytest.raises(CdqError):
        PF.scan_cdq(bytes(data))
    data = bytearray((GOLD / "cli_26.cdq").read_bytes())
    data[0] = ord("X")
    with pytest.raises(CdqError):
        PF.scan_cdq(bytes(data))


def test_bit_packers_mirror_reference(L):
    from cdq_lrr_b200 import pack_file as PF
    rng = np.random.default_rng(0)
    q = rng.integers(0, 26, (8, 32)).astype(np.uint8)
    for row in q:
        b = PF.pack_5bit_row(torch.from_numpy(row))
        assert b == O.pack_5bit(row[None])[0].tobytes()
        assert np.array_equal(PF.unpack_5bit_row(b).numpy(), row)
    q16 = rng.integers(0, 16, (8, 32)).astype(np.uint8)
    for row in q16:
        b = PF.pack_indices_nibble(torch.from_numpy(row))
        assert b == O.pack_nibble(row[None])[0].tobytes()
        assert np.array_equal(PF.unpack_nibble_row(b).numpy(), row)
    offs = torch.tensor([1, 7, 30], dtype=torch.uint8)
    vals = torch.tensor([0.5, -2.0, 3e-3], dtype=torch.bfloat16)
    blob = PF.pack_residuals(offs, vals)
    o2, v2 = PF.unpack_residuals(blob, 3)
    assert o2.tolist() == offs.tolist()
    assert torch.equal(v2.view(torch.int16), vals.view(torch.int16))
    ob, vb = O.pack_residual_blobs(np.array([3]), offs.numpy(), vals.view(torch.int16).numpy().view(np.uint16))
    assert ob.tobytes() == blob


def test_device_ingest_argument_checks():
    """The device ingest entry point rejects bad shapes, lattices and null
    buffers before touching the GPU."""
    import ctypes as C
    from cdq_lrr_b200 import _lib as L
    lib = L.lib()
    st = L.cdq_packed()
    P = C.c_void_p(16)
    assert lib.cdq_pack_from_reference_device(4, 32, 25, P, P, None, None, 0, C.byref(st), P, None) == 2
    assert lib.cdq_pack_from_reference_device(4, 33, 26, P, P, None, None, 0, C.byref(st), P, None) == 1
    assert lib.cdq_pack_from_reference_device(4, 32, 26, None, P, None, None, 0, C.byref(st), P, None) == 3
    assert lib.cdq_pack_from_reference_device(4, 32, 26, P, P, None, None, 0, C.byref(st), None, None) == 3
    assert lib.cdq_pack_from_reference_device(4, 32, 26, P, P, None, None, 5, C.byref(st), P, None) == 3


def test_file_checkpoints_match_record_walk(L):
    """cdq_file_checkpoints gives, for every span of tiles, the byte offset and
    first residual index that a walk over the records finds; truncated records
    are refused."""
    import ctypes as C
    from cdq_lrr_b200 import pack_file as PF
    data = (GOLD / "cli_26.cdq").read_bytes()
    ns, tabs = PF.scan_cdq(data)
    buf = np.frombuffer(data, dtype=np.uint8)
    for every in (1, 3, 256):
        for t in tabs:
            spans = -(-int(t.n_tiles) // every)
            bo = np.empty(spans, np.int64)
            ro = np.empty(spans, np.int64)
            assert L.lib().cdq_file_checkpoints(buf.ctypes.data_as(C.c_void_p), buf.size, ns, C.byref(t), every,
                                                bo.ctypes.data_as(C.c_void_p), ro.ctypes.data_as(C.c_void_p)) == 0
            pos, n = 0, 0
            for k in range(int(t.n_tiles)):
                if k % every == 0:
                    assert bo[k // every] == pos and ro[k // every] == n
                tc = data[t.record_offset + pos + 1]
                pos += 2 + 20 + (tc * 21 + 7) // 8
                n += tc
            assert pos == t.record_bytes and n == t.n_res
    t = tabs[0]
    short = buf[: t.record_offset + t.record_bytes - 1].copy()
    bo = np.empty(int(t.n_tiles), np.int64)
    ro = np.empty(int(t.n_tiles), np.int64)
    assert L.lib().cdq_file_checkpoints(short.ctypes.data_as(C.c_void_p), short.size, ns, C.byref(t), 1,
                                        bo.ctypes.data_as(C.c_void_p), ro.ctypes.data_as(C.c_void_p)) == 5


def test_compare_stats_argument_checks(L):
    """The quality reduction rejects bad arguments before any device work."""
    import ctypes as C
    P = C.c_void_p(64)
    assert L.lib().cdq_compare_stats(None, P, 10, 0, P, P, 1 << 20, None) == 3
    assert L.lib().cdq_compare_stats(P, P, 10, 2, P, P, 1 << 20, None) == 3
    assert L.lib().cdq_compare_stats(P, P, 0, 0, P, P, 1 << 20, None) == 3
    assert L.lib().cdq_compare_stats(P, P, 10, 0, P, P, 1024, None) == 7
