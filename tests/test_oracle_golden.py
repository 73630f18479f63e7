"""The CPU oracle against golden vectors recorded from the reference itself.

tests/golden/make_golden.py ran the reference Python (quantize_cdq_lrr,
dequantize, CDQLinear.forward, the cdq_pack.py CLI, read_cdq and load_cdq) and
stored what it returned. Every oracle function used as a checker elsewhere is
pinned here, bit for bit.
"""
import hashlib

import numpy as np
import pytest
import torch

from oracle import cdq_oracle as O
from cdq_lrr_b200.synth import synth_activation, synth_weight

CASES = ["small26", "small16", "rect26", "frac03125", "frac50", "onetile", "zeros",
         "constant", "zerotiles", "tiny", "huge", "wide16", "mid26", "nanweight", "infweight"]


def _nan_equal_bf16(a, b):
    a = np.asarray(a, dtype=np.uint16)
    b = np.asarray(b, dtype=np.uint16)
    an = (a & 0x7F80) == 0x7F80
    an &= (a & 0x7F) != 0
    bn = (b & 0x7F80) == 0x7F80
    bn &= (b & 0x7F) != 0
    return bool(np.array_equal(an, bn) and np.array_equal(a[~an], b[~bn]))


def _digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_lattice_bits(golden):
    assert np.array_equal(O.lattice_bits(26), golden["lattice26"])
    assert np.array_equal(O.lattice_bits(16), golden["lattice16"])


def test_fp8_encode_every_bf16(golden):
    allbf = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = O.fp8_e4m3fn_encode(O.bf16_bits_to_f32(allbf))
    assert np.array_equal(got, golden["fp8_encode_all_bf16"])


def test_fp8_scale_round_trip_every_bf16(golden):
    allbf = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    got = O.f32_to_bf16_bits(O.fp8_e4m3fn_decode(O.fp8_e4m3fn_encode(O.bf16_bits_to_f32(allbf))))
    assert _nan_equal_bf16(got, golden["fp8_scale_all_bf16"])


def test_fp8_decode_every_code(golden):
    got = O.f32_to_bf16_bits(O.fp8_e4m3fn_decode(np.arange(256, dtype=np.uint8)))
    assert _nan_equal_bf16(got, golden["fp8_decode_all"])


@pytest.mark.parametrize("name", CASES)
def test_quantize_matches_reference(golden, golden_meta, name):
    meta = golden_meta["cases"][name]
    p = O.quantize(golden[f"{name}.weight"], n_states=meta["n_states"], stc_frac=meta["stc_frac"])
    assert np.array_equal(p["quant_indices"], golden[f"{name}.quant_indices"])
    assert np.array_equal(p["scales_f8"], golden[f"{name}.scales_f8"])
    assert _nan_equal_bf16(p["scales_bf16"], golden[f"{name}.scales_bf16"])
    assert np.array_equal(p["residual_indices"], golden[f"{name}.residual_indices"])
    assert np.array_equal(p["residual_values"], golden[f"{name}.residual_values"])
    assert p["outlier_count"] == meta["outlier_count"]


@pytest.mark.parametrize("name", CASES)
def test_dequantize_matches_reference(golden, golden_meta, name):
    meta = golden_meta["cases"][name]
    p = O.quantize(golden[f"{name}.weight"], n_states=meta["n_states"], stc_frac=meta["stc_frac"])
    assert _nan_equal_bf16(O.dequantize(p), golden[f"{name}.w_hat"])


@pytest.mark.parametrize("name", CASES)
def test_linear_matches_reference(golden, golden_meta, name):
    """The fp64 dot of the oracle's w_hat, rounded to bf16, is within one bf16
    rounding of the reference's F.linear output (which accumulates in float32
    in an order of its own)."""
    meta = golden_meta["cases"][name]
    p = O.quantize(golden[f"{name}.weight"], n_states=meta["n_states"], stc_frac=meta["stc_frac"])
    what = O.dequantize(p)
    for m in (1, 3):
        y64 = O.linear_f64(what, golden[f"{name}.x{m}"], golden[f"{name}.bias"])
        yref = O.bf16_bits_to_f32(golden[f"{name}.y{m}"]).astype(np.float64)
        fin = np.isfinite(y64)
        assert np.array_equal(fin, np.isfinite(yref))
        err = np.abs(y64[fin] - yref[fin])
        assert np.all(err <= 2.0 ** -7 * np.abs(y64[fin]) + 1e-30), float(err.max())


def test_packer_cli_files_round_trip(golden, golden_meta):
    """read_cdq restatement on the reference CLI's files, and write_cdq
    restatement reproducing those files byte for byte."""
    from pathlib import Path
    gdir = Path(__file__).parent / "golden"
    cases = {nm: None for _, nm in golden_meta["cli_tensors"]}
    for states in (26, 16):
        data = (gdir / f"cli_{states}.cdq").read_bytes()
        rd = O.read_cdq(data)
        tensors = []
        for key, nm in golden_meta["cli_tensors"]:
            t = rd[key]
            tag = f"cli{states}.{nm}"
            assert np.array_equal(t["q"], golden[f"{tag}.q"])
            assert np.array_equal(t["scales_f8_u8"], golden[f"{tag}.scales"])
            assert np.array_equal(t["tag_counts"], golden[f"{tag}.tags"])
            w = golden[f"{nm}.weight"]
            p = O.quantize(w, n_states=states, stc_frac=0.0156)
            assert not p["topk_fallback"]
            tensors.append((key, p))
            # the record stream restated from the parsed file is the file's own
            assert np.array_equal(O.pack_from_records(t)["residual_indices"], p["residual_indices"])
        assert O.write_cdq(tensors, states) == data
    assert cases


def test_loader_buffers_and_forward(golden, golden_meta):
    from pathlib import Path
    data = (Path(__file__).parent / "golden" / "cli_26.cdq").read_bytes()
    rd = O.read_cdq(data)
    for key, nm in golden_meta["cli_tensors"]:
        p = O.pack_from_records(rd[key])
        tag = f"loader.{nm}"
        assert np.array_equal(p["quant_indices"], golden[f"{tag}.q"])
        assert _nan_equal_bf16(p["scales_bf16"], golden[f"{tag}.s"])
        assert np.array_equal(p["residual_indices"], golden[f"{tag}.offs"])
        assert np.array_equal(p["residual_values"], golden[f"{tag}.vals"])
        what = O.dequantize(p)
        y64 = O.linear_f64(what, golden[f"{tag}.x"], golden[f"{tag}.bias"])
        yref = O.bf16_bits_to_f32(golden[f"{tag}.y"]).astype(np.float64)
        fin = np.isfinite(y64)
        assert np.array_equal(fin, np.isfinite(yref))
        assert np.all(np.abs(y64[fin] - yref[fin]) <= 2.0 ** -7 * np.abs(y64[fin]) + 1e-30)


@pytest.mark.slow
@pytest.mark.parametrize("ns", [26, 16])
def test_projection_4864x896_digests(golden, golden_meta, ns):
    d = golden_meta["digests"][f"cfg1_{ns}"]
    w = synth_weight(4864, 896, std=0.02, seed=0)
    wb = w.view(torch.int16).numpy().view(np.uint16)
    assert _digest(wb) == d["weight"]
    p = O.quantize(wb, n_states=ns)
    assert p["outlier_count"] == d["outlier_count"]
    assert _digest(p["quant_indices"]) == d["quant_indices"]
    assert _digest(p["scales_f8"]) == d["scales_f8"]
    assert _digest(p["scales_bf16"]) == d["scales_bf16"]
    assert _digest(p["residual_indices"]) == d["residual_indices"]
    assert _digest(p["residual_values"]) == d["residual_values"]
    what = O.dequantize(p)
    assert _digest(what) == d["w_hat"]
    x = synth_activation(1, 896, seed=1).view(torch.int16).numpy().view(np.uint16)
    y64 = O.linear_f64(what, x)
    yref = O.bf16_bits_to_f32(golden[f"cfg1_{ns}.y1"]).astype(np.float64)
    assert np.all(np.abs(y64 - yref) <= 2.0 ** -7 * np.abs(y64) + 1e-30)


def test_oracle_without_guard_reproduces_reference_cli(golden, golden_meta):
    """The packer CLI quantizes without quantize_cdq_lrr's top-k tie guard
    (code/cdq_pack.py:279-291). On a checkpoint where the guard would fire (an
    all-zero and a constant tensor: every saliency ties), the oracle's
    guard-free restatement plus its writer reproduce the reference CLI's file
    byte for byte; with the guard the zero and constant tensors differ."""
    from pathlib import Path
    data = (Path(__file__).parent / "golden" / "cli_noguard_26.cdq").read_bytes()
    tensors, differs = [], []
    for key, nm in golden_meta["cli_noguard_tensors"]:
        w = golden[f"{nm}.weight"]
        p = O.quantize(w, n_states=26, stc_frac=0.0156, topk_guard=False)
        tensors.append((key, p))
        g = O.quantize(w, n_states=26, stc_frac=0.0156)
        differs.append(bool(g["topk_fallback"]) and g["outlier_count"] != p["outlier_count"])
    assert O.write_cdq(tensors, 26) == data
    assert differs == [True, True, False]
