"""The reference's drop-in entry points on the GPU, against the reference's
own outputs recorded in tests/golden:

* the packer CLI (code/cdq_pack.py:251-318) as pack_file.main: the .cdq
  bytes the reference CLI wrote for the same safetensors checkpoint;
* load_cdq and the loader CDQLinear (code/cdq_loader.py:43-110): the
  reference loader's buffers and outputs for the CLI's file;
* quantize_cdq_lrr's dict (code/cdq_lrr_qwen05.py:121-133): the reference's
  keys, types, dtypes and shapes, and its values.
"""
import json
import os
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import cdq_oracle as O

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).parent / "golden"


def _bf16(bits_u16):
    return torch.from_numpy(np.ascontiguousarray(bits_u16).view(np.int16)).view(torch.bfloat16)


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _checkpoint(golden, names, path):
    from safetensors.torch import save_file
    tensors = {key: _bf16(golden[f"{nm}.weight"]).contiguous() for key, nm in names}
    save_file(tensors, os.path.join(path, "model.safetensors"))


@pytest.mark.parametrize("states", [26, 16])
def test_packer_cli_reproduces_reference_file(golden, golden_meta, tmp_path, states):
    """pack_file.main on the checkpoint the reference CLI packed writes the
    same bytes, with the default guard (it does not fire on these tensors)
    and without it."""
    from cdq_lrr_b200 import pack_file
    _checkpoint(golden, golden_meta["cli_tensors"], tmp_path)
    want = (GOLD / f"cli_{states}.cdq").read_bytes()
    for extra in ([], ["--no-topk-guard"]):
        out = tmp_path / f"ours_{states}_{len(extra)}.cdq"
        pack_file.main(["--model", str(tmp_path), "--out", str(out), "--states", str(states), *extra])
        assert out.read_bytes() == want


def test_packer_cli_without_guard_matches_reference_on_ties(golden, golden_meta, tmp_path):
    """Where the top-k tie guard fires (all-zero and constant tensors), only
    --no-topk-guard reproduces the reference CLI, whose quantizer has no guard."""
    from cdq_lrr_b200 import pack_file
    _checkpoint(golden, golden_meta["cli_noguard_tensors"], tmp_path)
    want = (GOLD / "cli_noguard_26.cdq").read_bytes()
    out = tmp_path / "noguard.cdq"
    pack_file.main(["--model", str(tmp_path), "--out", str(out), "--states", "26", "--no-topk-guard"])
    assert out.read_bytes() == want
    guarded = tmp_path / "guarded.cdq"
    pack_file.main(["--model", str(tmp_path), "--out", str(guarded), "--states", "26"])
    assert guarded.read_bytes() != want


def test_load_cdq_matches_reference_loader(golden, golden_meta):
    """load_cdq on the reference CLI's file: the loader CDQLinear's q / s / offs
    / vals equal the reference loader's, and its forward is the fused GEMV
    (within the 1e-3 bar of the fp64 dot of w_hat, next to the reference
    loader's own bf16 output)."""
    from cdq_lrr_b200 import loader

    names = golden_meta["cli_tensors"]

    class Mlp(torch.nn.Module):
        def __init__(self, rows, cols):
            super().__init__()
            self.down_proj = torch.nn.Linear(cols, rows, bias=True)

    class Layer(torch.nn.Module):
        def __init__(self, rows, cols):
            super().__init__()
            self.mlp = Mlp(rows, cols)

    root = torch.nn.Module()
    root.model = torch.nn.Module()
    root.model.layers = torch.nn.ModuleList(
        [Layer(*golden[f"{nm}.weight"].shape) for _, nm in names]).to(torch.bfloat16).cuda()
    with torch.no_grad():
        for i, (_, nm) in enumerate(names):
            root.model.layers[i].mlp.down_proj.bias.copy_(_bf16(golden[f"loader.{nm}.bias"]).cuda())
    loader.load_cdq(root, str(GOLD / "cli_26.cdq"))
    for i, (_, nm) in enumerate(names):
        mod = root.model.layers[i].mlp.down_proj
        assert isinstance(mod, loader.CDQLinear)
        tag = f"loader.{nm}"
        assert np.array_equal(mod.q.numpy(), golden[f"{tag}.q"])
        assert np.array_equal(_bits(mod.s).ravel(), golden[f"{tag}.s"])
        assert np.array_equal(mod.offs.numpy(), golden[f"{tag}.offs"])
        assert np.array_equal(_bits(mod.vals), golden[f"{tag}.vals"])
        x = _bf16(golden[f"{tag}.x"]).cuda()
        with torch.no_grad():
            y = mod(x)
        assert y.dtype == torch.bfloat16 and y.shape == tuple(golden[f"{tag}.y"].shape)
        w_hat = _bits(__import__("cdq_lrr_b200.ops", fromlist=["dequant"]).dequant(mod.device_pack))
        ref64 = O.linear_f64(w_hat, golden[f"{tag}.x"], golden[f"{tag}.bias"])
        y64 = y.double().cpu().numpy()
        ref_loader = O.bf16_bits_to_f32(golden[f"{tag}.y"]).astype(np.float64)
        # the same outputs are non-finite (a scale beyond the fp8 range decodes to NaN)
        fin = np.isfinite(ref64)
        assert np.array_equal(fin, np.isfinite(y64)) and np.array_equal(fin, np.isfinite(ref_loader))
        if fin.any():  # bf16 outputs: within the rounding of the output
            assert np.linalg.norm(y64[fin] - ref64[fin]) <= 1e-2 * np.linalg.norm(ref64[fin])
            assert np.linalg.norm(y64[fin] - ref_loader[fin]) <= 1e-2 * np.linalg.norm(ref_loader[fin])


def test_quantize_dict_matches_reference_dict(golden, golden_meta):
    """quant.quantize_cdq_lrr returns the reference's dict: same keys, Python
    types, tensor dtypes and shapes, and the reference's values."""
    from cdq_lrr_b200 import quant
    spec = golden_meta["pack_dict"]
    nm = spec["case"]
    w = _bf16(golden[f"{nm}.weight"])
    pack = quant.quantize_cdq_lrr(w)
    assert set(pack) == set(spec["keys"])
    for k, s in spec["keys"].items():
        v = pack[k]
        if s["type"] == "tensor":
            assert isinstance(v, torch.Tensor), k
            assert str(v.dtype).replace("torch.", "") == s["dtype"], (k, v.dtype)
            assert list(v.shape) == s["shape"], (k, v.shape)
            assert v.device.type == "cpu", k
        else:
            assert type(v).__name__ == s["type"], (k, type(v))
            want = s["value"]
            assert (list(v) if isinstance(v, tuple) else v) == want, (k, v)
    assert np.array_equal(pack["quant_indices"].numpy(), golden[f"{nm}.quant_indices"])
    assert np.array_equal(pack["scales_f8"].view(torch.uint8).numpy().ravel(), golden[f"{nm}.scales_f8"])
    assert np.array_equal(_bits(pack["scales_bf16"]).ravel(), golden[f"{nm}.scales_bf16"])
    assert np.array_equal(pack["residual_indices"].numpy(), golden[f"{nm}.residual_indices"])
    assert np.array_equal(_bits(pack["residual_values"]), golden[f"{nm}.residual_values"])


@pytest.mark.parametrize("states", [26, 16])
def test_own_format_state_dict_is_validated(states):
    """CDQLinear buffers in this library's own layout, loaded from a state
    dict, are checked before any kernel reads them: a faithful copy loads and
    computes the same output; a 26-state pair code above 728, CSR bounds out
    of order and a residual column beyond the weight are refused with
    CDQ_ERR_FORMAT, and the module keeps its previous buffers."""
    from cdq_lrr_b200 import _lib as L
    from cdq_lrr_b200.quant import CAMKII_LATTICE, CAMKII_LATTICE_16, CDQLinear, quantize_cdq_lrr
    lat = CAMKII_LATTICE if states == 26 else CAMKII_LATTICE_16
    g = torch.Generator().manual_seed(5)
    w = (torch.randn(48, 256, generator=g) * 0.02).to(torch.bfloat16)
    w[3, 7] = 0.5
    w[40, 200] = -0.4
    lin = CDQLinear(quantize_cdq_lrr(w.cuda(), lattice=lat), 256, 48)
    x = (torch.randn(2, 256, generator=g)).to(torch.bfloat16).cuda()
    want = lin(x)
    sd = {k: v.clone() for k, v in lin.state_dict().items()}
    assert int(sd["res_ent"].numel()) > 0
    other = CDQLinear(quantize_cdq_lrr(torch.zeros_like(w).cuda(), lattice=lat), 256, 48)
    other.load_state_dict(sd)
    assert torch.equal(other(x), want)

    def refused(mutate):
        bad = {k: v.clone() for k, v in sd.items()}
        mutate(bad)
        tgt = CDQLinear(quantize_cdq_lrr(w.cuda(), lattice=lat), 256, 48)
        before = tgt.units.clone()
        with pytest.raises(L.CdqError) as ei:
            tgt.load_state_dict(bad)
        assert ei.value.status == 5
        assert torch.equal(tgt.units, before)

    if states == 26:
        def big_code(sd_):  # lane 0, code word 0: slot 0 = 1023
            sd_["units"][0] |= 0xFF
            sd_["units"][1] |= 0x03
        refused(big_code)

    def csr_order(sd_):
        sd_["res_ptr"][1] = sd_["res_ptr"][-1] + 1
    refused(csr_order)

    def col_out(sd_):
        sd_["res_ent"][0] = (sd_["res_ent"][0] & 0xFFFF) | (300 << 16)
    refused(col_out)

    def short_units(sd_):
        sd_["units"] = sd_["units"][:-16]
    refused(short_units)
