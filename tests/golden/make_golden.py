"""Generate the golden vectors that pin the CPU oracle to the reference.

Run where the reference source tree is available, with CDQ_REFERENCE set to
its root (the directory holding code/). It imports the reference's own Python
modules and records what they return:

* code/cdq_lrr_qwen05.py: CAMKII_LATTICE / CAMKII_LATTICE_16,
  fp8_quantize_scale, quantize_cdq_lrr, dequantize, CDQLinear.forward;
* code/cdq_pack.py: the packer CLI (run as a subprocess on a temporary
  safetensors checkpoint) and its write_cdq / read_cdq / bit packers;
* code/cdq_loader.py: load_cdq and the loader CDQLinear.forward.

Small cases are stored in full; the [4864, 896] workload is stored as SHA-256
digests of the reference's arrays plus a few scalars. Outputs go next to this
script: golden.npz, digests.json and *.cdq files. The weights come from
cdq_lrr_b200.synth (torch CPU generator, deterministic across machines).

    CDQ_REFERENCE=<reference root> python tests/golden/make_golden.py [--extras]

``--extras`` only adds to the existing fixtures: the packer CLI's file for a
checkpoint on which quantize_cdq_lrr's top-k tie guard fires (the CLI has no
guard: cli_noguard_26.cdq) and the key / type / dtype / shape record of the
quantize_cdq_lrr dict ("pack_dict" in digests.json).
"""
from __future__ import annotations

import hashlib
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))
if not os.environ.get("CDQ_REFERENCE"):
    raise SystemExit("set CDQ_REFERENCE to the reference source tree (the directory holding code/)")
REF = Path(os.environ["CDQ_REFERENCE"]) / "code"
sys.path.insert(0, str(REF))

import cdq_lrr_qwen05 as R  # noqa: E402
import cdq_pack as P  # noqa: E402
import cdq_loader as L  # noqa: E402

from cdq_lrr_b200.synth import synth_activation, synth_weight  # noqa: E402


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    if t.dtype == torch.float8_e4m3fn:
        return t.contiguous().view(torch.uint8).numpy().copy()
    return t.contiguous().numpy().copy()


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def weight_case(name: str) -> tuple[torch.Tensor, int, float]:
    """(bf16 weight, n_states, stc_frac) for a named small case."""
    g = torch.Generator().manual_seed(1234)
    if name == "small26":
        return synth_weight(64, 128, seed=11), 26, 0.0156
    if name == "small16":
        return synth_weight(64, 128, seed=11), 16, 0.0156
    if name == "rect26":
        return synth_weight(96, 320, std=0.015, seed=12), 26, 0.0156
    if name == "frac03125":
        return synth_weight(48, 256, seed=13), 16, 0.03125
    if name == "frac50":
        return synth_weight(32, 64, seed=14), 26, 0.5
    if name == "onetile":
        return synth_weight(1, 32, seed=15), 26, 0.0156
    if name == "zeros":
        return torch.zeros(8, 64, dtype=torch.bfloat16), 26, 0.0156
    if name == "constant":
        return torch.full((16, 64), 0.5, dtype=torch.bfloat16), 26, 0.0156
    if name == "zerotiles":
        w = synth_weight(32, 128, seed=16)
        w[3, :64] = 0
        w[7, 32:96] = 0
        w[10, :] = 1e-12
        return w, 26, 0.0156
    if name == "tiny":
        return (torch.randn(32, 96, generator=g) * 1e-5).to(torch.bfloat16), 26, 0.0156
    if name == "huge":
        w = synth_weight(16, 64, seed=17)
        w[2, 5] = 500.0
        w[4, 40] = -470.0
        w[6, 1] = 464.0
        w[9, 33] = 460.0
        return w, 26, 0.0156
    if name == "wide16":
        return synth_weight(16, 1024, seed=18), 16, 0.0156
    if name == "mid26":
        # values near lattice midpoints of sigma = 1 tiles
        lat = R.CAMKII_LATTICE.float()
        mids = ((lat[1:] + lat[:-1]) / 2)
        w = torch.empty(32, 64)
        w[:, 0] = 1.0
        w[:, 1:] = mids[torch.randint(0, 25, (32, 63), generator=g)]
        return w.to(torch.bfloat16), 26, 0.0156
    if name == "nanweight":
        w = synth_weight(8, 64, seed=19)
        w[1, 3] = float("nan")
        return w, 26, 0.0156
    if name == "infweight":
        w = synth_weight(8, 64, seed=20)
        w[5, 60] = float("inf")
        return w, 16, 0.0156
    raise KeyError(name)


SMALL_CASES = ["small26", "small16", "rect26", "frac03125", "frac50", "onetile", "zeros",
               "constant", "zerotiles", "tiny", "huge", "wide16", "mid26", "nanweight",
               "infweight"]


def lattice_of(n_states: int) -> torch.Tensor:
    return R.CAMKII_LATTICE if n_states == 26 else R.CAMKII_LATTICE_16


def record_pack(out: dict, tag: str, pack: dict) -> None:
    out[f"{tag}.quant_indices"] = bits(pack["quant_indices"])
    out[f"{tag}.scales_f8"] = bits(pack["scales_f8"]).ravel()
    out[f"{tag}.scales_bf16"] = bits(pack["scales_bf16"]).ravel()
    out[f"{tag}.residual_indices"] = bits(pack["residual_indices"])
    out[f"{tag}.residual_values"] = bits(pack["residual_values"])


def main() -> None:
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out: dict[str, np.ndarray] = {}
    meta: dict = {"torch": torch.__version__, "cases": {}}

    # lattices and the fp8 scale round trip over every bf16 bit pattern
    out["lattice26"] = bits(R.CAMKII_LATTICE)
    out["lattice16"] = bits(R.CAMKII_LATTICE_16)
    allbf = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    out["fp8_encode_all_bf16"] = bits(allbf.to(R.FP8_DTYPE))
    out["fp8_scale_all_bf16"] = bits(R.fp8_quantize_scale(allbf))
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(R.FP8_DTYPE)
    out["fp8_decode_all"] = bits(codes.to(torch.bfloat16))

    # quantizer, dequantizer and forward on small cases
    for name in SMALL_CASES:
        w, ns, frac = weight_case(name)
        pack = R.quantize_cdq_lrr(w, lattice=lattice_of(ns), stc_frac=frac)
        out[f"{name}.weight"] = bits(w)
        record_pack(out, name, pack)
        what = R.dequantize(pack)
        out[f"{name}.w_hat"] = bits(what)
        rows, cols = w.shape
        bias = synth_activation(1, rows, seed=99)[0]
        lin = R.CDQLinear(pack, cols, rows, bias=bias)
        for m in (1, 3):
            x = synth_activation(m, cols, seed=7 + m)
            out[f"{name}.x{m}"] = bits(x)
            with torch.no_grad():
                out[f"{name}.y{m}"] = bits(lin(x))
        out[f"{name}.bias"] = bits(bias)
        meta["cases"][name] = {"n_states": ns, "stc_frac": frac,
                               "outlier_count": pack["outlier_count"]}

    # packer CLI -> .cdq files, then read_cdq and load_cdq on them
    with tempfile.TemporaryDirectory() as td:
        from safetensors.torch import save_file
        tensors = {}
        names = []
        for i, nm in enumerate(["small26", "rect26", "zerotiles", "huge"]):
            w, _, _ = weight_case(nm)
            key = f"model.layers.{i}.mlp.down_proj.weight"
            tensors[key] = w.contiguous()
            names.append((key, nm))
        save_file(tensors, os.path.join(td, "model.safetensors"))
        for states in (26, 16):
            dst = HERE / f"cli_{states}.cdq"
            subprocess.run([sys.executable, str(REF / "cdq_pack.py"), "--model", td,
                            "--out", str(dst), "--states", str(states)],
                           check=True, capture_output=True)
            rd = P.read_cdq(str(dst))
            for key, nm in names:
                t = rd[key]
                tag = f"cli{states}.{nm}"
                out[f"{tag}.q"] = t["q"].numpy().copy()
                out[f"{tag}.scales"] = t["scales_f8_u8"].numpy().ravel().copy()
                out[f"{tag}.tags"] = t["tag_counts"].numpy().copy()
        meta["cli_tensors"] = names

        # loader: a module tree named like the checkpoint, patched from cli_26.cdq
        class Mlp(torch.nn.Module):
            def __init__(self, rows, cols):
                super().__init__()
                self.down_proj = torch.nn.Linear(cols, rows, bias=True)

        class Layer(torch.nn.Module):
            def __init__(self, rows, cols):
                super().__init__()
                self.mlp = Mlp(rows, cols)

        class Model(torch.nn.Module):
            def __init__(self):
                super().__init__()
                self.layers = torch.nn.ModuleList()
                for key, nm in names:
                    w, _, _ = weight_case(nm)
                    self.layers.append(Layer(*w.shape))

        model = Model()
        with torch.no_grad():
            for i, (key, nm) in enumerate(names):
                b = synth_activation(1, tensors[key].shape[0], seed=200 + i)[0]
                model.layers[i].mlp.down_proj.bias.copy_(b.float())
        model = model.to(torch.bfloat16)
        # load_cdq prefixes nothing: names must resolve from the root module
        wrapper = torch.nn.Module()
        wrapper.model = model
        L.load_cdq(wrapper, str(HERE / "cli_26.cdq"))
        for i, (key, nm) in enumerate(names):
            mod = wrapper.model.layers[i].mlp.down_proj
            tag = f"loader.{nm}"
            out[f"{tag}.q"] = bits(mod.q)
            out[f"{tag}.s"] = bits(mod.s).ravel()
            out[f"{tag}.offs"] = bits(mod.offs)
            out[f"{tag}.vals"] = bits(mod.vals)
            out[f"{tag}.bias"] = bits(mod.bias.data)
            x = synth_activation(2, tensors[key].shape[1], seed=300 + i)
            out[f"{tag}.x"] = bits(x)
            with torch.no_grad():
                out[f"{tag}.y"] = bits(mod(x))

    # the [4864, 896] workload: digests only
    dig: dict = {}
    for ns in (26, 16):
        w = synth_weight(4864, 896, std=0.02, seed=0)
        pack = R.quantize_cdq_lrr(w, lattice=lattice_of(ns))
        what = R.dequantize(pack)
        x = synth_activation(1, 896, seed=1)
        lin = R.CDQLinear(pack, 896, 4864)
        with torch.no_grad():
            y = lin(x)
        sal_n = pack["numel"]
        d = {
            "weight": digest(bits(w)),
            "quant_indices": digest(bits(pack["quant_indices"])),
            "scales_f8": digest(bits(pack["scales_f8"]).ravel()),
            "scales_bf16": digest(bits(pack["scales_bf16"]).ravel()),
            "residual_indices": digest(bits(pack["residual_indices"])),
            "residual_values": digest(bits(pack["residual_values"])),
            "w_hat": digest(bits(what)),
            "y1": digest(bits(y)),
            "outlier_count": pack["outlier_count"],
            "numel": sal_n,
        }
        out[f"cfg1_{ns}.y1"] = bits(y)
        dig[f"cfg1_{ns}"] = d
    meta["digests"] = dig

    np.savez_compressed(HERE / "golden.npz", **out)
    (HERE / "digests.json").write_text(json.dumps(meta, indent=1, sort_keys=True))
    print("wrote", HERE / "golden.npz", sum(v.nbytes for v in out.values()), "raw bytes")


def extras() -> None:
    """The packer CLI on tensors where the top-k tie guard fires, and the pack
    dict's structure, added to the existing fixtures."""
    meta = json.loads((HERE / "digests.json").read_text())
    with tempfile.TemporaryDirectory() as td:
        from safetensors.torch import save_file
        tensors, names = {}, []
        for i, nm in enumerate(["zeros", "constant", "small26"]):
            w, _, _ = weight_case(nm)
            key = f"model.layers.{i}.mlp.up_proj.weight"
            tensors[key] = w.contiguous()
            names.append((key, nm))
        save_file(tensors, os.path.join(td, "model.safetensors"))
        dst = HERE / "cli_noguard_26.cdq"
        subprocess.run([sys.executable, str(REF / "cdq_pack.py"), "--model", td, "--out", str(dst),
                        "--states", "26"], check=True, capture_output=True)
        meta["cli_noguard_tensors"] = names
    w, ns, frac = weight_case("small26")
    pack = R.quantize_cdq_lrr(w, lattice=lattice_of(ns), stc_frac=frac)
    spec = {}
    for k, v in pack.items():
        if isinstance(v, torch.Tensor):
            spec[k] = {"type": "tensor", "dtype": str(v.dtype).replace("torch.", ""), "shape": list(v.shape)}
        else:
            spec[k] = {"type": type(v).__name__, "value": list(v) if isinstance(v, (tuple, torch.Size)) else v}
    meta["pack_dict"] = {"case": "small26", "keys": spec}
    (HERE / "digests.json").write_text(json.dumps(meta, indent=1, sort_keys=True))
    print("wrote", dst, "and pack_dict")


if __name__ == "__main__":
    extras() if "--extras" in sys.argv else main()
