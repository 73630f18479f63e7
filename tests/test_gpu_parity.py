"""GPU parity: every kernel through the C ABI against the oracle.

* cdq_dequant: w_hat bit-exact (NaN compared as NaN) on every golden case;
* cdq_quantize: indices, fp8 scales, residual indices and values bit-exact
  with the reference's own outputs, including the [4864, 896] digests;
* cdq_linear / cdq_linear_f32: fp32 output within 1e-3 relative (normwise
  and per element against the fp64 dot of the oracle's w_hat); the bf16
  output is the fp32 output rounded once;
* cdq_linear_grouped: bit-identical to one launch per job.
"""
import hashlib

import numpy as np
import pytest
import torch

from oracle import cdq_oracle as O

pytestmark = pytest.mark.gpu

CASES = ["small26", "small16", "rect26", "frac03125", "frac50", "onetile", "zeros",
         "constant", "zerotiles", "tiny", "huge", "wide16", "mid26", "nanweight", "infweight"]
REL_TOL = 1e-3   # GEMV bar: fp32 accumulation vs the fp64 dot of the oracle's w_hat


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _nan_equal(a, b):
    a = np.asarray(a, np.uint16)
    b = np.asarray(b, np.uint16)
    an = ((a & 0x7F80) == 0x7F80) & ((a & 0x7F) != 0)
    bn = ((b & 0x7F80) == 0x7F80) & ((b & 0x7F) != 0)
    return bool(np.array_equal(an, bn) and np.array_equal(a[~an], b[~bn]))


def _digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _dev_pack(golden, name, n_states):
    from cdq_lrr_b200.ops import DevicePack
    w = golden[f"{name}.weight"]
    return DevicePack.from_reference(
        golden[f"{name}.quant_indices"], golden[f"{name}.scales_f8"],
        golden[f"{name}.residual_indices"], golden[f"{name}.residual_values"],
        w.shape[0], w.shape[1], n_states, device="cuda")


def _t(bits_u16: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits_u16).view(np.int16)).view(torch.bfloat16).cuda()


def _check_gemv(y32: torch.Tensor, y64: np.ndarray):
    y = y32.double().cpu().numpy()
    fin = np.isfinite(y64)
    assert np.array_equal(fin, np.isfinite(y)), "NaN/inf pattern differs"
    if fin.any():
        d = np.abs(y[fin] - y64[fin])
        norm = np.linalg.norm(y64[fin])
        assert np.linalg.norm(d) <= REL_TOL * max(norm, 1e-30), (np.linalg.norm(d), norm)
        scale = np.sqrt(np.mean(y64[fin] ** 2)) + 1e-30
        assert np.all(d <= REL_TOL * (np.abs(y64[fin]) + scale)), float(d.max())


@pytest.mark.parametrize("name", CASES)
def test_dequant_bit_exact(golden, golden_meta, name):
    from cdq_lrr_b200 import ops
    ns = golden_meta["cases"][name]["n_states"]
    dp = _dev_pack(golden, name, ns)
    w_hat = ops.dequant(dp)
    torch.cuda.synchronize()
    assert _nan_equal(_bits(w_hat), golden[f"{name}.w_hat"])


@pytest.mark.parametrize("name", CASES)
def test_quantize_bit_exact(golden, golden_meta, name):
    from cdq_lrr_b200 import ops
    meta = golden_meta["cases"][name]
    w = _t(golden[f"{name}.weight"])
    pack, info = ops.quantize(w, n_states=meta["n_states"], stc_frac=meta["stc_frac"])
    ref = pack.to_reference()
    assert info["n_res"] == meta["outlier_count"]
    assert np.array_equal(ref["quant_indices"], golden[f"{name}.quant_indices"])
    assert np.array_equal(ref["scales_f8"], golden[f"{name}.scales_f8"])
    assert np.array_equal(ref["residual_indices"], golden[f"{name}.residual_indices"])
    assert np.array_equal(ref["residual_values"], golden[f"{name}.residual_values"])
    p = O.quantize(golden[f"{name}.weight"], n_states=meta["n_states"], stc_frac=meta["stc_frac"])
    assert info["topk_fallback"] == p["topk_fallback"]
    if not np.isnan(p["threshold"]):
        assert np.float32(info["threshold"]) == p["threshold"]


@pytest.mark.parametrize("ns", [26, 16])
def test_quantize_4864x896_digests(golden_meta, ns):
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_weight
    d = golden_meta["digests"][f"cfg1_{ns}"]
    w = synth_weight(4864, 896, std=0.02, seed=0)
    assert _digest(_bits(w)) == d["weight"]
    pack, info = ops.quantize(w.cuda(), n_states=ns)
    ref = pack.to_reference()
    assert info["n_res"] == d["outlier_count"]
    assert _digest(ref["quant_indices"]) == d["quant_indices"]
    assert _digest(ref["scales_f8"]) == d["scales_f8"]
    assert _digest(ref["residual_indices"]) == d["residual_indices"]
    assert _digest(ref["residual_values"]) == d["residual_values"]
    assert _digest(_bits(ops.dequant(pack))) == d["w_hat"]


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("m", [1, 3, 8])
def test_linear_against_oracle(golden, golden_meta, name, m):
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation
    meta = golden_meta["cases"][name]
    dp = _dev_pack(golden, name, meta["n_states"])
    rows, cols = golden[f"{name}.weight"].shape
    x = synth_activation(m, cols, seed=40 + m)
    bias = golden[f"{name}.bias"]
    y32 = ops.linear(dp, x.cuda(), _t(bias), out_f32=True)
    y16 = ops.linear(dp, x.cuda(), _t(bias))
    y64 = O.linear_f64(golden[f"{name}.w_hat"], _bits(x), bias)
    _check_gemv(y32, y64)
    # the bf16 output is the fp32 result rounded once (same kernel, same order)
    assert _nan_equal(_bits(y16), O.f32_to_bf16_bits(y32.cpu().numpy()))


@pytest.mark.parametrize("shape,ns", [((256, 4864), 26), ((64, 2080), 26), ((45, 96), 26),
                                      ((33, 3104), 16), ((4864, 896), 26), ((896, 4864), 16)])
@pytest.mark.parametrize("m", [1, 4])
def test_linear_split_k_and_ragged(shape, ns, m):
    """Several residual groups per row (split K through the workspace), rows
    not a multiple of 32, a last group of one tile; repeated calls reuse the
    self-resetting workspace and give identical results."""
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight
    rows, cols = shape
    w = synth_weight(rows, cols, seed=rows + cols)
    p = O.quantize(_bits(w), n_states=ns)
    from cdq_lrr_b200.ops import DevicePack
    dp = DevicePack.from_reference(p["quant_indices"], p["scales_f8"], p["residual_indices"],
                                   p["residual_values"], rows, cols, ns, device="cuda")
    x = synth_activation(m, cols, seed=5).cuda()
    y1 = ops.linear(dp, x, out_f32=True)
    y2 = ops.linear(dp, x, out_f32=True)
    assert torch.equal(y1, y2)
    _check_gemv(y1, O.linear_f64(O.dequantize(p), _bits(x)))


@pytest.mark.parametrize("m", [1, 2, 5, 8])
def test_stream_cut_row_blocks_and_counters(m):
    """Long rows (several residual groups) in launches of every size: the row
    blocks that a warp's stretch boundary cuts are finished through the
    workspace's arrival counters. The result is bit-identical whether the job
    runs alone or among other jobs (different cuts), and every call leaves the
    counters at zero."""
    from cdq_lrr_b200 import _lib as L
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight
    shapes = [(896, 4864), (64, 18944), (1000, 2080), (16, 65504 // 32 * 32)]
    packs = [ops.quantize(synth_weight(r, c, seed=r + c).cuda(), n_states=26)[0] for r, c in shapes]
    xs = [synth_activation(m, c, seed=c).cuda() for _, c in shapes]
    singles = [ops.linear(p, x, out_f32=True) for p, x in zip(packs, xs)]
    filler = [ops.quantize(synth_weight(4864, 896, seed=i).cuda(), n_states=26)[0] for i in range(3)]
    for order in (0, 1):
        tasks = []
        jobs = list(zip(packs, xs))
        if order:
            jobs = jobs[::-1]
        for f in filler:
            tasks.append(ops.GemvTask(f, synth_activation(m, 896, seed=9).cuda(),
                                      torch.empty(m, 4864, dtype=torch.float32, device="cuda")))
        for p, x in jobs:
            tasks.append(ops.GemvTask(p, x, torch.empty(m, p.rows, dtype=torch.float32, device="cuda")))
        ops.linear_grouped(tasks, m)
        torch.cuda.synchronize()
        got = {id(t.pack): t.y for t in tasks}
        for p, s in zip(packs, singles):
            assert torch.equal(got[id(p)], s)
    for p, (r, c), x, s in zip(packs, shapes, xs, singles):
        ws = p.linear_workspace(m)
        nbytes = (r + 15) // 16 * 4
        assert int(ws[:nbytes].count_nonzero()) == 0
        _check_gemv(s, O.linear_f64(_bits(ops.dequant(p)), _bits(x)))


def test_linear_batch_above_8_splits():
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight
    w = synth_weight(128, 512, seed=9)
    p = O.quantize(_bits(w))
    dp = ops.DevicePack.from_reference(p["quant_indices"], p["scales_f8"], p["residual_indices"],
                                       p["residual_values"], 128, 512, 26, device="cuda")
    x = synth_activation(19, 512, seed=2).cuda()
    y = ops.linear(dp, x, out_f32=True)
    _check_gemv(y, O.linear_f64(O.dequantize(p), _bits(x)))


@pytest.mark.parametrize("shape,ns", [((128, 512), 26), ((64, 2080), 26), ((45, 96), 16), ((896, 4864), 16)])
@pytest.mark.parametrize("m", [9, 16, 33, 64])
def test_linear_wide_batch(shape, ns, m):
    """Batches 9..64: each unit is decoded once and multiplied against
    ceil(m/8) n-tiles; every row must match the oracle and equal the same
    row computed alone (a row's arithmetic does not depend on the batch)."""
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight
    rows, cols = shape
    w = synth_weight(rows, cols, seed=rows + cols + m)
    p = O.quantize(_bits(w), n_states=ns)
    dp = ops.DevicePack.from_reference(p["quant_indices"], p["scales_f8"], p["residual_indices"],
                                       p["residual_values"], rows, cols, ns, device="cuda")
    x = synth_activation(m, cols, seed=m).cuda()
    bias = synth_activation(1, rows, seed=3)[0].cuda()
    y = ops.linear(dp, x, bias, out_f32=True)
    ref = O.linear_f64(O.dequantize(p), _bits(x)) + O.bf16_bits_to_f32(_bits(bias)).astype(np.float64)
    _check_gemv(y, ref)
    for i in (0, m // 2, m - 1):
        assert torch.equal(y[i:i + 1], ops.linear(dp, x[i:i + 1], bias, out_f32=True))


@pytest.fixture
def tile_min_batch():
    """Sets the smallest batch that takes the tcgen05 tile path; restores 16."""
    from cdq_lrr_b200 import _lib as L
    yield L.set_tile_min_batch
    L.set_tile_min_batch(16)


def _tile_copies(rows: int) -> int:
    """Jobs of one projection that give a grouped launch enough 128-row tiles
    (one per two SMs of a B200) to take the tile path."""
    return -(-74 // -(-rows // 128))


@pytest.mark.parametrize("shape,ns", [((128, 512), 26), ((200, 2080), 26), ((45, 96), 16), ((896, 4864), 16),
                                      ((4864, 896), 26)])
@pytest.mark.parametrize("m", [1, 5, 16, 40])
def test_tile_path_against_oracle(tile_min_batch, shape, ns, m):
    """The tcgen05 tile path (forced for every batch here) against the oracle:
    one projection in enough jobs of a grouped launch to take the tile path,
    half of them on one shared activation matrix (prepared once) and half on
    their own; ragged row tiles (rows not a multiple of 128), odd tile counts
    (a phantom tile) and several residual groups included."""
    from cdq_lrr_b200 import _lib as L
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight
    tile_min_batch(1)
    rows, cols = shape
    w = synth_weight(rows, cols, seed=rows * 7 + cols + m)
    p = O.quantize(_bits(w), n_states=ns)
    dp = ops.DevicePack.from_reference(p["quant_indices"], p["scales_f8"], p["residual_indices"],
                                       p["residual_values"], rows, cols, ns, device="cuda")
    w_hat = O.dequantize(p)
    bias = synth_activation(1, rows, seed=4)[0].cuda()
    b64 = O.bf16_bits_to_f32(_bits(bias)).astype(np.float64)
    shared = synth_activation(m, cols, seed=m + 1).cuda()
    tasks = []
    for k in range(_tile_copies(rows)):
        x = shared if k % 2 == 0 else synth_activation(m, cols, seed=1000 + k).cuda()
        tasks.append(ops.GemvTask(dp, x, torch.empty(m, rows, dtype=torch.float32, device="cuda"), bias))
    ops.linear_grouped(tasks, m)
    torch.cuda.synchronize()
    assert L.kernel_error() == 0
    for k, t in enumerate(tasks[:4]):
        _check_gemv(t.y, O.linear_f64(w_hat, _bits(t.x)) + b64)


def test_tile_path_grouped_matches_streaming(tile_min_batch):
    """A grouped tile-path launch (jobs of both lattices and ragged shapes)
    matches the streaming path on the same jobs (single launches, which are
    too small for the tile path). The two add the same fp32 terms in a
    different order: the bar is 1e-5 of the output scale, far below the 1e-3
    oracle bar."""
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight
    tile_min_batch(1)
    shapes = [(896, 896, 26), (128, 896, 26), (4864, 896, 26), (896, 4864, 26), (96, 320, 16), (40, 2080, 16)]
    for m in (1, 24):
        by_ns = {}
        singles = []
        for rep in range(3):
            for i, (r, c, ns) in enumerate(shapes):
                pack, _ = ops.quantize(synth_weight(r, c, seed=400 + i).cuda(), n_states=ns)
                x = synth_activation(m, c, seed=500 + 10 * rep + i).cuda()
                t = ops.GemvTask(pack, x, torch.empty(m, r, dtype=torch.float32, device="cuda"))
                by_ns.setdefault(ns, []).append(t)
                singles.append((t, ops.linear(pack, x, out_f32=True)))
        for ts in by_ns.values():
            ops.linear_grouped(ts, m)
        torch.cuda.synchronize()
        for t, s in singles:
            tol = 1e-5 * (s.abs().max().item() + 1e-6)
            assert (t.y - s).abs().max().item() <= tol


@pytest.mark.parametrize("m", [1, 16, 64])
def test_tile_full_mode_many_jobs(tile_min_batch, m):
    """A grouped launch with many jobs on the tile path: the tile epilogue adds
    the residual entries and the bias and writes the final output (bf16 and
    float32 outputs, both lattices, rows not a multiple of 128, several
    residual groups per row)."""
    from cdq_lrr_b200 import _lib as L
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight
    tile_min_batch(1)
    shapes = [(896, 896, 26), (4864, 896, 26), (896, 4864, 26), (1000, 2080, 16), (4864, 896, 16),
              (200, 96, 26)] * 4
    refs, tasks = [], []
    for i, (r, c, ns) in enumerate(shapes):
        w = synth_weight(r, c, seed=600 + i)
        p = O.quantize(_bits(w), n_states=ns)
        dp = ops.DevicePack.from_reference(p["quant_indices"], p["scales_f8"], p["residual_indices"],
                                           p["residual_values"], r, c, ns, device="cuda")
        x = synth_activation(m, c, seed=700 + i).cuda()
        bias = synth_activation(1, r, seed=800 + i)[0].cuda() if i % 2 == 0 else None
        out_dtype = torch.float32 if i % 3 == 0 else torch.bfloat16
        tasks.append(ops.GemvTask(dp, x, torch.empty(m, r, dtype=out_dtype, device="cuda"), bias))
        ref = O.linear_f64(O.dequantize(p), _bits(x))
        if bias is not None:
            ref = ref + O.bf16_bits_to_f32(_bits(bias)).astype(np.float64)
        refs.append(ref)
    by_ns = {}
    for t, (_, _, ns) in zip(tasks, shapes):
        by_ns.setdefault(ns, []).append(t)
    for ts in by_ns.values():
        ops.linear_grouped(ts, m)
    torch.cuda.synchronize()
    assert L.kernel_error() == 0
    for t, ref in zip(tasks, refs):
        if t.y.dtype == torch.float32:
            _check_gemv(t.y, ref)
        else:
            err = np.abs(t.y.float().cpu().numpy() - ref).max()
            assert err <= 2 ** -7 * np.abs(ref).max() + 1e-3, err


def test_grouped_wide_batch_shared_pack():
    """One pack in several jobs of one wide-batch grouped launch: each job gets
    its own group-sum workspace."""
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight
    pack, _ = ops.quantize(synth_weight(896, 896, seed=5).cuda(), n_states=26)
    tasks, singles = [], []
    for i in range(3):
        x = synth_activation(24, 896, seed=300 + i).cuda()
        tasks.append(ops.GemvTask(pack, x, torch.empty(24, 896, dtype=torch.float32, device="cuda")))
        singles.append(ops.linear(pack, x, out_f32=True))
    ops.linear_grouped(tasks, 24)
    torch.cuda.synchronize()
    for t, s in zip(tasks, singles):
        assert torch.equal(t.y, s)


def test_grouped_equals_single_launches():
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight
    shapes = [(896, 896, 26), (128, 896, 26), (4864, 896, 26), (896, 4864, 26), (96, 320, 16),
              (40, 2080, 16)]
    tasks, singles = [], []
    for i, (r, c, ns) in enumerate(shapes):
        w = synth_weight(r, c, seed=100 + i).cuda()
        pack, _ = ops.quantize(w, n_states=ns)
        for m in (1,):
            x = synth_activation(m, c, seed=200 + i).cuda()
            y = torch.empty(m, r, dtype=torch.float32, device="cuda")
            tasks.append(ops.GemvTask(pack, x, y))
            singles.append(ops.linear(pack, x, out_f32=True))
    ops.linear_grouped(tasks, 1)
    torch.cuda.synchronize()
    for t, s in zip(tasks, singles):
        assert torch.equal(t.y, s)


def test_large_projection_properties():
    """[18944, 3584] (a 7B MLP projection, 67.9 M weights: beyond torch.quantile's
    limit, so no oracle run): quantizer invariants and GEMV vs the dequantized
    weight in fp64."""
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight
    rows, cols = 18944, 3584
    w = synth_weight(rows, cols, std=0.015, seed=7, device="cuda")
    pack, info = ops.quantize(w, n_states=26)
    k = int(round(rows * cols * 0.0156))
    assert not info["topk_fallback"]
    assert abs(info["n_res"] - k) <= max(2, k // 1000)
    w_hat = ops.dequant(pack)
    # residual positions hold the original weights exactly
    ent = pack.res_ent[: pack.n_res].long() & 0xFFFFFFFF
    rp = pack.res_ptr.long()
    counts = rp[1:] - rp[:-1]
    kg = (cols // 32 + 31) // 32
    b = torch.arange(counts.numel(), device="cuda")
    row_of = torch.repeat_interleave(b // kg, counts)  # buckets are (row, group), row major
    col = ent >> 16
    assert torch.equal(w_hat[row_of, col], w[row_of, col])
    # every non-residual weight is within half a lattice gap of sigma-scaled value
    x = synth_activation(2, cols, seed=3, device="cuda")
    y = ops.linear(pack, x, out_f32=True)
    y64 = (x.double() @ w_hat.double().T).cpu().numpy()
    _check_gemv(y, y64)


@pytest.mark.parametrize("shape,ns,m", [((896, 896), 26, 1), ((4864, 896), 26, 8),
                                        ((896, 4864), 16, 3), ((45, 1088), 26, 5),
                                        ((300, 2080), 26, 2), ((17, 96), 16, 7),
                                        ((130, 1056), 16, 1)])
def test_linear_shapes_batches_bias(shape, ns, m):
    """Odd tile counts (a phantom tile in the last pair), rows not a multiple
    of 16, every batch size, bias, both lattices."""
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight
    rows, cols = shape
    w = synth_weight(rows, cols, seed=rows + 3 * cols)
    p = O.quantize(_bits(w), n_states=ns)
    dp = ops.DevicePack.from_reference(p["quant_indices"], p["scales_f8"], p["residual_indices"],
                                       p["residual_values"], rows, cols, ns, device="cuda")
    x = synth_activation(m, cols, seed=9).cuda()
    bias = synth_activation(1, rows, seed=10)[0]
    y = ops.linear(dp, x, bias.cuda(), out_f32=True)
    torch.cuda.synchronize()
    _check_gemv(y, O.linear_f64(O.dequantize(p), _bits(x), _bits(bias)))


def _random_reference(rows, cols, ns, seed, frac=0.0156, pairs=True):
    rng = np.random.default_rng(seed)
    n = rows * cols
    q = rng.integers(0, ns, (n // 32, 32), dtype=np.uint8)
    sc = rng.integers(0, 0x7F, n // 32, dtype=np.uint8)
    k = int(round(n * frac))
    ri = rng.choice(n, k, replace=False)
    if pairs and k > 4:  # force some pairs whose two elements are both residuals
        ev = (ri[: k // 4] // 2) * 2
        ri = np.unique(np.concatenate([ri, ev, ev + 1]))
    ri = np.sort(np.unique(ri)).astype(np.int64)
    rv = rng.integers(0, 0xFFFF, ri.size, dtype=np.uint16)
    return q, sc, ri, rv


@pytest.mark.parametrize("shape,ns", [((45, 96), 26), ((200, 2080), 26), ((128, 512), 16), ((896, 4864), 26),
                                      ((33, 1088), 16), ((16, 32), 26)])
def test_device_ingest_matches_host(shape, ns):
    """The GPU converter from the reference format produces the host
    converter's device pack byte for byte (ragged row blocks, odd tile counts,
    several residual groups, adjacent residual pairs, both lattices)."""
    from cdq_lrr_b200 import ops
    rows, cols = shape
    q, sc, ri, rv = _random_reference(rows, cols, ns, seed=rows + cols + ns)
    host = ops.DevicePack.from_reference(q, sc, ri, rv, rows, cols, ns, device="cpu")
    dev = ops.DevicePack.from_reference_device(torch.from_numpy(q).cuda(), torch.from_numpy(sc).cuda(),
                                               torch.from_numpy(ri).cuda(),
                                               torch.from_numpy(rv.view(np.int16)).cuda(), rows, cols, ns)
    torch.cuda.synchronize()
    assert dev.n_res == host.n_res == ri.size
    assert torch.equal(dev.units.cpu(), host.units)
    assert torch.equal(dev.res_ptr.cpu(), host.res_ptr)
    assert torch.equal(dev.res_ent[: ri.size].cpu(), host.res_ent[: ri.size])
    assert torch.equal(dev.res_q[: ri.size].cpu(), host.res_q[: ri.size])


def test_device_ingest_golden_and_rejects_malformed(golden, golden_meta):
    """Golden reference packs ingested on the GPU dequantize to the oracle's
    w_hat; an out-of-range lattice index or unsorted residuals are refused."""
    from cdq_lrr_b200 import ops
    for name in CASES:
        ns = golden_meta["cases"][name]["n_states"]
        rows, cols = golden[f"{name}.weight"].shape
        p = {k: golden[f"{name}.{k}"] for k in ("quant_indices", "scales_f8", "residual_indices", "residual_values")}
        dp = ops.DevicePack.from_reference_device(
            torch.from_numpy(np.ascontiguousarray(p["quant_indices"])).cuda(),
            torch.from_numpy(np.ascontiguousarray(p["scales_f8"]).reshape(-1)).cuda(),
            torch.from_numpy(np.ascontiguousarray(p["residual_indices"]).astype(np.int64)).cuda(),
            torch.from_numpy(np.ascontiguousarray(p["residual_values"]).view(np.int16)).cuda(), rows, cols, ns)
        w_hat = ops.dequant(dp)
        torch.cuda.synchronize()
        assert _nan_equal(_bits(w_hat), golden[f"{name}.w_hat"]), name
    q, sc, ri, rv = _random_reference(32, 64, 26, seed=1)
    bad_q = q.copy()
    bad_q[0, 0] = 26
    with pytest.raises(ValueError):
        ops.DevicePack.from_reference_device(torch.from_numpy(bad_q).cuda(), torch.from_numpy(sc).cuda(),
                                             torch.from_numpy(ri).cuda(), torch.from_numpy(rv.view(np.int16)).cuda(),
                                             32, 64, 26)
    if ri.size > 1:
        bad_r = ri[::-1].copy()
        with pytest.raises(ValueError):
            ops.DevicePack.from_reference_device(torch.from_numpy(q).cuda(), torch.from_numpy(sc).cuda(),
                                                 torch.from_numpy(bad_r).cuda(),
                                                 torch.from_numpy(rv.view(np.int16)).cuda(), 32, 64, 26)


def test_device_file_decode_matches_host(tmp_path):
    """.cdq tile records unpacked on the GPU (256-tile spans from host
    checkpoints) give the host decoder's arrays: the CLI golden files and a
    written file with ragged spans, adjacent residuals and both lattices; and
    read_device_packs on a CUDA device builds the host path's packs byte for byte."""
    from pathlib import Path
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200 import pack_file as PF
    gold = Path(__file__).parent / "golden"
    files = [gold / "cli_26.cdq", gold / "cli_16.cdq"]
    for ns in (26, 16):
        tensors = {}
        for i, (r, c) in enumerate([(200, 2080), (45, 96), (33, 1088)]):
            q, sc, ri, rv = _random_reference(r, c, ns, seed=900 + i + ns)
            tensors[f"w{i}"] = {"rows": r, "cols": c, "quant_indices": q, "scales_f8": sc,
                                "residual_indices": ri, "residual_values": rv}
        p = tmp_path / f"rand{ns}.cdq"
        PF.write_cdq(p, tensors, n_states=ns)
        files.append(p)
    for path in files:
        data = path.read_bytes()
        ns, tabs = PF.scan_cdq(data)
        for t in tabs:
            h = PF.decode_tensor(data, ns, t)
            d = PF.decode_tensor_device(data, ns, t, "cuda")
            assert np.array_equal(d["quant_indices"].cpu().numpy(), h["quant_indices"])
            assert np.array_equal(d["scales_f8"].cpu().numpy(), h["scales_f8"])
            assert np.array_equal(d["residual_indices"].cpu().numpy(), h["residual_indices"])
            assert np.array_equal(d["residual_values"].cpu().numpy().view(np.uint16), h["residual_values"])
        dev = PF.read_device_packs(path, device="cuda")
        for t in tabs:
            h = PF.decode_tensor(data, ns, t)
            hp = ops.DevicePack.from_reference(h["quant_indices"], h["scales_f8"], h["residual_indices"],
                                               h["residual_values"], int(t.rows), int(t.cols), ns, device="cpu")
            dp = dev[t.name.decode()]
            assert torch.equal(dp.units.cpu(), hp.units) and torch.equal(dp.res_ptr.cpu(), hp.res_ptr)


def test_device_file_decode_rejects_bad_index():
    """A 26-state index of 26 or more in a record is refused by the device decoder."""
    from pathlib import Path
    from cdq_lrr_b200 import _lib as L
    from cdq_lrr_b200 import pack_file as PF
    data = bytearray((Path(__file__).parent / "golden" / "cli_26.cdq").read_bytes())
    ns, tabs = PF.scan_cdq(bytes(data))
    t = tabs[0]
    data[t.record_offset + 2] |= 0x1F  # first index of the first tile: 31
    with pytest.raises(L.CdqError):
        PF.decode_tensor_device(bytes(data), ns, t, "cuda")
