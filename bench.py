#!/usr/bin/env python
"""Benchmark of the CDQ-LRR batch-1 dequant-GEMV on B200.

Workload (default, "qwen05"): the 168 projection weights (q/k/v/o/gate/up/down
of 24 layers) of a random-init Qwen2.5-0.5B-architecture model, bf16
N(0, 0.02^2) with 1.5% of entries scaled by U(8, 20), quantised with the
26-state lattice and stc-frac 0.0156 by the GPU quantizer. A step is one
batch-1 dequant-GEMV over every one of those weights (independent seeded
N(0, 1) bf16 activations), issued as one grouped launch replayed from a CUDA
graph. The packed working set (about 261 MB) is larger than the 126 MB L2,
so no L2 flush is needed between steps.

  value  = algorithmic bytes of the step / device time of the step (GB/s);
           algorithmic bytes = the reference .cdq tile records of every
           weight (2 + 20 index bytes + ceil(21 * residuals / 8) per tile)
           plus the activations read and the outputs written.
  e2e    = the same metric through the public grouped-linear call with the
           activations copied in from pinned host memory and the outputs
           copied back every step.
  roofline = the GEMV kernel's achieved bandwidth against the measured HBM
           copy bandwidth (MEASURED_PEAKS.json).
  cpu_baseline = the reference's CPU forward (dequant + F.linear, restated
           with the same torch ops) on a sample of the workload.

``--impl reference`` times that CPU forward alone, on all host threads.
Multi-GPU (torchrun): every rank runs its own replica of the workload (weak
scaling, no collective on the data path); value = total bytes of all ranks /
the slowest rank's time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "dequant-GEMV HBM GB/s (% of B200 peak); batch-1 decode tokens/s"
UNIT = "GB/s"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("qwen05", "tp7b", "tp70b", "msweep", "tpsweep"), default="qwen05",
                    help="qwen05: the 168-projection batch-1 GEMV (default); tp7b: the 28-layer "
                         "Qwen2.5-7B-shape projection stack, tensor-parallel over the ranks; tp70b: "
                         "the Llama-70B MLP shapes [28672,8192] and [8192,28672], tensor-parallel; "
                         "msweep: the qwen05 projections at batch 1, 4, 16 and 64; tpsweep: tp7b "
                         "(batch 1 and 8) on 1, 2, 4 ... GPUs and tp70b in both tiers on all GPUs, "
                         "one-shot and NCCL all-reduce, in one launch")
    ap.add_argument("--states", type=int, choices=(26, 16), default=26, help="tp70b: lattice size")
    ap.add_argument("--batch", type=int, default=1, help="tp7b: activation rows (1 or 8)")
    ap.add_argument("--allreduce", choices=("oneshot", "nccl"), default="oneshot",
                    help="tp7b/tp70b: the row-parallel reduction")
    ap.add_argument("--tp-worlds", type=int, nargs="*", default=None,
                    help="tpsweep: the tensor-parallel widths to run at batch 1 (default 1, 2, 4 ... up to "
                         "the number of GPUs); batch 8, NCCL and the 70B shapes run on all GPUs")
    ap.add_argument("--tile-min-batch", type=int, default=16,
                    help="smallest batch that takes the tcgen05 tile path (the library default is 16)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="target CPU time of the cpu_baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp7b", type=int, default=1,
                    help="1: add the tensor-parallel Qwen2.5-7B-shape stack over all ranks to the default "
                         "line (0: skip)")
    ap.add_argument("--batch-sweep", type=int, default=1,
                    help="1: add the batch 1/4/16/64 sweep of the same projections to the line (tile path "
                         "from batch 16, and the streaming path at 16 and 64 beside it)")
    ap.add_argument("--decode-tokens", type=int, default=256,
                    help="greedy tokens decoded after a 128-token prompt by the full "
                         "Qwen2.5-0.5B-architecture model (0: skip the decode measurement)")
    ap.add_argument("--packs", choices=("quantized", "random"), default="quantized",
                    help="quantized: weights quantised by the GPU quantizer (the benchmark); "
                         "random: seeded random valid packs built on the host, so that the "
                         "only kernels of the run are the GEMV's (profiling)")
    return ap.parse_args()


def workload_config() -> dict:
    return {"workload": "Qwen2.5-0.5B-shape CDQ-26 projections (24 layers x 7), batch-1 "
                        "dequant-GEMV, stc-frac 0.0156",
            "batch": 1, "projections": 168, "lattice_states": 26,
            "weights": "bf16 N(0,0.02^2) + 1.5% x U(8,20), seeded",
            "l2": "packed working set > 126 MB L2; no flush needed",
            "launch": "one grouped launch per step, CUDA graph replay"}


def layer_list():
    from cdq_lrr_b200.synth import QWEN05, layer_shapes
    out = []
    for layer in range(QWEN05["layers"]):
        for name, rows, cols in layer_shapes(QWEN05):
            out.append((f"model.layers.{layer}.{name}", rows, cols))
    return out


def measured_peak() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """SM clock and throttle reasons sampled through NVML while the GPU works."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown",
               0x4: "sw_power_cap", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int):
        self.samples = []
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self._stop = threading.Event()
        self.t = None

    def start(self):
        if not self.ok:
            return
        def run():
            while not self._stop.is_set():
                try:
                    mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                    rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                    self.samples.append((time.perf_counter(), mhz, rs))
                except Exception:
                    pass
                time.sleep(0.002)
        self.t = threading.Thread(target=run, daemon=True)
        self.t.start()

    def stop(self):
        self._stop.set()
        if self.t:
            self.t.join()

    def summary(self, t0: float, t1: float) -> dict:
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        win = [s for s in self.samples if t0 <= s[0] <= t1]
        note = None
        if len(win) < 3:
            win = self.samples[-20:]
            note = "timed region shorter than the sampling period: last samples of the run"
        mhz = statistics.median([s[1] for s in win]) if win else None
        reasons = set()
        for _, _, rs in win:
            for bit, name in self.REASONS.items():
                if rs & bit:
                    reasons.add(name)
        out = {"sm_mhz": mhz, "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
               "samples": len(win)}
        if note:
            out["note"] = note
        return out


def dist_setup(n_gpus: int):
    import torch
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # keep stdout to the one JSON line
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(ws, v: float) -> float:
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(ws, v: float) -> float:
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# --------------------------------------------------------------- CPU baseline


def oracle_workload():
    """The benchmark workload for the reference's CPU forward: all 168
    projections as reference-format packs (seeded random valid indices, fp8
    scales in [2^-6, 2^-2) and round(0.0156 * numel) residuals at random
    positions, the sizes of the quantized workload: the forward's cost does
    not depend on the values) and the GPU arm's activations. Returns the
    modules, the activations and the algorithmic bytes of one pass."""
    import numpy as np
    from oracle import cdq_oracle as O
    from oracle.cdq_oracle_torch import OracleCDQLinear
    from cdq_lrr_b200.synth import synth_activation
    mods, xs = [], []
    for i, (_, rows, cols) in enumerate(layer_list()):
        rng = np.random.default_rng(i)
        n = rows * cols
        k = int(round(n * 0.0156))
        sc = rng.integers(0x08, 0x28, n // 32, dtype=np.uint8)
        p = {"quant_indices": rng.integers(0, 26, (n // 32, 32), dtype=np.uint8),
             "scales_bf16": O.f32_to_bf16_bits(O.fp8_e4m3fn_decode(sc)),
             "residual_indices": np.sort(rng.choice(n, k, replace=False)).astype(np.int64),
             "residual_values": rng.integers(0x3C00, 0x3F00, k, dtype=np.uint16),
             "lattice": O.lattice_bits(26), "orig_shape": (rows, cols)}
        mods.append(OracleCDQLinear(p))
        xs.append(synth_activation(1, cols, seed=10000 + i))
    step_bytes = sum(m.reference_bytes() + x.numel() * 2 + m.orig_shape[0] * 2 for m, x in zip(mods, xs))
    return mods, xs, step_bytes


def cpu_baseline(seconds: float) -> dict:
    """The reference CPU forward over the whole workload (all 168 projections),
    repeated for about `seconds`, on every host thread."""
    import torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    mods, xs, step_bytes = oracle_workload()
    with torch.no_grad():
        for m, x in zip(mods, xs):
            m(x)  # warm-up
        times = []
        t_end = time.perf_counter() + seconds
        while time.perf_counter() < t_end or len(times) < 3:
            t0 = time.perf_counter()
            for m, x in zip(mods, xs):
                m(x)
            times.append(time.perf_counter() - t0)
    med = statistics.median(times)
    return {"value": step_bytes / med / 1e9, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"the whole workload (168 projections, {step_bytes / 1e6:.2f} MB algorithmic) per pass, "
                      f"{len(times)} passes, median {med * 1e3:.1f} ms/pass; reference forward = lattice gather, "
                      f"bf16 scale multiply, residual scatter, F.linear (torch CPU, restated in "
                      f"oracle/cdq_oracle_torch.py)",
            "ms_per_pass": med * 1e3}


# ------------------------------------------------------------------- our arm


def random_pack(rows: int, cols: int, seed: int, device, stc_frac: float = 0.0156, n_states: int = 26):
    """A valid pack with seeded random symbols, fp8 scales in [2^-6, 2^-2)
    and round(stc_frac * numel) residuals at random positions, laid out on the
    host (no kernel launches)."""
    import numpy as np
    from cdq_lrr_b200 import ops
    rng = np.random.default_rng(seed)
    n = rows * cols
    q = rng.integers(0, n_states, (n // 32, 32), dtype=np.uint8)
    scales = rng.integers(0x08, 0x28, n // 32, dtype=np.uint8)
    k = int(round(n * stc_frac))
    ridx = np.sort(rng.choice(n, k, replace=False)).astype(np.int64)
    rval = rng.integers(0x3C00, 0x3F00, k, dtype=np.uint16)
    return ops.DevicePack.from_reference(q, scales, ridx, rval, rows, cols, n_states, device=device)


def run_decode(new_tokens: int, prompt_len: int = 128, alg_per_weight: float | None = None) -> dict:
    """Batch-1 greedy decode of the full Qwen2.5-0.5B-architecture model
    (random init, 168 CDQ-26 projections through the fused GEMV, bf16 tied
    lm_head), static KV cache, one-token step replayed from a CUDA graph; and
    the bytes a token reads (alg_per_weight: the workload's algorithmic bytes
    per projection weight, from the GEMV measurement)."""
    import torch
    from cdq_lrr_b200.synth import QWEN05
    from cdq_lrr_b200 import decode
    model = decode.build_model(seed=0, device="cuda")
    decode.patch_cdq(model)
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, 151936, (1, prompt_len), generator=g).cuda()
    decode.fused_greedy_decode(model, ids, 8)  # warm-up (allocations, lattice set-up)
    chain = decode.fused_greedy_decode(model, ids, new_tokens)
    decode.fused_greedy_decode(model, ids, 8, persistent=True)
    pers = decode.fused_greedy_decode(model, ids, new_tokens, persistent=True)
    same = bool(torch.equal(chain["tokens"].cpu(), pers["tokens"].cpu()))
    # the reported step: the faster of the two (both give the same tokens)
    r = pers if pers["tokens_per_s"] >= chain["tokens_per_s"] else chain
    decode.greedy_decode(model, ids, 8)
    h = decode.greedy_decode(model, ids, new_tokens)
    # the 16-state draft tier (README's draft/verify tiers): same model, 16-state packs
    from cdq_lrr_b200.quant import CAMKII_LATTICE_16
    del model
    torch.cuda.empty_cache()
    draft = decode.build_model(seed=0, device="cuda")
    decode.patch_cdq(draft, lattice=CAMKII_LATTICE_16)
    decode.fused_greedy_decode(draft, ids, 8)
    d16 = decode.fused_greedy_decode(draft, ids, new_tokens)
    decode.fused_greedy_decode(draft, ids, 8, persistent=True)
    d16p = decode.fused_greedy_decode(draft, ids, new_tokens, persistent=True)
    d16 = d16p if d16p["tokens_per_s"] >= d16["tokens_per_s"] else d16
    # speculative decoding: the 16-state tier drafts, the 26-state model verifies
    target = decode.build_model(seed=0, device="cuda")
    decode.patch_cdq(target)
    spec = {}
    runs = [("16_state_draft_k2", draft, 2), ("16_state_draft_k4", draft, 4),
            ("self_draft_k4", target, 4)]  # self-draft: every proposal agrees (the loop's upper bound)
    for tag, dm, k in runs:
        sp = decode.speculative_greedy_decode(target, dm, ids, new_tokens, k=k)
        spec[tag] = {"tokens_per_s": round(sp["tokens_per_s"], 2),
                     "accepted_drafts_per_verify": round(sp["accepted_per_verify"], 3),
                     "tokens_per_verify": round(sp["tokens_per_verify"], 3), "verifies": sp["verifies"],
                     "verify_pass_ms": round(sp["verify_ms"], 4),
                     "same_tokens_as_greedy": bool(torch.equal(sp["tokens"].view(-1).cpu(),
                                                               r["tokens"].view(-1).cpu()))}
    del target, draft
    torch.cuda.empty_cache()
    # bytes a token must read: the 168 projections' reference records (and their
    # activations and outputs), the tied bf16 lm_head, the KV cache at the mean
    # position of the run, one embedding row
    cfg = QWEN05
    proj = sum(rows * cols for _, rows, cols in layer_list())
    proj_bytes = int(round(proj * alg_per_weight)) if alg_per_weight else None
    lm_bytes = cfg["vocab"] * cfg["hidden"] * 2
    mean_pos = prompt_len + new_tokens / 2
    kv_bytes = int(cfg["layers"] * cfg["kv_heads"] * cfg["head_dim"] * 2 * 2 * mean_pos)
    tok_bytes = (proj_bytes or 0) + lm_bytes + kv_bytes + cfg["hidden"] * 2
    peak, peak_kind = measured_peak()
    out = {"tokens_per_s": round(r["tokens_per_s"], 2),
           "ms_per_token": round(r["decode_ms_per_token"], 4),
           "bytes_per_token": tok_bytes,
           "bytes_per_token_parts": {"projections": proj_bytes, "lm_head_bf16": lm_bytes, "kv_cache": kv_bytes},
           "roofline": {"bound": "hbm", "achieved_gb_s": round(tok_bytes * r["tokens_per_s"] / 1e9, 2),
                        "peak": peak, "frac": round(tok_bytes * r["tokens_per_s"] / 1e9 / peak, 4),
                        "peak_kind": f"of {peak_kind}"},
           "prefill_ms": round(r["prefill_ms"], 3), "prompt_tokens": prompt_len,
           "new_tokens": new_tokens, "cuda_graph": r["graphed"],
           "step": ("persistent decode step: one cooperative launch per token (every layer's norms, grouped "
                    "CDQ projections, rotary + cache append + GQA attention, SiLU-mul, the lm_head GEMV with "
                    "fused argmax and the token advance, grid-wide barriers between dependent steps)"
                    if r is pers else
                    "one-kernel-per-operation decode step, library kernels only (embedding + RMSNorm, per layer "
                    "add + RMSNorm, grouped CDQ projections, rotary + cache append + GQA attention, SiLU-mul; "
                    "lm_head GEMV with fused argmax; token advance), one CUDA graph per token, launches "
                    "programmatically dependent"),
           "persistent_step_tokens_per_s": round(pers["tokens_per_s"], 2),
           "one_kernel_per_op_step_tokens_per_s": round(chain["tokens_per_s"], 2),
           "steps_give_same_tokens": same,
           "hf_step_tokens_per_s": round(h["tokens_per_s"], 2),
           "draft_tier_16_state_tokens_per_s": round(d16["tokens_per_s"], 2),
           "speculative": spec,
           "speculative_note": "draft k tokens on the 16-state packs, verify k + 1 positions in one 26-state pass "
                               "(grouped CDQ linears at m = k + 1, multi-query attention), keep the agreeing "
                               "prefix plus the target's token; output identical to plain greedy. On this "
                               "random-init model the 16-state and 26-state greedy choices over 151936 near-flat "
                               "logits disagree, so drafts are rejected; the self-draft run shows the loop with "
                               "every draft accepted",
           "hf_step": "the same model through HF's Qwen2 forward (CDQ projections patched in), CUDA graph",
           "model": "Qwen2.5-0.5B architecture, random init, 168 CDQ-26 projections, bf16 tied lm_head",
           "timing": "CUDA events around the decode loop (device time incl. host launch gaps)"}
    return out


def run_ours(args) -> None:
    import numpy as np
    import torch
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight

    ws_, rank, local = dist_setup(args.gpus)
    kernel_name = ("res_sum_kernel<192> (residual pre-pass) then stream_kernel<26,1,192> (bulk-copy quad "
                   "ring + mma.sync, group sums finished in the kernel); one grouped call = two launches per step")
    dev = torch.device("cuda", torch.cuda.current_device())

    # weights: generated and quantised on the GPU, one at a time
    tasks = []
    alg_bytes = 0
    packed_bytes = 0
    for i, (name, rows, cols) in enumerate(layer_list()):
        if args.packs == "random":
            pack = random_pack(rows, cols, seed=i, device=dev)
        else:
            w = synth_weight(rows, cols, std=0.02, seed=i, device=dev)
            pack, info = ops.quantize(w, n_states=26, stc_frac=0.0156)
            del w
        x = synth_activation(1, cols, seed=10000 + i, device=dev)
        y = torch.empty(1, rows, dtype=torch.bfloat16, device=dev)
        tasks.append(ops.GemvTask(pack, x, y))
        alg_bytes += pack.reference_bytes() + x.numel() * 2 + y.numel() * 2
        packed_bytes += pack.device_bytes()
    torch.cuda.synchronize()
    grouped = ops.GroupedLinear(tasks, m=1)
    launches_per_step = grouped.launches

    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(3):
            grouped()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        grouped()

    sampler = ClockSampler(local)
    sampler.start()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    stream.synchronize()
    barrier(ws_)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
    stream.synchronize()
    t1 = time.perf_counter()
    barrier(ws_)
    torch.cuda.synchronize()
    sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = max_over_ranks(ws_, ms)
    total_bytes = sum_over_ranks(ws_, float(alg_bytes))
    value = total_bytes / (ms_max * 1e-3) / 1e9
    kernel_gbs = alg_bytes / (ms * 1e-3) / 1e9  # one grouped launch per step

    # end to end: host activations in, host outputs out, through the public call.
    # Two device buffer sets; per step i (set b = i % 2) the input copy runs on a
    # copy-in stream, the grouped call on the compute stream, the output copy on
    # a copy-out stream, ordered by events, so step i's copies overlap steps
    # i - 1 and i + 1's kernels as in a serving loop; every step still moves its
    # own inputs in and its own outputs out.
    xs_host = torch.empty(sum(t.x.numel() for t in tasks), dtype=torch.bfloat16).pin_memory()
    ys_host = [torch.empty(sum(t.y.numel() for t in tasks), dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    xs_dev = [torch.empty_like(xs_host, device=dev) for _ in range(2)]
    ys_dev = [torch.empty_like(ys_host[0], device=dev) for _ in range(2)]
    e2e_calls = []
    for b in range(2):
        xo = yo = 0
        e2e_tasks = []
        for t in tasks:
            nx, ny = t.x.numel(), t.y.numel()
            xs_dev[b][xo:xo + nx].copy_(t.x.view(-1))
            e2e_tasks.append(ops.GemvTask(t.pack, xs_dev[b][xo:xo + nx].view_as(t.x),
                                          ys_dev[b][yo:yo + ny].view_as(t.y)))
            xo += nx
            yo += ny
        e2e_calls.append(ops.GroupedLinear(e2e_tasks, m=1))
    xs_host.copy_(xs_dev[0].cpu())
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev = {k: [torch.cuda.Event() for _ in range(2)] for k in ("in", "comp", "out")}
    used = [False, False]

    def e2e_step(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            if used[b]:
                s_in.wait_event(ev["comp"][b])  # step i - 2 has read this input buffer
            xs_dev[b].copy_(xs_host, non_blocking=True)
            ev["in"][b].record(s_in)
        with torch.cuda.stream(stream):
            stream.wait_event(ev["in"][b])
            if used[b]:
                stream.wait_event(ev["out"][b])  # step i - 2's outputs have left this buffer
            e2e_calls[b]()
            ev["comp"][b].record(stream)
        with torch.cuda.stream(s_out):
            s_out.wait_event(ev["comp"][b])
            ys_host[b].copy_(ys_dev[b], non_blocking=True)
            ev["out"][b].record(s_out)
        used[b] = True

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize()
    barrier(ws_)
    s_in.wait_stream(s_out)
    e0.record(s_in)
    for i in range(args.steps):
        e2e_step(args.warmup + i)
    s_out.wait_stream(s_in)
    s_out.wait_stream(stream)
    e1.record(s_out)
    torch.cuda.synchronize()
    barrier(ws_)
    ms_e2e = max_over_ranks(ws_, e0.elapsed_time(e1) / args.steps)
    e2e_value = total_bytes / (ms_e2e * 1e-3) / 1e9
    # the e2e outputs equal the device-resident run's
    last = (args.warmup + args.steps - 1) % 2
    ok = torch.equal(ys_host[last].to(dev), torch.cat([t.y.view(-1) for t in tasks]))

    peak, peak_kind = measured_peak()
    # DRAM bytes of one step (both launches) from the ncu capture of this
    # workload with these kernels, summarised in profiles/ (ncu cannot run
    # inside a timed run)
    traffic = None
    traffic_src = os.path.join("profiles", "stream_kernel_qwen05_168proj.md")
    try:
        with open(os.path.join(ROOT, traffic_src)) as f:
            for line in f:
                if line.startswith("dram_bytes_per_step:"):
                    traffic = int(line.split(":", 1)[1])
    except OSError:
        traffic = None

    # the Qwen2.5-7B-shape stack tensor-parallel over every rank of this run
    # (one-shot all-reduce, and NCCL beside it), in every line
    tp7 = None
    if args.tp7b:
        from cdq_lrr_b200.synth import QWEN7B, layer_shapes
        import torch.distributed as dist
        kinds = {"q_proj": "col", "k_proj": "col", "v_proj": "col", "o_proj": "row",
                 "gate_proj": "col", "up_proj": "col", "down_proj": "row"}
        s7 = [(n, r, c, kinds[n]) for n, r, c in layer_shapes(QWEN7B)]
        grp = dist.group.WORLD if ws_ > 1 else None
        tp_args = argparse.Namespace(steps=max(args.steps // 4, 10), warmup=max(args.warmup, 3))
        one = tp_measure(tp_args, s7, QWEN7B["layers"], 26, 1, "oneshot", grp, ws_, rank, local, check=True)
        nccl = tp_measure(tp_args, s7, QWEN7B["layers"], 26, 1, "nccl", grp, ws_, rank, local) if ws_ > 1 else None
        if rank == 0:
            def brief(r):
                return {"ms_per_step": r["ms_per_step"], "aggregate_gb_s": r["value"],
                        "per_gpu_gb_s": r["roofline"]["achieved_per_gpu"],
                        "per_gpu_roofline_frac": r["roofline"]["frac"], "allreduce_error": r["allreduce_error"],
                        "clocks": r["clocks"]}
            tp7 = {"workload": "Qwen2.5-7B-shape projection stack (28 layers x 7, 26-state, seeded random packs), "
                               f"batch 1, tensor-parallel x{ws_}: q/k/v/gate/up split by output rows, o/down "
                               "split along K with a float32 all-reduce of their partial outputs",
                   "n_gpus": ws_, "steps": tp_args.steps, "algorithmic_gb_all_ranks": one["algorithmic_gb_all_ranks"],
                   "oneshot": brief(one), "nccl": brief(nccl) if nccl else None,
                   "allreduce_match": one.get("allreduce_match", True if ws_ == 1 else None),
                   "allreduce_match_rule": "one-shot sums == rank-order float32 sums of the NCCL-all-gathered "
                                           "partials, bit for bit, on every rank (trivially true at one GPU)",
                   "nccl_max_rel_diff": one.get("nccl_max_rel_diff")}

    cpu = None
    if rank == 0 and ws_ == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_seconds)

    bsweep = None
    if rank == 0 and ws_ == 1 and args.batch_sweep:
        packs = [t.pack for t in tasks]
        bsweep = batch_sweep(packs, (1, 4, 16, 64), 50, 5, 16, dev)
        bsweep += batch_sweep(packs, (16, 64), 50, 5, 65, dev)
        torch.cuda.synchronize()

    dec = None
    if rank == 0 and ws_ == 1 and args.decode_tokens > 0:
        n_weights = sum(r * c for _, r, c in layer_list())
        dec = run_decode(args.decode_tokens, alg_per_weight=(alg_bytes - sum(t.x.numel() * 2 + t.y.numel() * 2
                                                                             for t in tasks)) / n_weights)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": ws_,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": ("synthetic (seeded random-init weights and activations)" if args.packs == "quantized"
                     else "synthetic (seeded random packs, profiling mode)"),
            "config": {**workload_config(), "packed_mb_reference_format": round(alg_bytes / 1e6, 2),
                       "packed_mb_device_layout": round(packed_bytes / 1e6, 2),
                       "parallelism": f"replicas x{ws_}" if ws_ > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": round(kernel_gbs, 2), "peak": peak,
                         "unit": "GB/s", "frac": round(kernel_gbs / peak, 4),
                         "peak_kind": f"of {peak_kind}", "traffic": traffic,
                         "traffic_over_algorithmic": round(traffic / alg_bytes, 4) if traffic else None,
                         "traffic_source": f"{traffic_src}: ncu dram__bytes_read.sum + dram__bytes_write.sum of "
                                           f"both launches of one step" if traffic else None,
                         "kernel": kernel_name},
            "e2e": {"value": round(e2e_value, 2), "unit": UNIT,
                    "h2d_bytes_per_step": int(xs_host.numel() * 2),
                    "d2h_bytes_per_step": int(ys_host[0].numel() * 2),
                    "ms_per_step": round(ms_e2e, 5), "outputs_match": bool(ok),
                    "pipeline": "per step: one pinned-host-to-device copy of all activations, the "
                                "grouped call, one device-to-pinned-host copy of all outputs, on "
                                "three streams with two buffer sets, so a step's copies overlap "
                                "its neighbours' kernels; timed from the first copy-in to the "
                                "last copy-out"},
            "gpu_launches": int(args.steps * launches_per_step),
            "clocks": sampler.summary(t0, t1),
            "cpu_baseline": cpu,
            "decode": dec,
            "batch_sweep": bsweep,
            "tp7b": tp7,
        }
        print(json.dumps(line), flush=True)
    if ws_ > 1:
        import torch.distributed as dist
        del graph
        dist.destroy_process_group()


def run_reference(args) -> None:
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the reference arm runs on rank 0 only
    import torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    mods, xs, step_bytes = oracle_workload()
    with torch.no_grad():
        for _ in range(args.warmup):
            for m, x in zip(mods, xs):
                m(x)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            for m, x in zip(mods, xs):
                m(x)
        dt = (time.perf_counter() - t0) / args.steps
    value = step_bytes / dt / 1e9
    sample = (f"each step = the reference CPU forward (restated with the same torch CPU ops) over the whole "
              f"workload: all 168 projections, {step_bytes / 1e6:.2f} MB algorithmic, batch 1")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT,
            "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(),
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads,
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def batch_sweep(packs, batches, steps: int, warmup: int, tile_min_batch: int, device) -> list[dict]:
    """Grouped calls over `packs` at each batch size (seeded activations), one
    CUDA graph per step, timed with CUDA events: the path (the tcgen05 tile
    path from tile_min_batch rows, else the streaming kernels), ms per step,
    algorithmic GB/s (packs read once per step + activations + outputs) and
    TFLOP/s."""
    import torch
    from cdq_lrr_b200 import _lib as L
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation
    ref_bytes = sum(p.reference_bytes() for p in packs)
    out = []
    L.set_tile_min_batch(tile_min_batch)
    try:
        for M in batches:
            tasks = []
            io_bytes = 0
            for i, p in enumerate(packs):
                x = synth_activation(M, p.cols, seed=10000 + i, device=device)
                y = torch.empty(M, p.rows, dtype=torch.bfloat16, device=device)
                io_bytes += (x.numel() + y.numel()) * 2
                tasks.append(ops.GemvTask(p, x, y))
            g = ops.GroupedLinear(tasks, m=M)
            stream = torch.cuda.Stream(device=device)
            with torch.cuda.stream(stream):
                for _ in range(3):
                    g()
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                g()
            with torch.cuda.stream(stream):
                for _ in range(warmup):
                    graph.replay()
            stream.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                e0.record(stream)
                for _ in range(steps):
                    graph.replay()
                e1.record(stream)
            stream.synchronize()
            ms = e0.elapsed_time(e1) / steps
            flops = 2.0 * M * sum(p.rows * p.cols for p in packs)
            path = ("tcgen05 tile" if M >= tile_min_batch else
                    "mma.sync stream" if M <= 8 else "mma.sync wide stream")
            out.append({"batch": M, "path": path, "ms_per_step": round(ms, 5),
                        "gb_s": round((ref_bytes + io_bytes) / (ms * 1e-3) / 1e9, 2),
                        "tflop_s": round(flops / (ms * 1e-3) / 1e12, 3)})
            del graph, g, tasks
    finally:
        L.set_tile_min_batch(16)
    return out


def run_msweep(args) -> None:
    """Batch sweep (1, 4, 16, 64) over the 168 Qwen2.5-0.5B-shape projections:
    seeded random valid packs, one grouped call per step (batches above 8
    decode each unit once and multiply ceil(M/8) n-tiles of 8 rows)."""
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(0)
    packs = [random_pack(rows, cols, seed=i, device=dev) for i, (_, rows, cols) in enumerate(layer_list())]
    sweep = batch_sweep(packs, (1, 4, 16, 64), args.steps, args.warmup, args.tile_min_batch, dev)
    first = sweep[0]
    line = {"metric": METRIC, "value": first["gb_s"], "unit": UNIT, "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": first["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded random packs)",
            "config": {"workload": "Qwen2.5-0.5B-shape CDQ-26 projections (168), batch sweep",
                       "batches": [1, 4, 16, 64]},
            "sweep": sweep}
    print(json.dumps(line), flush=True)


def run_tp7b(args) -> None:
    from cdq_lrr_b200.synth import QWEN7B, layer_shapes
    kinds = {"q_proj": "col", "k_proj": "col", "v_proj": "col", "o_proj": "row",
             "gate_proj": "col", "up_proj": "col", "down_proj": "row"}
    shapes = [(n, r, c, kinds[n]) for n, r, c in layer_shapes(QWEN7B)]
    run_tp(args, shapes, QWEN7B["layers"], 26,
           "Qwen2.5-7B-shape projection stack (28 layers x 7)")


def run_tp70b(args) -> None:
    from cdq_lrr_b200.synth import LLAMA70B_SHAPES
    (r1, c1), (r2, c2) = LLAMA70B_SHAPES
    shapes = [("up_proj", r1, c1, "col"), ("down_proj", r2, c2, "row")]
    run_tp(args, shapes, 4, args.states,
           f"Llama-70B MLP shapes [{r1},{c1}] (rows split) and [{r2},{c2}] (K split), 4 copies, "
           f"{args.states}-state")


def tp_allreduce_check(layers, oar, group, world: int) -> dict:
    """One step's row-parallel reductions, checked across ranks: the one-shot
    all-reduce's sums must equal, bit for bit, the float32 sums in rank order
    (starting from zero) of the partials gathered from every rank by NCCL, and
    are compared with NCCL's own all-reduce of the same partials (whose
    summation order is NCCL's). Every rank takes the same collective steps."""
    import torch
    import torch.distributed as dist
    match, worst = True, 0.0
    for g, ys in layers[:2]:
        g()
        parts = [y.clone() for y in ys]
        for y in ys:
            oar(y)
        for y, p in zip(ys, parts):
            gathered = [torch.empty_like(p) for _ in range(world)]
            dist.all_gather(gathered, p, group=group)
            ref = torch.zeros_like(p)
            for q in gathered:
                ref = ref + q
            match = match and bool(torch.equal(y, ref))
            nc = p.clone()
            dist.all_reduce(nc, group=group)
            worst = max(worst, float((nc - y).abs().max() / (y.abs().max() + 1e-30)))
    torch.cuda.synchronize()
    t = torch.tensor([1.0 if match else 0.0], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return {"allreduce_match": bool(t.item() == 1.0), "nccl_max_rel_diff": worst}


def tp_measure(args, shapes, n_layers: int, n_states: int, batch: int, allreduce: str, group,
               world: int, rank: int, local: int, check: bool = False) -> dict | None:
    """Tensor-parallel GEMV stack on the ranks of `group` (world ranks): per
    layer, q/k/v/gate/up split by output rows (no collective) and o/down split
    along K with a float32 all-reduce of their partial outputs, by the
    one-shot peer-memory kernel (allreduce "oneshot") or NCCL ("nccl"). Each
    rank holds seeded random valid packs of its shards (the GEMV's speed does
    not depend on the code values; the sharding itself is tested for
    exactness separately). A step = every layer's grouped shard GEMV plus its
    two all-reduces, replayed from one CUDA graph. Returns the result on the
    group's rank 0 (None elsewhere)."""
    import torch
    import torch.distributed as dist
    from cdq_lrr_b200 import ops, tp
    from cdq_lrr_b200.synth import synth_activation

    dev = torch.device("cuda", torch.cuda.current_device())
    m = batch
    shard_host = {}
    for i, (name, rows, cols, kind) in enumerate(shapes):
        if kind == "col":
            r0, r1 = tp.row_bounds(rows, world, rank)
            shard_host[name] = random_pack(r1 - r0, cols, seed=100 * rank + i, device="cpu", n_states=n_states)
        else:
            c0, c1 = tp.k_bounds(cols, world, rank)
            shard_host[name] = random_pack(rows, c1 - c0, seed=100 * rank + i, device="cpu", n_states=n_states)
    layers = []
    alg_bytes = 0
    max_red = 0
    for li in range(n_layers):
        tasks, reduce_ys = [], []
        for name, rows, cols, kind in shapes:
            pack = shard_host[name].to(dev)
            x = synth_activation(m, pack.cols, seed=li * 7 + len(tasks), device=dev)
            if kind == "col":
                y = torch.empty(m, pack.rows, dtype=torch.bfloat16, device=dev)
            else:
                y = torch.empty(m, pack.rows, dtype=torch.float32, device=dev)
                reduce_ys.append(y)
                max_red = max(max_red, y.numel())
            tasks.append(ops.GemvTask(pack, x, y))
            alg_bytes += pack.reference_bytes() + x.numel() * 2 + y.numel() * (2 if y.dtype == torch.bfloat16 else 4)
        layers.append((ops.GroupedLinear(tasks, m=m), reduce_ys))
    oar = tp.OneShotAllReduce(max_red, group=group) if world > 1 and allreduce == "oneshot" else None
    checked = tp_allreduce_check(layers, oar, group, world) if check and oar is not None else None

    def step():
        for g, ys in layers:
            g()
            for y in ys:
                if oar is not None:
                    oar(y)
                elif world > 1:
                    dist.all_reduce(y, group=group)

    def gbar():
        if world > 1:
            dist.barrier(group=group)

    def gmax(v: float, op=None) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=op or dist.ReduceOp.MAX, group=group)
        return float(t.item())

    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(stream):
        for _ in range(3):
            step()
    stream.synchronize()
    gbar()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    sampler = ClockSampler(local)
    sampler.start()
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    stream.synchronize()
    gbar()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
    stream.synchronize()
    t1 = time.perf_counter()
    gbar()
    torch.cuda.synchronize()
    sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    ms_max = gmax(ms)
    total = gmax(float(alg_bytes), dist.ReduceOp.SUM if world > 1 else None)
    del graph  # holds NCCL work: released before the process group
    from cdq_lrr_b200 import _lib as L
    err = L.ar_error()
    if oar is not None:
        oar.close()
    layers.clear()
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    peak, peak_kind = measured_peak()
    per_gpu = total / world / (ms_max * 1e-3) / 1e9
    return {"n_gpus": world, "batch": m, "allreduce": allreduce if world > 1 else "none",
            "value": round(total / (ms_max * 1e-3) / 1e9, 2), "ms_per_step": round(ms_max, 5),
            "algorithmic_gb_all_ranks": round(total / 1e9, 3),
            "roofline": {"bound": "hbm", "achieved_per_gpu": round(per_gpu, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(per_gpu / peak, 4), "peak_kind": f"of {peak_kind}"},
            "allreduce_error": err, **(checked or {}), "clocks": sampler.summary(t0, t1)}


def tp_line(label: str, r: dict, steps: int, warmup: int) -> dict:
    ar = {"oneshot": "a one-shot peer-memory float32 all-reduce (own kernel)",
          "nccl": "a float32 NCCL all-reduce", "none": "no collective (one GPU)"}[r["allreduce"]]
    return {"metric": METRIC, "value": r["value"], "unit": UNIT, "n_gpus": r["n_gpus"], "steps": steps,
            "warmup": warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded random packs of the shard shapes)",
            "config": {"workload": f"{label}, batch {r['batch']}, tensor-parallel x{r['n_gpus']}: column-parallel "
                                   f"weights split by rows, row-parallel weights split along K with {ar}",
                       "batch": r["batch"], "algorithmic_gb_all_ranks": r["algorithmic_gb_all_ranks"],
                       "parallelism": f"tp{r['n_gpus']}", "allreduce": r["allreduce"],
                       "launch": "one CUDA graph per step (GEMVs + all-reduces)",
                       "l2": "packed working set far above the 126 MB L2"},
            "roofline": r["roofline"], "clocks": r["clocks"]}


def run_tp(args, shapes, n_layers: int, n_states: int, label: str) -> None:
    ws_, rank, local = dist_setup(args.gpus)
    import torch.distributed as dist
    group = dist.group.WORLD if ws_ > 1 else None
    r = tp_measure(args, shapes, n_layers, n_states, args.batch, args.allreduce, group, ws_, rank, local)
    if r is not None:
        print(json.dumps(tp_line(label, r, args.steps, args.warmup)), flush=True)
    if ws_ > 1:
        dist.destroy_process_group()


def run_tpsweep(args) -> None:
    """The tensor-parallel configurations in one launch: the 7B-shape stack at
    batch 1 on each width of --tp-worlds (subgroups of the first ranks; the
    others wait) with the one-shot all-reduce; on all GPUs also batch 1 with
    NCCL, batch 8, and the 70B MLP shapes in both lattice tiers. One JSON line
    (rank 0) with every result in "sweep"."""
    import torch
    import torch.distributed as dist
    from cdq_lrr_b200.synth import LLAMA70B_SHAPES, QWEN7B, layer_shapes
    ws_, rank, local = dist_setup(args.gpus)
    kinds = {"q_proj": "col", "k_proj": "col", "v_proj": "col", "o_proj": "row",
             "gate_proj": "col", "up_proj": "col", "down_proj": "row"}
    s7 = [(n, r, c, kinds[n]) for n, r, c in layer_shapes(QWEN7B)]
    (r1, c1), (r2, c2) = LLAMA70B_SHAPES
    s70 = [("up_proj", r1, c1, "col"), ("down_proj", r2, c2, "row")]
    worlds = [w for w in (1, 2, 4, 8) if w <= ws_ and (args.tp_worlds is None or w in args.tp_worlds)]
    if ws_ not in worlds:
        worlds.append(ws_)
    runs = []
    for w in worlds:
        runs.append(("7b", s7, QWEN7B["layers"], 26, 1, "oneshot", w))
    if ws_ > 1:
        runs.append(("7b", s7, QWEN7B["layers"], 26, 1, "nccl", ws_))
    runs.append(("7b", s7, QWEN7B["layers"], 26, 8, "oneshot", ws_))
    for ns in (26, 16):
        runs.append(("70b", s70, 4, ns, 1, "oneshot", ws_))
    results = []
    groups = {}
    for w in worlds:  # every rank creates every subgroup, in the same order
        groups[w] = dist.new_group(list(range(w))) if ws_ > 1 else None
    for tag, shapes, nl, ns, b, ar, w in runs:
        if rank < w:
            g = groups[w] if w > 1 else None
            r = tp_measure(args, shapes, nl, ns, b, ar, g, w, rank, local)
            if r is not None:
                r["workload"] = tag if tag == "7b" else f"70b-{ns}"
                results.append(r)
        if ws_ > 1:
            dist.barrier()
    if rank == 0:
        head = next((r for r in results if r["n_gpus"] == ws_ and r["workload"] == "7b"), results[0])
        line = tp_line("Qwen2.5-7B-shape projection stack (28 layers x 7)", head, args.steps, args.warmup)
        line["config"]["workloads"] = {"7b": "Qwen2.5-7B-shape projection stack (28 layers x 7), 26-state",
                                       "70b-26": f"Llama-70B MLP shapes [{r1},{c1}] and [{r2},{c2}], 4 copies, 26-state",
                                       "70b-16": f"Llama-70B MLP shapes [{r1},{c1}] and [{r2},{c2}], 4 copies, 16-state"}
        line["sweep"] = results
        print(json.dumps(line), flush=True)
    if ws_ > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    from cdq_lrr_b200 import _lib
    _lib.set_tile_min_batch(args.tile_min_batch)
    if args.workload == "tp7b":
        run_tp7b(args)
    elif args.workload == "tp70b":
        run_tp70b(args)
    elif args.workload == "msweep":
        run_msweep(args)
    elif args.workload == "tpsweep":
        run_tpsweep(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
