"""Tensor-parallel sharding: shards cut from the reference-format pack are
bit-identical parts of the unsharded weight; row-parallel partial products
summed across ranks (gloo, world size 2, CPU) equal the unsharded product; on
one GPU, ranks emulated in turn reproduce the unsharded fused linear."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import cdq_oracle as O


def _pack(rows, cols, seed, ns=26):
    from cdq_lrr_b200.synth import synth_weight
    w = synth_weight(rows, cols, seed=seed).view(torch.int16).numpy().view(np.uint16)
    return O.quantize(w, n_states=ns)


@pytest.mark.parametrize("rows,cols", [(96, 256), (45, 1088), (128, 96)])
@pytest.mark.parametrize("world", [2, 3, 4])
@pytest.mark.parametrize("kind", ["col", "row"])
def test_shards_are_exact_parts(rows, cols, world, kind):
    from cdq_lrr_b200 import tp
    p = _pack(rows, cols, seed=rows + cols)
    full = O.dequantize(p).reshape(rows, cols)
    covered = 0
    for r in range(world):
        s, rs, cs, off = tp.shard_reference(p, rows, cols, kind, world, r)
        sp = {**p, **s, "orig_shape": (rs, cs), "numel": rs * cs, "n_tiles": rs * cs // 32}
        part = O.dequantize(sp).reshape(rs, cs) if rs * cs else np.zeros((rs, cs), np.uint16)
        if kind == "col":
            assert np.array_equal(part, full[off:off + rs])
            covered += rs
        else:
            assert cs % 32 == 0
            assert np.array_equal(part, full[:, off:off + cs])
            covered += cs
    assert covered == (rows if kind == "col" else cols)


def _row_parallel_rank(rank, world, port, rows, cols, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cdq_lrr_b200 import tp
        from cdq_lrr_b200.synth import synth_activation
        p = _pack(rows, cols, seed=11)
        x = O.bf16_bits_to_f32(synth_activation(3, cols, seed=4).view(torch.int16).numpy().view(np.uint16))
        s, rs, cs, off = tp.shard_reference(p, rows, cols, "row", world, rank)
        sp = {**p, **s, "orig_shape": (rs, cs), "numel": rs * cs, "n_tiles": rs * cs // 32}
        w = O.bf16_bits_to_f32(O.dequantize(sp).reshape(rs, cs)).astype(np.float64)
        part = torch.from_numpy(x[:, off:off + cs].astype(np.float64) @ w.T)
        dist.all_reduce(part)
        full = O.bf16_bits_to_f32(O.dequantize(p).reshape(rows, cols)).astype(np.float64)
        ref = x.astype(np.float64) @ full.T
        q.put((rank, float(np.abs(part.numpy() - ref).max()), float(np.abs(ref).max())))
    finally:
        dist.destroy_process_group()


def test_row_parallel_allreduce_gloo():
    rows, cols, world = 64, 2048, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_row_parallel_rank, args=(r, world, port, rows, cols, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    for pr in procs:
        pr.join(timeout=300)
        assert pr.exitcode == 0
    res = [q.get(timeout=10) for _ in range(world)]
    for rank, err, scale in res:
        assert err <= 1e-9 * max(scale, 1.0), (rank, err, scale)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4])
def test_tp_emulated_on_one_gpu(world):
    from cdq_lrr_b200 import ops, tp
    from cdq_lrr_b200.synth import synth_activation
    for kind, rows, cols in (("col", 896, 896), ("row", 896, 4864)):
        p = _pack(rows, cols, seed=rows * 3 + cols)
        full = ops.DevicePack.from_reference(p["quant_indices"], p["scales_f8"], p["residual_indices"],
                                             p["residual_values"], rows, cols, 26, device="cuda")
        bias = synth_activation(1, rows, seed=8)[0].cuda()
        x = synth_activation(2, cols, seed=6).cuda()
        y_full32 = ops.linear(full, x, bias, out_f32=True)
        shards = [tp.TPLinear.from_reference(p, rows, cols, 26, kind, world, r, bias=bias) for r in range(world)]
        if kind == "col":
            y = torch.cat([s(x) for s in shards], dim=-1)
            # a row's computation does not depend on how rows are split: bit-identical
            assert torch.equal(y, ops.linear(full, x, bias))
        else:
            parts = [ops.linear(s.pack, x[..., s.offset:s.offset + s.pack.cols].contiguous(), None, out_f32=True)
                     for s in shards]
            y32 = torch.stack(parts).sum(0) + bias.float()
            err = (y32 - y_full32).abs().max().item()
            assert err <= 1e-3 * (y_full32.abs().max().item() + 1e-6), err


def test_allreduce_argument_checks():
    """The one-shot all-reduce rejects bad arguments before any device work."""
    import ctypes as C
    from cdq_lrr_b200 import _lib as L
    lib = L.lib()
    regions = (C.c_void_p * 8)()
    assert lib.cdq_allreduce_f32(None, 2, 0, 16, C.c_void_p(16), 8, None) == 3
    assert lib.cdq_allreduce_f32(regions, 9, 0, 16, C.c_void_p(16), 8, None) == 3    # > 8 ranks
    assert lib.cdq_allreduce_f32(regions, 2, 2, 16, C.c_void_p(16), 8, None) == 3    # rank >= world
    assert lib.cdq_allreduce_f32(regions, 2, 0, 16, C.c_void_p(16), 17, None) == 3   # n > cap
    assert lib.cdq_allreduce_f32(regions, 2, 0, 16, C.c_void_p(16), 8, None) == 3    # missing region
    h = L.cdq_ipc_handle()
    assert lib.cdq_ar_create(0, C.byref(C.c_void_p()), C.byref(h)) == 3
    assert lib.cdq_ar_open(None, None) == 3


@pytest.mark.gpu
def test_oneshot_allreduce_single_rank_graph():
    """One rank: the one-shot all-reduce is the identity, eagerly and replayed
    from a CUDA graph (alternating staging buffers), with no error recorded."""
    from cdq_lrr_b200 import _lib as L
    from cdq_lrr_b200 import tp
    ar = tp.OneShotAllReduce(5000)
    y = torch.randn(3, 1111, device="cuda")
    ref = y.clone()
    ar(y)
    assert torch.equal(y, ref)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ar(y)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            ar(y)
        for _ in range(5):
            g.replay()
    s.synchronize()
    assert torch.equal(y, ref)
    assert L.ar_error() == 0
    del g
    ar.close()


def _oneshot_rank(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from cdq_lrr_b200 import _lib as L
        from cdq_lrr_b200 import tp
        ar = tp.OneShotAllReduce(1 << 16)
        outs = []
        for it, n in enumerate((7, 3584, 65536, 3584, 1)):
            g = torch.Generator().manual_seed(1000 * it + rank)
            y = torch.randn(n, generator=g).cuda()
            ar(y)
            outs.append(y.cpu().numpy().copy())
        s = torch.cuda.Stream()
        y = torch.zeros(4096, device="cuda")
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=s):
                y.fill_(float(rank + 1))
                ar(y)
            for _ in range(4):
                graph.replay()
        s.synchronize()
        outs.append(y.cpu().numpy().copy())
        err = L.ar_error()
        del graph
        ar.close()
        q.put((rank, outs, err))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_oneshot_allreduce_two_ranks():
    """Two ranks on two GPUs: the sums equal the rank-order float32 sums bit for
    bit on both ranks, over alternating staging buffers, changing lengths and
    CUDA-graph replays. Skipped on a one-GPU machine."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 200
    procs = [ctx.Process(target=_oneshot_rank, args=(r, world, port, q)) for r in range(world)]
    for pr in procs:
        pr.start()
    res = {}
    try:
        for _ in range(world):
            rank, outs, err = q.get(timeout=240)
            res[rank] = (outs, err)
        for pr in procs:
            pr.join(timeout=60)
            assert pr.exitcode == 0
    finally:
        # a rank that died or hangs must not outlive the test holding GPU IPC regions
        for pr in procs:
            if pr.is_alive():
                pr.terminate()
                pr.join(timeout=30)
    for it, n in enumerate((7, 3584, 65536, 3584, 1)):
        parts = [torch.randn(n, generator=torch.Generator().manual_seed(1000 * it + r)).numpy() for r in range(world)]
        ref = np.float32(0) + parts[0]
        for p in parts[1:]:
            ref = (ref + p).astype(np.float32)
        for r in range(world):
            assert np.array_equal(res[r][0][it], ref), (it, r)
    for r in range(world):
        assert np.all(res[r][0][-1] == sum(range(1, world + 1)))
        assert res[r][1] == 0


@pytest.mark.gpu
def test_oneshot_allreduce_peer_wait_gives_up():
    """Failure detection without a fault: rank 0 of a two-rank all-reduce whose
    peer never arrives (the second region is never driven by anyone). With a
    short poll limit the flag wait gives up, the call records error 1 and the
    data keeps this rank's own partial; the context stays usable."""
    import ctypes as C
    from cdq_lrr_b200 import _lib as L
    lib = L.lib()
    cap = 4096
    regions = (C.c_void_p * 2)()
    handles = [L.cdq_ipc_handle(), L.cdq_ipc_handle()]
    for i in range(2):
        p = C.c_void_p()
        L.check(lib.cdq_ar_create(cap, C.byref(p), C.byref(handles[i])), "cdq_ar_create")
        regions[i] = p.value
    L.check(lib.cdq_ar_clear_error(), "cdq_ar_clear_error")
    L.check(lib.cdq_ar_set_spin_limit(1 << 12), "cdq_ar_set_spin_limit")
    try:
        y = torch.randn(cap, device="cuda")
        ref = y.clone()
        L.check(lib.cdq_allreduce_f32(regions, 2, 0, cap, C.c_void_p(y.data_ptr()), cap,
                                      C.c_void_p(torch.cuda.current_stream().cuda_stream)), "cdq_allreduce_f32")
        torch.cuda.synchronize()
        assert L.ar_error() == 1
        assert torch.equal(y, ref)
        z = torch.ones(8, device="cuda") * 2  # the context still works
        assert float(z.sum()) == 16.0
    finally:
        L.check(lib.cdq_ar_set_spin_limit(1 << 24), "cdq_ar_set_spin_limit")
        L.check(lib.cdq_ar_clear_error(), "cdq_ar_clear_error")
        for i in range(2):
            L.check(lib.cdq_ar_destroy(C.c_void_p(regions[i])), "cdq_ar_destroy")
