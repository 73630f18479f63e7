"""cdq_linear_noalloc: the fused linear for callers that cannot allocate.

Some hosts cannot call cudaMalloc on the decode path: a plugin whose host
process owns every byte of device memory through its own pool, or code where
an allocation (which may synchronise the device) is not allowed. For them
the library keeps its scratch (the row-block counters and per-group sums of
the streaming paths) in a fixed 4 MiB device array instead of a caller
workspace. These tests call it through the C ABI and check it
against cdq_linear on the same inputs, twice in a row (the array keeps the
previous call's contents), and check that a weight whose scratch would exceed
the array is refused. This file is collected last so that a run stopping at
the first failure has already run every other test.
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def _call_noalloc(L, pack, x, y, bias=None):
    st = pack.struct()
    return L.lib().cdq_linear_noalloc(
        C.byref(st), C.c_void_p(x.data_ptr()), x.shape[0], C.c_void_p(y.data_ptr()),
        C.c_void_p(bias.data_ptr()) if bias is not None else None,
        C.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("rows,cols,ns,m", [(256, 4864, 26, 1), (96, 2080, 16, 3),
                                            (4864, 896, 26, 8), (45, 1088, 26, 2)])
def test_noalloc_matches_workspace_linear(rows, cols, ns, m):
    from cdq_lrr_b200 import _lib as L
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight
    torch.cuda.set_device(0)
    w = synth_weight(rows, cols, seed=rows * 7 + cols).cuda()
    pack, _ = ops.quantize(w, n_states=ns)
    x = synth_activation(m, cols, seed=11).cuda()
    bias = synth_activation(1, rows, seed=12)[0].cuda()
    want = ops.linear(pack, x, bias)               # cdq_linear with its own workspace
    for _ in range(2):                             # two calls in a row on the shared array
        y = torch.full((m, rows), float("nan"), dtype=torch.bfloat16, device="cuda")
        L.check(_call_noalloc(L, pack, x, y, bias), "cdq_linear_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("rows,cols,ns,m", [(256, 4864, 26, 9), (128, 2080, 16, 16), (200, 1088, 26, 64)])
def test_noalloc_wide_batches_match_streaming_linear(rows, cols, ns, m):
    """Batches above 8 take the wide streaming kernel through the same array;
    cdq_linear with the tcgen05 tile path switched off takes the same kernel,
    so the outputs are bit-equal, again on two calls in a row."""
    from cdq_lrr_b200 import _lib as L
    from cdq_lrr_b200 import ops
    from cdq_lrr_b200.synth import synth_activation, synth_weight
    torch.cuda.set_device(0)
    w = synth_weight(rows, cols, seed=rows * 5 + cols).cuda()
    pack, _ = ops.quantize(w, n_states=ns)
    x = synth_activation(m, cols, seed=13).cuda()
    bias = synth_activation(1, rows, seed=14)[0].cuda()
    L.set_tile_min_batch(65)
    try:
        want = ops.linear(pack, x, bias)
    finally:
        L.set_tile_min_batch(16)
    for _ in range(2):
        y = torch.full((m, rows), float("nan"), dtype=torch.bfloat16, device="cuda")
        L.check(_call_noalloc(L, pack, x, y, bias), "cdq_linear_noalloc")
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int16), want.view(torch.int16))


def test_noalloc_rejects_oversized_scratch():
    """[8192, 28672] at m = 8 needs 7.3 MB of scratch: refused before any launch."""
    from cdq_lrr_b200 import _lib as L
    from cdq_lrr_b200 import ops
    torch.cuda.set_device(0)
    pack = ops.DevicePack.empty(8192, 28672, 26, 1, "cuda")
    x = torch.zeros(8, 28672, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(8, 8192, dtype=torch.bfloat16, device="cuda")
    assert _call_noalloc(L, pack, x, y) == 7  # CDQ_ERR_WORKSPACE
