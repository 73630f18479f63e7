"""Full-model parity and decode on the GPU: a Qwen2.5-0.5B-architecture model
(random init, outlier-bearing projections) with every projection replaced by
the fused CDQLinear, against the same model whose projections hold the
bit-exact w_hat: (a) in nn.Linear (torch's bf16 GEMM: the reference
CDQLinear.forward semantics, F.linear(x, w_hat), code/cdq_lrr_qwen05.py:
196-198) and (b) in an fp32-accumulated linear rounded once to bf16 (the
high-precision reference).

Bar: the fused model's logits are at least as close to (b) as torch's own
bf16 GEMM (a) is, within 1e-4 of cosine, at every position. A fixed 0.9999
logit cosine is not reachable on this 24-layer random-init model by any bf16
GEMM: two correct bf16 GEMMs with different summation orders differ at about
0.9988 after 24 layers, while one layer stays above 0.99998."""
import pytest
import torch
import torch.nn as nn

pytestmark = pytest.mark.gpu

MARGIN = 1e-4


@pytest.fixture(scope="module")
def cdq_model():
    from cdq_lrr_b200 import decode
    model = decode.build_model(seed=0, device="cuda")
    decode.patch_cdq(model)
    return model


def _prompt(n, seed=1, vocab=151936):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (1, n), generator=g).cuda()


class _F32Linear(nn.Module):
    """y = round_bf16(x @ w^T + b) with fp32 products and sums."""

    def __init__(self, lin: nn.Linear):
        super().__init__()
        self.w = lin.weight.detach().float()
        self.b = None if lin.bias is None else lin.bias.detach().float()

    def forward(self, x):
        y = x.float() @ self.w.T
        if self.b is not None:
            y = y + self.b
        return y.to(torch.bfloat16)


def _cos_min(a, b):
    return float(torch.nn.functional.cosine_similarity(a[0], b[0], dim=-1).min())


def test_full_model_logits_cosine(cdq_model):
    from cdq_lrr_b200 import decode
    from cdq_lrr_b200.synth import PROJ_NAMES
    ids = _prompt(32)
    with torch.no_grad():
        ours = cdq_model(input_ids=ids).logits.float()
    ref = decode.build_model(seed=0, device="cuda")
    decode.patch_cdq(ref)  # same packs: the quantizer is deterministic
    decode.materialize_reference(ref)
    with torch.no_grad():
        ref_bf16 = ref(input_ids=ids).logits.float()
    for layer in ref.model.layers:
        for name in PROJ_NAMES:
            parent = layer.self_attn if name in ("q_proj", "k_proj", "v_proj", "o_proj") else layer.mlp
            setattr(parent, name, _F32Linear(getattr(parent, name)))
    with torch.no_grad():
        ref_f32 = ref(input_ids=ids).logits.float()
    del ref
    assert torch.isfinite(ours).all()
    floor = _cos_min(ref_bf16, ref_f32)
    assert _cos_min(ours, ref_f32) >= floor - MARGIN, (_cos_min(ours, ref_f32), floor)
    assert _cos_min(ours, ref_bf16) >= floor - MARGIN, (_cos_min(ours, ref_bf16), floor)


def test_greedy_decode_graph_matches_eager(cdq_model):
    from cdq_lrr_b200 import decode
    ids = _prompt(16, seed=2)
    eager = decode.greedy_decode(cdq_model, ids, 12, use_graph=False)
    graphed = decode.greedy_decode(cdq_model, ids, 12, use_graph=True)
    assert torch.equal(eager["tokens"], graphed["tokens"])
    assert eager["tokens_per_s"] > 0 and graphed["tokens_per_s"] > 0


def test_one_layer_model_logits_cosine_0_9999():
    """Where bf16 summation-order noise has not compounded (one decoder layer),
    the fixed 0.9999 logit-cosine bar holds against torch's bf16 GEMM."""
    from cdq_lrr_b200 import decode
    ids = _prompt(32, seed=3)
    m = decode.build_model(seed=0, device="cuda", layers=1)
    decode.patch_cdq(m)
    with torch.no_grad():
        ours = m(input_ids=ids).logits.float()
    decode.materialize_reference(m)
    with torch.no_grad():
        ref = m(input_ids=ids).logits.float()
    assert _cos_min(ours, ref) >= 0.9999, _cos_min(ours, ref)
