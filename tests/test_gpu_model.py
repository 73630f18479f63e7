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


def test_decode_step_kernels_match_torch():
    """The decode-step kernels against the HF modules / torch ops they replace:
    RMSNorm with the residual add (Qwen2RMSNorm after a bf16 add), SiLU(gate)
    * up, and rotary embedding + cache append + grouped-query attention against
    HF's apply_rotary_pos_emb and an fp32 softmax attention."""
    import ctypes as C
    from transformers.models.qwen2.modeling_qwen2 import Qwen2RMSNorm, apply_rotary_pos_emb
    from cdq_lrr_b200 import _lib as L
    lib, s = L.lib(), torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device="cuda").manual_seed(0)
    n = 896
    h = torch.randn(n, generator=g, device="cuda").bfloat16()
    d = torch.randn(n, generator=g, device="cuda").bfloat16()
    norm = Qwen2RMSNorm(n, eps=1e-6).cuda().bfloat16()
    with torch.no_grad():
        norm.weight.copy_(torch.rand(n, generator=g, device="cuda") + 0.5)
    ref_h = h + d
    ref = norm(ref_h)
    hh, out = h.clone(), torch.empty_like(h)
    assert lib.cdq_add_rmsnorm(hh.data_ptr(), d.data_ptr(), norm.weight.data_ptr(), C.c_float(1e-6),
                               out.data_ptr(), n, s) == 0
    torch.cuda.synchronize()
    assert torch.equal(hh, ref_h)
    assert (out.float() - ref.float()).abs().max().item() <= 2 ** -7 * ref.float().abs().max().item()
    gt = torch.randn(4864, generator=g, device="cuda").bfloat16()
    up = torch.randn(4864, generator=g, device="cuda").bfloat16()
    act = torch.empty_like(gt)
    assert lib.cdq_silu_mul(gt.data_ptr(), up.data_ptr(), act.data_ptr(), 4864, s) == 0
    torch.cuda.synchronize()
    ref_act = torch.nn.functional.silu(gt) * up
    assert (act.float() - ref_act.float()).abs().max().item() <= 2 ** -7 * ref_act.float().abs().max().item()
    # attention at position P over a random cache
    H, KV, hd, T, P = 14, 2, 64, 64, 37
    q = torch.randn(H * hd, generator=g, device="cuda").bfloat16()
    k = torch.randn(KV * hd, generator=g, device="cuda").bfloat16()
    v = torch.randn(KV * hd, generator=g, device="cuda").bfloat16()
    kc = torch.randn(1, KV, T, hd, generator=g, device="cuda").bfloat16()
    vc = torch.randn(1, KV, T, hd, generator=g, device="cuda").bfloat16()
    ang = torch.arange(T, device="cuda")[:, None].float() * (1e6 ** (-torch.arange(0, hd, 2, device="cuda").float() / hd))
    emb = torch.cat([ang, ang], -1)
    cos, sin = emb.cos().bfloat16().contiguous(), emb.sin().bfloat16().contiguous()
    pos = torch.tensor([P], dtype=torch.int32, device="cuda")
    out = torch.empty(H * hd, dtype=torch.bfloat16, device="cuda")
    kc2, vc2 = kc.clone(), vc.clone()
    assert lib.cdq_attn_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                               pos.data_ptr(), kc2.data_ptr(), vc2.data_ptr(), T, H, KV, hd, C.c_float(0.125),
                               out.data_ptr(), s) == 0
    torch.cuda.synchronize()
    qr, kr = apply_rotary_pos_emb(q.view(1, H, 1, hd), k.view(1, KV, 1, hd), cos[P][None, None], sin[P][None, None])
    assert torch.equal(kc2[0, :, P], kr[0, :, 0]) and torch.equal(vc2[0, :, P], v.view(KV, hd))
    assert torch.equal(kc2[:, :, :P], kc[:, :, :P])
    keys = kc2[0, :, : P + 1].float().repeat_interleave(H // KV, 0)
    vals = vc2[0, :, : P + 1].float().repeat_interleave(H // KV, 0)
    att = torch.softmax((qr[0, :, 0].float()[:, None, :] * keys).sum(-1) * 0.125, -1)
    ref = (att[:, :, None] * vals).sum(1).reshape(-1)
    assert (out.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item()


def test_fused_decode_step_matches_hf_one_layer():
    """One decoder layer (where bf16 summation-order noise has not compounded):
    the fused decode step's logits match the HF step's on the same tokens
    (teacher-forced), cosine >= 0.9999 at every step, and its greedy token
    stream replays deterministically from the CUDA graph."""
    from cdq_lrr_b200 import decode
    m = decode.build_model(seed=0, device="cuda", layers=1)
    decode.patch_cdq(m)
    prompt = _prompt(16, seed=5)
    steps = 8
    fd = decode.FusedDecoder(m, prompt.shape[1] + steps + 4)
    tok0 = fd.prefill(prompt)
    fd.capture()
    fused = []
    for _ in range(steps):
        fd.step()
        fused.append(fd.logits.float().clone())
    toks = torch.cat([tok0.view(1), fd.tokens[: steps - 1]])
    hf = decode.GreedyDecoder(m, prompt.shape[1] + steps + 4, use_graph=False)
    hf.prefill(prompt)
    with torch.no_grad():
        for t in range(steps):
            hf.ids.copy_(toks[t].view(1, 1))
            hf.pos.fill_(prompt.shape[1] + t)
            hf.mask[..., prompt.shape[1] + t] = 0
            ref = hf.model(input_ids=hf.ids, attention_mask=hf.mask, past_key_values=hf.cache,
                           cache_position=hf.pos, position_ids=hf.pos[None], use_cache=True).logits[:, -1].float()
            cos = torch.nn.functional.cosine_similarity(fused[t], ref, dim=-1).item()
            assert cos >= 0.9999, (t, cos)
    # the graph replays the same tokens as eager fused steps
    fe = decode.FusedDecoder(m, prompt.shape[1] + steps + 4)
    fe.prefill(prompt)
    for _ in range(steps):
        fe.step()
    assert torch.equal(fe.tokens[:steps], fd.tokens[:steps])


def test_fused_decode_full_model(cdq_model):
    """24 layers: the fused step's first-step logits against the HF step's
    (cosine within the bf16 noise floor of this random-init model) and a
    graphed 32-token greedy run with no kernel error."""
    from cdq_lrr_b200 import _lib as L
    from cdq_lrr_b200 import decode
    prompt = _prompt(32, seed=6)
    r = decode.fused_greedy_decode(cdq_model, prompt, 32)
    assert r["tokens"].shape == (1, 32) and r["tokens_per_s"] > 0
    fd = decode.FusedDecoder(cdq_model, 40)
    tok = fd.prefill(prompt)
    fd.step()
    hf = decode.GreedyDecoder(cdq_model, 40, use_graph=False)
    assert torch.equal(hf.prefill(prompt).view(-1), tok.view(-1))
    with torch.no_grad():
        hf.ids.copy_(tok.view(1, 1))
        hf.pos.fill_(32)
        hf.mask[..., 32] = 0
        ref = hf.model(input_ids=hf.ids, attention_mask=hf.mask, past_key_values=hf.cache, cache_position=hf.pos,
                       position_ids=hf.pos[None], use_cache=True).logits[:, -1].float()
    cos = torch.nn.functional.cosine_similarity(fd.logits.float(), ref, dim=-1).item()
    assert cos >= 0.998, cos
    assert L.kernel_error() == 0


def test_quality_report_matches_torch():
    """The on-device quality sums against torch float64 (bf16 and float32
    inputs), bit-identical on repeat, and the quantize-and-report loop over a
    one-layer model against torch's MSE / cosine of each weight and its w_hat."""
    from cdq_lrr_b200 import decode, ops, quality
    g = torch.Generator(device="cuda").manual_seed(3)
    for dt in (torch.bfloat16, torch.float32):
        a = torch.randn(1_000_003, generator=g, device="cuda").to(dt)
        b = (a.float() + 0.01 * torch.randn(a.numel(), generator=g, device="cuda")).to(dt)
        r = quality.compare(a, b)
        a64, b64 = a.double(), b.double()
        mse = (a64 - b64).pow(2).mean().item()
        cos = (a64 @ b64 / (a64.norm() * b64.norm())).item()
        assert abs(r["mse"] - mse) <= 1e-9 * mse and abs(r["cos"] - cos) <= 1e-12
        assert quality.compare(a, b) == r
    m = decode.build_model(seed=0, device="cuda", layers=1)
    orig = {n: mod.weight.detach().clone() for n, mod in m.named_modules() if isinstance(mod, nn.Linear)}
    rep = quality.quantize_with_report(m)
    assert rep["linears"] == 7 and 0.99 < rep["weight_cos"] <= 1.0
    for name, r in rep["per_linear"].items():
        w = orig[name].double().reshape(-1)
        wh = ops.dequant(m.get_submodule(name).device_pack).double().reshape(-1)
        assert abs(r["cos"] - (w @ wh / (w.norm() * wh.norm())).item()) <= 1e-10
        assert abs(r["mse"] - (w - wh).pow(2).mean().item()) <= 1e-9 * max(r["mse"], 1e-30)
    lr = quality.logit_report(torch.ones(4, 8, device="cuda"), torch.ones(4, 8, device="cuda"))
    assert lr["logits_mse"] == 0.0 and abs(lr["logits_cos"] - 1.0) < 1e-12


def _flat_cos(a, b):
    """The reference's statistic: one cosine over the flattened logits
    (code/cdq_lrr_qwen05.py:303-304)."""
    return float(torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0))


@pytest.fixture(scope="module")
def ref_model():
    """The same model with every projection holding its bit-exact w_hat in
    nn.Linear: the reference dequant path (F.linear(x, w_hat))."""
    from cdq_lrr_b200 import decode
    ref = decode.build_model(seed=0, device="cuda")
    decode.patch_cdq(ref)  # same packs: the quantizer is deterministic
    decode.materialize_reference(ref)
    return ref


@pytest.mark.xfail(strict=False, reason=(
    "measured on a B200: 0.99942 / 0.99926 / 0.99948 (prompts 11, 1, 2) against the reference "
    "dequant path; torch's own bf16 GEMM scores 0.99939 / 0.99926 / 0.99947 against the fp32 "
    "model, so no bf16 GEMM meets 0.9999 after 24 layers of this random-init model; the "
    "per-layer check below holds 0.9999 at every layer"))
def test_full_model_flat_logit_cosine_0_9999(cdq_model, ref_model):
    """North-star bar in the reference's own form: the cosine of the flattened
    logits of a prompt, fused model against the reference dequant path, at
    full depth (24 layers), >= 0.9999. The bar is kept as stated; the measured
    values are in the expected-failure reason."""
    ids = _prompt(32, seed=11)
    with torch.no_grad():
        ours = cdq_model(input_ids=ids).logits.float()
        ref = ref_model(input_ids=ids).logits.float()
    cos = _flat_cos(ours, ref)
    assert cos >= 0.9999, cos


def test_full_model_flat_logit_cosine_vs_fp32(cdq_model, ref_model):
    """The reference's statistic against the fp32-accumulated model: the fused
    model is at least as close to it as the reference dequant path (torch's
    bf16 GEMM) is, within 1e-4."""
    from cdq_lrr_b200 import decode
    from cdq_lrr_b200.synth import PROJ_NAMES
    ids = _prompt(32, seed=11)
    with torch.no_grad():
        ours = cdq_model(input_ids=ids).logits.float()
        ref = ref_model(input_ids=ids).logits.float()
    f32 = decode.build_model(seed=0, device="cuda")
    decode.patch_cdq(f32)
    decode.materialize_reference(f32)
    for layer in f32.model.layers:
        for name in PROJ_NAMES:
            parent = layer.self_attn if name in ("q_proj", "k_proj", "v_proj", "o_proj") else layer.mlp
            setattr(parent, name, _F32Linear(getattr(parent, name)))
    with torch.no_grad():
        want = f32(input_ids=ids).logits.float()
    del f32
    assert _flat_cos(ours, want) >= _flat_cos(ref, want) - MARGIN, (_flat_cos(ours, want), _flat_cos(ref, want))


def test_per_layer_teacher_forced_cosine_0_9999(cdq_model, ref_model):
    """Each decoder layer of the fused model, fed the reference model's own
    input to that layer, matches the reference layer's output (flattened
    cosine >= 0.9999 at every one of the 24 layers): the kernel's error per
    layer, separated from the compounding of bf16 noise over depth."""
    ids = _prompt(32, seed=12)
    layers_ref = ref_model.model.layers
    captured = [None] * len(layers_ref)
    handles = []
    for i, layer in enumerate(layers_ref):
        def pre(mod, args, kwargs, i=i):
            captured[i] = [args, kwargs, None]
        def post(mod, args, kwargs, out, i=i):
            captured[i][2] = out[0] if isinstance(out, tuple) else out
        handles.append(layer.register_forward_pre_hook(pre, with_kwargs=True))
        handles.append(layer.register_forward_hook(post, with_kwargs=True))
    try:
        with torch.no_grad():
            ref_model(input_ids=ids, use_cache=False)
    finally:
        for h in handles:
            h.remove()
    worst = 1.0
    with torch.no_grad():
        for i, layer in enumerate(cdq_model.model.layers):
            args, kwargs, want = captured[i]
            got = layer(*args, **kwargs)
            got = got[0] if isinstance(got, tuple) else got
            cos = _flat_cos(got.float(), want.float())
            worst = min(worst, cos)
            assert cos >= 0.9999, (i, cos)
    assert worst >= 0.9999


def test_lm_head_argmax_kernel():
    """The tied lm_head GEMV with its fused argmax: bf16 logits within one
    rounding of torch's bf16 GEMV, the argmax equal to torch.argmax of the
    kernel's own logits (first index among equal values; a NaN logit wins),
    the key cleared after every call, rows not a multiple of the kernel's row
    group."""
    import ctypes as C
    from cdq_lrr_b200 import _lib as L
    lib = L.lib()
    g = torch.Generator().manual_seed(5)
    V, H = 5003, 896
    w = (torch.randn(V, H, generator=g) * 0.05).to(torch.bfloat16).cuda()
    x = torch.randn(H, generator=g).to(torch.bfloat16).cuda()
    logits = torch.empty(V, dtype=torch.bfloat16, device="cuda")
    best = torch.zeros(1, dtype=torch.int64, device="cuda")
    nxt = torch.zeros(1, dtype=torch.int64, device="cuda")
    s = torch.cuda.current_stream().cuda_stream

    def run():
        L.check(lib.cdq_lm_head_argmax(C.c_void_p(w.data_ptr()), C.c_void_p(x.data_ptr()), V, H,
                                       C.c_void_p(logits.data_ptr()), C.c_void_p(best.data_ptr()),
                                       C.c_void_p(nxt.data_ptr()), C.c_void_p(s)), "cdq_lm_head_argmax")
        torch.cuda.synchronize()

    run()
    ref = torch.nn.functional.linear(x.view(1, -1), w).float().view(-1)
    got = logits.float()
    assert torch.all((got - ref).abs() <= ref.abs() * 2 ** -7 + 1e-3)
    assert int(nxt) == int(torch.argmax(logits))
    assert int(best) == 0
    # a tie at the maximum: the first of the equal rows wins
    top = int(torch.argmax(logits))
    with torch.no_grad():
        w[V - 2].copy_(w[top])
        w[3].copy_(w[top])
    run()
    assert int(nxt) == min(3, top)
    # a NaN logit is the maximum
    with torch.no_grad():
        w[V - 1, 7] = float("nan")
    run()
    assert int(nxt) == V - 1 and int(best) == 0


def test_embed_rmsnorm_kernel():
    """Embedding row + the first input norm in one launch: the same bits as a
    row copy followed by cdq_add_rmsnorm without a delta."""
    import ctypes as C
    from cdq_lrr_b200 import _lib as L
    lib = L.lib()
    g = torch.Generator().manual_seed(6)
    V, H = 1000, 896
    table = torch.randn(V, H, generator=g).to(torch.bfloat16).cuda()
    wn = (1 + 0.1 * torch.randn(H, generator=g)).to(torch.bfloat16).cuda()
    s = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for tok in (0, 17, V - 1):
        ids = torch.tensor([tok], dtype=torch.int64, device="cuda")
        h, out = torch.empty(H, dtype=torch.bfloat16, device="cuda"), torch.empty(H, dtype=torch.bfloat16, device="cuda")
        L.check(lib.cdq_embed_rmsnorm(C.c_void_p(ids.data_ptr()), C.c_void_p(table.data_ptr()), V,
                                      C.c_void_p(h.data_ptr()), C.c_void_p(wn.data_ptr()), 1e-6,
                                      C.c_void_p(out.data_ptr()), H, s), "cdq_embed_rmsnorm")
        h2, out2 = table[tok].clone(), torch.empty(H, dtype=torch.bfloat16, device="cuda")
        L.check(lib.cdq_add_rmsnorm(C.c_void_p(h2.data_ptr()), None, C.c_void_p(wn.data_ptr()), 1e-6,
                                    C.c_void_p(out2.data_ptr()), H, s), "cdq_add_rmsnorm")
        torch.cuda.synchronize()
        assert torch.equal(h, table[tok]) and torch.equal(out, out2)


def test_verify_pass_matches_sequential_steps(cdq_model):
    """The speculative verify pass over n positions gives, bit for bit, the
    greedy tokens and cache contents of n sequential one-token steps."""
    from cdq_lrr_b200 import decode
    prompt = _prompt(24, seed=8)
    seq = decode.FusedDecoder(cdq_model, 64)
    tok = seq.prefill(prompt)
    toks = [int(tok)]
    for _ in range(4):
        seq.step()
        toks.append(int(seq.tokens[len(toks) - 1]))
    # the same 5 positions in one pass, fed the tokens the sequential steps saw
    par = decode.FusedDecoder(cdq_model, 64)
    par.prefill(prompt)
    ver = decode.VerifyStep(par, 5)
    ver.ids.copy_(torch.tensor(toks, device="cuda"))
    par.pos.fill_(24)
    ver.run()
    torch.cuda.synchronize()
    assert ver.next.tolist()[:4] == toks[1:]
    for a, b in zip(seq.cache.layers, par.cache.layers):
        assert torch.equal(a.keys[:, :, :28], b.keys[:, :, :28])
        assert torch.equal(a.values[:, :, :28], b.values[:, :, :28])


@pytest.mark.parametrize("k", [1, 3])
def test_speculative_decode_matches_greedy(cdq_model, k):
    """Draft tokens from the 16-state tier, verified k + 1 at a time by the
    26-state model: the output equals plain greedy decoding of the 26-state
    model token for token (the reference README's draft/verify tiers)."""
    from cdq_lrr_b200 import decode
    from cdq_lrr_b200.quant import CAMKII_LATTICE_16
    draft = decode.build_model(seed=0, device="cuda")
    decode.patch_cdq(draft, lattice=CAMKII_LATTICE_16)
    prompt = _prompt(32, seed=4)
    plain = decode.fused_greedy_decode(cdq_model, prompt, 40)["tokens"].view(-1).cpu()
    spec = decode.speculative_greedy_decode(cdq_model, draft, prompt, 40, k=k)
    assert torch.equal(spec["tokens"].view(-1).cpu(), plain)
    assert spec["verifies"] <= 39 and 0.0 <= spec["accepted_per_verify"] <= k


def test_speculative_self_draft_accepts_every_token(cdq_model):
    """With the target as its own draft every proposal agrees: each verify
    accepts all k drafts and adds the bonus token, and the output is still
    plain greedy (the rewind-free path of the loop)."""
    from cdq_lrr_b200 import decode
    prompt = _prompt(32, seed=5)
    plain = decode.fused_greedy_decode(cdq_model, prompt, 25)["tokens"].view(-1).cpu()
    spec = decode.speculative_greedy_decode(cdq_model, cdq_model, prompt, 25, k=3)
    assert torch.equal(spec["tokens"].view(-1).cpu(), plain)
    assert spec["accepted_per_verify"] == 3.0 and spec["verifies"] == 6


def test_persistent_step_matches_one_kernel_steps(cdq_model):
    """The persistent decode step (one cooperative launch per token) gives,
    bit for bit, the logits, tokens and cache contents of the
    one-kernel-per-operation step, eagerly and replayed from a CUDA graph."""
    from cdq_lrr_b200 import decode
    prompt = _prompt(24, seed=13)
    a = decode.FusedDecoder(cdq_model, 64)
    b = decode.FusedDecoder(cdq_model, 64, persistent=True)
    ta, tb = a.prefill(prompt), b.prefill(prompt)
    assert torch.equal(ta, tb)
    for _ in range(6):
        a.step()
        b.step()
        torch.cuda.synchronize()
        assert torch.equal(a.logits, b.logits)
        assert torch.equal(a.next, b.next) and torch.equal(a.pos, b.pos) and torch.equal(a.count, b.count)
    assert b.step_error() == 0
    for x, y in zip(a.cache.layers, b.cache.layers):
        assert torch.equal(x.keys[:, :, :30], y.keys[:, :, :30])
        assert torch.equal(x.values[:, :, :30], y.values[:, :, :30])
    plain = decode.fused_greedy_decode(cdq_model, prompt, 24)["tokens"].view(-1).cpu()
    pers = decode.fused_greedy_decode(cdq_model, prompt, 24, persistent=True)
    assert torch.equal(pers["tokens"].view(-1).cpu(), plain)


def test_persistent_step_16_state_and_error_word():
    """The 16-state draft tier on the persistent step equals its one-kernel
    step; a table run with the wrong lattice size sets error word 3 and
    touches nothing; cdq_step_reset clears it."""
    from cdq_lrr_b200 import decode
    from cdq_lrr_b200.quant import CAMKII_LATTICE_16
    m16 = decode.build_model(seed=0, device="cuda")
    decode.patch_cdq(m16, lattice=CAMKII_LATTICE_16)
    prompt = _prompt(16, seed=14)
    plain = decode.fused_greedy_decode(m16, prompt, 12)["tokens"].view(-1).cpu()
    pers = decode.fused_greedy_decode(m16, prompt, 12, persistent=True)["tokens"].view(-1).cpu()
    assert torch.equal(pers, plain)
    fd = decode.FusedDecoder(m16, 32, persistent=True)
    fd.prefill(prompt)
    pos = fd.pos.clone()
    s = torch.cuda.current_stream().cuda_stream
    fd._call("cdq_decode_step", fd.table.data_ptr(), 26, s)  # prepared for 16 states
    torch.cuda.synchronize()
    assert fd.step_error() == 3 and torch.equal(fd.pos, pos)
    fd._call("cdq_step_reset", fd.table.data_ptr(), s)
    torch.cuda.synchronize()
    assert fd.step_error() == 0
    fd.step()
    torch.cuda.synchronize()
    assert fd.step_error() == 0 and int(fd.pos) == int(pos) + 1
