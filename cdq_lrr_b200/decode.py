"""Batch-1 greedy decode of a Qwen2.5-0.5B-architecture model whose 168
projections run through the fused CDQ-LRR dequant-GEMV.

Mirrors the reference's model path: the reference quantizes every q/k/v/o/
gate/up/down projection of a Qwen2 model and patches a CDQLinear into its
place (code/cdq_lrr_qwen05.py:276-297), then runs the HF model unchanged
(code/cdq_lrr_qwen05.py:300-330). Weights here are random-init of that
architecture (no checkpoint is available): N(0, 0.02^2) with 1.5% of the
projection entries scaled by U(8, 20), seeded.

Decode runs with a static KV cache; the one-token step is captured in a CUDA
graph when HF's forward allows it (no host synchronisation in the step), and
replayed per token.
"""
from __future__ import annotations

import ctypes as C
import time

import torch
import torch.nn as nn

from .quant import CDQLinear
from .synth import PROJ_NAMES, QWEN05, synth_weight


def qwen05_config():
    from transformers import Qwen2Config
    c = QWEN05
    return Qwen2Config(vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=c["inter"],
                       num_hidden_layers=c["layers"], num_attention_heads=c["heads"],
                       num_key_value_heads=c["kv_heads"], head_dim=c["head_dim"],
                       tie_word_embeddings=True, max_position_embeddings=4096,
                       torch_dtype=torch.bfloat16)


def build_model(seed: int = 0, device="cuda", layers: int | None = None):
    """Random-init Qwen2.5-0.5B-architecture model in bf16 with outlier-bearing projections."""
    from transformers import Qwen2ForCausalLM
    cfg = qwen05_config()
    if layers is not None:
        cfg.num_hidden_layers = layers
    torch.manual_seed(seed)
    with torch.device(device):
        model = Qwen2ForCausalLM(cfg).to(torch.bfloat16)
    with torch.no_grad():
        for i, layer in enumerate(model.model.layers):
            for j, name in enumerate(PROJ_NAMES):
                mod = _proj(layer, name)
                rows, cols = mod.weight.shape
                mod.weight.copy_(synth_weight(rows, cols, std=0.02, seed=1000 + 7 * i + j,
                                              device=mod.weight.device))
    model.eval()
    return model


def _proj(layer, name: str) -> nn.Module:
    return getattr(layer.self_attn if name.endswith(("q_proj", "k_proj", "v_proj", "o_proj"))
                   else layer.mlp, name)


def _set_proj(layer, name: str, mod: nn.Module) -> None:
    parent = layer.self_attn if name in ("q_proj", "k_proj", "v_proj", "o_proj") else layer.mlp
    setattr(parent, name, mod)


def patch_cdq(model, lattice=None) -> dict:
    """Quantize every projection on the GPU and swap in the fused CDQLinear
    (the reference's quantize_model loop, code/cdq_lrr_qwen05.py:276-297).
    Returns {module name: reference-format pack}."""
    packs = {}
    for i, layer in enumerate(model.model.layers):
        for name in PROJ_NAMES:
            lin = _proj(layer, name)
            cdq, pack = CDQLinear.from_linear(lin, lattice=lattice)
            _set_proj(layer, name, cdq)
            packs[f"model.layers.{i}.{name}"] = pack
    return packs


def materialize_reference(model) -> None:
    """Replace every CDQLinear by an nn.Linear holding its w_hat (bit-exact),
    i.e. the reference CDQLinear.forward = F.linear(x, w_hat, bias)
    (code/cdq_lrr_qwen05.py:196-198) with torch's own GEMM."""
    for layer in model.model.layers:
        for name in PROJ_NAMES:
            cdq = _proj(layer, name)
            w = cdq.dequant_weight()
            lin = nn.Linear(cdq.in_features, cdq.out_features, bias=cdq.bias is not None,
                            device=w.device, dtype=torch.bfloat16)
            with torch.no_grad():
                lin.weight.copy_(w)
                if cdq.bias is not None:
                    lin.bias.copy_(cdq.bias)
            _set_proj(layer, name, lin)


class GreedyDecoder:
    """Static-cache greedy decoder for batch 1; the per-token step replays a
    CUDA graph when capture succeeds (`self.graphed`), else runs eagerly."""

    def __init__(self, model, max_len: int, use_graph: bool = True):
        from transformers import StaticCache
        self.model = model
        self.dev = next(model.parameters()).device
        self.cache = StaticCache(config=model.config, max_cache_len=max_len)
        self.ids = torch.zeros(1, 1, dtype=torch.long, device=self.dev)
        self.pos = torch.zeros(1, dtype=torch.long, device=self.dev)
        # explicit additive mask over the static cache: 0 for written positions,
        # -inf elsewhere (so the captured step carries no host-side mask logic)
        self.mask = torch.full((1, 1, 1, max_len), float("-inf"), dtype=torch.bfloat16, device=self.dev)
        self.next_tok = None
        self.graph = None
        self.use_graph = use_graph
        self.graphed = False

    def _step(self) -> torch.Tensor:
        out = self.model(input_ids=self.ids, attention_mask=self.mask, past_key_values=self.cache,
                         cache_position=self.pos, position_ids=self.pos[None], use_cache=True)
        return out.logits[:, -1].argmax(-1, keepdim=True)

    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        n = prompt.shape[1]
        pos = torch.arange(n, device=self.dev)
        out = self.model(input_ids=prompt, past_key_values=self.cache, cache_position=pos,
                         position_ids=pos[None], use_cache=True, logits_to_keep=1)
        self.mask[..., :n] = 0
        return out.logits[:, -1].argmax(-1, keepdim=True)

    @torch.no_grad()
    def capture(self, at: int) -> None:
        """Warm up and capture the one-token step; the warm-up steps write the
        cache at positions at, at+1, which decoding overwrites later."""
        if not self.use_graph:
            return
        self.pos.fill_(at)
        self.mask[..., at] = 0  # the warm-up steps attend to position `at` like the first real step
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.next_tok = self._step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.next_tok = self._step()
            self.graph = g
            self.graphed = True
        except Exception:  # HF forward not capturable in this version: eager steps
            self.graph = None
            self.graphed = False
            torch.cuda.synchronize(self.dev)
        self._rewind(at)

    def _rewind(self, at: int) -> None:
        """The static cache writes each step at its own on-device counter (it
        does not read cache_position), which the warm-up steps advanced: set
        it back to the next real position."""
        for layer in getattr(self.cache, "layers", []):
            n = getattr(layer, "cumulative_length", None)
            if torch.is_tensor(n):
                n.fill_(at)

    @torch.no_grad()
    def step(self, tok: torch.Tensor, position: int) -> torch.Tensor:
        self.ids.copy_(tok)
        self.pos.fill_(position)
        self.mask[..., position] = 0
        if self.graph is not None:
            self.graph.replay()
            return self.next_tok
        return self._step()


@torch.no_grad()
def greedy_decode(model, prompt: torch.Tensor, new_tokens: int, use_graph: bool = True) -> dict:
    """Prefill `prompt` (1, P) and decode `new_tokens` greedy tokens.
    Returns the tokens and the device-timed prefill and per-token times."""
    P = prompt.shape[1]
    dec = GreedyDecoder(model, P + new_tokens + 2, use_graph=use_graph)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    e[0].record()
    tok = dec.prefill(prompt)
    e[1].record()
    dec.capture(P)
    toks = [tok]
    e[2].record()
    for t in range(new_tokens - 1):
        tok = dec.step(tok, P + t).clone()
        toks.append(tok)
    e[3].record()
    torch.cuda.synchronize()
    steps = max(new_tokens - 1, 1)
    return {"tokens": torch.cat(toks, dim=1), "prefill_ms": e[0].elapsed_time(e[1]),
            "decode_ms_per_token": e[2].elapsed_time(e[3]) / steps,
            "tokens_per_s": 1e3 * steps / max(e[2].elapsed_time(e[3]), 1e-9), "graphed": dec.graphed}


class FusedDecoder:
    """Batch-1 greedy decoder whose one-token step runs on this library's
    kernels only: the embedding row with the first input norm; per layer, the
    fused residual-add + RMSNorm, one grouped CDQ call for q/k/v (with their
    biases), the rotary embedding + cache append + grouped-query attention
    kernel, o_proj, the second add + RMSNorm, one grouped call for gate/up,
    SiLU(gate) * up, down_proj; the final norm, the tied bf16 lm_head GEMV
    with its argmax, and the token advance. The step's token and position live
    on the device, so one CUDA graph of the step replays per token with no
    host work in between; every launch is programmatically dependent on the
    previous one, so launch latencies overlap. Prefill runs the
    HF model itself into the same static cache (the reference's forward,
    code/cdq_lrr_qwen05.py:300-330), whose [1, kv_heads, max_len, head_dim]
    tensors the attention kernel then reads and appends to.

    persistent=True runs the same step as one cooperative launch of the
    persistent decode-step kernel (cdq_decode_step: every layer, the lm_head
    and the advance in one kernel with grid-wide barriers), which computes the
    same bits without a launch per operation."""

    def __init__(self, model, max_len: int, persistent: bool = False):
        from transformers import StaticCache
        from . import _lib as L
        from . import ops
        self.L = L
        self.model = model
        cfg = model.config
        self.dev = next(model.parameters()).device
        self.max_len = max_len
        self.H = cfg.hidden_size
        self.n_heads, self.n_kv = cfg.num_attention_heads, cfg.num_key_value_heads
        self.hd = getattr(cfg, "head_dim", None) or self.H // self.n_heads
        self.eps = float(cfg.rms_norm_eps)
        self.cache = StaticCache(config=cfg, max_cache_len=max_len)
        bf16, dev = torch.bfloat16, self.dev
        pos_ids = torch.arange(max_len, device=dev)[None]
        with torch.no_grad():
            cos, sin = model.model.rotary_emb(torch.zeros(1, 1, self.H, dtype=bf16, device=dev), pos_ids)
        self.cos, self.sin = cos[0].contiguous(), sin[0].contiguous()
        z = lambda n, dt=bf16: torch.zeros(n, dtype=dt, device=dev)  # noqa: E731
        self.ids = z(1, torch.long)
        self.pos = z(1, torch.int32)
        self.count = z(1, torch.int32)
        self.tokens = z(max_len, torch.long)
        self.h, self.xn = z(self.H), z(self.H)
        qd, kvd = self.n_heads * self.hd, self.n_kv * self.hd
        self.q, self.k, self.v, self.att = z(qd), z(kvd), z(kvd), z(qd)
        self.o = z(self.H)
        self.inter = model.model.layers[0].mlp.gate_proj.out_features
        self.g, self.u, self.act, self.dn = z(self.inter), z(self.inter), z(self.inter), z(self.H)
        row = lambda t: t.view(1, -1)  # noqa: E731
        self.layers = []
        for layer in model.model.layers:
            a, mlp = layer.self_attn, layer.mlp
            T = lambda mod, x, y: ops.GemvTask(mod.device_pack, row(x), row(y), mod.bias)  # noqa: E731
            self.layers.append({
                "ln1": layer.input_layernorm.weight, "ln2": layer.post_attention_layernorm.weight,
                "qkv": ops.GroupedLinear([T(a.q_proj, self.xn, self.q), T(a.k_proj, self.xn, self.k),
                                          T(a.v_proj, self.xn, self.v)], m=1),
                "o": ops.GroupedLinear([T(a.o_proj, self.att, self.o)], m=1),
                "gu": ops.GroupedLinear([T(mlp.gate_proj, self.xn, self.g), T(mlp.up_proj, self.xn, self.u)], m=1),
                "down": ops.GroupedLinear([T(mlp.down_proj, self.act, self.dn)], m=1),
            })
        self.norm_w = model.model.norm.weight
        self.lm_w = model.lm_head.weight.contiguous()
        self.embed_w = model.model.embed_tokens.weight.contiguous()
        self.vocab = self.lm_w.shape[0]
        self.logits = torch.zeros(1, self.vocab, dtype=bf16, device=dev)
        self.best = z(1, torch.int64)   # the lm_head's argmax key (zero between steps)
        self.next = z(1, torch.int64)
        self.graph = None
        self.persistent = persistent
        self.table = None  # the persistent step's table, prepared once the cache exists (after prefill)

    def _prepare_persistent(self) -> None:
        """The persistent step's table: the model's shapes and buffers and,
        per layer, the seven projection jobs of the grouped calls above."""
        L = self.L
        p = lambda t: t.data_ptr()  # noqa: E731
        M = L.cdq_step_model()
        M.layers, M.hidden, M.heads, M.kv_heads = len(self.layers), self.H, self.n_heads, self.n_kv
        M.head_dim, M.inter, M.max_len, M.token_cap = self.hd, self.inter, self.max_len, self.max_len
        M.vocab, M.eps, M.scale = self.vocab, self.eps, float(self.hd) ** -0.5
        self.h1 = torch.zeros_like(self.h)
        for name, t in (("embed", self.embed_w), ("norm_w", self.norm_w), ("lm_w", self.lm_w), ("cos_t", self.cos),
                        ("sin_t", self.sin), ("pos", self.pos), ("ids", self.ids), ("tokens", self.tokens),
                        ("count", self.count), ("best", self.best), ("next", self.next), ("logits", self.logits),
                        ("h0", self.h), ("h1", self.h1), ("q", self.q), ("k", self.k), ("v", self.v),
                        ("att", self.att), ("o", self.o), ("g", self.g), ("u", self.u), ("dn", self.dn)):
            setattr(M, name, p(t))
        layers = (L.cdq_step_layer * len(self.layers))()
        ns = set()
        for li, (Ly, dst) in enumerate(zip(self.layers, layers)):
            qkv, o, gu, down = Ly["qkv"].jobs, Ly["o"].jobs, Ly["gu"].jobs, Ly["down"].jobs
            dst.q, dst.k, dst.v, dst.o = qkv[0], qkv[1], qkv[2], o[0]
            dst.gate, dst.up, dst.down = gu[0], gu[1], down[0]
            dst.ln1, dst.ln2 = p(Ly["ln1"]), p(Ly["ln2"])
            cl = self.cache.layers[li]
            dst.k_cache, dst.v_cache = p(cl.keys), p(cl.values)
            ns.update(t.pack.n_states for g in ("qkv", "o", "gu", "down") for t in Ly[g].tasks)
        if len(ns) != 1:
            raise ValueError("the persistent step needs one lattice size for every projection")
        self.n_states = ns.pop()
        nbytes = C.c_int64()
        L.check(L.lib().cdq_step_table_bytes(len(self.layers), C.byref(nbytes)), "cdq_step_table_bytes")
        self.table = torch.zeros(nbytes.value, dtype=torch.uint8, device=self.dev)
        self._step_model, self._step_layers = M, layers
        L.check(L.lib().cdq_step_prepare(C.byref(M), layers, self.table.data_ptr()), "cdq_step_prepare")

    def step_error(self) -> int:
        """The persistent step's error word (0: none)."""
        code = C.c_int32()
        self.L.check(self.L.lib().cdq_step_error(self.table.data_ptr(), C.byref(code)), "cdq_step_error")
        return code.value

    def _call(self, name: str, *args) -> None:
        self.L.check(getattr(self.L.lib(), name)(*args), name)

    def _step(self) -> None:
        p = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
        s = torch.cuda.current_stream(self.dev).cuda_stream
        if self.persistent:
            if self.table is None:
                self._prepare_persistent()
            self._call("cdq_decode_step", p(self.table), self.n_states, s)
            return
        for li, Ly in enumerate(self.layers):
            cl = self.cache.layers[li]
            if li == 0:  # the token's embedding row and the first input norm
                self._call("cdq_embed_rmsnorm", p(self.ids), p(self.embed_w), self.vocab, p(self.h), p(Ly["ln1"]),
                           self.eps, p(self.xn), self.H, s)
            else:
                self._call("cdq_add_rmsnorm", p(self.h), p(self.dn), p(Ly["ln1"]), self.eps, p(self.xn), self.H, s)
            Ly["qkv"]()
            self._call("cdq_attn_decode", p(self.q), p(self.k), p(self.v), p(self.cos), p(self.sin), p(self.pos),
                       p(cl.keys), p(cl.values), self.max_len, self.n_heads, self.n_kv, self.hd,
                       float(self.hd) ** -0.5, p(self.att), s)
            Ly["o"]()
            self._call("cdq_add_rmsnorm", p(self.h), p(self.o), p(Ly["ln2"]), self.eps, p(self.xn), self.H, s)
            Ly["gu"]()
            self._call("cdq_silu_mul", p(self.g), p(self.u), p(self.act), self.inter, s)
            Ly["down"]()
        self._call("cdq_add_rmsnorm", p(self.h), p(self.dn), p(self.norm_w), self.eps, p(self.xn), self.H, s)
        # the tied bf16 lm_head GEMV with its argmax fused in
        self._call("cdq_lm_head_argmax", p(self.lm_w), p(self.xn), self.vocab, self.H, p(self.logits),
                   p(self.best), p(self.next), s)
        self._call("cdq_decode_advance", p(self.next), p(self.ids), p(self.tokens), p(self.pos), p(self.count),
                   self.max_len, s)

    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        n = prompt.shape[1]
        pos = torch.arange(n, device=self.dev)
        out = self.model(input_ids=prompt, past_key_values=self.cache, cache_position=pos,
                         position_ids=pos[None], use_cache=True, logits_to_keep=1)
        tok = out.logits[:, -1].argmax(-1)
        self.reset(tok, n)
        if self.persistent and self.table is None:
            self._prepare_persistent()  # the static cache's tensors exist now
        return tok

    def reset(self, tok: torch.Tensor, position: int) -> None:
        self.ids.copy_(tok.view(1))
        self.pos.fill_(position)
        self.count.zero_()

    @torch.no_grad()
    def capture(self) -> None:
        """Two eager warm-up steps (they write the cache at the next two
        positions, which decoding overwrites), then the graph of one step;
        the token, position and count are restored afterwards."""
        tok, at = self.ids.clone(), int(self.pos.item())
        s = torch.cuda.Stream(device=self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self._step()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        self.reset(tok, at)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._step()
        self.graph = g
        self.reset(tok, at)

    @torch.no_grad()
    def step(self) -> None:
        if self.graph is not None:
            self.graph.replay()
        else:
            self._step()


@torch.no_grad()
def fused_greedy_decode(model, prompt: torch.Tensor, new_tokens: int, use_graph: bool = True,
                        persistent: bool = False) -> dict:
    """greedy_decode's contract on the fused decode step (FusedDecoder;
    persistent: the one-launch step)."""
    P = prompt.shape[1]
    dec = FusedDecoder(model, P + new_tokens + 2, persistent=persistent)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    e[0].record()
    tok = dec.prefill(prompt)
    e[1].record()
    if use_graph:
        dec.capture()
    e[2].record()
    for _ in range(new_tokens - 1):
        dec.step()
    e[3].record()
    torch.cuda.synchronize()
    steps = max(new_tokens - 1, 1)
    toks = torch.cat([tok.view(1, 1), dec.tokens[: new_tokens - 1].view(1, -1)], dim=1)
    return {"tokens": toks, "prefill_ms": e[0].elapsed_time(e[1]),
            "decode_ms_per_token": e[2].elapsed_time(e[3]) / steps,
            "tokens_per_s": 1e3 * steps / max(e[2].elapsed_time(e[3]), 1e-9), "graphed": use_graph}


class VerifyStep:
    """The target model's forward over n consecutive positions of one sequence
    at once (the speculative verify pass): the same kernels as the fused step,
    with n rows through the grouped CDQ linears (m = n) and a multi-query
    attention. Every row gets exactly the arithmetic of a one-token step, so
    its greedy tokens equal those of n sequential steps. Shares the target
    FusedDecoder's cache, tables and position (the first row's position)."""

    def __init__(self, fd: FusedDecoder, n: int):
        from . import ops
        self.fd, self.n = fd, n
        bf16, dev = torch.bfloat16, fd.dev
        z = lambda *shape, dt=bf16: torch.zeros(*shape, dtype=dt, device=dev)  # noqa: E731
        H, inter = fd.H, fd.inter
        qd, kvd = fd.n_heads * fd.hd, fd.n_kv * fd.hd
        self.ids = z(n, dt=torch.long)
        self.h, self.xn, self.o, self.dn = z(n, H), z(n, H), z(n, H), z(n, H)
        self.q, self.k, self.v, self.att = z(n, qd), z(n, kvd), z(n, kvd), z(n, qd)
        self.g, self.u, self.act = z(n, inter), z(n, inter), z(n, inter)
        self.best = z(n, dt=torch.int64)
        self.next = z(n, dt=torch.int64)
        self.layers = []
        for layer in fd.model.model.layers:
            a, mlp = layer.self_attn, layer.mlp
            T = lambda mod, x, y: ops.GemvTask(mod.device_pack, x, y, mod.bias)  # noqa: E731
            self.layers.append({
                "ln1": layer.input_layernorm.weight, "ln2": layer.post_attention_layernorm.weight,
                "qkv": ops.GroupedLinear([T(a.q_proj, self.xn, self.q), T(a.k_proj, self.xn, self.k),
                                          T(a.v_proj, self.xn, self.v)], m=n),
                "o": ops.GroupedLinear([T(a.o_proj, self.att, self.o)], m=n),
                "gu": ops.GroupedLinear([T(mlp.gate_proj, self.xn, self.g), T(mlp.up_proj, self.xn, self.u)], m=n),
                "down": ops.GroupedLinear([T(mlp.down_proj, self.act, self.dn)], m=n),
            })
        self.graph = None

    def _run(self) -> None:
        fd, n = self.fd, self.n
        p = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
        s = torch.cuda.current_stream(fd.dev).cuda_stream
        for li, Ly in enumerate(self.layers):
            cl = fd.cache.layers[li]
            if li == 0:
                fd._call("cdq_embed_rmsnorm_rows", p(self.ids), p(fd.embed_w), fd.vocab, p(self.h), p(Ly["ln1"]),
                         fd.eps, p(self.xn), fd.H, n, s)
            else:
                fd._call("cdq_add_rmsnorm_rows", p(self.h), p(self.dn), p(Ly["ln1"]), fd.eps, p(self.xn), fd.H, n, s)
            Ly["qkv"]()
            fd._call("cdq_attn_decode_multi", p(self.q), p(self.k), p(self.v), p(fd.cos), p(fd.sin), p(fd.pos),
                     p(cl.keys), p(cl.values), fd.max_len, fd.n_heads, fd.n_kv, fd.hd, float(fd.hd) ** -0.5,
                     p(self.att), n, s)
            Ly["o"]()
            fd._call("cdq_add_rmsnorm_rows", p(self.h), p(self.o), p(Ly["ln2"]), fd.eps, p(self.xn), fd.H, n, s)
            Ly["gu"]()
            fd._call("cdq_silu_mul", p(self.g), p(self.u), p(self.act), n * fd.inter, s)
            Ly["down"]()
        fd._call("cdq_add_rmsnorm_rows", p(self.h), p(self.dn), p(fd.norm_w), fd.eps, p(self.xn), fd.H, n, s)
        fd._call("cdq_lm_head_argmax_rows", p(fd.lm_w), p(self.xn), fd.vocab, fd.H, n, None, p(self.best),
                 p(self.next), s)

    @torch.no_grad()
    def capture(self) -> None:
        s = torch.cuda.Stream(device=self.fd.dev)
        s.wait_stream(torch.cuda.current_stream(self.fd.dev))
        with torch.cuda.stream(s):
            self._run()  # warm-up (writes cache slots that later passes overwrite)
        torch.cuda.current_stream(self.fd.dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._run()
        self.graph = g

    @torch.no_grad()
    def run(self) -> None:
        if self.graph is not None:
            self.graph.replay()
        else:
            self._run()


@torch.no_grad()
def speculative_greedy_decode(target, draft, prompt: torch.Tensor, new_tokens: int, k: int = 3,
                              use_graph: bool = True) -> dict:
    """Greedy decoding of `target` (the 26-state model) with `draft` (the same
    model on the 16-state lattice) proposing k tokens at a time: the draft
    decodes k tokens from the last accepted one, the target checks all k + 1
    positions in one verify pass, the longest prefix where the draft agrees
    with the target's own greedy choice is kept and the target's token at the
    first disagreement (or after the last draft token) follows. The output
    equals plain greedy decoding of the target token for token. Caches are
    static: slots beyond the accepted length are simply overwritten later."""
    P = prompt.shape[1]
    max_len = P + new_tokens + k + 4
    td = FusedDecoder(target, max_len)
    dd = FusedDecoder(draft, max_len)
    ver = VerifyStep(td, k + 1)
    e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    e[0].record()
    tok = td.prefill(prompt)
    dd.prefill(prompt)
    if use_graph:
        dd.capture()
        ver.capture()
    e[1].record()
    out = [int(tok.item())]
    pos = P  # position of `tok`
    verifies = accepted = 0
    while len(out) < new_tokens:
        dd.reset(torch.tensor([out[-1]], device=td.dev), pos)
        for _ in range(k):
            dd.step()
        ver.ids[0] = out[-1]
        ver.ids[1:].copy_(dd.tokens[:k])
        td.pos.fill_(pos)
        ver.run()
        drafts, ys = dd.tokens[:k].tolist(), ver.next.tolist()
        a = 0
        while a < k and drafts[a] == ys[a]:
            a += 1
        out += drafts[:a] + [ys[a]]
        verifies += 1
        accepted += a
        if a == k:  # the draft never consumed its last token: let it see it
            dd.reset(torch.tensor([drafts[k - 1]], device=td.dev), pos + k)
            dd.step()
        pos += a + 1
    e[2].record()
    torch.cuda.synchronize()
    ms = e[1].elapsed_time(e[2])
    n = len(out) - 1
    # the verify pass alone (device time of one graph replay, averaged)
    v0, v1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    td.pos.fill_(pos)
    v0.record()
    for _ in range(5):
        ver.run()
    v1.record()
    torch.cuda.synchronize()
    return {"tokens": torch.tensor(out[:new_tokens]).view(1, -1), "verifies": verifies,
            "accepted_per_verify": accepted / max(verifies, 1), "tokens_per_verify": n / max(verifies, 1),
            "tokens_per_s": 1e3 * n / max(ms, 1e-9), "k": k, "verify_ms": v0.elapsed_time(v1) / 5}


def main(argv=None) -> None:
    """Greedy generation on the random-init Qwen2.5-0.5B-architecture model
    with CDQ-26 projections (the reference's generate loop,
    code/cdq_lrr_qwen05.py:335-340), through the fused decode step; prints
    the tokens per second. --eager runs the steps without the CUDA graph, each
    step's launches inside the NVTX range "decode_step" (for a profiler's
    launch list)."""
    import argparse
    ap = argparse.ArgumentParser(prog="python -m cdq_lrr_b200.decode")
    ap.add_argument("--prompt", type=int, default=128, help="prompt tokens (seeded random ids)")
    ap.add_argument("--new-tokens", type=int, default=32)
    ap.add_argument("--eager", action="store_true", help="no CUDA graph; steps inside NVTX ranges")
    ap.add_argument("--persistent", action="store_true", help="the one-launch persistent decode step")
    args = ap.parse_args(argv)
    model = build_model(seed=0, device="cuda")
    patch_cdq(model)
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, model.config.vocab_size, (1, args.prompt), generator=g).cuda()
    if not args.eager:
        r = fused_greedy_decode(model, ids, args.new_tokens, persistent=args.persistent)
        print(f"{'persistent ' if args.persistent else ''}{r['tokens_per_s']:.1f} tok/s ({r['decode_ms_per_token']:.4f} ms per token), "
              f"tokens {r['tokens'][0, :8].tolist()} ...")
        return
    with torch.no_grad():
        dec = FusedDecoder(model, args.prompt + args.new_tokens + 2, persistent=args.persistent)
        dec.prefill(ids)
        dec._step()  # warm-up
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.new_tokens - 1):
            torch.cuda.nvtx.range_push("decode_step")
            dec._step()
            torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
    print(f"eager: {(args.new_tokens - 1) / dt:.1f} tok/s (host launch bound)")


if __name__ == "__main__":
    main()
