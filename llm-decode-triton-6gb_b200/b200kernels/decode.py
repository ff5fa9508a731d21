"""Greedy decode of a Mistral-shaped Hugging Face model with NF4 linears on the B200 kernels.

The reference decodes through ``model(input_ids, past_key_values, use_cache=True)`` one token at a
time (``profiling/common.py:80-85``, ``profiling/04_compare.py:21-31``); HF's ``DynamicCache`` grows
the KV tensors with ``torch.cat`` every step and Python launches every kernel, so the step cannot be
replayed as a CUDA graph. This engine decodes over a static KV cache ``[layers, B, KVH, S_max, D]``
with per-sequence lengths and captures one whole decode step (32 layers) in a CUDA graph:

* every NF4 linear -> the fused dequant + matmul kernel; with ``fused=True`` q/k/v share one launch
  and gate/up share one launch whose epilogue applies the SwiGLU;
* attention -> ``decode_attention`` (split-K partial + log-sum-exp combine);
* the glue ops (residual add + RMSNorm, rotary embedding + KV append) -> this library's kernels
  (``fused=True``), every launch a programmatic dependent of the previous one; or the HF modules
  themselves (``fused=False``);
* lm_head + argmax -> one ``lm_head_argmax`` launch at batch <= 64 (fused mode; vocabulary-parallel
  under tensor parallelism, the shards' maxima merged by one all-gather of 8-byte keys); otherwise
  torch ops. The embedding stays a torch op.

Prompts are prefilled through the HF forward (the reference's prefill path: SDPA, and dequant +
library GEMM for the many-row linears); the prompt's K/V are then copied into the static cache.
"""
from __future__ import annotations

import os

import torch
from transformers import MistralConfig, MistralForCausalLM
from transformers.cache_utils import DynamicCache
from transformers.models.mistral.modeling_mistral import apply_rotary_pos_emb

from . import _lib
from .decode_attention import decode_attention, decode_attention_append, l2_prefetch_hint
from .glue import add_rmsnorm, rope_kv_append, silu_mul
from .lm_head import MAX_M as LM_MAX_M, lm_head_argmax, merge_keys
from .linear4bit import quantize_model_linears
from .nf4_gemm import NF4Group, NF4Weight
from .tp import TPGroup, local_heads, shard_layer

# Mistral-7B-v0.3 shape (the checkpoint the reference profiles, profiling/common.py:11)
MISTRAL_7B = dict(hidden_size=4096, num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8,
                  head_dim=128, intermediate_size=14336, vocab_size=32768, rms_norm_eps=1e-5,
                  rope_parameters={"rope_type": "default", "rope_theta": 1e6}, sliding_window=None,
                  max_position_embeddings=32768 + 1024, tie_word_embeddings=False)


def build_random_mistral(seed: int = 0, dtype=torch.float16, device="cuda", nested: bool = True,
                         **overrides) -> MistralForCausalLM:
    """Random-init Mistral-shaped model (weights N(0, 0.02^2), RMSNorm weights 1) whose decoder
    linears are quantised to bitsandbytes NF4 on the device (blocksize 64, double-quantised scales
    with blocksize 256 when ``nested``). Embedding and lm_head stay dense in ``dtype``."""
    cfg = MistralConfig(**{**MISTRAL_7B, **overrides})
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    with torch.device(device):
        model = MistralForCausalLM(cfg)
    model.to(dtype)
    model.eval()
    quantize_model_linears(model.model, nested=nested)
    torch.cuda.empty_cache()
    return model


class DecodeEngine:
    """Static-cache, graph-captured greedy decode for a fixed batch size.

    ``fused=True`` (default) runs every per-layer op on this library's kernels, 9 launches per layer
    chained with programmatic dependent launch: add+RMSNorm, q/k/v in one NF4 launch, RoPE + KV
    append, attention (partial + combine), o_proj, add+RMSNorm, gate/up in one launch with the SwiGLU
    epilogue, down_proj (batch > 8: separate gate/up launches and a SiLU*mul kernel). ``fused=False``
    keeps the HF modules for the glue ops (the same torch code as the stock path) around the two hot
    kernels.

    ``tp`` (a ``TPGroup`` of world size > 1, one process per GPU) runs the tensor-parallel mode: this
    rank keeps its NF4 shards and its KV heads, and the o_proj / down_proj outputs are all-reduced
    inside the step's CUDA graph -- ``allreduce="fused"`` (batch <= 8): o_proj / down_proj push their
    partial products to every peer from the GEMM epilogue and the next add+RMSNorm sums them (no
    separate all-reduce launch); ``"peer"``: the one-shot NVLink peer-memory kernel
    (``b2d_allreduce``) between the GEMM and the add+RMSNorm (also used for batch > 8 under
    "fused"); ``"nccl"``: NCCL. All three give identical tokens. Requires ``fused=True``."""

    def __init__(self, model: MistralForCausalLM, batch: int, max_len: int, fused: bool = True,
                 tp: TPGroup | None = None, allreduce: str = "fused"):
        cfg = model.config
        self.model = model
        self.B, self.S = batch, max_len
        self.L = cfg.num_hidden_layers
        self.H, self.KVH = cfg.num_attention_heads, cfg.num_key_value_heads
        self.D = getattr(cfg, "head_dim", None) or cfg.hidden_size // self.H
        self.scale = self.D ** -0.5
        self.tp = tp if tp is not None and tp.world > 1 else None
        self.kv0 = 0
        if self.tp is not None:
            if not fused:
                raise ValueError("tensor parallel decode needs fused=True")
            _, self.H, self.kv0, self.KVH = local_heads(cfg, self.tp.world, self.tp.rank)
        p = next(model.parameters())
        self.device, self.dtype = p.device, model.model.embed_tokens.weight.dtype
        self.w = []
        for layer in model.model.layers:
            at, mlp = layer.self_attn, layer.mlp
            full = {n: NF4Weight(m.weight) for n, m in (
                ("q", at.q_proj), ("k", at.k_proj), ("v", at.v_proj), ("o", at.o_proj),
                ("gate", mlp.gate_proj), ("up", mlp.up_proj), ("down", mlp.down_proj))}
            if self.tp is not None:
                full = shard_layer(full, cfg, self.tp.world, self.tp.rank)
            self.w.append(full)
        kv_shape = (self.L, batch, self.KVH, max_len, self.D)
        self.k_cache = torch.zeros(kv_shape, dtype=self.dtype, device=self.device)
        self.v_cache = torch.zeros(kv_shape, dtype=self.dtype, device=self.device)
        self.ids = torch.zeros(batch, dtype=torch.long, device=self.device)      # input token per sequence
        self.pos = torch.zeros(batch, dtype=torch.long, device=self.device)      # its position
        self.next_ids = torch.zeros(batch, dtype=torch.long, device=self.device)
        self.logits = torch.zeros(batch, cfg.vocab_size, dtype=self.dtype, device=self.device)  # last step's
        self.bidx = torch.arange(batch, device=self.device)
        self.graph = None
        self.stream = torch.cuda.Stream(self.device)
        self.fused = fused
        if fused:
            self._init_fused(cfg)
        if allreduce not in ("fused", "peer", "nccl"):
            raise ValueError(f"allreduce must be 'fused', 'peer' or 'nccl', got {allreduce!r}")
        self.ar_fused = self.tp is not None and allreduce == "fused" and self.pair
        if self.ar_fused:
            self.tp.enable_fused_allreduce(batch, cfg.hidden_size, 2 * self.L, self.dtype, self.device)
            for g, w in zip(self.groups, self.w):
                g["o"] = NF4Group([w["o"]], mode="allreduce")
                g["down"] = NF4Group([w["down"]], mode="allreduce")
        elif self.tp is not None and allreduce in ("fused", "peer"):
            self.tp.enable_peer_allreduce(batch * cfg.hidden_size, self.dtype, self.device)
        head = model.lm_head
        self.lm_fused = (fused and batch <= LM_MAX_M and head.bias is None and head.weight.dtype == self.dtype
                         and cfg.hidden_size % 256 == 0
                         and (self.tp is None or cfg.vocab_size % self.tp.world == 0))
        if self.lm_fused:
            V = cfg.vocab_size
            if self.tp is None:
                self.lm_w, self.lm_off = head.weight.detach().contiguous(), 0
            else:   # vocabulary-parallel: this rank's rows of the head
                Vl = V // self.tp.world
                self.lm_off = self.tp.rank * Vl
                self.lm_w = head.weight.detach()[self.lm_off:self.lm_off + Vl].contiguous()
                self.logits_local = torch.zeros(batch, Vl, dtype=self.dtype, device=self.device)
                self.keys = torch.zeros(batch, dtype=torch.int64, device=self.device)
                self.keys_all = torch.zeros(self.tp.world * batch, dtype=torch.int64, device=self.device)

    def _init_fused(self, cfg):
        B, dev, dt = self.B, self.device, self.dtype
        hid, inter = cfg.hidden_size, self.w[0]["gate"].N
        self.eps = cfg.rms_norm_eps
        self.pair = B <= NF4Group.MAX_M
        self.groups = []
        for w in self.w:
            g = {"o": NF4Group([w["o"]]) if self.pair else None,
                 "down": NF4Group([w["down"]]) if self.pair else None}
            if self.pair:
                g["qkv"] = NF4Group([w["q"], w["k"], w["v"]])
                g["gateup"] = NF4Group([w["gate"], w["up"]], mode="silu_mul")
            self.groups.append(g)
        z = lambda *shape: torch.zeros(shape, dtype=dt, device=dev)
        self.r = z(B, hid)                                   # residual stream
        self.xn = z(B, hid)                                  # normalised activations
        self.q = z(B, self.H * self.D)
        self.k = z(B, self.KVH * self.D)
        self.v = z(B, self.KVH * self.D)
        self.attn = z(B, 1, self.H, self.D)
        self.o_out = z(B, hid)
        self.h_mlp = z(B, inter)
        self.g_out = None if self.pair else z(B, inter)
        self.down_out = z(B, hid)
        self.seqlens = torch.zeros(B, dtype=torch.int32, device=dev)
        # the streaming attention kernel also applies RoPE and appends the step's K/V (one launch fewer per
        # layer); B2D_ATTN_KERNEL=reg selects the separate rotary kernel + register-prefetch attention
        self.attn_append = os.environ.get("B2D_ATTN_KERNEL", "stream") != "reg"
        # B2D_ATTN_COMBINE=fused: the append launch's last split CTA combines (no combine launch)
        self.attn_flags = _lib.LAUNCH_PDL | (_lib.ATTN_FUSED_COMBINE if os.environ.get("B2D_ATTN_COMBINE") == "fused" else 0)
        # The attention launch prefetches the o_proj weights into L2 (B2D_L2_PREFETCH: "o" default, "o,gu"
        # adds gate/up, "none" off; measured at batch 8: "o" 2.206 -> 2.196 ms per step, "o,gu" 2.271)
        self.l2_pf = [t for t in os.environ.get("B2D_L2_PREFETCH", "o").split(",") if t and t != "none"]
        # rotary tables for every cache position, computed by the model's own rotary module
        pos = torch.arange(self.S, device=dev).view(1, -1)
        cos, sin = self.model.model.rotary_emb(self.r.view(B, 1, hid)[:1], pos)
        self.cos, self.sin = cos[0].to(dt).contiguous(), sin[0].to(dt).contiguous()

    @torch.inference_mode()
    def _step_fused(self):
        m = self.model.model
        B, H, KVH, D = self.B, self.H, self.KVH, self.D
        PDL, STATIC = _lib.LAUNCH_PDL, _lib.LAUNCH_PDL | _lib.STATIC_WEIGHTS
        torch.index_select(m.embed_tokens.weight, 0, self.ids, out=self.r)
        tp, arf = self.tp, self.ar_fused
        x_in = None

        def norm(weight, x, site):   # residual += x (or the all-reduced partials of `site`); xn = RMSNorm
            if site is None:
                add_rmsnorm(self.r, weight, self.eps, self.xn, x=x, flags=PDL)
            else:
                tp.allreduce_add_rmsnorm(site, self.r, weight, self.eps, self.xn, flags=PDL)

        for i, layer in enumerate(m.layers):
            w, g = self.w[i], self.groups[i]
            norm(layer.input_layernorm.weight, x_in, 2 * i - 1 if arf and i > 0 else None)
            if self.pair:
                g["qkv"].matmul(self.xn, [self.q, self.k, self.v], flags=STATIC)
            else:
                w["q"].matmul(self.xn, out=self.q); w["k"].matmul(self.xn, out=self.k); w["v"].matmul(self.xn, out=self.v)
            if self.attn_append:   # RoPE + KV append inside the attention launch
                if self.l2_pf:
                    names = {"o": ["o"], "gu": ["gate", "up"]}
                    pf = [w[n].packed for key in self.l2_pf for n in names[key]]
                    l2_prefetch_hint([t for t in pf if t.is_contiguous() and t.data_ptr() % 16 == 0])
                decode_attention_append(self.q, self.k, self.v, self.pos, self.cos, self.sin, self.k_cache[i],
                                        self.v_cache[i], self.scale, self.seqlens, self.attn, flags=self.attn_flags)
            else:
                q3 = self.q.view(B, H, D)
                rope_kv_append(self.q, self.k, self.v, self.pos, self.cos, self.sin, q3, self.k_cache[i],
                               self.v_cache[i], self.seqlens, flags=PDL)
                # the append above writes only each sequence's newest key/value: the older ones may be prefetched
                decode_attention(q3.view(B, H, 1, D), self.k_cache[i], self.v_cache[i], self.scale,
                                 seqlens=self.seqlens, out=self.attn, flags=PDL | _lib.KV_STATIC_PREFIX)
            a2 = self.attn.view(B, H * D)
            if arf:
                g["o"].matmul(a2, flags=STATIC, epilogue=tp.epilogue(2 * i))
            elif self.pair:
                g["o"].matmul(a2, [self.o_out], flags=STATIC)
            else:
                w["o"].matmul(a2, out=self.o_out)
            if tp is not None and not arf:
                tp.all_reduce(self.o_out)
            norm(layer.post_attention_layernorm.weight, self.o_out, 2 * i if arf else None)
            if self.pair:
                g["gateup"].matmul(self.xn, [self.h_mlp], flags=STATIC)
                if arf:
                    g["down"].matmul(self.h_mlp, flags=STATIC, epilogue=tp.epilogue(2 * i + 1))
                else:
                    g["down"].matmul(self.h_mlp, [self.down_out], flags=STATIC)
            else:
                w["gate"].matmul(self.xn, out=self.g_out); w["up"].matmul(self.xn, out=self.h_mlp)
                silu_mul(self.g_out, self.h_mlp, out=self.h_mlp, flags=PDL)
                w["down"].matmul(self.h_mlp, out=self.down_out)
            if tp is not None and not arf:
                tp.all_reduce(self.down_out)
            x_in = self.down_out
        norm(m.norm.weight, x_in, 2 * self.L - 1 if arf else None)
        if arf:
            tp.advance()
        if self.lm_fused and tp is None:
            lm_head_argmax(self.xn, self.lm_w, logits=self.logits, ids=self.next_ids, flags=STATIC)
        elif self.lm_fused:
            import torch.distributed as dist
            lm_head_argmax(self.xn, self.lm_w, logits=self.logits_local, keys=self.keys, vocab_offset=self.lm_off,
                           flags=STATIC)
            dist.all_gather_into_tensor(self.keys_all, self.keys, group=tp.group)
            merge_keys(self.keys_all.view(tp.world, B), out=self.next_ids)
        else:
            logits = self.model.lm_head(self.xn)                        # [B, vocab]
            self.logits.copy_(logits)
            torch.argmax(logits, -1, out=self.next_ids)
        self.ids.copy_(self.next_ids)
        self.pos.add_(1)

    # ----------------------------------------------------------------------------- one step
    @torch.inference_mode()
    def _step(self):
        """Consume ``ids`` at ``pos``, write the step's K/V, produce ``next_ids``, advance ``pos``."""
        if self.fused:
            return self._step_fused()
        m = self.model.model
        B, H, KVH, D = self.B, self.H, self.KVH, self.D
        h = m.embed_tokens(self.ids.view(B, 1))                      # [B, 1, hidden]
        cos, sin = m.rotary_emb(h, self.pos.view(B, 1))
        seqlens = (self.pos + 1).to(torch.int32)
        for i, layer in enumerate(m.layers):
            w = self.w[i]
            r = h
            x = layer.input_layernorm(h)
            q = w["q"].matmul(x).view(B, 1, H, D).transpose(1, 2)
            k = w["k"].matmul(x).view(B, 1, KVH, D).transpose(1, 2)
            v = w["v"].matmul(x).view(B, 1, KVH, D).transpose(1, 2)
            q, k = apply_rotary_pos_emb(q, k, cos, sin)
            self.k_cache[i][self.bidx, :, self.pos] = k[:, :, 0]
            self.v_cache[i][self.bidx, :, self.pos] = v[:, :, 0]
            a = decode_attention(q, self.k_cache[i], self.v_cache[i], self.scale, seqlens=seqlens)
            h = r + w["o"].matmul(a.reshape(B, 1, H * D))
            r = h
            x = layer.post_attention_layernorm(h)
            g = w["gate"].matmul(x)
            u = w["up"].matmul(x)
            h = r + w["down"].matmul(layer.mlp.act_fn(g) * u)
        logits = self.model.lm_head(m.norm(h))                       # [B, 1, vocab]
        self.logits.copy_(logits[:, -1])
        self.next_ids.copy_(logits[:, -1].argmax(-1))
        self.ids.copy_(self.next_ids)
        self.pos.add_(1)

    def capture(self):
        """Warm up (allocates every workspace on the capture stream) and capture one step."""
        saved = (self.ids.clone(), self.pos.clone(), self.next_ids.clone())
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            for _ in range(2):
                self._step()
                self.ids.copy_(saved[0]); self.pos.copy_(saved[1])
        torch.cuda.current_stream(self.device).wait_stream(self.stream)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self._step()
        self.ids.copy_(saved[0]); self.pos.copy_(saved[1]); self.next_ids.copy_(saved[2])
        torch.cuda.synchronize(self.device)

    def step(self):
        """One decode step on the current stream (graph replay once captured)."""
        if self.graph is None:
            self._step()
        else:
            self.graph.replay()
        return self.next_ids

    # ----------------------------------------------------------------------------- prefill / generate
    @torch.inference_mode()
    def prefill(self, prompt_ids: torch.Tensor) -> torch.Tensor:
        """Run the prompts [B, P] through the HF forward, copy their K/V into the static cache and
        set up the first decode input. Returns the first generated token per sequence."""
        B, P = prompt_ids.shape
        assert B == self.B and P < self.S, (prompt_ids.shape, self.B, self.S)
        past = DynamicCache()
        out = self.model(input_ids=prompt_ids.to(self.device), past_key_values=past, use_cache=True,
                         logits_to_keep=1)
        kv = slice(self.kv0, self.kv0 + self.KVH)   # this rank's KV heads (all of them without TP)
        for i in range(self.L):
            self.k_cache[i, :, :, :P] = past.layers[i].keys[:, kv]
            self.v_cache[i, :, :, :P] = past.layers[i].values[:, kv]
        first = out.logits[:, -1].argmax(-1)
        self.ids.copy_(first)
        self.next_ids.copy_(first)
        self.pos.fill_(P)
        return first

    def fill_random_cache(self, context: int, seed: int = 0):
        """Fill the first ``context`` cache slots with seeded N(0,1) K/V (long-context throughput runs)
        and set up decode from position ``context``."""
        g = torch.Generator(device=self.device).manual_seed(seed)
        for i in range(self.L):
            self.k_cache[i, :, :, :context].normal_(generator=g)
            self.v_cache[i, :, :, :context].normal_(generator=g)
        self.pos.fill_(context)
        self.ids.random_(0, self.model.config.vocab_size, generator=g)

    def check_peers(self) -> None:
        """Raise if a tensor-parallel peer wait of this rank has timed out since the engine was built.

        The peer all-reduce kernels bound every wait and count a timeout in a device-side error word
        instead of hanging; after one, the sums of later steps are not trustworthy (a wait that
        timed out reads whatever the peer's slot held). ``generate`` and ``teacher_forced`` call this
        at their end; a caller driving ``step`` itself should call it (one device read) before it
        trusts the tokens. A no-op without tensor parallelism."""
        if self.tp is not None:
            n = self.tp.peer_errors()
            if n:
                raise RuntimeError(f"tensor-parallel rank {self.tp.rank}: {n} peer all-reduce wait(s) timed out; "
                                   "the decoded tokens since then are invalid")

    def full_logits(self) -> torch.Tensor:
        """The last step's logits [B, vocab]. Under tensor parallelism with the vocabulary-parallel
        head, every rank holds its slice and this gathers them (a collective: all ranks call it)."""
        if self.tp is None or not self.lm_fused:
            return self.logits
        import torch.distributed as dist
        W, (B, Vl) = self.tp.world, self.logits_local.shape
        buf = torch.empty(W * B, Vl, dtype=self.dtype, device=self.device)
        dist.all_gather_into_tensor(buf, self.logits_local, group=self.tp.group)
        self.logits.copy_(buf.view(W, B, Vl).permute(1, 0, 2).reshape(B, W * Vl))
        return self.logits

    @torch.inference_mode()
    def teacher_forced(self, prompt_ids: torch.Tensor, tokens: torch.Tensor):
        """Decode consuming the given tokens [B, T] (instead of our own argmax): returns our argmax
        and logits (float) for steps 1..T-1, i.e. the prediction after consuming tokens[:, t-1]."""
        self.prefill(prompt_ids)
        if self.graph is None:
            self.capture()
        preds, logits = [], []
        for t in range(1, tokens.shape[1]):
            self.ids.copy_(tokens[:, t - 1])
            preds.append(self.step().clone())
            logits.append(self.full_logits().float())
        self.check_peers()
        return torch.stack(preds, 1), torch.stack(logits, 1)

    @torch.inference_mode()
    def generate(self, prompt_ids: torch.Tensor, new_tokens: int) -> torch.Tensor:
        """Greedy decode: [B, P] prompts -> [B, new_tokens] generated ids (first from prefill)."""
        out = [self.prefill(prompt_ids)]
        if self.graph is None:
            self.capture()
        for _ in range(new_tokens - 1):
            out.append(self.step().clone())
        self.check_peers()
        return torch.stack(out, dim=1)


@torch.inference_mode()
def hf_greedy(model, prompt_ids: torch.Tensor, new_tokens: int, return_logits: bool = False):
    """The reference's greedy loop (``profiling/04_compare.py:21-31``) through the HF forward with a
    ``DynamicCache``: whatever forward the model's modules currently have (stock or patched)."""
    past = DynamicCache()
    out = model(input_ids=prompt_ids, past_key_values=past, use_cache=True, logits_to_keep=1)
    nxt = out.logits[:, -1:].argmax(-1)
    toks, logits = [nxt], [out.logits[:, -1].float()]
    for _ in range(new_tokens - 1):
        out = model(input_ids=nxt, past_key_values=past, use_cache=True)
        nxt = out.logits[:, -1:].argmax(-1)
        toks.append(nxt)
        if return_logits:
            logits.append(out.logits[:, -1].float())
    toks = torch.cat(toks, dim=1)
    return (toks, torch.stack(logits, 1)) if return_logits else toks
