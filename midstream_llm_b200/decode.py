"""Incremental next-token logits with a KV cache.

The reference samples by calling `next_token_logits(model, context, device)` for every new token
(Midstream-LLM src/jishui/generate_torch.py:278-285), which re-runs the whole context through the
model and keeps logits[0, -1]: O(T) work per token, O(T^2) per generation. `KVCacheDecoder` keeps
the post-RoPE keys and values of every layer: a context that extends the previous one by new tokens
runs only those tokens (embedding, M = 1 GEMMs with the RoPE position chosen by the table row,
single-query attention over the cache, `jx_attn_decode`); any other context (a new prompt, or the
reference's sliding window `history[-limit:]` once it exceeds the context length) is prefilled from
scratch with the batched forward. Numerics are the training forward's fp16 recipe.
"""
from __future__ import annotations

from typing import Sequence

import numpy as np
import torch

from . import ops
from .model import JishuiForCausalLM, rope_tables

F16, F32 = torch.float16, torch.float32


class KVCacheDecoder:
    """Per-model decoding state: keys / values of the last context for every layer (batch 1). The cache is
    rebuilt when the context does not extend the previous one or the weights changed since."""

    def __init__(self, model: JishuiForCausalLM, max_len: int | None = None):
        c = model.config
        self.model = model
        self.max_len = max_len or c.max_position_embeddings
        dev = next(model.parameters()).device
        if dev.type != "cuda":
            raise RuntimeError("KVCacheDecoder: the model must be on a CUDA device (there is no CPU path)")
        L, d, F, H, hd = c.num_hidden_layers, c.hidden_size, c.intermediate_size, c.num_attention_heads, c.head_dim
        self.kc = torch.empty(L, 1, self.max_len, d, device=dev, dtype=F16)
        self.vc = torch.empty(L, 1, self.max_len, d, device=dev, dtype=F16)
        self.cos, self.sin = rope_tables(self.max_len, hd, c.rope_theta, dev)
        e = lambda *s, t=F16: torch.empty(*s, device=dev, dtype=t)  # noqa: E731
        self.x, self.h, self.o, self.xmid, self.h2 = e(1, d), e(1, d), e(1, d), e(1, d), e(1, d)
        self.qkv = e(1, 3 * d)
        self.gate, self.up, self.act = e(1, F), e(1, F), e(1, F)
        self.mean, self.rstd = e(1, t=F32), e(1, t=F32)
        self.logits = e(1, c.vocab_size)
        self.ws = e(ops.attn_decode_workspace_bytes(1, H, self.max_len) // 4 + 4, t=F32)
        self.tok = torch.empty(1, device=dev, dtype=torch.int64)
        # CUDA-graph inputs: token and position in device memory, staged through pinned host buffers.
        self.pos = torch.zeros(1, device=dev, dtype=torch.int64)
        self.len32 = torch.ones(1, device=dev, dtype=torch.int32)
        self.cos_row = torch.empty(1, hd // 2, device=dev, dtype=F32)
        self.sin_row = torch.empty(1, hd // 2, device=dev, dtype=F32)
        self.host_in = torch.zeros(64, 2, dtype=torch.int64).pin_memory()  # ring of staging slots
        self._slot = 0
        self.use_graph = True
        self._graph = None
        self._graph_key = None
        self.context: list[int] = []
        self._generation = -1  # weights generation the cache was built with
        self._fl = None        # the model's flat weight storage the cache and graph were built with

    @torch.no_grad()
    def next_token_logits(self, context: Sequence[int]) -> np.ndarray:
        """float32 logits [V] of the token after `context` (generate_torch.py:278-285)."""
        ctx = [int(t) for t in context]
        if not ctx:
            raise ValueError("empty context")
        if len(ctx) > self.max_len:
            raise ValueError("context exceeds the decoder's maximum length")
        # The flat weight buffers are re-validated (a walk over every parameter) only when prefilling; a decode
        # step reuses them while the model still holds the same storage object.
        fl = self._fl if self._fl is not None and self.model._flat is self._fl else self.model.flat()
        fl.refresh_f16()
        n = len(self.context)
        if 0 < n < len(ctx) and ctx[:n] == self.context and fl.generation == self._generation and fl is self._fl:
            for p in range(n, len(ctx)):
                self._decode(ctx[p], p)
        else:
            fl = self.model.flat()
            fl.refresh_f16()
            self._fl = fl
            self._prefill(ctx)
        self.context = ctx
        self._generation = fl.generation
        return self.logits[0].float().cpu().numpy()

    # ---------------------------------------------------------------- internals
    def _prefill(self, ctx: list[int]) -> None:
        m, c = self.model, self.model.config
        T = len(ctx)
        Tp = (T + 255) // 256 * 256  # attention tiles; the padding follows the context, so causality hides it
        d, L = c.hidden_size, c.num_hidden_layers
        dev = self.kc.device
        ids = torch.zeros(Tp, device=dev, dtype=torch.int64)
        ids[:T] = torch.tensor(ctx, dtype=torch.int64)
        fl = self._fl
        ws = m._workspace(1, Tp, False)
        e16 = fl.p16_rows("embed_tokens.weight", c.vocab_size, d)
        ops.embed_fwd(ids, e16, out=ws.xs[0])
        A = ws.acts[0]
        for i in range(L):
            m._layer_fwd(m._layer_weights(fl, i), ws, ws.xs[i % 2], ws.xs[(i + 1) % 2], A)
            self.kc[i, 0, :T].copy_(A.qkv[:T, d:2 * d])
            self.vc[i, 0, :T].copy_(A.qkv[:T, 2 * d:])
        x_last = ws.xs[L % 2][T - 1:T]
        m._norm_fwd(x_last, fl.p32_view("norm.weight", (d,)), m._bias_view(fl.p32_view, "norm.bias"), self.h,
                    self.mean, self.rstd)
        ops.gemm_f16(self.h, e16, out=self.logits)

    def _decode(self, token: int, p: int) -> None:
        """One new token at position p: a replay of the captured step (token and position are device inputs),
        or an eager step that also captures the graph when there is none for the current weights buffers."""
        j = self._slot % self.host_in.shape[0]
        if j == 0 and self._slot:
            torch.cuda.current_stream().synchronize()  # every slot's copy has landed before the ring wraps
        self._slot += 1
        self.host_in[j, 0], self.host_in[j, 1] = token, p
        self.tok.copy_(self.host_in[j, :1], non_blocking=True)
        self.pos.copy_(self.host_in[j, 1:], non_blocking=True)
        key = id(self._fl)
        if self._graph is not None and self._graph_key == key:
            self._graph.replay()
            return
        self._step()  # eager (and the first use of every kernel of the step, outside any capture)
        if self.use_graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._step()
            self._graph, self._graph_key = g, key

    def _step(self) -> None:
        """The decode step on device inputs self.tok / self.pos (graph-capturable: no host reads)."""
        m, c = self.model, self.model.config
        d, F, H, hd, L = c.hidden_size, c.intermediate_size, c.num_attention_heads, c.head_dim, c.num_hidden_layers
        fl = self._fl
        e16 = fl.p16_rows("embed_tokens.weight", c.vocab_size, d)
        ops.embed_fwd(self.tok, e16, out=self.x)
        torch.index_select(self.cos, 0, self.pos, out=self.cos_row)  # RoPE of position p as a 1-row table
        torch.index_select(self.sin, 0, self.pos, out=self.sin_row)
        self.len32.copy_(self.pos + 1)
        cos, sin = self.cos_row, self.sin_row
        for i in range(L):
            w = m._layer_weights(fl, i)
            m._norm_fwd(self.x, w["g1"], w["b1"], self.h, self.mean, self.rstd)
            ops.gemm_qkv_rope(self.h, w["wqkv"], d, cos, sin, 1, hd, out=self.qkv)
            ops.attn_decode(self.qkv, self.kc[i], self.vc[i], self.max_len, H, hd, self.ws, out=self.o,
                            length_dev=self.len32)
            ops.gemm_f16(self.o, w["wo"], resid=self.x, out=self.xmid)
            m._norm_fwd(self.xmid, w["g2"], w["b2"], self.h2, self.mean, self.rstd)
            ops.gemm_swiglu_fwd(self.h2, w["wgu"], F, gate=self.gate, up=self.up, act=self.act)
            ops.gemm_f16(self.act, w["wd"], resid=self.xmid, out=self.x)
        m._norm_fwd(self.x, fl.p32_view("norm.weight", (d,)), m._bias_view(fl.p32_view, "norm.bias"), self.h,
                    self.mean, self.rstd)
        ops.gemm_f16(self.h, e16, out=self.logits)


def next_token_logits(model: JishuiForCausalLM, context: Sequence[int], device=None) -> np.ndarray:
    """Drop-in for generate_torch.next_token_logits: the same result, with a KV cache kept on the model
    across calls."""
    dec = getattr(model, "_kv_decoder", None)
    if dec is None:
        dec = model._kv_decoder = KVCacheDecoder(model)
    return dec.next_token_logits(context)
