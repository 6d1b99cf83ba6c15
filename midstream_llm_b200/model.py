"""Drop-in `JishuiForCausalLM` whose forward and backward run on the B200 kernels.

Mirrors Midstream-LLM src/jishui/model_torch.py:
  * identical module tree, parameter names and shapes (model_torch.py:28-84),
    so `state_dict()` / `load_state_dict(strict=True)` interoperate with the
    reference and with checkpoints written by either trainer;
  * `forward(input_ids) -> logits [B, T, V]` in fp16 (model_torch.py:86-98);
  * `causal_lm_loss(model, inputs, targets)` -> mean CE (model_torch.py:102-104),
    which here runs the fused head + cross-entropy and never materialises fp32
    logits.

Numerics follow the reference's fp16 autocast recipe (pretrain_torch.py:212):
fp32 master weights, fp16 GEMM operands with fp32 accumulation, fp16 residual
stream, fp32 norm statistics (RMSNorm, or LayerNorm run in fp32 as autocast runs it) /
RoPE / softmax / CE. The B200 path always
computes this recipe (there is no fp32 or CPU path); it raises if the
configuration is outside what the kernels implement.

Storage: at first use on a CUDA device every parameter is re-pointed into
one flat fp32 buffer (named_parameters() order, 64-element aligned); `.grad`
tensors are views into a flat fp32 gradient buffer, and an fp16 copy of the
flat weights feeds the GEMMs (refreshed by the fused optimizer, or re-cast
when a parameter was modified in place). Because q/k/v and gate/up are
adjacent in that order, the fused [q;k;v] and [gate;up] weight matrices are
plain views.
"""
from __future__ import annotations

import math
import weakref
from dataclasses import dataclass, field

import torch
from torch import nn

from . import _lib, ops
from .config import ModelConfig

_ALIGN = 64
# The flat buffers are padded to a multiple of this many elements, so that 1, 2, 4 or 8 data-parallel ranks
# get equal contiguous shards that start on 64-element (256-byte) boundaries.
_SHARD_ALIGN = 512

# Parameter -> weak reference to the JishuiForCausalLM that owns it; lets the
# optimizer, GradScaler and clip_grad_norm_ find the model's flat buffers from
# `model.parameters()` without putting attributes on the Parameter objects.
# Keyed by id(); the stored weak reference to the parameter guards against id reuse.
_PARAM_OWNER: dict[int, tuple] = {}


def owner_of(params) -> "JishuiForCausalLM":
    """The single JishuiForCausalLM owning all of `params` (raises otherwise)."""
    owners = set()
    model = None
    for p in params:
        entry = _PARAM_OWNER.get(id(p))
        model = entry[1]() if entry is not None and entry[0]() is p else None
        if model is None:
            raise RuntimeError("parameter does not belong to a B200 JishuiForCausalLM")
        owners.add(id(model))
    if len(owners) != 1:
        raise RuntimeError("parameters from more than one model were given")
    return model


def _round_up(n: int, a: int = _ALIGN) -> int:
    return (n + a - 1) // a * a


def rope_tables(seq_len: int, head_dim: int, theta: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    """cos/sin [seq_len, head_dim/2] computed with the reference's own fp32 ops
    (model_torch.py:20-22) so the tables are bit-identical to its angles."""
    inv = theta ** (-torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim)
    angles = torch.arange(seq_len, device=device, dtype=torch.float32)[:, None] * inv
    return angles.cos().contiguous(), angles.sin().contiguous()


# Sequence tile of the attention kernels: a batch's rows are padded to a multiple of it. Causal attention
# never lets a real position see the padding, the padded targets are ignored by the loss, and their
# logit gradients are zero, so results at the real positions are those of the unpadded sequence.
_SEQ_TILE = 256


def _pad_rows(t: torch.Tensor, fill: int) -> torch.Tensor:
    """[B, T] integer rows padded on the right to a multiple of the sequence tile with `fill`."""
    T = t.shape[-1]
    Tp = -(-T // _SEQ_TILE) * _SEQ_TILE
    if Tp == T:
        return t
    out = torch.full((t.shape[0], Tp), fill, dtype=t.dtype, device=t.device)
    out[:, :T] = t
    return out


def _unpad_logits(ws: "Workspace", T: int) -> torch.Tensor:
    """A copy of the workspace logits at the first T positions of each row, [B, T, V]."""
    full = ws.logits.view(ws.B, ws.T, -1)
    return full[:, :T].clone() if T != ws.T else full.clone()


def check_supported(config: ModelConfig) -> None:
    """Raises for configurations the sm_100a kernels do not implement (no silent fallback)."""
    problems = []
    if config.attention_bias or config.mlp_bias:
        problems.append("attention_bias / mlp_bias are not supported")
    if not config.tie_word_embeddings:
        problems.append("untied LM head is not supported")
    if config.num_key_value_heads != config.num_attention_heads:
        problems.append("grouped-query attention is not supported")
    if config.head_dim != 64:
        problems.append("head_dim must be 64")
    if config.hidden_size % 64 or config.intermediate_size % 8 or config.hidden_size > 4096:
        problems.append("hidden_size must be a multiple of 64 (<= 4096) and intermediate_size a multiple of 8")
    if problems:
        raise ValueError("unsupported Jishui configuration for the B200 kernels: " + "; ".join(problems))


# --------------------------------------------------------------------------- module tree
def make_norm(config: ModelConfig) -> nn.Module:
    """The reference's norm choice (model_torch.py:12-15): RMSNorm, or LayerNorm with optional bias."""
    if config.norm_type == "rmsnorm":
        return nn.RMSNorm(config.hidden_size, eps=config.norm_eps)
    return nn.LayerNorm(config.hidden_size, eps=config.norm_eps, bias=config.norm_bias)


class CausalSelfAttention(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        self.config = config
        d = config.hidden_size
        kv = config.num_key_value_heads * config.head_dim
        self.q_proj = nn.Linear(d, d, bias=config.attention_bias)
        self.k_proj = nn.Linear(d, kv, bias=config.attention_bias)
        self.v_proj = nn.Linear(d, kv, bias=config.attention_bias)
        self.o_proj = nn.Linear(d, d, bias=config.attention_bias)


class SwiGLU(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        d, f = config.hidden_size, config.intermediate_size
        self.gate_proj = nn.Linear(d, f, bias=config.mlp_bias)
        self.up_proj = nn.Linear(d, f, bias=config.mlp_bias)
        self.down_proj = nn.Linear(f, d, bias=config.mlp_bias)


class TransformerBlock(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        self.input_norm = make_norm(config)
        self.attention = CausalSelfAttention(config)
        self.post_attention_norm = make_norm(config)
        self.mlp = SwiGLU(config)


# --------------------------------------------------------------------------- flat storage
class FlatParams:
    """Flat fp32 master weights, fp32 grads and the fp16 weight copy of one model."""

    def __init__(self, model: "JishuiForCausalLM", device: torch.device):
        named = list(model.named_parameters())
        self.names = [n for n, _ in named]
        self.params = [p for _, p in named]
        self.offsets: dict[str, int] = {}
        off = 0
        for n, p in named:
            self.offsets[n] = off
            off += _round_up(p.numel())
        self.numel = _round_up(off, _SHARD_ALIGN)
        self.device = device
        self.p32 = torch.zeros(self.numel, dtype=torch.float32, device=device)
        self.g32 = torch.zeros(self.numel, dtype=torch.float32, device=device)
        self.p16 = torch.zeros(self.numel, dtype=torch.float16, device=device)
        with torch.no_grad():
            for n, p in named:
                view = self.p32_view(n, p.shape)
                view.copy_(p.detach().to(device=device, dtype=torch.float32))
                p.data = view
        # Flat indices of the parameters the kernels read in fp32 (the 1-D norm gains and biases; every matrix
        # is read from the fp16 copy). A sharded update must hand their new values to every rank.
        idx = [torch.arange(self.offsets[n], self.offsets[n] + p.numel()) for n, p in named if p.dim() == 1]
        self.f32_read_index = (torch.cat(idx) if idx else torch.zeros(0, dtype=torch.long)).to(device)
        self._versions: list[int] | None = None
        self.generation = 0  # bumped whenever the fp16 weights are rewritten (caches derived from them go stale)
        # Per-update state filled by GradScaler.unscale_ / clip_grad_norm_ and
        # consumed by the fused optimizer step.
        self.inv_scale: torch.Tensor | None = None
        self.found_inf: torch.Tensor | None = None
        self.clip: torch.Tensor | None = None
        self.stats_ready = False  # stats_partial holds this update's sums of squares
        self.stats_parts = ops.grad_stats_parts(self.numel)
        self.stats_partial = torch.zeros(self.stats_parts, dtype=torch.float32, device=device)
        self.stats_count = self.stats_parts  # partial sums written by the last statistics pass
        self.norm_out = torch.zeros(2, dtype=torch.float32, device=device)
        self.refresh_f16(force=True)

    def p32_view(self, name: str, shape) -> torch.Tensor:
        o = self.offsets[name]
        n = math.prod(shape)
        return self.p32[o:o + n].view(shape)

    def g32_view(self, name: str, shape) -> torch.Tensor:
        o = self.offsets[name]
        return self.g32[o:o + math.prod(shape)].view(shape)

    def p16_rows(self, first: str, rows: int, cols: int) -> torch.Tensor:
        o = self.offsets[first]
        return self.p16[o:o + rows * cols].view(rows, cols)

    def g32_rows(self, first: str, rows: int, cols: int) -> torch.Tensor:
        o = self.offsets[first]
        return self.g32[o:o + rows * cols].view(rows, cols)

    def owns(self, model: "JishuiForCausalLM") -> bool:
        for n, p in model.named_parameters():
            o = self.offsets.get(n)
            if o is None or p.device != self.device or p.data_ptr() != self.p32.data_ptr() + 4 * o:
                return False
        return True

    def refresh_f16(self, force: bool = False) -> None:
        """Re-casts the fp16 weight copy if any parameter was modified in place."""
        versions = [p._version for p in self.params]
        if force or versions != self._versions:
            ops.cast_f32_f16(self.p32, self.p16)
            self._versions = versions
            self.generation += 1

    def mark_f16_current(self) -> None:
        """Called after a fused update that rewrote p32 and p16 together."""
        self._versions = [p._version for p in self.params]
        self.generation += 1

    def prepare_grads(self) -> bool:
        """Attaches flat-buffer views as `.grad`; returns True to accumulate into
        the existing gradient, False when every gradient was unset (overwrite)."""
        grads = [p.grad for p in self.params]
        if all(g is None for g in grads):
            for n, p in zip(self.names, self.params):
                p.grad = self.g32_view(n, p.shape)
            return False
        with torch.no_grad():
            for n, p in zip(self.names, self.params):
                view = self.g32_view(n, p.shape)
                if p.grad is None:
                    view.zero_()
                elif p.grad.data_ptr() != view.data_ptr():
                    view.copy_(p.grad)
                p.grad = view
        return True


# --------------------------------------------------------------------------- activation workspace
@dataclass
class LayerActs:
    h1: torch.Tensor
    mean1: torch.Tensor               # LayerNorm only (unused for RMSNorm)
    rstd1: torch.Tensor
    qkv: torch.Tensor
    o: torch.Tensor
    lse: torch.Tensor
    xmid: torch.Tensor
    h2: torch.Tensor
    mean2: torch.Tensor
    rstd2: torch.Tensor
    gate: torch.Tensor
    up: torch.Tensor
    act: torch.Tensor


@dataclass
class Workspace:
    B: int
    T: int
    xs: torch.Tensor                  # [L+1, M, d] residual stream at every layer boundary
    acts: list[LayerActs]             # per layer, or a single recompute slot under checkpointing
    hf: torch.Tensor
    meanf: torch.Tensor
    rstdf: torch.Tensor
    logits: torch.Tensor              # [M, V] fp16; overwritten in place by dlogits in backward
    ce_lse: torch.Tensor
    row_loss: torch.Tensor
    ce_parts: torch.Tensor            # [M, ceil(V/128), 2] head-epilogue cross-entropy statistics
    dx: torch.Tensor
    dxmid: torch.Tensor
    dh: torch.Tensor
    do: torch.Tensor
    dqkv: torch.Tensor
    dgu: torch.Tensor
    attn_ws: torch.Tensor
    attn_fwd_ws: torch.Tensor
    norm_part: torch.Tensor
    wgrad_ws: torch.Tensor
    cos: torch.Tensor
    sin: torch.Tensor
    extra: dict = field(default_factory=dict)


def _wgrad_splits(n: int, k: int, tokens: int = 16384, pairs: int = 74) -> int:
    """Split count for a weight-gradient GEMM with [n, k] output reducing over
    `tokens`, for the 2-SM kernel (a CTA pair per 256 x 256 tile, `pairs` pairs
    resident): minimises (waves x per-split main loop) + the split-K cost (clearing
    and reading back the one fp32 accumulator, the splits' reduce-adds in L2), at
    ~14.8 TFLOP/s per pair and 6 TB/s."""
    tiles = -(-n // 256) * -(-k // 256)
    tile_us = 2.0 * 256 * 256 * tokens / 14.8e6  # one tile over all tokens, microseconds
    best, best_t = 1, None
    for s in range(1, 9):
        if tokens // s < 1024:
            break
        t = math.ceil(tiles * s / pairs) * tile_us / s
        if s > 1:
            t += (2.0 + 0.25 * s) * n * k * 4 / 6e6
        if best_t is None or t < best_t * 0.97:
            best, best_t = s, t
    return best


# --------------------------------------------------------------------------- the model
class JishuiForCausalLM(nn.Module):
    def __init__(self, config: ModelConfig):
        super().__init__()
        check_supported(config)
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList([TransformerBlock(config) for _ in range(config.num_hidden_layers)])
        self.norm = make_norm(config)
        self._flat: FlatParams | None = None
        self._ws: dict = {}
        self._gen = 0
        self.grad_reducer = None  # set by midstream_llm_b200.distributed for data-parallel runs
        ref = weakref.ref(self)
        for p in self.parameters():
            _PARAM_OWNER[id(p)] = (weakref.ref(p), ref)

    # ---- storage -------------------------------------------------------
    def flat(self) -> FlatParams:
        dev = self.embed_tokens.weight.device
        if dev.type != "cuda":
            raise RuntimeError("JishuiForCausalLM (B200) runs on CUDA only: move it with .cuda() / .to('cuda')")
        if self._flat is None or not self._flat.owns(self):
            self._flat = FlatParams(self, dev)
            self._ws.clear()
        return self._flat

    def _workspace(self, B: int, T: int, train: bool) -> Workspace:
        key = (B, T, train, bool(self.config.gradient_checkpointing and train))
        ws = self._ws.get(key)
        if ws is not None:
            return ws
        c = self.config
        dev = self.embed_tokens.weight.device
        M, d, F, H = B * T, c.hidden_size, c.intermediate_size, c.num_attention_heads
        f16 = dict(dtype=torch.float16, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        L = c.num_hidden_layers
        nslots = 1 if (not train or c.gradient_checkpointing) else L

        def acts():
            return LayerActs(h1=torch.empty(M, d, **f16), mean1=torch.empty(M, **f32), rstd1=torch.empty(M, **f32),
                             qkv=torch.empty(M, 3 * d, **f16),
                             o=torch.empty(M, d, **f16), lse=torch.empty(B, H, T, **f32), xmid=torch.empty(M, d, **f16),
                             h2=torch.empty(M, d, **f16), mean2=torch.empty(M, **f32), rstd2=torch.empty(M, **f32),
                             gate=torch.empty(M, F, **f16), up=torch.empty(M, F, **f16), act=torch.empty(M, F, **f16))

        cos, sin = rope_tables(T, c.head_dim, c.rope_theta, dev)
        nparts = _lib.query("jx_rmsnorm_bwd_parts", M)
        wmax = 0
        if train:
            for n, k in ((3 * d, d), (d, d), (2 * F, d), (d, F), (c.vocab_size, d)):
                s = _wgrad_splits(n, k, M)
                wmax = max(wmax, ops.wgrad_workspace_bytes(n, k, s))
        xs_slots = L + 1 if train else 2
        ws = Workspace(
            B=B, T=T, xs=torch.empty(xs_slots, M, d, **f16), acts=[acts() for _ in range(nslots)],
            hf=torch.empty(M, d, **f16), meanf=torch.empty(M, **f32), rstdf=torch.empty(M, **f32), logits=torch.empty(M, c.vocab_size, **f16),
            ce_lse=torch.empty(M, **f32), row_loss=torch.empty(M, **f32),
            ce_parts=torch.empty(M, ops.ce_parts_blocks(c.vocab_size), 2, **f32),
            dx=torch.empty(M, d, **f16) if train else None, dxmid=torch.empty(M, d, **f16) if train else None,
            dh=torch.empty(M, d, **f16) if train else None, do=torch.empty(M, d, **f16) if train else None,
            dqkv=torch.empty(M, 3 * d, **f16) if train else None, dgu=torch.empty(M, 2 * F, **f16) if train else None,
            attn_ws=torch.empty(ops.attn_bwd_workspace_bytes(B, T, H, c.head_dim) // 4 + 4, **f32) if train else None,
            attn_fwd_ws=torch.empty(ops.attn_fwd_workspace_bytes(B, T, H, c.head_dim) // 4 + 4, **f32),
            norm_part=torch.empty(2 * nparts * d, **f32), wgrad_ws=torch.empty(max(wmax // 4, 4), **f32),
            cos=cos, sin=sin)
        self._ws[key] = ws
        return ws

    # ---- weight views ------------------------------------------------------
    def _layer_weights(self, fl: FlatParams, i: int):
        c = self.config
        d, F = c.hidden_size, c.intermediate_size
        pre = f"layers.{i}."
        q, k, v = (pre + f"attention.{x}_proj.weight" for x in "qkv")
        g, u = pre + "mlp.gate_proj.weight", pre + "mlp.up_proj.weight"
        if fl.offsets[k] != fl.offsets[q] + d * d or fl.offsets[v] != fl.offsets[k] + d * d:
            raise RuntimeError("q/k/v weights are not adjacent in the flat buffer")
        if fl.offsets[u] != fl.offsets[g] + F * d:
            raise RuntimeError("gate/up weights are not adjacent in the flat buffer")
        return dict(
            wqkv=fl.p16_rows(q, 3 * d, d), wo=fl.p16_rows(pre + "attention.o_proj.weight", d, d),
            wgu=fl.p16_rows(g, 2 * F, d), wd=fl.p16_rows(pre + "mlp.down_proj.weight", d, F),
            g1=fl.p32_view(pre + "input_norm.weight", (d,)), g2=fl.p32_view(pre + "post_attention_norm.weight", (d,)),
            gqkv=fl.g32_rows(q, 3 * d, d), go=fl.g32_rows(pre + "attention.o_proj.weight", d, d),
            ggu=fl.g32_rows(g, 2 * F, d), gd=fl.g32_rows(pre + "mlp.down_proj.weight", d, F),
            gg1=fl.g32_view(pre + "input_norm.weight", (d,)), gg2=fl.g32_view(pre + "post_attention_norm.weight", (d,)),
            b1=self._bias_view(fl.p32_view, pre + "input_norm.bias"),
            b2=self._bias_view(fl.p32_view, pre + "post_attention_norm.bias"),
            gb1=self._bias_view(fl.g32_view, pre + "input_norm.bias"),
            gb2=self._bias_view(fl.g32_view, pre + "post_attention_norm.bias"),
            lo=fl.offsets[pre + "input_norm.weight"],
            hi=fl.offsets[pre + "mlp.down_proj.weight"] + _round_up(d * F))

    def _bias_view(self, view, name: str):
        """fp32 view of a LayerNorm bias (None when the configuration has none)."""
        if self.config.norm_type == "rmsnorm" or not self.config.norm_bias:
            return None
        return view(name, (self.config.hidden_size,))

    # ---- norm dispatch (RMSNorm or LayerNorm, model_torch.py:12-15) ------------
    def _norm_fwd(self, x, gamma, beta, out, mean, rstd) -> None:
        c = self.config
        if c.norm_type == "rmsnorm":
            ops.rmsnorm_fwd(x, gamma, c.norm_eps, out=out, rstd=rstd)
        else:
            ops.layernorm_fwd(x, gamma, beta, c.norm_eps, out=out, mean=mean, rstd=rstd)

    def _norm_bwd(self, dy, x, mean, rstd, gamma, dgamma, dbeta, acc, dresid, out, part) -> None:
        if self.config.norm_type == "rmsnorm":
            ops.rmsnorm_bwd(dy, x, rstd, gamma, dresid=dresid, out=out, dgamma=dgamma, accumulate=acc, part=part)
        else:
            ops.layernorm_bwd(dy, x, mean, rstd, gamma, dgamma=dgamma, dbeta=dbeta, accumulate=acc, dresid=dresid,
                              out=out, part=part)

    # ---- forward pieces ------------------------------------------------------
    def _layer_fwd(self, w, ws: Workspace, x_in: torch.Tensor, x_out: torch.Tensor, A: LayerActs) -> None:
        c = self.config
        B, T = ws.B, ws.T
        d, F, H, hd = c.hidden_size, c.intermediate_size, c.num_attention_heads, c.head_dim
        self._norm_fwd(x_in, w["g1"], w["b1"], A.h1, A.mean1, A.rstd1)
        ops.gemm_qkv_rope(A.h1, w["wqkv"], d, ws.cos, ws.sin, T, hd, out=A.qkv)
        ops.attn_fwd(A.qkv, B, T, H, hd, out=A.o, lse=A.lse, workspace=ws.attn_fwd_ws)
        ops.gemm_f16(A.o, w["wo"], resid=x_in, out=A.xmid)
        self._norm_fwd(A.xmid, w["g2"], w["b2"], A.h2, A.mean2, A.rstd2)
        ops.gemm_swiglu_fwd(A.h2, w["wgu"], F, gate=A.gate, up=A.up, act=A.act)
        ops.gemm_f16(A.act, w["wd"], resid=A.xmid, out=x_out)

    def _trunk_fwd(self, ids: torch.Tensor, train: bool, ce: bool = False) -> Workspace:
        c = self.config
        B, T = ids.shape  # already padded to the sequence tile (callers check the unpadded length)
        if T % _SEQ_TILE:
            raise ValueError(f"internal: sequence length {T} is not a multiple of {_SEQ_TILE}")
        fl = self.flat()
        fl.refresh_f16()
        ws = self._workspace(B, T, train)
        e16 = fl.p16_rows("embed_tokens.weight", c.vocab_size, c.hidden_size)
        ops.embed_fwd(ids.reshape(-1), e16, out=ws.xs[0])
        ckpt = train and c.gradient_checkpointing
        for i in range(c.num_hidden_layers):
            w = self._layer_weights(fl, i)
            if train:
                x_in, x_out = ws.xs[i], ws.xs[i + 1]
            else:
                x_in, x_out = ws.xs[i % 2], ws.xs[(i + 1) % 2]
            A = ws.acts[0 if (ckpt or not train) else i]
            self._layer_fwd(w, ws, x_in, x_out, A)
        x_last = ws.xs[c.num_hidden_layers] if train else ws.xs[c.num_hidden_layers % 2]
        self._norm_fwd(x_last, fl.p32_view("norm.weight", (c.hidden_size,)), self._bias_view(fl.p32_view, "norm.bias"),
                       ws.hf, ws.meanf, ws.rstdf)
        if ce:  # the head also leaves the cross-entropy statistics of its logits (ce_fwd_parts)
            ops.gemm_f16_ce_parts(ws.hf, e16, out=ws.logits, parts=ws.ce_parts)
        else:
            ops.gemm_f16(ws.hf, e16, out=ws.logits)
        ws.extra["x_last"] = x_last
        return ws

    # ---- public forward ------------------------------------------------------
    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        """logits [B, T, V] in fp16 (model_torch.py:86-98), for any T up to max_position_embeddings."""
        T = input_ids.shape[-1]
        if T > self.config.max_position_embeddings:
            raise ValueError("sequence exceeds configured context length")
        ids = _pad_rows(input_ids.to(torch.int64).contiguous(), 0)
        if torch.is_grad_enabled() and self.embed_tokens.weight.requires_grad:
            return _LogitsFn.apply(self, ids, T, *self.parameters())
        ws = self._trunk_fwd(ids, train=False)
        return _unpad_logits(ws, T)

    def loss(self, inputs: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100) -> torch.Tensor:
        """Mean cross-entropy of next-token prediction through the fused head (any T up to
        max_position_embeddings; padded positions are ignored targets)."""
        if inputs.shape[-1] > self.config.max_position_embeddings:
            raise ValueError("sequence exceeds configured context length")
        if targets.shape != inputs.shape:
            raise ValueError(f"targets {tuple(targets.shape)} and inputs {tuple(inputs.shape)} differ in shape")
        ids = _pad_rows(inputs.to(torch.int64).contiguous(), 0)
        tg = _pad_rows(targets.to(torch.int64).contiguous(), ignore_index)
        if torch.is_grad_enabled() and self.embed_tokens.weight.requires_grad:
            return _LossFn.apply(self, ids, tg, ignore_index, *self.parameters())
        ws = self._trunk_fwd(ids, train=False, ce=True)
        return self._ce_forward(ws, tg.reshape(-1), ignore_index)[2].clone()

    def _ce_forward(self, ws: Workspace, tg: torch.Tensor, ignore_index: int) -> torch.Tensor:
        """Loss from the statistics the head left in ws.ce_parts (the trunk ran with ce=True)."""
        ops.ce_fwd_parts(ws.ce_parts, ws.logits, tg, ignore_index, lse=ws.ce_lse, row_loss=ws.row_loss)
        out = torch.empty(3, dtype=torch.float32, device=ws.logits.device)
        ops.ce_loss(ws.row_loss, tg, ignore_index, out=out)
        return out

    # ---- backward ------------------------------------------------------------
    def _backward_from_dlogits(self, ws: Workspace, ids: torch.Tensor) -> None:
        """ws.logits holds f16 dlogits; writes every parameter's gradient."""
        c = self.config
        fl = self.flat()
        accumulate = fl.prepare_grads()
        fl.stats_ready, fl.clip = False, None  # the gradients change: earlier norm statistics are stale
        d, V, L = c.hidden_size, c.vocab_size, c.num_hidden_layers
        reducer = self.grad_reducer
        if reducer is not None:
            reducer.begin(fl)
        e16 = fl.p16_rows("embed_tokens.weight", V, d)
        ge = fl.g32_rows("embed_tokens.weight", V, d)
        ops.gemm_f16(ws.logits, e16, b_mn_major=True, out=ws.dh)
        ops.gemm_wgrad(ws.logits, ws.hf, ge, accumulate, _wgrad_splits(V, d, ws.B * ws.T), ws.wgrad_ws)
        x_last = ws.extra["x_last"]
        self._norm_bwd(ws.dh, x_last, ws.meanf, ws.rstdf, fl.p32_view("norm.weight", (d,)),
                       fl.g32_view("norm.weight", (d,)), self._bias_view(fl.g32_view, "norm.bias"), accumulate, None,
                       ws.dx, ws.norm_part)
        if reducer is not None:
            o = fl.offsets["norm.weight"]
            last = "norm.bias" if "norm.bias" in fl.offsets else "norm.weight"
            reducer.ready(o, fl.offsets[last] + _round_up(d))
        ckpt = c.gradient_checkpointing
        for i in reversed(range(L)):
            w = self._layer_weights(fl, i)
            A = ws.acts[0 if ckpt else i]
            if ckpt:
                scratch = ws.extra.setdefault("ckpt_out", torch.empty_like(ws.dx))
                self._layer_fwd(w, ws, ws.xs[i], scratch, A)
            self._layer_bwd(w, ws, A, ws.xs[i], accumulate)
            if reducer is not None:
                reducer.ready(w["lo"], w["hi"])
        ops.embed_bwd(ids.reshape(-1), ws.dx, ge)
        if reducer is not None:
            reducer.ready(0, _round_up(V * d))
            reducer.finish()

    def _layer_bwd(self, w, ws: Workspace, A: LayerActs, x_in: torch.Tensor, acc: bool) -> None:
        c = self.config
        B, T = ws.B, ws.T
        M = B * T
        d, F, H, hd = c.hidden_size, c.intermediate_size, c.num_attention_heads, c.head_dim
        ops.gemm_swiglu_bwd(ws.dx, w["wd"], A.gate, A.up, out=ws.dgu)
        ops.gemm_wgrad(ws.dx, A.act, w["gd"], acc, _wgrad_splits(d, F, M), ws.wgrad_ws)
        ops.gemm_f16(ws.dgu, w["wgu"], b_mn_major=True, out=ws.dh)
        ops.gemm_wgrad(ws.dgu, A.h2, w["ggu"], acc, _wgrad_splits(2 * F, d, M), ws.wgrad_ws)
        self._norm_bwd(ws.dh, A.xmid, A.mean2, A.rstd2, w["g2"], w["gg2"], w["gb2"], acc, ws.dx, ws.dxmid, ws.norm_part)
        ops.gemm_f16(ws.dxmid, w["wo"], b_mn_major=True, out=ws.do)
        ops.gemm_wgrad(ws.dxmid, A.o, w["go"], acc, _wgrad_splits(d, d, M), ws.wgrad_ws)
        ops.attn_bwd(A.qkv, A.o, ws.do, A.lse, B, T, H, hd, cos=ws.cos, sin=ws.sin, out=ws.dqkv, workspace=ws.attn_ws)
        ops.gemm_f16(ws.dqkv, w["wqkv"], b_mn_major=True, out=ws.dh)
        ops.gemm_wgrad(ws.dqkv, A.h1, w["gqkv"], acc, _wgrad_splits(3 * d, d, M), ws.wgrad_ws)
        self._norm_bwd(ws.dh, x_in, A.mean1, A.rstd1, w["g1"], w["gg1"], w["gb1"], acc, ws.dxmid, ws.dx, ws.norm_part)


class _LossFn(torch.autograd.Function):
    """Whole-model forward + fused CE; backward writes every parameter's .grad
    directly (the flat gradient buffer) and returns None for the parameters."""

    @staticmethod
    def forward(ctx, model: JishuiForCausalLM, ids, targets, ignore_index, *params):
        ws = model._trunk_fwd(ids, train=True, ce=True)
        tg = targets.reshape(-1)
        out = model._ce_forward(ws, tg, ignore_index)
        model._gen += 1
        ctx.model, ctx.gen, ctx.ws = model, model._gen, ws
        ctx.ignore_index = ignore_index
        ctx.save_for_backward(ids, tg, out)
        return out[2].clone()

    @staticmethod
    def backward(ctx, grad_loss):
        model, ws = ctx.model, ctx.ws
        if model._gen != ctx.gen:
            raise RuntimeError("another training forward ran before this backward; activations were overwritten")
        ids, tg, out = ctx.saved_tensors
        g = grad_loss.detach().to(torch.float32).reshape(1).contiguous()
        ops.ce_bwd(ws.logits, tg, ws.ce_lse, g, out[1:2], ctx.ignore_index)
        model._backward_from_dlogits(ws, ids)
        return (None, None, None, None) + (None,) * (len(ctx.needs_input_grad) - 4)


class _LogitsFn(torch.autograd.Function):
    """forward() under autograd: returns fp16 logits; backward takes dlogits."""

    @staticmethod
    def forward(ctx, model: JishuiForCausalLM, ids, T: int, *params):
        ws = model._trunk_fwd(ids, train=True)
        model._gen += 1
        ctx.model, ctx.gen, ctx.ws, ctx.T = model, model._gen, ws, T
        ctx.save_for_backward(ids)
        return _unpad_logits(ws, T)

    @staticmethod
    def backward(ctx, dlogits):
        model, ws = ctx.model, ctx.ws
        if model._gen != ctx.gen:
            raise RuntimeError("another training forward ran before this backward; activations were overwritten")
        (ids,) = ctx.saved_tensors
        B, Tp = ids.shape
        full = ws.logits.view(B, Tp, -1)
        full[:, :ctx.T].copy_(dlogits)
        full[:, ctx.T:].zero_()  # padded positions: no gradient
        model._backward_from_dlogits(ws, ids)
        return (None, None, None) + (None,) * (len(ctx.needs_input_grad) - 3)


def causal_lm_loss(model: JishuiForCausalLM, inputs: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Mean next-token cross-entropy (model_torch.py:102-104) through the fused head + CE."""
    return model.loss(inputs, targets)
