"""Tensor-level wrappers over the C ABI.

Every function takes CUDA tensors, validates dtype / device / layout, and
launches on torch's current stream. Outputs are allocated here (by torch's
caching allocator) unless passed in. There is no CPU path: a CPU tensor or a
missing library raises.
"""
from __future__ import annotations

import math

import torch

from . import _lib

F16, F32, I64 = torch.float16, torch.float32, torch.int64

# When set to a list, every GEMM launch appends (algorithmic FLOPs, start event,
# end event) recorded on the launching stream (used by bench.py's roofline).
_GEMM_PROFILE: list | None = None


def set_gemm_profile(records: list | None) -> None:
    global _GEMM_PROFILE
    _GEMM_PROFILE = records


class _GemmTimer:
    """Records (flops, algorithmic bytes, start event, end event) of one GEMM launch when profiling is on.
    Algorithmic bytes: each operand read once and each output written once (fp16 2 B, fp32 4 B)."""
    __slots__ = ("flops", "bytes", "start")

    def __init__(self, flops: float, nbytes: float = 0.0):
        self.flops = flops
        self.bytes = nbytes
        self.start = None

    def __enter__(self):
        if _GEMM_PROFILE is not None:
            self.start = torch.cuda.Event(enable_timing=True)
            self.start.record()
        return self

    def __exit__(self, *exc):
        if self.start is not None and _GEMM_PROFILE is not None:
            end = torch.cuda.Event(enable_timing=True)
            end.record()
            _GEMM_PROFILE.append((self.flops, self.bytes, self.start, end))


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _check(t: torch.Tensor, dtype: torch.dtype, name: str, contiguous: bool = True) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (the Jishui B200 kernels have no CPU path)")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


# ---------------------------------------------------------------- RMSNorm
def rmsnorm_fwd(x: torch.Tensor, gamma: torch.Tensor, eps: float, resid: torch.Tensor | None = None,
                out: torch.Tensor | None = None, sum_out: torch.Tensor | None = None,
                rstd: torch.Tensor | None = None):
    """Returns (y, rstd, s) where s = x (+ resid) is the normalised input."""
    _check(x, F16, "x")
    _check(gamma, F32, "gamma")
    cols = x.shape[-1]
    rows = x.numel() // cols
    y = out if out is not None else torch.empty_like(x)
    rstd = rstd if rstd is not None else torch.empty(rows, device=x.device, dtype=F32)
    s = x
    if resid is not None:
        _check(resid, F16, "resid")
        s = sum_out if sum_out is not None else torch.empty_like(x)
    _lib.call("jx_rmsnorm_fwd", x.data_ptr(), _ptr(resid), _ptr(s) if resid is not None else None, gamma.data_ptr(),
              y.data_ptr(), rstd.data_ptr(), rows, cols, float(eps), _stream())
    return y, rstd, s


def rmsnorm_bwd(dy: torch.Tensor, x: torch.Tensor, rstd: torch.Tensor, gamma: torch.Tensor,
                dresid: torch.Tensor | None = None, dgamma: torch.Tensor | None = None, accumulate: bool = False,
                out: torch.Tensor | None = None, part: torch.Tensor | None = None):
    """Returns (dx, dgamma); dgamma is accumulated into when `accumulate` and given."""
    _check(dy, F16, "dy")
    _check(x, F16, "x")
    _check(rstd, F32, "rstd")
    _check(gamma, F32, "gamma")
    cols = x.shape[-1]
    rows = x.numel() // cols
    dx = out if out is not None else torch.empty_like(x)
    nparts = _lib.query("jx_rmsnorm_bwd_parts", rows)
    if part is None or part.numel() < nparts * cols:
        part = torch.empty(nparts * cols, device=x.device, dtype=F32)
    if dresid is not None:
        _check(dresid, F16, "dresid")
    _lib.call("jx_rmsnorm_bwd", dy.data_ptr(), x.data_ptr(), rstd.data_ptr(), gamma.data_ptr(), _ptr(dresid),
              dx.data_ptr(), part.data_ptr(), rows, cols, _stream())
    if dgamma is None:
        dgamma = torch.empty(cols, device=x.device, dtype=F32)
        accumulate = False
    _lib.call("jx_rmsnorm_dgamma_reduce", part.data_ptr(), nparts, cols, dgamma.data_ptr(), int(accumulate), _stream())
    return dx, dgamma


def layernorm_fwd(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor | None, eps: float,
                  out: torch.Tensor | None = None, mean: torch.Tensor | None = None, rstd: torch.Tensor | None = None):
    """LayerNorm in fp32 over fp16 rows, fp16 output: returns (y, mean, rstd)."""
    _check(x, F16, "x")
    _check(gamma, F32, "gamma")
    if beta is not None:
        _check(beta, F32, "beta")
    cols = x.shape[-1]
    rows = x.numel() // cols
    y = out if out is not None else torch.empty_like(x)
    mean = mean if mean is not None else torch.empty(rows, device=x.device, dtype=F32)
    rstd = rstd if rstd is not None else torch.empty(rows, device=x.device, dtype=F32)
    _lib.call("jx_layernorm_fwd", x.data_ptr(), gamma.data_ptr(), _ptr(beta), y.data_ptr(), mean.data_ptr(),
              rstd.data_ptr(), rows, cols, float(eps), _stream())
    return y, mean, rstd


def layernorm_bwd(dy: torch.Tensor, x: torch.Tensor, mean: torch.Tensor, rstd: torch.Tensor, gamma: torch.Tensor,
                  dgamma: torch.Tensor | None = None, dbeta: torch.Tensor | None = None, accumulate: bool = False,
                  dresid: torch.Tensor | None = None, out: torch.Tensor | None = None,
                  part: torch.Tensor | None = None):
    """Returns (dx, dgamma, dbeta); dgamma / dbeta are accumulated into when `accumulate` and given.
    dbeta is computed only when a tensor is passed for it."""
    _check(dy, F16, "dy")
    _check(x, F16, "x")
    _check(gamma, F32, "gamma")
    cols = x.shape[-1]
    rows = x.numel() // cols
    dx = out if out is not None else torch.empty_like(x)
    nparts = _lib.query("jx_rmsnorm_bwd_parts", rows)
    if part is None or part.numel() < 2 * nparts * cols:
        part = torch.empty(2 * nparts * cols, device=x.device, dtype=F32)
    if dresid is not None:
        _check(dresid, F16, "dresid")
    pb = part[nparts * cols:] if dbeta is not None else None
    _lib.call("jx_layernorm_bwd", dy.data_ptr(), x.data_ptr(), mean.data_ptr(), rstd.data_ptr(), gamma.data_ptr(),
              _ptr(dresid), dx.data_ptr(), part.data_ptr(), _ptr(pb), rows, cols, _stream())
    if dgamma is None:
        dgamma = torch.empty(cols, device=x.device, dtype=F32)
        accumulate = False
    _lib.call("jx_rmsnorm_dgamma_reduce", part.data_ptr(), nparts, cols, dgamma.data_ptr(), int(accumulate), _stream())
    if dbeta is not None:
        _lib.call("jx_rmsnorm_dgamma_reduce", pb.data_ptr(), nparts, cols, dbeta.data_ptr(), int(accumulate),
                  _stream())
    return dx, dgamma, dbeta


# ---------------------------------------------------------------- embedding
def embed_fwd(ids: torch.Tensor, table16: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    _check(ids, I64, "ids")
    _check(table16, F16, "table16")
    vocab, cols = table16.shape
    y = out if out is not None else torch.empty(*ids.shape, cols, device=ids.device, dtype=F16)
    _lib.call("jx_embed_fwd", ids.data_ptr(), ids.numel(), table16.data_ptr(), vocab, cols, y.data_ptr(), _stream())
    return y


def embed_bwd(ids: torch.Tensor, dout16: torch.Tensor, dtable: torch.Tensor) -> None:
    _check(ids, I64, "ids")
    _check(dout16, F16, "dout16")
    _check(dtable, F32, "dtable")
    vocab, cols = dtable.shape
    _lib.call("jx_embed_bwd", ids.data_ptr(), ids.numel(), dout16.data_ptr(), vocab, cols, dtable.data_ptr(),
              _stream())


# ---------------------------------------------------------------- GEMMs
def _ld(t: torch.Tensor) -> int:
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError("GEMM operands must be 2-D with unit column stride")
    return t.stride(0)


def gemm_f16(a: torch.Tensor, b: torch.Tensor, a_mn_major: bool = False, b_mn_major: bool = False,
             resid: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """C[m][n] = sum_k A[m][k] B[n][k] (fp16 out). a is [M,K] (or [K,M] if a_mn_major);
    b is [N,K] (or [K,N] if b_mn_major)."""
    _check(a, F16, "a", contiguous=False)
    _check(b, F16, "b", contiguous=False)
    M, K = (a.shape[1], a.shape[0]) if a_mn_major else a.shape
    N, Kb = (b.shape[1], b.shape[0]) if b_mn_major else b.shape
    if K != Kb:
        raise ValueError(f"inner dimensions differ: {K} vs {Kb}")
    c = out if out is not None else torch.empty(M, N, device=a.device, dtype=F16)
    if resid is not None:
        _check(resid, F16, "resid", contiguous=False)
    with _GemmTimer(2.0 * M * N * K, 2.0 * (M * K + N * K + M * N * (2 if resid is not None else 1))):
        _lib.call("jx_gemm_f16", a.data_ptr(), _ld(a), int(a_mn_major), b.data_ptr(), _ld(b), int(b_mn_major), M, N,
                  K, c.data_ptr(), _ld(c), _ptr(resid), _ld(resid) if resid is not None else 0, _stream())
    return c


def gemm_qkv_rope(x: torch.Tensor, w: torch.Tensor, hidden: int, cos: torch.Tensor, sin: torch.Tensor, seq_len: int,
                  head_dim: int, out: torch.Tensor | None = None) -> torch.Tensor:
    _check(x, F16, "x")
    _check(w, F16, "w")
    _check(cos, F32, "cos")
    _check(sin, F32, "sin")
    M, K = x.shape
    c = out if out is not None else torch.empty(M, 3 * hidden, device=x.device, dtype=F16)
    with _GemmTimer(2.0 * M * 3 * hidden * K, 2.0 * (M * K + 3 * hidden * K + M * 3 * hidden)):
        _lib.call("jx_gemm_qkv_rope", x.data_ptr(), K, w.data_ptr(), M, hidden, K, c.data_ptr(), _ld(c),
                  cos.data_ptr(), sin.data_ptr(), seq_len, head_dim, _stream())
    return c


def gemm_swiglu_fwd(x: torch.Tensor, wgu: torch.Tensor, F: int, gate=None, up=None, act=None):
    _check(x, F16, "x")
    _check(wgu, F16, "wgu")
    M, K = x.shape
    mk = lambda: torch.empty(M, F, device=x.device, dtype=F16)  # noqa: E731
    gate = gate if gate is not None else mk()
    up = up if up is not None else mk()
    act = act if act is not None else mk()
    with _GemmTimer(2.0 * M * 2 * F * K, 2.0 * (M * K + 2 * F * K + 3 * M * F)):
        _lib.call("jx_gemm_swiglu_fwd", x.data_ptr(), K, wgu.data_ptr(), M, F, K, gate.data_ptr(), up.data_ptr(),
                  act.data_ptr(), F, _stream())
    return gate, up, act


def gemm_swiglu_bwd(dy: torch.Tensor, wd: torch.Tensor, gate: torch.Tensor, up: torch.Tensor,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """dy [M, d], wd [d, F] -> dgu [M, 2F] = [d gate | d up]."""
    _check(dy, F16, "dy")
    _check(wd, F16, "wd")
    M, K = dy.shape
    F = wd.shape[1]
    dgu = out if out is not None else torch.empty(M, 2 * F, device=dy.device, dtype=F16)
    with _GemmTimer(2.0 * M * F * K, 2.0 * (M * K + F * K + 2 * M * F + 2 * M * F)):
        _lib.call("jx_gemm_swiglu_bwd", dy.data_ptr(), K, wd.data_ptr(), M, F, K, gate.data_ptr(), up.data_ptr(), F,
                  dgu.data_ptr(), _ld(dgu), _stream())
    return dgu


def wgrad_workspace_bytes(N: int, K: int, splits: int) -> int:
    return _lib.query("jx_gemm_wgrad_workspace_bytes", N, K, splits)


def gemm_wgrad(dy: torch.Tensor, x: torch.Tensor, g: torch.Tensor, accumulate: bool, splits: int = 1,
               workspace: torch.Tensor | None = None) -> None:
    """g[n][k] (+)= f32(f16(sum_t dy[t][n] x[t][k]))."""
    _check(dy, F16, "dy", contiguous=False)
    _check(x, F16, "x", contiguous=False)
    _check(g, F32, "g", contiguous=False)
    T, N = dy.shape
    K = x.shape[1]
    if splits > 1:
        need = wgrad_workspace_bytes(N, K, splits)
        if workspace is None or workspace.numel() * workspace.element_size() < need:
            workspace = torch.empty(need // 4 + 1, device=dy.device, dtype=F32)
    with _GemmTimer(2.0 * T * N * K, 2.0 * (T * N + T * K) + 4.0 * N * K * (2 if accumulate else 1)):
        _lib.call("jx_gemm_wgrad", dy.data_ptr(), _ld(dy), x.data_ptr(), _ld(x), T, N, K, g.data_ptr(), _ld(g),
                  int(accumulate), splits, _ptr(workspace), _stream())


# ---------------------------------------------------------------- attention
def attn_fwd_workspace_bytes(B: int, T: int, H: int, D: int) -> int:
    return _lib.query("jx_attn_fwd_workspace_bytes", B, T, H, D)


def attn_fwd(qkv: torch.Tensor, B: int, T: int, H: int, D: int, out: torch.Tensor | None = None,
             lse: torch.Tensor | None = None, workspace: torch.Tensor | None = None):
    """Causal attention forward: (out f16 [B*T, H*D], lse f32 [B, H, T]). `workspace` holds the
    kernel's work counter; without one a fresh buffer is taken from torch's allocator."""
    _check(qkv, F16, "qkv")
    o = out if out is not None else torch.empty(B * T, H * D, device=qkv.device, dtype=F16)
    lse = lse if lse is not None else torch.empty(B, H, T, device=qkv.device, dtype=F32)
    need = attn_fwd_workspace_bytes(B, T, H, D)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need // 4 + 4, device=qkv.device, dtype=F32)
    _lib.call("jx_attn_fwd", qkv.data_ptr(), o.data_ptr(), lse.data_ptr(), workspace.data_ptr(), B, T, H, D,
              1.0 / math.sqrt(D), _stream())
    return o, lse


def attn_bwd_workspace_bytes(B: int, T: int, H: int, D: int) -> int:
    return _lib.query("jx_attn_bwd_workspace_bytes", B, T, H, D)


def attn_bwd(qkv, o, do, lse, B, T, H, D, cos=None, sin=None, out=None, workspace=None):
    """dqkv f16 [B*T, 3*H*D]; q/k gradients rotated back through RoPE when tables are given."""
    _check(do, F16, "do")
    dqkv = out if out is not None else torch.empty_like(qkv)
    need = attn_bwd_workspace_bytes(B, T, H, D)
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty(need // 4 + 4, device=qkv.device, dtype=F32)
    _lib.call("jx_attn_bwd", qkv.data_ptr(), o.data_ptr(), do.data_ptr(), lse.data_ptr(), workspace.data_ptr(),
              dqkv.data_ptr(), B, T, H, D, 1.0 / math.sqrt(D), _ptr(cos), _ptr(sin), _stream())
    return dqkv


def attn_decode_workspace_bytes(B: int, H: int, max_len: int) -> int:
    return _lib.query("jx_attn_decode_workspace_bytes", B, H, max_len)


def attn_decode(qkv: torch.Tensor, kcache: torch.Tensor, vcache: torch.Tensor, length: int, H: int, D: int,
                workspace: torch.Tensor, out: torch.Tensor | None = None,
                length_dev: torch.Tensor | None = None) -> torch.Tensor:
    """One new token per sequence against the KV cache. qkv [B, 3*H*D] (the new rows), kcache / vcache
    [B, max_len, H*D] holding positions < length-1; appends the new k / v at length-1; returns [B, H*D].
    With `length_dev` (int32 scalar on the device) the length is read there and `length` is its upper bound."""
    _check(qkv, F16, "qkv")
    _check(kcache, F16, "kcache")
    _check(vcache, F16, "vcache")
    B = qkv.shape[0]
    if kcache.stride() != vcache.stride() or kcache.shape[1] < length:
        raise ValueError("attn_decode: caches must share a layout and hold `length` positions")
    o = out if out is not None else torch.empty(B, H * D, device=qkv.device, dtype=F16)
    if length_dev is not None and length_dev.dtype != torch.int32:
        raise ValueError("attn_decode: length_dev must be int32")
    _lib.call("jx_attn_decode", qkv.data_ptr(), _ld(qkv), kcache.data_ptr(), vcache.data_ptr(), kcache.stride(1),
              kcache.stride(0), B, length, _ptr(length_dev), H, D, 1.0 / math.sqrt(D), workspace.data_ptr(),
              o.data_ptr(), _ld(o), _stream())
    return o


# ---------------------------------------------------------------- cross-entropy
def ce_fwd(logits16: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100, lse=None, row_loss=None):
    _check(targets, I64, "targets")
    rows, vocab = logits16.shape
    lse = lse if lse is not None else torch.empty(rows, device=logits16.device, dtype=F32)
    row_loss = row_loss if row_loss is not None else torch.empty(rows, device=logits16.device, dtype=F32)
    _lib.call("jx_ce_fwd", logits16.data_ptr(), rows, vocab, _ld(logits16), targets.data_ptr(), ignore_index,
              lse.data_ptr(), row_loss.data_ptr(), _stream())
    return lse, row_loss


def ce_parts_blocks(vocab: int) -> int:
    """Number of 128-column blocks of the head's cross-entropy partial statistics."""
    return (vocab + 127) // 128


def gemm_f16_ce_parts(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor | None = None,
                      parts: torch.Tensor | None = None):
    """The tied head C = a b^T (fp16 logits, as gemm_f16) plus parts [M, ceil(N/128), 2] fp32: (max,
    sum exp(v - max)) of each 128-column block of the fp16 logits v, for ce_fwd_parts."""
    _check(a, F16, "a", contiguous=False)
    _check(b, F16, "b", contiguous=False)
    M, K = a.shape
    N, Kb = b.shape
    if K != Kb:
        raise ValueError(f"inner dimensions differ: {K} vs {Kb}")
    c = out if out is not None else torch.empty(M, N, device=a.device, dtype=F16)
    nblk = ce_parts_blocks(N)
    if parts is None:
        parts = torch.empty(M, nblk, 2, device=a.device, dtype=F32)
    _check(parts, F32, "parts")
    if parts.numel() < M * nblk * 2:
        raise ValueError("parts is too small")
    with _GemmTimer(2.0 * M * N * K, 2.0 * (M * K + N * K + M * N)):
        _lib.call("jx_gemm_f16_ce_parts", a.data_ptr(), _ld(a), b.data_ptr(), _ld(b), M, N, K, c.data_ptr(), _ld(c),
                  parts.data_ptr(), _stream())
    return c, parts


def ce_fwd_parts(parts: torch.Tensor, logits16: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100,
                 lse=None, row_loss=None):
    """ce_fwd from the head GEMM's partial statistics (only the target logits are read)."""
    _check(targets, I64, "targets")
    _check(parts, F32, "parts")
    rows, vocab = logits16.shape
    lse = lse if lse is not None else torch.empty(rows, device=logits16.device, dtype=F32)
    row_loss = row_loss if row_loss is not None else torch.empty(rows, device=logits16.device, dtype=F32)
    _lib.call("jx_ce_fwd_parts", parts.data_ptr(), ce_parts_blocks(vocab), logits16.data_ptr(), rows, vocab,
              _ld(logits16), targets.data_ptr(), ignore_index, lse.data_ptr(), row_loss.data_ptr(), _stream())
    return lse, row_loss


def ce_loss(row_loss: torch.Tensor, targets: torch.Tensor, ignore_index: int = -100,
            out: torch.Tensor | None = None, accumulate: bool = False) -> torch.Tensor:
    out = out if out is not None else torch.zeros(3, device=row_loss.device, dtype=F32)
    _lib.call("jx_ce_loss", row_loss.data_ptr(), targets.data_ptr(), ignore_index, row_loss.numel(), out.data_ptr(),
              int(accumulate), _stream())
    return out


def ce_bwd(logits16, targets, lse, grad_loss: torch.Tensor, count: torch.Tensor, ignore_index: int = -100) -> None:
    rows, vocab = logits16.shape
    _lib.call("jx_ce_bwd", logits16.data_ptr(), rows, vocab, _ld(logits16), targets.data_ptr(), ignore_index,
              lse.data_ptr(), grad_loss.data_ptr(), count.data_ptr(), _stream())


# ---------------------------------------------------------------- optimizer
def grad_stats(grad: torch.Tensor, inv_scale: torch.Tensor, partial: torch.Tensor, found_inf: torch.Tensor,
               unscaled_out: torch.Tensor | None = None) -> int:
    """Per-block sums of (g * inv_scale)^2 into `partial`, found_inf = 1 on a non-finite element; with
    `unscaled_out` (f32, may be `grad` itself) the unscaled gradients are written there too."""
    n = grad.numel()
    nparts = _lib.query("jx_grad_stats_parts", n)
    if unscaled_out is not None:
        _check(unscaled_out, F32, "unscaled_out")
        if unscaled_out.numel() != n:
            raise ValueError("unscaled_out must have as many elements as grad")
    _lib.call("jx_grad_stats", grad.data_ptr(), int(grad.dtype == F16), n, inv_scale.data_ptr(), partial.data_ptr(),
              found_inf.data_ptr(), _ptr(unscaled_out), _stream())
    return nparts


def grad_stats_parts(n: int) -> int:
    return _lib.query("jx_grad_stats_parts", n)


def grad_finalize(partial: torch.Tensor, nparts: int, max_norm: float, out: torch.Tensor) -> None:
    _lib.call("jx_grad_finalize", partial.data_ptr(), nparts, float(max_norm), out.data_ptr(), _stream())


def adamw_step(p, grad, m, v, p16, inv_scale, clip, found_inf, step_state, lr, beta1, beta2, eps, wd) -> None:
    """step_state: f32[4] device tensor; [0] is the completed-update count, advanced on
    the device unless *found_inf != 0."""
    _lib.call("jx_adamw_step", p.data_ptr(), grad.data_ptr(), int(grad.dtype == F16), m.data_ptr(), v.data_ptr(),
              _ptr(p16), p.numel(), _ptr(inv_scale), _ptr(clip), _ptr(found_inf), step_state.data_ptr(), float(lr),
              float(beta1), float(beta2), float(eps), float(wd), _stream())


def scaler_update(scale, tracker, found_inf, growth=2.0, backoff=0.5, interval=2000) -> None:
    _lib.call("jx_scaler_update", scale.data_ptr(), tracker.data_ptr(), found_inf.data_ptr(), float(growth),
              float(backoff), int(interval), _stream())


def cast_f32_f16(src: torch.Tensor, dst: torch.Tensor) -> None:
    _lib.call("jx_cast_f32_f16", src.data_ptr(), dst.data_ptr(), src.numel(), _stream())


def transpose_f16(src: torch.Tensor, dst: torch.Tensor | None = None) -> torch.Tensor:
    rows, cols = src.shape
    dst = dst if dst is not None else torch.empty(cols, rows, device=src.device, dtype=F16)
    _lib.call("jx_transpose_f16", src.data_ptr(), dst.data_ptr(), rows, cols, _stream())
    return dst
