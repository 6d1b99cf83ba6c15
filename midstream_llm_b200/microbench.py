"""Operator microbenchmarks of the bandwidth-bound path and the dense kernels.

    python -m midstream_llm_b200.microbench [--op all|rmsnorm|ce|adamw|gemm|attn] [--iters N]

Shapes (the operator workload of the Jishui-200M step):
  rmsnorm  fwd with residual add and bwd with residual gradient on fp16 [16384, 1024];
           algorithmic bytes 4*M*d*2 = 134,217,728 each way (+ rstd / gamma)
  ce       fused chunked cross-entropy: hidden [16384, 1024] x tied embedding
           [32000, 1024], Zipf(1.1) labels: logits GEMM, CE fwd, CE bwd (in place),
           dH and dE GEMMs = 3 x 2*M*V*d = 3.221 TFLOP; the softmax sub-steps are
           also reported against the 2.097 GB an fp16 logits read + dlogits write costs
  adamw    unscale + non-finite check + global norm + clip + AdamW over 200M fp32
           parameters with fp16 gradients N(0, 1e-3): 28 B/param (5.6 GB); a flagged
           step with 1 % +inf gradients runs the statistics pass only (2 B/param)
  gemm     the decoder's GEMM shapes with their fused epilogues
  attn     causal flash attention fwd / bwd at (B 16, T 1024) and (B 4, T 4096), 16 heads x 64
  eval     validation forward (no autograd, fused head + CE) of the 200M model at 16 x 1024
  decode   next-token logits with the KV cache vs re-running the whole context (200M, context ~1000)
Each line is JSON with the time per call (CUDA events, after warm-up, inputs
larger than L2 unless noted), the achieved rate against the measured peaks and
the SM clock read just before the timed calls (`sm_mhz`). The B200 is power-capped:
after seconds of dense GEMMs the SM clock drops (to ~1240 MHz) and takes a second
or two to recover, so `--op all` pauses between operator groups.
"""
from __future__ import annotations

import argparse
import json
import math
import time
from pathlib import Path

import torch

from . import ops
from .data import ZipfBatches

ROOT = Path(__file__).resolve().parents[1]


def _peaks() -> dict:
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "fallback": True}


_NVML = None


def _sm_mhz() -> int | None:
    """Current SM clock of device 0 (NVML), or None where NVML is unavailable."""
    global _NVML
    try:
        import pynvml
        if _NVML is None:
            pynvml.nvmlInit()
            _NVML = pynvml.nvmlDeviceGetHandleByIndex(torch.cuda.current_device())
        return int(pynvml.nvmlDeviceGetClockInfo(_NVML, pynvml.NVML_CLOCK_SM))
    except Exception:
        return None


_LAST_MHZ = None


def _time(fn, iters: int, warmup: int = 3) -> float:
    global _LAST_MHZ
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    _LAST_MHZ = _sm_mhz()
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters / 1000.0  # seconds per call


def _emit(name: str, seconds: float, work: float, unit: str, peak: float, **extra) -> dict:
    rate = work / seconds / (1e9 if unit == "GB/s" else 1e12)
    line = {"op": name, "us": seconds * 1e6, "achieved": rate, "unit": unit, "peak": peak, "frac": rate / peak,
            "sm_mhz": _LAST_MHZ}
    line.update(extra)
    print(json.dumps(line), flush=True)
    return line


def bench_rmsnorm(iters: int) -> None:
    pk = _peaks()
    M, d = 16384, 1024
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(M, d, device="cuda", generator=g).half()
    r = torch.randn(M, d, device="cuda", generator=g).half()
    gamma = torch.ones(d, device="cuda")
    y, s = torch.empty_like(x), torch.empty_like(x)
    rstd = torch.empty(M, device="cuda")
    t = _time(lambda: ops.rmsnorm_fwd(x, gamma, 1e-5, resid=r, out=y, sum_out=s, rstd=rstd), iters)
    _emit("rmsnorm_fwd_residual [16384,1024]", t, 4 * M * d * 2 + M * 4 + d * 4, "GB/s", pk["hbm_gbs"])
    t = _time(lambda: ops.rmsnorm_fwd(x, gamma, 1e-5, out=y, rstd=rstd), iters)  # the training step's form
    _emit("rmsnorm_fwd [16384,1024]", t, 2 * M * d * 2 + M * 4 + d * 4, "GB/s", pk["hbm_gbs"])
    dy = torch.randn(M, d, device="cuda", generator=g).half()
    dres = torch.randn(M, d, device="cuda", generator=g).half()
    dx = torch.empty_like(x)
    dgamma = torch.zeros(d, device="cuda")
    part = torch.empty(ops._lib.query("jx_rmsnorm_bwd_parts", M) * d, device="cuda")
    t = _time(lambda: ops.rmsnorm_bwd(dy, s, rstd, gamma, dresid=dres, out=dx, dgamma=dgamma, part=part), iters)
    _emit("rmsnorm_bwd_residual [16384,1024] (incl. dgamma reduce)", t, 4 * M * d * 2 + M * 4 + d * 4, "GB/s",
          pk["hbm_gbs"])


def bench_ce(iters: int) -> None:
    pk = _peaks()
    M, d, V = 16384, 1024, 32000
    g = torch.Generator(device="cuda").manual_seed(1)
    h = (torch.randn(M, d, device="cuda", generator=g) * 0.5).half()
    E = (torch.randn(V, d, device="cuda", generator=g) * 0.02).half()
    tg = torch.from_numpy(ZipfBatches(V, 16, 1023, seed=2).next_rows().reshape(-1)[:M].copy()).cuda()
    logits = torch.empty(M, V, device="cuda", dtype=torch.float16)
    lse = torch.empty(M, device="cuda")
    row_loss = torch.empty(M, device="cuda")
    lsc = torch.zeros(3, device="cuda")
    dh = torch.empty(M, d, device="cuda", dtype=torch.float16)
    dE = torch.zeros(V, d, device="cuda")
    grad = torch.tensor([65536.0 / 4], device="cuda")

    parts = torch.empty(M, ops.ce_parts_blocks(V), 2, device="cuda")

    def step():  # the model's path: head GEMM with the CE statistics in its epilogue
        ops.gemm_f16_ce_parts(h, E, out=logits, parts=parts)
        ops.ce_fwd_parts(parts, logits, tg, lse=lse, row_loss=row_loss)
        ops.ce_loss(row_loss, tg, out=lsc)
        ops.ce_bwd(logits, tg, lse, grad, lsc[1:2])
        ops.gemm_f16(logits, E, b_mn_major=True, out=dh)
        ops.gemm_wgrad(logits, h, dE, False, 1)

    t = _time(step, iters)
    _emit("fused_ce fwd+bwd h[16384,1024] x E[32000,1024]", t, 3 * 2.0 * M * V * d, "TFLOP/s",
          pk.get("bf16_tflops_sustained", pk["bf16_tflops"]), flops=3 * 2.0 * M * V * d)
    # The bandwidth-bound softmax sub-steps: the statistics merge (parts + target logits) and the backward
    # read / write of the fp16 logits; the unfused form reads the logits once more in the forward.
    t_fwd = _time(lambda: ops.ce_fwd_parts(parts, logits, tg, lse=lse, row_loss=row_loss), iters)
    t_bwd = _time(lambda: ops.ce_bwd(logits, tg, lse, grad, lsc[1:2]), iters)
    t_unf = _time(lambda: ops.ce_fwd(logits, tg, lse=lse, row_loss=row_loss), iters)
    moved = parts.numel() * 4 + 2 * M * V * 2
    _emit("ce_softmax_substeps (statistics merge + bwd read/write of fp16 logits)", t_fwd + t_bwd, moved, "GB/s",
          pk["hbm_gbs"], fwd_us=t_fwd * 1e6, bwd_us=t_bwd * 1e6, unfused_fwd_us=t_unf * 1e6,
          unfused_bytes=3 * M * V * 2)


def bench_adamw(iters: int) -> None:
    pk = _peaks()
    n = 200_000_000
    g = torch.Generator(device="cuda").manual_seed(3)
    p = torch.randn(n, device="cuda", generator=g) * 0.02
    grad = (torch.randn(n, device="cuda", generator=g) * 1e-3).half()
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    p16 = None
    inv = torch.tensor([1.0 / 1024], device="cuda")
    parts = ops.grad_stats_parts(n)
    partial = torch.empty(parts, device="cuda")
    found = torch.zeros(1, device="cuda")
    fin = torch.empty(2, device="cuda")
    state = torch.zeros(4, device="cuda")

    def step():
        found.zero_()
        ops.grad_stats(grad, inv, partial, found)
        ops.grad_finalize(partial, parts, 1.0, fin)
        ops.adamw_step(p, grad, m, v, p16, inv, fin[1:2], found, state, 3e-4, 0.9, 0.95, 1e-5, 0.1)

    t = _time(step, iters)
    _emit("unscale+norm+clip+adamw 200M fp32 params, fp16 grads", t, 28.0 * n, "GB/s", pk["hbm_gbs"],
          bytes_per_param=28)
    idx = torch.randperm(n, device="cuda", generator=g)[: n // 100]
    grad_inf = grad.clone()
    grad_inf[idx] = float("inf")
    p0 = p.clone()

    def flagged():
        found.zero_()
        ops.grad_stats(grad_inf, inv, partial, found)
        ops.grad_finalize(partial, parts, 1.0, fin)
        ops.adamw_step(p, grad_inf, m, v, p16, inv, fin[1:2], found, state, 3e-4, 0.9, 0.95, 1e-5, 0.1)

    t = _time(flagged, iters)
    torch.cuda.synchronize()
    skipped = bool(torch.equal(p, p0)) and float(found) == 1.0
    _emit("flagged step (1% +inf): stats pass only, update skipped on the device", t, 2.0 * n, "GB/s",
          pk["hbm_gbs"], bytes_per_param=2, update_skipped=skipped)


def gemm_cases():
    """Every GEMM call of one micro-batch of the 200M step (16 x 1024 tokens), issued as the model issues it
    (same entry points, operand majors, epilogues and split-K counts). Each case: (name, launches per
    micro-batch, FLOPs, algorithmic bytes -- operands read once, outputs written once, an accumulated fp32
    gradient read and written --, the call)."""
    from .model import _wgrad_splits, rope_tables
    M, d, F, V = 16384, 1024, 2816, 32000
    hh = lambda *s: (torch.randn(*s, device="cuda") * 0.5).half()  # noqa: E731
    x, wqkv, wo, wgu, wd, E = hh(M, d), hh(3 * d, d), hh(d, d), hh(2 * F, d), hh(d, F), hh(V, d)
    cos, sin = rope_tables(1024, 64, 10000.0, "cuda")
    qkv = torch.empty(M, 3 * d, device="cuda", dtype=torch.half)
    gt, up, act = (torch.empty(M, F, device="cuda", dtype=torch.half) for _ in range(3))
    out = torch.empty(M, d, device="cuda", dtype=torch.half)
    out2 = torch.empty(M, d, device="cuda", dtype=torch.half)
    dgu = torch.empty(M, 2 * F, device="cuda", dtype=torch.half)
    dq = hh(M, 3 * d)
    logits = torch.empty(M, V, device="cuda", dtype=torch.half)
    parts = torch.empty(M, ops.ce_parts_blocks(V), 2, device="cuda")
    gqkv, go, ggu, gd = (torch.zeros(n, k, device="cuda") for n, k in ((3 * d, d), (d, d), (2 * F, d), (d, F)))
    GV = torch.zeros(V, d, device="cuda")
    ws = torch.empty(64 << 20, device="cuda")
    sp = lambda n, k: _wgrad_splits(n, k, M)  # noqa: E731
    b16 = lambda *n: 2.0 * sum(n)  # noqa: E731
    wg = lambda n, k: 2.0 * M * (n + k) + 8.0 * n * k  # noqa: E731  (accumulated fp32 gradient: read + write)
    return [
        ("qkv+rope [16384x3072x1024]", 16, 2 * M * 3 * d * d, b16(M * d, 3 * d * d, M * 3 * d),
         lambda: ops.gemm_qkv_rope(x, wqkv, d, cos, sin, 1024, 64, out=qkv)),
        ("o_proj+residual [16384x1024x1024]", 16, 2 * M * d * d, b16(M * d, d * d, 2 * M * d),
         lambda: ops.gemm_f16(x, wo, resid=x, out=out)),
        ("gate|up+swiglu [16384x5632x1024]", 16, 2 * M * 2 * F * d, b16(M * d, 2 * F * d, 3 * M * F),
         lambda: ops.gemm_swiglu_fwd(x, wgu, F, gate=gt, up=up, act=act)),
        ("down+residual [16384x1024x2816]", 16, 2 * M * d * F, b16(M * F, d * F, 2 * M * d),
         lambda: ops.gemm_f16(act, wd, resid=x, out=out)),
        ("tied head + CE statistics [16384x32000x1024]", 1, 2 * M * V * d, b16(M * d, V * d, M * V),
         lambda: ops.gemm_f16_ce_parts(x, E, out=logits, parts=parts)),
        ("down dgrad+swiglu bwd [16384x2816x1024]", 16, 2 * M * F * d, b16(M * d, F * d, 4 * M * F),
         lambda: ops.gemm_swiglu_bwd(x, wd, gt, up, out=dgu)),
        (f"down wgrad [1024x2816, 16384 tokens, {sp(d, F)} splits]", 16, 2 * M * d * F, wg(d, F),
         lambda: ops.gemm_wgrad(out, act, gd, True, sp(d, F), ws)),
        ("gate|up dgrad [16384x1024x5632]", 16, 2 * M * 2 * F * d, b16(M * 2 * F, 2 * F * d, M * d),
         lambda: ops.gemm_f16(dgu, wgu, b_mn_major=True, out=out)),
        (f"gate|up wgrad [5632x1024, 16384 tokens, {sp(2 * F, d)} splits]", 16, 2 * M * 2 * F * d, wg(2 * F, d),
         lambda: ops.gemm_wgrad(dgu, x, ggu, True, sp(2 * F, d), ws)),
        ("o dgrad [16384x1024x1024]", 16, 2 * M * d * d, b16(M * d, d * d, M * d),
         lambda: ops.gemm_f16(out, wo, b_mn_major=True, out=out2)),
        (f"o wgrad [1024x1024, 16384 tokens, {sp(d, d)} splits]", 16, 2 * M * d * d, wg(d, d),
         lambda: ops.gemm_wgrad(out, x, go, True, sp(d, d), ws)),
        ("qkv dgrad [16384x1024x3072]", 16, 2 * M * 3 * d * d, b16(M * 3 * d, 3 * d * d, M * d),
         lambda: ops.gemm_f16(dq, wqkv, b_mn_major=True, out=out)),
        (f"qkv wgrad [3072x1024, 16384 tokens, {sp(3 * d, d)} splits]", 16, 2 * M * 3 * d * d, wg(3 * d, d),
         lambda: ops.gemm_wgrad(dq, x, gqkv, True, sp(3 * d, d), ws)),
        ("head dgrad [16384x1024x32000]", 1, 2 * M * V * d, b16(M * V, V * d, M * d),
         lambda: ops.gemm_f16(logits, E, b_mn_major=True, out=out)),
        ("head wgrad [32000x1024, 16384 tokens]", 1, 2 * M * V * d, wg(V, d),
         lambda: ops.gemm_wgrad(logits, x, GV, True, 1, ws)),
    ]


def bench_gemm(iters: int) -> None:
    """The step's GEMM calls one after another (3 warm-up + `iters` timed launches each)."""
    pk = _peaks()
    peak = pk.get("bf16_tflops", 1590.0)
    for name, per_mb, fl, nbytes, fn in gemm_cases():
        _emit("gemm " + name, _time(fn, iters), fl, "TFLOP/s", peak, peak_kind="bf16_tflops (burst)",
              launches_per_microbatch=per_mb, algorithmic_bytes=nbytes)


def bench_attn(iters: int) -> None:
    pk = _peaks()
    for B, T in ((16, 1024), (4, 4096)):
        H, D = 16, 64
        qkv = (torch.randn(B * T, 3 * H * D, device="cuda") * 0.5).half()
        o, lse = ops.attn_fwd(qkv, B, T, H, D)
        do = torch.randn_like(o)
        ws = torch.empty(ops.attn_bwd_workspace_bytes(B, T, H, D) // 4 + 4, device="cuda")
        wsf = torch.empty(ops.attn_fwd_workspace_bytes(B, T, H, D) // 4 + 4, device="cuda")
        dqkv = torch.empty_like(qkv)
        fl = 2.0 * B * H * T * T * D  # causal forward: two T x T x D products, half of them
        _emit(f"attn_fwd causal B{B} T{T} H16 D64", _time(lambda: ops.attn_fwd(qkv, B, T, H, D, out=o, lse=lse,
                                                                             workspace=wsf), iters),
              fl, "TFLOP/s", pk.get("bf16_tflops", 1590.0))
        _emit(f"attn_bwd causal B{B} T{T} H16 D64", _time(lambda: ops.attn_bwd(qkv, o, do, lse, B, T, H, D, out=dqkv,
                                                                              workspace=ws), iters),
              2.5 * fl, "TFLOP/s", pk.get("bf16_tflops", 1590.0))
        _bench_sdpa(qkv, do, B, T, H, D, fl, iters, pk.get("bf16_tflops", 1590.0))


def _bench_sdpa(qkv, do, B, T, H, D, fl, iters, peak) -> None:
    """torch's F.scaled_dot_product_attention at the same shapes (what the reference calls,
    model_torch.py:48), with contiguous [B, H, T, D] fp16 operands, for every backend torch offers here."""
    from torch.nn.attention import SDPBackend, sdpa_kernel
    from torch.nn.functional import scaled_dot_product_attention as sdpa
    q, k, v = (qkv.view(B, T, 3, H, D)[:, :, i].transpose(1, 2).contiguous().requires_grad_(True) for i in range(3))
    dout = do.view(B, T, H, D).transpose(1, 2).contiguous()
    for name, backend in (("default", None), ("flash", SDPBackend.FLASH_ATTENTION),
                          ("cudnn", SDPBackend.CUDNN_ATTENTION), ("efficient", SDPBackend.EFFICIENT_ATTENTION)):
        try:
            ctx = sdpa_kernel(backend) if backend is not None else torch.enable_grad()
            with ctx:
                out = sdpa(q, k, v, is_causal=True)
                tf = _time(lambda: sdpa(q, k, v, is_causal=True), iters)
                tb = _time(lambda: torch.autograd.grad(out, (q, k, v), dout, retain_graph=True), iters)
        except Exception as exc:  # a backend that does not support this shape or GPU
            print(json.dumps({"op": f"torch sdpa[{name}] B{B} T{T}", "unavailable": str(exc).splitlines()[0][:160]}),
                  flush=True)
            continue
        _emit(f"torch sdpa[{name}] fwd causal B{B} T{T} H16 D64", tf, fl, "TFLOP/s", peak)
        _emit(f"torch sdpa[{name}] bwd causal B{B} T{T} H16 D64", tb, 2.5 * fl, "TFLOP/s", peak)


def bench_eval(iters: int) -> None:
    """Validation forward (pretrain_torch.py:42-58): no autograd, fused head + CE, 200M model, 16 x 1024."""
    from .config import jishui_200m
    from .data import ZipfBatches
    from .model import JishuiForCausalLM
    pk = _peaks()
    cfg = jishui_200m(1024)
    torch.manual_seed(0)
    model = JishuiForCausalLM(cfg).cuda()
    with torch.no_grad():
        for p in model.parameters():
            if p.dim() == 2:
                p.normal_(0.0, 0.02)
    rows = torch.from_numpy(ZipfBatches(cfg.vocab_size, 16, 1024, seed=7).next_rows()).cuda()
    x, y = rows[:, :-1].contiguous(), rows[:, 1:].contiguous()
    d, F, V, L = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.num_hidden_layers
    fwd_flops = 2.0 * 16 * 1024 * (L * (4 * d * d + 3 * d * F) + V * d) + 2.0 * L * 16 * 16 * 1024 * 1024 * 64
    with torch.no_grad():
        t = _time(lambda: model.loss(x, y), iters)
    _emit("eval forward+CE 200M B16 T1024 (tokens/s: %.0f)" % (16 * 1024 / t), t, fwd_flops, "TFLOP/s",
          pk.get("bf16_tflops", 1590.0))


def bench_decode(iters: int) -> None:
    """Next-token logits at context 1024 of the 200M model: one KV-cache step against re-running the whole
    context (what generate_torch.next_token_logits does, here through this library's forward)."""
    from .config import jishui_200m
    from .decode import KVCacheDecoder
    from .model import JishuiForCausalLM
    cfg = jishui_200m(1024)
    torch.manual_seed(0)
    model = JishuiForCausalLM(cfg).cuda()
    with torch.no_grad():
        for p in model.parameters():
            if p.dim() == 2:
                p.normal_(0.0, 0.02)
    ctx = torch.randint(3, cfg.vocab_size, (1024,)).tolist()
    dec = KVCacheDecoder(model)
    dec.next_token_logits(ctx[:1000])
    state = {"n": 1000}

    def step():
        if state["n"] >= 1024:
            dec.next_token_logits(ctx[:1000])
            state["n"] = 1000
        state["n"] += 1
        dec.next_token_logits(ctx[:state["n"]])

    t = _time(step, iters)
    print(json.dumps({"op": "decode step (KV cache) 200M, context ~1000", "us": t * 1e6,
                      "tokens_per_s": 1.0 / t}), flush=True)
    full = torch.tensor([ctx], device="cuda")
    with torch.no_grad():
        tf = _time(lambda: model(full)[0, -1].float().cpu(), max(2, iters // 4))
    print(json.dumps({"op": "full-context recompute per token 200M, context 1024", "us": tf * 1e6,
                      "tokens_per_s": 1.0 / tf}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--op", default="all", choices=("all", "rmsnorm", "ce", "adamw", "gemm", "attn", "eval", "decode"))
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args()
    torch.cuda.set_device(0)
    for name, fn in (("rmsnorm", bench_rmsnorm), ("ce", bench_ce), ("adamw", bench_adamw), ("gemm", bench_gemm),
                     ("attn", bench_attn), ("eval", bench_eval),
                     ("decode", bench_decode)):
        if a.op in ("all", name):
            if a.op == "all":
                torch.cuda.synchronize()
                time.sleep(3.0)  # let the SM clock recover from the previous group under the power cap
            fn(a.iters)
            torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
