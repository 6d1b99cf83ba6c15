"""Training-throughput benchmark of the Jishui decoder step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--workload 200m|long|base]

One step = one optimizer update. Workloads (token ids Zipf(1.1) from a seed,
weights N(0, 0.02)):
  200m  Jishui-200M (V 32000, d 1024, 16 layers, 16 heads x 64, SwiGLU 2816,
        RMSNorm, tied), seq 1024, micro-batch 16; grad-accum 4 on 1 GPU,
        grad-accum 1 per GPU when N > 1 (data parallel, 25 MB NCCL buckets
        overlapped with backward; weak scaling).
  long  the same model at seq 4096, micro-batch 4, every layer recomputed in
        backward (gradient checkpointing), grad-accum 1.
Rank 0 prints one JSON line:
  value      K updates with the batches already in HBM (CUDA events, barrier +
             synchronize around, max over ranks); nothing but the reducer's two
             overlap events per update is recorded inside that region;
  e2e        K more through the same public API with each update's tokens copied
             from pinned host memory and the loss read back;
  roofline   a third pass of K updates with CUDA events around every GEMM launch
             (the dominant kernel family), so that instrumentation stays out of
             `value`;
  per_gpu_accum1 (1 GPU, workload 200m) K updates of one micro-batch each, the
             data-parallel runs' per-GPU configuration;
  exposed_comm_ms_per_step (N > 1) the part of the gradient all-reduce the
             backward did not hide;
  gpu_reference (1 GPU) the reference recipe in eager PyTorch on the same GPU;
  cpu_baseline (1 GPU) the reference update on the host cores.
`--impl reference` times the reference's update step (the oracle restatement
of Midstream-LLM's model_torch + pretrain_torch update, fp32, no autocast) on
the host CPU cores on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

MEASURED = ROOT / "MEASURED_PEAKS.json"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks() -> tuple[dict, str]:
    try:
        return json.loads(MEASURED.read_text()), "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


def workload(name: str, n_gpus: int) -> dict:
    if name == "200m":
        return dict(name="jishui-200m-seq1024", seq=1024, micro=16, accum=4 if n_gpus == 1 else 1, ckpt=False)
    if name == "long":
        return dict(name="jishui-200m-seq4096-recompute", seq=4096, micro=4, accum=1, ckpt=True)
    if name == "base":
        # The reference's production run (configs/jishui-200m-cuda-4b.json): 16,384 tokens per update
        # (batch 1 x accum 8 there; one micro-batch of 8 x 2048 here, the same update).
        return dict(name="jishui-200m-base-layernorm-seq2048", seq=2048, micro=8, accum=1, ckpt=False, cfg="base")
    raise SystemExit(f"unknown workload {name}")


def workload_config(wl: dict):
    from midstream_llm_b200.config import jishui_200m, jishui_200m_base
    if wl.get("cfg") == "base":
        return jishui_200m_base(wl["ckpt"])
    return jishui_200m(wl["seq"], gradient_checkpointing=wl["ckpt"])


def model_flops_per_token(cfg, seq: int) -> tuple[float, float]:
    """(6*N_mm + 6*L*T*d, PaLM 6*N_mm + 12*L*T*d): GEMM weights incl. the tied head; no recompute."""
    d, F, V, L = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size, cfg.num_hidden_layers
    n_mm = L * (4 * d * d + 3 * d * F) + V * d
    return 6.0 * n_mm + 6.0 * L * seq * d, 6.0 * n_mm + 12.0 * L * seq * d


def init_weights(model, seed: int) -> None:
    """N(0, 0.02) for every 2-D parameter in named_parameters() order, gains 1."""
    gen = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if p.dim() == 2:
                p.copy_(torch.randn(p.shape, generator=gen) * 0.02)
            else:
                p.fill_(0.0 if name.endswith(".bias") else 1.0)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, device_index: int):
        self.path = Path(tempfile.mkstemp(prefix="clocks_", suffix=".csv")[1])
        self.proc = None
        self.device_index = device_index

    def start(self):
        try:
            uuid = str(torch.cuda.get_device_properties(self.device_index).uuid)
            sel = ["-i", uuid if uuid.startswith("GPU-") else "GPU-" + uuid]
        except Exception:
            sel = ["-i", str(self.device_index)]
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", *sel], stdout=self.path.open("w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons, power = [], [], set(), []
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(self.NAMES, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        loaded = [s for s in sm if s > 0.5 * max(sm)] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


def cpu_reference_rate(steps: int, warmup: int, seq: int, cfg, seed: int = 0) -> dict:
    """The reference update (oracle restatement, fp32, no autocast) on the host cores:
    the workload's model at micro-batch 1 x seq, tokens/s over `steps` updates."""
    from oracle import jishui_ref as oracle
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    from dataclasses import replace
    cfg = replace(cfg, gradient_checkpointing=False)
    torch.manual_seed(seed)
    model = oracle.JishuiRef(cfg)
    oracle.init_weights(model, seed)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), eps=1e-5, weight_decay=0.1)
    rows = oracle.zipf_tokens(cfg.vocab_size, 1, seq, seed)
    batch = [(rows[:, :-1], rows[:, 1:])]
    for _ in range(warmup):
        oracle.reference_update(model, opt, None, lambda: batch, 1, 1.0, 3e-4, device_type="cpu")
    t0 = time.perf_counter()
    for _ in range(steps):
        oracle.reference_update(model, opt, None, lambda: batch, 1, 1.0, 3e-4, device_type="cpu")
    dt = time.perf_counter() - t0
    return {"value": steps * seq / dt, "unit": "tokens/s", "cores": threads, "kind": "port",
            "sample": f"{steps} fp32 updates of {cfg.name} at micro-batch 1x{seq} on {threads} host threads "
                      f"(oracle restatement of model_torch + pretrain_torch update, no autocast)"}


def recompute_flops_per_token(cfg, seq: int) -> float:
    """Forward FLOPs per token that gradient checkpointing runs a second time (every layer, not the head)."""
    d, F, L = cfg.hidden_size, cfg.intermediate_size, cfg.num_hidden_layers
    return 2.0 * L * (4 * d * d + 3 * d * F) + 2.0 * L * seq * d


def gpu_reference_rate(cfg, B: int, T: int, accum: int, batches: list, dev) -> dict:
    """The reference recipe on the same GPU: the oracle's restatement of the reference modules run the way
    pretrain_torch.py:204-235 runs them (fp16 autocast, torch.amp.GradScaler(65536), torch.optim.AdamW(
    fused=True), TF32 off, grad clip 1.0), on the workload's micro-batches; tokens/s over 3 timed updates
    after 2 warm-up updates (CUDA events; the loop's own host reads included, as in the reference)."""
    from oracle import jishui_ref as oracle
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    ref = oracle.JishuiRef(cfg)
    oracle.init_weights(ref, 0)
    ref = ref.to(dev)
    opt = torch.optim.AdamW(ref.parameters(), lr=3e-4, betas=(0.9, 0.95), eps=1e-5, weight_decay=0.1, fused=True)
    scaler = torch.amp.GradScaler("cuda", init_scale=65536.0)

    def upd(b):
        return oracle.reference_update(ref, opt, scaler, lambda: b, accum, 1.0, 3e-4)

    for b in batches[:2]:
        upd(b)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for b in batches[2:]:
        upd(b)
    e.record()
    torch.cuda.synchronize()
    n = len(batches) - 2
    ms = s.elapsed_time(e) / n
    rate = B * T * accum / (ms / 1000.0)
    del ref, opt, scaler
    torch.cuda.empty_cache()
    return {"value": rate, "unit": "tokens/s", "ms_per_step": ms, "steps": n,
            "recipe": "reference modules (oracle restatement) in eager PyTorch: fp16 autocast, cuBLAS GEMMs, "
                      "F.scaled_dot_product_attention, GradScaler, AdamW(fused=True), TF32 off",
            "gradient_checkpointing": bool(cfg.gradient_checkpointing)}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    wl = workload(args.workload, args.gpus)
    cfg = workload_config(wl)
    steps = max(1, min(args.steps, 3))
    base = cpu_reference_rate(steps, min(args.warmup, 1), wl["seq"], cfg)
    f_model, _ = model_flops_per_token(cfg, wl["seq"])
    line = {"metric": "train tokens/s", "value": base["value"], "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": steps, "warmup": min(args.warmup, 1), "ms_per_step": 1000.0 * wl["seq"] / base["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": wl["name"] + " (reference CPU sample: micro-batch 1)", "model": cfg.name,
                       "seq_len": wl["seq"], "global_batch": wl["micro"] * wl["accum"] * args.gpus,
                       "parallelism": f"dp{args.gpus}"},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "mfu_model_flops": base["value"] * f_model}
    emit(line)


_RESULT_FD: int | None = None


def _keep_stdout_for_result() -> None:
    """The driver reads one JSON line from stdout: anything else that writes to file descriptor 1 (NCCL's
    version banner, library warnings) is sent to stderr, and the result goes to the original stdout."""
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)


def emit(line: dict) -> None:
    out = json.dumps(line) + "\n"
    if _RESULT_FD is None:
        sys.stdout.write(out)
        sys.stdout.flush()
    else:
        os.write(_RESULT_FD, out.encode())


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=8)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--workload", choices=("200m", "long", "base"), default="200m")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--sm-reserve", type=int, default=int(os.environ.get("JX_SM_RESERVE", "0")),
                    help="SMs the persistent kernels leave to NCCL while gradient buckets are in flight (N > 1)")
    ap.add_argument("--shard-optimizer", type=int, default=int(os.environ.get("JX_SHARD_OPTIMIZER", "1")),
                    help="N > 1: reduce each gradient bucket to its owning rank, update 1/N of the parameters "
                         "per rank and all-gather the fp16 weights (1) instead of all-reducing (0)")
    ap.add_argument("--no-gpu-reference", action="store_true",
                    help="skip timing the reference recipe (eager torch modules) on the same GPU")
    args = ap.parse_args()
    _keep_stdout_for_result()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
        return

    import torch.distributed as dist
    from midstream_llm_b200 import AdamW, GradScaler, JishuiForCausalLM, _lib, ops, train_update
    from midstream_llm_b200.data import ZipfBatches
    from midstream_llm_b200.distributed import GradReducer, LaunchEnvironment, build_runtime_plan, initialize_runtime

    env = LaunchEnvironment.from_environ()
    if env.world_size != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={env.world_size}; launch N>1 with torch.distributed.run")
    ctx = initialize_runtime(build_runtime_plan("cuda", env), timeout_s=600)
    dev = ctx.torch_device
    rank, world = env.rank, env.world_size
    wl = workload(args.workload, world)
    B, T, accum = wl["micro"], wl["seq"], wl["accum"]
    cfg = workload_config(wl)

    model = JishuiForCausalLM(cfg)
    init_weights(model, seed=0)  # identical on every rank
    model.to(dev)
    opt = AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), eps=1e-5, weight_decay=0.1, fused=True)
    scaler = GradScaler("cuda", init_scale=65536.0)
    if world > 1:
        model.grad_reducer = GradReducer(bucket_bytes=25 * 1024 * 1024, sm_reserve=args.sm_reserve,
                                         shard_optimizer=bool(args.shard_optimizer))

    stream = ZipfBatches(cfg.vocab_size, B, T, seed=1000 + rank)
    n_host = (args.warmup + args.steps) * accum
    host_rows = [torch.from_numpy(stream.next_rows()).pin_memory() for _ in range(n_host)]
    dev_rows = [r.to(dev) for r in host_rows]

    def device_batches(step):
        rows = dev_rows[(step * accum) % len(dev_rows):][:accum]
        return [(r[:, :-1], r[:, 1:]) for r in rows]

    def host_batches(step):
        out = []
        for r in host_rows[(step * accum) % len(host_rows):][:accum]:
            t = r.to(dev, non_blocking=True)
            out.append((t[:, :-1], t[:, 1:]))
        return out

    def one_update(batches):
        return train_update(model, opt, scaler, lambda: batches, accum, 1.0, 3e-4)

    for s in range(args.warmup):
        one_update(device_batches(s))
    torch.cuda.synchronize()

    def timed(get_batches, collect_gemm: bool = False, n_steps: int | None = None, update=None):
        n_steps = args.steps if n_steps is None else n_steps
        update = update or one_update
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        prof = [] if collect_gemm else None
        ops.set_gemm_profile(prof)
        launches0 = _lib.launch_count()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        results = []
        for s in range(n_steps):
            results.append(update(get_batches(args.warmup + s)))
        end.record()
        torch.cuda.synchronize()
        ops.set_gemm_profile(None)
        launches = _lib.launch_count() - launches0
        ms = start.elapsed_time(end)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t)
            dist.barrier()
        return ms, results, launches, prof

    # 1. The headline value: K updates, batches resident in HBM, no instrumentation inside the timed region
    #    beyond the communication-overlap events of the data-parallel reducer (two per update).
    reducer = model.grad_reducer
    if reducer is not None:
        reducer.exposed_events = []
    clocks = ClockSampler(dev.index or 0) if rank == 0 else None
    if clocks:
        clocks.start()
    ms, results, launches, _ = timed(device_batches)
    clock_info = clocks.stop() if clocks else None
    exposed_ms = None
    if reducer is not None:
        ev = reducer.exposed_events
        reducer.exposed_events = None
        t = torch.tensor([sum(a.elapsed_time(b) for a, b in ev) / max(args.steps, 1)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        exposed_ms = float(t)
    # 2. The same updates end to end through the public API: tokens copied from pinned host memory every
    #    update, the loss read back.
    e2e_ms = None
    if not args.no_e2e:
        e2e_ms, _, _, _ = timed(host_batches)
    # 3. A separate, untimed-for-value pass with every GEMM launch bracketed by CUDA events (the roofline of
    #    the dominant kernel family).
    _, _, _, prof = timed(device_batches, collect_gemm=True)
    # 4. One GPU: the per-GPU rate at grad-accum 1 (the data-parallel runs' per-GPU configuration).
    accum1_ms = None
    if world == 1 and accum > 1:
        def one_micro(batches):
            return train_update(model, opt, scaler, lambda: batches[:1], 1, 1.0, 3e-4)
        accum1_ms, _, _, _ = timed(device_batches, update=one_micro)

    tokens_per_step = B * T * accum * world
    value = tokens_per_step * args.steps / (ms / 1000.0)
    pk, pk_kind = peaks()
    f_model, f_palm = model_flops_per_token(cfg, T)
    line = None
    gpu_ref = None
    if world == 1 and not args.no_gpu_reference:
        gpu_ref = gpu_reference_rate(cfg, B, T, accum, [device_batches(s) for s in range(2 + 3)], dev)
    if rank == 0:
        gemm_flops = sum(p[0] for p in prof)
        gemm_ms = sum(p[2].elapsed_time(p[3]) for p in prof)
        gemm_bytes = sum(p[1] for p in prof) / max(len(prof), 1)
        gemm_tflops = gemm_flops / (gemm_ms / 1000.0) / 1e12 if gemm_ms > 0 else None
        peak = pk["bf16_tflops_sustained"] if "bf16_tflops_sustained" in pk else pk["bf16_tflops"]
        traffic = None
        tfile = ROOT / "profiles" / "gemm_traffic.json"
        if tfile.exists():
            traffic = json.loads(tfile.read_text()).get("bytes_per_launch")
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            cpu = cpu_reference_rate(2, 1, T, cfg)
        line = {
            "metric": "train tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic (Zipf 1.1 tokens, N(0,0.02) weights)",
            "config": {"workload": wl["name"], "model": cfg.name, "global_batch": B * accum * world, "micro_batch": B,
                       "grad_accum": accum, "seq_len": T,
                       "parallelism": f"dp{world}" + (" (25 MB buckets reduced to their owning rank, sharded AdamW, "
                                                      "fp16 weights all-gathered)" if world > 1 and args.shard_optimizer
                                                      else ""),
                       "gradient_checkpointing": bool(wl["ckpt"]),
                       "l2": f"working set (activations, {4 * sum(p.numel() for p in model.parameters()) / 1e6:.0f} MB "
                             "fp32 grads) far exceeds the 126 MB L2"},
            "mfu": value * f_model / (world * pk["bf16_tflops"] * 1e12),
            "mfu_palm": value * f_palm / (world * pk["bf16_tflops"] * 1e12),
            "peak_kind": pk_kind,
            "roofline": {"kernel": "gemm_kernel (tcgen05, all GEMM launches of one pass of K updates)",
                         "bound": "tensor", "achieved": gemm_tflops, "peak": peak, "unit": "TFLOP/s",
                         "frac": (gemm_tflops / peak) if gemm_tflops else None, "traffic": traffic,
                         "launches": len(prof), "share_of_step": gemm_ms / ms if ms > 0 else None,
                         "algorithmic_bytes_per_launch": gemm_bytes,
                         "peak_note": f"bf16_tflops_sustained ({pk_kind}); timed in a separate pass with events "
                                      "around every GEMM launch"},
            "gpu_launches": launches,
            "sm_reserve": args.sm_reserve if world > 1 else 0,
            "sharded_update": bool(args.shard_optimizer) and world > 1,
            "clocks": clock_info,
            "loss_last": results[-1]["loss"],
        }
        if wl["ckpt"]:
            line["hfu"] = value * (f_model + recompute_flops_per_token(cfg, T)) / (world * pk["bf16_tflops"] * 1e12)
        if exposed_ms is not None:
            line["exposed_comm_ms_per_step"] = exposed_ms
        if accum1_ms is not None:
            line["per_gpu_accum1"] = {"value": B * T * args.steps / (accum1_ms / 1000.0), "unit": "tokens/s",
                                      "ms_per_step": accum1_ms / args.steps,
                                      "note": "the same micro-batch with grad-accum 1 (the data-parallel per-GPU "
                                              "configuration): optimizer every micro-batch"}
        if e2e_ms is not None:
            line["e2e"] = {"value": tokens_per_step * args.steps / (e2e_ms / 1000.0), "unit": "tokens/s",
                           "h2d_bytes_per_step": B * (T + 1) * 8 * accum, "d2h_bytes_per_step": 3 * 4}
        if gpu_ref is not None:
            line["gpu_reference"] = gpu_ref
        if cpu is not None:
            line["cpu_baseline"] = cpu
        emit(line)
    ctx.close()


if __name__ == "__main__":
    main()
