"""Worker for tests/test_dp_gpu.py, launched with torch.distributed.run (one rank per GPU).

Each rank computes the decoder's gradients on its own Zipf micro-batch with the
bucketed NCCL reducer averaging them during backward; rank 0 then recomputes
the same update as one process accumulating every rank's micro-batch with
loss / world_size (the data-parallel oracle) and writes the comparison."""
import json
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from midstream_llm_b200 import AdamW, GradScaler, JishuiForCausalLM, causal_lm_loss, train_update  # noqa: E402
from midstream_llm_b200.config import ModelConfig  # noqa: E402
from midstream_llm_b200.data import ZipfBatches  # noqa: E402
from midstream_llm_b200.distributed import (GradReducer, LaunchEnvironment, build_runtime_plan,  # noqa: E402
                                            initialize_runtime)

CFG = ModelConfig(name="dp", vocab_size=4096, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=4, head_dim=64, intermediate_size=688, norm_type="rmsnorm", norm_bias=False,
                  max_position_embeddings=1024, gradient_checkpointing=False)


def model_on(dev):
    torch.manual_seed(0)
    m = JishuiForCausalLM(CFG)
    gen = torch.Generator().manual_seed(0)
    with torch.no_grad():
        for _, p in m.named_parameters():
            p.copy_(torch.randn(p.shape, generator=gen) * 0.02 if p.dim() == 2 else torch.ones(p.shape))
    return m.to(dev)


def batch(rank, dev):
    rows = torch.from_numpy(ZipfBatches(CFG.vocab_size, 2, 256, seed=100 + rank).next_rows()).to(dev)
    return rows[:, :-1].contiguous(), rows[:, 1:].contiguous()


def main():
    env = LaunchEnvironment.from_environ()
    ctx = initialize_runtime(build_runtime_plan("cuda", env), timeout_s=120)
    dev, world, rank = ctx.torch_device, env.world_size, env.rank
    scale = 1024.0
    m = model_on(dev)
    m.grad_reducer = GradReducer(bucket_bytes=1 << 20)
    x, y = batch(rank, dev)
    (causal_lm_loss(m, x, y) * scale).backward()
    torch.cuda.synchronize()
    dp_grads = {n: p.grad.detach().clone() for n, p in m.named_parameters()}
    # one DP optimizer update through the public API, identical on every rank afterwards
    opt = AdamW(m.parameters(), lr=1e-3, betas=(0.9, 0.95), eps=1e-5, weight_decay=0.1)
    scaler = GradScaler("cuda", init_scale=scale)
    r = train_update(m, opt, scaler, lambda: [(x, y)], 1, 1.0, 1e-3)
    # Gradient accumulation over 2 micro-batches: only the last micro-step's backward all-reduces
    # (no_sync rule); the update still leaves identical parameters on every rank.
    per_backward = len(m.grad_reducer.launched)
    before = m.grad_reducer.collectives
    x2, y2 = batch(rank + 50, dev)
    train_update(m, opt, scaler, lambda: [(x, y), (x2, y2)], 2, 1.0, 1e-3)
    accum_collectives = m.grad_reducer.collectives - before
    flat = torch.cat([p.detach().reshape(-1) for p in m.parameters()])
    gathered = [torch.empty_like(flat) for _ in range(world)]
    dist.all_gather(gathered, flat)
    params_agree = all(torch.equal(g, gathered[0]) for g in gathered)
    # The sharded (ZeRO-1-style) update: this rank's shard of the gradients is reduced to it, AdamW runs on
    # the shard, the fp16 weights are all-gathered. Compared against the replicated update from the same
    # start: gradients on the own shard, fp16 weights everywhere, master weights after gather_full_state.
    ms = model_on(dev)
    ms.grad_reducer = GradReducer(bucket_bytes=1 << 20, shard_optimizer=True)
    mr = model_on(dev)
    mr.grad_reducer = GradReducer(bucket_bytes=1 << 20)
    opt_s = AdamW(ms.parameters(), lr=1e-3, betas=(0.9, 0.95), eps=1e-5, weight_decay=0.1)
    opt_r = AdamW(mr.parameters(), lr=1e-3, betas=(0.9, 0.95), eps=1e-5, weight_decay=0.1)
    sc_s, sc_r = GradScaler("cuda", init_scale=scale), GradScaler("cuda", init_scale=scale)
    x3, y3 = batch(rank + 70, dev)
    rs = train_update(ms, opt_s, sc_s, lambda: [(x3, y3)], 1, 1.0, 1e-3)
    rr = train_update(mr, opt_r, sc_r, lambda: [(x3, y3)], 1, 1.0, 1e-3)
    fs, fr = ms.flat(), mr.flat()
    # The norm gains are read by the kernels in fp32: after the sharded update every rank holds the
    # owner's new values (no gather_full_state needed), equal to the replicated update's.
    norm32 = fs.p32.index_select(0, fs.f32_read_index)
    n32 = [torch.empty_like(norm32) for _ in range(world)]
    dist.all_gather(n32, norm32)
    norm_equal_ranks = all(torch.equal(g, n32[0]) for g in n32)
    norm_err = float((norm32 - fr.p32.index_select(0, fr.f32_read_index)).norm() / norm32.norm())
    # A second update from the updated weights: the sharded and replicated losses still agree.
    x4, y4 = batch(rank + 90, dev)
    rs2 = train_update(ms, opt_s, sc_s, lambda: [(x4, y4)], 1, 1.0, 1e-3)
    rr2 = train_update(mr, opt_r, sc_r, lambda: [(x4, y4)], 1, 1.0, 1e-3)
    lo, hi = ms.grad_reducer.shard_range(fs)
    shard_grad_err = float((fs.g32[lo:hi] - fr.g32[lo:hi]).norm() / fr.g32[lo:hi].norm())
    g16 = [torch.empty_like(fs.p16) for _ in range(world)]
    dist.all_gather(g16, fs.p16)
    f16_equal_ranks = all(torch.equal(g, g16[0]) for g in g16)
    f16_err = float((fs.p16.float() - fr.p16.float()).norm() / fr.p16.float().norm())
    ms.grad_reducer.gather_full_state(opt_s)
    p32_err = float((fs.p32 - fr.p32).norm() / fr.p32.norm())
    m_err = float((opt_s._m - opt_r._m).norm() / opt_r._m.norm())
    sharded = {"shard_grad_err": shard_grad_err, "f16_equal_ranks": f16_equal_ranks, "f16_err": f16_err,
               "p32_err": p32_err, "m_err": m_err, "grad_norm": [rs["grad_norm"], rr["grad_norm"]],
               "loss": [rs["loss"], rr["loss"]], "norm_equal_ranks": norm_equal_ranks, "norm_err": norm_err,
               "loss2": [rs2["loss"], rr2["loss"]]}
    if rank == 0:
        ref = model_on(dev)
        for rr in range(world):
            xr, yr = batch(rr, dev)
            (causal_lm_loss(ref, xr, yr) * (scale / world)).backward()
        torch.cuda.synchronize()
        errs = {}
        for n, p in ref.named_parameters():
            a, b = dp_grads[n].double(), p.grad.double()
            errs[n] = float((a - b).norm() / b.norm().clamp_min(1e-30))
        out = {"world": world, "max_rel_err": max(errs.values()), "errs": errs, "params_agree": params_agree,
               "attempts": r["attempts"], "buckets": per_backward, "accum_collectives": accum_collectives,
               "sharded": sharded}
        Path(os.environ["DP_TEST_OUT"]).write_text(json.dumps(out))
    dist.barrier()
    ctx.close()


if __name__ == "__main__":
    main()
