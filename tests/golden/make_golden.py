"""Generates the golden fixtures that pin the oracle to the reference.

Run where the reference project is available; MIDSTREAM_REF must name its
`src` directory (the one holding the `jishui` package). The tests only read the fixtures it writes.

    MIDSTREAM_REF=<reference checkout>/src python tests/golden/make_golden.py

Writes tests/golden/reference_golden.json with:
  * the tiny debug config's 10-step fp32 AdamW run from the reference package
    (losses, grad norms, per-parameter sums of the final weights) on seeded
    N(0, 0.02) weights and Zipf(1.1) tokens, and the same run through
    oracle/jishui_ref.py, which must agree bit for bit;
  * the 200M architecture's parameter names/shapes and count;
  * RoPE and causal-attention known answers;
  * the learning rates of the 200-step cosine-warm-restart schedule.
"""
from __future__ import annotations

import json
import os
import sys
from dataclasses import replace
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
REF = os.environ.get("MIDSTREAM_REF")
if not REF:
    raise SystemExit("set MIDSTREAM_REF to the reference project's src directory (it holds the jishui package)")
sys.path.insert(0, str(ROOT))
sys.path.insert(0, REF)

from jishui import model_torch as ref_model  # noqa: E402
from jishui.config import ModelConfig, TrainConfig  # noqa: E402
from jishui.schedules_torch import continuation_lr, make_continuation_schedule  # noqa: E402

from oracle import jishui_ref as oracle  # noqa: E402

TINY = ModelConfig(name="tiny-debug", vocab_size=24000, hidden_size=256, num_hidden_layers=4, num_attention_heads=4,
                   num_key_value_heads=4, head_dim=64, intermediate_size=688, norm_type="rmsnorm", norm_eps=1e-5,
                   norm_bias=False, rope_theta=10000.0, max_position_embeddings=2048, tie_word_embeddings=True,
                   gradient_checkpointing=False)
M200 = replace(TINY, name="jishui-200m", vocab_size=32000, hidden_size=1024, num_hidden_layers=16,
               num_attention_heads=16, num_key_value_heads=16, intermediate_size=2816)


def run_tiny(model_cls, steps=10, seed=0):
    torch.manual_seed(seed)
    torch.set_num_threads(1)
    model = model_cls(TINY)
    oracle.init_weights(model, seed)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), eps=1e-5, weight_decay=0.1)
    tokens = oracle.zipf_tokens(TINY.vocab_size, 4, 256, seed)
    x, y = tokens[:, :-1], tokens[:, 1:]
    with torch.no_grad():
        logits0 = model(x)
    out = {"logits0_sum": float(logits0.double().sum()), "logits0_sq": float(logits0.double().square().sum()),
           "losses": [], "grad_norms": []}
    for _ in range(steps):
        r = oracle.reference_update(model, opt, None, lambda: [(x, y)], 1, 1.0, 3e-4, device_type="cpu")
        out["losses"].append(r["loss"])
        out["grad_norms"].append(r["grad_norm"])
    out["param_sums"] = {n: [float(p.double().sum()), float(p.double().square().sum())]
                         for n, p in model.named_parameters()}
    out["tokens_sum"] = int(tokens.sum())
    return out


def main() -> None:
    golden = {"config_tiny": TINY.to_dict(), "config_200m": M200.to_dict()}
    ref = run_tiny(ref_model.JishuiForCausalLM)
    mine = run_tiny(oracle.JishuiRef)
    if ref != mine:
        raise SystemExit("oracle/jishui_ref.py disagrees with the reference package on the tiny run")
    golden["tiny_fp32_10_steps"] = ref

    big = ref_model.JishuiForCausalLM(M200)
    golden["params_200m"] = [[n, list(p.shape)] for n, p in big.named_parameters()]
    golden["param_count_200m"] = sum(p.numel() for p in big.parameters())
    del big

    torch.manual_seed(4)
    x = torch.randn(1, 2, 5, 64)
    golden["rope_case"] = {"input": x.flatten().tolist(), "output": ref_model.rope(x, 10000.0).flatten().tolist()}

    torch.manual_seed(5)
    q, k, v = (torch.randn(1, 2, 7, 64) for _ in range(3))
    y = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
    golden["attention_case"] = {"q": q.flatten().tolist(), "k": k.flatten().tolist(), "v": v.flatten().tolist(),
                                "out": y.flatten().tolist()}

    cfg = TrainConfig(learning_rate=3e-4, min_learning_rate=3e-5, warmup_steps=20)
    sched = make_continuation_schedule({"schedule": "cosine_warm_restarts", "cycles": 2}, cfg, 0, 200, 3e-5)
    golden["schedule_200"] = {"schedule": sched, "lr": [continuation_lr(sched, k) for k in range(0, 201)]}
    sched2 = make_continuation_schedule({"schedule": "cosine_from_imported_lr"}, cfg, 55200, 244141, 3.6e-5)
    golden["schedule_imported"] = {"schedule": sched2,
                                   "lr": [continuation_lr(sched2, k) for k in range(55200, 244142, 4999)]}

    out = Path(__file__).with_name("reference_golden.json")
    out.write_text(json.dumps(golden, indent=1))
    print(f"wrote {out} ({out.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
