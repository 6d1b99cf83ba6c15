"""Whole-model parity on the GPU: the B200 decoder against the oracle (the
reference decoder restated) running the reference's own CUDA recipe — fp16
autocast, GradScaler, torch AdamW(fused=True) — on identical seeded weights
and Zipf token batches.

Tolerances (stated by the task): per-op outputs/gradients rel 2e-3, attention /
CE gradients 1e-2 (whole-model gradients pass through both, so 1e-2 applies),
loss after 200 steps within 0.5 % relative."""
import copy
import math
from dataclasses import replace

import pytest
import torch

from conftest import rel_err
from oracle import jishui_ref as oracle

pytestmark = pytest.mark.gpu

SMALL = dict(name="small", vocab_size=4096, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
             num_key_value_heads=4, head_dim=64, intermediate_size=688, norm_type="rmsnorm", norm_eps=1e-5,
             norm_bias=False, rope_theta=10000.0, max_position_embeddings=1024, tie_word_embeddings=True,
             gradient_checkpointing=False)


# The reference's production architecture (configs/jishui-200m-cuda-4b.json: LayerNorm with bias, d 704,
# 11 heads, F 1856, V 32768, seq 2048) with 2 layers: hidden sizes that are not multiples of 128 and an odd
# head count exercise the partial GEMM tiles and the attention work split.
PROD2 = dict(SMALL, name="prod2", vocab_size=32768, hidden_size=704, num_attention_heads=11, num_key_value_heads=11,
             intermediate_size=1856, norm_type="layernorm", norm_bias=True, max_position_embeddings=2048)


def _cfg(**kw):
    from midstream_llm_b200.config import ModelConfig
    return ModelConfig(**dict(SMALL, **kw))


def _pair(cfg, seed=0):
    from midstream_llm_b200.model import JishuiForCausalLM
    ref = oracle.JishuiRef(cfg)
    oracle.init_weights(ref, seed)
    mine = JishuiForCausalLM(cfg)
    mine.load_state_dict(ref.state_dict())
    return ref.cuda(), mine.cuda()


def _batch(cfg, B, T, seed):
    rows = oracle.zipf_tokens(cfg.vocab_size, B, T, seed).cuda()
    return rows[:, :-1].contiguous(), rows[:, 1:].contiguous()


def test_forward_logits_and_loss():
    cfg = _cfg()
    ref, mine = _pair(cfg)
    x, y = _batch(cfg, 2, 256, 1)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.float16):
        ref_logits = ref(x)
        ref_loss = oracle.causal_lm_loss(ref, x, y)
    with torch.no_grad():
        logits = mine(x)
        loss = mine.loss(x, y)
    assert logits.dtype == torch.float16 and logits.shape == ref_logits.shape
    assert rel_err(logits, ref_logits) < 2e-3
    assert abs(float(loss) - float(ref_loss)) / float(ref_loss) < 1e-3


@pytest.mark.parametrize("ckpt", [False, True])
def test_backward_gradients(ckpt):
    cfg = _cfg(gradient_checkpointing=ckpt)
    ref, mine = _pair(cfg)
    x, y = _batch(cfg, 2, 256, 2)
    scale = 1024.0
    with torch.autocast("cuda", dtype=torch.float16):
        ref_loss = oracle.causal_lm_loss(ref, x, y)
    (ref_loss * scale).backward()
    from midstream_llm_b200.model import causal_lm_loss
    loss = causal_lm_loss(mine, x, y)
    (loss * scale).backward()
    assert abs(float(loss) - float(ref_loss)) / float(ref_loss) < 1e-3
    for (n, pr), (n2, pm) in zip(ref.named_parameters(), mine.named_parameters()):
        assert n == n2
        assert pm.grad is not None, n
        e = rel_err(pm.grad, pr.grad)
        assert e < 1e-2, (n, e)


def test_checkpointing_matches_plain():
    from midstream_llm_b200.model import JishuiForCausalLM, causal_lm_loss
    cfg = _cfg()
    ref, a = _pair(cfg)
    b = JishuiForCausalLM(replace(cfg, gradient_checkpointing=True))
    b.load_state_dict(ref.state_dict())
    b.cuda()
    x, y = _batch(cfg, 2, 256, 3)
    for m in (a, b):
        (causal_lm_loss(m, x, y) * 512).backward()
    for (n, pa), (_, pb) in zip(a.named_parameters(), b.named_parameters()):
        assert rel_err(pb.grad, pa.grad) < 1e-6, n


def test_grad_accumulation_adds():
    from midstream_llm_b200.model import causal_lm_loss
    cfg = _cfg()
    _, mine = _pair(cfg)
    x1, y1 = _batch(cfg, 2, 256, 4)
    x2, y2 = _batch(cfg, 2, 256, 5)
    (causal_lm_loss(mine, x1, y1) * 256).backward()
    g1 = {n: p.grad.clone() for n, p in mine.named_parameters()}
    mine.zero_grad(set_to_none=True)
    (causal_lm_loss(mine, x2, y2) * 256).backward()
    g2 = {n: p.grad.clone() for n, p in mine.named_parameters()}
    mine.zero_grad(set_to_none=True)
    (causal_lm_loss(mine, x1, y1) * 256).backward()
    (causal_lm_loss(mine, x2, y2) * 256).backward()
    for n, p in mine.named_parameters():
        assert rel_err(p.grad, g1[n] + g2[n]) < 1e-5, n


def _train(cfg, steps, accum, B, T, seed, mine_side: bool, init_scale=65536.0, sched=None):
    from midstream_llm_b200 import AdamW, GradScaler, train_update
    from midstream_llm_b200.schedules import continuation_lr
    ref, mine = _pair(cfg, seed)
    losses, attempts = [], []
    if mine_side:
        model = mine
        opt = AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), eps=1e-5, weight_decay=0.1, fused=True)
        scaler = GradScaler("cuda", init_scale=init_scale)
    else:
        model = ref
        opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), eps=1e-5, weight_decay=0.1,
                                fused=True)
        scaler = torch.amp.GradScaler("cuda", init_scale=init_scale)
    for step in range(steps):
        micro = [_batch(cfg, B, T, seed * 100000 + step * accum + i) for i in range(accum)]
        lr = continuation_lr(sched, step) if sched else 3e-4
        if mine_side:
            r = train_update(model, opt, scaler, lambda: micro, accum, 1.0, lr)
        else:
            r = oracle.reference_update(model, opt, scaler, lambda: micro, accum, 1.0, lr)
        losses.append(r["loss"])
        attempts.append(r["attempts"])
    return losses, attempts, scaler.get_scale()


@pytest.mark.slow
def test_training_200_steps_loss_parity():
    from midstream_llm_b200.config import TrainConfig
    from midstream_llm_b200.schedules import make_continuation_schedule
    cfg = _cfg()
    sched = make_continuation_schedule({"schedule": "cosine_warm_restarts", "cycles": 2},
                                       TrainConfig(learning_rate=3e-4, min_learning_rate=3e-5, warmup_steps=20),
                                       0, 200, 3e-5)
    ref_l, _, _ = _train(cfg, 200, 2, 4, 256, 7, mine_side=False, sched=sched)
    my_l, _, _ = _train(cfg, 200, 2, 4, 256, 7, mine_side=True, sched=sched)
    assert my_l[0] == pytest.approx(ref_l[0], rel=1e-3)
    tail_ref = sum(ref_l[-10:]) / 10
    tail_me = sum(my_l[-10:]) / 10
    assert abs(tail_me - tail_ref) / tail_ref < 5e-3, (tail_me, tail_ref)
    assert my_l[-1] < my_l[0] - 1.0  # it learns


def test_overflow_skip_and_retry():
    cfg = _cfg()
    ref_l, ref_att, ref_scale = _train(cfg, 3, 1, 2, 256, 9, mine_side=False, init_scale=2.0 ** 20)
    my_l, my_att, my_scale = _train(cfg, 3, 1, 2, 256, 9, mine_side=True, init_scale=2.0 ** 20)
    assert my_att[0] > 1 and ref_att[0] > 1
    assert abs(my_att[0] - ref_att[0]) <= 1
    assert my_l[-1] == pytest.approx(ref_l[-1], rel=5e-3)


def test_checkpoint_resume_is_bit_identical(tmp_path):
    """A restored checkpoint holds exactly the saved weights, optimizer moments and step, and scaler state, so the
    next update's forward (loss) is bit-identical. The update's parameters then agree to fp32 rounding, not bit
    for bit: two accumulations in the backward have no fixed order (rows of the embedding gradient that repeat
    in a batch are scattered with atomic adds, and each query tile's dQ gathers its key blocks by reduce-add),
    as in the reference's own CUDA backward."""
    from midstream_llm_b200 import AdamW, GradScaler, JishuiForCausalLM, train_update
    from midstream_llm_b200.checkpoints import load_checkpoint, save_checkpoint
    cfg = _cfg()
    _, model = _pair(cfg)
    opt = AdamW(model.parameters(), lr=1e-4, betas=(0.9, 0.95), eps=1e-5, weight_decay=0.1)
    scaler = GradScaler("cuda", init_scale=65536.0)
    micro = [_batch(cfg, 2, 256, 11)]
    train_update(model, opt, scaler, lambda: micro, 1, 1.0, 1e-4)
    state = {"model": cfg.to_dict(), "step": 1, "tokens_seen": 512}
    path = save_checkpoint(tmp_path, state, model, opt, scaler)
    saved_params = [p.detach().clone() for p in model.parameters()]
    saved_opt = copy.deepcopy(opt.state_dict())  # its tensors may view the live moment buffers
    saved_scaler = copy.deepcopy(scaler.state_dict())
    expected = train_update(model, opt, scaler, lambda: micro, 1, 1.0, 1e-4)
    restored = JishuiForCausalLM(cfg).cuda()
    ropt = AdamW(restored.parameters(), lr=0.5)
    rscaler = GradScaler("cuda")
    assert load_checkpoint(path, restored, ropt, rscaler) == state
    for a, b in zip(saved_params, restored.parameters()):
        assert torch.equal(a, b)
    rs = ropt.state_dict()
    assert rs["param_groups"] == saved_opt["param_groups"]
    for k, st in saved_opt["state"].items():
        for name, v in st.items():
            w = rs["state"][k][name]
            assert torch.equal(torch.as_tensor(v), torch.as_tensor(w)), (k, name)
    assert rscaler.state_dict() == saved_scaler
    got = train_update(restored, ropt, rscaler, lambda: micro, 1, 1.0, 1e-4)
    assert got["loss"] == expected["loss"]
    for a, b in zip(model.parameters(), restored.parameters()):
        assert rel_err(b, a) < 1e-6


def test_checkpoint_loads_into_reference_optimizer(tmp_path):
    """A bundle written by the B200 trainer restores the reference's torch objects."""
    from midstream_llm_b200 import AdamW, GradScaler, train_update
    from midstream_llm_b200.checkpoints import save_checkpoint
    cfg = _cfg()
    ref, model = _pair(cfg)
    opt = AdamW(model.parameters(), lr=1e-4, betas=(0.9, 0.95), eps=1e-5, weight_decay=0.1)
    scaler = GradScaler("cuda", init_scale=65536.0)
    train_update(model, opt, scaler, lambda: [_batch(cfg, 2, 256, 12)], 1, 1.0, 1e-4)
    path = save_checkpoint(tmp_path, {"model": cfg.to_dict(), "step": 1}, model, opt, scaler)
    bundle = torch.load(path / "training.pt", map_location="cpu", weights_only=True)
    ref.load_state_dict(bundle["model"], strict=True)
    topt = torch.optim.AdamW(ref.parameters(), lr=1e-4, fused=True)
    topt.load_state_dict(bundle["optimizer"])
    tscaler = torch.amp.GradScaler("cuda")
    tscaler.load_state_dict(bundle["scaler"])
    assert tscaler.get_scale() == scaler.get_scale()
    for p in ref.parameters():
        assert float(topt.state[p]["step"]) == 1.0


@pytest.mark.parametrize("kw,B,T", [(PROD2, 1, 2048), (dict(SMALL, norm_type="layernorm", norm_bias=False), 2, 256)])
def test_layernorm_model_parity(kw, B, T):
    """Forward loss and every parameter gradient of LayerNorm configurations against the oracle's fp16 recipe.
    Bound per parameter: rel 1e-2, or 1.5x the reference's own spread between its fp16 recipe and an fp32 run
    of the same model when that is larger (the last layer's q/k gradients of the production shape are ~1e-3 of
    the v gradients and their fp16 rounding noise alone is ~3 %)."""
    import copy
    from midstream_llm_b200.config import ModelConfig
    from midstream_llm_b200.model import causal_lm_loss
    cfg = ModelConfig(**kw)
    ref, mine = _pair(cfg)
    ref32 = copy.deepcopy(ref)
    x, y = _batch(cfg, B, T, 3)
    scale = 256.0
    with torch.autocast("cuda", dtype=torch.float16):
        ref_loss = oracle.causal_lm_loss(ref, x, y)
    (ref_loss * scale).backward()
    (oracle.causal_lm_loss(ref32, x, y) * scale).backward()
    loss = causal_lm_loss(mine, x, y)
    (loss * scale).backward()
    assert abs(float(loss) - float(ref_loss)) / float(ref_loss) < 1e-3
    names = [n for n, _ in ref.named_parameters()]
    assert names == [n for n, _ in mine.named_parameters()]
    assert any(n.endswith("norm.bias") for n in names) == bool(cfg.norm_bias)
    for (n, pr), (_, p32), (_, pm) in zip(ref.named_parameters(), ref32.named_parameters(), mine.named_parameters()):
        assert pm.grad is not None, n
        e = rel_err(pm.grad, pr.grad)
        bound = max(1e-2, 1.5 * rel_err(p32.grad, pr.grad))
        assert e < bound, (n, e, bound)


def test_evaluate_matches_reference_recipe():
    """evaluate() against the reference's evaluate body (no_grad + fp16 autocast causal_lm_loss, mean of the
    per-batch losses) on the same rows; no parameter gradient is created."""
    import numpy as np
    from midstream_llm_b200.trainer import evaluate
    cfg = _cfg()
    ref, mine = _pair(cfg)
    rows = [oracle.zipf_tokens(cfg.vocab_size, 2, 256, 50 + i).numpy().astype(np.uint16) for i in range(3)]
    losses = []
    with torch.no_grad():
        for r in rows:
            t = torch.as_tensor(r.astype(np.int64), device="cuda")
            with torch.autocast("cuda", dtype=torch.float16):
                losses.append(float(oracle.causal_lm_loss(ref, t[:, :-1], t[:, 1:])))
    got = evaluate(mine, iter(rows), 3, "cuda")
    assert abs(got - sum(losses) / 3) / (sum(losses) / 3) < 1e-3
    assert mine.training and all(p.grad is None for p in mine.parameters())
