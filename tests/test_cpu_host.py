"""Host-side logic on CPU: the C-ABI library loads and exports every declared
symbol, configuration validation, schedules, checkpoint retention, launch
environment / runtime plan, Zipf data, and that the product path refuses CPU
tensors instead of falling back. Mirrors Midstream-LLM tests/test_checkpoints.py,
tests/test_distributed.py and tests/test_torch_continuation.py:125-169."""
import json
import re
from dataclasses import replace
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]


def test_library_exports_every_declared_symbol():
    from midstream_llm_b200 import _lib
    lib = _lib.load()
    header = (ROOT / "include" / "jishui_b200.h").read_text()
    declared = set(re.findall(r"\b(jx_[a-z0-9_]+)\s*\(", header))
    assert declared, "no declarations found"
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(_lib.EXPORTED)
    assert lib.jx_version() >= 100


def test_pure_host_queries():
    from midstream_llm_b200 import _lib
    # one norm-backward block (one partial row) per SM, 148 without a device; fewer for short inputs
    assert _lib.query("jx_rmsnorm_bwd_parts", 16384) == 148
    assert _lib.query("jx_rmsnorm_bwd_parts", 100) == 13
    assert _lib.query("jx_grad_stats_parts", 238_322_688) >= 148
    assert _lib.query("jx_gemm_wgrad_workspace_bytes", 1024, 1024, 4) == 1024 * 1024 * 4
    assert _lib.query("jx_gemm_wgrad_workspace_bytes", 1024, 1024, 1) == 0


def test_invalid_arguments_are_rejected_with_text():
    from midstream_llm_b200 import _lib
    with pytest.raises(_lib.JxError, match="head_dim must be 64"):
        _lib.call("jx_attn_fwd", 16, 16, 16, 16, 1, 128, 1, 32, 0.125, None)
    with pytest.raises(_lib.JxError, match="cols must be a multiple of 8"):
        _lib.call("jx_rmsnorm_fwd", 16, None, None, 16, 16, 16, 4, 12, 1e-5, None)


def test_ops_refuse_cpu_tensors():
    from midstream_llm_b200 import ops
    x = torch.zeros(4, 8, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.rmsnorm_fwd(x, torch.ones(8), 1e-5)


def test_model_refuses_cpu_forward_and_unsupported_configs():
    from midstream_llm_b200 import JishuiForCausalLM
    from midstream_llm_b200.config import jishui_tiny
    m = JishuiForCausalLM(jishui_tiny())
    with pytest.raises(RuntimeError, match="CUDA only"):
        m(torch.zeros(1, 8, dtype=torch.long))
    for bad in (dict(num_key_value_heads=2), dict(attention_bias=True), dict(tie_word_embeddings=False)):
        with pytest.raises(ValueError, match="unsupported"):
            JishuiForCausalLM(replace(jishui_tiny(), **bad))


def test_layernorm_model_has_reference_parameter_names():
    """LayerNorm configurations build the reference's module tree (model_torch.py:12-15): weight and bias per
    norm, in named_parameters() order, so state dicts move both ways."""
    import sys
    sys.path.insert(0, str(ROOT))
    from oracle import jishui_ref as oracle
    from midstream_llm_b200 import JishuiForCausalLM
    from midstream_llm_b200.config import jishui_tiny
    for bias in (True, False):
        cfg = replace(jishui_tiny(), norm_type="layernorm", norm_bias=bias)
        ref, mine = oracle.JishuiRef(cfg), JishuiForCausalLM(cfg)
        names = [(n, tuple(p.shape)) for n, p in mine.named_parameters()]
        assert names == [(n, tuple(p.shape)) for n, p in ref.named_parameters()]
        assert ("norm.bias", (cfg.hidden_size,)) in names if bias else all("bias" not in n for n, _ in names)
        mine.load_state_dict(ref.state_dict(), strict=True)


def test_config_validation_matches_reference_rules():
    from midstream_llm_b200.config import ModelConfig, TrainConfig, jishui_200m
    with pytest.raises(ValueError, match="hidden_size must equal"):
        replace(jishui_200m(), hidden_size=1000)
    with pytest.raises(ValueError, match="divisible"):
        replace(jishui_200m(), num_key_value_heads=3)
    with pytest.raises(ValueError, match="even"):
        ModelConfig(name="x", vocab_size=10, hidden_size=3, num_hidden_layers=1, num_attention_heads=1,
                    num_key_value_heads=1, head_dim=3, intermediate_size=4)
    with pytest.raises(ValueError):
        TrainConfig(loss_scale=0.0)
    with pytest.raises(ValueError):
        TrainConfig(optimizer_checkpoints=5, max_checkpoints=3)
    cfg = jishui_200m()
    assert ModelConfig.from_dict(json.loads(json.dumps(cfg.to_dict()))) == cfg


def test_restart_schedule_endpoints_and_sgdr_equivalence():
    from midstream_llm_b200.config import TrainConfig
    from midstream_llm_b200.schedules import continuation_lr, make_continuation_schedule
    config = TrainConfig(learning_rate=1e-4, min_learning_rate=1e-5, warmup_steps=1000)
    s = make_continuation_schedule({"schedule": "cosine_warm_restarts", "cycles": 3}, config, 55200, 244141, 3.60865e-5)
    assert s["cycle_boundaries"] == [55200, 118181, 181161, 244141]
    assert continuation_lr(s, 55200) == pytest.approx(3.60865e-5)
    assert continuation_lr(s, 56199) == pytest.approx(1e-4)
    for b in (118180, 181160, 244140):
        assert continuation_lr(s, b) == pytest.approx(1e-5)
    restored = json.loads(json.dumps(s))
    for step in (55200, 55600, 80000, 118180, 118181, 181161, 244140, 244141):
        assert continuation_lr(restored, step) == continuation_lr(s, step)
    config0 = TrainConfig(learning_rate=1e-4, min_learning_rate=1e-5, warmup_steps=0)
    s0 = make_continuation_schedule({"schedule": "cosine_warm_restarts", "cycles": 3}, config0, 10, 310, 3.6e-5)
    p = torch.nn.Parameter(torch.zeros(1))
    sgd = torch.optim.SGD([p], lr=1e-4)
    ref = torch.optim.lr_scheduler.CosineAnnealingWarmRestarts(sgd, T_0=100, eta_min=1e-5)
    for cycle in range(3):
        for offset in (0, 1, 25, 50, 98):
            ref.step(cycle * 100 + offset * 100 / 99)
            assert continuation_lr(s0, 10 + cycle * 100 + offset) == pytest.approx(ref.get_last_lr()[0])
    for cycles in (0, -1, 1.5, 100):
        with pytest.raises(ValueError):
            make_continuation_schedule({"schedule": "cosine_warm_restarts", "cycles": cycles}, config, 10, 3010, 3.6e-5)


def test_checkpoint_retention(tmp_path):
    from midstream_llm_b200.checkpoints import latest_checkpoint, prune_checkpoints
    root = tmp_path / "checkpoints"
    root.mkdir()
    for step in (200, 400, 600, 800):
        (root / f"step_{step:08d}").mkdir()
        (root / f"step_{step:08d}" / "optimizer.npz").write_bytes(b"adam")
    (root / ".step_00001000.tmp").mkdir()
    (root / "step_notes").mkdir()
    prune_checkpoints(tmp_path, max_checkpoints=3)
    assert sorted(p.name for p in root.iterdir()) == [".step_00001000.tmp", "step_00000400", "step_00000600",
                                                     "step_00000800", "step_notes"]
    assert latest_checkpoint(tmp_path).name == "step_00000800"
    prune_checkpoints(tmp_path, max_checkpoints=3, optimizer_checkpoints=1)
    assert not (root / "step_00000400" / "optimizer.npz").exists()
    assert (root / "step_00000800" / "optimizer.npz").exists()


def test_launch_environment_and_runtime_plan():
    from midstream_llm_b200.distributed import DistributedCapabilityError, LaunchEnvironment, build_runtime_plan
    with pytest.raises(DistributedCapabilityError, match="incomplete torchrun environment"):
        LaunchEnvironment.from_environ({"WORLD_SIZE": "8"})
    env = LaunchEnvironment.from_environ({"RANK": "5", "LOCAL_RANK": "1", "WORLD_SIZE": "8"})
    assert env == LaunchEnvironment(rank=5, local_rank=1, world_size=8)
    with pytest.raises(DistributedCapabilityError):
        LaunchEnvironment.from_environ({"RANK": "9", "LOCAL_RANK": "1", "WORLD_SIZE": "8"})
    plan = build_runtime_plan("cuda", env)
    assert (plan.device, plan.process_group_backend, plan.distributed) == ("cuda:1", "nccl", True)
    assert build_runtime_plan("cpu").process_group_backend == "gloo"
    with pytest.raises(DistributedCapabilityError, match="cannot mix accelerator types"):
        build_runtime_plan("cuda,ascend-npu")
    with pytest.raises(DistributedCapabilityError, match="not supported"):
        build_runtime_plan("apple-ane")


def test_zipf_stream_is_deterministic_and_resumable():
    from midstream_llm_b200.data import ZipfBatches
    a = ZipfBatches(32000, 2, 16, seed=3)
    first = a.next_rows()
    state = a.state_dict()
    second = a.next_rows()
    b = ZipfBatches(32000, 2, 16, seed=3)
    b.load_state_dict(json.loads(json.dumps(state)))
    assert np.array_equal(b.next_rows(), second)
    c = ZipfBatches(32000, 2, 16, seed=3)
    assert np.array_equal(c.next_rows(), first)
    big = ZipfBatches(32000, 64, 1024, seed=0).next_rows()
    # Zipf(1.1): id 0 is the most frequent token, ~ 1/H(1.1) of all draws.
    assert (big == 0).mean() > 0.08 and big.max() < 32000


def test_oracle_and_product_zipf_streams_agree():
    from midstream_llm_b200.data import ZipfBatches
    from oracle import jishui_ref as oracle
    rows = ZipfBatches(4096, 2, 64, seed=7).next_rows()
    assert np.array_equal(rows, oracle.zipf_tokens(4096, 2, 64, 7).numpy())


def test_product_does_not_import_the_oracle():
    for path in (ROOT / "midstream_llm_b200").rglob("*.py"):
        text = path.read_text()
        assert "import oracle" not in text and "from oracle" not in text, path


def test_evaluate_host_logic():
    """evaluate(): mean of per-batch losses over eval_batches rows of the iterator, train mode restored, a
    non-finite mean raises (pretrain_torch.py:42-58); validation_report() asks for one iterator per category."""
    from midstream_llm_b200.trainer import evaluate, validation_report

    class Stub(torch.nn.Module):
        def __init__(self, values):
            super().__init__()
            self.values, self.seen = list(values), []

        def loss(self, x, y):
            assert not self.training and not torch.is_grad_enabled()
            assert x.dtype == torch.int64 and x.shape == (2, 8) and torch.equal(x[:, 1:], y[:, :-1])
            self.seen.append(int(x[0, 0]))
            return torch.tensor(self.values.pop(0))

    rows = (np.arange(5 * 2 * 9, dtype=np.uint16).reshape(5, 2, 9))
    m = Stub([1.0, 2.0, 4.0])
    assert evaluate(m, iter(rows), 3, "cpu") == pytest.approx(7.0 / 3)
    assert m.training and m.seen == [0, 18, 36]
    with pytest.raises(FloatingPointError, match="non-finite"):
        evaluate(Stub([1.0, float("inf")]), iter(rows), 2, "cpu")
    asked = []

    def make(c):
        asked.append(c)
        return iter(rows)

    rep = validation_report(Stub([1.0] * 3), make, 1, "cpu", step=200, categories=(2, 5))
    assert asked == [None, 2, 5] and rep == {"step": 200, "loss": 1.0, "per_category_loss": {2: 1.0, 5: 1.0}}
