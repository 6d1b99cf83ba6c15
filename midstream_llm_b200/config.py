"""Run configuration: the same dataclasses, fields, defaults and validation as
the reference (Midstream-LLM src/jishui/config.py:11-112), so JSON run configs
and checkpoint `train_state.json` records load unchanged."""
from __future__ import annotations

import json
import math
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any


@dataclass(frozen=True)
class ModelConfig:
    """Decoder architecture (config.py:11-41). Validation matches the reference."""
    name: str
    vocab_size: int
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    norm_type: str = "layernorm"
    norm_eps: float = 1.0e-5
    norm_bias: bool = True
    rope_theta: float = 10_000.0
    max_position_embeddings: int = 2048
    tie_word_embeddings: bool = True
    attention_bias: bool = False
    mlp_bias: bool = False
    gradient_checkpointing: bool = True

    def __post_init__(self) -> None:
        if self.hidden_size != self.num_attention_heads * self.head_dim:
            raise ValueError(
                "hidden_size must equal num_attention_heads * head_dim: "
                f"{self.hidden_size} != {self.num_attention_heads} * {self.head_dim}")
        if self.num_attention_heads % self.num_key_value_heads != 0:
            raise ValueError("num_attention_heads must be divisible by num_key_value_heads")
        if self.head_dim % 2:
            raise ValueError("head_dim must be even for RoPE")
        if self.norm_type not in {"layernorm", "rmsnorm"}:
            raise ValueError("norm_type must be layernorm or rmsnorm")

    @classmethod
    def from_dict(cls, value: dict[str, Any]) -> "ModelConfig":
        return cls(**value)

    @classmethod
    def from_json(cls, path: str | Path) -> "ModelConfig":
        with Path(path).open(encoding="utf-8") as handle:
            return cls.from_dict(json.load(handle))

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


@dataclass(frozen=True)
class TrainConfig:
    """Optimizer / AMP / loop inputs (config.py:57-99)."""
    seed: int = 42
    dtype: str = "float16"
    loss_scale: float = 1.0
    seq_len: int = 2048
    batch_size: int = 1
    grad_accum_steps: int = 8
    max_steps: int = 10_000
    learning_rate: float = 3.0e-4
    min_learning_rate: float = 3.0e-5
    warmup_steps: int = 200
    weight_decay: float = 0.1
    beta1: float = 0.9
    beta2: float = 0.95
    adam_eps: float = 1.0e-5
    grad_clip: float = 1.0
    log_interval: int = 1
    eval_interval: int = 200
    eval_batches: int = 10
    save_interval: int = 200
    max_checkpoints: int = 3
    optimizer_checkpoints: int = 3
    sampling_mode: str = "target"
    eod_token_id: int = 2
    compile_step: bool = True

    def __post_init__(self) -> None:
        if self.dtype not in {"float32", "float16", "bfloat16"}:
            raise ValueError("dtype must be float32, float16, or bfloat16")
        if not math.isfinite(self.loss_scale) or self.loss_scale <= 0:
            raise ValueError("loss_scale must be finite and positive")
        if min(self.seq_len, self.batch_size, self.grad_accum_steps, self.max_steps) < 1:
            raise ValueError("sequence, batch, accumulation, and step values must be positive")
        if self.sampling_mode not in {"target", "weights"}:
            raise ValueError("sampling_mode must be target or weights")
        if self.adam_eps <= 0:
            raise ValueError("adam_eps must be positive")
        if self.max_checkpoints < 1:
            raise ValueError("max_checkpoints must be positive")
        if self.optimizer_checkpoints < 0 or self.optimizer_checkpoints > self.max_checkpoints:
            raise ValueError("optimizer_checkpoints must be between 0 and max_checkpoints")

    @classmethod
    def from_dict(cls, value: dict[str, Any]) -> "TrainConfig":
        return cls(**value)

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


def load_run_config(path: str | Path) -> tuple[ModelConfig, TrainConfig]:
    """Reads the {model, training, ...} JSON run config (config.py:109-112)."""
    with Path(path).open(encoding="utf-8") as handle:
        raw = json.load(handle)
    return ModelConfig.from_dict(raw["model"]), TrainConfig.from_dict(raw["training"])


def jishui_200m(seq_len: int = 1024, gradient_checkpointing: bool = False) -> ModelConfig:
    """The 200M decoder measured here: V 32000, d 1024, 16 layers x 16 heads of 64,
    SwiGLU 2816, RMSNorm, RoPE 10000, tied embeddings."""
    return ModelConfig(name="jishui-200m", vocab_size=32000, hidden_size=1024, num_hidden_layers=16,
                       num_attention_heads=16, num_key_value_heads=16, head_dim=64, intermediate_size=2816,
                       norm_type="rmsnorm", norm_eps=1e-5, norm_bias=False, rope_theta=10000.0,
                       max_position_embeddings=max(2048, seq_len), tie_word_embeddings=True,
                       gradient_checkpointing=gradient_checkpointing)


def jishui_200m_base(gradient_checkpointing: bool = False) -> ModelConfig:
    """The reference's production decoder (configs/jishui-200m-cuda-4b.json): V 32768, d 704, 30 layers x 11
    heads of 64, SwiGLU 1856, LayerNorm with bias, RoPE 10000, context 2048, tied embeddings."""
    return ModelConfig(name="Jishui-200M-Base", vocab_size=32768, hidden_size=704, num_hidden_layers=30,
                       num_attention_heads=11, num_key_value_heads=11, head_dim=64, intermediate_size=1856,
                       norm_type="layernorm", norm_eps=1e-5, norm_bias=True, rope_theta=10000.0,
                       max_position_embeddings=2048, tie_word_embeddings=True,
                       gradient_checkpointing=gradient_checkpointing)


def jishui_tiny(gradient_checkpointing: bool = False) -> ModelConfig:
    """Tiny debug decoder: V 24000, d 256, 4 layers x 4 heads of 64, SwiGLU 688."""
    return ModelConfig(name="jishui-tiny", vocab_size=24000, hidden_size=256, num_hidden_layers=4,
                       num_attention_heads=4, num_key_value_heads=4, head_dim=64, intermediate_size=688,
                       norm_type="rmsnorm", norm_eps=1e-5, norm_bias=False, rope_theta=10000.0,
                       max_position_embeddings=2048, tie_word_embeddings=True,
                       gradient_checkpointing=gradient_checkpointing)
