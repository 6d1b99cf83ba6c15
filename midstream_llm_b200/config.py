"""Run configuration records for the Jishui decoder and its trainer.

The field names, their order and their defaults are an interface shared with
Midstream-LLM (src/jishui/config.py:11-99): run-config JSON files
(`{"model": {...}, "training": {...}}`) and the `model` record stored in every
checkpoint's `train_state.json` are written by one trainer and read by the
other, so both records round-trip through `to_dict()` / `from_dict()`
unchanged. The checks below are derived from what each field means to the
model and the update loop; each record reports every violated constraint at
once in a single ValueError.

`JishuiForCausalLM` accepts any object carrying these attributes, including the
reference's own `ModelConfig`.
"""
from __future__ import annotations

import json
import math
from dataclasses import asdict, dataclass
from pathlib import Path
from typing import Any, Iterator

NORM_TYPES = ("layernorm", "rmsnorm")
COMPUTE_DTYPES = ("float32", "float16", "bfloat16")
SAMPLING_MODES = ("target", "weights")


class _Record:
    """JSON round-trip shared by both records: unknown keys are an error (TypeError from the constructor)."""

    @classmethod
    def from_dict(cls, value: dict[str, Any]):
        return cls(**value)

    @classmethod
    def from_json(cls, path: str | Path):
        return cls.from_dict(json.loads(Path(path).read_text(encoding="utf-8")))

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    def _violations(self) -> Iterator[str]:  # pragma: no cover - overridden
        return iter(())

    def __post_init__(self) -> None:
        problems = list(self._violations())
        if problems:
            raise ValueError(f"invalid {type(self).__name__}: " + "; ".join(problems))


@dataclass(frozen=True)
class ModelConfig(_Record):
    """Decoder architecture (the reference's config.py:11-28 fields)."""
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

    def _violations(self) -> Iterator[str]:
        # The attention heads tile the hidden state exactly.
        if self.num_attention_heads * self.head_dim != self.hidden_size:
            yield (f"hidden_size must equal num_attention_heads * head_dim ({self.hidden_size} != "
                   f"{self.num_attention_heads} * {self.head_dim})")
        # Each key/value head serves a whole group of query heads.
        if self.num_key_value_heads < 1 or self.num_attention_heads % self.num_key_value_heads:
            yield "num_attention_heads must be divisible by num_key_value_heads"
        # RoPE rotates the two halves of every head against each other.
        if self.head_dim % 2:
            yield "head_dim must be even for RoPE"
        if self.norm_type not in NORM_TYPES:
            yield f"norm_type must be one of {', '.join(NORM_TYPES)} (got {self.norm_type!r})"


@dataclass(frozen=True)
class TrainConfig(_Record):
    """Optimizer, AMP and loop inputs (the reference's config.py:57-83 fields)."""
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

    def _violations(self) -> Iterator[str]:
        if self.dtype not in COMPUTE_DTYPES:
            yield f"dtype must be one of {', '.join(COMPUTE_DTYPES)} (got {self.dtype!r})"
        # The initial GradScaler scale multiplies the loss.
        if not (math.isfinite(self.loss_scale) and self.loss_scale > 0):
            yield "loss_scale must be finite and positive"
        sizes = {"seq_len": self.seq_len, "batch_size": self.batch_size,
                 "grad_accum_steps": self.grad_accum_steps, "max_steps": self.max_steps}
        for key, value in sizes.items():
            if value < 1:
                yield f"{key} must be positive (got {value})"
        if self.sampling_mode not in SAMPLING_MODES:
            yield f"sampling_mode must be one of {', '.join(SAMPLING_MODES)} (got {self.sampling_mode!r})"
        # AdamW divides by sqrt(v) + eps.
        if not self.adam_eps > 0:
            yield "adam_eps must be positive"
        if self.max_checkpoints < 1:
            yield "max_checkpoints must be positive"
        # Optimizer state is kept in a subset of the retained checkpoints.
        if not 0 <= self.optimizer_checkpoints <= self.max_checkpoints:
            yield "optimizer_checkpoints must be between 0 and max_checkpoints"


def load_run_config(path: str | Path) -> tuple[ModelConfig, TrainConfig]:
    """Both records of a `{"model": ..., "training": ...}` run-config file."""
    raw = json.loads(Path(path).read_text(encoding="utf-8"))
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
