"""B200-native Jishui decoder training step.

Drop-in for the step Midstream-LLM's `jishui.model_torch` and
`jishui.pretrain_torch` run: the same module / parameter names, fp16 AMP with
GradScaler skip-and-retry, AdamW + continuation schedules and the
`checkpoints_torch` layout, with every forward/backward/optimizer kernel a
hand-written sm_100a kernel in libjishui_b200.so (C ABI: include/jishui_b200.h).
"""
from .config import ModelConfig, TrainConfig, jishui_200m, jishui_tiny, load_run_config
from .model import JishuiForCausalLM, causal_lm_loss
from .optim import AdamW, GradScaler, clip_grad_norm_
from .schedules import continuation_lr, make_continuation_schedule
from .trainer import evaluate, train_update, validation_report

__all__ = ["ModelConfig", "TrainConfig", "jishui_200m", "jishui_tiny", "load_run_config", "JishuiForCausalLM",
           "causal_lm_loss", "AdamW", "GradScaler", "clip_grad_norm_", "continuation_lr",
           "make_continuation_schedule", "train_update", "evaluate", "validation_report"]
