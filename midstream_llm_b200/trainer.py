"""One optimizer update of the Jishui decoder — the reference trainer's hot loop body.

Follows Midstream-LLM src/jishui/pretrain_torch.py:204-235:
  zero_grad(set_to_none) -> grad_accum micro-batches of
  scaler.scale(loss / accum).backward() -> scaler.unscale_ -> clip_grad_norm_(grad_clip)
  -> lr from the schedule -> non-finite grad norm: scaler.update(new_scale=scale/2)
  and replay the SAME samples (at most 8 attempts) -> else scaler.step + scaler.update().

Differences in mechanics (not in results): the loss, non-finite checks and the
grad norm stay on the device until one host read at the end of the attempt
(the reference blocks on the host 2x per micro-batch and 2x per update); the
optimizer kernel skips itself on the device when the gradients overflowed, so
the skip needs no host round trip. A non-finite loss still raises
FloatingPointError without applying an update.
"""
from __future__ import annotations

import math
from typing import Callable, Sequence

import torch

from .data import tensor_batch
from .model import JishuiForCausalLM, causal_lm_loss
from .optim import AdamW, GradScaler, clip_grad_norm_

Batch = tuple[torch.Tensor, torch.Tensor]


def train_update(model: JishuiForCausalLM, optimizer: AdamW, scaler: GradScaler,
                 micro_batches: Callable[[], Sequence[Batch]], grad_accum_steps: int, grad_clip: float, lr: float,
                 max_attempts: int = 8, on_retry: Callable[[int, float], None] | None = None) -> dict:
    """Runs one update. `micro_batches()` returns this update's micro-batches; it is
    called again on a retry and must replay the same samples (the reference
    restores its sampler state for that, pretrain_torch.py:204-207)."""
    for attempt in range(max_attempts):
        optimizer.zero_grad(set_to_none=True)
        total = None
        batches = micro_batches()
        if len(batches) != grad_accum_steps:
            raise ValueError(f"expected {grad_accum_steps} micro-batches, got {len(batches)}")
        reducer = model.grad_reducer
        for i, (x, y) in enumerate(batches):
            # Data parallel: only the last micro-step's backward all-reduces the accumulated gradients
            # (the reference's no_sync rule, docs/torch-distributed.md:65); AVG is linear, so the sum of
            # the micro-steps' gradients is averaged across ranks once.
            if reducer is not None:
                reducer.enabled = i == len(batches) - 1
            loss = causal_lm_loss(model, x, y)
            total = loss.detach() if total is None else total + loss.detach()
            scaler.scale(loss / grad_accum_steps).backward()
        if reducer is not None:
            reducer.enabled = True
        scaler.unscale_(optimizer)
        grad_norm = clip_grad_norm_(model.parameters(), grad_clip)
        for group in optimizer.param_groups:
            group["lr"] = lr
        # A non-finite loss forces the device-side skip as well, so no update is
        # applied before the host sees it and raises.
        found = scaler.found_inf
        found.copy_(torch.maximum(found, (~torch.isfinite(total)).float().reshape(1)))
        optimizer.step()  # skipped on the device when found_inf != 0
        loss_sum, norm, inf = torch.stack([total, grad_norm, found[0]]).tolist()
        if not math.isfinite(loss_sum):
            raise FloatingPointError("non-finite loss")
        if inf != 0.0 or not math.isfinite(norm):
            scaler.update(new_scale=scaler.get_scale() / 2)
            if on_retry is not None:
                on_retry(attempt + 1, scaler.get_scale())
            continue
        scaler.update()
        return {"loss": loss_sum / grad_accum_steps, "grad_norm": norm, "attempts": attempt + 1, "lr": lr}
    raise FloatingPointError("gradient overflow persisted after 8 retries")


@torch.no_grad()
def evaluate(model: JishuiForCausalLM, iterator, eval_batches: int, device) -> float:
    """Mean validation loss over `eval_batches` batches of `iterator` (any object whose next() returns
    [B, T+1] integer rows, like the reference's SequentialBatchIterator), as pretrain_torch.py:42-58:
    eval mode, no autograd, the fp16 recipe, mean of the per-batch mean losses, train mode restored,
    FloatingPointError on a non-finite result. The per-batch losses are summed on the device in float64
    and read once (the reference reads each one)."""
    if eval_batches <= 0:
        raise ValueError("eval_batches must be positive")
    model.eval()
    total = torch.zeros((), dtype=torch.float64, device=device)
    for _ in range(eval_batches):
        x, y = tensor_batch(next(iterator), device)
        total += causal_lm_loss(model, x, y).double()
    model.train()
    result = float(total) / eval_batches
    if not math.isfinite(result):
        raise FloatingPointError("non-finite validation loss")
    return result


def validation_report(model: JishuiForCausalLM, make_iterator: Callable, eval_batches: int, device, step: int,
                      categories: Sequence[int] = ()) -> dict:
    """Overall and per-category validation loss (pretrain_torch.py:61-69): `make_iterator(category)` returns
    a fresh validation iterator (category None = all); `categories` lists those present in the split."""
    overall = evaluate(model, make_iterator(None), eval_batches, device)
    per_category = {c: evaluate(model, make_iterator(c), eval_batches, device) for c in categories}
    return {"step": step, "loss": overall, "per_category_loss": per_category}
