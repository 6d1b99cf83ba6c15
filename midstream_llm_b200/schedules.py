"""Learning-rate schedule inputs, indexed by completed optimizer updates.

Same schedule dictionaries and formulas as the reference
(Midstream-LLM src/jishui/schedules_torch.py:7-59): "cosine_from_imported_lr"
and SGDR-style "cosine_warm_restarts" with an optional linear warmup in the
first cycle. A schedule saved by either implementation is accepted by both.
"""
from __future__ import annotations

import math


def make_continuation_schedule(continuation, config, start_step, end_step, imported_lr):
    """Builds the schedule dict (schedules_torch.py:7-31)."""
    mode = continuation["schedule"]
    common = {"mode": mode, "start_step": start_step, "end_step": end_step,
              "start_lr": imported_lr, "end_lr": config.min_learning_rate}
    if mode == "cosine_from_imported_lr":
        return common
    if mode != "cosine_warm_restarts":
        raise ValueError("unsupported continuation schedule")
    cycles = continuation.get("cycles", 3)
    if type(cycles) is not int or cycles < 1:
        raise ValueError("cycles must be a positive integer")
    width, extra = divmod(end_step - start_step, cycles)
    if width < 2 or config.warmup_steps < 0 or config.warmup_steps == 1:
        raise ValueError("cycles need at least two updates; warmup must be zero or >=2")
    finite = all(math.isfinite(v) for v in (imported_lr, config.learning_rate, config.min_learning_rate))
    if not finite or not 0 < config.min_learning_rate <= imported_lr <= config.learning_rate:
        raise ValueError("restart schedule requires 0 < min_lr <= imported_lr <= peak_lr")
    boundaries = [start_step]
    for i in range(cycles):
        boundaries.append(boundaries[-1] + width + (1 if i < extra else 0))
    if config.warmup_steps > boundaries[1] - start_step - 2:
        raise ValueError("first cycle must leave at least two cosine decay updates after warmup")
    return dict(common, peak_lr=config.learning_rate, warmup_steps=config.warmup_steps,
                cycle_boundaries=boundaries)


def _cosine(lo: float, hi: float, progress: float) -> float:
    return lo + 0.5 * (hi - lo) * (1 + math.cos(math.pi * progress))


def continuation_lr(schedule: dict, completed_step: int) -> float:
    """LR for the NEXT update (schedules_torch.py:34-59): each restart cycle's first
    and last update use exactly the peak and minimum LR; only the first cycle warms up
    linearly from the imported LR."""
    mode = schedule.get("mode", "cosine_from_imported_lr")
    if mode == "cosine_from_imported_lr":
        span = max(1, schedule["end_step"] - schedule["start_step"])
        progress = min(1.0, max(0.0, (completed_step - schedule["start_step"]) / span))
        return _cosine(schedule["end_lr"], schedule["start_lr"], progress)
    if mode != "cosine_warm_restarts":
        raise ValueError("unsupported continuation schedule")
    if completed_step >= schedule["end_step"]:
        return schedule["end_lr"]
    completed_step = max(schedule["start_step"], completed_step)
    bounds = schedule["cycle_boundaries"]
    for cycle, (begin, end) in enumerate(zip(bounds, bounds[1:])):
        if begin <= completed_step < end:
            offset = completed_step - begin
            warmup = schedule["warmup_steps"] if cycle == 0 else 0
            if offset < warmup:
                return schedule["start_lr"] + (schedule["peak_lr"] - schedule["start_lr"]) * offset / (warmup - 1)
            progress = (offset - warmup) / (end - begin - warmup - 1)
            return _cosine(schedule["end_lr"], schedule["peak_lr"], progress)
    raise ValueError("invalid cycle boundaries")
