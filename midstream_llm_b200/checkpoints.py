"""Checkpoint layout shared with the reference's CUDA trainer.

`training.pt` bundle v1 + `train_state.json`, written into a temporary
directory, fsynced, renamed to `step_%08d`, then `latest.json` is replaced
atomically and old checkpoints pruned (Midstream-LLM
src/jishui/checkpoints_torch.py:69-112, src/jishui/checkpoints.py:1-66).
The optimizer entry is a torch-AdamW-format state dict, so a bundle written
here loads into the reference trainer and vice versa.
"""
from __future__ import annotations

import json
import os
from pathlib import Path

import torch


def check_model_config(saved: dict, requested: dict) -> None:
    """Architectures must match; gradient_checkpointing is ignored (checkpoints_torch.py:16-22)."""
    saved, requested = dict(saved), dict(requested)
    saved.pop("gradient_checkpointing", None)
    requested.pop("gradient_checkpointing", None)
    if saved != requested:
        raise ValueError("checkpoint architecture differs from requested model")


def _checkpoint_directories(run_dir: Path) -> list[Path]:
    root = Path(run_dir) / "checkpoints"
    return sorted(p for p in root.glob("step_*")
                  if p.is_dir() and p.name.startswith("step_") and p.name[5:].isdigit())


def latest_checkpoint(run_dir: Path) -> Path:
    found = _checkpoint_directories(run_dir)
    if not found:
        raise FileNotFoundError(f"no checkpoints under {Path(run_dir) / 'checkpoints'}")
    return found[-1]


def _remove_tree(path: Path) -> None:
    try:
        children = list(path.iterdir())
    except FileNotFoundError:
        return
    for child in children:
        if child.is_dir() and not child.is_symlink():
            _remove_tree(child)
        else:
            child.unlink(missing_ok=True)
    try:
        path.rmdir()
    except FileNotFoundError:
        pass


def prune_checkpoints(run_dir: Path, max_checkpoints: int, optimizer_checkpoints: int | None = None) -> None:
    """Keeps the newest `max_checkpoints` complete directories (checkpoints.py:43-66)."""
    if max_checkpoints < 1:
        raise ValueError("max_checkpoints must be positive")
    if optimizer_checkpoints is not None and not 0 <= optimizer_checkpoints <= max_checkpoints:
        raise ValueError("optimizer_checkpoints must be between 0 and max_checkpoints")
    found = _checkpoint_directories(run_dir)
    for old in found[:-max_checkpoints]:
        _remove_tree(old)
    if optimizer_checkpoints is not None:
        kept = found[-max_checkpoints:]
        trim = kept[:-optimizer_checkpoints] if optimizer_checkpoints else kept
        for path in trim:
            (path / "optimizer.npz").unlink(missing_ok=True)


def save_checkpoint(run_dir: Path, state: dict, model, optimizer, scaler, keep: int = 3) -> Path:
    """Atomic complete checkpoint (checkpoints_torch.py:69-97)."""
    run_dir = Path(run_dir)
    root = run_dir / "checkpoints"
    root.mkdir(parents=True, exist_ok=True)
    destination = root / f"step_{state['step']:08d}"
    if destination.exists():
        raise FileExistsError(destination)
    temporary = root / f".step_{state['step']:08d}.{os.getpid()}.tmp"
    temporary.mkdir(exist_ok=False)
    bundle = {
        "format_version": 1, "model": model.state_dict(),
        "optimizer": optimizer.state_dict(), "scaler": scaler.state_dict(),
        "rng": torch.get_rng_state(),
        "cuda_rng": torch.cuda.get_rng_state_all() if torch.cuda.is_available() else [],
        "state": state,
    }
    with (temporary / "training.pt").open("wb") as handle:
        torch.save(bundle, handle)
        handle.flush()
        os.fsync(handle.fileno())
    with (temporary / "train_state.json").open("w", encoding="utf-8") as handle:
        json.dump(state, handle, ensure_ascii=False, indent=2)
        handle.flush()
        os.fsync(handle.fileno())
    temporary.rename(destination)
    latest = run_dir / ".latest.json.tmp"
    latest.write_text(json.dumps({"checkpoint": str(destination), "step": state["step"]}, indent=2))
    latest.replace(run_dir / "latest.json")
    prune_checkpoints(run_dir, keep)
    return destination


def load_checkpoint(path: Path, model, optimizer, scaler) -> dict:
    """Strict restore of model, optimizer, scaler and RNG (checkpoints_torch.py:100-112)."""
    bundle = torch.load(Path(path) / "training.pt", map_location="cpu", weights_only=True, mmap=True)
    if bundle["format_version"] != 1:
        raise ValueError("unsupported CUDA checkpoint format")
    state = bundle["state"]
    check_model_config(state["model"], model.config.to_dict())
    model.load_state_dict(bundle["model"], strict=True)
    optimizer.load_state_dict(bundle["optimizer"])
    scaler.load_state_dict(bundle["scaler"])
    torch.set_rng_state(bundle["rng"])
    if bundle["cuda_rng"] and torch.cuda.is_available():
        torch.cuda.set_rng_state_all(bundle["cuda_rng"])
    return state
