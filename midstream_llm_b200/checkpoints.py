"""Checkpoints in the on-disk layout the reference's CUDA trainer reads and writes.

Layout (the format of Midstream-LLM src/jishui/checkpoints_torch.py:69-112 and
src/jishui/checkpoints.py:43-66):

    <run>/checkpoints/step_<step, 8 digits>/training.pt       torch.save of the bundle below
    <run>/checkpoints/step_<step, 8 digits>/train_state.json  the loop's `state` record as JSON
    <run>/latest.json   {"checkpoint": "<that directory>", "step": <step>}

    bundle = {"format_version": 1, "model": state_dict, "optimizer": AdamW state_dict,
              "scaler": GradScaler state_dict, "rng": CPU RNG state,
              "cuda_rng": per-device CUDA RNG states (or []), "state": the same record}

Only directories named `step_` followed by digits are checkpoints. A checkpoint
appears under that name only when both of its files are complete and synced:
it is assembled in a hidden staging directory next to it and renamed in one
step, so a crash leaves either the old set or the new one. The optimizer entry
uses torch.optim.AdamW's state-dict format and the scaler entry
torch.amp.GradScaler's, so a bundle moves between this trainer and the
reference in both directions.
"""
from __future__ import annotations

import json
import os
import re
import shutil
import tempfile
from pathlib import Path

import torch

FORMAT_VERSION = 1
_STEP_DIR = re.compile(r"step_(\d+)")
# Fields of the model record that change how the model runs but not its parameters.
_RUNTIME_ONLY_FIELDS = frozenset({"gradient_checkpointing"})


def _architecture(record: dict) -> dict:
    return {k: v for k, v in dict(record).items() if k not in _RUNTIME_ONLY_FIELDS}


def check_model_config(saved: dict, requested: dict) -> None:
    """Raises ValueError unless the two model records describe the same parameters (recompute settings
    are not compared)."""
    a, b = _architecture(saved), _architecture(requested)
    if a != b:
        keys = sorted(k for k in a.keys() | b.keys() if a.get(k, ...) != b.get(k, ...))
        raise ValueError(f"checkpoint architecture differs from requested model: {', '.join(keys)}")


def _checkpoint_directories(run_dir: Path) -> list[Path]:
    """Complete checkpoint directories of a run, oldest step first."""
    root = Path(run_dir) / "checkpoints"
    if not root.is_dir():
        return []
    found = []
    for entry in root.iterdir():
        match = _STEP_DIR.fullmatch(entry.name)
        if match and entry.is_dir():
            found.append((int(match.group(1)), entry))
    return [path for _, path in sorted(found)]


def latest_checkpoint(run_dir: Path) -> Path:
    found = _checkpoint_directories(run_dir)
    if not found:
        raise FileNotFoundError(f"no checkpoints under {Path(run_dir) / 'checkpoints'}")
    return found[-1]


def prune_checkpoints(run_dir: Path, max_checkpoints: int, optimizer_checkpoints: int | None = None) -> None:
    """Deletes all but the newest `max_checkpoints` checkpoints. With `optimizer_checkpoints` set, only that
    many of the kept ones (the newest) keep their `optimizer.npz` (the reference's MLX Adam state file)."""
    if max_checkpoints < 1:
        raise ValueError("max_checkpoints must be positive")
    if optimizer_checkpoints is not None and not 0 <= optimizer_checkpoints <= max_checkpoints:
        raise ValueError("optimizer_checkpoints must be between 0 and max_checkpoints")
    found = _checkpoint_directories(run_dir)
    kept = found[-max_checkpoints:]
    for path in found[:len(found) - len(kept)]:
        shutil.rmtree(path, ignore_errors=True)
    if optimizer_checkpoints is not None:
        for path in kept[:len(kept) - optimizer_checkpoints]:
            (path / "optimizer.npz").unlink(missing_ok=True)


def _fsync_dir(path: Path) -> None:
    fd = os.open(path, os.O_RDONLY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def _write_synced(path: Path, write) -> None:
    with path.open("wb") as handle:
        write(handle)
        handle.flush()
        os.fsync(handle.fileno())


def save_checkpoint(run_dir: Path, state: dict, model, optimizer, scaler, keep: int = 3) -> Path:
    """Writes checkpoint `state["step"]`, points latest.json at it and prunes to `keep` checkpoints.
    Raises FileExistsError if that step was already saved."""
    run_dir = Path(run_dir)
    root = run_dir / "checkpoints"
    root.mkdir(parents=True, exist_ok=True)
    final = root / f"step_{state['step']:08d}"
    if final.exists():
        raise FileExistsError(final)
    bundle = {"format_version": FORMAT_VERSION, "model": model.state_dict(), "optimizer": optimizer.state_dict(),
              "scaler": scaler.state_dict(), "rng": torch.get_rng_state(),
              "cuda_rng": torch.cuda.get_rng_state_all() if torch.cuda.is_available() else [], "state": state}
    staging = Path(tempfile.mkdtemp(prefix=f".{final.name}.", suffix=".tmp", dir=root))
    try:
        _write_synced(staging / "training.pt", lambda h: torch.save(bundle, h))
        _write_synced(staging / "train_state.json",
                      lambda h: h.write(json.dumps(state, ensure_ascii=False, indent=2).encode("utf-8")))
        staging.rename(final)
    except BaseException:
        shutil.rmtree(staging, ignore_errors=True)
        raise
    _fsync_dir(root)
    pointer = json.dumps({"checkpoint": str(final), "step": state["step"]}, indent=2).encode("utf-8")
    fd, tmp = tempfile.mkstemp(prefix=".latest.", suffix=".tmp", dir=run_dir)
    with os.fdopen(fd, "wb") as handle:
        handle.write(pointer)
        handle.flush()
        os.fsync(handle.fileno())
    os.replace(tmp, run_dir / "latest.json")
    prune_checkpoints(run_dir, keep)
    return final


def load_checkpoint(path: Path, model, optimizer, scaler) -> dict:
    """Restores model (strict), optimizer, scaler and RNG states from a checkpoint directory and returns
    its `state` record. The model's architecture must match the saved one."""
    bundle = torch.load(Path(path) / "training.pt", map_location="cpu", weights_only=True, mmap=True)
    if bundle.get("format_version") != FORMAT_VERSION:
        raise ValueError(f"unsupported checkpoint format {bundle.get('format_version')!r}")
    state = bundle["state"]
    check_model_config(state["model"], model.config.to_dict())
    model.load_state_dict(bundle["model"], strict=True)
    optimizer.load_state_dict(bundle["optimizer"])
    scaler.load_state_dict(bundle["scaler"])
    torch.set_rng_state(bundle["rng"])
    if bundle["cuda_rng"] and torch.cuda.is_available():
        torch.cuda.set_rng_state_all(bundle["cuda_rng"])
    return state
