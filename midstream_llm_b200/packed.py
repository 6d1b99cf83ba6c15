"""Packed corpus rows built on the device.

The reference trainer draws packed rows on the host (Midstream-LLM src/jishui/data.py:233-330
PackedBatchIterator for training, :333-379 SequentialBatchIterator for validation): each row of
seq_len + 1 tokens is filled with spans of uint16 documents, an end-of-document token after every
document that ends inside the row, then copied to the GPU per micro-batch (pretrain_torch.py:38-40).

Here the same random draws decide the same spans (the *plan* of a row: a few (column, token, count)
runs), the token shards stay resident in device memory, and `jx_pack_rows` writes the int64 rows on
the device; only the plan (tens of bytes per document span) crosses PCIe. A background thread plans
the next batches while the GPU works. Rows are identical to the reference iterators' for the same
index, sampling weights and seed.

The index argument is the reference's `PretrainIndex` (or any object with the same fields:
shards, offsets, lengths, categories, splits, token_shards, indices_for).
"""
from __future__ import annotations

import queue
import threading

import numpy as np
import torch

from . import _lib

SPLIT_TO_ID = {"train": 0, "val": 1, "test": 2}


def _split_ids(index, split: str) -> np.ndarray:
    """Documents of a split with a known category (data.py:86-90 indices_for)."""
    if hasattr(index, "indices_for"):
        return index.indices_for(split)
    mask = (index.splits == SPLIT_TO_ID[split]) & (index.categories > 0)
    return np.flatnonzero(mask)


class DeviceTokenStore:
    """Every token shard of the index in one device buffer (uint16 bits), with the global start of
    each shard. 4B tokens take 8 GB of HBM."""

    def __init__(self, index, device):
        shards = list(index.token_shards)
        sizes = [int(s.shape[0]) for s in shards]
        self.base = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
        self.ntokens = int(self.base[-1])
        self.tokens = torch.empty(self.ntokens, dtype=torch.int16, device=device)
        for s, start in zip(shards, self.base[:-1]):
            host = torch.from_numpy(np.ascontiguousarray(s, dtype=np.uint16).view(np.int16))
            self.tokens[int(start):int(start) + host.numel()].copy_(host)

    def token_start(self, shard: int, offset: int) -> int:
        return int(self.base[shard]) + offset


class _Plan:
    """Runs of one batch: int64 [n, 3] (dst column, src token or -(eod+1), count) and int32
    row starts [rows + 1]."""

    __slots__ = ("runs", "row_start")

    def __init__(self):
        self.runs: list[tuple[int, int, int]] = []
        self.row_start: list[int] = [0]

    def end_row(self) -> None:
        self.row_start.append(len(self.runs))


class PackedRowPlanner:
    """The draws of PackedBatchIterator (data.py:233-330), producing row plans instead of rows."""

    def __init__(self, index, sampling: dict, seq_len: int, batch_size: int, seed: int, mode: str = "target",
                 eod_token_id: int = 2):
        self.index, self.seq_len, self.batch_size = index, seq_len, batch_size
        self.eod_token_id, self.mode = eod_token_id, mode
        self.rng = np.random.default_rng(seed)
        self.batches_emitted = 0
        train_ids = _split_ids(index, "train")
        self._groups: dict[int, np.ndarray] = {}
        self._cumulative: dict[int, np.ndarray] = {}
        totals: dict[int, int] = {}
        for category in range(1, 7):
            ids = train_ids[index.categories[train_ids] == category]
            if len(ids) == 0:
                continue
            self._groups[category] = ids
            cumulative = np.cumsum(index.lengths[ids], dtype=np.uint64)
            self._cumulative[category] = cumulative
            totals[category] = int(cumulative[-1])
        self.category_ids = np.asarray(sorted(self._groups), dtype=np.uint8)
        if mode == "target":
            raw = np.asarray([float(sampling["target_mix"][str(c)]) for c in self.category_ids], dtype=np.float64)
        elif mode == "weights":
            raw = np.asarray([totals[int(c)] * float(sampling["weights_by_category"][str(c)])
                              for c in self.category_ids], dtype=np.float64)
        else:
            raise ValueError(f"unknown sampling mode: {mode}")
        self.category_probabilities = raw / raw.sum()

    def plan(self, store: DeviceTokenStore) -> _Plan:
        plan = _Plan()
        selected = self.rng.choice(self.category_ids, size=self.batch_size, p=self.category_probabilities)
        for category in selected:
            self._plan_row(plan, int(category), store)
            plan.end_row()
        self.batches_emitted += 1
        return plan

    def _plan_row(self, plan: _Plan, category: int, store: DeviceTokenStore) -> None:
        ids, cumulative, idx = self._groups[category], self._cumulative[category], self.index
        width = self.seq_len + 1
        position = 0
        while position < width:
            token_position = int(self.rng.integers(0, int(cumulative[-1])))
            local_doc = int(np.searchsorted(cumulative, token_position, side="right"))
            previous = int(cumulative[local_doc - 1]) if local_doc else 0
            start_in_doc = token_position - previous
            doc_index = int(ids[local_doc])
            available = int(idx.lengths[doc_index]) - start_in_doc
            count = min(available, width - position)
            src = store.token_start(int(idx.shards[doc_index]), int(idx.offsets[doc_index]) + start_in_doc)
            plan.runs.append((position, src, count))
            position += count
            if count == available and position < width:
                plan.runs.append((position, -(self.eod_token_id + 1), 1))
                position += 1

    def state_dict(self) -> dict:
        return {"batches_emitted": self.batches_emitted, "rng_state": self.rng.bit_generator.state}

    def load_state_dict(self, state: dict) -> None:
        self.batches_emitted = int(state["batches_emitted"])
        self.rng.bit_generator.state = state["rng_state"]


class SequentialRowPlanner:
    """The document stream of SequentialBatchIterator (data.py:333-379), producing row plans."""

    def __init__(self, index, split: str, seq_len: int, batch_size: int, eod_token_id: int = 2,
                 category: int | None = None):
        self.index = index
        self.doc_ids = _split_ids(index, split)
        if category is not None:
            self.doc_ids = self.doc_ids[index.categories[self.doc_ids] == category]
        if len(self.doc_ids) == 0:
            label = f"{split} category={category}" if category is not None else split
            raise ValueError(f"no usable documents in {label}")
        self.seq_len, self.batch_size, self.eod_token_id = seq_len, batch_size, eod_token_id
        self.doc_position = 0
        self.token_position = 0

    def plan(self, store: DeviceTokenStore) -> _Plan:
        plan = _Plan()
        for _ in range(self.batch_size):
            self._plan_row(plan, store)
            plan.end_row()
        return plan

    def _plan_row(self, plan: _Plan, store: DeviceTokenStore) -> None:
        idx, width = self.index, self.seq_len + 1
        position = 0
        while position < width:
            doc_index = int(self.doc_ids[self.doc_position])
            length = int(idx.lengths[doc_index])
            available = length - self.token_position
            count = min(available, width - position)
            src = store.token_start(int(idx.shards[doc_index]), int(idx.offsets[doc_index]) + self.token_position)
            plan.runs.append((position, src, count))
            position += count
            self.token_position += count
            if self.token_position == length:
                self.doc_position = (self.doc_position + 1) % len(self.doc_ids)
                self.token_position = 0
                if position < width:
                    plan.runs.append((position, -(self.eod_token_id + 1), 1))
                    position += 1

    def state_dict(self) -> dict:
        return {"doc_position": self.doc_position, "token_position": self.token_position}

    def load_state_dict(self, state: dict) -> None:
        self.doc_position = int(state["doc_position"])
        self.token_position = int(state["token_position"])


def pack_rows(store: DeviceTokenStore, runs: torch.Tensor, row_start: torch.Tensor, rows: int, width: int,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """int64 [rows, width] token rows on the device from a plan already on the device."""
    if runs.device.type != "cuda" or row_start.device.type != "cuda":
        raise RuntimeError("pack_rows: the plan must be on the CUDA device (there is no CPU path)")
    out = out if out is not None else torch.empty(rows, width, dtype=torch.int64, device=runs.device)
    _lib.call("jx_pack_rows", store.tokens.data_ptr(), store.ntokens, runs.data_ptr(), row_start.data_ptr(), rows,
              width, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return out


class DeviceBatches:
    """Iterator of int64 [batch, seq+1] rows on the device for a planner (PackedRowPlanner or
    SequentialRowPlanner). A background thread plans up to `prefetch` batches ahead into pinned host
    memory; next() copies one plan on the current stream and gathers the rows there. state_dict() is
    the planner's state before the first batch not yet returned, so a checkpoint resumes exactly."""

    def __init__(self, planner, store: DeviceTokenStore, prefetch: int = 4):
        self.planner, self.store = planner, store
        self.width = planner.seq_len + 1
        self.prefetch = max(1, prefetch)
        self._state = planner.state_dict()
        self._start()

    def _start(self) -> None:
        self._queue: queue.Queue = queue.Queue(maxsize=self.prefetch)
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._work, name="jx-row-planner", daemon=True)
        self._thread.start()

    def _work(self) -> None:
        try:
            while not self._stop.is_set():
                plan = self.planner.plan(self.store)
                runs = torch.tensor(plan.runs, dtype=torch.int64).pin_memory()
                starts = torch.tensor(plan.row_start, dtype=torch.int32).pin_memory()
                item = (runs, starts, self.planner.state_dict())
                while not self._stop.is_set():
                    try:
                        self._queue.put(item, timeout=0.1)
                        break
                    except queue.Full:
                        continue
        except BaseException as exc:  # surfaced by the consumer
            self._queue.put(exc)

    def __iter__(self) -> "DeviceBatches":
        return self

    def __next__(self) -> torch.Tensor:
        item = self._queue.get()
        if isinstance(item, BaseException):
            raise item
        runs, starts, state_after = item
        dev = self.store.tokens.device
        rows = starts.numel() - 1
        out = pack_rows(self.store, runs.to(dev, non_blocking=True), starts.to(dev, non_blocking=True), rows,
                        self.width)
        self._state = state_after
        return out

    def close(self) -> None:
        self._stop.set()
        self._thread.join(timeout=5)

    def state_dict(self) -> dict:
        return self._state

    def load_state_dict(self, state: dict) -> None:
        self.close()
        self.planner.load_state_dict(state)
        self._state = self.planner.state_dict()
        self._start()
