"""Data-parallel runtime: launch environment, runtime plan, and the bucketed
gradient all-reduce that overlaps the decoder's backward.

Launch / plan semantics follow Midstream-LLM src/jishui/distributed.py:35-67
(`LaunchEnvironment.from_environ`: RANK/LOCAL_RANK/WORLD_SIZE all or
nothing), :302-349 (`build_runtime_plan`: cuda -> nccl on cuda:LOCAL_RANK,
cpu -> gloo, one accelerator type per job) and :371-409
(`initialize_runtime`: bind the device, init the process group from env://).
The reference has no gradient exchange; the rules it documents for one
(docs/torch-distributed.md:62-67: rank-seeded samplers, no all-reduce on
non-final accumulation micro-steps, rank-0 checkpoints then a barrier) are
what `GradReducer` and the trainer implement.
"""
from __future__ import annotations

import os
from dataclasses import asdict, dataclass
from typing import Mapping

import torch
import torch.distributed as dist


class DistributedCapabilityError(RuntimeError):
    """The requested process topology cannot run here."""


# torchrun exports these three together; each maps to one LaunchEnvironment field.
_TORCHRUN_VARS = {"RANK": "rank", "LOCAL_RANK": "local_rank", "WORLD_SIZE": "world_size"}


@dataclass(frozen=True)
class LaunchEnvironment:
    """This process's place in the job. A single process (no torchrun variables) is rank 0 of 1."""
    rank: int = 0
    local_rank: int = 0
    world_size: int = 1

    def __post_init__(self) -> None:
        if self.world_size < 1:
            raise DistributedCapabilityError(f"WORLD_SIZE must be at least 1 (got {self.world_size})")
        if self.rank < 0 or self.rank >= self.world_size:
            raise DistributedCapabilityError(f"RANK {self.rank} is outside [0, {self.world_size})")
        if self.local_rank < 0:
            raise DistributedCapabilityError(f"LOCAL_RANK must not be negative (got {self.local_rank})")

    @classmethod
    def from_environ(cls, environ: Mapping[str, str] | None = None) -> "LaunchEnvironment":
        """Reads RANK / LOCAL_RANK / WORLD_SIZE: all three or none of them must be set."""
        source = os.environ if environ is None else environ
        found = {var: source[var] for var in _TORCHRUN_VARS if var in source}
        if not found:
            return cls()
        absent = [var for var in _TORCHRUN_VARS if var not in found]
        if absent:
            raise DistributedCapabilityError(f"incomplete torchrun environment: {', '.join(absent)} not set")
        fields = {}
        for var, text in found.items():
            try:
                fields[_TORCHRUN_VARS[var]] = int(text)
            except ValueError:
                raise DistributedCapabilityError(f"{var}={text!r} is not an integer") from None
        return cls(**fields)


@dataclass(frozen=True)
class RuntimePlan:
    accelerator: str
    device: str
    process_group_backend: str | None
    rank: int
    local_rank: int
    world_size: int

    @property
    def distributed(self) -> bool:
        return self.world_size > 1

    def to_dict(self) -> dict:
        d = asdict(self)
        d["distributed"] = self.distributed
        return d


def build_runtime_plan(accelerators, launch: LaunchEnvironment | None = None) -> RuntimePlan:
    """cuda -> NCCL on cuda:LOCAL_RANK; cpu -> gloo. Mixed accelerators are rejected."""
    launch = launch or LaunchEnvironment()
    items = accelerators.split(",") if isinstance(accelerators, str) else list(accelerators)
    requested = tuple(dict.fromkeys(a.strip().lower() for a in items if a.strip()))
    if requested == ("auto",):
        requested = ("cuda" if torch.cuda.is_available() else "cpu",)
    if len(requested) != 1:
        raise DistributedCapabilityError(
            f"one DDP process group cannot mix accelerator types ({', '.join(requested)}); use a homogeneous job")
    acc = requested[0]
    if acc not in {"cuda", "cpu"}:
        raise DistributedCapabilityError(f"accelerator {acc!r} is not supported by the B200 build (cuda or cpu)")
    return RuntimePlan(accelerator=acc, device=f"cuda:{launch.local_rank}" if acc == "cuda" else "cpu",
                       process_group_backend="nccl" if acc == "cuda" else "gloo", rank=launch.rank,
                       local_rank=launch.local_rank, world_size=launch.world_size)


@dataclass
class RuntimeContext:
    plan: RuntimePlan
    torch_device: torch.device
    created_process_group: bool

    def close(self) -> None:
        if self.created_process_group and dist.is_initialized():
            dist.destroy_process_group()
        self.created_process_group = False

    def __enter__(self) -> "RuntimeContext":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


def initialize_runtime(plan: RuntimePlan, timeout_s: float | None = None) -> RuntimeContext:
    """Binds the local device and (for world_size > 1) creates the process group."""
    if plan.accelerator == "cuda":
        if not torch.cuda.is_available():
            raise DistributedCapabilityError("cuda runtime is unavailable")
        if plan.local_rank >= torch.cuda.device_count():
            raise DistributedCapabilityError(
                f"LOCAL_RANK={plan.local_rank} exceeds the {torch.cuda.device_count()} visible cuda device(s)")
        torch.cuda.set_device(plan.local_rank)
    created = False
    if plan.distributed:
        if dist.is_initialized():
            raise DistributedCapabilityError("a torch process group is already initialized")
        kwargs = {}
        if timeout_s is not None:
            import datetime
            kwargs["timeout"] = datetime.timedelta(seconds=timeout_s)
        if plan.accelerator == "cuda":
            kwargs["device_id"] = torch.device(plan.device)
        dist.init_process_group(backend=plan.process_group_backend, init_method="env://", rank=plan.rank,
                                world_size=plan.world_size, **kwargs)
        created = True
    return RuntimeContext(plan=plan, torch_device=torch.device(plan.device), created_process_group=created)


class GradReducer:
    """Reduces the flat fp32 gradient buffer across ranks while backward runs.

    The decoder's backward calls `ready(lo, hi)` each time a contiguous range
    of the flat gradient buffer is final (the final norm, then each layer from
    the last to the first, then the tied embedding). Ranges are merged into
    buckets of about `bucket_bytes`, each launched asynchronously on NCCL's
    stream as soon as it fills, so communication of layer l overlaps the
    backward of layers l-1..0. `finish()` makes the compute stream wait for
    every outstanding bucket. Set `enabled = False` for non-final
    gradient-accumulation micro-steps.

    Two modes:
      * replicated (default): every bucket is all-reduced (AVG); every rank then
        holds the mean gradient and runs the whole optimizer update;
      * sharded (`shard_optimizer=True`, a ZeRO-1-style update): the flat buffer
        is split into `world_size` equal contiguous shards; each bucket piece is
        reduced (SUM) to the rank that owns it, which is about half an
        all-reduce's traffic. GradScaler.unscale_ folds the 1/world_size of the
        mean into its unscale pass over the local shard and all-reduces only
        its partial sums of squares and the inf flag; AdamW updates the local
        shard and all-gathers the fp16 weights in place, and the fp32 values the
        kernels read (norm gains and biases) are shared by `sync_f32_params`.
        Otherwise each rank's fp32 master weights and moments are current on its
        own shard only:
        `gather_full_state(optimizer)` (a collective: every rank calls it)
        makes them whole again, e.g. before rank 0 writes a checkpoint.
    """

    def __init__(self, group=None, bucket_bytes: int = 25 * 1024 * 1024, sm_reserve: int = 0,
                 shard_optimizer: bool = False):
        self.group = group
        # SMs the persistent GEMM / attention kernels leave to NCCL while buckets are in flight.
        self.sm_reserve = int(sm_reserve)
        self._reserving = False
        self.shard_optimizer = bool(shard_optimizer)
        self.bucket_elems = max(1, bucket_bytes // 4)
        self.enabled = True
        self._works: list = []
        self._lo = self._hi = None
        self._flat = None
        self.launched: list[tuple[int, int]] = []
        self.collectives = 0  # gradient collectives issued over this reducer's lifetime
        # When a list, finish() appends (start, end) CUDA events on the compute stream around its wait for
        # the outstanding buckets: end - start is the communication time the backward did not hide.
        self.exposed_events: list | None = None

    # ---- sharding ---------------------------------------------------------
    def sharded(self) -> bool:
        return self.shard_optimizer and self.world_size() > 1

    def shard_size(self, numel: int) -> int:
        n = self.world_size()
        if numel % n:
            raise ValueError(f"flat buffer of {numel} elements does not split into {n} equal shards")
        return numel // n

    def shard_range(self, flat) -> tuple[int, int]:
        """[lo, hi) of the flat buffers that this rank updates."""
        size = self.shard_size(flat.numel)
        r = dist.get_rank(self.group)
        return r * size, (r + 1) * size

    def pieces(self, lo: int, hi: int, numel: int) -> list[tuple[int, int, int]]:
        """[lo, hi) cut at shard boundaries: (owner rank in the group, start, end) per piece."""
        size = self.shard_size(numel)
        out = []
        a = lo
        while a < hi:
            owner = a // size
            b = min(hi, (owner + 1) * size)
            out.append((owner, a, b))
            a = b
        return out

    def reduce_stats(self, partial: torch.Tensor, found_inf: torch.Tensor) -> None:
        """Sums the shards' partial sums of squares and inf flags across ranks (stream-ordered)."""
        dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
        dist.all_reduce(found_inf, op=dist.ReduceOp.SUM, group=self.group)

    def gather_f16(self, flat) -> None:
        """All ranks' updated fp16 shards into every rank's fp16 weight copy (in place)."""
        lo, hi = self.shard_range(flat)
        dist.all_gather_into_tensor(flat.p16, flat.p16[lo:hi], group=self.group)

    def sync_f32_params(self, flat) -> None:
        """After a sharded update: the parameters the kernels read in fp32 (norm gains and biases,
        `flat.f32_read_index`) get their owner's new value on every rank. Each rank contributes the
        elements of its own shard and zeros elsewhere; the sum is exact (one non-zero per element)."""
        idx = getattr(flat, "f32_read_index", None)
        if idx is None or idx.numel() == 0:
            return
        lo, hi = self.shard_range(flat)
        vals = flat.p32.index_select(0, idx)
        vals = torch.where((idx >= lo) & (idx < hi), vals, torch.zeros_like(vals))
        dist.all_reduce(vals, op=dist.ReduceOp.SUM, group=self.group)
        flat.p32.index_copy_(0, idx, vals)

    def gather_full_state(self, optimizer=None) -> None:
        """Makes the fp32 master weights (and the optimizer's moments) whole on every rank. A collective."""
        flat = self._flat if optimizer is None else optimizer._ensure_state()
        if not self.sharded() or flat is None:
            return
        lo, hi = self.shard_range(flat)
        bufs = [flat.p32]
        if optimizer is not None and optimizer._m is not None:
            bufs += [optimizer._m, optimizer._v]
        for b in bufs:
            dist.all_gather_into_tensor(b, b[lo:hi].clone(), group=self.group)
        flat.mark_f16_current()

    def world_size(self) -> int:
        return dist.get_world_size(self.group) if dist.is_initialized() else 1

    def begin(self, flat) -> None:
        self._flat = flat
        self._works.clear()
        self._lo = self._hi = None
        self.launched = []

    def _set_reserve(self, on: bool) -> None:
        if self.sm_reserve and on != self._reserving and self._flat is not None and self._flat.g32.is_cuda:
            from . import _lib
            _lib.call("jx_set_sm_reserve", self.sm_reserve if on else 0)
            self._reserving = on

    def _launch(self, lo: int, hi: int) -> None:
        self._set_reserve(True)
        if self.sharded():
            for owner, a, b in self.pieces(lo, hi, self._flat.numel):
                dst = owner if self.group is None else dist.get_global_rank(self.group, owner)
                work = dist.reduce(self._flat.g32[a:b], dst=dst, op=dist.ReduceOp.SUM, group=self.group,
                                   async_op=True)
                self._works.append((work, None, None))
                self.collectives += 1
            self.launched.append((lo, hi))
            return
        view = self._flat.g32[lo:hi]
        op = dist.ReduceOp.AVG if dist.get_backend(self.group) == "nccl" else dist.ReduceOp.SUM
        work = dist.all_reduce(view, op=op, group=self.group, async_op=True)
        self._works.append((work, view, op))
        self.launched.append((lo, hi))
        self.collectives += 1

    def ready(self, lo: int, hi: int) -> None:
        if not self.enabled or self.world_size() == 1:
            return
        if self._lo is None:
            self._lo, self._hi = lo, hi
        elif hi == self._lo:
            self._lo = lo
        else:  # not adjacent: flush what we have and start a new span
            self._launch(self._lo, self._hi)
            self._lo, self._hi = lo, hi
        while self._hi - self._lo >= self.bucket_elems:
            self._launch(self._hi - self.bucket_elems, self._hi)
            self._hi -= self.bucket_elems

    def finish(self) -> None:
        if not self.enabled or self.world_size() == 1:
            return
        if self._lo is not None and self._hi > self._lo:
            self._launch(self._lo, self._hi)
        self._lo = self._hi = None
        ws = self.world_size()
        start = end = None
        if self.exposed_events is not None and self._works and torch.cuda.is_available() and self._flat.g32.is_cuda:
            start = torch.cuda.Event(enable_timing=True)
            start.record()
        for work, view, op in self._works:
            work.wait()
            if op == dist.ReduceOp.SUM:
                view.div_(ws)
        if start is not None:
            end = torch.cuda.Event(enable_timing=True)
            end.record()
            self.exposed_events.append((start, end))
        self._works.clear()
        self._set_reserve(False)
