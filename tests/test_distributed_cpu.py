"""Data-parallel host logic with real process groups on CPU (gloo, world size 2):
the bucketed gradient reducer averages exactly, issues the same collectives in
the same order on every rank, honours the no-all-reduce rule for non-final
accumulation micro-steps, and a rank that dies before its collective makes the
survivor's collective fail with an error after the process-group timeout
instead of hanging."""
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _FakeFlat:
    def __init__(self, n, rank):
        g = torch.Generator().manual_seed(100 + rank)
        self.g32 = torch.randn(n, generator=g)


# flat layout: [embed 0:4096) [layer0 4096:10240) [layer1 10240:16384) [norm 16384:16448)
_RANGES = [(16384, 16448), (10240, 16384), (4096, 10240), (0, 4096)]


def _reducer_worker(rank, world, port, out_q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from midstream_llm_b200.distributed import GradReducer
        flat = _FakeFlat(16448, rank)
        expect = sum(_FakeFlat(16448, r).g32 for r in range(world)) / world
        red = GradReducer(bucket_bytes=3000 * 4)
        red.begin(flat)
        for lo, hi in _RANGES:
            red.ready(lo, hi)
        red.finish()
        ok = torch.allclose(flat.g32, expect, rtol=1e-6, atol=1e-7)
        launched = list(red.launched)
        covered = sorted(launched)
        contiguous = covered[0][0] == 0 and covered[-1][1] == 16448 and all(
            a[1] == b[0] for a, b in zip(covered, covered[1:]))
        sizes_ok = all(hi - lo <= 3000 for lo, hi in launched[:-1])
        gathered = [None] * world
        dist.all_gather_object(gathered, launched)
        same_order = all(g == gathered[0] for g in gathered)
        # Non-final accumulation micro-step: no collective, gradients untouched.
        flat2 = _FakeFlat(16448, rank)
        before = flat2.g32.clone()
        red.enabled = False
        red.begin(flat2)
        for lo, hi in _RANGES:
            red.ready(lo, hi)
        red.finish()
        untouched = torch.equal(flat2.g32, before) and red.launched == []
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, ok, contiguous, sizes_ok, same_order, untouched, len(launched)))
    except Exception:
        out_q.put((rank, "error", traceback.format_exc()))


def test_grad_reducer_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_reducer_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for r in results:
        assert r[1] != "error", r[2]
        rank, ok, contiguous, sizes_ok, same_order, untouched, n = r
        assert ok and contiguous and sizes_ok and same_order and untouched, r
        assert n >= 6  # 16448 elements in buckets of <= 3000


class _FakeFlatN:
    def __init__(self, n, rank):
        g = torch.Generator().manual_seed(100 + rank)
        self.g32 = torch.randn(n, generator=g)
        self.numel = n


def _sharded_worker(rank, world, port, out_q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from midstream_llm_b200.distributed import GradReducer
        n = 16448  # a bucket (3000 elements) straddles the shard boundary at 8224
        flat = _FakeFlatN(n, rank)
        total = sum(_FakeFlatN(n, r).g32 for r in range(world))
        red = GradReducer(bucket_bytes=3000 * 4, shard_optimizer=True)
        red.begin(flat)
        for lo, hi in _RANGES:
            red.ready(lo, hi)
        red.finish()
        lo, hi = red.shard_range(flat)
        ok = torch.allclose(flat.g32[lo:hi], total[lo:hi], rtol=1e-6, atol=1e-6)
        pieces = red.pieces(7000, 10000, n)
        split_ok = pieces == [(0, 7000, 8224), (1, 8224, 10000)]
        covered = sorted(red.launched)
        full = covered[0][0] == 0 and covered[-1][1] == n
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, ok, split_ok, full, (lo, hi), red.collectives))
    except Exception:
        out_q.put((rank, "error", traceback.format_exc()))


def test_sharded_reducer_gloo_two_ranks():
    """The sharded update's gradient exchange: every bucket is cut at the shard boundary and each piece is
    reduced (summed) to the rank that owns it; each rank then holds the exact sum on its own shard."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sharded_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    shards = set()
    for r in results:
        assert r[1] != "error", r[2]
        rank, ok, split_ok, full, rng, collectives = r
        assert ok and split_ok and full, r
        assert collectives > len(_RANGES)  # straddling buckets became two reductions
        shards.add(rng)
    assert shards == {(0, 8224), (8224, 16448)}


class _FakeFlatP:
    def __init__(self, n, rank, idx):
        g = torch.Generator().manual_seed(200 + rank)
        self.p32 = torch.randn(n, generator=g)
        self.numel = n
        self.f32_read_index = idx


def _sync_worker(rank, world, port, out_q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from midstream_llm_b200.distributed import GradReducer
        n = 16448
        # three fp32-read ranges: inside shard 0, straddling the boundary at 8224, inside shard 1
        idx = torch.cat([torch.arange(100, 356), torch.arange(8000, 8512), torch.arange(12000, 12100)])
        flat = _FakeFlatP(n, rank, idx)
        before = flat.p32.clone()
        owners = [_FakeFlatP(n, r, idx).p32 for r in range(world)]
        red = GradReducer(shard_optimizer=True)
        red.sync_f32_params(flat)
        size = red.shard_size(n)
        want = torch.stack([owners[int(i) // size][int(i)] for i in idx])
        ok_idx = torch.equal(flat.p32[idx], want)
        mask = torch.ones(n, dtype=torch.bool)
        mask[idx] = False
        ok_rest = torch.equal(flat.p32[mask], before[mask])
        dist.barrier()
        dist.destroy_process_group()
        out_q.put((rank, ok_idx, ok_rest))
    except Exception:
        out_q.put((rank, "error", traceback.format_exc()))


def test_sharded_update_shares_fp32_norm_parameters_gloo():
    """After a sharded update each rank holds new master weights on its own shard only; the parameters the
    kernels read in fp32 (norm gains and biases) must then carry their owner's value on every rank, including
    a range that straddles the shard boundary, while everything else stays as it was."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sync_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for r in results:
        assert r[1] != "error", r[2]
        assert r[1] and r[2], r


def _dead_rank_worker(rank, world, port, out_q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        out_q.put((rank, "left"))
        out_q.close()
        out_q.join_thread()  # flush the message before leaving
        os._exit(0)  # leaves between steps, with no collective in flight
    t = torch.ones(8)
    try:
        dist.all_reduce(t)
        out_q.put((rank, "completed"))
    except Exception as exc:  # the survivor learns of it from the timeout
        out_q.put((rank, "error:" + type(exc).__name__))


def test_dead_rank_surfaces_as_error_not_hang():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=90) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert results[1] == "left"
    assert results[0].startswith("error:"), results
