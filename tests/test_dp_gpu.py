"""Data-parallel gradients on 2+ GPUs (NCCL, bucketed all-reduce during backward)
equal one process accumulating every rank's micro-batch with loss / world
(the DP oracle), within fp16 tolerance; a grad-accum-2 update all-reduces only
on its last micro-step; after the updates every rank holds bit-identical
parameters. The sharded (ZeRO-1-style) update matches the replicated one: the
gradients of each rank's own shard, the fp16 weights on every rank, and the
master weights and moments once gathered."""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_dp_matches_single_process_accumulation(tmp_path):
    world = min(torch.cuda.device_count(), 8)
    out = tmp_path / "dp.json"
    env = dict(os.environ, DP_TEST_OUT=str(out), NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_port()}",
           str(ROOT / "tests" / "dp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["world"] == world
    assert res["max_rel_err"] < 2e-3, res["errs"]
    assert res["params_agree"]
    assert res["buckets"] > 1
    assert res["accum_collectives"] == res["buckets"]  # the non-final micro-step issued none
    sh = res["sharded"]
    assert sh["shard_grad_err"] < 1e-6, sh  # reduce-to-owner sums equal the all-reduce on the own shard
    assert sh["f16_equal_ranks"], sh
    assert sh["f16_err"] < 1e-3 and sh["p32_err"] < 1e-6 and sh["m_err"] < 1e-5, sh
    assert abs(sh["grad_norm"][0] - sh["grad_norm"][1]) <= 1e-5 * sh["grad_norm"][1], sh
    # norm gains (read in fp32 by the kernels) carry the owner's update on every rank
    assert sh["norm_equal_ranks"] and sh["norm_err"] < 1e-6, sh
    assert abs(sh["loss2"][0] - sh["loss2"][1]) <= 2e-5 * abs(sh["loss2"][1]), sh
