"""The sharded decode over real ranks: one process per GPU, exchanges by NCCL all-gathers or by
libqsa's all-gather over NVLink peer memory, the indexer caches sharded or replicated (2 GPUs or
more).

Runs tests/shard_nccl_worker.py under torch.distributed.run on min(4, visible GPUs) ranks and
requires its SHARD_NCCL line to report ok (selections identical to the unsharded qsa_decode on
every rank, outputs within the parity tolerance and identical across ranks, clean status).
"""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

TESTS = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(n, exchange, index, delay=""):
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes", "1",
           "--nproc-per-node", str(n), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(TESTS, "shard_nccl_worker.py"), exchange, index] + ([delay] if delay else [])
    r = subprocess.run(cmd, capture_output=True, text=True, env=dict(os.environ, NCCL_NVLS_ENABLE="0"))
    lines = [l for l in r.stdout.splitlines() if l.startswith("SHARD_NCCL ")]
    assert r.returncode == 0 and lines, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(lines[-1][len("SHARD_NCCL "):])
    assert res["ok"] and res["world"] == n, res


@pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")
@pytest.mark.parametrize("index", ["sharded", "replicated"])
def test_sharded_decode_c_entry_one_rank(index):
    """qsa_decode_sharded (the step with its NCCL all-gathers behind the C ABI) on a one-rank
    communicator: the same selection as qsa_decode and the output within the parity tolerance."""
    _run(1, "nccl_capi", index)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange,index,delay", [("nccl", "sharded", ""), ("peer", "sharded", ""),
                                                 ("peer", "replicated", ""), ("peer", "replicated", "delay"),
                                                 ("peer", "sharded", "delay"), ("nccl_capi", "sharded", ""),
                                                 ("nccl_capi", "replicated", "")])
def test_sharded_decode_over_ranks(exchange, index, delay):
    """`delay`: three steps back to back, the last rank's host sleeping between each peer push and
    its wait (later rounds published before its wait launches).  nccl_capi: qsa_decode_sharded with
    the process group's communicator."""
    n = min(4, torch.cuda.device_count())
    _run(n, exchange, index, delay)
