"""KV-sequence-sharded decode on the CPU: the block split, the exactness of the two-stage
selection, the state/merge arithmetic, and the ShardedDecoder's exchange over gloo ranks.

The compute steps run on the oracle (tests/shard_oracle_backend.py); the GPU tests check the
library's kernels for the same steps against the unsharded qsa_decode.
"""
from __future__ import annotations

import os
import socket
import sys
import tempfile
from datetime import timedelta

import numpy as np
import pytest
import torch

import oracle
from helpers import rel_err
from qwfnfer_b200._abi import TYPE_F16, TYPE_Q8_0, k_blocks, make_desc
from qwfnfer_b200.shard import ShardedDecoder, shard_blocks
from shard_oracle_backend import OracleShardBackend

TESTS = os.path.dirname(os.path.abspath(__file__))


def test_shard_blocks_cover_the_cache_once():
    for n, w in [(64, 1), (64, 2), (100, 3), (16384, 8), (17, 5)]:
        ranges = [shard_blocks(n, w, g) for g in range(w)]
        assert ranges[0][0] == 0 and ranges[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
        sizes = [hi - lo for lo, hi in ranges]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_blocks(3, 4, 0)


def make_host_cache(d, n_tok, seed):
    g = np.random.default_rng(seed)
    kv_dim = d.n_head_kv * d.head_dim
    kc, vc, ic, _ = oracle.cache_arrays(d)
    K = (g.standard_normal((n_tok, kv_dim)) / 16).astype(np.float32)
    V = g.standard_normal((n_tok, kv_dim)).astype(np.float32)
    ki = (g.standard_normal((n_tok, d.idx_dim)) * 1.012).astype(np.float32)
    oracle.append(d, kc, vc, ic, 0, K, V, ki)
    nb = n_tok // d.ratio
    _, pool16 = oracle.pool_blocks(d, ic, 0, nb)
    pool = np.zeros((d.n_ctx // d.ratio, d.idx_dim), np.uint16)
    pool[:nb] = pool16
    return kc, vc, pool


@pytest.mark.parametrize("type_", [TYPE_F16, TYPE_Q8_0])
def test_merged_states_equal_attention(type_):
    """Attention over a selection = merge of the states of any partition of its blocks."""
    d = make_desc(n_ctx=4096, top_k_blocks=8, window=128, type_k=type_, type_v=type_)
    kc, vc, pool = make_host_cache(d, 4000, seed=1)
    g = np.random.default_rng(2)
    Q = g.standard_normal((3, d.n_head, d.head_dim)).astype(np.float32)
    q_pos = [3999, 2500, 700]
    KB = k_blocks(d)
    sel = np.full((3, KB), -1, np.int32)
    for t, q in enumerate(q_pos):
        blocks = sorted(g.choice((q + 1) // d.ratio + 1, size=min(KB, (q + 1) // d.ratio + 1), replace=False))
        sel[t, :len(blocks)] = blocks
    want = oracle.attend(d, kc, vc, q_pos, sel, Q)
    for n_parts in (1, 2, 3):
        parts = []
        for p in range(n_parts):
            sp = np.where(sel % n_parts == p, sel, -1)      # blocks dealt round-robin over the parts
            parts.append(oracle.attend_state(d, kc, vc, q_pos, sp, Q))
        got = oracle.merge_states(d, np.stack(parts))
        assert rel_err(got, want) < 1e-5, n_parts


@pytest.mark.parametrize("world", [1, 2, 3, 5])
@pytest.mark.parametrize("window", [0, 128])
def test_two_stage_selection_is_the_global_selection(world, window):
    """Each shard's best KB blocks, merged by (score, lower block), give the global selection --
    including the many zero-score ties (relu of a single indexer head)."""
    d = make_desc(n_ctx=8192, top_k_blocks=16, window=window, type_k=TYPE_F16, type_v=TYPE_F16)
    kc, vc, pool = make_host_cache(d, 8000, seed=3)
    g = np.random.default_rng(4)
    positions = [7999, 5000, 1023, 640, 64, 3]
    q_idx = (g.standard_normal((len(positions), d.idx_dim)) * 1.012).astype(np.float32)
    n_blocks = d.n_ctx // d.ratio
    backs = [OracleShardBackend(d, kc, vc, pool, shard_blocks(n_blocks, world, r)) for r in range(world)]
    cands = torch.stack([b.candidates(positions, len(positions), 8000, b.blocks, q_idx) for b in backs])
    sc = oracle.scores(d, pool, n_blocks, q_idx)
    n_zero = 0
    for t, q in enumerate(positions):
        want, _ = oracle.select(d, sc[t], q)
        got = backs[0].global_selection(cands.numpy(), q, t)
        assert got == [int(b) for b in want if b >= 0], (world, q)
        n_zero += int((sc[t, :(q + 1) // d.ratio] == 0).sum())
    assert n_zero > 0          # the tie rule was exercised


def _gloo_worker(rank, world, port, outdir):
    sys.path[:0] = [TESTS, os.path.dirname(TESTS)]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        d = make_desc(n_ctx=8192, top_k_blocks=16, window=128, type_k=TYPE_Q8_0, type_v=TYPE_Q8_0)
        kc, vc, pool = make_host_cache(d, 8000, seed=5)           # every rank derives the same cache
        backend = OracleShardBackend(d, kc, vc, pool, shard_blocks(d.n_ctx // d.ratio, world, rank))
        dec = ShardedDecoder(d, backend=backend, rank=rank, world=world)
        g = np.random.default_rng(6)
        positions = [7999, 4100, 900]
        B = len(positions)
        q = torch.from_numpy(g.standard_normal((B, d.n_head, d.head_dim)).astype(np.float32))
        q_idx = torch.from_numpy((g.standard_normal((B, d.idx_dim)) * 1.012).astype(np.float32))
        sel = torch.empty((B, k_blocks(d)), dtype=torch.int32)
        out = dec.step(positions, B, 8000, q, q_idx, sel_out=sel)
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), out=out.numpy(), sel=sel.numpy(),
                 blocks=np.array(dec.blocks))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2])
def test_sharded_decoder_over_gloo_matches_the_unsharded_node(world):
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as outdir:
        mp.start_processes(_gloo_worker, args=(world, _free_port(), outdir), nprocs=world, join=True,
                           start_method="spawn")
        res = [np.load(os.path.join(outdir, f"rank{r}.npz")) for r in range(world)]
    d = make_desc(n_ctx=8192, top_k_blocks=16, window=128, type_k=TYPE_Q8_0, type_v=TYPE_Q8_0)
    kc, vc, pool = make_host_cache(d, 8000, seed=5)
    g = np.random.default_rng(6)
    positions = [7999, 4100, 900]
    Q = g.standard_normal((3, d.n_head, d.head_dim)).astype(np.float32)
    q_idx = (g.standard_normal((3, d.idx_dim)) * 1.012).astype(np.float32)
    out, sel, _ = oracle.node(d, kc, vc, pool, positions, Q, q_idx)
    assert [tuple(r["blocks"]) for r in res] == [shard_blocks(d.n_ctx // d.ratio, world, i) for i in range(world)]
    for r in res:                                        # every rank ends with the same result
        assert np.array_equal(r["sel"], sel)
        assert rel_err(r["out"], out) < 1e-5
