"""The decode selection on a B200 against the oracle, exactly (no near-tie allowance).

The scores are exact functions of the pooled keys (f16 x f16 products are exact in f32, summed in
double, rounded once), so the GPU and the oracle score every block identically and the selected
lists must be equal entry for entry, ties included (ties go to the lower block).  The pooled keys
are written directly (the selection reads nothing else), so contexts of any length are cheap:
  - random keys from 70 to 33,000 blocks (1 to 16 selecting warps, one to several rounds of
    candidates per warp, passes that read four keys per thread ahead beyond 4,096 candidates);
  - 128 to 512 blocks kept, up to 36,000 blocks (close to the 160 KB of scores one CTA holds);
  - every score equal (equal keys; all-zero keys), a few distinct scores (ties at the cut), fewer
    positive scores than wanted (the cut falls among the zeros), a cut inside one f32 exponent.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
from helpers import forced_blocks
from qwfnfer_b200._abi import QSA_OK, QsaLayerCache, check, k_blocks, lib, make_desc
from qwfnfer_b200.qsa import QsaNode, decode_items

pytestmark = pytest.mark.gpu


def _select(d, pool: torch.Tensor, q_pos: int, q_idx: torch.Tensor) -> np.ndarray:
    node = QsaNode(d)
    c = QsaLayerCache()
    c.pool = pool.data_ptr()
    c.k = c.v = c.idx = pool.data_ptr()         # never read by the selection
    items = decode_items([c], [q_pos])
    ws = node.workspace("decode", 1, q_pos + 1)
    sel = torch.full((1, k_blocks(d)), -7, dtype=torch.int32, device="cuda")
    check(lib().qsa_decode_select(ctypes.byref(d), items.data_ptr(), 1, q_pos + 1, q_idx.data_ptr(), sel.data_ptr(),
                                  ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream), "select")
    assert node.check(ws) == QSA_OK
    torch.cuda.synchronize()
    return sel.cpu().numpy()[0]


def _run(n_blocks: int, pool_rows: np.ndarray, top_k: int = 64, seed: int = 0, q_idx: np.ndarray | None = None):
    """Select for the query whose position completes block n_blocks - 1 (all n_blocks visible)."""
    n_ctx = max(8192, 64 * (n_blocks + 2))
    d = make_desc(n_ctx=n_ctx, top_k_blocks=top_k, window=128)
    pool = torch.zeros(n_ctx // 64, d.idx_dim, dtype=torch.int16, device="cuda")
    pool[:n_blocks] = torch.from_numpy(pool_rows.view(np.int16)).cuda()
    if q_idx is None:
        q_idx = np.random.default_rng(seed).normal(0, 1.0, d.idx_dim).astype(np.float32)
    q_pos = 64 * n_blocks - 1
    assert min(forced_blocks(d, q_pos)) == n_blocks - 3
    got = _select(d, pool, q_pos, torch.from_numpy(q_idx.reshape(1, 1, -1)).cuda())
    sc = oracle.scores(d, pool_rows.view(np.uint16), n_blocks, q_idx)[0]
    want, _ = oracle.select(d, sc, q_pos)
    assert np.array_equal(got, want), (
        f"n_blocks={n_blocks}: gpu-only {sorted(set(got) - set(want))[:20]} "
        f"oracle-only {sorted(set(want) - set(got))[:20]}")
    return sc, got


def _f16(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, np.float32).astype(np.float16))


@pytest.mark.parametrize("n_blocks", [70, 900, 1900, 2560, 4000, 8100, 8192, 16384, 20000, 33000])
def test_random_keys_every_layout(n_blocks):
    rng = np.random.default_rng(n_blocks)
    rows = _f16(rng.normal(0, 1.012 / 8, (n_blocks, 128)))
    _run(n_blocks, rows, seed=n_blocks)


@pytest.mark.parametrize("top_k,n_blocks", [(128, 16384), (256, 20000), (512, 36000), (512, 30000)])
def test_wider_selections(top_k, n_blocks):
    """More blocks kept, over long contexts: a cut bin larger than the collected list at the first
    digits, ranks from a deeper level."""
    rng = np.random.default_rng(top_k + n_blocks)
    rows = _f16(rng.normal(0, 1.012 / 8, (n_blocks, 128)))
    _run(n_blocks, rows, top_k=top_k, seed=top_k)


@pytest.mark.parametrize("n_blocks", [500, 2560, 20000])
def test_all_scores_equal(n_blocks):
    """Equal positive scores, then all-zero scores: the lowest blocks are kept."""
    rng = np.random.default_rng(1)
    row = _f16(rng.normal(0, 0.2, 128))
    q = (row.astype(np.float32) * 3).astype(np.float32)            # positive dot product
    n_cand = n_blocks - 3                                          # the last three blocks are forced
    for rows, q_idx in ((np.tile(row, (n_blocks, 1)), q), (np.zeros((n_blocks, 128), np.float16), None)):
        sc, got = _run(n_blocks, rows, q_idx=q_idx)
        assert np.all(sc[:n_cand] == sc[0])
        kept = [int(b) for b in got if 0 <= b < n_cand]
        assert kept == list(range(min(64, n_cand)))
    assert sc[0] == 0


@pytest.mark.parametrize("n_blocks,n_distinct", [(2560, 3), (2560, 40), (16384, 5)])
def test_few_distinct_scores(n_blocks, n_distinct):
    """Blocks drawn from a few key vectors: the cut falls inside a run of equal scores."""
    rng = np.random.default_rng(n_distinct)
    protos = _f16(rng.normal(0, 0.3, (n_distinct, 128)))
    rows = protos[rng.integers(0, n_distinct, n_blocks)]
    _run(n_blocks, rows, seed=7)


def test_fewer_positive_scores_than_wanted():
    """30 blocks with positive scores, the rest relu-cut to zero: all 30 kept, then the lowest
    zero-score blocks."""
    n_blocks = 3000
    rng = np.random.default_rng(3)
    q = np.abs(rng.normal(0, 1, 128)).astype(np.float32)
    rows = -np.abs(rng.normal(0, 0.1, (n_blocks, 128)))
    pos = rng.choice(n_blocks - 3, 30, replace=False)
    rows[pos] = np.abs(rows[pos])
    sc, got = _run(n_blocks, _f16(rows), q_idx=q)
    assert int((sc[:n_blocks - 3] > 0).sum()) == 30
    assert set(pos.tolist()) <= set(got.tolist())


def test_cut_inside_one_exponent():
    """Every score in [1, 2): the first digit (the exponent) separates nothing."""
    n_blocks = 4000
    rng = np.random.default_rng(5)
    q = np.zeros(128, np.float32)
    q[0] = 1.0
    rows = np.zeros((n_blocks, 128), np.float32)
    rows[:, 0] = rng.uniform(1.0, 1.99, n_blocks)
    sc, _ = _run(n_blocks, _f16(rows), q_idx=q)
    assert np.all((sc[:n_blocks - 3] >= 1) & (sc[:n_blocks - 3] < 2))


def test_batch_of_long_queries():
    """Eight queries at different positions over one long cache: the batch's scoring grid (18
    CTAs of 448 blocks per query, in one wave) and eight selecting CTAs; each query's selection
    equals the oracle's."""
    n_blocks, B = 9000, 8
    rng = np.random.default_rng(11)
    rows = _f16(rng.normal(0, 1.012 / 8, (n_blocks, 128)))
    n_ctx = 64 * (n_blocks + 2)
    d = make_desc(n_ctx=n_ctx, top_k_blocks=64, window=128)
    pool = torch.zeros(n_ctx // 64, d.idx_dim, dtype=torch.int16, device="cuda")
    pool[:n_blocks] = torch.from_numpy(rows.view(np.int16)).cuda()
    positions = [64 * (n_blocks - 37 * i) - 1 for i in range(B)]
    q_idx = rng.normal(0, 1.0, (B, 1, d.idx_dim)).astype(np.float32)
    node = QsaNode(d)
    c = QsaLayerCache()
    c.pool = pool.data_ptr()
    c.k = c.v = c.idx = pool.data_ptr()
    items = decode_items([c] * B, positions)
    max_n_kv = max(positions) + 1
    ws = node.workspace("decode", B, max_n_kv)
    sel = torch.full((B, k_blocks(d)), -7, dtype=torch.int32, device="cuda")
    qd = torch.from_numpy(q_idx).cuda()
    check(lib().qsa_decode_select(ctypes.byref(d), items.data_ptr(), B, max_n_kv, qd.data_ptr(), sel.data_ptr(),
                                  ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream), "select")
    assert node.check(ws) == QSA_OK
    got = sel.cpu().numpy()
    for i, q_pos in enumerate(positions):
        nb = (q_pos + 1) // 64
        sc = oracle.scores(d, rows[:nb].view(np.uint16), nb, q_idx[i, 0])[0]
        want, _ = oracle.select(d, sc, q_pos)
        assert np.array_equal(got[i], want), f"query {i}"
