"""KV-sequence-sharded decode on one GPU: every shard's caches and calls on the same device, the
exchanges done by stacking (what the all-gathers deliver).  The sharded result must equal the
unsharded qsa_decode's: the same caches (bytes), the same selection (exactly), the same attention
output within the parity tolerance.  The NCCL path over real ranks is test_zz_shard_nccl.py.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import ATTN_TOL, rel_err
from qwfnfer_b200._abi import QSA_ERR_DEVICE_ARG, QSA_OK, TYPE_F16, TYPE_Q8_0, k_blocks, make_desc
from qwfnfer_b200.configs import fill_cache, token_inputs
from qwfnfer_b200.qsa import QsaNode, QsaState, decode_items
from qwfnfer_b200.shard import LibShardBackend, ShardedDecoder, shard_blocks

pytestmark = pytest.mark.gpu


def build(d, world, n_toks, seeds):
    """Unsharded caches of len(n_toks) sequences, and each emulated rank's shard of them."""
    node = QsaNode(d)
    full = [QsaState(d) for _ in n_toks]
    for st, n, s in zip(full, n_toks, seeds):
        fill_cache(node, st, 0, n, s)
    ranks = []
    for r in range(world):
        dec = ShardedDecoder(d, backend=LibShardBackend(d), rank=r, world=world)
        sts = [QsaState(d, blocks=dec.blocks) for _ in n_toks]
        for st, n, s in zip(sts, n_toks, seeds):
            fill_cache(node, st, 0, n, s, append=dec.append)
        ranks.append((dec, sts))
    return node, full, ranks


def assert_shard_caches_equal(d, full, ranks, n_rows):
    r = d.ratio
    for dec, sts in ranks:
        lo, hi = dec.blocks
        for f, s, n in zip(full, sts, n_rows):
            c0, c1 = lo * r, min(hi * r, n)
            if c1 <= c0:
                continue
            for a, b in ((f.k[0], s.k[0]), (f.v[0], s.v[0]), (f.idx[0], s.idx[0])):
                assert torch.equal(a[c0:c1], b[:c1 - c0])
            nb = min(hi, n // r)
            if nb > lo:
                assert torch.equal(f.pool[0][lo:nb], s.pool[0][:nb - lo])


def sharded_step(d, ranks, positions, max_n_kv, q, q_idx, k=None, v=None, ki=None):
    """One step through every emulated rank: returns (out, [sel of each rank])."""
    B = len(positions)
    cands, items = [], []
    for dec, sts in ranks:
        it = decode_items([s.layer() for s in sts], positions)
        items.append(it)
        cands.append(dec.backend.candidates(it, B, max_n_kv, dec.blocks, q_idx, k, v, ki))
    gathered = torch.stack(cands)
    states, sels = [], []
    for (dec, _), it in zip(ranks, items):
        sel = torch.empty((B, k_blocks(d)), dtype=torch.int32, device="cuda")
        states.append(dec.backend.attend(it, B, max_n_kv, dec.blocks, gathered, q, sel_out=sel))
        sels.append(sel)
    out = ranks[0][0].backend.merge(torch.stack(states))
    for dec, _ in ranks:
        assert dec.backend.check(B, max_n_kv) == QSA_OK
    return out, sels


@pytest.mark.parametrize("world,type_", [(2, TYPE_Q8_0), (3, TYPE_Q8_0), (4, TYPE_F16)])
def test_sharded_decode_equals_unsharded(world, type_):
    d = make_desc(n_ctx=32768, top_k_blocks=64, window=128, type_k=type_, type_v=type_)
    # sequence 0 decodes the token completing block 468 (the pooled-key update on its owner);
    # sequence 1 is short: the upper shards hold nothing of it (empty states)
    positions = [30015, 9000]
    node, full, ranks = build(d, world, positions, seeds=[21, 22])
    assert_shard_caches_equal(d, full, ranks, positions)
    q, q_idx, k, v, ki = token_inputs(d, 2, seed=23, q_dtype=torch.float32 if type_ == TYPE_F16 else torch.bfloat16)
    max_n_kv = max(positions) + 1
    sel_ref = torch.empty((2, k_blocks(d)), dtype=torch.int32, device="cuda")
    items_full = decode_items([s.layer() for s in full], positions)
    out_ref = node.sparse_attn_decode(items_full, 2, max_n_kv, q, q_idx, k, v, ki, sel_out=sel_ref)
    out, sels = sharded_step(d, ranks, positions, max_n_kv, q, q_idx, k, v, ki)
    torch.cuda.synchronize()
    for s in sels:
        assert torch.equal(s, sel_ref)
    assert rel_err(out.cpu().numpy(), out_ref.cpu().numpy()) <= ATTN_TOL
    assert_shard_caches_equal(d, full, ranks, [p + 1 for p in positions])


def test_shard_select_drops_impossible_candidates():
    """A candidate list no shard could have produced (a block past the query) is dropped and
    reported through the status word; the step still completes with the valid candidates."""
    d = make_desc(n_ctx=8192, top_k_blocks=16, window=128)
    positions = [5000]
    node, full, ranks = build(d, 2, positions, seeds=[31])
    q, q_idx, _, _, _ = token_inputs(d, 1, seed=32)
    dec, sts = ranks[0]
    it = decode_items([s.layer() for s in sts], positions)
    cands = [r[0].backend.candidates(decode_items([s.layer() for s in r[1]], positions), 1, 5001, r[0].blocks, q_idx)
             for r in ranks]
    gathered = torch.stack(cands).clone()
    gathered[1, 0, 0, 0] = 120                       # block 120 is past the query's block 78
    state = dec.backend.attend(it, 1, 5001, dec.blocks, gathered, q)
    assert dec.backend.check(1, 5001) == QSA_ERR_DEVICE_ARG
    assert not torch.isnan(state).any()


@pytest.mark.parametrize("case", ["all_equal", "tie_at_cut"])
def test_shard_select_equal_keys_by_lower_block(case):
    """Global selection from hand-made candidate lists of 2 shards whose scores tie: equal keys
    are kept by lower block (slot order), also when every key is equal."""
    d = make_desc(n_ctx=8192, top_k_blocks=16, window=128)
    pos = 5000                                        # 78 whole blocks visible; forced 76..78
    node, full, ranks = build(d, 2, [pos], seeds=[33])
    q, _, _, _, _ = token_inputs(d, 1, seed=34)
    KB = k_blocks(d)
    want = KB - 3
    lists = [list(range(0, 19)), list(range(64, 76))]  # what the two shards could send (ascending)
    f32 = lambda x: int(np.float32(x).view(np.int32))
    if case == "all_equal":
        keys = [[f32(0.5)] * 19, [f32(0.5)] * 12]
        expect = list(range(0, want))
    else:
        keys = [[f32(0.25)] * 19, [f32(1.0)] * 6 + [f32(0.25)] * 6]
        expect = list(range(0, want - 6)) + list(range(64, 70))
    expect = sorted(expect) + [76, 77, 78]
    gathered = torch.full((2, 2, 1, KB), -1, dtype=torch.int32)
    for s in range(2):
        gathered[s, 0, 0, :len(lists[s])] = torch.tensor(lists[s], dtype=torch.int32)
        gathered[s, 1, 0, :len(keys[s])] = torch.tensor(keys[s], dtype=torch.int32)
    gathered = gathered.cuda()
    for dec, sts in ranks:
        it = decode_items([s.layer() for s in sts], [pos])
        sel = torch.empty(1, KB, dtype=torch.int32, device="cuda")
        dec.backend.attend(it, 1, pos + 1, dec.blocks, gathered, q, sel_out=sel)
        assert dec.backend.check(1, pos + 1) == QSA_OK
        assert sel.cpu().numpy()[0].tolist() == expect


@pytest.mark.parametrize("world,type_", [(2, TYPE_Q8_0), (3, TYPE_F16)])
def test_sharded_decode_replicated_index_equals_unsharded(world, type_):
    """Replicated indexer caches: every emulated rank holds all raw and pooled keys (byte-equal to
    the unsharded caches) and its shard's K/V rows; each selects globally (the unsharded
    selection, exactly), attends its own blocks, and the merged states equal qsa_decode's output."""
    d = make_desc(n_ctx=32768, top_k_blocks=64, window=128, type_k=type_, type_v=type_)
    positions = [30015, 9000]
    node = QsaNode(d)
    full = [QsaState(d) for _ in positions]
    for st, n, s in zip(full, positions, [21, 22]):
        fill_cache(node, st, 0, n, s)
    ranks = []
    for r in range(world):
        dec = ShardedDecoder(d, backend=LibShardBackend(d), rank=r, world=world, index="replicated")
        sts = [QsaState(d, blocks=dec.blocks, index_full=True) for _ in positions]
        for st, n, s in zip(sts, positions, [21, 22]):
            fill_cache(node, st, 0, n, s, append=dec.append)
        ranks.append((dec, sts))
    q, q_idx, k, v, ki = token_inputs(d, 2, seed=23, q_dtype=torch.float32 if type_ == TYPE_F16 else torch.bfloat16)
    max_n_kv = max(positions) + 1
    sel_ref = torch.empty((2, k_blocks(d)), dtype=torch.int32, device="cuda")
    out_ref = node.sparse_attn_decode(decode_items([s.layer() for s in full], positions), 2, max_n_kv, q, q_idx,
                                      k, v, ki, sel_out=sel_ref)
    states, sels = [], []
    for dec, sts in ranks:
        sel = torch.empty((2, k_blocks(d)), dtype=torch.int32, device="cuda")
        states.append(dec.backend.decode_ri(decode_items([s.layer() for s in sts], positions), 2, max_n_kv,
                                            dec.blocks, q, q_idx, k, v, ki, sel_out=sel))
        sels.append(sel)
    out = ranks[0][0].backend.merge(torch.stack(states))
    torch.cuda.synchronize()
    for dec, _ in ranks:
        assert dec.backend.check(2, max_n_kv) == QSA_OK
    for s in sels:
        assert torch.equal(s, sel_ref)
    assert rel_err(out.cpu().numpy(), out_ref.cpu().numpy()) <= ATTN_TOL
    r = d.ratio
    for dec, sts in ranks:                             # caches after the step's append
        lo, hi = dec.blocks
        for f, s, n in zip(full, sts, [p + 1 for p in positions]):
            assert torch.equal(f.idx[0][:n], s.idx[0][:n])
            assert torch.equal(f.pool[0][:n // r], s.pool[0][:n // r])
            c0, c1 = lo * r, min(hi * r, n)
            if c1 > c0:
                assert torch.equal(f.k[0][c0:c1], s.k[0][:c1 - c0])
                assert torch.equal(f.v[0][c0:c1], s.v[0][:c1 - c0])
