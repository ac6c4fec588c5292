"""Parity at the full sizes of the benchmark's prefill and 1M-context configurations, on a B200.

  - Prefill (config 4): 8,192 new tokens on a 155,648-token q8_0 prefix (2,560 blocks once the chunk
    is appended), top-64 + 128-token window, in one chunk and in two.  About 290 queries spread over
    the chunk are checked against the oracle: selections bit-exact outside near-ties, attention within
    2e-3; the pooled keys of the 128 blocks the chunk completes within 1e-5 (f32) and 1 f16 ulp; and
    the result does not depend on the chunking.  Each CTA of the block-grouped attention here runs
    about 14 chunks of 16 entries through its Q/S double buffers and TMEM phases.
  - Decode at 1,048,576 tokens (config 5): top-128 of 16,384 blocks, unsharded and as 8- and 16-shard
    single-GPU emulations of the sequence-sharded step (16 x 131 candidates exceed the global
    selection's 2,048-key sort and take its radix path): selections equal, outputs within 2e-3, the
    unsharded output against the oracle.

The oracle reads the bytes the GPU wrote (caches copied to the host).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from helpers import ATTN_TOL, POOL_TOL, check_selection, rel_err
from qwfnfer_b200._abi import QSA_OK, TYPE_BF16, TYPE_Q8_0, k_blocks, make_desc
from qwfnfer_b200.configs import CONFIGS, fill_cache, token_inputs
from qwfnfer_b200.qsa import QsaNode, QsaState, decode_items
from qwfnfer_b200.shard import LibShardBackend, ShardedDecoder

pytestmark = pytest.mark.gpu


def _bf16_bits(q):
    return q.view(torch.int16).cpu().numpy().view(np.uint16)


def _prefill(d, n_past, T, chunks, seed):
    node, st = QsaNode(d), QsaState(d)
    fill_cache(node, st, 0, n_past, seed)
    q, q_idx, k, v, ki = token_inputs(d, T, seed + 1)
    out = torch.empty(T, d.n_head, d.head_dim, device="cuda")
    sel = torch.empty(T, k_blocks(d), dtype=torch.int32, device="cuda")
    off = 0
    for c in chunks:
        node.sparse_attn(st.layer(), n_past + off, q[off:off + c], q_idx[off:off + c], k[off:off + c],
                         v[off:off + c], ki[off:off + c], out=out[off:off + c], sel_out=sel[off:off + c])
        assert node.check(node.workspace("prefill", c, n_past + off + c)) == QSA_OK
        off += c
    torch.cuda.synchronize()
    return node, st, (q, q_idx), out, sel


def test_prefill_config4_full_size():
    cfg = CONFIGS[4]
    d = cfg.desc()
    n_past, T = cfg.n_past, cfg.prefill_T
    node, st, (q, q_idx), out, sel = _prefill(d, n_past, T, [T], 301)
    out1, sel1 = out.cpu().numpy(), sel.cpu().numpy()
    n_rows = n_past + T
    kc = st.k[0][:n_rows].cpu().numpy()
    vc = st.v[0][:n_rows].cpu().numpy()
    ic = st.idx[0][:n_rows].cpu().numpy().view(np.uint16)
    pool = st.pool[0].cpu().numpy().view(np.uint16)
    # the 128 blocks completed by the chunk: f32 values (recomputed by the same kernel the append
    # runs) within 1e-5 of the oracle, the f16 the prefill stored equal to that kernel's and within
    # 1 ulp of the oracle's
    b0, nb = n_past // d.ratio, T // d.ratio
    p32 = torch.empty(nb, d.idx_dim, device="cuda")
    before = st.pool[0][b0:b0 + nb].clone()
    node.qsa_pool_rebuild(st.layer(), nb, blk0=b0, pooled_f32=p32)
    torch.cuda.synchronize()
    assert torch.equal(before, st.pool[0][b0:b0 + nb])
    ref32, ref16 = oracle.pool_blocks(d, ic, b0, nb)
    assert np.abs(p32.cpu().numpy() - ref32).max() <= POOL_TOL
    assert np.abs(pool[b0:b0 + nb].astype(np.int32) - ref16.astype(np.int32)).max() <= 1
    # sampled queries: selection and attention against the oracle
    qh = _bf16_bits(q)
    qi = q_idx.cpu().numpy()
    samples = sorted(set(list(range(0, T, 29)) + [1, 63, 64, 65, T - 65, T - 64, T - 2, T - 1]))
    for t in samples:
        qp = n_past + t
        sc = oracle.scores(d, pool, (qp + 1) // d.ratio, qi[t])[0]
        check_selection(d, sel1[t], sc, qp)
    ref = oracle.attend(d, kc, vc, [n_past + t for t in samples], sel1[samples], qh[samples], q_type=TYPE_BF16)
    errs = [rel_err(out1[t], ref[i]) for i, t in enumerate(samples)]
    assert max(errs) <= ATTN_TOL, f"worst query {samples[int(np.argmax(errs))]}: {max(errs):.2e}"
    # the same tokens in two chunks: the same selections, outputs within the tolerance
    del node, st
    torch.cuda.empty_cache()
    _, _, _, out2, sel2 = _prefill(d, n_past, T, [3000, T - 3000], 301)
    assert np.array_equal(sel2.cpu().numpy(), sel1)
    assert rel_err(out2.cpu().numpy(), out1) <= ATTN_TOL


def _oracle_cache_rows(st, sel_row, q_pos, r, row_bytes_k, row_bytes_v):
    """Host K/V byte arrays of q_pos + 1 rows holding only the selected blocks' rows (the oracle reads
    nothing else); untouched pages of the zeroed arrays are never materialised."""
    n = q_pos + 1
    kc = np.zeros((n, row_bytes_k), np.uint8)
    vc = np.zeros((n, row_bytes_v), np.uint8)
    for b in sel_row:
        if b < 0:
            continue
        c0, c1 = b * r, min((b + 1) * r, n)
        kc[c0:c1] = st.k[0][c0:c1].cpu().numpy()
        vc[c0:c1] = st.v[0][c0:c1].cpu().numpy()
    return kc, vc


@pytest.fixture(scope="module")
def config5_unsharded():
    cfg = CONFIGS[5]
    d = cfg.desc()
    n_past = cfg.n_past
    node, st = QsaNode(d), QsaState(d)
    fill_cache(node, st, 0, n_past, 401)
    q, q_idx, k, v, ki = token_inputs(d, 1, 402)
    sel = torch.empty(1, k_blocks(d), dtype=torch.int32, device="cuda")
    out = node.sparse_attn_decode(decode_items([st.layer()], [n_past]), 1, n_past + 1, q, q_idx, k, v, ki,
                                  sel_out=sel)
    assert node.check(node.workspace("decode", 1, n_past + 1)) == QSA_OK
    res = dict(d=d, n_past=n_past, node=node, st=st, inputs=(q, q_idx, k, v, ki), out=out.cpu().numpy(),
               sel=sel.cpu().numpy())
    yield res
    del res["node"], res["st"]
    torch.cuda.empty_cache()


def test_decode_config5_full_size_against_oracle(config5_unsharded):
    c = config5_unsharded
    d, n_past, st = c["d"], c["n_past"], c["st"]
    q, q_idx, _, _, _ = c["inputs"]
    pool = st.pool[0].cpu().numpy().view(np.uint16)
    sc = oracle.scores(d, pool, (n_past + 1) // d.ratio, q_idx[0].cpu().numpy())[0]
    check_selection(d, c["sel"][0], sc, n_past)
    kc, vc = _oracle_cache_rows(st, c["sel"][0], n_past, d.ratio, st.k[0].shape[1], st.v[0].shape[1])
    ref = oracle.attend(d, kc, vc, [n_past], c["sel"][0][None], _bf16_bits(q)[0][None], q_type=TYPE_BF16)[0]
    assert rel_err(c["out"][0], ref) <= ATTN_TOL


@pytest.mark.parametrize("world", [8, 16])
def test_decode_config5_full_size_sharded_emulation(config5_unsharded, world):
    """Every emulated rank holds its contiguous 1/world of the blocks (caches filled from the same
    random stream), appends the token if it holds its cell, proposes its best blocks; the global
    selection, each rank's attention state and the merge must give the unsharded result."""
    c = config5_unsharded
    d, n_past = c["d"], c["n_past"]
    q, q_idx, k, v, ki = c["inputs"]
    node = c["node"]
    ranks = []
    for r in range(world):
        dec = ShardedDecoder(d, backend=LibShardBackend(d), rank=r, world=world)
        st = QsaState(d, blocks=dec.blocks)
        fill_cache(node, st, 0, n_past, 401, append=dec.append)
        ranks.append((dec, st))
    B, max_n_kv = 1, n_past + 1
    items = [decode_items([st.layer()], [n_past]) for _, st in ranks]
    cands = [dec.backend.candidates(it, B, max_n_kv, dec.blocks, q_idx, k, v, ki) for (dec, _), it in zip(ranks, items)]
    gathered = torch.stack(cands)
    states, sels = [], []
    for (dec, _), it in zip(ranks, items):
        sel = torch.empty((B, k_blocks(d)), dtype=torch.int32, device="cuda")
        states.append(dec.backend.attend(it, B, max_n_kv, dec.blocks, gathered, q, sel_out=sel))
        sels.append(sel)
    out = ranks[0][0].backend.merge(torch.stack(states))
    for dec, _ in ranks:
        assert dec.backend.check(B, max_n_kv) == QSA_OK
    torch.cuda.synchronize()
    for s in sels:
        assert np.array_equal(s.cpu().numpy(), c["sel"])
    assert rel_err(out.cpu().numpy(), c["out"]) <= ATTN_TOL
    # the token's row landed on the rank holding its cell, with the bytes of the unsharded append
    owner = next((dec, st) for dec, st in ranks if dec.blocks[0] * d.ratio <= n_past < dec.blocks[1] * d.ratio)
    row = n_past - owner[0].blocks[0] * d.ratio
    assert torch.equal(owner[1].k[0][row], c["st"].k[0][n_past])
    assert torch.equal(owner[1].v[0][row], c["st"].v[0][n_past])
