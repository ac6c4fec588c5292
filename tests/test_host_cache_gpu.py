"""Caches in pinned host memory (qsa_desc.placement: QSA_KV_HOST, QSA_IDX_HOST), as the
reference's state_config kv_host / idx_host place them (src/qwfn_state.h:31-36), on a B200.

The device reads and writes them over the bus: appends store the rows there, the pooled-key
update reads the raw keys from there, and the attention copies the selected K/V rows into shared
memory with ordinary loads (the prefill takes the query-major attention, the block-grouped one
reading the caches by TMA).  Against a twin set of device caches filled with the same tokens: the
cache bytes are equal, decode selections and outputs are bit-identical (the same arithmetic on the
same bytes), prefill selections are equal and outputs within the parity tolerance (two attention
paths), and the oracle agrees on sampled queries.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from helpers import ATTN_TOL, check_selection, rel_err
from qwfnfer_b200._abi import QSA_OK, TYPE_BF16, k_blocks, make_desc
from qwfnfer_b200.configs import fill_cache, token_inputs
from qwfnfer_b200.qsa import QsaNode, QsaState, decode_items

pytestmark = pytest.mark.gpu


def descs(**kw):
    base = dict(n_ctx=32768, top_k_blocks=64, window=128)
    return make_desc(**base, **kw), make_desc(**base)


@pytest.mark.parametrize("kv_host,idx_host", [(True, True), (True, False), (False, True)])
def test_decode_over_host_caches(kv_host, idx_host):
    dh, dd = descs(kv_host=kv_host, idx_host=idx_host)
    nh, nd = QsaNode(dh), QsaNode(dd)
    lengths = [20031, 7000]                       # the first token completes block 313 (pool update)
    host = [QsaState(dh) for _ in lengths]
    dev = [QsaState(dd) for _ in lengths]
    assert host[0].k[0].is_cuda != kv_host and host[0].idx[0].is_cuda != idx_host
    for i, n in enumerate(lengths):
        fill_cache(nh, host[i], 0, n, seed=300 + i)
        fill_cache(nd, dev[i], 0, n, seed=300 + i)
    B, KB = len(lengths), k_blocks(dd)
    q, q_idx, k, v, ki = token_inputs(dd, B, 301)
    sel_h = torch.empty(B, KB, dtype=torch.int32, device="cuda")
    sel_d = torch.empty_like(sel_h)
    out_h = nh.sparse_attn_decode(decode_items([s.layer() for s in host], lengths), B, max(lengths) + 1, q, q_idx, k, v,
                                  ki, sel_out=sel_h)
    out_d = nd.sparse_attn_decode(decode_items([s.layer() for s in dev], lengths), B, max(lengths) + 1, q, q_idx, k, v,
                                  ki, sel_out=sel_d)
    torch.cuda.synchronize()
    assert nh.check(nh.workspace("decode", B, max(lengths) + 1)) == QSA_OK
    assert torch.equal(sel_h, sel_d)
    assert torch.equal(out_h, out_d)
    for a, b, n in zip(host, dev, lengths):
        for x, y in ((a.k[0], b.k[0]), (a.v[0], b.v[0]), (a.idx[0], b.idx[0])):
            assert torch.equal(x[:n + 1].cpu(), y[:n + 1].cpu())
        assert torch.equal(a.pool[0][:(n + 1) // 64], b.pool[0][:(n + 1) // 64])


def test_prefill_over_host_caches():
    dh, dd = descs(kv_host=True, idx_host=True)
    nh, nd = QsaNode(dh), QsaNode(dd)
    n_past, T = 9000, 200
    a, b = QsaState(dh), QsaState(dd)
    fill_cache(nh, a, 0, n_past, seed=310)
    fill_cache(nd, b, 0, n_past, seed=310)
    q, q_idx, k, v, ki = token_inputs(dd, T, 311)
    KB = k_blocks(dd)
    sel_h = torch.empty(T, KB, dtype=torch.int32, device="cuda")
    sel_d = torch.empty_like(sel_h)
    out_h = nh.sparse_attn(a.layer(), n_past, q, q_idx, k, v, ki, sel_out=sel_h)
    out_d = nd.sparse_attn(b.layer(), n_past, q, q_idx, k, v, ki, sel_out=sel_d)
    torch.cuda.synchronize()
    assert torch.equal(sel_h, sel_d)
    assert rel_err(out_h.cpu().numpy(), out_d.cpu().numpy()) <= ATTN_TOL
    kc, vc = a.k[0][:n_past + T].numpy(), a.v[0][:n_past + T].numpy()
    pool = a.pool[0].cpu().numpy().view(np.uint16)
    qh = q.view(torch.int16).cpu().numpy().view(np.uint16)
    out = out_h.cpu().numpy()
    sel = sel_h.cpu().numpy()
    for t in (0, 63, 64, 150, T - 1):
        qp = n_past + t
        sc = oracle.scores(dd, pool, (qp + 1) // 64, q_idx[t].cpu().numpy())[0]
        check_selection(dd, sel[t], sc, qp)
        ref = oracle.attend(dd, kc, vc, [qp], sel[t][None], qh[t][None], q_type=TYPE_BF16)[0]
        assert rel_err(out[t], ref) <= ATTN_TOL
