"""qsa_decode_noalloc: the decode entry point for callers that cannot allocate device memory.

An operator running inside another framework's planned graph, or a serving loop with a fixed
memory budget, cannot hand the library a workspace; this entry point keeps its scratch in a fixed
device array inside libqsa.so.  The tests call it through the C ABI and check that it gives the
workspace entry point's results (same selections, attention within the parity tolerance):
  - on two calls in a row, then on a call with another batch size (the scratch layout moves);
  - with the token's K/V/raw-key rows appended by the call, twice in a row (the cache bytes too);
  - on a call whose workspace is exactly the 8 MiB maximum, without sel_out; one past it is refused.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import ATTN_TOL, rel_err
from qwfnfer_b200._abi import QSA_OK, TYPE_BF16, TYPE_Q8_0, k_blocks, lib, make_desc
from qwfnfer_b200.configs import fill_cache, token_inputs
from qwfnfer_b200.qsa import QsaNode, QsaState, decode_items

pytestmark = pytest.mark.gpu

SCRATCH_MAX = 8 << 20          # the library's fixed scratch array


def _p(t):
    return None if t is None else t.data_ptr()


def noalloc_decode(d, items, batch, max_n_kv, q, q_idx, out, sel, k=None, v=None, ki=None):
    return lib().qsa_decode_noalloc(ctypes.byref(d), items.data_ptr(), batch, max_n_kv, q.data_ptr(), TYPE_BF16,
                                    q_idx.data_ptr(), _p(k), _p(v), _p(ki), out.data_ptr(), _p(sel),
                                    torch.cuda.current_stream().cuda_stream)


def test_noalloc_decode_matches_workspace_decode():
    d = make_desc(n_ctx=32768, top_k_blocks=64, window=128, type_k=TYPE_Q8_0, type_v=TYPE_Q8_0)
    node, st = QsaNode(d), QsaState(d)
    n_tok = 30000
    fill_cache(node, st, 0, n_tok, seed=5)
    KB = k_blocks(d)
    cases = [([29999], 11), ([29000], 12), ([29999, 20000], 13)]      # two calls in a row, then batch 2
    for positions, seed in cases:
        B = len(positions)
        q, q_idx, _, _, _ = token_inputs(d, B, seed)
        items = decode_items([st.layer()] * B, positions)
        sel_ref = torch.empty(B, KB, dtype=torch.int32, device="cuda")
        out_ref = node.sparse_attn_decode(items, B, n_tok, q, q_idx, sel_out=sel_ref)
        out = torch.empty_like(out_ref)
        sel = torch.empty_like(sel_ref)
        assert noalloc_decode(d, items, B, n_tok, q, q_idx, out, sel) == QSA_OK
        torch.cuda.synchronize()
        assert np.array_equal(sel.cpu().numpy(), sel_ref.cpu().numpy())
        assert rel_err(out.cpu().numpy(), out_ref.cpu().numpy()) <= ATTN_TOL


def test_noalloc_decode_with_append_matches_workspace_decode():
    """The call appends each token's K/V/raw key (and the pooled key of the block it completes)
    itself: two tokens in a row per sequence, the second completing a block, caches compared
    byte for byte with a twin pair of caches driven through the workspace entry point."""
    d = make_desc(n_ctx=16384, top_k_blocks=32, window=128, type_k=TYPE_Q8_0, type_v=TYPE_Q8_0)
    node = QsaNode(d)
    lengths = [9982, 5000]                      # the second token of sequence 0 completes block 155
    mine = [QsaState(d) for _ in lengths]
    twin = [QsaState(d) for _ in lengths]
    for i, n in enumerate(lengths):
        fill_cache(node, mine[i], 0, n, seed=31 + i)
        fill_cache(node, twin[i], 0, n, seed=31 + i)
    B, KB = len(lengths), k_blocks(d)
    for step in range(2):
        positions = [n + step for n in lengths]
        q, q_idx, k, v, ki = token_inputs(d, B, 40 + step)
        max_n_kv = max(positions) + 1
        sel_ref = torch.empty(B, KB, dtype=torch.int32, device="cuda")
        out_ref = node.sparse_attn_decode(decode_items([s.layer() for s in twin], positions), B, max_n_kv, q, q_idx,
                                          k, v, ki, sel_out=sel_ref)
        out = torch.empty_like(out_ref)
        sel = torch.empty_like(sel_ref)
        items = decode_items([s.layer() for s in mine], positions)
        assert noalloc_decode(d, items, B, max_n_kv, q, q_idx, out, sel, k, v, ki) == QSA_OK
        torch.cuda.synchronize()
        assert np.array_equal(sel.cpu().numpy(), sel_ref.cpu().numpy())
        assert rel_err(out.cpu().numpy(), out_ref.cpu().numpy()) <= ATTN_TOL
        for a, b, p in zip(mine, twin, positions):      # the written rows (the rest is uninitialised)
            for x, y in ((a.k, b.k), (a.v, b.v), (a.idx, b.idx)):
                assert torch.equal(x[0][:p + 1], y[0][:p + 1])
            nb = (p + 1) // d.ratio
            assert torch.equal(a.pool[0][:nb], b.pool[0][:nb])


def test_noalloc_decode_at_its_scratch_limit():
    """A batch whose decode workspace is exactly the 8 MiB maximum runs (sel_out NULL) and matches
    the workspace entry point; the next batch size is refused before anything runs."""
    d = make_desc(n_ctx=32768, top_k_blocks=64, window=128, type_k=TYPE_Q8_0, type_v=TYPE_Q8_0)
    L = lib()
    B = 3792
    sizes = {n: L.qsa_decode_workspace_size(ctypes.byref(d), B, n) for n in range(30000, 32769)}
    fits = [n for n, s in sizes.items() if s <= SCRATCH_MAX]
    exact = [n for n in fits if sizes[n] == SCRATCH_MAX]
    n_kv = exact[0] if exact else max(fits, key=lambda n: sizes[n])
    assert sizes[n_kv] > SCRATCH_MAX - (64 << 10)          # at the limit, not well inside it
    node, st = QsaNode(d), QsaState(d)
    fill_cache(node, st, 0, n_kv, seed=7)
    positions = [n_kv - 1 - (i * 7) % 10000 for i in range(B)]
    q, q_idx, _, _, _ = token_inputs(d, B, 17)
    items = decode_items([st.layer()] * B, positions)
    out_ref = node.sparse_attn_decode(items, B, n_kv, q, q_idx)
    out = torch.empty_like(out_ref)
    for _ in range(2):
        out.zero_()
        assert noalloc_decode(d, items, B, n_kv, q, q_idx, out, None) == QSA_OK
        torch.cuda.synchronize()
        assert rel_err(out.cpu().numpy(), out_ref.cpu().numpy()) <= ATTN_TOL
    over = next(b for b in range(B + 1, B + 4096) if L.qsa_decode_workspace_size(ctypes.byref(d), b, n_kv) > SCRATCH_MAX)
    items_over = decode_items([st.layer()] * over, [n_kv - 1] * over)
    q2, qi2, _, _, _ = token_inputs(d, over, 18)
    out2 = torch.zeros(over, d.n_head, d.head_dim, device="cuda")
    assert noalloc_decode(d, items_over, over, n_kv, q2, qi2, out2, None) == 5      # QSA_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert float(out2.abs().max()) == 0.0                                          # nothing ran


def test_noalloc_rejects_a_call_beyond_its_scratch():
    d = make_desc(n_ctx=1 << 20, top_k_blocks=128, window=128)
    # 4096 queries at 1M context need ~256 MB of scratch: refused before anything runs
    items = torch.zeros(4096 * 48, dtype=torch.uint8, device="cuda")
    dummy = torch.zeros(16, device="cuda")
    rc = lib().qsa_decode_noalloc(ctypes.byref(d), items.data_ptr(), 4096, 1 << 20, dummy.data_ptr(), TYPE_BF16,
                                  dummy.data_ptr(), None, None, None, dummy.data_ptr(), None,
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 5          # QSA_ERR_WORKSPACE
