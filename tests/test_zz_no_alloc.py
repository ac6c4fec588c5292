"""qsa_decode_noalloc: the decode entry point for callers that cannot allocate device memory.

An operator running inside another framework's planned graph, or a serving loop with a fixed
memory budget, cannot hand the library a workspace; this entry point keeps its scratch in a fixed
device array inside libqsa.so.  The test calls it through the C ABI and checks that it gives the
workspace entry point's results (same selections, attention within the parity tolerance) on two
calls in a row, then on a call with another batch size (the scratch layout moves with it).
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


def noalloc_decode(d, items, batch, max_n_kv, q, q_idx, out, sel):
    return lib().qsa_decode_noalloc(ctypes.byref(d), items.data_ptr(), batch, max_n_kv, q.data_ptr(), TYPE_BF16,
                                    q_idx.data_ptr(), None, None, None, out.data_ptr(), sel.data_ptr(),
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


def test_noalloc_rejects_a_call_beyond_its_scratch():
    d = make_desc(n_ctx=1 << 20, top_k_blocks=128, window=128)
    # 4096 queries at 1M context need ~256 MB of scratch: refused before anything runs
    items = torch.zeros(4096 * 48, dtype=torch.uint8, device="cuda")
    dummy = torch.zeros(16, device="cuda")
    rc = lib().qsa_decode_noalloc(ctypes.byref(d), items.data_ptr(), 4096, 1 << 20, dummy.data_ptr(), TYPE_BF16,
                                  dummy.data_ptr(), None, None, None, dummy.data_ptr(), None,
                                  torch.cuda.current_stream().cuda_stream)
    assert rc == 5          # QSA_ERR_WORKSPACE
