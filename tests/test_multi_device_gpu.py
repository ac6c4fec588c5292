"""One process driving two GPUs: the library's kernels with large dynamic shared memory (the
decode selection and attention, the prefill tcgen05 scores and the block-grouped attention) need a
function attribute that is a per-device setting.  The same decode and prefill run on cuda:0 and
then cuda:1 must succeed on both and give the same bits."""
from __future__ import annotations

import pytest
import torch

from qwfnfer_b200._abi import make_desc
from qwfnfer_b200.configs import fill_cache, token_inputs
from qwfnfer_b200.qsa import QsaNode, QsaState, decode_items

pytestmark = pytest.mark.gpu


def run_on(dev: int):
    name = f"cuda:{dev}"
    with torch.cuda.device(dev):
        d = make_desc(n_ctx=8192, top_k_blocks=16, window=128)
        node = QsaNode(d, device=name)
        st = QsaState(d, device=name)
        fill_cache(node, st, 0, 5000, 71, device=name)
        q, qi, k, v, ki = token_inputs(d, 1, 72, device=name)
        dec = node.sparse_attn_decode(decode_items([st.layer()], [5000], device=name), 1, 5001, q, qi, k, v, ki)
        T = 128                                   # >= 64 tokens: tcgen05 scores and the block-grouped attention
        qp, qip, kp, vp, kip = token_inputs(d, T, 73, device=name)
        pre = node.sparse_attn(st.layer(), 5001, qp, qip, kp, vp, kip)
        torch.cuda.synchronize()
        return dec.cpu(), pre.cpu()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_kernels_on_two_devices_of_one_process():
    d0, p0 = run_on(0)
    d1, p1 = run_on(1)
    assert torch.equal(d0, d1)
    assert torch.equal(p0, p1)
    assert torch.isfinite(p0).all()
