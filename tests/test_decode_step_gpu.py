"""QsaDecodeStep (one captured decode step per token, inputs and output through pinned host
memory) against the eager qsa_decode call on a second copy of the same caches: the same output
bits, the same selection and the same cache bytes, token after token (one of them completing a
block, so the pooled-key update runs inside the replay)."""
from __future__ import annotations

import pytest
import torch

from qwfnfer_b200._abi import QsaError, TYPE_F16, TYPE_Q8_0, make_desc
from qwfnfer_b200.configs import fill_cache, token_inputs
from qwfnfer_b200.qsa import QsaNode, QsaState, decode_items

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("type_,q_dtype", [(TYPE_Q8_0, torch.bfloat16), (TYPE_F16, torch.float32)])
def test_decode_step_equals_eager(type_, q_dtype):
    d = make_desc(n_ctx=16384, top_k_blocks=32, window=128, type_k=type_, type_v=type_)
    node = QsaNode(d)
    starts = [9021, 4000]                       # sequence 0 completes block 140 at its third token
    ref = [QsaState(d) for _ in starts]
    mine = [QsaState(d) for _ in starts]
    for a, b, n, s in zip(ref, mine, starts, (41, 42)):
        fill_cache(node, a, 0, n, s)
        fill_cache(node, b, 0, n, s)
    max_n_kv = max(starts) + 8
    step = node.decode_step([s.layer() for s in mine], max_n_kv, q_dtype=q_dtype, sel_out=True)
    for t in range(5):
        pos = [n + t for n in starts]
        q, qi, k, v, ki = token_inputs(d, 2, seed=100 + t, q_dtype=q_dtype)
        sel_ref = torch.empty_like(step.sel)
        out_ref = node.sparse_attn_decode(decode_items([s.layer() for s in ref], pos), 2, max_n_kv, q, qi, k, v, ki,
                                          sel_out=sel_ref)
        step.wait()
        step.set_positions(pos)
        for name, x in (("q", q), ("q_idx", qi), ("k_new", k), ("v_new", v), ("kidx_new", ki)):
            step.host[name].copy_(x.cpu())
        host_out = step.run(sync=True)
        assert torch.equal(host_out, out_ref.cpu())
        assert torch.equal(step.sel, sel_ref)
    torch.cuda.synchronize()
    for a, b, n in zip(ref, mine, starts):
        n_rows = n + 5
        for x, y in ((a.k[0], b.k[0]), (a.v[0], b.v[0]), (a.idx[0], b.idx[0])):
            assert torch.equal(x[:n_rows], y[:n_rows])
        assert torch.equal(a.pool[0][:n_rows // d.ratio], b.pool[0][:n_rows // d.ratio])
    assert node.check(step.ws) == 0


def test_decode_step_packed_row_and_shape_checks():
    """load() fills the activations from one packed host row; positions past the captured shape
    are refused on the host."""
    d = make_desc(n_ctx=8192, top_k_blocks=16, window=128)
    node = QsaNode(d)
    st = QsaState(d)
    fill_cache(node, st, 0, 3000, 51)
    step = node.decode_step([st.layer()], 3001)
    with pytest.raises(QsaError):
        step.set_positions([3001])
    step.set_positions([3000])
    q, qi, k, v, ki = token_inputs(d, 1, seed=52)
    row = torch.zeros(step.row_bytes - step.input_offset, dtype=torch.uint8)
    o = 0
    for x in (q, qi, k, v, ki):
        b = x.contiguous().view(torch.uint8).reshape(-1).cpu()
        row[o:o + b.numel()] = b
        o += (b.numel() + 15) // 16 * 16
    step.load(row)
    for name, x in (("q", q), ("q_idx", qi), ("k_new", k), ("v_new", v), ("kidx_new", ki)):
        assert torch.equal(step.host[name], x.cpu())
    got = step.run(sync=True).clone()
    ref = QsaState(d)
    fill_cache(node, ref, 0, 3000, 51)
    out_ref = node.sparse_attn_decode(decode_items([ref.layer()], [3000]), 1, 3001, q, qi, k, v, ki)
    assert torch.equal(got, out_ref.cpu())


def test_stage_copy_directions_and_refusals():
    """qsa_stage_copy moves bytes host->device, device->host and device->device; it refuses (on the
    host, launching nothing) unaligned or ragged sizes and host memory that is not pinned."""
    import ctypes

    import numpy as np

    from qwfnfer_b200._abi import QSA_ERR_INVALID, QSA_OK, lib

    L = lib()
    st = torch.cuda.current_stream().cuda_stream
    n = 12352                                         # 772 pieces of 16 bytes
    src_h = torch.randint(0, 256, (n,), dtype=torch.uint8).pin_memory()
    dev = torch.zeros(n, dtype=torch.uint8, device="cuda")
    dev2 = torch.zeros(n, dtype=torch.uint8, device="cuda")
    back = torch.zeros(n, dtype=torch.uint8).pin_memory()
    assert L.qsa_stage_copy(dev.data_ptr(), src_h.data_ptr(), n, st) == QSA_OK
    assert L.qsa_stage_copy(dev2.data_ptr(), dev.data_ptr(), n, st) == QSA_OK
    assert L.qsa_stage_copy(back.data_ptr(), dev2.data_ptr(), n, st) == QSA_OK
    torch.cuda.synchronize()
    assert torch.equal(back, src_h)
    assert torch.equal(dev.cpu(), src_h)
    plain = np.zeros(n, dtype=np.uint8)               # pageable host memory: not reachable by a kernel
    assert L.qsa_stage_copy(dev.data_ptr(), ctypes.c_void_p(plain.ctypes.data), n, st) == QSA_ERR_INVALID
    assert L.qsa_stage_copy(dev.data_ptr(), src_h.data_ptr(), n - 8, st) == QSA_ERR_INVALID
    assert L.qsa_stage_copy(dev.data_ptr() + 8, src_h.data_ptr(), 16, st) == QSA_ERR_INVALID
    assert L.qsa_stage_copy(None, src_h.data_ptr(), 16, st) == QSA_ERR_INVALID
    torch.cuda.synchronize()
