"""The output gate fused into the attention's final store (qsa_decode_gated, qsa_prefill_gated) and
the output projection of the gated product (qsa_output_z), on a B200.

The gated store computes z = out * sigmoid(gate) with the arithmetic qsa_output applies to (out,
gate) before its products, so the chain decode_gated -> output_z must give the same y as decode ->
output: bit for bit (same z values, same kernels after them).  z itself is checked against the
ungated output times torch's sigmoid within one bf16 step (bf16 z) or 1e-6 (f32 z: the device and
torch exp may round apart), and the f32 output written beside it equals the ungated call's.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from qwfnfer_b200._abi import QsaError, TYPE_Q8_0, k_blocks, make_desc
from qwfnfer_b200.configs import fill_cache, q8_0_rows, token_inputs
from qwfnfer_b200.qsa import QsaNode, QsaOutput, QsaState, decode_items

pytestmark = pytest.mark.gpu


def check_z(z: torch.Tensor, out: torch.Tensor, gate: torch.Tensor) -> None:
    ref = out.reshape(out.shape[0], -1) * torch.sigmoid(gate)
    if z.dtype == torch.bfloat16:
        err = (z.float() - ref).abs()
        assert torch.all(err <= 2.0 ** -7 * ref.abs() + 1e-30), float(err.max())
    else:
        assert torch.allclose(z, ref, rtol=1e-6, atol=1e-30), float((z - ref).abs().max())


@pytest.mark.parametrize("z_dtype,lengths", [(torch.bfloat16, [30000]), (torch.float32, [30000, 9000, 4000])])
def test_decode_gated_matches_decode(z_dtype, lengths):
    """Batch 1 (one query split over many CTAs: the gate is applied by the merge) and a ragged
    batch; the f32 output written beside z is the ungated call's."""
    d = make_desc(n_ctx=32768, top_k_blocks=64, window=128, type_k=TYPE_Q8_0, type_v=TYPE_Q8_0)
    node = QsaNode(d)
    states = [QsaState(d) for _ in lengths]
    for i, (st, n) in enumerate(zip(states, lengths)):
        fill_cache(node, st, 0, n, seed=200 + i)
    B = len(lengths)
    q, q_idx, _, _, _ = token_inputs(d, B, 201)
    gate = 2 * torch.randn(B, d.n_head * d.head_dim, generator=torch.Generator(device="cuda").manual_seed(202),
                           device="cuda")
    items = decode_items([st.layer() for st in states], [n - 1 for n in lengths])     # the last written rows
    max_n_kv = max(lengths)
    out_ref = node.sparse_attn_decode(items, B, max_n_kv, q, q_idx)
    out = torch.full_like(out_ref, float("nan"))
    z = node.sparse_attn_decode_gated(items, B, max_n_kv, q, q_idx, gate, z_dtype=z_dtype, out=out)
    torch.cuda.synchronize()
    assert torch.equal(out, out_ref)
    check_z(z, out_ref, gate)
    # without the f32 output
    z2 = node.sparse_attn_decode_gated(items, B, max_n_kv, q, q_idx, gate, z_dtype=z_dtype)
    torch.cuda.synchronize()
    assert torch.equal(z2, z)


@pytest.mark.parametrize("T", [100, 20])
def test_prefill_gated_matches_prefill(T):
    """The block-grouped path (T >= 64: the gate is applied by its merge) and the query-major path."""
    d = make_desc(n_ctx=16384, top_k_blocks=32, window=128, type_k=TYPE_Q8_0, type_v=TYPE_Q8_0)
    node = QsaNode(d)
    n_past = 9000
    a, b = QsaState(d), QsaState(d)
    fill_cache(node, a, 0, n_past, seed=210)
    fill_cache(node, b, 0, n_past, seed=210)
    q, q_idx, k, v, ki = token_inputs(d, T, 211)
    gate = torch.randn(T, d.n_head * d.head_dim, generator=torch.Generator(device="cuda").manual_seed(212), device="cuda")
    out_ref = node.sparse_attn(a.layer(), n_past, q, q_idx, k, v, ki)
    z = node.sparse_attn_gated(b.layer(), n_past, q, q_idx, gate, k, v, ki)
    torch.cuda.synchronize()
    check_z(z, out_ref, gate)


@pytest.mark.parametrize("T,q8", [(1, False), (40, False), (3, True), (24, True)])
def test_output_z_chain_equals_output(T, q8):
    """decode_gated -> output_z gives decode -> output's y bit for bit (bf16 z with bf16 weights, f32 z
    with q8_0 weights; GEMV up to 16 tokens, tcgen05 GEMM above)."""
    d = make_desc(n_ctx=8192, top_k_blocks=16, window=128)
    node, st = QsaNode(d), QsaState(d)
    n_past = 6000
    fill_cache(node, st, 0, n_past, seed=220)
    q, q_idx, _, _, _ = token_inputs(d, T, 221)
    g = torch.Generator(device="cuda").manual_seed(222)
    gate = torch.randn(T, d.n_head * d.head_dim, generator=g, device="cuda")
    positions = [n_past - 1 - 37 * i for i in range(T)]
    items = decode_items([st.layer()] * T, positions)
    wf = torch.randn(2560, d.n_head * d.head_dim, generator=g, device="cuda") * 0.02
    op = QsaOutput(d, q8_0_rows(wf) if q8 else wf.to(torch.bfloat16))
    attn = node.sparse_attn_decode(items, T, n_past, q, q_idx)
    y_ref = op.project(attn, gate)
    z = node.sparse_attn_decode_gated(items, T, n_past, q, q_idx, gate, z_dtype=torch.float32 if q8 else torch.bfloat16)
    y = op.project_z(z)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref), float((y - y_ref).abs().max())


def test_gated_argument_errors():
    d = make_desc(n_ctx=8192, top_k_blocks=16, window=128)
    node = QsaNode(d)
    st = QsaState(d)
    q, q_idx, _, _, _ = token_inputs(d, 1, 230)
    items = decode_items([st.layer()], [10])
    gate = torch.zeros(1, d.n_head * d.head_dim, device="cuda")
    buf = torch.zeros(d.n_head * d.head_dim + 1, device="cuda")
    with pytest.raises(QsaError):            # the gate is read as 16-byte vectors: a misaligned one is refused
        node.sparse_attn_decode_gated(items, 1, 11, q, q_idx, buf[1:].view(1, -1))
    op = QsaOutput(d, q8_0_rows(torch.zeros(256, d.n_head * d.head_dim, device="cuda")))
    with pytest.raises(QsaError):            # bf16 z with q8_0 weights: they quantise the f32 product
        op.project_z(torch.zeros(1, d.n_head * d.head_dim, dtype=torch.bfloat16, device="cuda"))
    assert np.isfinite(gate.cpu().numpy()).all()
