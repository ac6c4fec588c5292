"""Parity of the CUDA path (libqsa.so through its C ABI) with the CPU oracle, on a B200.

Bars: q8_0/f16 cache bytes bit-exact; pooled keys within 1e-5 (f32 before
the f16 store); selected block sets bit-exact excluding near-ties; attention within 2e-3 max
relative error (fp32 softmax).  The oracle always reads the bytes the GPU wrote.
"""
import math

import numpy as np
import pytest
import torch

import oracle
from helpers import ATTN_TOL, POOL_TOL, check_selection, forced_blocks, host_caches, rel_err, sel_matrix
from qwfnfer_b200._abi import QSA_OK, TYPE_BF16, TYPE_F16, TYPE_F32, TYPE_Q8_0, k_blocks, lib, make_desc
from qwfnfer_b200.configs import IDX_STD, K_SCALE, fill_cache, token_inputs
from qwfnfer_b200.qsa import QsaNode, QsaState, decode_items

pytestmark = pytest.mark.gpu


def desc_for(kv_type, n_ctx, top_k=64, window=128, ratio=64):
    return make_desc(n_head=16, n_head_kv=2, head_dim=256, idx_n_head=1, idx_dim=128, ratio=ratio,
                     top_k_blocks=top_k, window=window, n_ctx=n_ctx, type_k=kv_type, type_v=kv_type)


def q_host(q):
    if q.dtype == torch.bfloat16:
        return q.view(torch.int16).cpu().numpy().view(np.uint16), TYPE_BF16
    return q.float().cpu().numpy(), TYPE_F32


@pytest.mark.parametrize("kv_type", [TYPE_Q8_0, TYPE_F16])
def test_append_rows_bit_exact(kv_type):
    d = desc_for(kv_type, 4096)
    node, st = QsaNode(d), QsaState(d, zero=True)
    g = torch.Generator(device="cuda").manual_seed(11)
    n, pos0 = 200, 37
    K = torch.randn(n, 512, generator=g, device="cuda") * 3.0
    V = torch.randn(n, 512, generator=g, device="cuda")
    ki = torch.randn(n, 128, generator=g, device="cuda") * IDX_STD
    node.append(st.layer(), pos0, K, V, ki)
    torch.cuda.synchronize()
    kc, vc, ic, _ = oracle.cache_arrays(d)
    oracle.append(d, kc, vc, ic, pos0, K.cpu().numpy(), V.cpu().numpy(), ki.cpu().numpy())
    gk, gv, gi, _ = host_caches(st, 0, d.n_ctx)
    assert np.array_equal(gk, kc)
    assert np.array_equal(gv, vc)
    assert np.array_equal(gi, ic)


@pytest.mark.parametrize("blk0,n_blk,n_ctx", [(0, 96, 64 * 128), (16290, 94, 1 << 20)])
def test_pool_rebuild_matches_oracle(blk0, n_blk, n_ctx):
    d = desc_for(TYPE_Q8_0, n_ctx)
    node = QsaNode(d)
    st = QsaState(d)
    g = torch.Generator(device="cuda").manual_seed(blk0 + 5)
    rows = torch.randn(n_blk * 64, 128, generator=g, device="cuda") * IDX_STD
    st.idx[0][blk0 * 64:(blk0 + n_blk) * 64] = rows.half().view(torch.int16)
    out32 = torch.empty(n_blk, 128, device="cuda")
    node.qsa_pool_rebuild(st.layer(), n_blk, blk0=blk0, pooled_f32=out32)
    torch.cuda.synchronize()
    ic = np.zeros(((blk0 + n_blk) * 64, 128), np.uint16)
    ic[blk0 * 64:] = st.idx[0][blk0 * 64:(blk0 + n_blk) * 64].cpu().numpy().view(np.uint16)
    ref32, ref16 = oracle.pool_blocks(d, ic, blk0, n_blk)
    got32 = out32.cpu().numpy()
    assert np.abs(got32 - ref32).max() <= POOL_TOL
    got16 = st.pool[0][blk0:blk0 + n_blk].cpu().numpy().view(np.uint16)
    diff = got16 != ref16
    # f16 storage agrees except where the f32 values straddle a rounding boundary
    assert diff.mean() < 1e-3
    assert np.all(np.abs(got16[diff].astype(np.int32) - ref16[diff].astype(np.int32)) <= 1)


def run_decode_case(d, n_past, seed, q_dtype=torch.bfloat16, batch_lengths=None, inputs=None):
    """Fill caches, decode one token per sequence (append included), compare everything.
    inputs: the tokens' (q, q_idx, k, v, kidx) when given (e.g. from qsa_front), else seeded."""
    lengths = batch_lengths or [n_past]
    node = QsaNode(d)
    states = [QsaState(d) for _ in lengths]
    for i, (st, L) in enumerate(zip(states, lengths)):
        fill_cache(node, st, 0, L, seed + 100 * i)
    B = len(lengths)
    q, q_idx, k, v, ki = inputs if inputs is not None else token_inputs(d, B, seed + 7, q_dtype)
    items = decode_items([st.layer() for st in states], lengths)
    KB = k_blocks(d)
    sel = torch.full((B, KB), -7, dtype=torch.int32, device="cuda")
    out = node.sparse_attn_decode(items, B, max(lengths) + 1, q, q_idx, k, v, ki, sel_out=sel)
    ws = node.workspace("decode", B, max(lengths) + 1)
    assert node.check(ws) == QSA_OK
    out, sel = out.cpu().numpy(), sel.cpu().numpy()
    qh, qt = q_host(q)
    for i, (st, L) in enumerate(zip(states, lengths)):
        kc, vc, ic, pool = host_caches(st, 0, L + 1)
        # the appended row, bit-exact
        rk, rv, ri, _ = oracle.cache_arrays(make_desc(**{**_desc_kwargs(d), "n_ctx": 64}))
        oracle.append(d, rk, rv, ri, 0, k[i:i + 1].cpu().numpy(), v[i:i + 1].cpu().numpy(), ki[i:i + 1].cpu().numpy())
        assert np.array_equal(kc[L], rk[0]) and np.array_equal(vc[L], rv[0]) and np.array_equal(ic[L], ri[0])
        # the pooled key of the block this token completed
        if (L + 1) % d.ratio == 0:
            b = L // d.ratio
            _, p16 = oracle.pool_blocks(d, ic, b, 1)
            assert np.abs(p16[0].astype(np.int32) - pool[b].astype(np.int32)).max() <= 1
        # selection, from the GPU's pooled keys
        nb = (L + 1) // d.ratio
        sc = oracle.scores(d, pool, max(nb, 1), q_idx[i].cpu().numpy())[0]
        check_selection(d, sel[i], sc, L)
        # attention over the GPU's selection
        ref = oracle.attend(d, kc, vc, [L], sel[i][None], qh[i][None], q_type=qt)[0]
        e = rel_err(out[i], ref)
        assert e <= ATTN_TOL, f"seq {i} (n_past {L}): rel err {e:.2e}"
    return out, sel


def _desc_kwargs(d):
    return dict(n_head=d.n_head, n_head_kv=d.n_head_kv, head_dim=d.head_dim, idx_n_head=d.idx_n_head,
                idx_dim=d.idx_dim, ratio=d.ratio, top_k_blocks=d.top_k_blocks, window=d.window, n_ctx=d.n_ctx,
                type_k=d.type_k, type_v=d.type_v, rope_dim=d.rope_dim, sections=tuple(d.sections),
                rms_eps=d.rms_eps, rope_freq_base=d.rope_freq_base)


def test_decode_config1_shape_f16():
    """Benchmark config 1 shape: 4K context, f16 KV, top-16 + window, f32 query."""
    run_decode_case(desc_for(TYPE_F16, 4096, top_k=16), 4095, seed=0, q_dtype=torch.float32)


def test_decode_config2_full_size_q8_0():
    """Benchmark config 2: 163,840-token q8_0 cache, top-64 of 2560 + window, bf16 query."""
    run_decode_case(desc_for(TYPE_Q8_0, 163840), 163839, seed=1)


@pytest.mark.parametrize("n_past,window,top_k", [(5000, 0, 16), (5055, 0, 16), (100, 128, 64), (64 * 70 + 3, 128, 64),
                                                 (0, 128, 64), (63, 0, 4)])
def test_decode_edge_cases(n_past, window, top_k):
    """Reference tail rule (window 0), partial/complete blocks, everything selected, first token."""
    run_decode_case(desc_for(TYPE_Q8_0, 8192, top_k=top_k, window=window), n_past, seed=3 + n_past)


def test_batched_decode_ragged_lengths():
    """Benchmark config 3 pattern: independent sequences of different lengths in one call."""
    lengths = [4096, 163839, 70000, 4095, 1000, 130000 + 63, 64 * 67, 99999]
    run_decode_case(desc_for(TYPE_Q8_0, 163840), None, seed=2, batch_lengths=lengths)


def test_dense_equivalence_against_torch_fp32():
    """All cells selected: the node equals dense causal attention (torch fp32 reference)."""
    d = desc_for(TYPE_Q8_0, 4096, top_k=64)
    node, st = QsaNode(d), QsaState(d)
    n_past = 2000                                  # 32 blocks < 67 kept: everything selected
    fill_cache(node, st, 0, n_past, 9)
    q, q_idx, k, v, ki = token_inputs(d, 1, 10, torch.float32)
    out = node.sparse_attn_decode(decode_items([st.layer()], [n_past]), 1, n_past + 1, q, q_idx, k, v, ki)
    kc, vc, _, _ = host_caches(st, 0, n_past + 1)
    Kd = torch.from_numpy(oracle.q8_0_dequantize(kc)).view(n_past + 1, 2, 256).cuda()
    Vd = torch.from_numpy(oracle.q8_0_dequantize(vc)).view(n_past + 1, 2, 256).cuda()
    Kd, Vd = Kd.half().float(), Vd.half().float()
    qf = q[0].half().float().view(2, 8, 256)
    s = torch.einsum("ghd,cgd->ghc", qf, Kd) / math.sqrt(256)
    ref = torch.einsum("ghc,cgd->ghd", torch.softmax(s, dim=-1), Vd).reshape(16, 256)
    assert rel_err(out[0].cpu().numpy(), ref.cpu().numpy()) <= ATTN_TOL


def run_prefill(d, n_past, T, chunks, seed):
    node, st = QsaNode(d), QsaState(d)
    fill_cache(node, st, 0, n_past, seed)
    q, q_idx, k, v, ki = token_inputs(d, T, seed + 1)
    KB = k_blocks(d)
    out = torch.empty(T, 16, 256, device="cuda")
    sel = torch.empty(T, KB, dtype=torch.int32, device="cuda")
    off = 0
    for c in chunks:
        node.sparse_attn(st.layer(), n_past + off, q[off:off + c], q_idx[off:off + c], k[off:off + c],
                         v[off:off + c], ki[off:off + c], out=out[off:off + c], sel_out=sel[off:off + c])
        off += c
    assert off == T
    torch.cuda.synchronize()
    return node, st, (q, q_idx, k, v, ki), out.cpu().numpy(), sel.cpu().numpy()


def test_prefill_parity_and_chunk_invariance():
    d = desc_for(TYPE_Q8_0, 8192)
    n_past, T = 3000, 300
    node, st, (q, q_idx, k, v, ki), out1, sel1 = run_prefill(d, n_past, T, [T], 21)
    _, _, _, out3, sel3 = run_prefill(d, n_past, T, [100, 150, 50], 21)
    assert np.array_equal(sel1, sel3)
    # same selections; outputs differ only by the split-K order of the f16 P tiles (each is
    # within ATTN_TOL of the oracle below)
    assert rel_err(out3, out1) <= ATTN_TOL
    kc, vc, ic, pool = host_caches(st, 0, n_past + T)
    # the whole-block pooled keys the prefill produced
    nb = (n_past + T) // 64
    _, p16 = oracle.pool_blocks(d, ic, 0, nb)
    assert np.abs(p16.astype(np.int32) - pool[:nb].astype(np.int32)).max() <= 1
    qh, qt = q_host(q)
    qi = q_idx.cpu().numpy()
    for t in list(range(0, T, 13)) + [T - 1]:
        qp = n_past + t
        sc = oracle.scores(d, pool, max((qp + 1) // 64, 1), qi[t])[0]
        check_selection(d, sel1[t], sc, qp)
        ref = oracle.attend(d, kc, vc, [qp], sel1[t][None], qh[t][None], q_type=qt)[0]
        assert rel_err(out1[t], ref) <= ATTN_TOL


@pytest.mark.parametrize("kv_type,top_k", [(TYPE_Q8_0, 16), (TYPE_Q8_0, 40), (TYPE_F16, 16)])
def test_prefill_radix_selection_and_attention(kv_type, top_k):
    """More visible blocks than top_k: the radix cut of the warp-per-query selection (not the
    take-everything branch), then the block-grouped attention, against the oracle; chunking the
    same tokens gives the same selections."""
    d = desc_for(kv_type, 16384, top_k=top_k)
    n_past, T = 9000, 200                          # 140..143 whole blocks visible
    node, st, (q, q_idx, k, v, ki), out1, sel1 = run_prefill(d, n_past, T, [T], 71)
    _, _, _, out2, sel2 = run_prefill(d, n_past, T, [64, 136], 71)
    assert np.array_equal(sel1, sel2)
    assert rel_err(out2, out1) <= ATTN_TOL
    kc, vc, _, pool = host_caches(st, 0, n_past + T)
    qh, qt = q_host(q)
    qi = q_idx.cpu().numpy()
    for t in list(range(0, T, 17)) + [T - 1]:
        qp = n_past + t
        sc = oracle.scores(d, pool, (qp + 1) // 64, qi[t])[0]
        check_selection(d, sel1[t], sc, qp)
        ref = oracle.attend(d, kc, vc, [qp], sel1[t][None], qh[t][None], q_type=qt)[0]
        assert rel_err(out1[t], ref) <= ATTN_TOL


@pytest.mark.parametrize("n_past,T", [(0, 300), (0, 64), (130, 65), (4000, 63)])
def test_prefill_first_chunks_and_path_boundary(n_past, T):
    """Prefill from an empty cache (early queries see no whole block: only the window) and chunk
    sizes on both sides of the block-grouped path's threshold (64 tokens), against the oracle."""
    d = desc_for(TYPE_Q8_0, 8192, top_k=16)
    node, st, (q, q_idx, k, v, ki), out, sel = run_prefill(d, n_past, T, [T], 81)
    assert np.isfinite(out).all()
    kc, vc, _, pool = host_caches(st, 0, n_past + T)
    qh, qt = q_host(q)
    qi = q_idx.cpu().numpy()
    for t in sorted(set([0, 1, T // 2, T - 1] + list(range(0, T, 29)))):
        qp = n_past + t
        nb = (qp + 1) // 64
        if nb > 0:
            sc = oracle.scores(d, pool, nb, qi[t])[0]
            check_selection(d, sel[t], sc, qp)
        else:                                         # no whole block yet: the window alone
            assert {int(x) for x in sel[t] if x >= 0} == forced_blocks(d, qp)
        ref = oracle.attend(d, kc, vc, [qp], sel[t][None], qh[t][None], q_type=qt)[0]
        assert rel_err(out[t], ref) <= ATTN_TOL


@pytest.mark.parametrize("kv_type", [TYPE_Q8_0, TYPE_F16])
def test_prefill_ignores_unwritten_cells(kv_type):
    """Cells at or past n_past + T of the last block are never written; with their bytes all 0xFF
    (NaN scales and values) the output must still be finite and equal the oracle's."""
    d = desc_for(kv_type, 8192)
    node, st = QsaNode(d), QsaState(d)
    for t in st.k + st.v + st.idx:
        t.fill_(-1)
    n_past, T = 3010, 100                         # ends inside block 48 (cells 3072..3135)
    fill_cache(node, st, 0, n_past, 61)
    q, q_idx, k, v, ki = token_inputs(d, T, 62)
    sel = torch.empty(T, k_blocks(d), dtype=torch.int32, device="cuda")
    out = node.sparse_attn(st.layer(), n_past, q, q_idx, k, v, ki, sel_out=sel)
    torch.cuda.synchronize()
    assert node.check(node.workspace("prefill", T, n_past + T)) == QSA_OK
    out, sel = out.cpu().numpy(), sel.cpu().numpy()
    assert np.isfinite(out).all()
    kc, vc, _, _ = host_caches(st, 0, n_past + T)
    qh, qt = q_host(q)
    for t in [0, 37, 61, T - 1]:
        ref = oracle.attend(d, kc, vc, [n_past + t], sel[t][None], qh[t][None], q_type=qt)[0]
        assert rel_err(out[t], ref) <= ATTN_TOL


def test_decode_equals_prefill_at_same_position():
    d = desc_for(TYPE_Q8_0, 8192)
    n_past, T = 4000, 70
    _, st, (q, q_idx, k, v, ki), out_p, sel_p = run_prefill(d, n_past, T, [T], 33)
    # decode the last token again over the same caches (its row is rewritten with the same bytes)
    node = QsaNode(d)
    t = T - 1
    sel = torch.empty(1, k_blocks(d), dtype=torch.int32, device="cuda")
    out = node.sparse_attn_decode(decode_items([st.layer()], [n_past + t]), 1, n_past + T, q[t:t + 1],
                                  q_idx[t:t + 1], k[t:t + 1], v[t:t + 1], ki[t:t + 1], sel_out=sel)
    sel_d = sel.cpu().numpy()[0]
    # decode scores are exactly rounded, prefill scores are tensor-core f32 sums: both selections
    # equal the oracle's outside near-ties, and the outputs agree whenever the selections do
    _, _, _, pool = host_caches(st, 0, n_past + T)
    qp = n_past + t
    sc = oracle.scores(d, pool, (qp + 1) // 64, q_idx[t].cpu().numpy())[0]
    check_selection(d, sel_d, sc, qp)
    check_selection(d, sel_p[t], sc, qp)
    if np.array_equal(sel_d, sel_p[t]):
        assert rel_err(out.cpu().numpy()[0], out_p[t]) <= ATTN_TOL


def test_out_of_range_position_is_reported_not_faulted():
    d = desc_for(TYPE_Q8_0, 4096)
    node, st = QsaNode(d), QsaState(d)
    fill_cache(node, st, 0, 1000, 1)
    q, q_idx, k, v, ki = token_inputs(d, 2, 2)
    items = decode_items([st.layer(), st.layer()], [999, 4096 + 5])   # second is past n_ctx
    out = node.sparse_attn_decode(items, 2, 4096, q, q_idx, k, v, ki)
    ws = node.workspace("decode", 2, 4096)
    from qwfnfer_b200._abi import STATUS_NAMES
    assert STATUS_NAMES[node.check(ws)] == "QSA_ERR_DEVICE_ARG"
    assert node.check(ws) == QSA_OK                      # cleared
    o = out.cpu().numpy()
    assert np.all(o[1] == 0) and np.all(np.isfinite(o[0]))


def test_host_argument_errors():
    d = desc_for(TYPE_Q8_0, 4096)
    node = QsaNode(d)
    from qwfnfer_b200._abi import QsaError
    st = QsaState(d)
    q, q_idx, k, v, ki = token_inputs(d, 1, 2)
    with pytest.raises(QsaError):
        node.append(st.layer(), 4090, k.repeat(10, 1), v.repeat(10, 1), ki.repeat(10, 1))   # past n_ctx
    with pytest.raises(QsaError):   # workspace too small
        node.sparse_attn_decode(decode_items([st.layer()], [10]), 1, 4096, q, q_idx,
                                ws=torch.zeros(64, dtype=torch.uint8, device="cuda"))
