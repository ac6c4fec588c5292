"""The CPU oracle against everything that pins it (no GPU).

- q8_0 and f16 rounding: the committed golden vectors (tests/golden/make_golden.py, gguf-py's
  ggml-quants reference codec and numpy's IEEE float16 cast);
- selection: a literal restatement of the reference's host-side bias code
  (src/qwfn_engine.cpp:926-950 prefill, :748-759 decode, tools/qwfn_logits.cpp:151-176) followed by
  a top-k over score + bias, which is what ggml_top_k sees;
- attention: equal to dense causal attention (fp64) whenever every cell is selected
  (src/qwfn_graph.h:29-35);
- pooled keys: an independent numpy restatement of qsa_pool_blocks (src/qwfn_graph.cpp:412-429).
"""
import math
import os

import numpy as np
import pytest

import oracle
from qwfnfer_b200._abi import TYPE_F16, TYPE_Q8_0, k_blocks, make_desc

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_q8_0_matches_ggml_reference_codec():
    g = np.load(os.path.join(GOLDEN, "q8_0_ggml_ref.npz"))
    q = oracle.q8_0_quantize(g["x"])
    assert q.shape == g["q"].shape
    assert np.array_equal(q, g["q"]), f"{np.sum(np.any(q != g['q'], axis=1))} blocks differ"
    # dequantize: d * q in f32
    d = g["q"][:, :2].copy().view(np.float16).astype(np.float32)
    qs = g["q"][:, 2:].view(np.int8).astype(np.float32)
    assert np.array_equal(oracle.q8_0_dequantize(g["q"]), (d * qs).astype(np.float32))


def test_f16_rounding_is_ieee_rne():
    g = np.load(os.path.join(GOLDEN, "f16_rne.npz"))
    assert np.array_equal(oracle.f32_to_f16(g["x"]), g["h"])
    back = oracle.f16_to_f32(g["h"])
    assert np.array_equal(back, g["h"].view(np.float16).astype(np.float32))


# ---------------------------------------------------------------- selection rules
def ref_prefill_bias(n_past_c: int, Tc: int, r: int) -> np.ndarray:
    """engine::build_attn_inputs bias rows, src/qwfn_engine.cpp:926-950 (literal)."""
    n_kv = n_past_c + Tc
    n_blocks = (n_kv + r - 1) // r
    n_bid = n_kv // r
    have_dead = n_bid < n_blocks
    dead = n_bid if have_dead else n_blocks - 1
    bi = np.empty((Tc, n_blocks), np.float32)
    for i in range(Tc):
        q = n_past_c + i
        tail_b = min(n_bid, (q + 1) // r)
        row = bi[i]
        row[:tail_b] = 0.0
        row[tail_b:n_bid] = 1e9
        row[n_bid:] = -np.inf
        if have_dead:
            row[dead] = 1e9
        for b in range(tail_b, n_blocks):
            if row[b] > 0.0 and b * r > q:
                row[b] = -1e9
    return bi


def ref_decode_bias(n_past: int, r: int, NBmax: int):
    """engine::qsa_decode_prepare after a prefill (the full rewrite, src/qwfn_engine.cpp:761-768)
    plus the per-token window (:748-753) and the bucket rule (:755-759)."""
    b_last = n_past // r
    n_bid = (n_past + 1) // r
    full = np.full(NBmax, -np.inf, np.float32)
    full[: min(n_bid, NBmax)] = 0.0
    if b_last < NBmax:
        full[b_last] = 0.0 if b_last < n_bid else 1e9
    NB = ((b_last + 1 + 255) // 256) * 256
    NB = min(max(NB, 768), NBmax)
    return full, NB


def topk_set(v: np.ndarray, k: int) -> set:
    order = np.argsort(-v, kind="stable")
    return set(int(b) for b in order[:k])


def visible(sel_blocks, q, r):
    return {b for b in sel_blocks if b * r <= q}


@pytest.mark.parametrize("r,idx_top_k_cells,n_past,T", [(4, 64, 0, 300), (4, 64, 37, 41), (64, 1024, 1000, 200),
                                                        (64, 64 * 16 - 63, 4000, 96), (8, 24, 5, 60)])
def test_selection_equals_reference_prefill_bias_rule(r, idx_top_k_cells, n_past, T):
    """window=0 reproduces graph_builder::qsa_top_k with build_attn_inputs' bias."""
    rng = np.random.default_rng(r * 1000 + n_past)
    width_blocks = (idx_top_k_cells + r - 1 + r - 1) // r      # kb = ceil((top_k + r - 1) / r)
    d = make_desc(ratio=r, top_k_blocks=width_blocks - 1, window=0, n_ctx=((n_past + T) // r + 2) * r)
    bias = ref_prefill_bias(n_past, T, r)
    n_blocks = bias.shape[1]
    n_kv = n_past + T
    for i in range(T):
        q = n_past + i
        sc = rng.random(n_blocks).astype(np.float32) * 10.0  # distinct: no ties
        width = min(n_kv, idx_top_k_cells + r - 1)
        kb = min(n_blocks, (width + r - 1) // r)
        ref = visible(topk_set(sc + bias[i], kb), q, r)
        sel, _ = oracle.select(d, sc, q)
        ours = {int(b) for b in sel if b >= 0}
        assert ours == ref, f"q={q}: ours-ref {sorted(ours - ref)} ref-ours {sorted(ref - ours)}"


@pytest.mark.parametrize("r,top_blocks,n_past", [(64, 16, 4095), (64, 16, 4000), (4, 16, 299), (4, 512, 163839 // 64),
                                                 (64, 64, 163839), (64, 64, 100)])
def test_selection_equals_reference_decode_bias_rule(r, top_blocks, n_past):
    rng = np.random.default_rng(n_past)
    NBmax = (n_past + 1 + r - 1) // r + 3
    d = make_desc(ratio=r, top_k_blocks=top_blocks, window=0, n_ctx=NBmax * r)
    bias, NB = ref_decode_bias(n_past, r, NBmax)
    sc = rng.random(NBmax).astype(np.float32)
    kb = min(top_blocks + 1, NB)
    ref = visible(topk_set(sc[:NB] + bias[:NB], kb), n_past, r)
    sel, _ = oracle.select(d, sc, n_past)
    assert {int(b) for b in sel if b >= 0} == ref


@pytest.mark.parametrize("q", [0, 63, 64, 127, 128, 129, 4095, 5000, 163839])
def test_selection_window_contract(q):
    """window > 0: blocks b_q-2..b_q forced (+1e9), KB = k + 3, else as the reference bias."""
    r, k = 64, 16
    d = make_desc(ratio=r, top_k_blocks=k, window=128, n_ctx=(q // r + 2) * r)
    rng = np.random.default_rng(q)
    n_blocks = q // r + 1
    sc = rng.random(n_blocks).astype(np.float32)
    bias = ref_prefill_bias(q, 1, r)[0] if q > 0 else ref_prefill_bias(0, 1, r)[0]
    bq = q // r
    bias[max(0, bq - 2): bq + 1] = 1e9
    ref = visible(topk_set(sc + bias[:n_blocks], k + 3), q, r)
    sel, forced = oracle.select(d, sc, q)
    ours = {int(b) for b in sel if b >= 0}
    assert ours == ref
    assert {int(b) for b, f in zip(sel, forced) if f} == set(range(max(0, bq - 2), bq + 1))
    assert k_blocks(d) == k + 3


# ---------------------------------------------------------------- attention
def make_cache(d, n_tok, seed):
    rng = np.random.default_rng(seed)
    kv_dim = d.n_head_kv * d.head_dim
    K = (rng.standard_normal((n_tok, kv_dim)) / math.sqrt(d.head_dim)).astype(np.float32)
    V = rng.standard_normal((n_tok, kv_dim)).astype(np.float32)
    kc, vc, ic, pool = oracle.cache_arrays(d)
    oracle.append(d, kc, vc, ic, 0, K, V, None)
    return kc, vc


def dequant_rows(d, c, type_, n_tok, round_f16):
    kv_dim = d.n_head_kv * d.head_dim
    if type_ == TYPE_Q8_0:
        x = oracle.q8_0_dequantize(c[:n_tok]).reshape(n_tok, kv_dim)
        if round_f16:
            x = x.astype(np.float16).astype(np.float32)
    else:
        x = c[:n_tok].view(np.uint16).view(np.float16).astype(np.float32).reshape(n_tok, kv_dim)
    return x


@pytest.mark.parametrize("type_", [TYPE_Q8_0, TYPE_F16])
@pytest.mark.parametrize("flags", [0, oracle.DEFAULT_FLAGS])
def test_attention_dense_equivalence(type_, flags):
    """Every cell selected -> the node is dense causal attention (src/qwfn_graph.h:29-35)."""
    d = make_desc(n_head=8, n_head_kv=2, head_dim=64, ratio=16, top_k_blocks=64, window=0, n_ctx=512,
                  type_k=type_, type_v=type_)
    n_tok = 300
    kc, vc = make_cache(d, n_tok, 1)
    rng = np.random.default_rng(2)
    q_pos = np.array([0, 15, 16, 150, 299])
    Q = rng.standard_normal((len(q_pos), d.n_head, d.head_dim)).astype(np.float32)
    nblk = n_tok // d.ratio + 1
    sel = np.full((len(q_pos), k_blocks(d)), -1, np.int32)
    for t, q in enumerate(q_pos):
        blocks = np.arange(q // d.ratio + 1)
        sel[t, : len(blocks)] = blocks
    out = oracle.attend(d, kc, vc, q_pos, sel, Q, flags=flags)
    kr = bool(flags & oracle.KV_F16_ROUND)
    Kd = dequant_rows(d, kc, type_, n_tok, kr).astype(np.float64)
    Vd = dequant_rows(d, vc, type_, n_tok, kr).astype(np.float64)
    Qd = Q.astype(np.float16).astype(np.float64) if flags & oracle.Q_F16 else Q.astype(np.float64)
    gqa = d.n_head // d.n_head_kv
    for t, q in enumerate(q_pos):
        for h in range(d.n_head):
            g = h // gqa
            k = Kd[: q + 1, g * d.head_dim:(g + 1) * d.head_dim]
            v = Vd[: q + 1, g * d.head_dim:(g + 1) * d.head_dim]
            s = k @ Qd[t, h] / math.sqrt(d.head_dim)
            p = np.exp(s - s.max())
            ref = p @ v / p.sum()
            np.testing.assert_allclose(out[t, h], ref, rtol=0, atol=2e-6)
    assert nblk > 0


def test_ggml_f16_accumulator_mode_is_close_but_distinct():
    """ORC_GGML_FA|ORC_GGML_V_F16 emulates ggml-cpu's F16 V accumulator; recorded, not asserted tight."""
    d = make_desc(n_head=8, n_head_kv=1, head_dim=64, ratio=64, top_k_blocks=16, window=128, n_ctx=4096)
    kc, vc = make_cache(d, 4096, 3)
    Q = np.random.default_rng(4).standard_normal((1, 8, 64)).astype(np.float32)
    sel = np.arange(k_blocks(d), dtype=np.int32)[None]
    a = oracle.attend(d, kc, vc, [4095], sel, Q)
    b = oracle.attend(d, kc, vc, [4095], sel, Q, flags=oracle.DEFAULT_FLAGS | oracle.GGML_FA)
    c = oracle.attend(d, kc, vc, [4095], sel, Q, flags=oracle.DEFAULT_FLAGS | oracle.GGML_FA | oracle.GGML_V_F16)
    rel = lambda x: float(np.abs(x - a).max() / np.abs(a).max())
    assert rel(b) < 1e-5          # f32 online softmax == exact within f32 rounding
    assert 0.0 < rel(c) < 5e-2    # the f16 accumulator is visibly coarser


# ---------------------------------------------------------------- pooled keys
def numpy_pool(d, ic, b, w=None):
    """Independent restatement of qsa_pool_blocks for block b (f32 steps, double sum of squares)."""
    r, D, nd = d.ratio, d.idx_dim, d.rope_dim
    x = ic[b * r:(b + 1) * r].view(np.float16).astype(np.float32)
    s = x[0].copy()
    for i in range(1, r):
        s = (s + x[i]).astype(np.float32)
    s = (s * np.float32(1.0 / r)).astype(np.float32)
    ss = float(np.sum((s * s).astype(np.float64)))
    mean = np.float32(ss / D)
    scale = np.float32(1.0) / np.sqrt(np.float32(mean + np.float32(d.rms_eps)), dtype=np.float32)
    y = (s * scale).astype(np.float32)
    if w is not None:
        y = (y * w).astype(np.float32)
    theta_scale = np.float32(math.pow(d.rope_freq_base, -2.0 / nd))
    th = np.float32(b * r)
    out = y.copy()
    for i in range(nd // 2):
        c, sn = np.float32(math.cos(th)), np.float32(math.sin(th))
        x0, x1 = y[i], y[i + nd // 2]
        out[i] = x0 * c - x1 * sn
        out[i + nd // 2] = x0 * sn + x1 * c
        th = np.float32(th * theta_scale)
    return out


@pytest.mark.parametrize("blk", [0, 1, 17, 2559])
def test_pool_blocks_match_numpy_restatement(blk):
    d = make_desc(ratio=64, n_ctx=64 * 2560)
    rng = np.random.default_rng(blk)
    ic = np.zeros((d.n_ctx, d.idx_dim), np.uint16)
    rows = (rng.standard_normal((64, d.idx_dim)) * 1.02).astype(np.float32)
    ic[blk * 64:(blk + 1) * 64] = rows.astype(np.float16).view(np.uint16)
    w = (1.0 + 0.1 * rng.standard_normal(d.idx_dim)).astype(np.float32)
    o32, o16 = oracle.pool_blocks(d, ic, blk, 1, w)
    ref = numpy_pool(d, ic, blk, w)
    np.testing.assert_allclose(o32[0], ref, rtol=0, atol=1e-5)
    assert np.array_equal(o16[0], o32[0].astype(np.float16).view(np.uint16))
