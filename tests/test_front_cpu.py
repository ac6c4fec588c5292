"""The oracle's projection front (orc_front) on the CPU: against an independent numpy restatement,
and pinned to the pooled-key path (orc_pool_blocks), whose norm and IMRoPE the front shares.

The numpy restatement keeps ggml's f32 angle recurrence (theta advanced by f32 multiplies, which
at positions near 160K moves the angle far from the exact value) and does the rest in float64."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from qwfnfer_b200._abi import make_desc


def bf16_bits(a: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def bits_to_f64(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def weights(d, n_embd, seed):
    rng = np.random.default_rng(seed)
    hd = d.head_dim

    def w(rows):
        return bf16_bits(rng.standard_normal((rows, n_embd), dtype=np.float32) * 0.02)

    return {"wq": w(2 * hd * d.n_head), "wk": w(hd * d.n_head_kv), "wv": w(hd * d.n_head_kv),
            "wq_idx": w(d.idx_dim * d.idx_n_head), "wk_idx": w(d.idx_dim),
            "q_norm": (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32),
            "k_norm": (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32),
            "q_idx_norm": (1 + 0.1 * rng.standard_normal(d.idx_dim)).astype(np.float32)}


def np_norm_rope(d, v, w, pos):
    """rms_norm * w, then IMRoPE with ggml's f32 angle chain (cos/sin in float64 of that angle)."""
    y = v / np.sqrt(np.mean(v * v) + np.float64(np.float32(d.rms_eps))) * w.astype(np.float64)
    nd, half = d.rope_dim, d.rope_dim // 2
    ts = np.float32(np.power(np.float32(d.rope_freq_base), np.float32(-2.0 / nd)))
    s = list(d.sections)
    sect = sum(s)
    out = y.copy()
    th = np.float32(pos)
    for i in range(half):
        sec = i % sect
        use = (sec % 3 == 1 and sec < 3 * s[1]) or (sec % 3 == 2 and sec < 3 * s[2]) or (sec % 3 == 0 and sec < 3 * s[0])
        a = float(th) if use else 0.0
        c, sn = np.cos(a), np.sin(a)
        out[i] = y[i] * c - y[i + half] * sn
        out[i + half] = y[i] * sn + y[i + half] * c
        th = np.float32(th * ts)
    return out


def np_front(d, w, pos, x):
    hd, nh, nkv, H, D = d.head_dim, d.n_head, d.n_head_kv, d.idx_n_head, d.idx_dim
    xb = bits_to_f64(bf16_bits(x))
    y = {k: xb @ bits_to_f64(w[k]).T for k in ("wq", "wk", "wv", "wq_idx", "wk_idx")}
    T = x.shape[0]
    out = {"q": np.zeros((T, nh, hd)), "gate": np.zeros((T, nh * hd)), "q_idx": np.zeros((T, H, D)),
           "k": np.zeros((T, nkv * hd)), "v": y["wv"], "kidx": y["wk_idx"]}
    for t in range(T):
        for h in range(nh):
            out["q"][t, h] = np_norm_rope(d, y["wq"][t, 2 * h * hd:2 * h * hd + hd], w["q_norm"], pos[t])
            out["gate"][t, h * hd:(h + 1) * hd] = y["wq"][t, (2 * h + 1) * hd:(2 * h + 2) * hd]
        for j in range(nkv):
            out["k"][t, j * hd:(j + 1) * hd] = np_norm_rope(d, y["wk"][t, j * hd:(j + 1) * hd], w["k_norm"], pos[t])
        for h in range(H):
            out["q_idx"][t, h] = np_norm_rope(d, y["wq_idx"][t, h * D:(h + 1) * D], w["q_idx_norm"], pos[t])
    return out


@pytest.mark.parametrize("idx_n_head,n_embd,positions", [(1, 512, [0, 5, 163839]), (4, 256, [77777, 1048575])])
def test_oracle_front_matches_numpy(idx_n_head, n_embd, positions):
    d = make_desc(idx_n_head=idx_n_head, n_ctx=1 << 20)
    w = weights(d, n_embd, seed=idx_n_head)
    x = np.random.default_rng(9).standard_normal((len(positions), n_embd), dtype=np.float32)
    pos = np.array(positions, np.int32)
    got = oracle.front(d, w, pos, x)
    ref = np_front(d, w, pos, x)
    for k in ("gate", "v", "kidx"):                          # projections: one f32 rounding of a double sum
        assert np.allclose(got[k], ref[k], rtol=1e-6, atol=1e-7 * np.abs(ref[k]).max()), k
    for k in ("q", "k", "q_idx"):                            # normed and roped
        err = np.abs(got[k] - ref[k]).max() / np.abs(ref[k]).max()
        assert err < 2e-6, (k, err)


@pytest.mark.parametrize("b", [0, 5, 2000])
def test_front_norm_rope_is_the_pooled_keys(b):
    """One-hot activations and indexer-query weights holding a vector u (exact in bf16 and f16)
    give q_idx = norm-rope(u) at position p; a block whose r raw keys all equal u pools to
    norm-rope(u) at position b*r.  With p = b*r and q_norm = k_norm the two are bit-equal."""
    r = 64
    d = make_desc(n_ctx=(b + 1) * r, idx_n_head=1)
    rng = np.random.default_rng(b)
    u = (rng.integers(-32, 33, d.idx_dim) / 8.0).astype(np.float32)
    gamma = (1 + 0.1 * rng.standard_normal(d.idx_dim)).astype(np.float32)
    n_embd, j = 64, 13
    w = weights(d, n_embd, seed=1)
    wq_idx = np.zeros((d.idx_dim, n_embd), np.float32)
    wq_idx[:, j] = u
    w["wq_idx"], w["q_idx_norm"] = bf16_bits(wq_idx), gamma
    x = np.zeros((1, n_embd), np.float32)
    x[0, j] = 1.0
    got = oracle.front(d, w, np.array([b * r], np.int32), x)["q_idx"][0, 0]
    ic = np.zeros(((b + 1) * r, d.idx_dim), np.uint16)
    ic[b * r:] = oracle.f32_to_f16(u)[None, :]
    p32, _ = oracle.pool_blocks(d, ic, b, 1, k_norm_w=gamma)
    assert np.array_equal(got, p32[0])


def test_oracle_output_matches_numpy():
    """orc_output: attn * sigmoid(gate) rounded to bf16, then the attn_output projection."""
    d = make_desc()
    rng = np.random.default_rng(4)
    n_in, n_embd, T = d.n_head * d.head_dim, 384, 3
    wo = bf16_bits(rng.standard_normal((n_embd, n_in), dtype=np.float32) * 0.02)
    attn = rng.standard_normal((T, d.n_head, d.head_dim), dtype=np.float32)
    gate = 2 * rng.standard_normal((T, n_in), dtype=np.float32)
    got = oracle.output(d, wo, attn, gate)
    sg = (np.float32(1) / (np.float32(1) + np.exp(-gate))).astype(np.float32)
    z = bits_to_f64(bf16_bits((attn.reshape(T, n_in) * sg).astype(np.float32)))
    W = bits_to_f64(wo)
    ref = z @ W.T
    bound = 1e-6 * (np.abs(z) @ np.abs(W).T) + 2 ** -7 * np.max(np.abs(z)[:, None, :] * np.abs(W)[None], axis=2)
    assert np.all(np.abs(got - ref) <= bound)


def q8_rows(a: np.ndarray) -> np.ndarray:
    """f32 [rows][n] -> q8_0 rows uint8 [rows][n/32*34] with the pinned reference quantiser."""
    return oracle.q8_0_quantize(np.ascontiguousarray(a, np.float32))


def np_q8_dot_rows(wq: np.ndarray, x: np.ndarray) -> np.ndarray:
    """ggml_vec_dot_q8_0_q8_0 of every q8_0 weight row with x quantised to q8_0 (numpy, float64 sums
    of the f32 block terms): per block the integer sum of products times f32(d_w) * f32(d_x)."""
    n = x.shape[-1]
    nb = n // 32
    xq = q8_rows(x[None])[0].reshape(nb, 34)
    xd = xq[:, :2].copy().view(np.float16).astype(np.float32)[:, 0]
    xi = xq[:, 2:].view(np.int8).astype(np.int64)
    w = wq.reshape(wq.shape[0], nb, 34)
    wd = w[:, :, :2].copy().view(np.float16).astype(np.float32)[:, :, 0]
    wi = w[:, :, 2:].view(np.int8).astype(np.int64)
    sumi = (wi * xi[None]).sum(axis=2).astype(np.float32)
    terms = sumi * (wd * xd[None]).astype(np.float32)
    return terms.astype(np.float64).sum(axis=1).astype(np.float32)


def test_oracle_q8_0_weights_front_and_output():
    """q8_0 projection weights (what quantised GGUF checkpoints carry): the oracle quantises the
    activations to q8_0 and takes integer block dots scaled by both f16 scales, as ggml's CPU
    mul_mat does; checked against an independent numpy restatement, rows exact to f32 rounding."""
    d = make_desc(idx_n_head=2)
    n_embd = 512
    rng = np.random.default_rng(3)
    hd = d.head_dim
    wf = {k: rng.standard_normal((r, n_embd), dtype=np.float32) * 0.02
          for k, r in (("wq", 2 * hd * d.n_head), ("wk", hd * d.n_head_kv), ("wv", hd * d.n_head_kv),
                       ("wq_idx", d.idx_dim * d.idx_n_head), ("wk_idx", d.idx_dim))}
    w = {k: q8_rows(v) for k, v in wf.items()}
    x = rng.standard_normal((2, n_embd), dtype=np.float32)
    pos = np.array([7, 150000], np.int32)
    got = oracle.front(d, w, pos, x, w_type=8)
    for t in range(2):
        gate = np.concatenate([np_q8_dot_rows(w["wq"][(2 * h + 1) * hd:(2 * h + 2) * hd], x[t]) for h in range(d.n_head)])
        np.testing.assert_allclose(got["gate"][t], gate, rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(got["v"][t], np_q8_dot_rows(w["wv"], x[t]), rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(got["kidx"][t], np_q8_dot_rows(w["wk_idx"], x[t]), rtol=1e-6, atol=1e-6)
    # the q8_0 result tracks the f32 product to the quantisation error
    exact = x @ wf["wv"].T
    assert np.abs(got["v"] - exact).max() <= 0.02 * np.abs(exact).max()
    # output side
    wo32 = rng.standard_normal((96, d.n_head * hd), dtype=np.float32) * 0.02
    attn = rng.standard_normal((2, d.n_head, hd), dtype=np.float32)
    g = rng.standard_normal((2, d.n_head * hd), dtype=np.float32)
    y = oracle.output(d, q8_rows(wo32), attn, g, w_type=8)
    z = attn.reshape(2, -1) * (np.float32(1) / (np.float32(1) + np.exp(-g)))
    for t in range(2):
        np.testing.assert_allclose(y[t], np_q8_dot_rows(q8_rows(wo32), z[t].astype(np.float32)), rtol=1e-5, atol=1e-6)


def test_synthetic_q8_0_weights_use_the_pinned_rounding():
    """configs.q8_0_rows (the torch quantiser of the synthetic q8_0 weights) gives the bytes of the
    oracle's quantiser, which the gguf-py golden vectors pin to ggml's reference rounding."""
    from qwfnfer_b200.configs import q8_0_rows, q8_0_rows_dequant
    x = torch.randn(48, 512, generator=torch.Generator().manual_seed(5)) * 0.02
    x[3, :32] = 0.0                                     # an all-zero block (d = 0)
    x[4, 40] = 1e-3                                     # a block with one large value
    q = q8_0_rows(x).numpy()
    assert np.array_equal(q, oracle.q8_0_quantize(x.numpy()))
    assert np.array_equal(q8_0_rows_dequant(torch.from_numpy(q)).numpy(), oracle.q8_0_dequantize(q))
