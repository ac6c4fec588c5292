"""Pins the oracle's IMRoPE against an independent implementation (no GPU).

The oracle restates ggml_rope_multi with GGML_ROPE_TYPE_IMROPE (src/qwfn_graph.cpp:272-273, 425-427:
sections [11, 11, 10, 0], text positions (p, p, p, 0)): per pair i the section rule picks the
position, NEOX pairs (i, i + rope_dim/2), frequency base^(-2i/rope_dim), dims past rope_dim pass
through.  transformers' Qwen3.5 text rotary embedding implements the same interleaved multi-section
rope from its own code (inverse frequencies, interleaving of the t/h/w sections, rotate_half,
partial rotary).  Here the oracle's pooled-key path runs on blocks whose 64 raw-key rows are equal,
so the mean is the row itself, and its output must equal transformers' rms-norm followed by its
rope at the block's first position: within 1e-4 for the first 20 blocks (positions up to 1,216),
and for all 200 (up to 12,736) within the f32 precision of the angle (the two compute it as a chain
of f32 multiplies and as inverse frequency x position; at an angle of 7,700 rad one rounding is
~1e-3 rad).  A pairing of adjacent dims, other frequencies or a rotated tail would miss by O(1).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from qwfnfer_b200._abi import make_desc

m = pytest.importorskip("transformers.models.qwen3_5.modeling_qwen3_5")
cfg_mod = pytest.importorskip("transformers.models.qwen3_5.configuration_qwen3_5")

N_BLK = 200
RATIO = 64


def _transformers_rope(x: torch.Tensor, positions: torch.Tensor, base: float, rope_dim: int, head_dim: int,
                       sections) -> torch.Tensor:
    cfg = cfg_mod.Qwen3_5TextConfig(head_dim=head_dim, max_position_embeddings=1 << 20,
                                    rope_parameters={"rope_type": "default", "rope_theta": base,
                                                     "partial_rotary_factor": rope_dim / head_dim,
                                                     "mrope_section": list(sections)})
    rot = m.Qwen3_5TextRotaryEmbedding(cfg)
    cos, sin = rot(x, positions[None, :])                 # text positions: t = h = w
    q = x[None, None]                                     # [batch 1, heads 1, tokens, head_dim]
    out, _ = m.apply_rotary_pos_emb(q, q, cos, sin)
    return out[0, 0]


def test_pooled_key_rope_matches_transformers():
    d = make_desc(n_ctx=RATIO * N_BLK, rope_dim=64, sections=(11, 11, 10, 0), rope_freq_base=1e7, rms_eps=1e-6)
    assert d.idx_dim == 128 and d.ratio == RATIO
    rng = np.random.default_rng(21)
    rows = rng.normal(0, 1.0, (N_BLK, d.idx_dim)).astype(np.float16)
    ic = np.repeat(rows, RATIO, axis=0).view(np.uint16)   # block b: 64 copies of row b
    out32, _ = oracle.pool_blocks(d, ic, 0, N_BLK)

    x = torch.from_numpy(rows.astype(np.float32))
    xn = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + d.rms_eps)
    positions = torch.arange(N_BLK, dtype=torch.int64) * RATIO
    want = _transformers_rope(xn, positions, d.rope_freq_base, d.rope_dim, d.idx_dim, (11, 11, 10)).numpy()

    assert np.isfinite(out32).all()
    np.testing.assert_allclose(out32[:, d.rope_dim:], want[:, d.rope_dim:], rtol=1e-5, atol=1e-6)   # passed through
    np.testing.assert_allclose(out32[:20], want[:20], rtol=1e-4, atol=1e-4)
    # beyond: |error| <= |x| x (f32 rounding of the largest angle of the block, a few ulp)
    angle = positions.numpy()[:, None].astype(np.float64)
    bound = 8 * np.abs(xn.numpy()).max(axis=1, keepdims=True) * angle * 2.0 ** -24 + 1e-5
    assert (np.abs(out32 - want) <= bound).all()
    # the layout is what is pinned: NEOX pairs and not adjacent ones, the sections' frequencies
    assert np.abs(out32[1:, :d.rope_dim] - xn.numpy()[1:, :d.rope_dim]).max() > 0.1
