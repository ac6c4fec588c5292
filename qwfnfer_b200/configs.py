"""The benchmark configurations of the QSA path and their seeded synthetic inputs.

Stand-ins (no checkpoint or dataset is involved): K, V ~ N(0,1) with K scaled by 1/sqrt(256) after
norm/rope, stored q8_0 (or f16); Q ~ N(0,1) in bf16 (f32 for the f16 config); the indexer query and
raw indexer keys ~ N(0, 1.012^2), the spread of a N(0,0.02) [128 x 2560] projection of N(0,1)
activations; k_norm weights = 1.  Layer descriptor: 16 query heads, 2 KV heads, head_dim 256,
one indexer head of dim 128, blocks of 64 cells, IMRoPE (rope_dim 64, sections 11/11/10/0,
base 1e7), a 128-token causal window forced at block granularity.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from ._abi import TYPE_F16, TYPE_Q8_0, QsaDesc, make_desc

IDX_STD = 1.012   # sqrt(2560) * 0.02
K_SCALE = 1.0 / 16.0


@dataclass
class Config:
    name: str
    n_ctx: int
    top_k: int
    kv_type: int
    seed: int
    n_past: int = 0                    # decode: position of the decoded token
    batch: int = 1
    layers: int = 1
    prefill_T: int = 0
    lengths: list[int] = field(default_factory=list)

    def desc(self, n_ctx: int | None = None) -> QsaDesc:
        return make_desc(n_head=16, n_head_kv=2, head_dim=256, idx_n_head=1, idx_dim=128, ratio=64,
                         top_k_blocks=self.top_k, window=128, n_ctx=n_ctx or self.n_ctx,
                         type_k=self.kv_type, type_v=self.kv_type)


def config3_lengths(n: int = 64, lo: int = 4096, hi: int = 163840, seed: int = 2) -> list[int]:
    g = torch.Generator().manual_seed(seed)
    return [int(x) for x in torch.randint(lo, hi + 1, (n,), generator=g)]


CONFIGS = {
    1: Config("cpu_decode_4k_f16", n_ctx=4096, top_k=16, kv_type=TYPE_F16, seed=0, n_past=4095),
    2: Config("decode_160k_q8_0", n_ctx=163840, top_k=64, kv_type=TYPE_Q8_0, seed=1, n_past=163839),
    3: Config("batched_decode_64_q8_0", n_ctx=163840, top_k=64, kv_type=TYPE_Q8_0, seed=2, batch=64),
    4: Config("prefill_8192_on_155648_q8_0", n_ctx=163840, top_k=64, kv_type=TYPE_Q8_0, seed=3,
              n_past=155648, prefill_T=8192),
    5: Config("decode_1m_12_layers_q8_0", n_ctx=1048576, top_k=128, kv_type=TYPE_Q8_0, seed=4,
              n_past=1048575, layers=12),
}


def fill_cache(node, state, il: int, n_tok: int, seed: int, chunk: int = 1 << 16, device="cuda",
               append=None) -> None:
    """Append n_tok seeded random tokens at rows [0, n_tok) through the library's append path
    (q8_0 quantisation, raw indexer keys, pooled keys of the completed blocks).  `append(cache,
    pos0, K, V, kidx)` replaces node.append (a shard's append keeps the rows in its cells; the
    random stream is the same, so shards hold exactly the rows of the unsharded cache)."""
    d = node.desc
    append = append or node.append
    kv_dim = d.n_head_kv * d.head_dim
    g = torch.Generator(device=device).manual_seed(seed)
    for pos in range(0, n_tok, chunk):
        n = min(chunk, n_tok - pos)
        K = torch.randn(n, kv_dim, generator=g, device=device) * K_SCALE
        V = torch.randn(n, kv_dim, generator=g, device=device)
        ki = torch.randn(n, d.idx_dim, generator=g, device=device) * IDX_STD
        append(state.layer(il), pos, K, V, ki)


def token_inputs(d: QsaDesc, n: int, seed: int, q_dtype=torch.bfloat16, device="cuda"):
    """(q [n, n_head, hd], q_idx [n, idx_n_head, idx_dim], k_new, v_new, kidx_new) for n tokens."""
    g = torch.Generator(device=device).manual_seed(seed)
    kv_dim = d.n_head_kv * d.head_dim
    q = torch.randn(n, d.n_head, d.head_dim, generator=g, device=device).to(q_dtype)
    q_idx = torch.randn(n, d.idx_n_head, d.idx_dim, generator=g, device=device) * IDX_STD
    k = torch.randn(n, kv_dim, generator=g, device=device) * K_SCALE
    v = torch.randn(n, kv_dim, generator=g, device=device)
    ki = torch.randn(n, d.idx_dim, generator=g, device=device) * IDX_STD
    return q, q_idx, k, v, ki


N_EMBD = 2560     # model width of the synthetic projection weights


def front_weights(d: QsaDesc, n_embd: int = N_EMBD, seed: int = 0, gammas: bool = False, device="cuda",
                  q8_0: bool = False) -> dict:
    """Synthetic weights of the projection front (qsa_front): ~ N(0, 0.02) row-major [out][n_embd]
    for attn_q (query and gate interleaved per head), attn_k, attn_v, indexer.q_proj,
    indexer.k_proj, in bf16 or (q8_0=True) as q8_0 rows; f32 norm weights, 1 (the stand-in) or with
    gammas=True ~ 1 + N(0, 0.1) to exercise the multiply."""
    g = torch.Generator(device=device).manual_seed(seed)
    hd = d.head_dim

    def w(rows):
        f = torch.randn(rows, n_embd, generator=g, device=device) * 0.02
        return q8_0_rows(f) if q8_0 else f.to(torch.bfloat16)

    def gamma(n):
        if not gammas:
            return torch.ones(n, device=device)
        return 1.0 + 0.1 * torch.randn(n, generator=g, device=device)

    return {"wq": w(2 * hd * d.n_head), "wk": w(hd * d.n_head_kv), "wv": w(hd * d.n_head_kv),
            "wq_idx": w(d.idx_dim * d.idx_n_head), "wk_idx": w(d.idx_dim),
            "q_norm": gamma(hd), "k_norm": gamma(hd), "q_idx_norm": gamma(d.idx_dim)}


def q8_0_rows(w: torch.Tensor) -> torch.Tensor:
    """f32 [rows][n] (n % 32 == 0) -> q8_0 rows as bytes uint8 [rows][n/32*34], with ggml's reference
    rounding (quantize_row_q8_0_ref): per block d = amax/127, id = 1/d (0 when d == 0), q = x*id
    rounded half away from zero, d stored as f16 ahead of the block's 32 int8 values."""
    rows, n = w.shape
    x = w.float().reshape(rows, n // 32, 32)
    d = x.abs().amax(dim=2, keepdim=True) / 127.0
    inv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
    v = x * inv
    q = (torch.sign(v) * torch.floor(v.abs() + 0.5)).to(torch.int8)
    out = torch.empty(rows, n // 32, 34, dtype=torch.uint8, device=w.device)
    out[:, :, :2] = d.half().view(torch.uint8).reshape(rows, n // 32, 2)
    out[:, :, 2:] = q.view(torch.uint8)
    return out.reshape(rows, n // 32 * 34)


def q8_0_rows_dequant(q: torch.Tensor) -> torch.Tensor:
    """q8_0 rows uint8 [rows][n/32*34] -> f32 [rows][n] (f32(d) * q)."""
    rows = q.shape[0]
    b = q.reshape(rows, -1, 34)
    d = b[:, :, :2].contiguous().view(torch.float16).float()
    return (d * b[:, :, 2:].contiguous().view(torch.int8).float()).reshape(rows, -1)
