"""QSA layer descriptors from a GGUF file's metadata.

The keys, their defaults and the layer rule follow the reference's loader and engine:
  model_index::read_metadata          src/qwfn_model.cpp:111-152 (keys under "<arch>.", defaults)
  hparams::is_attn_layer              src/qwfn_hparams.h: (il + 1) % full_attention_interval == 0
  engine::init, decode QSA state      src/qwfn_engine.cpp:384-431: the ratio of an attention layer is
                                      compress_ratios[il] (0 = a dense attention layer, no QSA);
                                      k_blocks = ceil((idx_top_k + r - 1) / r), the tail block included
The reference forces only the query's incomplete block (window 0), so top_k_blocks = k_blocks - 1.
A descriptor can be refused by qsa_desc_check for shapes these kernels do not handle (for example
more than 8 query heads per KV head); layer_desc raises QsaError then.
"""
from __future__ import annotations

import ctypes

from ._abi import QsaError, TYPE_Q8_0, check, lib, make_desc


def read_hparams(path: str) -> dict:
    """The metadata the node needs, with the reference loader's defaults for absent keys."""
    from gguf import GGUFReader

    r = GGUFReader(path)

    def get(key, default=None):
        f = r.fields.get(key)
        return default if f is None else f.contents()

    arch = get("general.architecture", "")
    A = arch + "."
    secs = list(get(A + "rope.dimension_sections", [])) or [11, 11, 10, 0]
    hp = {
        "arch": arch,
        "n_layer": int(get(A + "block_count", 0)),
        "n_embd": int(get(A + "embedding_length", 0)),
        "n_ctx_train": int(get(A + "context_length", 0)),
        "n_head": int(get(A + "attention.head_count", 0)),
        "n_head_kv": int(get(A + "attention.head_count_kv", 0)),
        "head_dim": int(get(A + "attention.key_length", 0)),
        "rms_eps": float(get(A + "attention.layer_norm_rms_epsilon", 1e-6)),
        "full_attention_interval": int(get(A + "full_attention_interval", 4)),
        "compress_ratios": [int(v) for v in get(A + "attention.compress_ratios", [])],
        "rope_freq_base": float(get(A + "rope.freq_base", 10000000.0)),
        "rope_dim": int(get(A + "rope.dimension_count", 64)),
        "sections": [int(v) for v in (secs + [0, 0, 0, 0])[:4]],
        "idx_n_head": int(get(A + "attention.indexer.head_count", 4)),
        "idx_dim": int(get(A + "attention.indexer.key_length", 128)),
        "idx_top_k": int(get(A + "attention.indexer.top_k", 2048)),
    }
    return hp


def is_attn_layer(hp: dict, il: int) -> bool:
    return (il + 1) % hp["full_attention_interval"] == 0


def qsa_layers(hp: dict) -> list[int]:
    """Attention layers with a compression ratio: the layers the node runs on."""
    cr = hp["compress_ratios"]
    return [il for il in range(hp["n_layer"]) if is_attn_layer(hp, il) and il < len(cr) and cr[il] > 0]


def layer_desc(hp: dict, il: int, n_ctx: int, window: int = 0, type_k: int = TYPE_Q8_0, type_v: int = TYPE_Q8_0,
               k_norm_w: int | None = None):
    """The qsa_desc of attention layer il for a cache of n_ctx cells (rounded up to whole blocks)."""
    if il not in qsa_layers(hp):
        raise QsaError(1, f"layer {il} is not a sparse-attention layer")
    r = hp["compress_ratios"][il]
    k_blocks = (hp["idx_top_k"] + r - 1 + r - 1) // r
    d = make_desc(n_head=hp["n_head"], n_head_kv=hp["n_head_kv"], head_dim=hp["head_dim"], idx_n_head=hp["idx_n_head"],
                  idx_dim=hp["idx_dim"], ratio=r, top_k_blocks=k_blocks - 1, window=window,
                  n_ctx=(n_ctx + r - 1) // r * r, type_k=type_k, type_v=type_v, rope_dim=hp["rope_dim"],
                  sections=tuple(hp["sections"]), rms_eps=hp["rms_eps"], rope_freq_base=hp["rope_freq_base"],
                  k_norm_w=k_norm_w)
    check(lib().qsa_desc_check(ctypes.byref(d)), f"layer {il} descriptor")
    return d
