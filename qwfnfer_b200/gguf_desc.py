"""QSA layer descriptors from a GGUF file's metadata, through libqsa's C reader.

The metadata is parsed by the library's host code (qsa_gguf_read_hparams in csrc/qsa_gguf.cpp),
with the reference loader's keys, typed getters and defaults:
  model_index::read_metadata          src/qwfn_model.cpp:111-152 (keys under "<arch>.", defaults)
  hparams::is_attn_layer              (il + 1) % full_attention_interval == 0
  engine::init, decode QSA state      src/qwfn_engine.cpp:384-431: the ratio of an attention layer is
                                      compress_ratios[il] (0 = a dense attention layer, no QSA);
                                      k_blocks = ceil((idx_top_k + r - 1) / r), the tail block included
The reference forces only the query's incomplete block (window 0), so top_k_blocks = k_blocks - 1.
A descriptor can be refused by qsa_desc_check for shapes these kernels do not handle (for example
more than 8 query heads per KV head); layer_desc raises QsaError then.  This module only converts
between the C structures and Python values.
"""
from __future__ import annotations

import ctypes

from ._abi import QSA_OK, QsaDesc, QsaError, QsaGgufHparams, TYPE_Q8_0, lib


def read_hparams_struct(path: str) -> QsaGgufHparams:
    hp = QsaGgufHparams()
    err = ctypes.create_string_buffer(256)
    s = lib().qsa_gguf_read_hparams(str(path).encode(), ctypes.byref(hp), err, len(err))
    if s != QSA_OK:
        raise QsaError(s, f"qsa_gguf_read_hparams: {err.value.decode(errors='replace')}")
    return hp


def read_hparams(path: str) -> dict:
    """The metadata the node needs, with the reference loader's defaults for absent keys."""
    hp = read_hparams_struct(path)
    out = {f: getattr(hp, f) for f, _ in QsaGgufHparams._fields_ if f not in ("arch", "compress_ratios", "sections")}
    out["arch"] = hp.arch.decode()
    out["compress_ratios"] = [hp.compress_ratios[i] for i in range(hp.n_compress)]
    out["sections"] = [hp.sections[i] for i in range(4)]
    out["_struct"] = hp
    return out


def _struct(hp) -> QsaGgufHparams:
    return hp["_struct"] if isinstance(hp, dict) else hp


def is_attn_layer(hp: dict, il: int) -> bool:
    return (il + 1) % hp["full_attention_interval"] == 0


def qsa_layers(hp) -> list[int]:
    """Attention layers with a compression ratio: the layers the node runs on (qsa_gguf_is_qsa_layer)."""
    h = _struct(hp)
    return [il for il in range(h.n_layer) if lib().qsa_gguf_is_qsa_layer(ctypes.byref(h), il)]


def layer_desc(hp, il: int, n_ctx: int, window: int = 0, type_k: int = TYPE_Q8_0, type_v: int = TYPE_Q8_0,
               k_norm_w: int | None = None) -> QsaDesc:
    """The qsa_desc of sparse-attention layer il for a cache of n_ctx cells (qsa_gguf_layer_desc)."""
    d = QsaDesc()
    s = lib().qsa_gguf_layer_desc(ctypes.byref(_struct(hp)), il, n_ctx, window, type_k, type_v, k_norm_w,
                                  ctypes.byref(d))
    if s != QSA_OK:
        raise QsaError(s, f"layer {il} descriptor")
    return d
