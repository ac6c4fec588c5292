"""QSA descriptors from GGUF metadata (qwfnfer_b200.gguf_desc) against the reference loader's keys,
defaults and layer rule, on synthetic GGUF files written with gguf-py (metadata only)."""
from __future__ import annotations

import pytest

from qwfnfer_b200._abi import QSA_ERR_UNSUPPORTED, QsaError, k_blocks
from qwfnfer_b200.configs import CONFIGS
from qwfnfer_b200.gguf_desc import layer_desc, qsa_layers, read_hparams


def write_gguf(path, kv: dict):
    from gguf import GGUFWriter

    w = GGUFWriter(str(path), "qwen4exp")
    A = "qwen4exp."
    for k, v in kv.items():
        if isinstance(v, list):
            w.add_array(A + k, v)
        elif isinstance(v, float):
            w.add_float32(A + k, v)
        else:
            w.add_uint32(A + k, v)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


STANDIN = {"block_count": 8, "embedding_length": 2560, "context_length": 262144, "attention.head_count": 16,
           "attention.head_count_kv": 2, "attention.key_length": 256, "attention.value_length": 256,
           "attention.layer_norm_rms_epsilon": 1e-6, "full_attention_interval": 4,
           "attention.compress_ratios": [0, 0, 0, 64, 0, 0, 0, 64], "rope.freq_base": 1e7, "rope.dimension_count": 64,
           "rope.dimension_sections": [11, 11, 10, 0], "attention.indexer.head_count": 1,
           "attention.indexer.key_length": 128, "attention.indexer.top_k": 4033}


def test_standin_layer_descriptor(tmp_path):
    """A file with the benchmark stand-in's shapes: layers 3 and 7 are the sparse-attention layers;
    top_k 4033 at r = 64 keeps ceil((4033 + 63) / 64) = 64 blocks, the tail block among them."""
    p = tmp_path / "standin.gguf"
    write_gguf(p, STANDIN)
    hp = read_hparams(str(p))
    assert hp["arch"] == "qwen4exp" and hp["n_embd"] == 2560
    assert qsa_layers(hp) == [3, 7]
    d = layer_desc(hp, 3, n_ctx=163840)
    ref = CONFIGS[2].desc()
    for f in ("n_head", "n_head_kv", "head_dim", "idx_n_head", "idx_dim", "ratio", "n_ctx", "rope_dim"):
        assert getattr(d, f) == getattr(ref, f), f
    assert list(d.sections) == [11, 11, 10, 0]
    assert d.window == 0 and k_blocks(d) == 64
    assert abs(d.rms_eps - 1e-6) < 1e-12 and d.rope_freq_base == 1e7
    with pytest.raises(QsaError):
        layer_desc(hp, 2, n_ctx=4096)                  # a recurrent layer


def test_defaults_and_context_rounding(tmp_path):
    """Absent optional keys take the reference loader's defaults; n_ctx is rounded up to whole blocks."""
    kv = {k: v for k, v in STANDIN.items()
          if not k.startswith(("rope.", "attention.indexer.", "full_attention", "attention.layer_norm"))}
    kv["block_count"] = 4
    kv["attention.compress_ratios"] = [0, 0, 0, 64]
    p = tmp_path / "defaults.gguf"
    write_gguf(p, kv)
    hp = read_hparams(str(p))
    assert hp["rope_freq_base"] == 1e7 and hp["rope_dim"] == 64 and hp["sections"] == [11, 11, 10, 0]
    assert (hp["idx_n_head"], hp["idx_dim"], hp["idx_top_k"]) == (4, 128, 2048)
    assert hp["full_attention_interval"] == 4 and abs(hp["rms_eps"] - 1e-6) < 1e-12
    d = layer_desc(hp, 3, n_ctx=1000)
    assert d.n_ctx == 1024 and k_blocks(d) == (2048 + 63 + 63) // 64


def test_checkpoint_shape_is_refused_cleanly(tmp_path):
    """The shipped checkpoint's attention (24 query heads on 2 KV heads, ratio 4, 4 indexer heads):
    12 query heads per KV head is beyond what these kernels pack (8), so the descriptor is refused
    with QSA_ERR_UNSUPPORTED rather than run."""
    kv = dict(STANDIN, **{"attention.head_count": 24, "attention.compress_ratios": [0, 0, 0, 4, 0, 0, 0, 4],
                          "attention.indexer.head_count": 4, "attention.indexer.top_k": 2048})
    p = tmp_path / "ckpt.gguf"
    write_gguf(p, kv)
    hp = read_hparams(str(p))
    assert qsa_layers(hp) == [3, 7]
    with pytest.raises(QsaError) as e:
        layer_desc(hp, 7, n_ctx=262144)
    assert e.value.status == QSA_ERR_UNSUPPORTED


def test_c_reader_typed_getters(tmp_path):
    """The library's C reader follows the reference loader's getters: integer keys of any integer
    width, f32 keys only when stored as F32 (an F64 value falls back to the default), integer
    arrays of 64-bit elements, a partial sections array completed from the defaults."""
    from gguf import GGUFValueType, GGUFWriter

    p = tmp_path / "typed.gguf"
    w = GGUFWriter(str(p), "qwen4exp")
    A = "qwen4exp."
    w.add_uint64(A + "block_count", 4)
    w.add_uint16(A + "attention.head_count", 16)
    w.add_int32(A + "attention.head_count_kv", 2)
    w.add_uint32(A + "attention.key_length", 256)
    w.add_uint32(A + "embedding_length", 2560)
    w.add_float64(A + "attention.layer_norm_rms_epsilon", 1e-5)      # not F32: the default 1e-6 holds
    w.add_array(A + "attention.compress_ratios", [0, 0, 0, 64])
    w.add_key_value(A + "rope.dimension_sections", [12, 12], GGUFValueType.ARRAY, sub_type=GGUFValueType.INT64)
    w.add_uint8(A + "attention.indexer.head_count", 1)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    hp = read_hparams(str(p))
    assert (hp["n_layer"], hp["n_head"], hp["n_head_kv"], hp["idx_n_head"]) == (4, 16, 2, 1)
    assert abs(hp["rms_eps"] - 1e-6) < 1e-12
    assert hp["compress_ratios"] == [0, 0, 0, 64]
    assert hp["sections"] == [12, 12, 10, 0]
    assert qsa_layers(hp) == [3]


def test_c_reader_refusals(tmp_path):
    """Another architecture is refused as the reference loader refuses it; a file that is not GGUF
    or is cut short is reported, not read past its end."""
    from gguf import GGUFWriter

    p = tmp_path / "other.gguf"
    w = GGUFWriter(str(p), "llama")
    w.add_uint32("llama.block_count", 2)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(QsaError) as e:
        read_hparams(str(p))
    assert e.value.status == QSA_ERR_UNSUPPORTED and "architecture" in str(e.value)
    junk = tmp_path / "junk.gguf"
    junk.write_bytes(b"not a gguf file at all")
    with pytest.raises(QsaError):
        read_hparams(str(junk))
    good = tmp_path / "standin.gguf"
    write_gguf(good, STANDIN)
    cut = tmp_path / "cut.gguf"
    cut.write_bytes(good.read_bytes()[:100])
    with pytest.raises(QsaError):
        read_hparams(str(cut))
    with pytest.raises(QsaError):
        read_hparams(str(tmp_path / "missing.gguf"))
