"""ctypes view of include/qsa.h and the loader of libqsa.so.

This is the binding a Python caller of the C ABI writes; the structures mirror the header field
for field.  The library is loaded from this package directory (built in-tree by
``qwfnfer_b200.build``); there is no fallback: a missing library is an ImportError-like failure.
"""
from __future__ import annotations

import ctypes
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libqsa.so")

QSA_OK = 0
QSA_ERR_INVALID, QSA_ERR_CUDA, QSA_ERR_TIMEOUT, QSA_ERR_UNSUPPORTED, QSA_ERR_WORKSPACE, QSA_ERR_DEVICE_ARG = 1, 2, 3, 4, 5, 6
STATUS_NAMES = {
    0: "QSA_OK", 1: "QSA_ERR_INVALID", 2: "QSA_ERR_CUDA", 3: "QSA_ERR_TIMEOUT",
    4: "QSA_ERR_UNSUPPORTED", 5: "QSA_ERR_WORKSPACE", 6: "QSA_ERR_DEVICE_ARG",
}

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_BF16 = 0, 1, 8, 30
KV_HOST, IDX_HOST = 1, 2          # qsa_desc.placement bits


class QsaDesc(ctypes.Structure):
    """struct qsa_desc (include/qsa.h)."""
    _fields_ = [
        ("n_head", ctypes.c_int32), ("n_head_kv", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("idx_n_head", ctypes.c_int32), ("idx_dim", ctypes.c_int32), ("ratio", ctypes.c_int32),
        ("top_k_blocks", ctypes.c_int32), ("window", ctypes.c_int32), ("n_ctx", ctypes.c_int32),
        ("type_k", ctypes.c_int32), ("type_v", ctypes.c_int32), ("rope_dim", ctypes.c_int32),
        ("sections", ctypes.c_int32 * 4), ("rms_eps", ctypes.c_float),
        ("rope_freq_base", ctypes.c_float), ("k_norm_w", ctypes.c_void_p), ("placement", ctypes.c_uint32),
    ]

    def copy(self) -> "QsaDesc":
        d = QsaDesc()
        ctypes.pointer(d)[0] = self
        return d


class QsaLayerCache(ctypes.Structure):
    """struct qsa_layer_cache."""
    _fields_ = [("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                ("idx", ctypes.c_void_p), ("pool", ctypes.c_void_p)]


class QsaDecodeItem(ctypes.Structure):
    """struct qsa_decode_item (48 bytes)."""
    _fields_ = [("cache", QsaLayerCache), ("n_past", ctypes.c_int32),
                ("reserved", ctypes.c_int32 * 3)]


class QsaPeerSlots(ctypes.Structure):
    """struct qsa_peer_slots: one channel of the NVLink peer exchange (every rank's gather region
    of it in this process, the rank count and index, this rank's epoch counter of the channel)."""
    _fields_ = [("region", ctypes.c_void_p * 8), ("n_ranks", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("epoch", ctypes.c_void_p)]


class QsaFrontWeights(ctypes.Structure):
    """struct qsa_front_weights (include/qsa.h)."""
    _fields_ = [("wq", ctypes.c_void_p), ("wk", ctypes.c_void_p), ("wv", ctypes.c_void_p),
                ("wq_idx", ctypes.c_void_p), ("wk_idx", ctypes.c_void_p),
                ("q_norm", ctypes.c_void_p), ("k_norm", ctypes.c_void_p), ("q_idx_norm", ctypes.c_void_p),
                ("n_embd", ctypes.c_int32), ("w_type", ctypes.c_int32)]


GGUF_MAX_LAYERS = 256


class QsaGgufHparams(ctypes.Structure):
    """struct qsa_gguf_hparams (include/qsa.h)."""
    _fields_ = [
        ("arch", ctypes.c_char * 64), ("n_layer", ctypes.c_int32), ("n_embd", ctypes.c_int32),
        ("n_ctx_train", ctypes.c_int32), ("n_head", ctypes.c_int32), ("n_head_kv", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("rms_eps", ctypes.c_float), ("full_attention_interval", ctypes.c_int32),
        ("n_compress", ctypes.c_int32), ("compress_ratios", ctypes.c_int32 * GGUF_MAX_LAYERS),
        ("rope_freq_base", ctypes.c_float), ("rope_dim", ctypes.c_int32), ("sections", ctypes.c_int32 * 4),
        ("idx_n_head", ctypes.c_int32), ("idx_dim", ctypes.c_int32), ("idx_top_k", ctypes.c_int32),
    ]


def make_desc(n_head=16, n_head_kv=2, head_dim=256, idx_n_head=1, idx_dim=128, ratio=64,
              top_k_blocks=64, window=128, n_ctx=4096, type_k=TYPE_Q8_0, type_v=TYPE_Q8_0,
              rope_dim=64, sections=(11, 11, 10, 0), rms_eps=1e-6, rope_freq_base=1e7,
              k_norm_w=None, kv_host=False, idx_host=False) -> QsaDesc:
    d = QsaDesc()
    d.n_head, d.n_head_kv, d.head_dim = n_head, n_head_kv, head_dim
    d.idx_n_head, d.idx_dim, d.ratio = idx_n_head, idx_dim, ratio
    d.top_k_blocks, d.window, d.n_ctx = top_k_blocks, window, n_ctx
    d.type_k, d.type_v, d.rope_dim = type_k, type_v, rope_dim
    for i in range(4):
        d.sections[i] = sections[i]
    d.rms_eps, d.rope_freq_base = rms_eps, rope_freq_base
    d.k_norm_w = k_norm_w
    d.placement = (KV_HOST if kv_host else 0) | (IDX_HOST if idx_host else 0)
    return d


def k_blocks(d: QsaDesc) -> int:
    """KB: top_k_blocks plus the forced-window blocks (qsa_k_blocks)."""
    nf = (d.window + d.ratio - 1) // d.ratio + 1 if d.window > 0 else 1
    return d.top_k_blocks + nf


def row_bytes(d: QsaDesc, which: int) -> int:
    kv_dim = d.n_head_kv * d.head_dim
    if which in (0, 1):
        t = d.type_k if which == 0 else d.type_v
        return kv_dim // 32 * 34 if t == TYPE_Q8_0 else kv_dim * 2
    return d.idx_dim * 2


_lib = None


class QsaError(RuntimeError):
    def __init__(self, status: int, where: str):
        super().__init__(f"{where}: {STATUS_NAMES.get(status, status)}")
        self.status = status


def lib() -> ctypes.CDLL:
    """Load libqsa.so (built in-tree).  Raises if it is missing: there is no other path."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libqsa.so is not built ({LIB_PATH}); run __graft_entry__.build()")
    L = ctypes.CDLL(LIB_PATH)
    P, I32, SZ, VP = ctypes.POINTER, ctypes.c_int32, ctypes.c_size_t, ctypes.c_void_p
    D = P(QsaDesc)
    C = P(QsaLayerCache)
    sigs = {
        "qsa_status_string": (ctypes.c_char_p, [I32]),
        "qsa_desc_check": (I32, [D]),
        "qsa_k_blocks": (I32, [D]),
        "qsa_row_bytes": (SZ, [D, I32]),
        "qsa_cache_bytes": (SZ, [D, I32]),
        "qsa_append": (I32, [D, C, I32, I32, VP, VP, VP, VP]),
        "qsa_pool_rebuild": (I32, [D, C, I32, I32, VP, VP]),
        "qsa_decode_workspace_size": (SZ, [D, I32, I32]),
        "qsa_shard_workspace_size": (SZ, [D, I32, I32, I32, I32]),
        "qsa_workspace_init": (I32, [VP, SZ, VP]),
        "qsa_decode": (I32, [D, VP, I32, I32, VP, I32, VP, VP, VP, VP, VP, VP, VP, SZ, VP]),
        "qsa_decode_append": (I32, [D, VP, I32, I32, VP, VP, VP, VP, SZ, VP]),
        "qsa_decode_select": (I32, [D, VP, I32, I32, VP, VP, VP, SZ, VP]),
        "qsa_decode_attend": (I32, [D, VP, I32, I32, VP, I32, VP, VP, SZ, VP]),
        "qsa_decode_noalloc": (I32, [D, VP, I32, I32, VP, I32, VP, VP, VP, VP, VP, VP, VP]),
        "qsa_decode_gated": (I32, [D, VP, I32, I32, VP, I32, VP, VP, VP, VP, VP, VP, I32, VP, VP, VP, SZ, VP]),
        "qsa_prefill_gated": (I32, [D, C, I32, I32, VP, I32, VP, VP, VP, VP, VP, VP, I32, VP, VP, VP, SZ, VP]),
        "qsa_output_z": (I32, [D, VP, I32, I32, I32, VP, I32, VP, VP, SZ, VP]),
        "qsa_shard_state_floats": (SZ, [D]),
        "qsa_shard_append": (I32, [D, C, I32, I32, I32, I32, VP, VP, VP, VP]),
        "qsa_shard_append_ri": (I32, [D, C, I32, I32, I32, I32, VP, VP, VP, VP]),
        "qsa_shard_decode_ri": (I32, [D, VP, I32, I32, I32, I32, VP, I32, VP, VP, VP, VP, VP, VP, VP, SZ, VP]),
        "qsa_shard_candidates": (I32, [D, VP, I32, I32, I32, I32, VP, VP, VP, VP, VP, VP, SZ, VP]),
        "qsa_shard_attend": (I32, [D, VP, I32, I32, I32, I32, I32, VP, I32, VP, I32, VP, VP, VP, SZ, VP]),
        "qsa_merge_states": (I32, [D, I32, I32, VP, VP, VP]),
        "qsa_decode_sharded_workspace_size": (SZ, [D, I32, I32, I32, I32, I32]),
        "qsa_decode_sharded": (I32, [D, VP, I32, I32, I32, I32, I32, VP, I32, VP, I32, VP, VP, VP, VP, VP, VP, VP, SZ, VP]),
        "qsa_ipc_handle": (I32, [VP, VP, P(SZ)]),
        "qsa_ipc_open": (I32, [VP, P(VP)]),
        "qsa_ipc_close": (I32, [VP]),
        "qsa_peer_buffer_bytes": (SZ, [I32, SZ]),
        "qsa_peer_push": (I32, [VP, I32, I32, VP, SZ, VP, VP, VP]),
        "qsa_peer_wait": (I32, [VP, I32, SZ, VP, VP, SZ, VP]),
        "qsa_shard_decode_ri_peer": (I32, [D, VP, I32, I32, I32, I32, VP, I32, VP, VP, VP, VP, P(QsaPeerSlots), VP, VP,
                                           SZ, VP]),
        "qsa_merge_states_peer": (I32, [D, P(QsaPeerSlots), I32, VP, VP, SZ, VP]),
        "qsa_prefill_workspace_size": (SZ, [D, I32, I32]),
        "qsa_prefill": (I32, [D, C, I32, I32, VP, I32, VP, VP, VP, VP, VP, VP, VP, SZ, VP]),
        "qsa_check": (I32, [VP, SZ, VP]),
        "qsa_stage_copy": (I32, [VP, VP, SZ, VP]),
        "qsa_front_workspace_size": (SZ, [D, P(QsaFrontWeights), I32]),
        "qsa_front": (I32, [D, P(QsaFrontWeights), I32, VP, VP, VP, VP, VP, VP, VP, VP, VP, SZ, VP]),
        "qsa_output_workspace_size": (SZ, [D, I32, I32, I32]),
        "qsa_output": (I32, [D, VP, I32, I32, I32, VP, VP, VP, VP, SZ, VP]),
        "qsa_version": (I32, []),
        "qsa_gguf_read_hparams": (I32, [ctypes.c_char_p, P(QsaGgufHparams), ctypes.c_char_p, SZ]),
        "qsa_gguf_is_qsa_layer": (I32, [P(QsaGgufHparams), I32]),
        "qsa_gguf_layer_desc": (I32, [P(QsaGgufHparams), I32, I32, I32, I32, I32, VP, D]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype, fn.argtypes = res, args
    _lib = L
    return L


def check(status: int, where: str) -> None:
    if status != QSA_OK:
        raise QsaError(status, where)


# Every symbol include/qsa.h declares (the CPU test checks the library exports each one).
HEADER_SYMBOLS = [
    "qsa_status_string", "qsa_desc_check", "qsa_k_blocks", "qsa_row_bytes", "qsa_cache_bytes",
    "qsa_append", "qsa_pool_rebuild", "qsa_decode_workspace_size", "qsa_workspace_init",
    "qsa_decode", "qsa_decode_append", "qsa_decode_select", "qsa_decode_attend", "qsa_decode_noalloc",
    "qsa_shard_state_floats", "qsa_shard_workspace_size", "qsa_shard_append", "qsa_shard_candidates", "qsa_shard_attend",
    "qsa_shard_append_ri", "qsa_shard_decode_ri",
    "qsa_merge_states", "qsa_decode_sharded_workspace_size", "qsa_decode_sharded",
    "qsa_ipc_handle", "qsa_ipc_open", "qsa_ipc_close", "qsa_peer_buffer_bytes", "qsa_peer_push", "qsa_peer_wait",
    "qsa_shard_decode_ri_peer", "qsa_merge_states_peer",
    "qsa_prefill_workspace_size", "qsa_prefill", "qsa_front_workspace_size", "qsa_front", "qsa_output_workspace_size", "qsa_output",
    "qsa_decode_gated", "qsa_prefill_gated", "qsa_output_z",
    "qsa_gguf_read_hparams", "qsa_gguf_is_qsa_layer", "qsa_gguf_layer_desc",
    "qsa_stage_copy",
    "qsa_check", "qsa_version",
]
