"""numpy binding of the CPU oracle (oracle/libqsa_oracle.so).

TEST INFRASTRUCTURE ONLY: loaded by tests/, __graft_entry__.smoke() and bench.py's CPU legs as
the checker / CPU baseline.  The product (qwfnfer_b200, libqsa.so) never imports it.
Each wrapper names the function of qsa_oracle.cpp it calls; that file cites the reference lines.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from qwfnfer_b200._abi import QsaDesc, TYPE_BF16, TYPE_F32, TYPE_Q8_0, k_blocks, row_bytes

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqsa_oracle.so")

# orc_attend flags (qsa_oracle.cpp)
KV_F16_ROUND, Q_F16, GGML_FA, GGML_V_F16 = 1, 2, 4, 8
DEFAULT_FLAGS = KV_F16_ROUND | Q_F16

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} missing: run `make -C oracle` or __graft_entry__.build()")
        L = ctypes.CDLL(LIB_PATH)
        VP, I64, I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32
        D = ctypes.POINTER(QsaDesc)
        sigs = {
            "orc_version": (ctypes.c_int, []),
            "orc_max_threads": (ctypes.c_int, []),
            "orc_set_threads": (None, [ctypes.c_int]),
            "orc_f32_to_f16": (None, [VP, VP, I64]),
            "orc_f16_to_f32": (None, [VP, VP, I64]),
            "orc_q8_0_quantize": (None, [VP, VP, I64]),
            "orc_q8_0_dequantize": (None, [VP, VP, I64]),
            "orc_append": (None, [D, VP, VP, VP, I64, I64, VP, VP, VP]),
            "orc_pool_blocks": (None, [D, VP, I64, I64, VP, VP, VP]),
            "orc_scores": (None, [D, VP, I64, I64, VP, VP]),
            "orc_select": (ctypes.c_int, [D, VP, I64, VP, VP]),
            "orc_attend": (None, [D, VP, VP, I64, VP, VP, I64, VP, I32, VP, I32]),
            "orc_attend_state": (None, [D, VP, VP, I64, VP, VP, I64, VP, I32, VP, I32]),
            "orc_k_blocks": (ctypes.c_int, [D]),
            "orc_node": (None, [D, VP, VP, VP, I64, VP, VP, I32, VP, VP, VP, VP, I32]),
            "orc_front": (None, [D, VP, VP, VP, VP, VP, VP, VP, VP, I64, I64, VP, VP, VP, VP, VP, VP, VP, VP]),
            "orc_output": (None, [D, VP, I64, I64, VP, VP, VP]),
            "orc_front_w": (None, [D, I32, VP, VP, VP, VP, VP, VP, VP, VP, I64, I64, VP, VP, VP, VP, VP, VP, VP, VP]),
            "orc_output_w": (None, [D, I32, VP, I64, I64, VP, VP, VP]),
        }
        for name, (res, args) in sigs.items():
            fn = getattr(L, name)
            fn.restype, fn.argtypes = res, args
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def max_threads() -> int:
    return lib().orc_max_threads()


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_f16(_p(x), _p(y), x.size)
    return y


def f16_to_f32(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    y = np.empty(x.shape, dtype=np.float32)
    lib().orc_f16_to_f32(_p(x), _p(y), x.size)
    return y


def q8_0_quantize(x: np.ndarray) -> np.ndarray:
    """f32 [..., n] (n % 32 == 0) -> uint8 [..., n//32*34]  (orc_q8_0_quantize)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    out = np.empty(x.shape[:-1] + (n // 32 * 34,), dtype=np.uint8)
    lib().orc_q8_0_quantize(_p(x), _p(out), x.size)
    return out


def q8_0_dequantize(q: np.ndarray) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.uint8)
    nb = q.shape[-1] // 34
    out = np.empty(q.shape[:-1] + (nb * 32,), dtype=np.float32)
    lib().orc_q8_0_dequantize(_p(q), _p(out), out.size)
    return out


def append(d: QsaDesc, kc: np.ndarray, vc: np.ndarray, ic: np.ndarray, pos0: int,
           k: np.ndarray | None, v: np.ndarray | None, kidx: np.ndarray | None) -> None:
    """Write rows [pos0, pos0+n) of the byte caches kc/vc (uint8 [n_ctx, row_bytes]) and the F16
    idx cache ic (uint16 [n_ctx, idx_dim]) in place (orc_append)."""
    n = (k if k is not None else kidx).shape[0]
    f = lambda a: None if a is None else np.ascontiguousarray(a, dtype=np.float32)
    k, v, kidx = f(k), f(v), f(kidx)
    lib().orc_append(ctypes.byref(d), _p(kc), _p(vc), _p(ic), pos0, n, _p(k), _p(v), _p(kidx))


def pool_blocks(d: QsaDesc, ic: np.ndarray, blk0: int, n_blk: int, k_norm_w: np.ndarray | None = None):
    """Pooled keys of blocks [blk0, blk0+n_blk): (f32 [n_blk, idx_dim], f16 bits [n_blk, idx_dim])."""
    out32 = np.empty((n_blk, d.idx_dim), dtype=np.float32)
    out16 = np.empty((n_blk, d.idx_dim), dtype=np.uint16)
    w = None if k_norm_w is None else np.ascontiguousarray(k_norm_w, dtype=np.float32)
    lib().orc_pool_blocks(ctypes.byref(d), _p(np.ascontiguousarray(ic)), blk0, n_blk, _p(w), _p(out32), _p(out16))
    return out32, out16


def scores(d: QsaDesc, pool: np.ndarray, nb: int, q_idx: np.ndarray) -> np.ndarray:
    """Head-summed relu scores of n_q queries against blocks [0, nb): f32 [n_q, nb]."""
    q_idx = np.ascontiguousarray(q_idx, dtype=np.float32).reshape(-1, d.idx_n_head * d.idx_dim)
    out = np.empty((q_idx.shape[0], nb), dtype=np.float32)
    lib().orc_scores(ctypes.byref(d), _p(np.ascontiguousarray(pool)), nb, q_idx.shape[0], _p(q_idx), _p(out))
    return out


def select(d: QsaDesc, sc: np.ndarray, q: int):
    """(sel int32 [KB] ascending -1 padded, forced uint8 [KB]) for the query at position q."""
    KB = k_blocks(d)
    sel = np.empty(KB, dtype=np.int32)
    forced = np.empty(KB, dtype=np.uint8)
    sc = np.ascontiguousarray(sc, dtype=np.float32)
    lib().orc_select(ctypes.byref(d), _p(sc), q, _p(sel), _p(forced))
    return sel, forced


def attend(d: QsaDesc, kc: np.ndarray, vc: np.ndarray, q_pos, sel: np.ndarray, Q: np.ndarray,
           q_type: int = TYPE_F32, flags: int = DEFAULT_FLAGS) -> np.ndarray:
    """Attention of n_q queries over their selected blocks: f32 [n_q, n_head, head_dim].
    Q is f32, or uint16 bf16 bits with q_type=TYPE_BF16."""
    q_pos = np.ascontiguousarray(np.atleast_1d(q_pos), dtype=np.int64)
    n_q = q_pos.size
    sel = np.ascontiguousarray(sel, dtype=np.int32).reshape(n_q, -1)
    Q = np.ascontiguousarray(Q)
    assert Q.size == n_q * d.n_head * d.head_dim
    out = np.empty((n_q, d.n_head, d.head_dim), dtype=np.float32)
    lib().orc_attend(ctypes.byref(d), _p(np.ascontiguousarray(kc)), _p(np.ascontiguousarray(vc)), n_q,
                     _p(q_pos), _p(sel), sel.shape[1], _p(Q), q_type, _p(out), flags)
    return out


def attend_state(d: QsaDesc, kc: np.ndarray, vc: np.ndarray, q_pos, sel: np.ndarray, Q: np.ndarray,
                 q_type: int = TYPE_F32, flags: int = DEFAULT_FLAGS) -> np.ndarray:
    """Unnormalised attention state f32 [n_q, 32 + 16*head_dim] ([M 16][L 16][O 16 x hd], rows
    8*kv_head + head, M in the log2 domain) over the selected blocks; orc_attend_state."""
    q_pos = np.ascontiguousarray(np.atleast_1d(q_pos), dtype=np.int64)
    n_q = q_pos.size
    sel = np.ascontiguousarray(sel, dtype=np.int32).reshape(n_q, -1)
    Q = np.ascontiguousarray(Q)
    out = np.empty((n_q, 32 + 16 * d.head_dim), dtype=np.float32)
    lib().orc_attend_state(ctypes.byref(d), _p(np.ascontiguousarray(kc)), _p(np.ascontiguousarray(vc)), n_q,
                           _p(q_pos), _p(sel), sel.shape[1], _p(Q), q_type, _p(out), flags)
    return out


def merge_states(d: QsaDesc, states: np.ndarray) -> np.ndarray:
    """Log-sum-exp merge of states [n_parts, n_q, 32 + 16*hd] -> f32 [n_q, n_head, hd], in double:
    M = max_p M_p;  out = sum_p 2^(M_p - M) O_p / sum_p 2^(M_p - M) L_p."""
    P, n_q, _ = states.shape
    hd, gqa = d.head_dim, d.n_head // d.n_head_kv
    M = states[:, :, :16].astype(np.float64)
    L = states[:, :, 16:32].astype(np.float64)
    O = states[:, :, 32:].astype(np.float64).reshape(P, n_q, 16, hd)
    Mx = M.max(axis=0)
    Mu = np.where(np.isneginf(Mx), 0.0, Mx)
    w = np.exp2(M - Mu[None])                                   # [P, n_q, 16]
    Ls = (w * L).sum(axis=0)
    Os = (w[..., None] * O).sum(axis=0)
    res = np.where(Ls[..., None] > 0, Os / np.where(Ls > 0, Ls, 1.0)[..., None], 0.0)
    rows = [8 * g + h for g in range(d.n_head_kv) for h in range(gqa)]
    return res[:, rows, :].astype(np.float32)


def node(d: QsaDesc, kc, vc, pool, q_pos, Q, q_idx, q_type: int = TYPE_F32, flags: int = DEFAULT_FLAGS):
    """Scores + selection + attention for queries at q_pos over caches whose pooled keys are
    current.  Returns (out f32 [n_q, n_head, hd], sel int32 [n_q, KB], scores f32 [n_q, nb])."""
    q_pos = np.ascontiguousarray(np.atleast_1d(q_pos), dtype=np.int64)
    n_q = q_pos.size
    KB = k_blocks(d)
    nb = max(int((q_pos.max() + 1) // d.ratio), 1)
    out = np.empty((n_q, d.n_head, d.head_dim), dtype=np.float32)
    sel = np.empty((n_q, KB), dtype=np.int32)
    sc = np.zeros((n_q, nb), dtype=np.float32)
    q_idx = np.ascontiguousarray(q_idx, dtype=np.float32)
    lib().orc_node(ctypes.byref(d), _p(np.ascontiguousarray(kc)), _p(np.ascontiguousarray(vc)),
                   _p(np.ascontiguousarray(pool)), n_q, _p(q_pos), _p(np.ascontiguousarray(Q)), q_type,
                   _p(q_idx), _p(out), _p(sel), _p(sc), flags)
    return out, sel, sc


def cache_arrays(d: QsaDesc):
    """Zeroed host caches in the reference layouts: (K bytes, V bytes, idx f16, pool f16)."""
    n = d.n_ctx
    return (np.zeros((n, row_bytes(d, 0)), np.uint8), np.zeros((n, row_bytes(d, 1)), np.uint8),
            np.zeros((n, d.idx_dim), np.uint16), np.zeros((n // d.ratio, d.idx_dim), np.uint16))


def front(d: QsaDesc, w: dict, pos: np.ndarray, x: np.ndarray, w_type: int = TYPE_BF16) -> dict:
    """orc_front_w: the projections, norms and IMRoPE feeding the node for T tokens.
    w: wq, wk, wv, wq_idx, wk_idx as uint16 bf16 bits [out][n_embd] (w_type TYPE_BF16), or as uint8
    q8_0 rows [out][n_embd/32*34] (TYPE_Q8_0); q_norm, k_norm, q_idx_norm f32 (or None).
    pos int32 [T], x f32 [T][n_embd].  Returns q, gate, q_idx, k, v, kidx (f32)."""
    T, n_embd = x.shape
    hd, nh, nkv, H, D = d.head_dim, d.n_head, d.n_head_kv, d.idx_n_head, d.idx_dim
    out = {"q": np.zeros((T, nh, hd), np.float32), "gate": np.zeros((T, nh * hd), np.float32),
           "q_idx": np.zeros((T, H, D), np.float32), "k": np.zeros((T, nkv * hd), np.float32),
           "v": np.zeros((T, nkv * hd), np.float32), "kidx": np.zeros((T, D), np.float32)}
    wdt = np.uint8 if w_type == TYPE_Q8_0 else np.uint16
    ws = [np.ascontiguousarray(w[k], dtype=wdt) for k in ("wq", "wk", "wv", "wq_idx", "wk_idx")]
    ns = [None if w.get(k) is None else np.ascontiguousarray(w[k], dtype=np.float32)
          for k in ("q_norm", "k_norm", "q_idx_norm")]
    pos = np.ascontiguousarray(pos, dtype=np.int32)
    x = np.ascontiguousarray(x, dtype=np.float32)
    lib().orc_front_w(ctypes.byref(d), w_type, *[_p(a) for a in ws], *[_p(a) for a in ns], n_embd, T, _p(pos), _p(x),
                      *[_p(out[k]) for k in ("q", "gate", "q_idx", "k", "v", "kidx")])
    return out


def output(d: QsaDesc, wo: np.ndarray, attn: np.ndarray, gate: np.ndarray, w_type: int = TYPE_BF16) -> np.ndarray:
    """orc_output_w: y = attn_output (attn * sigmoid(gate)); wo uint16 bf16 bits [n_embd][n_head*head_dim]
    (or uint8 q8_0 rows with w_type TYPE_Q8_0), attn f32 [T][n_head][head_dim], gate f32
    [T][n_head*head_dim] -> y f32 [T][n_embd]."""
    wo = np.ascontiguousarray(wo, dtype=np.uint8 if w_type == TYPE_Q8_0 else np.uint16)
    attn = np.ascontiguousarray(attn, dtype=np.float32)
    gate = np.ascontiguousarray(gate, dtype=np.float32)
    T, n_embd = attn.shape[0], wo.shape[0]
    y = np.zeros((T, n_embd), np.float32)
    lib().orc_output_w(ctypes.byref(d), w_type, _p(wo), n_embd, T, _p(attn), _p(gate), _p(y))
    return y
