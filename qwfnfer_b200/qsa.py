"""Host-side mirror of the reference's QSA node interface over the C ABI (libqsa.so).

Names follow the reference so that callers and tests read like it:
  QsaState           qwfn::state (src/qwfn_state.cpp:18-96) K/V/idx caches of the attention layers
                     plus the engine's pooled-key cache (src/qwfn_engine.cpp:389-397)
  QsaNode.sparse_attn_decode   graph_builder::sparse_attn_decode (src/qwfn_graph.cpp:450-546)
  QsaNode.sparse_attn          graph_builder::sparse_attn / qsa_top_k (src/qwfn_graph.cpp:235-408)
  QsaNode.qsa_pool_rebuild     graph_builder::qsa_pool_rebuild (src/qwfn_graph.cpp:431-448)
Errors raise QsaError carrying the qsa_status (the reference aborts; the library never does).
PyTorch provides device memory and streams only; every computation runs in libqsa.so.
"""
from __future__ import annotations

import ctypes

import torch

from . import _abi
from ._abi import (QsaDecodeItem, QsaDesc, QsaError, QsaLayerCache, TYPE_BF16, TYPE_F32, check, k_blocks,
                   lib, row_bytes)


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    assert t.is_cuda and t.is_contiguous(), "device tensors must be contiguous CUDA tensors"
    return t.data_ptr()


def _stream(stream: torch.cuda.Stream | None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


class QsaState:
    """Per-sequence caches of `n_layers` QSA layers, reference layouts (include/qsa.h).

    blocks=(lo, hi): a shard's caches, holding blocks [lo, hi) only (row 0 = cell lo*ratio);
    with index_full the raw-key and pooled-key caches still cover every block (the sharded decode
    with replicated indexer caches)."""

    def __init__(self, desc: QsaDesc, n_layers: int = 1, device: str | torch.device = "cuda", zero: bool = False,
                 blocks: tuple[int, int] | None = None, index_full: bool = False):
        check(lib().qsa_desc_check(ctypes.byref(desc)), "qsa_desc_check")
        self.desc = desc
        self.device = torch.device(device)
        self.blocks = blocks if blocks is not None else (0, desc.n_ctx // desc.ratio)
        n = (self.blocks[1] - self.blocks[0]) * desc.ratio
        ni = desc.n_ctx if index_full else n
        alloc = torch.zeros if zero else torch.empty
        self.k = [alloc((n, row_bytes(desc, 0)), dtype=torch.uint8, device=self.device) for _ in range(n_layers)]
        self.v = [alloc((n, row_bytes(desc, 1)), dtype=torch.uint8, device=self.device) for _ in range(n_layers)]
        self.idx = [alloc((ni, desc.idx_dim), dtype=torch.int16, device=self.device) for _ in range(n_layers)]
        self.pool = [torch.zeros((ni // desc.ratio, desc.idx_dim), dtype=torch.int16, device=self.device)
                     for _ in range(n_layers)]

    def layer(self, il: int = 0) -> QsaLayerCache:
        c = QsaLayerCache()
        c.k, c.v, c.idx, c.pool = (self.k[il].data_ptr(), self.v[il].data_ptr(),
                                   self.idx[il].data_ptr(), self.pool[il].data_ptr())
        return c

    def bytes(self) -> int:
        return sum(t.numel() * t.element_size() for ts in (self.k, self.v, self.idx, self.pool) for t in ts)


def decode_items(caches: list[QsaLayerCache], n_past: list[int], device="cuda") -> torch.Tensor:
    """Device table of qsa_decode_item (48 bytes each) for qsa_decode."""
    arr = (QsaDecodeItem * len(caches))()
    for i, (c, n) in enumerate(zip(caches, n_past)):
        arr[i].cache = c
        arr[i].n_past = int(n)
    raw = bytes(arr)
    host = torch.frombuffer(bytearray(raw), dtype=torch.uint8)
    return host.to(device)


def set_n_past(items: torch.Tensor, n_past: list[int]) -> None:
    """Rewrite the n_past fields of a device item table in place (the per-token update)."""
    stride = ctypes.sizeof(QsaDecodeItem)
    off = QsaDecodeItem.n_past.offset
    view = items.view(-1, stride)
    vals = torch.tensor(n_past, dtype=torch.int32).view(torch.uint8).view(-1, 4)
    view[:, off:off + 4] = vals.to(items.device)


class QsaNode:
    """The QSA node of one layer description; workspaces are sized per call shape and cached."""

    def __init__(self, desc: QsaDesc, device: str | torch.device = "cuda"):
        check(lib().qsa_desc_check(ctypes.byref(desc)), "qsa_desc_check")
        self.desc = desc
        self.device = torch.device(device)
        self.kb = k_blocks(desc)
        self._ws: dict[tuple, torch.Tensor] = {}

    def workspace(self, kind: str, n_q: int, max_n_kv: int, stream=None) -> torch.Tensor:
        fn = lib().qsa_decode_workspace_size if kind == "decode" else lib().qsa_prefill_workspace_size
        size = fn(ctypes.byref(self.desc), n_q, max_n_kv)
        if size == 0:
            raise QsaError(_abi.QSA_OK + 1, "workspace size")
        key = (kind, size)
        ws = self._ws.get(key)
        if ws is None:
            ws = torch.empty(size, dtype=torch.uint8, device=self.device)
            check(lib().qsa_workspace_init(ws.data_ptr(), size, _stream(stream)), "qsa_workspace_init")
            self._ws[key] = ws
        return ws

    # ------------------------------------------------------------------ append / pool
    def append(self, cache: QsaLayerCache, pos0: int, k: torch.Tensor | None, v: torch.Tensor | None,
               kidx: torch.Tensor | None, stream=None) -> None:
        n = (k if k is not None else kidx).shape[0]
        check(lib().qsa_append(ctypes.byref(self.desc), ctypes.byref(cache), pos0, n, _ptr(k), _ptr(v), _ptr(kidx),
                               _stream(stream)), "qsa_append")

    def qsa_pool_rebuild(self, cache: QsaLayerCache, n_whole: int, blk0: int = 0,
                         pooled_f32: torch.Tensor | None = None, stream=None) -> None:
        check(lib().qsa_pool_rebuild(ctypes.byref(self.desc), ctypes.byref(cache), blk0, n_whole, _ptr(pooled_f32),
                                     _stream(stream)), "qsa_pool_rebuild")

    # ------------------------------------------------------------------ decode / prefill
    def sparse_attn_decode(self, items: torch.Tensor, batch: int, max_n_kv: int, q: torch.Tensor,
                           q_idx: torch.Tensor, k_new=None, v_new=None, kidx_new=None,
                           out: torch.Tensor | None = None, sel_out: torch.Tensor | None = None,
                           ws: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        d = self.desc
        if out is None:
            out = torch.empty((batch, d.n_head, d.head_dim), dtype=torch.float32, device=self.device)
        q_type = TYPE_BF16 if q.dtype == torch.bfloat16 else TYPE_F32
        if ws is None:
            ws = self.workspace("decode", batch, max_n_kv, stream)
        check(lib().qsa_decode(ctypes.byref(d), _ptr(items), batch, max_n_kv, _ptr(q), q_type, _ptr(q_idx),
                               _ptr(k_new), _ptr(v_new), _ptr(kidx_new), _ptr(out), _ptr(sel_out),
                               ws.data_ptr(), ws.numel(), _stream(stream)), "qsa_decode")
        return out

    def sparse_attn(self, cache: QsaLayerCache, n_past: int, q: torch.Tensor, q_idx: torch.Tensor,
                    k_new=None, v_new=None, kidx_new=None, out: torch.Tensor | None = None,
                    sel_out: torch.Tensor | None = None, ws: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        d = self.desc
        T = q.shape[0]
        if out is None:
            out = torch.empty((T, d.n_head, d.head_dim), dtype=torch.float32, device=self.device)
        q_type = TYPE_BF16 if q.dtype == torch.bfloat16 else TYPE_F32
        if ws is None:
            ws = self.workspace("prefill", T, n_past + T, stream)
        check(lib().qsa_prefill(ctypes.byref(d), ctypes.byref(cache), n_past, T, _ptr(q), q_type, _ptr(q_idx),
                                _ptr(k_new), _ptr(v_new), _ptr(kidx_new), _ptr(out), _ptr(sel_out),
                                ws.data_ptr(), ws.numel(), _stream(stream)), "qsa_prefill")
        return out

    def check(self, ws: torch.Tensor, stream=None) -> int:
        """qsa_check: synchronise and return (and clear) the device status as a qsa_status."""
        return lib().qsa_check(ws.data_ptr(), ws.numel(), _stream(stream))
