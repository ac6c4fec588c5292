"""Host-side mirror of the reference's QSA node interface over the C ABI (libqsa.so).

Names follow the reference so that callers and tests read like it:
  QsaState           qwfn::state (src/qwfn_state.cpp:18-96) K/V/idx caches of the attention layers
                     plus the engine's pooled-key cache (src/qwfn_engine.cpp:389-397)
  QsaNode.sparse_attn_decode   graph_builder::sparse_attn_decode (src/qwfn_graph.cpp:450-546)
  QsaNode.sparse_attn          graph_builder::sparse_attn / qsa_top_k (src/qwfn_graph.cpp:235-408)
  QsaNode.qsa_pool_rebuild     graph_builder::qsa_pool_rebuild (src/qwfn_graph.cpp:431-448)
  QsaDecodeStep      one captured decode step per token, as the engine computes one graph per step
                     (src/qwfn_engine.cpp:814)
  QsaFront           the projections, norms and IMRoPE feeding the node (src/qwfn_graph.cpp:465,
                     479-484, 505-518)
  QsaOutput          the gated output projection after it (src/qwfn_graph.cpp:543-545)
Errors raise QsaError carrying the qsa_status (the reference aborts; the library never does).
PyTorch provides device memory and streams only; every computation runs in libqsa.so.
"""
from __future__ import annotations

import ctypes

import torch

from . import _abi
from ._abi import (QsaDecodeItem, QsaDesc, QsaError, QsaFrontWeights, QsaLayerCache, TYPE_BF16, TYPE_F32, check,
                   k_blocks, lib, row_bytes)


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
    with replicated indexer caches).  The descriptor's placement puts K/V (KV_HOST) and/or the raw
    indexer keys (IDX_HOST) in pinned host memory, as state_config's kv_host / idx_host do
    (src/qwfn_state.h:31-36); the pooled keys stay on the device."""

    def __init__(self, desc: QsaDesc, n_layers: int = 1, device: str | torch.device = "cuda", zero: bool = False,
                 blocks: tuple[int, int] | None = None, index_full: bool = False):
        check(lib().qsa_desc_check(ctypes.byref(desc)), "qsa_desc_check")
        self.desc = desc
        self.device = torch.device(device)
        self.blocks = blocks if blocks is not None else (0, desc.n_ctx // desc.ratio)
        n = (self.blocks[1] - self.blocks[0]) * desc.ratio
        ni = desc.n_ctx if index_full else n
        def alloc(shape, dtype, host):
            if host:                       # pinned, mapped into the device's address space (UVA)
                t = torch.empty(shape, dtype=dtype, pin_memory=True)
                return t.zero_() if zero else t
            return (torch.zeros if zero else torch.empty)(shape, dtype=dtype, device=self.device)

        kv_host, idx_host = bool(desc.placement & _abi.KV_HOST), bool(desc.placement & _abi.IDX_HOST)
        self.k = [alloc((n, row_bytes(desc, 0)), torch.uint8, kv_host) for _ in range(n_layers)]
        self.v = [alloc((n, row_bytes(desc, 1)), torch.uint8, kv_host) for _ in range(n_layers)]
        self.idx = [alloc((ni, desc.idx_dim), torch.int16, idx_host) for _ in range(n_layers)]
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

    def sparse_attn_decode_gated(self, items: torch.Tensor, batch: int, max_n_kv: int, q: torch.Tensor,
                                 q_idx: torch.Tensor, gate: torch.Tensor, k_new=None, v_new=None, kidx_new=None,
                                 z_dtype=torch.bfloat16, out: torch.Tensor | None = None,
                                 sel_out: torch.Tensor | None = None, ws: torch.Tensor | None = None,
                                 stream=None) -> torch.Tensor:
        """qsa_decode_gated: the decode with the output gate applied in the attention's final store;
        returns z = out * sigmoid(gate) [batch][n_head*head_dim] in z_dtype (bf16 or f32); `out`
        (optional) also receives the ungated f32 output."""
        d = self.desc
        z = torch.empty((batch, d.n_head * d.head_dim), dtype=z_dtype, device=self.device)
        q_type = TYPE_BF16 if q.dtype == torch.bfloat16 else TYPE_F32
        if ws is None:
            ws = self.workspace("decode", batch, max_n_kv, stream)
        check(lib().qsa_decode_gated(ctypes.byref(d), _ptr(items), batch, max_n_kv, _ptr(q), q_type, _ptr(q_idx),
                                     _ptr(k_new), _ptr(v_new), _ptr(kidx_new), _ptr(gate), _ptr(z), _z_type(z_dtype),
                                     _ptr(out), _ptr(sel_out), ws.data_ptr(), ws.numel(), _stream(stream)),
              "qsa_decode_gated")
        return z

    def sparse_attn_gated(self, cache: QsaLayerCache, n_past: int, q: torch.Tensor, q_idx: torch.Tensor,
                          gate: torch.Tensor, k_new=None, v_new=None, kidx_new=None, z_dtype=torch.bfloat16,
                          out: torch.Tensor | None = None, sel_out: torch.Tensor | None = None,
                          ws: torch.Tensor | None = None, stream=None) -> torch.Tensor:
        """qsa_prefill_gated: a prefill chunk with the output gate applied in the final store (see
        sparse_attn_decode_gated)."""
        d = self.desc
        T = q.shape[0]
        z = torch.empty((T, d.n_head * d.head_dim), dtype=z_dtype, device=self.device)
        q_type = TYPE_BF16 if q.dtype == torch.bfloat16 else TYPE_F32
        if ws is None:
            ws = self.workspace("prefill", T, n_past + T, stream)
        check(lib().qsa_prefill_gated(ctypes.byref(d), ctypes.byref(cache), n_past, T, _ptr(q), q_type, _ptr(q_idx),
                                      _ptr(k_new), _ptr(v_new), _ptr(kidx_new), _ptr(gate), _ptr(z), _z_type(z_dtype),
                                      _ptr(out), _ptr(sel_out), ws.data_ptr(), ws.numel(), _stream(stream)),
              "qsa_prefill_gated")
        return z

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

    def decode_step(self, caches: list[QsaLayerCache], max_n_kv: int, q_dtype=torch.bfloat16,
                    sel_out: bool = False) -> "QsaDecodeStep":
        """A captured decode step of these caches (one token per cache, at most max_n_kv cells)."""
        return QsaDecodeStep(self, caches, max_n_kv, q_dtype, sel_out)


def _z_type(dtype) -> int:
    if dtype == torch.bfloat16:
        return TYPE_BF16
    if dtype == torch.float32:
        return TYPE_F32
    raise QsaError(_abi.QSA_ERR_INVALID, "gated output: bfloat16 or float32")


class QsaDecodeStep:
    """One decode step of fixed shape, captured once as a CUDA graph and replayed per token, the way
    the engine submits one compute graph per step to its backend (src/qwfn_engine.cpp:814).

    A replay is qsa_stage_copy of the step's packed pinned host buffer to the device (the item
    table with this token's positions, then q, q_idx, k_new, v_new, kidx_new) and qsa_decode,
    whose last kernel stores the output straight into pinned host memory (mapped at its host
    address): kernels on the compute engine only, no copy-engine hand-over.  Between replays: wait(), write the inputs (the views in `host`,
    or a packed row through load()) and the positions (set_positions()), run(), then read
    `host_out` once the stream has synchronised (run(sync=True) does that)."""

    def __init__(self, node: QsaNode, caches: list[QsaLayerCache], max_n_kv: int, q_dtype=torch.bfloat16,
                 sel_out: bool = False):
        d = node.desc
        if q_dtype not in (torch.bfloat16, torch.float32):
            raise QsaError(_abi.QSA_ERR_INVALID, "q dtype must be bfloat16 or float32")
        self.node, self.batch, self.max_n_kv, self.q_dtype = node, len(caches), int(max_n_kv), q_dtype
        B, kv_dim = self.batch, d.n_head_kv * d.head_dim
        item_bytes = ctypes.sizeof(QsaDecodeItem)
        parts = [("items", (B * item_bytes,), torch.uint8), ("q", (B, d.n_head, d.head_dim), q_dtype),
                 ("q_idx", (B, d.idx_n_head, d.idx_dim), torch.float32), ("k_new", (B, kv_dim), torch.float32),
                 ("v_new", (B, kv_dim), torch.float32), ("kidx_new", (B, d.idx_dim), torch.float32)]
        layout, o = [], 0
        for name, shape, dt in parts:
            n = torch.Size(shape).numel() * torch.empty(0, dtype=dt).element_size()
            layout.append((name, shape, dt, o, n))
            o += (n + 15) // 16 * 16                 # every part starts on 16 bytes
        self.row_bytes = o
        self.input_offset = layout[1][3]            # q..kidx_new: the per-token activations
        self.host_in = torch.zeros(o, dtype=torch.uint8).pin_memory()
        self.dev_in = torch.empty(o, dtype=torch.uint8, device=node.device)

        def views(buf):
            return {name: buf[off:off + n].view(dt).view(shape) for name, shape, dt, off, n in layout}

        self.host, self.dev = views(self.host_in), views(self.dev_in)
        table = (QsaDecodeItem * B)()
        for i, c in enumerate(caches):
            table[i].cache = c
        self.host["items"].copy_(torch.frombuffer(bytearray(bytes(table)), dtype=torch.uint8))
        self._n_past = self.host["items"].view(torch.int32).view(B, item_bytes // 4)[:, QsaDecodeItem.n_past.offset // 4]
        self.host_out = torch.empty((B, d.n_head, d.head_dim), dtype=torch.float32).pin_memory()
        self.sel = torch.empty((B, node.kb), dtype=torch.int32, device=node.device) if sel_out else None
        self.ws = node.workspace("decode", B, self.max_n_kv)
        self.done = torch.cuda.Event()
        self.graph: torch.cuda.CUDAGraph | None = None

    def set_positions(self, n_past: list[int]) -> None:
        """Cells already cached per sequence: this token is appended at n_past and attends n_past + 1."""
        if len(n_past) != self.batch or any(n < 0 or n + 1 > self.max_n_kv for n in n_past):
            raise QsaError(_abi.QSA_ERR_INVALID, "positions outside the captured step's shape")
        self._n_past.copy_(torch.tensor(n_past, dtype=torch.int32))

    def load(self, row: torch.Tensor) -> None:
        """Copy one packed host row of the activations (q..kidx_new, the layout of host_in past the
        item table) into the pinned input buffer."""
        self.host_in[self.input_offset:].copy_(row)

    def wait(self) -> None:
        """Block until the last replay has finished with the host buffers."""
        self.done.synchronize()

    def _call(self) -> None:
        d, dv, st = self.node.desc, self.dev, _stream(None)
        check(lib().qsa_stage_copy(self.dev_in.data_ptr(), self.host_in.data_ptr(), self.row_bytes, st),
              "qsa_stage_copy (inputs)")
        q_type = TYPE_BF16 if self.q_dtype == torch.bfloat16 else TYPE_F32
        check(lib().qsa_decode(ctypes.byref(d), self.dev_in.data_ptr(), self.batch, self.max_n_kv,
                               dv["q"].data_ptr(), q_type, dv["q_idx"].data_ptr(), dv["k_new"].data_ptr(),
                               dv["v_new"].data_ptr(), dv["kidx_new"].data_ptr(), self.host_out.data_ptr(),
                               _ptr(self.sel), self.ws.data_ptr(), self.ws.numel(), st), "qsa_decode")

    def run(self, sync: bool = False) -> torch.Tensor:
        """Replay the step on the current stream (captured on first use); returns host_out."""
        if self.graph is None:
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, capture_error_mode="relaxed"):
                self._call()
        self.graph.replay()
        self.done.record()
        if sync:
            self.done.synchronize()
        return self.host_out


def _weight_format(t: torch.Tensor) -> tuple[int, int]:
    """(qsa type, row length in values) of a projection weight held as ggml holds it: bf16
    [out][n], or q8_0 rows as bytes uint8 [out][n/32*34]."""
    if t.dim() == 2 and t.dtype == torch.bfloat16:
        return TYPE_BF16, int(t.shape[1])
    if t.dim() == 2 and t.dtype == torch.uint8 and t.shape[1] % 34 == 0:
        return _abi.TYPE_Q8_0, int(t.shape[1]) // 34 * 32
    raise QsaError(_abi.QSA_ERR_INVALID, "projection weights: bf16 [out][n] or q8_0 bytes uint8 [out][n/32*34]")


class QsaFront:
    """The projections feeding the node of one layer (qsa_front): weights row-major [out][n_embd]
    as ggml holds them (attn_q with query and gate interleaved per head, attn_k, attn_v,
    indexer.q_proj, indexer.k_proj), bf16 or q8_0 (uint8 rows of n_embd/32 blocks of 34 bytes),
    and the f32 norm weights.  project() returns qsa_decode's inputs: q (f32, QSA_TYPE_F32), q_idx,
    k_new, v_new, kidx_new, and the gate."""

    def __init__(self, desc: QsaDesc, wq: torch.Tensor, wk: torch.Tensor, wv: torch.Tensor, wq_idx: torch.Tensor,
                 wk_idx: torch.Tensor, q_norm: torch.Tensor | None = None, k_norm: torch.Tensor | None = None,
                 q_idx_norm: torch.Tensor | None = None):
        fmts = {_weight_format(t) for t in (wq, wk, wv, wq_idx, wk_idx)}
        if len(fmts) != 1:
            raise QsaError(_abi.QSA_ERR_INVALID, "front weights: one format and row length for all five")
        (w_type, n_embd), = fmts
        for t in (q_norm, k_norm, q_idx_norm):
            if t is not None and t.dtype != torch.float32:
                raise QsaError(_abi.QSA_ERR_INVALID, "front norm weights: f32")
        self.desc, self.device, self.n_embd, self.w_type = desc, wq.device, n_embd, w_type
        self._keep = (wq, wk, wv, wq_idx, wk_idx, q_norm, k_norm, q_idx_norm)
        w = QsaFrontWeights()
        w.wq, w.wk, w.wv, w.wq_idx, w.wk_idx = (_ptr(t) for t in (wq, wk, wv, wq_idx, wk_idx))
        w.q_norm, w.k_norm, w.q_idx_norm = (_ptr(t) for t in (q_norm, k_norm, q_idx_norm))
        w.n_embd, w.w_type = self.n_embd, w_type
        self.w = w
        self._ws: torch.Tensor | None = None

    def workspace(self, T: int, stream=None) -> torch.Tensor:
        size = lib().qsa_front_workspace_size(ctypes.byref(self.desc), ctypes.byref(self.w), T)
        if size == 0:
            raise QsaError(_abi.QSA_ERR_INVALID, "qsa_front_workspace_size")
        if self._ws is None or self._ws.numel() < size:
            self._ws = torch.empty(size, dtype=torch.uint8, device=self.device)
            check(lib().qsa_workspace_init(self._ws.data_ptr(), size, _stream(stream)), "qsa_workspace_init")
        return self._ws

    def project(self, x: torch.Tensor, pos: torch.Tensor, stream=None):
        """x f32 [T][n_embd], pos int32 [T] (device) -> (q, gate, q_idx, k, v, kidx) f32."""
        d = self.desc
        T = x.shape[0]
        if x.dtype != torch.float32 or x.shape[1] != self.n_embd or pos.dtype != torch.int32 or pos.numel() != T:
            raise QsaError(_abi.QSA_ERR_INVALID, "front inputs: x f32 [T][n_embd], pos int32 [T]")
        f = dict(dtype=torch.float32, device=self.device)
        kv = d.n_head_kv * d.head_dim
        q = torch.empty((T, d.n_head, d.head_dim), **f)
        gate = torch.empty((T, d.n_head * d.head_dim), **f)
        q_idx = torch.empty((T, d.idx_n_head, d.idx_dim), **f)
        k, v = torch.empty((T, kv), **f), torch.empty((T, kv), **f)
        kidx = torch.empty((T, d.idx_dim), **f)
        ws = self.workspace(T, stream)
        check(lib().qsa_front(ctypes.byref(d), ctypes.byref(self.w), T, _ptr(pos), _ptr(x), _ptr(q), _ptr(gate),
                              _ptr(q_idx), _ptr(k), _ptr(v), _ptr(kidx), ws.data_ptr(), ws.numel(), _stream(stream)),
              "qsa_front")
        return q, gate, q_idx, k, v, kidx


class QsaOutput:
    """The output side of the node (qsa_output): y = attn_output.weight (attn * sigmoid(gate)), the
    weight row-major [n_embd][n_head*head_dim] in bf16, or q8_0 bytes uint8 [n_embd][n_head*head_dim/32*34]."""

    def __init__(self, desc: QsaDesc, wo: torch.Tensor):
        self.w_type, n_in = _weight_format(wo)
        if n_in != desc.n_head * desc.head_dim:
            raise QsaError(_abi.QSA_ERR_INVALID, "attn_output weight: [n_embd][n_head*head_dim]")
        self.desc, self.wo, self.n_embd = desc, wo, int(wo.shape[0])
        self._ws: torch.Tensor | None = None

    def workspace(self, T: int, stream=None) -> torch.Tensor | None:
        """The workspace of a T-token call (none up to 16 tokens; above, the GEMM path's)."""
        size = lib().qsa_output_workspace_size(ctypes.byref(self.desc), self.n_embd, self.w_type, T)
        if size == 0:
            return None
        if self._ws is None or self._ws.numel() < size:
            self._ws = torch.empty(size, dtype=torch.uint8, device=self.wo.device)
            check(lib().qsa_workspace_init(self._ws.data_ptr(), size, _stream(stream)), "qsa_workspace_init")
        return self._ws

    def project(self, attn: torch.Tensor, gate: torch.Tensor, out: torch.Tensor | None = None, stream=None):
        """attn f32 [T][n_head][head_dim], gate f32 [T][n_head*head_dim] -> y f32 [T][n_embd]."""
        T = attn.shape[0]
        if out is None:
            out = torch.empty((T, self.n_embd), dtype=torch.float32, device=self.wo.device)
        ws = self.workspace(T, stream)
        check(lib().qsa_output(ctypes.byref(self.desc), _ptr(self.wo), self.n_embd, self.w_type, T, _ptr(attn), _ptr(gate),
                               _ptr(out), None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(),
                               _stream(stream)), "qsa_output")
        return out

    def project_z(self, z: torch.Tensor, out: torch.Tensor | None = None, stream=None):
        """qsa_output_z: y = attn_output.weight z for a gated product z [T][n_head*head_dim] (bf16 with
        bf16 weights, or f32) written by the gated decode / prefill -> y f32 [T][n_embd]."""
        T = z.shape[0]
        if out is None:
            out = torch.empty((T, self.n_embd), dtype=torch.float32, device=self.wo.device)
        ws = self.workspace(T, stream)
        check(lib().qsa_output_z(ctypes.byref(self.desc), _ptr(self.wo), self.n_embd, self.w_type, T, _ptr(z),
                                 _z_type(z.dtype), _ptr(out), None if ws is None else ws.data_ptr(),
                                 0 if ws is None else ws.numel(), _stream(stream)), "qsa_output_z")
        return out
