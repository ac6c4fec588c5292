"""KV-sequence-sharded QSA decode: one process per GPU over torch.distributed.

The reference decodes a sequence on one device (its engine keeps one KV cache per layer,
src/qwfn_state.cpp:18-96).  For contexts whose caches do not fit one GPU, or decode faster spread
over several, the cells of every layer are split into contiguous block ranges, one per rank, and
one decode step of one layer becomes:

  1. candidates (libqsa): the rank holding the new token's cell appends it (K, V, raw key, and the
     pooled key of a block it completes); every rank scores its own visible blocks and keeps its
     best KB blocks outside the forced window, with their scores;
  2. one all-gather of the candidates ([2, batch, KB] int32 per rank: ids, then score bits), by NCCL
     or by libqsa's push/wait over NVLink peer memory (exchange="peer");
  3. attend (libqsa): the exact global selection, identical on every rank and to the unsharded
     qsa_decode's (a block among the global best is among its owner's best), then attention over
     the rank's part of it into an unnormalised state [M | L | O] per query;
  4. one all-gather of the states;
  5. merge (libqsa): log-sum-exp combination of the states in rank order.

The two exchanges carry O(batch x KB) and O(batch x 16 x head_dim) words, independent of the
context length; the cache reads stay local.  The backend computes steps 1, 3 and 5; the default is
the library on this rank's GPU.  PyTorch provides memory, streams and the collectives only.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from ._abi import QsaDesc, QsaError, QsaLayerCache, QsaPeerSlots, TYPE_BF16, TYPE_F32, check, k_blocks, lib


def shard_blocks(n_blocks: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous block range [lo, hi) of `rank`: an even split, the first n_blocks % world ranks
    holding one block more."""
    if world <= 0 or not 0 <= rank < world or n_blocks < world:
        raise ValueError(f"cannot split {n_blocks} blocks over {world} ranks (rank {rank})")
    base, extra = divmod(n_blocks, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    assert t.is_cuda and t.is_contiguous(), "device tensors must be contiguous CUDA tensors"
    return t.data_ptr()


class LibShardBackend:
    """Steps 1, 3 and 5 on this rank's GPU through libqsa's sharded entry points."""

    def __init__(self, desc: QsaDesc, device: str | torch.device = "cuda"):
        check(lib().qsa_desc_check(ctypes.byref(desc)), "qsa_desc_check")
        self.desc = desc
        self.device = torch.device(device)
        self.kb = k_blocks(desc)
        self.state_floats = lib().qsa_shard_state_floats(ctypes.byref(desc))
        self._ws: dict[int, torch.Tensor] = {}
        self._blocks: tuple[int, int] | None = None       # the shard range of the last call

    def _stream(self) -> int:
        return torch.cuda.current_stream(self.device).cuda_stream

    def workspace(self, batch: int, max_n_kv: int, blocks: tuple[int, int] | None = None) -> torch.Tensor:
        blocks = blocks if blocks is not None else self._blocks
        if blocks is None:
            raise ValueError("no shard block range yet")
        self._blocks = tuple(blocks)
        size = lib().qsa_shard_workspace_size(ctypes.byref(self.desc), batch, max_n_kv, blocks[0], blocks[1])
        if size == 0:
            raise ValueError("invalid decode shape")
        ws = self._ws.get(size)
        if ws is None:
            ws = torch.empty(size, dtype=torch.uint8, device=self.device)
            check(lib().qsa_workspace_init(ws.data_ptr(), size, self._stream()), "qsa_workspace_init")
            self._ws[size] = ws
        return ws

    def append(self, cache: QsaLayerCache, blocks: tuple[int, int], pos0: int, k, v, kidx) -> None:
        n = (k if k is not None else kidx).shape[0]
        check(lib().qsa_shard_append(ctypes.byref(self.desc), ctypes.byref(cache), blocks[0], blocks[1], pos0, n,
                                     _ptr(k), _ptr(v), _ptr(kidx), self._stream()), "qsa_shard_append")

    def append_ri(self, cache: QsaLayerCache, blocks: tuple[int, int], pos0: int, k, v, kidx) -> None:
        """Replicated indexer caches: every row's raw key (and pooled keys), the shard's K/V rows."""
        n = (k if k is not None else kidx).shape[0]
        check(lib().qsa_shard_append_ri(ctypes.byref(self.desc), ctypes.byref(cache), blocks[0], blocks[1], pos0, n,
                                        _ptr(k), _ptr(v), _ptr(kidx), self._stream()), "qsa_shard_append_ri")

    def decode_ri(self, items, batch: int, max_n_kv: int, blocks: tuple[int, int], q, q_idx, k_new=None, v_new=None,
                  kidx_new=None, sel_out: torch.Tensor | None = None, state: torch.Tensor | None = None) -> torch.Tensor:
        """Replicated indexer caches: append, the global selection and the attention over this
        shard's selected blocks, into an unnormalised state f32 [batch, state_floats]."""
        if state is None:
            state = torch.empty((batch, self.state_floats), dtype=torch.float32, device=self.device)
        q_type = TYPE_BF16 if q.dtype == torch.bfloat16 else TYPE_F32
        ws = self.workspace(batch, max_n_kv, blocks)
        check(lib().qsa_shard_decode_ri(ctypes.byref(self.desc), _ptr(items), batch, max_n_kv, blocks[0], blocks[1],
                                        _ptr(q), q_type, _ptr(q_idx), _ptr(k_new), _ptr(v_new), _ptr(kidx_new),
                                        state.data_ptr(), _ptr(sel_out), ws.data_ptr(), ws.numel(), self._stream()),
              "qsa_shard_decode_ri")
        return state

    def decode_ri_peer(self, items, batch: int, max_n_kv: int, blocks: tuple[int, int], q, q_idx, slots: QsaPeerSlots,
                       k_new=None, v_new=None, kidx_new=None, sel_out: torch.Tensor | None = None) -> None:
        """decode_ri whose state goes straight into slot `rank` of every rank's region of one peer
        channel (`slots`), published there by a release flag: no push or wait launch."""
        q_type = TYPE_BF16 if q.dtype == torch.bfloat16 else TYPE_F32
        ws = self.workspace(batch, max_n_kv, blocks)
        check(lib().qsa_shard_decode_ri_peer(ctypes.byref(self.desc), _ptr(items), batch, max_n_kv, blocks[0],
                                             blocks[1], _ptr(q), q_type, _ptr(q_idx), _ptr(k_new), _ptr(v_new),
                                             _ptr(kidx_new), ctypes.byref(slots), _ptr(sel_out), ws.data_ptr(),
                                             ws.numel(), self._stream()), "qsa_shard_decode_ri_peer")

    def merge_peer(self, slots: QsaPeerSlots, batch: int, status: torch.Tensor,
                   out: torch.Tensor | None = None) -> torch.Tensor:
        """Wait (bounded; the status word of `status`) for every rank's state of the round in this
        rank's region of the channel, then merge them into out f32 [batch, n_head, head_dim]."""
        d = self.desc
        if out is None:
            out = torch.empty((batch, d.n_head, d.head_dim), dtype=torch.float32, device=self.device)
        check(lib().qsa_merge_states_peer(ctypes.byref(d), ctypes.byref(slots), batch, out.data_ptr(),
                                          status.data_ptr(), status.numel(), self._stream()), "qsa_merge_states_peer")
        return out

    def candidates(self, items, batch: int, max_n_kv: int, blocks: tuple[int, int], q_idx,
                   k_new=None, v_new=None, kidx_new=None, out: torch.Tensor | None = None) -> torch.Tensor:
        """This rank's candidates, int32 [2, batch, KB]: block ids (-1 padded), then score bits."""
        if out is None:
            out = torch.empty((2, batch, self.kb), dtype=torch.int32, device=self.device)
        ws = self.workspace(batch, max_n_kv, blocks)
        check(lib().qsa_shard_candidates(ctypes.byref(self.desc), _ptr(items), batch, max_n_kv, blocks[0], blocks[1],
                                         _ptr(q_idx), _ptr(k_new), _ptr(v_new), _ptr(kidx_new), _ptr(out),
                                         ws.data_ptr(), ws.numel(), self._stream()), "qsa_shard_candidates")
        return out

    def attend(self, items, batch: int, max_n_kv: int, blocks: tuple[int, int], gathered: torch.Tensor, q,
               sel_out: torch.Tensor | None = None, state: torch.Tensor | None = None,
               n_shards: int | None = None, cand_stride: int = 0) -> torch.Tensor:
        """gathered: every rank's candidates in rank order, int32 [n_shards, 2, batch, KB], or a flat
        tensor whose shard slices are cand_stride elements apart."""
        n_shards = n_shards if n_shards is not None else gathered.shape[0]
        if state is None:
            state = torch.empty((batch, self.state_floats), dtype=torch.float32, device=self.device)
        q_type = TYPE_BF16 if q.dtype == torch.bfloat16 else TYPE_F32
        ws = self.workspace(batch, max_n_kv, blocks)
        check(lib().qsa_shard_attend(ctypes.byref(self.desc), _ptr(items), batch, max_n_kv, blocks[0], blocks[1],
                                     n_shards, _ptr(gathered), cand_stride, _ptr(q), q_type, state.data_ptr(),
                                     _ptr(sel_out), ws.data_ptr(), ws.numel(), self._stream()), "qsa_shard_attend")
        return state

    def merge(self, states: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """states: f32 [n_parts, batch, state_floats] -> f32 [batch, n_head, head_dim]."""
        P, B = states.shape[0], states.shape[1]
        d = self.desc
        if out is None:
            out = torch.empty((B, d.n_head, d.head_dim), dtype=torch.float32, device=self.device)
        check(lib().qsa_merge_states(ctypes.byref(d), P, B, _ptr(states.contiguous()), out.data_ptr(), self._stream()),
              "qsa_merge_states")
        return out

    def check(self, batch: int, max_n_kv: int, blocks: tuple[int, int] | None = None) -> int:
        ws = self.workspace(batch, max_n_kv, blocks)
        return lib().qsa_check(ws.data_ptr(), ws.numel(), self._stream())


class PeerExchange:
    """All-gathers of fixed-size slices over NVLink peer memory (libqsa's qsa_peer_push/_wait):
    one buffer per rank holding a gather region per channel, mapped by every rank through CUDA
    IPC.  `all_gather(channel, src)` returns a view [world, *src.shape] of this rank's region; the
    view stays valid until the same channel's next all_gather (every rank must call the channels
    in the same order)."""

    def __init__(self, slot_bytes: list[int], group=None, device: str | torch.device = "cuda"):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)
        L = lib()
        self.slot = [int(b) for b in slot_bytes]
        assert all(b % 4 == 0 for b in self.slot), "slots are 4-byte multiples"
        self.stride = [(b + 15) // 16 * 16 for b in self.slot]
        region = [L.qsa_peer_buffer_bytes(self.world, b) for b in self.slot]
        self.offsets = [0]
        for r in region[:-1]:
            self.offsets.append(self.offsets[-1] + ((r + 255) // 256) * 256)
        total = self.offsets[-1] + ((region[-1] + 255) // 256) * 256
        self.buf = torch.zeros(total, dtype=torch.uint8, device=self.device)
        self.sync = torch.zeros(len(self.slot), 2, dtype=torch.int32, device=self.device)   # epoch, counter
        handle = (ctypes.c_char * 64)()
        off = ctypes.c_size_t()
        check(L.qsa_ipc_handle(self.buf.data_ptr(), handle, ctypes.byref(off)), "qsa_ipc_handle")
        everyone = [None] * self.world
        dist.all_gather_object(everyone, (bytes(handle), off.value), group=group)
        self._opened = []
        bases = []
        for r, (h, o) in enumerate(everyone):
            if r == self.rank:
                bases.append(self.buf.data_ptr())
                continue
            hb = (ctypes.c_char * 64).from_buffer_copy(h)
            base = ctypes.c_void_p()
            check(L.qsa_ipc_open(hb, ctypes.byref(base)), "qsa_ipc_open")
            self._opened.append(base.value)
            bases.append(base.value + o)
        # per channel, every rank's region address (host list, and a device array for the push)
        self.regions = [[b + off_c for b in bases] for off_c in self.offsets]
        self.ptrs = [torch.tensor(r, dtype=torch.int64, device=self.device) for r in self.regions]
        self._slots: dict[int, QsaPeerSlots] = {}
        self.status = torch.zeros(64, dtype=torch.uint8, device=self.device)   # status word of the waits
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)

    def all_gather(self, channel: int, src: torch.Tensor):
        """(gathered, stride): gathered = this rank's region as a flat tensor of src's dtype, the
        slices `stride` elements apart (a [world, *src.shape] view when there is no padding)."""
        L = lib()
        nb = src.numel() * src.element_size()
        assert src.is_contiguous() and nb == self.slot[channel]
        stream = torch.cuda.current_stream(self.device).cuda_stream
        region = self.buf.data_ptr() + self.offsets[channel]
        epoch = self.sync[channel].data_ptr()
        check(L.qsa_peer_push(self.ptrs[channel].data_ptr(), self.world, self.rank, src.data_ptr(), nb, epoch,
                              epoch + 4, stream), "qsa_peer_push")
        check(L.qsa_peer_wait(region, self.world, nb, epoch, self.status.data_ptr(), self.status.numel(), stream),
              "qsa_peer_wait")
        st = self.stride[channel]
        flat = self.buf[self.offsets[channel]:self.offsets[channel] + self.world * st].view(src.dtype)
        stride = st // src.element_size()
        if st == nb:
            return flat.view((self.world,) + tuple(src.shape)), stride
        return flat, stride

    def slots(self, channel: int) -> QsaPeerSlots:
        """The channel as qsa_shard_decode_ri_peer / qsa_merge_states_peer see it (at most 8 ranks)."""
        s = self._slots.get(channel)
        if s is None:
            if self.world > 8:
                raise QsaError(1, "the fused peer exchange serves at most 8 ranks")
            s = QsaPeerSlots()
            for r, a in enumerate(self.regions[channel]):
                s.region[r] = a
            s.n_ranks, s.rank = self.world, self.rank
            s.epoch = self.sync[channel].data_ptr()
            self._slots[channel] = s
        return s

    def check(self) -> int:
        return lib().qsa_check(self.status.data_ptr(), self.status.numel(),
                               torch.cuda.current_stream(self.device).cuda_stream)

    def close(self) -> None:
        for b in self._opened:
            lib().qsa_ipc_close(b)
        self._opened = []


class ShardedDecoder:
    """The per-rank driver of the sharded decode step (module docstring).  `group` is a
    torch.distributed process group (default: the world); world size 1 runs without collectives."""

    def __init__(self, desc: QsaDesc, backend=None, group=None, rank: int | None = None,
                 world: int | None = None, exchange: str = "nccl", batch: int = 1, index: str = "sharded"):
        """exchange: "nccl" (all-gathers of the process group), "nccl_capi" (the whole step in libqsa's
        qsa_decode_sharded with the process group's NCCL communicator), "peer" (libqsa's all-gather
        over NVLink peer memory, GPUs of one node; sized for `batch` queries per step; with
        replicated indexer caches and at most 8 ranks, the states are stored into the peers by the
        attention itself and published by flag) or "peer_push" (the same buffers, every exchange by
        a push and a wait launch).
        index: "sharded"
        (each rank holds its blocks' raw and pooled keys; candidates are exchanged) or "replicated"
        (every rank holds all of them, QsaState(index_full=True), and selects globally itself: one
        exchange per step).

        With the peer exchange and replicated indexer caches, consecutive steps alternate two state
        channels (a rank's push of step s+1 lands only after its peers read step s).  A CUDA graph
        fixes each captured step's channel, so a graph replayed back to back must hold an even
        number of steps."""
        if index not in ("sharded", "replicated"):
            raise ValueError("index is 'sharded' or 'replicated'")
        self.index_replicated = index == "replicated"
        self.desc = desc
        self.group = group
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = world if world is not None else (dist.get_world_size(group) if dist_on else 1)
        self.rank = rank if rank is not None else (dist.get_rank(group) if dist_on else 0)
        self.blocks = shard_blocks(desc.n_ctx // desc.ratio, self.world, self.rank)
        self.backend = backend if backend is not None else LibShardBackend(desc)
        self.kb = k_blocks(desc)
        self.peer = None
        self._steps = 0
        self.comm = 0
        if exchange == "nccl_capi":
            pg = group if group is not None else dist.group.WORLD
            dev = self.backend.device
            dist.all_reduce(torch.zeros(1, device=dev), group=pg)        # the communicator exists after a collective
            self.comm = pg._get_backend(dev)._comm_ptr()
            if not self.comm:
                raise QsaError(1, "no NCCL communicator behind the process group")
        self.fused = exchange == "peer"
        if exchange in ("peer", "peer_push") and self.world > 1:
            # Channels: 0 candidates, 1 and 2 states.  A push overwrites the peers' slots without
            # waiting for them to finish reading the last round, so consecutive pushes into one
            # channel are always separated by a wait on another: the sharded-index step alternates
            # candidates and states; the replicated-index step (states only) alternates 1 and 2.
            # A rank's push of round e+2 into a channel then follows its wait of round e+1, which
            # needs every peer's push of e+1, which each peer issues after its merge read round e.
            state_floats = lib().qsa_shard_state_floats(ctypes.byref(desc))
            sb = batch * state_floats * 4
            self.peer = PeerExchange([2 * batch * self.kb * 4, sb, sb], group=group, device=self.backend.device)

    def _all_gather(self, t: torch.Tensor, channel: int = 0):
        """(gathered, stride): every rank's t in rank order, slices `stride` elements apart
        ([world, *t.shape] when dense)."""
        if self.world == 1:
            return t.unsqueeze(0), t.numel()
        t = t.contiguous()
        if self.peer is not None:
            return self.peer.all_gather(channel, t)
        out = torch.empty((self.world * t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t, group=self.group)
        return out.view((self.world,) + tuple(t.shape)), t.numel()

    def append(self, cache: QsaLayerCache, pos0: int, k, v, kidx) -> None:
        """Append global rows [pos0, pos0+n): the rows inside this rank's cells are written (with
        replicated indexer caches: every row's raw key, the K/V rows inside this rank's cells)."""
        if self.index_replicated:
            self.backend.append_ri(cache, self.blocks, pos0, k, v, kidx)
            return
        n = (k if k is not None else kidx).shape[0]
        r = self.desc.ratio
        lo, hi = max(pos0, self.blocks[0] * r), min(pos0 + n, self.blocks[1] * r)
        if lo >= hi:
            return
        sl = slice(lo - pos0, hi - pos0)
        self.backend.append(cache, self.blocks, lo, None if k is None else k[sl], None if v is None else v[sl],
                            None if kidx is None else kidx[sl])

    def step(self, items, batch: int, max_n_kv: int, q, q_idx, k_new=None, v_new=None, kidx_new=None,
             sel_out: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
        """One decode step of one layer for `batch` queries (items: this rank's device item table,
        global n_past, local caches).  Returns f32 [batch, n_head, head_dim] on every rank, in `out`
        when given (device memory, or pinned host memory: the last kernel stores into it)."""
        if self.comm:
            return self._step_capi(items, batch, max_n_kv, q, q_idx, k_new, v_new, kidx_new, sel_out, out)
        if self.index_replicated:
            channel = 1 + (self._steps & 1)
            self._steps += 1
            if self.peer is not None and self.fused and self.world <= 8:
                # the attention stores the state into every rank's region itself and publishes it;
                # the merge waits for the flags (no push or wait launch)
                if batch * self.backend.state_floats * 4 != self.peer.slot[channel]:
                    raise QsaError(1, "batch differs from the one the peer exchange was sized for")
                slots = self.peer.slots(channel)
                self.backend.decode_ri_peer(items, batch, max_n_kv, self.blocks, q, q_idx, slots, k_new, v_new,
                                            kidx_new, sel_out=sel_out)
                return self.backend.merge_peer(slots, batch, self.peer.status, out)
            state = self.backend.decode_ri(items, batch, max_n_kv, self.blocks, q, q_idx, k_new, v_new, kidx_new,
                                           sel_out=sel_out)
            states, _ = self._all_gather(state, channel)
            return self.backend.merge(states.view(self.world, batch, -1), out)
        cand = self.backend.candidates(items, batch, max_n_kv, self.blocks, q_idx, k_new, v_new, kidx_new)
        gathered, cstride = self._all_gather(cand, 0)
        state = self.backend.attend(items, batch, max_n_kv, self.blocks, gathered, q, sel_out=sel_out,
                                    n_shards=self.world, cand_stride=cstride)
        states, _ = self._all_gather(state, 1)
        return self.backend.merge(states.view(self.world, batch, -1), out)

    def _step_capi(self, items, batch, max_n_kv, q, q_idx, k_new, v_new, kidx_new, sel_out, out=None):
        """The step as one qsa_decode_sharded call (its all-gathers on the NCCL communicator)."""
        d = self.desc
        L = lib()
        size = L.qsa_decode_sharded_workspace_size(ctypes.byref(d), batch, max_n_kv, self.blocks[0], self.blocks[1],
                                                    self.world)
        if size == 0:
            raise QsaError(1, "invalid sharded decode shape")
        ws = self.backend._ws.get(("capi", size))
        stream = torch.cuda.current_stream(self.backend.device).cuda_stream
        if ws is None:
            ws = torch.empty(size, dtype=torch.uint8, device=self.backend.device)
            check(L.qsa_workspace_init(ws.data_ptr(), size, stream), "qsa_workspace_init")
            self.backend._ws[("capi", size)] = ws
        if out is None:
            out = torch.empty((batch, d.n_head, d.head_dim), dtype=torch.float32, device=self.backend.device)
        q_type = TYPE_BF16 if q.dtype == torch.bfloat16 else TYPE_F32
        check(L.qsa_decode_sharded(ctypes.byref(d), _ptr(items), batch, max_n_kv, self.blocks[0], self.blocks[1],
                                   1 if self.index_replicated else 0, self.comm, self.world, _ptr(q), q_type,
                                   _ptr(q_idx), _ptr(k_new), _ptr(v_new), _ptr(kidx_new), out.data_ptr(), _ptr(sel_out),
                                   ws.data_ptr(), ws.numel(), stream), "qsa_decode_sharded")
        return out

    def check(self, batch: int, max_n_kv: int) -> int:
        """qsa_check of the workspace this decoder's steps used (synchronises the stream)."""
        if self.comm:
            size = lib().qsa_decode_sharded_workspace_size(ctypes.byref(self.desc), batch, max_n_kv, self.blocks[0],
                                                          self.blocks[1], self.world)
            ws = self.backend._ws.get(("capi", size))
            if ws is None:
                return 0
            return lib().qsa_check(ws.data_ptr(), ws.numel(), torch.cuda.current_stream(self.backend.device).cuda_stream)
        return self.backend.check(batch, max_n_kv, self.blocks)
