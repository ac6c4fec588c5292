"""Launch order: a call's first kernel waits for all earlier work in the stream.

The kernels after the first of a call start early (programmatic dependent launch) and read the
call's inputs (the item table, q, q_idx, the caches) before they wait for the kernel ahead of
them.  That is only safe if the call's first kernel started after the work that wrote those
inputs had completed (or, the decode append, waits for the kernel ahead before it reads or lets
the next kernel start).  These tests write the inputs with qsa_stage_copy, whose kernel lets its
successor start at once, at the end of a 64 MB copy from pinned host memory (about a millisecond
over PCIe), with different, stale values already in place; the decode with and without its
append (the append first, or the selection) and the attention alone must give the outputs of the
same calls on settled inputs, bit for bit, and the append must write the row it is given.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from qwfnfer_b200._abi import TYPE_BF16, check, lib, make_desc
from qwfnfer_b200.configs import fill_cache, token_inputs
from qwfnfer_b200.qsa import QsaNode, QsaState, decode_items

pytestmark = pytest.mark.gpu

BULK = 64 << 20            # bytes copied ahead of the inputs


def _pack(parts: list[torch.Tensor]) -> tuple[torch.Tensor, list[int]]:
    """The tensors' bytes back to back on 16-byte boundaries (a uint8 host tensor) and their offsets."""
    offs, o = [], 0
    for p in parts:
        offs.append(o)
        o += (p.numel() * p.element_size() + 15) // 16 * 16
    buf = torch.zeros(o, dtype=torch.uint8)
    for p, off in zip(parts, offs):
        b = p.contiguous().view(torch.uint8).reshape(-1).cpu()
        buf[off:off + b.numel()].copy_(b)
    return buf, offs


def _setup():
    """The desc, node, cache (kept alive by the caller: the item tables point into it), position,
    pinned source, device buffer, stale and new input bytes, and the inputs' offsets (items, q,
    q_idx, k_new, v_new, kidx_new)."""
    d = make_desc(n_ctx=32768, top_k_blocks=64, window=128)
    node = QsaNode(d)
    st = QsaState(d)
    n_past = 20000
    fill_cache(node, st, 0, n_past + 1, 61)            # the token at n_past is already cached
    new_in = token_inputs(d, 1, seed=5)
    old_in = token_inputs(d, 1, seed=6)
    new, offs = _pack([decode_items([st.layer()], [n_past]).cpu(), *new_in])
    old, _ = _pack([decode_items([st.layer()], [n_past - 700]).cpu(), *old_in])
    host = torch.zeros(BULK + new.numel(), dtype=torch.uint8).pin_memory()
    host[BULK:].copy_(new)
    dev = torch.zeros(BULK + new.numel(), dtype=torch.uint8, device="cuda")
    views = {name: (BULK + off, None) for name, off in zip(("items", "q", "q_idx", "k", "v", "kidx"), offs)}
    return d, node, st, n_past, host, dev, old, new, views


def _ptr(dev: torch.Tensor, off: int) -> int:
    return dev.data_ptr() + off


@pytest.mark.parametrize("append", [False, True])
def test_decode_waits_for_staged_inputs(append):
    d, node, st, n_past, host, dev, old, new, v = _setup()
    L, D, s = lib(), ctypes.byref(d), torch.cuda.current_stream().cuda_stream
    ws = node.workspace("decode", 1, n_past + 1)
    rows = (_ptr(dev, v["k"][0]), _ptr(dev, v["v"][0]), _ptr(dev, v["kidx"][0])) if append else (None, None, None)

    def call(out):
        check(L.qsa_decode(D, _ptr(dev, v["items"][0]), 1, n_past + 1, _ptr(dev, v["q"][0]), TYPE_BF16,
                           _ptr(dev, v["q_idx"][0]), *rows, out.data_ptr(), None, ws.data_ptr(), ws.numel(), s),
              "decode")

    # the reference: the same call on the settled new inputs (with the append, it writes the row
    # at n_past, which every later call rewrites with the same bytes)
    dev[BULK:].copy_(new.cuda())
    want = torch.empty(1, d.n_head, d.head_dim, device="cuda")
    call(want)
    torch.cuda.synchronize()
    assert torch.isfinite(want).all()
    cache = [x.clone() for x in (st.k[0], st.v[0], st.idx[0], st.pool[0])]
    for _ in range(3):
        dev[BULK:].copy_(old.cuda())                    # stale inputs in place
        torch.cuda.synchronize()
        got = torch.full_like(want, float("nan"))
        check(L.qsa_stage_copy(dev.data_ptr(), host.data_ptr(), host.numel(), s), "stage")
        call(got)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        for x, y in zip(cache, (st.k[0], st.v[0], st.idx[0], st.pool[0])):
            assert torch.equal(x, y)                    # no row written at a stale position
    assert node.check(ws) == 0


def test_attend_alone_waits_for_staged_query():
    d, node, st, n_past, host, dev, old, new, v = _setup()
    L, D, s = lib(), ctypes.byref(d), torch.cuda.current_stream().cuda_stream
    ws = node.workspace("decode", 1, n_past + 1)
    dev[BULK:].copy_(new.cuda())
    check(L.qsa_decode_select(D, _ptr(dev, v["items"][0]), 1, n_past + 1, _ptr(dev, v["q_idx"][0]), None,
                              ws.data_ptr(), ws.numel(), s), "select")
    want = torch.empty(1, d.n_head, d.head_dim, device="cuda")
    check(L.qsa_decode_attend(D, _ptr(dev, v["items"][0]), 1, n_past + 1, _ptr(dev, v["q"][0]), TYPE_BF16,
                              want.data_ptr(), ws.data_ptr(), ws.numel(), s), "attend")
    torch.cuda.synchronize()
    assert torch.isfinite(want).all()
    for _ in range(3):
        dev[BULK:].copy_(old.cuda())
        dev[v["items"][0]:v["q"][0]].copy_(new[:v["q"][0] - BULK].cuda())    # the same position: only q is stale
        torch.cuda.synchronize()
        got = torch.full_like(want, float("nan"))
        check(L.qsa_stage_copy(dev.data_ptr(), host.data_ptr(), host.numel(), s), "stage")
        check(L.qsa_decode_attend(D, _ptr(dev, v["items"][0]), 1, n_past + 1, _ptr(dev, v["q"][0]), TYPE_BF16,
                                  got.data_ptr(), ws.data_ptr(), ws.numel(), s), "attend")
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    assert node.check(ws) == 0
