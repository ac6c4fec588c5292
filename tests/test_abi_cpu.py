"""The C ABI library on a machine without a GPU: it loads, exports every function include/qsa.h
declares, and its host-only functions (validation, sizes) behave.  No kernel is launched."""
import ctypes
import os
import re

import pytest

from qwfnfer_b200 import _abi
from qwfnfer_b200._abi import TYPE_F16, TYPE_Q8_0, lib, make_desc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "qsa.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(qsa_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_header_function():
    L = lib()
    names = header_functions()
    assert names, "no functions parsed from include/qsa.h"
    assert set(names) == set(_abi.HEADER_SYMBOLS)
    for n in names:
        assert hasattr(L, n), f"libqsa.so does not export {n}"


def test_desc_check_and_sizes():
    L = lib()
    d = make_desc(n_ctx=163840)
    assert L.qsa_desc_check(ctypes.byref(d)) == 0
    assert L.qsa_k_blocks(ctypes.byref(d)) == 67
    assert L.qsa_row_bytes(ctypes.byref(d), 0) == 544
    assert L.qsa_row_bytes(ctypes.byref(d), 2) == 256
    assert L.qsa_cache_bytes(ctypes.byref(d), 0) == 163840 * 544
    assert L.qsa_cache_bytes(ctypes.byref(d), 3) == 2560 * 256
    f16 = make_desc(n_ctx=4096, type_k=TYPE_F16, type_v=TYPE_F16, top_k_blocks=16)
    assert L.qsa_row_bytes(ctypes.byref(f16), 1) == 1024
    assert L.qsa_k_blocks(ctypes.byref(f16)) == 19
    w0 = make_desc(n_ctx=4096, window=0, top_k_blocks=512, ratio=4)
    assert L.qsa_k_blocks(ctypes.byref(w0)) == 513          # ceil((2048 + 4 - 1) / 4), the reference's k_blocks
    s1 = L.qsa_decode_workspace_size(ctypes.byref(d), 1, 163840)
    s64 = L.qsa_decode_workspace_size(ctypes.byref(d), 64, 163840)
    assert 0 < s1 < s64
    assert L.qsa_decode_workspace_size(ctypes.byref(d), 0, 163840) == 0


@pytest.mark.parametrize("field,value,status", [
    ("n_ctx", 1000, 1), ("n_head_kv", 3, 1), ("ratio", 0, 1), ("top_k_blocks", 0, 1), ("window", -1, 1),
    ("type_k", 2, 1), ("head_dim", 128, 4), ("idx_dim", 64, 4), ("n_head_kv", 1, 4), ("top_k_blocks", 5000, 4)])
def test_desc_check_rejects(field, value, status):
    d = make_desc(n_ctx=4096)
    setattr(d, field, value)
    assert lib().qsa_desc_check(ctypes.byref(d)) == status


def test_status_strings():
    L = lib()
    for s, name in _abi.STATUS_NAMES.items():
        assert L.qsa_status_string(s)
    assert L.qsa_version() >= 100


def test_struct_layouts_match_header():
    assert ctypes.sizeof(_abi.QsaLayerCache) == 32
    assert ctypes.sizeof(_abi.QsaDecodeItem) == 48
    assert _abi.QsaDecodeItem.n_past.offset == 32
    assert ctypes.sizeof(_abi.QsaDesc) == 4 * 12 + 16 + 8 + 8 + 8      # + placement (and tail padding)
    assert _abi.QsaDesc.placement.offset == 80


def test_peer_slots_layout():
    assert ctypes.sizeof(_abi.QsaPeerSlots) == 8 * 8 + 4 + 4 + 8
    assert _abi.QsaPeerSlots.epoch.offset == 72


def test_front_weights_layout():
    assert ctypes.sizeof(_abi.QsaFrontWeights) == 8 * 8 + 2 * 4
    assert _abi.QsaFrontWeights.n_embd.offset == 64


# Fake device addresses: 16-byte aligned, never dereferenced (every case below is refused on the
# host before any CUDA call is made).
A = 1 << 20


def front_call(w=None, T=1, x=A, ws_bytes=1 << 30):
    d = make_desc(n_ctx=4096)
    if w is None:
        w = _abi.QsaFrontWeights(A, A, A, A, A, None, None, None, 2560, _abi.TYPE_BF16)
    outs = [A] * 6
    return lib().qsa_front(ctypes.byref(d), ctypes.byref(w), T, A, x, *outs, A, ws_bytes, None)


def test_front_host_refusals():
    d = make_desc(n_ctx=4096)
    w = _abi.QsaFrontWeights(A, A, A, A, A, None, None, None, 2560, _abi.TYPE_BF16)
    assert lib().qsa_front_workspace_size(ctypes.byref(d), ctypes.byref(w), 1) > 0
    assert front_call(T=0) == _abi.QSA_ERR_INVALID
    assert front_call(x=A + 4) == _abi.QSA_ERR_INVALID                    # misaligned activations
    assert front_call(ws_bytes=16) == _abi.QSA_ERR_WORKSPACE
    for field, value, status in (("w_type", _abi.TYPE_F16, _abi.QSA_ERR_UNSUPPORTED),
                                 ("n_embd", 2564, _abi.QSA_ERR_UNSUPPORTED), ("n_embd", 1 << 15, _abi.QSA_ERR_UNSUPPORTED),
                                 ("wv", None, _abi.QSA_ERR_INVALID), ("wk_idx", A + 8, _abi.QSA_ERR_INVALID)):
        bad = _abi.QsaFrontWeights.from_buffer_copy(w)
        setattr(bad, field, value)
        assert front_call(w=bad) == status, field


def test_output_host_refusals():
    d = make_desc(n_ctx=4096)
    L = lib()
    call = lambda wt=_abi.TYPE_BF16, n_embd=2560, attn=A, T=1, ws_bytes=0: L.qsa_output(
        ctypes.byref(d), A, n_embd, wt, T, attn, A, A, A if ws_bytes else None, ws_bytes, None)
    assert call(wt=TYPE_F16) == _abi.QSA_ERR_UNSUPPORTED
    assert call(attn=A + 4) == _abi.QSA_ERR_INVALID
    assert call(n_embd=0) == _abi.QSA_ERR_INVALID
    assert call(T=0) == _abi.QSA_ERR_INVALID
    assert L.qsa_output_workspace_size(ctypes.byref(d), 2560, _abi.TYPE_BF16, 16) == 0   # the GEMV path needs none
    assert L.qsa_output_workspace_size(ctypes.byref(d), 2560, TYPE_F16, 64) == 0         # no such weight type
    assert (L.qsa_output_workspace_size(ctypes.byref(d), 2560, _abi.TYPE_Q8_0, 64) >
            L.qsa_output_workspace_size(ctypes.byref(d), 2560, _abi.TYPE_BF16, 64))      # + attn_output as f16
    need = L.qsa_output_workspace_size(ctypes.byref(d), 2560, _abi.TYPE_BF16, 64)
    assert need >= 64 * 4096 * 2
    assert call(T=64) == _abi.QSA_ERR_WORKSPACE                                   # the GEMM path without one
    assert call(T=64, ws_bytes=need - 16) == _abi.QSA_ERR_WORKSPACE


def test_stage_copy_host_refusals():
    L = lib()
    assert L.qsa_stage_copy(None, A, 16, None) == _abi.QSA_ERR_INVALID
    assert L.qsa_stage_copy(A, A, 20, None) == _abi.QSA_ERR_INVALID          # not a multiple of 16 bytes
    assert L.qsa_stage_copy(A + 8, A, 16, None) == _abi.QSA_ERR_INVALID      # misaligned
    assert L.qsa_stage_copy(A, A, 0, None) == _abi.QSA_ERR_INVALID


def _slots(n=2, rank=0, epoch=A, regions=None):
    s = _abi.QsaPeerSlots()
    for r in range(min(n, 8)):
        s.region[r] = regions[r] if regions else A + r * (1 << 24)
    s.n_ranks, s.rank, s.epoch = n, rank, epoch
    return s


def test_fused_peer_exchange_host_refusals():
    """qsa_shard_decode_ri_peer / qsa_merge_states_peer refuse bad channel descriptions on the host:
    more than 8 ranks, a rank outside them, no epoch word, a region off 16 bytes; and the merge a
    batch of 0 or a status word under 16 bytes."""
    d = make_desc(n_ctx=4096)
    L = lib()
    dec = lambda s, batch=1: L.qsa_shard_decode_ri_peer(ctypes.byref(d), A, batch, 4096, 0, 32, A, _abi.TYPE_BF16, A,
                                                        None, None, None, ctypes.byref(s), None, A, 1 << 30, None)
    mrg = lambda s, batch=1, ws_bytes=64: L.qsa_merge_states_peer(ctypes.byref(d), ctypes.byref(s), batch, A, A,
                                                                  ws_bytes, None)
    for bad in (_slots(n=9), _slots(n=0), _slots(rank=2), _slots(rank=-1), _slots(epoch=None),
                _slots(regions=[A, A + 4])):
        assert dec(bad) == _abi.QSA_ERR_INVALID
        assert mrg(bad) == _abi.QSA_ERR_INVALID
    assert dec(_slots(), batch=0) == _abi.QSA_ERR_INVALID
    assert mrg(_slots(), batch=0) == _abi.QSA_ERR_INVALID
    assert mrg(_slots(), ws_bytes=8) == _abi.QSA_ERR_WORKSPACE
