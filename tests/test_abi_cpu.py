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
    assert ctypes.sizeof(_abi.QsaDesc) == 4 * 12 + 16 + 8 + 8
