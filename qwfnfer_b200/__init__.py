"""qwfnfer_b200 -- B200-native sparse-attention (QSA) hot path of the QwFNfer engine.

The compute lives in libqsa.so (hand-written sm_100a CUDA behind the C ABI of include/qsa.h);
this package holds its ctypes binding and a host mirror of the reference's node interface.
"""
from ._abi import (QsaDecodeItem, QsaDesc, QsaError, QsaLayerCache, TYPE_BF16, TYPE_F16, TYPE_F32, TYPE_Q8_0,
                   k_blocks, lib, make_desc, row_bytes)

__all__ = ["QsaDecodeItem", "QsaDesc", "QsaError", "QsaLayerCache", "TYPE_BF16", "TYPE_F16", "TYPE_F32",
           "TYPE_Q8_0", "k_blocks", "lib", "make_desc", "row_bytes"]
