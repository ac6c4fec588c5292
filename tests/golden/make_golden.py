"""Generate the committed golden vectors under tests/golden/ (run once; outputs are committed).

q8_0: gguf-py's Q8_0.quantize_blocks, whose source states "bit-exact same results as reference
implementation in ggml-quants.c" (quantize_row_q8_0_ref) -- the rounding ggml uses for q8_0 K/V
cache rows.  f16: numpy's float32 -> float16 cast, IEEE round-to-nearest-even, which is what
ggml's GGML_FP32_TO_FP16 (F16C) produces for the F16 indexer and pooled-key caches.

usage: python tests/golden/make_golden.py   (needs the `gguf` package; not needed at test time)
"""
import os

import numpy as np
from gguf.quants import Q8_0

HERE = os.path.dirname(os.path.abspath(__file__))


def q8_0_inputs() -> np.ndarray:
    rng = np.random.default_rng(20261201)
    blocks = [rng.standard_normal((256, 32)).astype(np.float32)]             # N(0,1) K/V rows
    blocks.append((rng.standard_normal((64, 32)) / 16).astype(np.float32))    # K scaled 1/sqrt(256)
    blocks.append((rng.standard_normal((32, 32)) * 1e4).astype(np.float32))   # large magnitudes
    blocks.append((rng.standard_normal((32, 32)) * 1e-6).astype(np.float32))  # f16-subnormal scales
    blocks.append(np.zeros((2, 32), np.float32))                              # amax == 0 -> d = 0
    # exact half-way products x*id = k + 0.5 (round half away from zero, not to even)
    ties = np.zeros((8, 32), np.float32)
    for i in range(8):
        ties[i, 0] = 127.0
        ties[i, 1:] = (np.arange(31, dtype=np.float32) - 15.0) + 0.5 * (1 if i % 2 else -1)
    blocks.append(ties)
    one_hot = np.zeros((4, 32), np.float32)
    one_hot[np.arange(4), np.arange(4) * 7] = np.array([1.0, -3.5, 65504.0, -1e-3], np.float32)
    blocks.append(one_hot)
    return np.concatenate(blocks, axis=0)


def f16_inputs() -> np.ndarray:
    rng = np.random.default_rng(7)
    vals = [rng.standard_normal(4096).astype(np.float32),
            (rng.standard_normal(512) * 1e-6).astype(np.float32),   # subnormal range of f16
            np.array([0.0, -0.0, 65504.0, 65520.0, 1e9, -1e9, 6.1e-5, 5.96e-8, 2.98e-8,
                      1.0 + 2 ** -11, 1.0 + 3 * 2 ** -11, np.inf, -np.inf], np.float32)]
    return np.concatenate(vals)


def main() -> None:
    x = q8_0_inputs()
    q = Q8_0.quantize_blocks(x.copy())
    assert q.shape == (x.shape[0], 34) and q.dtype == np.uint8
    np.savez_compressed(os.path.join(HERE, "q8_0_ggml_ref.npz"), x=x, q=q)
    f = f16_inputs()
    with np.errstate(over="ignore"):
        h = f.astype(np.float16).view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "f16_rne.npz"), x=f, h=h)
    print("wrote", x.shape[0], "q8_0 blocks and", f.size, "f16 values")


if __name__ == "__main__":
    main()
