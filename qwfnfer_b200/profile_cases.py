"""Small, fixed workloads of the QSA kernels for profilers (ncu captures one launch of them).

    python -m qwfnfer_b200.profile_cases batch B STEPS    # B decode queries over one config-2 cache
    python -m qwfnfer_b200.profile_cases decode STEPS     # the config-2 decode step (append + select + attend)
    python -m qwfnfer_b200.profile_cases prefill T N_PAST STEPS   # one qsa_prefill chunk (config-4 shape)

`batch` places the B queries at positions 163839 - 64 i of one 160K q8_0 cache (no append), so the attention runs in its
multi-tile streaming regime with 220 MB of caches on the device; `decode` is one token of config 2.  `prefill` appends
T tokens at N_PAST of a q8_0 cache and runs the whole chunk (T=4096 at 77824 keeps config 4's ~210 queries per block
with about 2.5 GB on the device).  Each step is preceded by a 256 MB L2 flush; the device time of every step is printed.
"""
from __future__ import annotations

import sys

import torch

from .configs import CONFIGS, fill_cache, token_inputs
from .qsa import QsaNode, QsaState, decode_items


def main(argv: list[str]) -> None:
    kind = argv[0] if argv else "batch"
    if kind == "prefill":
        return prefill(argv[1:])
    cfg = CONFIGS[2]
    d = cfg.desc()
    node, st = QsaNode(d), QsaState(d)
    fill_cache(node, st, 0, cfg.n_past + 1, cfg.seed)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    if kind == "batch":
        B = int(argv[1]) if len(argv) > 1 else 16
        steps = int(argv[2]) if len(argv) > 2 else 3
        q, qi, _, _, _ = token_inputs(d, B, 99)
        items = decode_items([st.layer()] * B, [cfg.n_past - 64 * i for i in range(B)])
        ws = node.workspace("decode", B, cfg.n_past + 1)
        run = lambda: node.sparse_attn_decode(items, B, cfg.n_past + 1, q, qi, ws=ws)
    else:
        steps = int(argv[1]) if len(argv) > 1 else 3
        q, qi, k, v, ki = token_inputs(d, 1, 99)
        items = decode_items([st.layer()], [cfg.n_past])
        ws = node.workspace("decode", 1, cfg.n_past + 1)
        run = lambda: node.sparse_attn_decode(items, 1, cfg.n_past + 1, q, qi, k, v, ki, ws=ws)
    torch.cuda.synchronize()
    ev = []
    for _ in range(steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        run()
        b.record()
        ev.append((a, b))
    torch.cuda.synchronize()
    print("us per step:", [round(a.elapsed_time(b) * 1e3, 1) for a, b in ev])


def prefill(argv: list[str]) -> None:
    T = int(argv[0]) if argv else 4096
    n_past = int(argv[1]) if len(argv) > 1 else 77824
    steps = int(argv[2]) if len(argv) > 2 else 3
    cfg = CONFIGS[4]
    d = cfg.desc(n_ctx=n_past + T)
    node, st = QsaNode(d), QsaState(d)
    fill_cache(node, st, 0, n_past, cfg.seed)
    q, qi, k, v, ki = token_inputs(d, T, cfg.seed + 1000)
    ws = node.workspace("prefill", T, n_past + T)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    ev = []
    for _ in range(steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        node.sparse_attn(st.layer(), n_past, q, qi, k, v, ki, ws=ws)
        b.record()
        ev.append((a, b))
    torch.cuda.synchronize()
    print("us per step:", [round(a.elapsed_time(b) * 1e3, 1) for a, b in ev])


if __name__ == "__main__":
    main(sys.argv[1:])
