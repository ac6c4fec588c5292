"""Small, fixed workloads of the QSA kernels for profilers (ncu captures one launch of them).

    python profile_cases.py batch B STEPS    # B decode queries over one config-2 cache
    python profile_cases.py decode STEPS     # the config-2 decode step (append + select + attend)
    python profile_cases.py prefill T N_PAST STEPS   # one qsa_prefill chunk (config-4 shape)
    python profile_cases.py front T STEPS    # qsa_front for T tokens (n_embd 2560, bf16 weights)
    python profile_cases.py output T STEPS   # qsa_output for T tokens (4096 -> 2560, bf16 weights)
    python -m torch.distributed.run --nproc-per-node N ... profile_cases.py shard5 peer|nccl [lb] [ri]
                                                          # config-5 sharded step: per-kernel timeline per rank

`batch` places the B queries at positions 163839 - 64 i of one 160K q8_0 cache (no append), so the attention runs in its
multi-tile streaming regime with 220 MB of caches on the device; `decode` is one token of config 2.  `prefill` appends
T tokens at N_PAST of a q8_0 cache and runs the whole chunk (T=4096 at 77824 keeps config 4's ~210 queries per block
with about 2.5 GB on the device).  Each step is preceded by a 256 MB L2 flush; the device time of every step is printed.
`front` projects T tokens through the layer's 48.5 MB of bf16 projection weights (the config-2 descriptor), each
step after the 256 MB L2 flush, so the weights come from DRAM.
`shard5` replays the config-5 sharded decode step (one layer after another, or with `lb` the 12 layers as one batch,
captured twice per replay so that the state exchange's two channels alternate; `ri`: indexer caches replicated;
exchange `peer` (states stored by the attention into every rank's buffer), `peer_push` or `nccl`)
from a CUDA graph under torch.profiler and prints, per rank, each kernel's median start offset and duration within
the step (CUPTI activity records; a breakdown, not a bench value).
"""
from __future__ import annotations

import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from qwfnfer_b200.configs import CONFIGS, fill_cache, token_inputs  # noqa: E402
from qwfnfer_b200.qsa import QsaNode, QsaState, decode_items  # noqa: E402


def main(argv: list[str]) -> None:
    kind = argv[0] if argv else "batch"
    if kind == "prefill":
        return prefill(argv[1:])
    if kind == "shard5":
        return shard5(argv[1:])
    if kind == "front":
        return front(argv[1:])
    if kind == "output":
        return output(argv[1:])
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


def front(argv: list[str]) -> None:
    from qwfnfer_b200.configs import front_weights
    from qwfnfer_b200.qsa import QsaFront

    T = int(argv[0]) if argv else 1
    steps = int(argv[1]) if len(argv) > 1 else 3
    d = CONFIGS[2].desc()
    fr = QsaFront(d, **front_weights(d, seed=5))
    x = torch.randn(T, fr.n_embd, generator=torch.Generator(device="cuda").manual_seed(6), device="cuda")
    pos = torch.arange(CONFIGS[2].n_past - T + 1, CONFIGS[2].n_past + 1, dtype=torch.int32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    ev = []
    for _ in range(steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fr.project(x, pos)
        b.record()
        ev.append((a, b))
    torch.cuda.synchronize()
    print("us per step:", [round(a.elapsed_time(b) * 1e3, 1) for a, b in ev])


def output(argv: list[str]) -> None:
    from qwfnfer_b200.configs import N_EMBD
    from qwfnfer_b200.qsa import QsaOutput

    T = int(argv[0]) if argv else 1
    steps = int(argv[1]) if len(argv) > 1 else 3
    d = CONFIGS[2].desc()
    g = torch.Generator(device="cuda").manual_seed(7)
    n_in = d.n_head * d.head_dim
    op = QsaOutput(d, (torch.randn(N_EMBD, n_in, generator=g, device="cuda") * 0.02).to(torch.bfloat16))
    attn = torch.randn(T, d.n_head, d.head_dim, generator=g, device="cuda")
    gate = torch.randn(T, n_in, generator=g, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    ev = []
    for _ in range(steps):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        op.project(attn, gate)
        b.record()
        ev.append((a, b))
    torch.cuda.synchronize()
    print("us per step:", [round(a.elapsed_time(b) * 1e3, 1) for a, b in ev])


def shard5(argv: list[str]) -> None:
    import os
    import statistics
    from datetime import timedelta

    import torch.distributed as dist
    from torch.profiler import ProfilerActivity, profile

    from qwfnfer_b200._abi import k_blocks
    from qwfnfer_b200.shard import ShardedDecoder

    local, ws = int(os.environ.get("LOCAL_RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    rank = dist.get_rank() if ws > 1 else 0
    exchange = argv[0] if argv else "peer"
    lb = "lb" in argv
    cfg = CONFIGS[5]
    d = cfg.desc()
    NL, n_past = cfg.layers, cfg.n_past
    index = "replicated" if "ri" in argv else "sharded"
    dec = ShardedDecoder(d, rank=rank, world=ws, exchange=exchange, batch=NL if lb else 1, index=index)
    node = QsaNode(d, dev)
    st = QsaState(d, n_layers=NL, device=dev, blocks=dec.blocks, index_full=dec.index_replicated)
    for il in range(NL):
        fill_cache(node, st, il, n_past, cfg.seed * 1000 + il, append=dec.append)
    items = [decode_items([st.layer(il)], [n_past], device=dev) for il in range(NL)]
    items_all = decode_items([st.layer(il) for il in range(NL)], [n_past] * NL, device=dev)
    q, qi, k, v, ki = token_inputs(d, NL, cfg.seed + 100)
    sel = torch.empty(NL, k_blocks(d), dtype=torch.int32, device=dev)

    def step():
        if lb:
            dec.step(items_all, NL, n_past + 1, q, qi, k, v, ki, sel_out=sel)
            return
        for il in range(NL):
            dec.step(items[il], 1, n_past + 1, q[il:il + 1], qi[il:il + 1], k[il:il + 1], v[il:il + 1],
                     ki[il:il + 1], sel_out=sel[il:il + 1])

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    # the batched step twice per replay: the replicated-index state exchange alternates two peer
    # channels per step, which a graph of one step would fix to one
    reps = 2 if lb else 1
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        for _ in range(reps):
            step()
    for _ in range(5):
        g.replay()
    torch.cuda.synchronize()
    if ws > 1:
        dist.barrier()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(10):
            flush.zero_()
            g.replay()
        torch.cuda.synchronize()
    evs = sorted((e for e in prof.events() if e.device_type.name == "CUDA"), key=lambda e: e.time_range.start)
    steps, cur = [], None
    for e in evs:                              # a step is the kernels (libqsa's, NCCL's) after each flush
        if "FillFunctor" in e.name:
            cur = []
            steps.append(cur)
        elif cur is not None:
            cur.append((e.name, e.time_range.start, e.time_range.end))
    rows, spans = {}, []
    for s_ in steps[2:]:
        if not s_:
            continue
        t0 = s_[0][1]
        spans.append(s_[-1][2] - t0)
        for i, (n, a, b) in enumerate(s_):
            rows.setdefault(f"{i:02d} {n.split('(')[0]}", []).append((a - t0, b - a))
    lines = [f"rank {rank} of {ws}, exchange {exchange}, {'12 layers as one batch' if lb else 'layer after layer'}: "
             f"replay of {reps} token(s) {statistics.median(spans):.1f} us (median of {len(spans)})"]
    for key, vals in list(rows.items())[:64]:
        lines.append(f"  {key:48s} start {statistics.median([x for x, _ in vals]):8.1f} us  "
                     f"duration {statistics.median([y for _, y in vals]):7.1f} us")
    print("\n".join(lines), flush=True)
    del g
    if dec.peer is not None:
        torch.cuda.synchronize()
        dist.barrier()
        dec.peer.close()
    if ws > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1:])
