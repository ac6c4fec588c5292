"""One rank of the sharded decode over NCCL (launched by tests/test_zz_shard_nccl.py):

    python -m torch.distributed.run --nnodes 1 --nproc-per-node N --master-addr 127.0.0.1 \
        --master-port P tests/shard_nccl_worker.py [nccl|peer] [sharded|replicated] [delay]

The exchange is NCCL's all-gather or libqsa's all-gather over NVLink peer memory; the indexer
caches are sharded with the K/V (candidates exchanged) or replicated on every rank.

Every rank fills its shard of two sequences' caches, runs one ShardedDecoder step (append of the
new token, the two all-gathers, the merge), and checks its status.  Rank 0 also builds the
unsharded caches on its GPU and runs qsa_decode on them; every rank's output and selection are
gathered to rank 0 and compared with it.  Rank 0 prints one line `SHARD_NCCL {...}`; the exit
code is 0 only if every check passed.

With `delay`, the step runs three times back to back and the last rank's host sleeps before
launching each wait for the peers (the wait of a push, or the state merge that waits for the
states the other ranks' kernels stored into its region), so the other ranks publish later rounds
while its wait has not been launched yet: the exchange must neither time out nor let a later
round overwrite slots still being read (every step's output is checked).
"""
from __future__ import annotations

import json
import os
import sys
import time
from datetime import timedelta

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "tests")]

from qwfnfer_b200._abi import QSA_OK, k_blocks, make_desc  # noqa: E402
from qwfnfer_b200.configs import fill_cache, token_inputs  # noqa: E402
from qwfnfer_b200.qsa import QsaNode, QsaState, decode_items  # noqa: E402
from qwfnfer_b200.shard import ShardedDecoder  # noqa: E402

ATTN_TOL = 2e-3


def _delay_waits(peer, seconds):
    """Make this rank's host sleep before launching each wait for the peers."""
    import qwfnfer_b200.shard as shard_mod
    real = shard_mod.lib

    class Slow:
        def __getattr__(self, name):
            fn = getattr(real(), name)
            if name not in ("qsa_peer_wait", "qsa_merge_states_peer"):
                return fn

            def wait(*a):
                torch.cuda.synchronize()        # the push has run; the peers may move on meanwhile
                time.sleep(seconds)
                return fn(*a)
            return wait

    shard_mod.lib = lambda: Slow()


def main() -> int:
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    rank, world = dist.get_rank(), dist.get_world_size()
    d = make_desc(n_ctx=65536, top_k_blocks=64, window=128)
    positions = [60031, 20000]                   # 60032 = 938 * 64: the token completes block 937
    seeds = [41, 42]
    exchange = sys.argv[1] if len(sys.argv) > 1 else "nccl"
    index = sys.argv[2] if len(sys.argv) > 2 else "sharded"
    delay = len(sys.argv) > 3 and sys.argv[3] == "delay"
    dec = ShardedDecoder(d, exchange=exchange, batch=2, index=index)
    if delay and dec.peer is not None and rank == world - 1:
        _delay_waits(dec.peer, 0.05)
    node = QsaNode(d)
    sts = [QsaState(d, blocks=dec.blocks, index_full=dec.index_replicated) for _ in positions]
    for st, n, s in zip(sts, positions, seeds):
        fill_cache(node, st, 0, n, s, append=dec.append)
    q, q_idx, k, v, ki = token_inputs(d, 2, seed=43)
    items = decode_items([s.layer() for s in sts], positions)
    B, KB, max_n_kv = len(positions), k_blocks(d), max(positions) + 1
    sel = torch.empty((B, KB), dtype=torch.int32, device=dev)
    # with `delay`, the same step (it rewrites the token's row with the same bytes) three times
    step_outs = [dec.step(items, B, max_n_kv, q, q_idx, k, v, ki, sel_out=sel).clone() for _ in range(3 if delay else 1)]
    out = step_outs[-1]
    steps_equal = all(torch.equal(o, out) for o in step_outs)
    st_code = dec.check(B, max_n_kv)
    if dec.peer is not None and st_code == QSA_OK:
        st_code = dec.peer.check()
    status = torch.tensor([st_code], dtype=torch.int32, device=dev)
    outs = [torch.empty_like(out) for _ in range(world)]
    sels = [torch.empty_like(sel) for _ in range(world)]
    stats = [torch.empty_like(status) for _ in range(world)]
    dist.all_gather(outs, out)
    dist.all_gather(sels, sel)
    dist.all_gather(stats, status)
    ok = True
    if rank == 0:
        full = [QsaState(d) for _ in positions]
        for st, n, s in zip(full, positions, seeds):
            fill_cache(node, st, 0, n, s)
        sel_ref = torch.empty_like(sel)
        out_ref = node.sparse_attn_decode(decode_items([s.layer() for s in full], positions), B, max_n_kv,
                                          q, q_idx, k, v, ki, sel_out=sel_ref)
        torch.cuda.synchronize()
        ref_max = out_ref.abs().max().item()
        errs = [((o - out_ref).abs().max().item()) / ref_max for o in outs]
        sel_ok = [bool(torch.equal(s, sel_ref)) for s in sels]
        same = all(torch.equal(o, outs[0]) for o in outs)
        statuses = [int(s.item()) for s in stats]
        ok = (all(sel_ok) and max(errs) <= ATTN_TOL and same and all(s == QSA_OK for s in statuses)
              and steps_equal)
        print("SHARD_NCCL " + json.dumps({"world": world, "exchange": exchange, "index": index, "blocks": dec.blocks,
                                          "delay": delay, "steps_equal": steps_equal,
                                          "rel_err": errs, "sel_equal": sel_ok,
                                          "ranks_identical": same, "status": statuses, "ok": ok}), flush=True)
    flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
    dist.broadcast(flag, 0)
    if dec.peer is not None:
        torch.cuda.synchronize()
        dist.barrier()
        dec.peer.close()
    dist.destroy_process_group()
    return 0 if flag.item() == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
