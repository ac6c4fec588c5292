"""A CPU backend of the sharded decode built on the oracle (test infrastructure only).

It implements the three compute steps that qwfnfer_b200.shard.ShardedDecoder asks of a backend --
candidates, attend (global selection + attention state), merge -- with the oracle's scores,
selection rule and attention, on one shard's slice of host caches, so that the decoder's host
logic (block split, exchange order, packing, the merge) runs on gloo ranks without a GPU.  The
selection is restated here as a sort by (score descending, block ascending): the rule of
orc_select (oracle/qsa_oracle.cpp), which the tests check it against.
"""
from __future__ import annotations

import numpy as np
import torch

import oracle
from qwfnfer_b200._abi import TYPE_BF16, TYPE_F32, k_blocks


def forced_range(d, q):
    """Forced blocks [f_lo, f_hi] of the query at q (empty when f_lo > f_hi)."""
    bq = q // d.ratio
    if d.window > 0:
        return max(0, bq - (-(-d.window // d.ratio) + 1) + 1), bq
    return (bq, bq) if (q + 1) % d.ratio else (1, 0)


class OracleShardBackend:
    def __init__(self, d, kc, vc, pool, blocks):
        """kc, vc, pool: the GLOBAL host caches; the backend keeps only blocks [lo, hi) of them."""
        self.d = d
        self.kb = k_blocks(d)
        lo, hi = blocks
        r = d.ratio
        self.kc = np.ascontiguousarray(kc[lo * r:hi * r])
        self.vc = np.ascontiguousarray(vc[lo * r:hi * r])
        self.pool = np.ascontiguousarray(pool[lo:hi])
        self.blocks = blocks
        self.state_floats = 32 + 16 * d.head_dim

    def candidates(self, items, batch, max_n_kv, blocks, q_idx, k_new=None, v_new=None, kidx_new=None):
        assert k_new is None and v_new is None and kidx_new is None, "append is not restated here"
        assert tuple(blocks) == tuple(self.blocks)
        d, lo, hi = self.d, self.blocks[0], self.blocks[1]
        positions = list(items)
        q_idx = np.asarray(q_idx, dtype=np.float32).reshape(batch, -1)
        sc = oracle.scores(d, self.pool, hi - lo, q_idx)                # [batch, hi - lo]
        out = np.full((2, batch, self.kb), -1, np.int32)
        out[1] = 0
        for t, q in enumerate(positions):
            f_lo, f_hi = forced_range(d, q)
            want = self.kb - max(0, f_hi - f_lo + 1)
            n_vis = (q + 1) // d.ratio
            cands = [(-float(sc[t, b - lo]), b) for b in range(lo, min(hi, n_vis)) if not f_lo <= b <= f_hi]
            cands.sort()
            for i, (neg, b) in enumerate(cands[:want]):
                out[0, t, i] = b
                out[1, t, i] = np.float32(-neg).view(np.int32)
        return torch.from_numpy(out)

    def global_selection(self, gathered: np.ndarray, q: int, t: int) -> list[int]:
        d = self.d
        f_lo, f_hi = forced_range(d, q)
        want = self.kb - max(0, f_hi - f_lo + 1)
        pairs = []
        for sh in range(gathered.shape[0]):
            for j in range(self.kb):
                b = int(gathered[sh, 0, t, j])
                if b >= 0:
                    pairs.append((-float(np.int32(gathered[sh, 1, t, j]).view(np.float32)), b))
        pairs.sort()
        chosen = [b for _, b in pairs[:want]] + list(range(f_lo, f_hi + 1))
        return sorted(chosen)

    def attend(self, items, batch, max_n_kv, blocks, gathered, q, sel_out=None, n_shards=None, cand_stride=0):
        d, lo, hi = self.d, self.blocks[0], self.blocks[1]
        r = d.ratio
        gathered = gathered.numpy()
        positions = list(items)
        q_np = q.numpy() if q.dtype != torch.bfloat16 else q.view(torch.int16).numpy().view(np.uint16)
        q_type = TYPE_BF16 if q.dtype == torch.bfloat16 else TYPE_F32
        states = np.empty((batch, self.state_floats), np.float32)
        for t, qp in enumerate(positions):
            sel = self.global_selection(gathered, qp, t)
            if sel_out is not None:
                sel_out[t, :] = -1
                sel_out[t, :len(sel)] = torch.tensor(sel, dtype=torch.int32)
            mine = [b - lo for b in sel if lo <= b < hi]
            local = np.full(self.kb, -1, np.int32)
            local[:len(mine)] = mine
            # local cells: block b - lo, position qp - lo*r (negative: nothing of this shard is visible)
            states[t] = oracle.attend_state(d, self.kc, self.vc, [qp - lo * r], local, q_np[t:t + 1], q_type)[0]
        return torch.from_numpy(states)

    def merge(self, states, out=None):
        merged = torch.from_numpy(oracle.merge_states(self.d, states.numpy()))
        if out is None:
            return merged
        out.copy_(merged.view_as(out))
        return out
