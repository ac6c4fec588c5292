"""Shared checks of the parity tests: the CUDA path (libqsa.so) against the CPU oracle."""
from __future__ import annotations

import numpy as np

import oracle
from qwfnfer_b200._abi import k_blocks

ATTN_TOL = 2e-3      # max |out - ref| / max |ref| over the [n_head, head_dim] output (fp32 softmax)
POOL_TOL = 1e-5      # pooled keys, f32 before the f16 store


def host_caches(state, il, n_rows):
    """Host copies (K bytes, V bytes, idx f16 bits, pool f16 bits) of layer il's caches."""
    kc = state.k[il][:n_rows].cpu().numpy()
    vc = state.v[il][:n_rows].cpu().numpy()
    ic = state.idx[il][:n_rows].cpu().numpy().view(np.uint16)
    pool = state.pool[il].cpu().numpy().view(np.uint16)
    return kc, vc, ic, pool


def forced_blocks(d, q):
    r = d.ratio
    bq = q // r
    if d.window > 0:
        nf = -(-d.window // r) + 1
        return set(range(max(0, bq - nf + 1), bq + 1))
    return {bq} if (q + 1) % r else set()


def check_selection(d, sel_gpu_row, scores_row, q):
    """Selected block sets equal, excluding blocks whose score is within 4 ulp of the k-th kept
    score (near-ties, which the reference's own backends order differently).  Returns the
    number of near-tie blocks excluded (0 means the sets were compared whole)."""
    sel_o, _ = oracle.select(d, scores_row, q)
    got = {int(b) for b in sel_gpu_row if b >= 0}
    want = {int(b) for b in sel_o if b >= 0}
    forced = forced_blocks(d, q)
    kept = sorted((scores_row[b] for b in want - forced), reverse=True)
    ties = set()
    if kept:
        kth = np.float32(kept[-1])
        ulp = np.spacing(np.abs(kth)) if kth != 0 else np.float32(1e-30)
        n_vis = (q + 1) // d.ratio
        ties = {b for b in range(n_vis) if b not in forced and abs(scores_row[b] - kth) <= 4 * ulp}
    assert got - ties == want - ties, f"q={q}: gpu-only {sorted(got - want)} oracle-only {sorted(want - got)}"
    assert len(got) == len(want)
    return len(ties & (got ^ want))


def rel_err(out, ref):
    return float(np.abs(out - ref).max() / max(np.abs(ref).max(), 1e-30))


def sel_matrix(sel_list, d):
    KB = k_blocks(d)
    m = np.full((len(sel_list), KB), -1, np.int32)
    for i, s in enumerate(sel_list):
        s = [b for b in s if b >= 0]
        m[i, :len(s)] = s
    return m
