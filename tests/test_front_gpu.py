"""qsa_front (the projections, norms and IMRoPE feeding the node) and qsa_output (the gated output
projection after it) on a B200 against the CPU oracle; the front pinned to the GPU's own pooled keys
and chained into qsa_decode and qsa_output.

Tolerances: a projection's f32 sum may differ from the oracle's (double sum, one rounding) by the
f32 accumulation error, bounded here by 1e-5 of the row's sum of |w * x|; the normed and roped
outputs within 1e-4 of their largest magnitude."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
from qwfnfer_b200._abi import (QSA_ERR_INVALID, QSA_ERR_UNSUPPORTED, QSA_ERR_WORKSPACE, QsaFrontWeights, TYPE_BF16,
                               TYPE_F16, TYPE_Q8_0, lib, make_desc)
from qwfnfer_b200.configs import fill_cache, front_weights
from qwfnfer_b200.qsa import QsaFront, QsaNode, QsaOutput, QsaState, decode_items
from test_gpu_parity import desc_for, run_decode_case

pytestmark = pytest.mark.gpu

PROJ_TOL = 1e-5      # of the row's sum of |w * x|
NORMED_TOL = 1e-4    # of the output's largest magnitude


def host_weights(w: dict) -> dict:
    out = {}
    for k, t in w.items():
        out[k] = t.view(torch.int16).cpu().numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.cpu().numpy()
    return out


def abs_row_sums(wt: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """[T][rows] sums of |w * bf16(x)| (the scale of a row's rounding error)."""
    return x.to(torch.bfloat16).float().abs() @ wt.float().abs().T


@pytest.mark.parametrize("idx_n_head,T", [(1, 1), (1, 6), (4, 3)])
def test_front_matches_oracle(idx_n_head, T):
    d = make_desc(idx_n_head=idx_n_head, n_ctx=1 << 20)
    w = front_weights(d, seed=11 + T, gammas=True)
    front = QsaFront(d, **w)
    g = torch.Generator(device="cuda").manual_seed(12)
    x = torch.randn(T, front.n_embd, generator=g, device="cuda")
    pos_list = [163839, 0, 70000, 1048575, 5, 129][:T]
    pos = torch.tensor(pos_list, dtype=torch.int32, device="cuda")
    q, gate, q_idx, k, v, kidx = front.project(x, pos)
    torch.cuda.synchronize()
    ref = oracle.front(d, host_weights(w), np.array(pos_list, np.int32), x.cpu().numpy())
    hd = d.head_dim
    wq_gate = w["wq"].view(d.n_head, 2, hd, -1)[:, 1].reshape(d.n_head * hd, -1)
    for name, got, wt in (("gate", gate, wq_gate), ("v", v, w["wv"]), ("kidx", kidx, w["wk_idx"])):
        bound = PROJ_TOL * abs_row_sums(wt, x).cpu().numpy()
        err = np.abs(got.cpu().numpy() - ref[name])
        assert np.all(err <= bound + 1e-30), (name, float(err.max()), float(bound.max()))
    for name, got in (("q", q), ("k", k), ("q_idx", q_idx)):
        e = np.abs(got.cpu().numpy() - ref[name]).max() / np.abs(ref[name]).max()
        assert e <= NORMED_TOL, (name, e)


GEMM_PROJ_TOL = 1e-4    # the GEMM path: the tensor cores' f32 accumulation order, of the row's sum of |w * x|


@pytest.mark.parametrize("idx_n_head,T", [(1, 17), (2, 40)])
def test_front_gemm_path_matches_oracle(idx_n_head, T):
    """Above 16 tokens (a prefill chunk) the projections run as one tcgen05 GEMM (bf16 products,
    f32 accumulation) whose epilogue applies the norms and IMRoPE (17 and 40 tokens: a partly
    filled 128-row tile); the outputs agree with the oracle as the GEMV path's do."""
    d = make_desc(idx_n_head=idx_n_head, n_ctx=1 << 20)
    w = front_weights(d, seed=50 + T, gammas=True)
    front = QsaFront(d, **w)
    g = torch.Generator(device="cuda").manual_seed(51)
    x = torch.randn(T, front.n_embd, generator=g, device="cuda")
    pos_list = [int(p) for p in torch.randint(0, 163840, (T,), generator=torch.Generator().manual_seed(T))]
    pos = torch.tensor(pos_list, dtype=torch.int32, device="cuda")
    q, gate, q_idx, k, v, kidx = front.project(x, pos)
    torch.cuda.synchronize()
    ref = oracle.front(d, host_weights(w), np.array(pos_list, np.int32), x.cpu().numpy())
    hd = d.head_dim
    wq_gate = w["wq"].view(d.n_head, 2, hd, -1)[:, 1].reshape(d.n_head * hd, -1)
    for name, got, wt in (("gate", gate, wq_gate), ("v", v, w["wv"]), ("kidx", kidx, w["wk_idx"])):
        bound = GEMM_PROJ_TOL * abs_row_sums(wt, x).cpu().numpy()
        err = np.abs(got.cpu().numpy() - ref[name])
        assert np.all(err <= bound + 1e-30), (name, float(err.max()), float(bound.max()))
    for name, got in (("q", q), ("k", k), ("q_idx", q_idx)):
        e = np.abs(got.cpu().numpy() - ref[name]).max() / np.abs(ref[name]).max()
        assert e <= NORMED_TOL, (name, e)


@pytest.mark.parametrize("b", [3, 2000])
def test_front_q_idx_equals_gpu_pooled_key(b):
    """The front's indexer query of one-hot activations over weights holding u, at position b*r,
    equals (as f16 bits) the pooled key the append path computes for a block of r raw keys equal to
    u, with the same norm weight: the two kernels share the norm and IMRoPE arithmetic."""
    r = 64
    gamma = (1 + 0.1 * torch.randn(128, generator=torch.Generator().manual_seed(b))).cuda()
    d = make_desc(n_ctx=(b + 1) * r, idx_n_head=1, k_norm_w=gamma.data_ptr())
    rng = np.random.default_rng(b)
    u = torch.from_numpy((rng.integers(-32, 33, d.idx_dim) / 8.0).astype(np.float32)).cuda()
    node, st = QsaNode(d), QsaState(d)
    kv = d.n_head_kv * d.head_dim
    node.append(st.layer(), b * r, torch.zeros(r, kv, device="cuda"), torch.zeros(r, kv, device="cuda"),
                u[None, :].repeat(r, 1).contiguous())
    w = front_weights(d, n_embd=64, seed=3)
    j = 13
    wq_idx = torch.zeros(d.idx_dim, 64, device="cuda")
    wq_idx[:, j] = u
    w["wq_idx"], w["q_idx_norm"] = wq_idx.to(torch.bfloat16), gamma
    x = torch.zeros(1, 64, device="cuda")
    x[0, j] = 1.0
    _, _, q_idx, _, _, _ = QsaFront(d, **w).project(x, torch.tensor([b * r], dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    got16 = q_idx[0, 0].cpu().numpy().astype(np.float16).view(np.uint16)
    pool16 = st.pool[0][b].cpu().numpy().view(np.uint16)
    assert np.array_equal(got16, pool16)


@pytest.mark.parametrize("kv_type,n_past", [(TYPE_Q8_0, 30015), (TYPE_F16, 4095)])
def test_front_then_decode(kv_type, n_past):
    """qsa_front's outputs are qsa_decode's inputs as they are: q as QSA_TYPE_F32, the indexer query,
    the new K/V rows (appended bit-exact) and the raw indexer key; the decode then meets every
    parity bar against the oracle over the caches it wrote."""
    d = desc_for(kv_type, 32768)
    w = front_weights(d, seed=21, gammas=True)
    x = torch.randn(1, w["wq"].shape[1], generator=torch.Generator(device="cuda").manual_seed(22), device="cuda")
    q, _, q_idx, k, v, kidx = QsaFront(d, **w).project(x, torch.tensor([n_past], dtype=torch.int32, device="cuda"))
    run_decode_case(d, n_past, seed=23, inputs=(q, q_idx, k, v, kidx))


def test_front_argument_errors():
    """Refused on the host before anything is launched."""
    d = make_desc(n_ctx=4096)
    w = front_weights(d, n_embd=64, seed=1)
    front = QsaFront(d, **w)
    x = torch.zeros(1, 64, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    outs = [torch.empty(4096, device="cuda") for _ in range(6)]
    ws = front.workspace(1)
    L = lib()

    def call(wts, xp=x.data_ptr(), ws_bytes=ws.numel()):
        return L.qsa_front(ctypes.byref(d), ctypes.byref(wts), 1, pos.data_ptr(), xp, *[o.data_ptr() for o in outs],
                           ws.data_ptr(), ws_bytes, torch.cuda.current_stream().cuda_stream)

    bad = QsaFrontWeights.from_buffer_copy(front.w)
    bad.w_type = TYPE_F16
    assert call(bad) == QSA_ERR_UNSUPPORTED
    bad = QsaFrontWeights.from_buffer_copy(front.w)
    bad.n_embd = 60
    assert call(bad) == QSA_ERR_UNSUPPORTED
    assert call(front.w, xp=x.data_ptr() + 4) == QSA_ERR_INVALID
    assert call(front.w, ws_bytes=16) == QSA_ERR_WORKSPACE
    bad = QsaFrontWeights.from_buffer_copy(front.w)
    bad.wk = None
    assert call(bad) == QSA_ERR_INVALID
    torch.cuda.synchronize()


def output_bound(wo: torch.Tensor, attn: torch.Tensor, gate: torch.Tensor, tol: float = PROJ_TOL) -> np.ndarray:
    """Per (token, row): 1e-5 of the sum of |w * z| plus one bf16 rounding step of the largest term
    (the device and host expf may round one gated value to a neighbouring bf16)."""
    T = attn.shape[0]
    z = (attn.reshape(T, -1) * torch.sigmoid(gate)).abs()
    W = wo.float().abs()
    s = z @ W.T
    m = torch.stack([(z[t][None, :] * W).max(dim=1).values for t in range(T)])
    return (tol * s + 2 ** -7 * m).cpu().numpy()


@pytest.mark.parametrize("T,n_embd", [(1, 2560), (5, 2560), (2, 1000)])
def test_output_matches_oracle(T, n_embd):
    d = make_desc()
    g = torch.Generator(device="cuda").manual_seed(31 + T)
    n_in = d.n_head * d.head_dim
    wo = (torch.randn(n_embd, n_in, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    attn = torch.randn(T, d.n_head, d.head_dim, generator=g, device="cuda")
    gate = 2 * torch.randn(T, n_in, generator=g, device="cuda")
    y = QsaOutput(d, wo).project(attn, gate)
    torch.cuda.synchronize()
    ref = oracle.output(d, wo.view(torch.int16).cpu().numpy().view(np.uint16), attn.cpu().numpy(), gate.cpu().numpy())
    err = np.abs(y.cpu().numpy() - ref)
    bound = output_bound(wo, attn, gate)
    assert np.all(err <= bound), float((err / bound).max())


@pytest.mark.parametrize("T,n_embd", [(17, 2560), (48, 1000)])
def test_output_gemm_path_matches_oracle(T, n_embd):
    """Above 16 tokens the output side is one tcgen05 GEMM (bf16 products, f32 accumulation) over
    the gated activations rounded to bf16; the bound takes its accumulation order (GEMM_PROJ_TOL)."""
    d = make_desc()
    g = torch.Generator(device="cuda").manual_seed(61 + T)
    n_in = d.n_head * d.head_dim
    wo = (torch.randn(n_embd, n_in, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    attn = torch.randn(T, d.n_head, d.head_dim, generator=g, device="cuda")
    gate = 2 * torch.randn(T, n_in, generator=g, device="cuda")
    y = QsaOutput(d, wo).project(attn, gate)
    torch.cuda.synchronize()
    ref = oracle.output(d, wo.view(torch.int16).cpu().numpy().view(np.uint16), attn.cpu().numpy(), gate.cpu().numpy())
    err = np.abs(y.cpu().numpy() - ref)
    bound = output_bound(wo, attn, gate, GEMM_PROJ_TOL)
    assert np.all(err <= bound), float((err / bound).max())


def test_front_decode_output_chain():
    """The node end to end for one token: qsa_front -> qsa_decode -> qsa_output, each stage's
    output feeding the next as it is; the output stage checked against the oracle on the GPU's own
    intermediates (the earlier stages have their own parity tests)."""
    d = desc_for(TYPE_Q8_0, 16384)
    n_past = 12000
    node, st = QsaNode(d), QsaState(d)
    fill_cache(node, st, 0, n_past, 41)
    w = front_weights(d, seed=42, gammas=True)
    g = torch.Generator(device="cuda").manual_seed(43)
    x = torch.randn(1, w["wq"].shape[1], generator=g, device="cuda")
    q, gate, q_idx, k, v, kidx = QsaFront(d, **w).project(x, torch.tensor([n_past], dtype=torch.int32, device="cuda"))
    attn = node.sparse_attn_decode(decode_items([st.layer()], [n_past]), 1, n_past + 1, q, q_idx, k, v, kidx)
    wo = (torch.randn(2560, d.n_head * d.head_dim, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    y = QsaOutput(d, wo).project(attn, gate)
    torch.cuda.synchronize()
    ref = oracle.output(d, wo.view(torch.int16).cpu().numpy().view(np.uint16), attn.cpu().numpy(), gate.cpu().numpy())
    assert np.all(np.abs(y.cpu().numpy() - ref) <= output_bound(wo, attn, gate))
    assert np.isfinite(ref).all()


def test_output_argument_errors():
    d = make_desc()
    n_in = d.n_head * d.head_dim
    wo = torch.zeros(64, n_in, dtype=torch.bfloat16, device="cuda")
    attn = torch.zeros(1, n_in + 4, device="cuda")
    gate = torch.zeros(1, n_in, device="cuda")
    y = torch.zeros(1, 64, device="cuda")
    L, st = lib(), torch.cuda.current_stream().cuda_stream

    def call(w_type=TYPE_BF16, n_embd=64, ap=attn.data_ptr(), T=1):
        return L.qsa_output(ctypes.byref(d), wo.data_ptr(), n_embd, w_type, T, ap, gate.data_ptr(), y.data_ptr(),
                            None, 0, st)

    assert call(w_type=TYPE_F16) == QSA_ERR_UNSUPPORTED
    assert call(ap=attn.data_ptr() + 4) == QSA_ERR_INVALID
    assert call(n_embd=0) == QSA_ERR_INVALID
    assert call(T=32) == QSA_ERR_WORKSPACE            # above 16 tokens the GEMM path needs a workspace
    torch.cuda.synchronize()


@pytest.mark.parametrize("which", ["front", "output"])
def test_projection_gemm_full_chunk_sampled(which):
    """A whole 8192-token prefill chunk through the GEMM path (64 row tiles; every weight tile of the
    front, or of attn_output at n_embd 2560), checked against the oracle on 40 sampled tokens (the
    projections of a token depend on that token only)."""
    d = make_desc(n_ctx=1 << 20)
    T = 8192
    g = torch.Generator(device="cuda").manual_seed(71)
    samples = sorted(set([0, 1, 127, 128, 4095, 8190, 8191] + list(range(5, T, 251))))[:40]
    if which == "front":
        w = front_weights(d, seed=72, gammas=True)
        front = QsaFront(d, **w)
        x = torch.randn(T, front.n_embd, generator=g, device="cuda")
        pos = torch.randint(0, 1 << 20, (T,), generator=g, device="cuda", dtype=torch.int32)
        outs = front.project(x, pos)
        torch.cuda.synchronize()
        xs = x[samples]
        ref = oracle.front(d, host_weights(w), pos[samples].cpu().numpy(), xs.cpu().numpy())
        q, gate, q_idx, k, v, kidx = (t[samples] for t in outs)
        hd = d.head_dim
        wq_gate = w["wq"].view(d.n_head, 2, hd, -1)[:, 1].reshape(d.n_head * hd, -1)
        for name, got, wt in (("gate", gate, wq_gate), ("v", v, w["wv"]), ("kidx", kidx, w["wk_idx"])):
            bound = GEMM_PROJ_TOL * abs_row_sums(wt, xs).cpu().numpy()
            err = np.abs(got.cpu().numpy() - ref[name])
            assert np.all(err <= bound + 1e-30), (name, float(err.max()), float(bound.max()))
        for name, got in (("q", q), ("k", k), ("q_idx", q_idx)):
            e = np.abs(got.cpu().numpy() - ref[name]).max() / np.abs(ref[name]).max()
            assert e <= NORMED_TOL, (name, e)
    else:
        n_in = d.n_head * d.head_dim
        wo = (torch.randn(2560, n_in, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        attn = torch.randn(T, d.n_head, d.head_dim, generator=g, device="cuda")
        gate = 2 * torch.randn(T, n_in, generator=g, device="cuda")
        y = QsaOutput(d, wo).project(attn, gate)
        torch.cuda.synchronize()
        a_s, g_s = attn[samples], gate[samples]
        ref = oracle.output(d, wo.view(torch.int16).cpu().numpy().view(np.uint16), a_s.cpu().numpy(), g_s.cpu().numpy())
        err = np.abs(y[samples].cpu().numpy() - ref)
        assert np.all(err <= output_bound(wo, a_s, g_s, GEMM_PROJ_TOL)), float(err.max())


# q8_0 projection weights.  GEMV path (up to 16 tokens): integer block dots (dp4a) of the q8_0
# weights with the q8_0-quantised activations, f32 sums of the block terms, as ggml's mul_mat; bound
# 1e-5 of the row's sum of |w x| over the dequantised operands.  GEMM path: the tensor-core products
# of the f16 roundings of every d * q (2^-11 relative each), bound 2e-4 of that sum and 2e-3 of the
# largest normed output (the q8_0 quantisation itself moves the result by ~1%).
Q8_GEMV_TOL, Q8_GEMM_TOL, Q8_GEMM_NORMED_TOL = 1e-5, 2e-4, 2e-3


def q8_abs_row_sums(wq8: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """[T][rows] sums of |w * x| over the dequantised q8_0 weight and q8_0-quantised activation."""
    from qwfnfer_b200.configs import q8_0_rows, q8_0_rows_dequant
    xd = q8_0_rows_dequant(q8_0_rows(x))
    return xd.abs() @ q8_0_rows_dequant(wq8).abs().T


@pytest.mark.parametrize("T", [1, 5, 40])
def test_front_q8_0_weights_match_oracle(T):
    d = make_desc(n_ctx=1 << 20, idx_n_head=1)
    w = front_weights(d, seed=90 + T, gammas=True, q8_0=True)
    front = QsaFront(d, **w)
    assert front.n_embd == 2560
    g = torch.Generator(device="cuda").manual_seed(91)
    x = torch.randn(T, front.n_embd, generator=g, device="cuda")
    pos_list = [int(p) for p in torch.randint(0, 163840, (T,), generator=torch.Generator().manual_seed(T))]
    pos = torch.tensor(pos_list, dtype=torch.int32, device="cuda")
    q, gate, q_idx, k, v, kidx = front.project(x, pos)
    torch.cuda.synchronize()
    hw = {kk: t.cpu().numpy() for kk, t in w.items()}
    ref = oracle.front(d, hw, np.array(pos_list, np.int32), x.cpu().numpy(), w_type=TYPE_Q8_0)
    gemm = T > 16
    tol, ntol = (Q8_GEMM_TOL, Q8_GEMM_NORMED_TOL) if gemm else (Q8_GEMV_TOL, NORMED_TOL)
    hd = d.head_dim
    wq_gate = w["wq"].view(d.n_head, 2, hd, -1)[:, 1].reshape(d.n_head * hd, -1)
    for name, got, wt in (("gate", gate, wq_gate), ("v", v, w["wv"]), ("kidx", kidx, w["wk_idx"])):
        bound = tol * q8_abs_row_sums(wt, x).cpu().numpy()
        err = np.abs(got.cpu().numpy() - ref[name])
        assert np.all(err <= bound + 1e-30), (name, float(err.max()), float(bound.max()))
    for name, got in (("q", q), ("k", k), ("q_idx", q_idx)):
        e = np.abs(got.cpu().numpy() - ref[name]).max() / np.abs(ref[name]).max()
        assert e <= ntol, (name, e)


@pytest.mark.parametrize("T", [1, 3, 24])
def test_output_q8_0_weights_match_oracle(T):
    from qwfnfer_b200.configs import q8_0_rows
    d = make_desc()
    g = torch.Generator(device="cuda").manual_seed(95 + T)
    n_in = d.n_head * d.head_dim
    wo = q8_0_rows(torch.randn(2560, n_in, generator=g, device="cuda") * 0.02)
    attn = torch.randn(T, d.n_head, d.head_dim, generator=g, device="cuda")
    gate = 2 * torch.randn(T, n_in, generator=g, device="cuda")
    y = QsaOutput(d, wo).project(attn, gate)
    torch.cuda.synchronize()
    ref = oracle.output(d, wo.cpu().numpy(), attn.cpu().numpy(), gate.cpu().numpy(), w_type=TYPE_Q8_0)
    z = attn.reshape(T, -1) * torch.sigmoid(gate)
    tol = Q8_GEMM_TOL if T > 16 else Q8_GEMV_TOL
    # the device and host expf may round one gated value apart, which can move its q8_0 value one step
    # (or its block's scale): one step of the largest quantised term per row on top of the bound
    from qwfnfer_b200.configs import q8_0_rows_dequant
    wd = q8_0_rows_dequant(wo).abs()
    step = (z.abs().amax(dim=1, keepdim=True) / 127.0) @ wd.amax(dim=1, keepdim=True).T
    bound = tol * q8_abs_row_sums(wo, z).cpu().numpy() + 2.0 * step.cpu().numpy()
    err = np.abs(y.cpu().numpy() - ref)
    assert np.all(err <= bound), float((err / bound).max())
