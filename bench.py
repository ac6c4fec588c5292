"""Benchmark of the QSA sparse-attention hot path on B200 (one JSON line on stdout, rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 2|3|5]

Default workload (benchmark config 2): decode of one token on one sparse-attention layer at
163,840-token context, q8_0 KV, 16 query / 2 KV heads, head_dim 256, one 128-dim indexer head,
top-64 of 2560 blocks of 64 cells + a 128-token window (67 blocks, 4288 cells).  A step is the
whole node: append of the token's K/V/raw key (+ the pooled key of the block it completes),
indexer scores + top-k, and split-K attention.  Metric: microseconds per layer-token (lower is
better).  Inputs are resident in HBM; L2 is flushed (256 MB write) before every timed step.
The default line also carries the other configurations as sub-objects, each with its own timing,
clocks and roofline (--headline-only skips them):
  "batched"  config 3: 64 sequences, lengths U[4096, 163840] (seed 2), one batched decode step;
             with N ranks each GPU decodes its 64/N sequences (data parallel, no collective);
  "prefill"  config 4: chunked prefill of 8192 tokens at position 155,648 (tok/s, tensor roofline);
  "sharded"  config 5: one token through 12 layers at 1,048,576 tokens, top-128, the KV sequence
             sharded over the N ranks (layer after layer, and the 12 independent layers as one batch).
  --config 3|4|5 runs one of them alone as the line.
With N > 1 GPUs (torchrun) each rank runs config 2 on its own GPU ("replicas");
value = total units / max-over-ranks time.
--impl reference times the reference's CPU algorithm (the oracle/ port, all host cores).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HBM_FALLBACK_GBS, BF16_FALLBACK_TFS = 6650.0, 1590.0
METRIC = "sparse-attn decode us/layer @160K q8_0"


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        j = json.load(open(p))
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), "measured"
    return HBM_FALLBACK_GBS, BF16_FALLBACK_TFS, "fallback"


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of the config-2 decode
# attention, from one ncu capture of this kernel (not measured by this run; the capture's command
# and figures are in profiles/attn_decode_config2.md).
ATTN_CONFIG2_NCU_TRAFFIC = 4716288


NVML_SAMPLER = r"""
import sys, time
import pynvml
pynvml.nvmlInit()
h = pynvml.nvmlDeviceGetHandleByIndex(int(sys.argv[1]))
mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
out = sys.stdout
while True:
    sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
    bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
    out.write("%.6f,%d,%d,%d\n" % (time.time(), sm, mx, bits))
    time.sleep(0.0005)
"""


class ClockSampler:
    """SM clocks and throttle reasons while running (read-only queries): a child process samples
    NVML every ~0.5 ms and stamps each sample with its wall time, so that even millisecond timed
    regions get samples inside them whatever the main process is doing; nvidia-smi at 5 ms runs
    beside it (its lines arrive buffered, so they only count towards the reasons seen in the run)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    NVML_BITS = (("hw_slowdown", 0x8), ("hw_thermal_slowdown", 0x40), ("sw_thermal_slowdown", 0x20),
                 ("sw_power_cap", 0x4))

    def __init__(self, gpu_index: str):
        self.samples, self.proc, self.gpu = [], None, gpu_index
        self.t0 = self.t1 = None
        self.nvml_proc, self.nvml_samples = None, []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "5", "-i", self.gpu], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        try:                                   # unbuffered child writing to a file: nothing is lost at stop
            self.nvml_file = tempfile.TemporaryFile(mode="w+")
            self.nvml_proc = subprocess.Popen([sys.executable, "-u", "-c", NVML_SAMPLER, str(int(self.gpu))],
                                              stdout=self.nvml_file, stderr=subprocess.DEVNULL, text=True)
            t_end = time.time() + 5.0          # the timed region starts once the child is sampling
            while time.time() < t_end and self.nvml_proc.poll() is None and os.fstat(self.nvml_file.fileno()).st_size == 0:
                time.sleep(0.01)
        except (OSError, ValueError):
            self.nvml_proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), [x.strip() for x in line.split(",")]))

    def mark(self, which):
        setattr(self, which, time.time())

    def stop(self):
        if self.nvml_proc:
            self.nvml_proc.terminate()
            try:
                self.nvml_proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.nvml_proc.kill()
                self.nvml_proc.wait()
            self.nvml_file.seek(0)
            out = self.nvml_file.read()
            self.nvml_file.close()
            for line in out.splitlines():
                try:
                    t, sm, mx, bits = line.split(",")
                    self.nvml_samples.append((float(t), int(sm), int(mx), int(bits)))
                except ValueError:
                    continue
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        marked = self.t0 is not None and self.t1 is not None
        nv_inside = [x for x in self.nvml_samples if marked and self.t0 <= x[0] <= self.t1]
        sm, mx, reasons = [], [], set()
        nv_use = nv_inside or self.nvml_samples[-20:]
        for _, f, m, bits in nv_use:
            sm.append(float(f))
            mx.append(float(m))
            for n, bit in self.NVML_BITS:
                if bits & bit:
                    reasons.add(n)
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for _, s in self.samples:
            try:
                if not nv_use:
                    sm.append(float(s[1]))
                    mx.append(float(s[2]))
            except (ValueError, IndexError):
                continue
            for i, n in enumerate(names[1:], start=5):
                if i < len(s) and s[i].lower().startswith("active") and n != "sw_power_cap":
                    reasons.add(n)            # a slowdown seen anywhere in the run is reported
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock samples"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(nv_use) if nv_use else len(self.samples), "samples_in_timed_region": len(nv_inside),
                "sources": "NVML every 0.5 ms (child process) + nvidia-smi -lms 5"}


# ------------------------------------------------------------------------------------------------
def dist_setup(backend):
    import torch
    import torch.distributed as dist
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        from datetime import timedelta
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=timedelta(seconds=120))
    return ws, rank, local


def max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t)
    return float(t.item())


def attended_cells(sel_row, q, r):
    return sum(max(0, min(r, q - int(b) * r + 1)) for b in sel_row if b >= 0)


# ------------------------------------------------------------------------------------------------
def cpu_baseline_config2(d, kc, vc, pool, q_host, qi_host, n_past, budget_s=12.0, max_iter=200):
    """The oracle's ggml-mode node (scores, top-k, f32 online softmax with an F16 V accumulator as
    ggml-cpu's flash attention) on all host cores, one query per iteration, bounded to ~budget_s."""
    import numpy as np

    import oracle
    from qwfnfer_b200._abi import TYPE_BF16
    threads = len(os.sched_getaffinity(0))   # every host core this process may use (torchrun sets OMP_NUM_THREADS=1)
    oracle.set_threads(threads)
    flags = oracle.DEFAULT_FLAGS | oracle.GGML_FA | oracle.GGML_V_F16
    times = []
    t_end = time.perf_counter() + budget_s
    i = 0
    while time.perf_counter() < t_end and i < max_iter:
        s = i % q_host.shape[0]
        t0 = time.perf_counter()
        oracle.node(d, kc, vc, pool, [n_past], q_host[s:s + 1], qi_host[s:s + 1], q_type=TYPE_BF16, flags=flags)
        times.append(time.perf_counter() - t0)
        i += 1
    us = statistics.median(times) * 1e6
    return {"value": round(us, 1), "unit": "us/layer-token", "cores": threads, "kind": "port",
            "sample": f"{len(times)} single-query decodes of config 2 (scores over 2560 blocks, top-64+3, "
                      f"attention over 4288 cells x 16 heads), median, oracle ggml-mode, {threads} threads"}


def run_ours_config2(args, ws, rank, local):
    import numpy as np
    import torch

    from qwfnfer_b200._abi import TYPE_BF16, check, k_blocks, lib
    from qwfnfer_b200.configs import CONFIGS, fill_cache, token_inputs
    from qwfnfer_b200.qsa import QsaNode, QsaState, decode_items, _stream
    import ctypes

    cfg = CONFIGS[2]
    d = cfg.desc()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    n_past = cfg.n_past
    node, st = QsaNode(d, dev), QsaState(d, device=dev)
    fill_cache(node, st, 0, n_past, cfg.seed + 17 * rank)
    S = 8
    q, qi, k, v, ki = token_inputs(d, S, cfg.seed + 1000 + rank)
    items = decode_items([st.layer()], [n_past], device=dev)
    KB = k_blocks(d)
    wsb = node.workspace("decode", 1, n_past + 1)
    # static buffers for graph replay (slices of one device buffer); slot inputs are copied in
    # before each timed step
    parts = [x[:1] for x in (q, qi, k, v, ki)]
    nbytes = [x.numel() * x.element_size() for x in parts]
    offs = [sum(nbytes[:i]) for i in range(len(nbytes))]
    assert all(o % 16 == 0 for o in offs)
    dstage = torch.empty(sum(nbytes), dtype=torch.uint8, device=dev)
    sq, sqi, sk, sv, ski = (dstage[o:o + n].view(x.dtype).view(x.shape) for x, o, n in zip(parts, offs, nbytes))
    out = torch.empty(1, d.n_head, d.head_dim, device=dev)
    sel = torch.empty(1, KB, dtype=torch.int32, device=dev)
    L = lib()
    D = ctypes.byref(d)

    def load(s):
        sq.copy_(q[s:s + 1]); sqi.copy_(qi[s:s + 1]); sk.copy_(k[s:s + 1]); sv.copy_(v[s:s + 1]); ski.copy_(ki[s:s + 1])

    def step_api(stream_ptr):
        check(L.qsa_decode(D, items.data_ptr(), 1, n_past + 1, sq.data_ptr(), TYPE_BF16, sqi.data_ptr(),
                           sk.data_ptr(), sv.data_ptr(), ski.data_ptr(), out.data_ptr(), sel.data_ptr(),
                           wsb.data_ptr(), wsb.numel(), stream_ptr), "qsa_decode")

    def attend_api(stream_ptr):
        check(L.qsa_decode_attend(D, items.data_ptr(), 1, n_past + 1, sq.data_ptr(), TYPE_BF16, out.data_ptr(),
                                  wsb.data_ptr(), wsb.numel(), stream_ptr), "qsa_decode_attend")

    def select_api(stream_ptr):
        check(L.qsa_decode_select(D, items.data_ptr(), 1, n_past + 1, sqi.data_ptr(), sel.data_ptr(),
                                  wsb.data_ptr(), wsb.numel(), stream_ptr), "qsa_decode_select")

    for s in range(max(args.warmup, 3)):
        load(s % S)
        step_api(_stream(None))
    torch.cuda.synchronize()
    g_step, g_attn, g_sel = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_step):
        step_api(_stream(None))
    with torch.cuda.graph(g_attn):
        attend_api(_stream(None))
    with torch.cuda.graph(g_sel):
        select_api(_stream(None))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    K = args.steps

    def timed(graph, n):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for i in range(n):
            load(i % S)
            flush.zero_()
            ev[i][0].record()
            graph.replay()
            ev[i][1].record()
        torch.cuda.synchronize()
        return [a.elapsed_time(b) * 1e3 for a, b in ev]   # us

    launches = _launches_per_replay(g_step)
    clocks = ClockSampler(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local]
                          if "CUDA_VISIBLE_DEVICES" in os.environ else str(local))
    clocks.start()
    for _ in range(max(args.warmup, 3)):
        timed(g_step, 50)            # warm-up under load (also settles clocks)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.mark("t0")
    step_us = timed(g_step, K)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.mark("t1")
    attn_us = timed(g_attn, K)
    sel_us = timed(g_sel, K)
    # e2e through the public API: QsaDecodeStep replays, per token, the copy of the token's packed
    # pinned host row (item table with the position, q, q_idx, k, v, kidx) to the device,
    # qsa_decode and the copy of the output back to pinned host memory
    dstep = node.decode_step([st.layer()], n_past + 1)
    dstep.set_positions([n_past])
    rows = torch.zeros(S, dstep.row_bytes - dstep.input_offset, dtype=torch.uint8).pin_memory()
    for s_, row in enumerate(rows):
        o = 0
        for x in (q, qi, k, v, ki):
            b = x[s_:s_ + 1].contiguous().view(torch.uint8).reshape(-1).cpu()
            row[o:o + b.numel()].copy_(b)
            o += (b.numel() + 15) // 16 * 16
    for s_ in range(max(args.warmup, 3)):
        dstep.wait()
        dstep.load(rows[s_ % S])
        dstep.run()
    e2e = []
    for i in range(K):
        dstep.wait()                 # the previous token's output is back before its successor is written
        dstep.load(rows[i % S])
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dstep.run()
        b.record()
        e2e.append((a, b))
    torch.cuda.synchronize()
    e2e_us = [a.elapsed_time(b) * 1e3 for a, b in e2e]
    clocks.stop()
    h2d = dstep.row_bytes
    d2h = dstep.host_out.numel() * dstep.host_out.element_size()
    check(node.check(wsb), "qsa_check")          # the step graphs and the e2e step share this workspace

    total_us = max_over_ranks(sum(step_us), ws)
    e2e_total = max_over_ranks(sum(e2e_us), ws)
    units = K * ws
    value = total_us / units
    sel_h = sel.cpu().numpy()[0]
    cells = attended_cells(sel_h, n_past, d.ratio)
    attn_bytes = cells * 2 * 544 + q[:1].numel() * 2 + out.numel() * 4 + KB * 4
    attn_mean = statistics.mean(attn_us)
    hbm, _, src = peaks()
    achieved = attn_bytes / (attn_mean * 1e-6) / 1e9
    step_bytes = attn_bytes + (n_past + 1) // 64 * 256 + 2 * 544 + 256 + 64 * 256
    res = {
        "metric": METRIC, "value": round(value, 3), "unit": "us/layer-token", "n_gpus": ws, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(statistics.mean(step_us) / 1e3, 6), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "q8_0 KV, bf16 Q, f16 MMA / f32 softmax", "data": "synthetic",
        "config": {"workload": "config2: decode 1 token, 1 layer, ctx 163840, q8_0 KV, top-64 of 2560 blocks + "
                               "128-token window (67 blocks, 4288 cells), batch 1",
                   "global_batch": ws, "seq_len": n_past + 1, "parallelism": f"replicas x{ws}" if ws > 1 else "1 GPU",
                   "l2": "flushed (256 MB write) before every timed step", "cuda_graph": True},
        "roofline": {"bound": "hbm", "kernel": "attn_kernel<q8_0> (qsa_decode_attend)",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "peak_source": f"{src} hbm_gbs (burst)",
                     "traffic": ATTN_CONFIG2_NCU_TRAFFIC,
                     "traffic_source": "ncu capture of this kernel at this workload (profiles/attn_decode_config2.md), "
                                       "not measured in this run",
                     "algorithmic_bytes_per_launch": attn_bytes, "launch_us": round(attn_mean, 3)},
        "step_roofline": {"algorithmic_bytes": step_bytes,
                          "achieved_gbs": round(step_bytes / (statistics.mean(step_us) * 1e-6) / 1e9, 1)},
        "stages_us": {"step": round(statistics.mean(step_us), 3), "select": round(statistics.mean(sel_us), 3),
                      "attend": round(attn_mean, 3)},
        "e2e": {"value": round(e2e_total / units, 3), "unit": "us/layer-token", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches * K,       # libqsa kernels per replay (CUPTI count) x timed steps
        "clocks": clocks.summary(),
    }
    res["front"] = front_stage(d, dev, n_past, flush, K, cfg.seed)
    res["output"] = output_stage(d, dev, flush, K, cfg.seed)
    res["front_q8_0"] = front_stage(d, dev, n_past, flush, K, cfg.seed, q8_0=True)
    res["output_q8_0"] = output_stage(d, dev, flush, K, cfg.seed, q8_0=True)
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        kc = st.k[0][:n_past + 1].cpu().numpy()
        vc = st.v[0][:n_past + 1].cpu().numpy()
        pool = st.pool[0].cpu().numpy().view(np.uint16)
        qh = q.view(torch.int16).cpu().numpy().view(np.uint16)
        res["cpu_baseline"] = cpu_baseline_config2(d, kc, vc, pool, qh, qi.cpu().numpy(), n_past)
    return res


def _stage_time(fn, flush, n, graph):
    """Mean device time (us) of n calls of fn, each after the L2 flush: replayed from a CUDA graph
    (decode-sized calls, where launches matter) or called directly (prefill-sized ones)."""
    import torch

    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    run = fn
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        run = g.replay
    ev = []
    for _ in range(n):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        run()
        b.record()
        ev.append((a, b))
    torch.cuda.synchronize()
    return statistics.mean(a.elapsed_time(b) * 1e3 for a, b in ev)


def _stage_roofline(T, us, nbytes, flops):
    """HBM roofline for decode-sized calls (the weights dominate), tensor roofline above 16 tokens."""
    hbm, tfs, src = peaks()
    if T <= 16:
        ach = nbytes / (us * 1e-6) / 1e9
        return {"bound": "hbm", "algorithmic_bytes": nbytes, "achieved_gbs": round(ach, 1), "peak": hbm,
                "frac": round(ach / hbm, 4), "peak_source": f"{src} hbm_gbs (burst)"}
    ach = flops / (us * 1e-6) / 1e12
    return {"bound": "tensor", "flops": flops, "achieved_tflops": round(ach, 1), "peak": tfs,
            "frac": round(ach / tfs, 4), "peak_source": f"{src} bf16_tflops (burst)"}


def front_stage(d, dev, n_past, flush, K, seed, T=1, q8_0=False):
    """The projection front feeding the node (qsa_front: attn_q/k/v and the indexer projections over
    n_embd 2560, their norms and IMRoPE) for T tokens ending at n_past, L2 flushed before each call:
    the bf16 GEMV up to 16 tokens, the tcgen05 projection GEMM (norms and IMRoPE in its epilogue) above."""
    import torch

    from qwfnfer_b200.configs import front_weights
    from qwfnfer_b200.qsa import QsaFront

    w = front_weights(d, seed=seed + 50, device=dev, q8_0=q8_0)
    front = QsaFront(d, **w)
    x = torch.randn(T, front.n_embd, generator=torch.Generator(device=dev).manual_seed(seed + 51), device=dev)
    pos = torch.arange(n_past - T + 1, n_past + 1, dtype=torch.int32, device=dev)
    outs = front.project(x, pos)
    us = _stage_time(lambda: front.project(x, pos), flush, max(K, 20) if T <= 16 else max(K, 5), graph=T <= 16)
    w_bytes = sum(t.numel() * t.element_size() for t in w.values())
    rows = sum(t.shape[0] for k, t in w.items() if k.startswith("w"))
    nbytes = w_bytes + x.numel() * 4 + sum(o.numel() * 4 for o in outs)
    fmt = "q8_0" if q8_0 else "bf16"
    if T <= 16:
        path = f"front_kernel{'_q8' if q8_0 else ''} ({fmt} GEMV)"
    else:
        path = ("act_q8_f16 + q8_to_f16 (weights) + " if q8_0 else "to_bf16 + ") + \
               "rope table + proj_gemm_kernel (tcgen05, fused norm/IMRoPE epilogue)"
    return {"kernel": f"qsa_front, {T} token(s), n_embd 2560, {fmt} weights: {path}", "us": round(us, 3),
            **_stage_roofline(T, us, nbytes, 2 * T * rows * front.n_embd), "launches": 1 if T <= 16 else (8 if q8_0 else 3)}


def output_stage(d, dev, flush, K, seed, T=1, q8_0=False):
    """The output side after the node (qsa_output: attention output times sigmoid(gate), then the
    bf16 attn_output projection to n_embd 2560) for T tokens, L2 flushed before each call."""
    import torch

    from qwfnfer_b200.configs import N_EMBD, q8_0_rows
    from qwfnfer_b200.qsa import QsaOutput

    g = torch.Generator(device=dev).manual_seed(seed + 60)
    n_in = d.n_head * d.head_dim
    wf = torch.randn(N_EMBD, n_in, generator=g, device=dev) * 0.02
    wo = q8_0_rows(wf) if q8_0 else wf.to(torch.bfloat16)
    del wf
    attn = torch.randn(T, d.n_head, d.head_dim, generator=g, device=dev)
    gate = torch.randn(T, n_in, generator=g, device=dev)
    out = torch.empty(T, N_EMBD, device=dev)
    op = QsaOutput(d, wo)
    us = _stage_time(lambda: op.project(attn, gate, out=out), flush, max(K, 20) if T <= 16 else max(K, 5),
                     graph=T <= 16)
    nbytes = wo.numel() * wo.element_size() + attn.numel() * 4 + gate.numel() * 4 + out.numel() * 4
    fmt = "q8_0" if q8_0 else "bf16"
    if T <= 16:
        path = f"output_kernel{'_q8' if q8_0 else ''} ({fmt} GEMV)"
    else:
        path = ("act_q8_f16 + q8_to_f16 (weights)" if q8_0 else "gate_bf16_kernel") + " + proj_gemm_kernel (tcgen05)"
    return {"kernel": f"qsa_output, {T} token(s), 4096 -> n_embd 2560, {fmt} weights: {path}", "us": round(us, 3),
            **_stage_roofline(T, us, nbytes, 2 * T * N_EMBD * n_in), "launches": 1 if T <= 16 else (3 if q8_0 else 2)}


def _timed_replays(graph, n, before=None):
    """Device time (us) of n replays of `graph`, each after `before()` (input load + L2 flush)."""
    import torch
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
    for i in range(n):
        if before:
            before(i)
        ev[i][0].record()
        graph.replay()
        ev[i][1].record()
    torch.cuda.synchronize()
    return [a.elapsed_time(b) * 1e3 for a, b in ev]


def _launches_per_replay(graph):
    """libqsa kernels in one replay of `graph`, counted from CUPTI kernel records (torch.profiler)
    of a replay outside the timed region."""
    import torch
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        graph.replay()
        torch.cuda.synchronize()
    return sum(1 for e in prof.events() if e.device_type.name == "CUDA" and "qsa" in e.name)


def _clock_sampler(local):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    return ClockSampler(vis.split(",")[local] if vis else str(local))


def run_ours_config3(args, ws, rank, local):
    """Batched decode of 64 sequences (lengths U[4096, 163840], seed 2), one layer; with N ranks
    each GPU decodes its contiguous share of the sequences (data parallel, no collective)."""
    import ctypes

    import torch

    from qwfnfer_b200._abi import TYPE_BF16, check, k_blocks, lib
    from qwfnfer_b200.configs import CONFIGS, config3_lengths, fill_cache, token_inputs
    from qwfnfer_b200.qsa import QsaNode, QsaState, _stream, decode_items

    cfg = CONFIGS[3]
    d = cfg.desc()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    lengths = config3_lengths()
    if len(lengths) % ws:
        raise SystemExit(f"config 3: {len(lengths)} sequences do not split over {ws} ranks")
    per = len(lengths) // ws
    mine = lengths[rank * per:(rank + 1) * per]
    positions = [n - 1 for n in mine]                 # the decoded token is the sequence's last
    node = QsaNode(d, dev)
    states = []
    for j, n in enumerate(positions):
        st = QsaState(d, device=dev)
        fill_cache(node, st, 0, n, cfg.seed * 1000 + rank * per + j)
        states.append(st)
    B, KB = len(positions), k_blocks(d)
    max_n_kv = max(positions) + 1
    items = decode_items([st.layer() for st in states], positions, device=dev)
    S = 4
    ins = [token_inputs(d, B, cfg.seed + 100 * s + rank) for s in range(S)]
    sq, sqi, sk, sv, ski = (torch.empty_like(x) for x in ins[0])
    out = torch.empty(B, d.n_head, d.head_dim, device=dev)
    sel = torch.empty(B, KB, dtype=torch.int32, device=dev)
    wsb = node.workspace("decode", B, max_n_kv)
    L, D = lib(), ctypes.byref(d)

    def load(s):
        for dst, src in zip((sq, sqi, sk, sv, ski), ins[s % S]):
            dst.copy_(src)

    def step_api(stream_ptr):
        check(L.qsa_decode(D, items.data_ptr(), B, max_n_kv, sq.data_ptr(), TYPE_BF16, sqi.data_ptr(), sk.data_ptr(),
                           sv.data_ptr(), ski.data_ptr(), out.data_ptr(), sel.data_ptr(), wsb.data_ptr(), wsb.numel(),
                           stream_ptr), "qsa_decode")

    def attend_api(stream_ptr):
        check(L.qsa_decode_attend(D, items.data_ptr(), B, max_n_kv, sq.data_ptr(), TYPE_BF16, out.data_ptr(),
                                  wsb.data_ptr(), wsb.numel(), stream_ptr), "qsa_decode_attend")

    for s in range(args.warmup):
        load(s)
        step_api(_stream(None))
    torch.cuda.synchronize()
    g_step, g_attn = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_step):
        step_api(_stream(None))
    with torch.cuda.graph(g_attn):
        attend_api(_stream(None))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def before(i):
        load(i)
        flush.zero_()

    K = args.steps
    launches = _launches_per_replay(g_step)
    clocks = _clock_sampler(local)
    clocks.start()
    _timed_replays(g_step, 20, before)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.mark("t0")
    step_us = _timed_replays(g_step, K, before)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.mark("t1")
    attn_us = _timed_replays(g_attn, K, before)
    # e2e through the public QsaDecodeStep: per step, this rank's packed pinned host rows (item
    # table with the positions, q, q_idx, k, v, kidx of every sequence) staged in by a kernel,
    # qsa_decode, and the output stored by its last kernel into pinned host memory
    dstep = node.decode_step([st.layer() for st in states], max_n_kv)
    dstep.set_positions(positions)
    rows = []
    for s_ in range(S):
        for name, x in zip(("q", "q_idx", "k_new", "v_new", "kidx_new"), ins[s_]):
            dstep.host[name].copy_(x.cpu())
        rows.append(dstep.host_in[dstep.input_offset:].clone().pin_memory())
    for s_ in range(max(args.warmup, 3)):
        dstep.wait()
        dstep.load(rows[s_ % S])
        dstep.run()
    e2e = []
    for i in range(K):
        dstep.wait()
        dstep.load(rows[i % S])
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        dstep.run()
        b.record()
        e2e.append((a, b))
    torch.cuda.synchronize()
    e2e_us = [a.elapsed_time(b) * 1e3 for a, b in e2e]
    clocks.stop()
    check(node.check(wsb), "qsa_check")
    check(node.check(dstep.ws), "qsa_check (e2e step)")
    h2d = dstep.row_bytes
    d2h = dstep.host_out.numel() * dstep.host_out.element_size()
    sel_h = sel.cpu().numpy()
    cells = sum(attended_cells(sel_h[t], positions[t], d.ratio) for t in range(B))
    attn_bytes = cells * 2 * 544 + sum(x.numel() * x.element_size() for x in (sq, out)) + B * KB * 4
    attn_mean = statistics.mean(attn_us)
    hbm, _, src = peaks()
    achieved = attn_bytes / (attn_mean * 1e-6) / 1e9
    step_bytes = attn_bytes + sum((p + 1) // d.ratio for p in positions) * 256
    total_us = max_over_ranks(statistics.mean(step_us), ws)
    e2e_max = max_over_ranks(statistics.mean(e2e_us), ws)
    n_tok = B * ws
    return {
        "metric": "batched sparse-attn decode us/token, 64 seqs @4K-160K q8_0", "value": round(total_us / n_tok, 4),
        "unit": "us/token", "n_gpus": ws, "steps": K, "warmup": args.warmup, "ms_per_step": round(total_us / 1e3, 6),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "q8_0 KV, bf16 Q, f16 MMA / f32 softmax", "data": "synthetic",
        "config": {"workload": f"config3: one decode step of 64 sequences, lengths U[4096,163840] seed 2, q8_0, "
                               f"top-64 + 128-token window; {per} sequences per GPU",
                   "global_batch": len(lengths), "seq_len": max(lengths),
                   "parallelism": f"data parallel x{ws}" if ws > 1 else "1 GPU",
                   "l2": "flushed (256 MB write) before every timed step", "cuda_graph": True},
        "roofline": {"bound": "hbm", "kernel": "attn_kernel<q8_0> (qsa_decode_attend), rank 0",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "peak_source": f"{src} hbm_gbs (burst)", "traffic": None,
                     "algorithmic_bytes_per_launch": attn_bytes, "launch_us": round(attn_mean, 3)},
        "step_roofline": {"algorithmic_bytes": step_bytes,
                          "achieved_gbs": round(step_bytes / (statistics.mean(step_us) * 1e-6) / 1e9, 1)},
        "stages_us": {"step": round(statistics.mean(step_us), 3), "attend": round(attn_mean, 3)},
        "e2e": {"value": round(e2e_max / n_tok, 4), "unit": "us/token", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "gpu_launches": launches * K,       # libqsa kernels per replay (CUPTI count) x timed steps
        "clocks": clocks.summary(),
    }


def run_ours_config5(args, ws, rank, local):
    """One token through 12 sparse-attention layers at 1,048,576 tokens of context (top-128), the
    KV sequence sharded over the ranks: per layer, shard-local candidates, an all-gather, the
    global selection and local attention, an all-gather of the states, the merge."""
    import numpy as np
    import torch

    from qwfnfer_b200._abi import check, k_blocks, lib
    from qwfnfer_b200.configs import CONFIGS, fill_cache, token_inputs
    from qwfnfer_b200.qsa import QsaNode, QsaState, _stream, decode_items
    from qwfnfer_b200.shard import ShardedDecoder

    cfg = CONFIGS[5]
    L = lib()
    d = cfg.desc()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    NL, n_past = cfg.layers, cfg.n_past
    lb = args.layer_batch                      # the 12 independent layers as one batch of 12 items
    dec = ShardedDecoder(d, rank=rank, world=ws, exchange=args.exchange, batch=NL if lb else 1, index=args.index)
    node = QsaNode(d, dev)
    st = QsaState(d, n_layers=NL, device=dev, blocks=dec.blocks, index_full=dec.index_replicated)
    for il in range(NL):                       # every rank draws the same stream, keeps its cells
        fill_cache(node, st, il, n_past, cfg.seed * 1000 + il, append=dec.append)
    items = [decode_items([st.layer(il)], [n_past], device=dev) for il in range(NL)]
    items_all = decode_items([st.layer(il) for il in range(NL)], [n_past] * NL, device=dev)
    KB = k_blocks(d)
    S = 4
    ins = [token_inputs(d, NL, cfg.seed + 100 * s) for s in range(S)]     # identical on every rank
    slots = [torch.empty_like(x) for x in ins[0]]
    sel = torch.empty(NL, KB, dtype=torch.int32, device=dev)

    def load(s):
        for dst, src in zip(slots, ins[s % S]):
            dst.copy_(src)

    def step(slots=slots, out=None):
        """The 12 layers' step; `out` (f32 [NL, n_head, head_dim]) receives the outputs when given."""
        q, qi, k, v, ki = slots
        if lb:                                 # one exchange of candidates and one of states for all layers
            dec.step(items_all, NL, n_past + 1, q, qi, k, v, ki, sel_out=sel, out=out)
            return
        for il in range(NL):
            dec.step(items[il], 1, n_past + 1, q[il:il + 1], qi[il:il + 1], k[il:il + 1], v[il:il + 1],
                     ki[il:il + 1], sel_out=sel[il:il + 1], out=None if out is None else out[il:il + 1])

    # Tokens per graph replay.  The replicated-index step's state exchange alternates two peer
    # channels per step, so that a rank's push of step s+1 lands only after the peer read step s;
    # a graph fixes the channel of every step it holds, so one of a single step would reuse one
    # channel every replay.  The 12 layers after one another already alternate inside the graph;
    # the batched step is captured twice.
    reps = 2 if lb else 1
    for s in range(args.warmup):
        load(s)
        step()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, capture_error_mode="thread_local"):
        for _ in range(reps):
            step()
    # the attention stage alone (the dominant kernel), on this rank's share: layer 0, or all 12
    # layers in one launch with --layer-batch (with replicated indexer caches: selection + attention)
    a_items, a_b = (items_all, NL) if lb else (items[0], 1)
    if dec.index_replicated:
        torch.cuda.synchronize()
        g_attn = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_attn):
            dec.backend.decode_ri(a_items, a_b, n_past + 1, dec.blocks, slots[0][:a_b], slots[1][:a_b])
    else:
        cand = dec.backend.candidates(a_items, a_b, n_past + 1, dec.blocks, slots[1][:a_b])
        gathered, cstride = dec._all_gather(cand, 0)
        torch.cuda.synchronize()
        g_attn = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_attn):
            dec.backend.attend(a_items, a_b, n_past + 1, dec.blocks, gathered, slots[0][:a_b], n_shards=dec.world,
                               cand_stride=cstride)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def before(i):
        load(i)
        flush.zero_()

    K = args.steps
    launches = _launches_per_replay(g)
    clocks = _clock_sampler(local)
    clocks.start()
    _timed_replays(g, 10, before)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.mark("t0")
    step_us = _timed_replays(g, K, before)
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.mark("t1")
    attn_us = _timed_replays(g_attn, K, lambda i: flush.zero_())
    # e2e: the public ShardedDecoder.step of the 12 layers captured with its host side, as a user
    # drives it per token: qsa_stage_copy of this rank's packed pinned row (q, q_idx, k, v, kidx of
    # every layer) into one device buffer, the step, and the outputs stored by the state merge
    # straight into pinned host memory
    offs, o = [], 0
    for x in ins[0]:
        offs.append(o)
        o += (x.numel() * x.element_size() + 15) // 16 * 16
    dev_in = torch.empty(reps, o, dtype=torch.uint8, device=dev)
    host_in = torch.empty(reps, o, dtype=torch.uint8).pin_memory()
    e_slots = [[dev_in[r_, off:off + x.numel() * x.element_size()].view(x.dtype).view(x.shape)
                for x, off in zip(ins[0], offs)] for r_ in range(reps)]
    rows = []
    for t_ in ins:
        r = torch.zeros(o, dtype=torch.uint8)
        for x, off in zip(t_, offs):
            r[off:off + x.numel() * x.element_size()].copy_(x.contiguous().view(torch.uint8).reshape(-1).cpu())
        rows.append(r.pin_memory())
    hout = torch.empty(reps, NL, d.n_head, d.head_dim).pin_memory()

    def step_e2e():
        for r_ in range(reps):               # each token's row staged, its step, its outputs stored to the host
            check(L.qsa_stage_copy(dev_in[r_].data_ptr(), host_in[r_].data_ptr(), o, _stream(None)), "qsa_stage_copy")
            step(e_slots[r_], hout[r_])

    for r_ in range(reps):
        host_in[r_].copy_(rows[r_])
    step_e2e()
    torch.cuda.synchronize()
    g_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_e2e, capture_error_mode="thread_local"):
        step_e2e()
    e2e = []
    for i in range(K):
        torch.cuda.synchronize()               # the previous token's output is back before its successor is written
        for r_ in range(reps):
            host_in[r_].copy_(rows[(reps * i + r_) % S])
        flush.zero_()
        if ws > 1:
            torch.distributed.barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g_e2e.replay()
        b.record()
        e2e.append((a, b))
    torch.cuda.synchronize()
    e2e_us = [a.elapsed_time(b) * 1e3 for a, b in e2e]
    clocks.stop()
    if dec.backend.check(NL if lb else 1, n_past + 1) != 0:
        raise SystemExit("device status error")
    sel_h = sel.cpu().numpy()
    lo, hi = dec.blocks
    local_cells = sum(attended_cells([b for b in sel_h[il] if lo <= b < hi], n_past, d.ratio) for il in range(NL))
    scored = (n_past + 1) // d.ratio if dec.index_replicated else max(0, min(hi, (n_past + 1) // d.ratio) - lo)
    sf = 16 * (2 + d.head_dim) * 4
    step_bytes = local_cells * 2 * 544 + NL * (scored * 256 + 2 * 544 + 256 + (ws + 1) * sf)
    attn_layers = range(NL) if lb else range(1)
    attn_cells0 = sum(attended_cells([b for b in sel_h[il] if lo <= b < hi], n_past, d.ratio) for il in attn_layers)
    attn_bytes = attn_cells0 * 2 * 544 + len(attn_layers) * (16 * 256 * 2 + sf)
    attn_mean = statistics.mean(attn_us)
    hbm, _, src = peaks()
    achieved = attn_bytes / (attn_mean * 1e-6) / 1e9
    total_us = max_over_ranks(statistics.mean(step_us), ws) / reps
    e2e_max = max_over_ranks(statistics.mean(e2e_us), ws) / reps
    res = {
        "metric": "sparse-attn decode us/layer @1M q8_0, 12 layers, KV-sequence-sharded",
        "value": round(total_us / NL, 3), "unit": "us/layer-token", "n_gpus": ws, "steps": K,
        "warmup": args.warmup, "ms_per_step": round(total_us / 1e3, 6), "higher_is_better": False,
        "scaling": "strong", "vs_baseline": None, "dtype": "q8_0 KV, bf16 Q, f16 MMA / f32 softmax",
        "data": "synthetic",
        "config": {"workload": "config5: decode 1 token through 12 layers, ctx 1048576, q8_0, top-128 of 16384 "
                               "blocks + 128-token window (131 blocks)"
                               + (", the 12 independent layers issued as one batch (one candidate and one state "
                                  "exchange per token for all layers)" if lb else ", layer after layer"),
                   "global_batch": 1, "seq_len": n_past + 1, "layers": NL,
                   "parallelism": (f"KV-sequence-sharded x{ws} ("
                                   + {"peer": "NVLink peer memory: states stored by the attention, published by flag"
                                      if dec.index_replicated else "NVLink peer-memory all-gathers",
                                      "peer_push": "NVLink peer-memory all-gathers",
                                      "nccl": "NCCL all-gathers"}[args.exchange]
                                   + (", indexer caches replicated" if dec.index_replicated else "")
                                   + ")") if ws > 1 else "1 GPU",
                   "blocks_per_gpu": hi - lo,
                   "l2": "flushed (256 MB write) before every timed step", "cuda_graph": True,
                   "tokens_per_replay": reps},
        "roofline": {"bound": "hbm", "kernel": "attn_kernel<q8_0> (qsa_shard_attend), "
                               + ("all 12 layers in one launch" if lb else "layer 0") + ", rank 0",
                     "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                     "peak_source": f"{src} hbm_gbs (burst)", "traffic": None,
                     "algorithmic_bytes_per_launch": attn_bytes, "launch_us": round(attn_mean, 3)},
        "step_roofline": {"algorithmic_bytes_per_gpu": step_bytes,
                          "achieved_gbs": round(step_bytes / (statistics.mean(step_us) / reps * 1e-6) / 1e9, 1)},
        "e2e": {"value": round(e2e_max / NL, 3), "unit": "us/layer-token",
                "h2d_bytes_per_step": sum(x.numel() * x.element_size() for x in ins[0]),
                "d2h_bytes_per_step": NL * d.n_head * d.head_dim * 4},
        "gpu_launches": launches * K,       # libqsa kernels per replay (CUPTI count) x timed steps
        "clocks": clocks.summary(),
    }
    del g, g_attn                               # graphs holding NCCL work go before the process group
    if dec.peer is not None:
        torch.cuda.synchronize()
        torch.distributed.barrier()
        dec.peer.close()
    return res


def run_ours_config4(args, ws, rank, local):
    """Chunked prefill (benchmark config 4): 8192 new tokens appended at position 155,648 of a
    q8_0 cache; a step is one qsa_prefill call (append of the chunk's K/V/raw keys and pooled
    keys, indexer scores of every query, per-query top-k + window, sparse attention)."""
    import ctypes

    import numpy as np
    import torch

    from qwfnfer_b200._abi import TYPE_BF16, check, k_blocks, lib
    from qwfnfer_b200.configs import CONFIGS, fill_cache, token_inputs
    from qwfnfer_b200.qsa import QsaNode, QsaState, _stream

    cfg = CONFIGS[4]
    d = cfg.desc()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    T, n_past = cfg.prefill_T, cfg.n_past
    node, st = QsaNode(d, dev), QsaState(d, device=dev)
    fill_cache(node, st, 0, n_past, cfg.seed + 17 * rank)
    q, qi, k, v, ki = token_inputs(d, T, cfg.seed + 1000 + rank)
    out = torch.empty(T, d.n_head, d.head_dim, device=dev)
    KB = k_blocks(d)
    sel = torch.empty(T, KB, dtype=torch.int32, device=dev)
    wsb = node.workspace("prefill", T, n_past + T)
    L, D = lib(), ctypes.byref(d)
    cache = st.layer()

    def step_api(stream_ptr, qq=q, qqi=qi, kk=k, vv=v, kki=ki, oo=out):
        check(L.qsa_prefill(D, ctypes.byref(cache), n_past, T, qq.data_ptr(), TYPE_BF16, qqi.data_ptr(), kk.data_ptr(),
                            vv.data_ptr(), kki.data_ptr(), oo.data_ptr(), sel.data_ptr(), wsb.data_ptr(), wsb.numel(),
                            stream_ptr), "qsa_prefill")

    for _ in range(args.warmup):
        step_api(_stream(None))
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step_api(_stream(None))
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    K = args.steps
    launches = _launches_per_replay(g)
    clocks = _clock_sampler(local)
    clocks.start()
    _timed_replays(g, 2, lambda i: flush.zero_())
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.mark("t0")
    step_us = _timed_replays(g, K, lambda i: flush.zero_())
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    clocks.mark("t1")
    # e2e: qsa_prefill with the chunk's inputs copied from pinned host memory and the output read back
    hq, hqi, hk, hv, hki = (x.cpu().pin_memory() for x in (q, qi, k, v, ki))
    hout = torch.empty_like(out, device="cpu").pin_memory()
    sq, sqi, sk, sv, ski = (torch.empty_like(x) for x in (q, qi, k, v, ki))
    e2e = []
    for i in range(min(K, 5)):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for dst, src in zip((sq, sqi, sk, sv, ski), (hq, hqi, hk, hv, hki)):
            dst.copy_(src, non_blocking=True)
        step_api(torch.cuda.current_stream().cuda_stream, sq, sqi, sk, sv, ski, out)
        hout.copy_(out, non_blocking=True)
        b.record()
        e2e.append((a, b))
    torch.cuda.synchronize()
    e2e_us = [a.elapsed_time(b) * 1e3 for a, b in e2e]
    clocks.stop()
    check(node.check(wsb), "qsa_check")
    sel_h = sel.cpu().numpy()
    cells = sum(attended_cells(sel_h[t], n_past + t, d.ratio) for t in range(0, T, 64)) * 64
    nb = (n_past + T) // d.ratio
    flops_idx = 2.0 * T * nb * d.idx_dim * d.idx_n_head
    flops_attn = 4.0 * cells * d.n_head * d.head_dim
    step_mean = statistics.mean(step_us)
    total_us = max_over_ranks(step_mean, ws)
    e2e_max = max_over_ranks(statistics.mean(e2e_us), ws)
    _, tfs, src = peaks()
    achieved = (flops_idx + flops_attn) / (step_mean * 1e-6) / 1e12
    toks = T * ws
    res = {
        "metric": "sparse-attn prefill tok/s @8192 on 155648 q8_0", "value": round(toks / (total_us * 1e-6), 1),
        "unit": "tok/s", "n_gpus": ws, "steps": K, "warmup": args.warmup, "ms_per_step": round(total_us / 1e3, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q8_0 KV, bf16 Q, f16 MMA / f32 softmax", "data": "synthetic",
        "config": {"workload": "config4: one chunk of 8192 tokens at n_past 155648 (append + indexer + top-64 + window "
                               "+ attention), q8_0", "global_batch": toks, "seq_len": n_past + T,
                   "parallelism": f"replicas x{ws}" if ws > 1 else "1 GPU",
                   "l2": "flushed (256 MB write) before every timed step; inputs exceed L2", "cuda_graph": True},
        "roofline": {"bound": "tensor", "kernel": "whole qsa_prefill step (indexer + attention FLOPs)",
                     "achieved": round(achieved, 2), "peak": tfs, "unit": "TFLOP/s", "frac": round(achieved / tfs, 4),
                     "peak_source": f"{src} bf16_tflops (burst)", "traffic": None,
                     "flops_per_step": flops_idx + flops_attn, "indexer_flops": flops_idx},
        "e2e": {"value": round(toks / (e2e_max * 1e-6), 1), "unit": "tok/s",
                "h2d_bytes_per_step": sum(x.numel() * x.element_size() for x in (q, qi, k, v, ki)),
                "d2h_bytes_per_step": out.numel() * out.element_size()},
        "gpu_launches": launches * K,       # libqsa kernels per replay (CUPTI count) x timed steps
        "clocks": clocks.summary(),
    }
    # the projections around the node for this chunk, reported beside the node's metric
    res["front"] = front_stage(d, dev, n_past + T - 1, flush, K, cfg.seed, T=T)
    res["output"] = output_stage(d, dev, flush, K, cfg.seed, T=T)
    res["front_q8_0"] = front_stage(d, dev, n_past + T - 1, flush, K, cfg.seed, T=T, q8_0=True)
    res["output_q8_0"] = output_stage(d, dev, flush, K, cfg.seed, T=T, q8_0=True)
    return res


def run_reference_config2(args):
    """The reference's CPU algorithm (oracle port, ggml mode, all host cores) on config 2."""
    import numpy as np

    import oracle
    from qwfnfer_b200._abi import TYPE_BF16
    from qwfnfer_b200.configs import CONFIGS, IDX_STD, K_SCALE
    cfg = CONFIGS[2]
    d = cfg.desc()
    n_past = cfg.n_past
    threads = len(os.sched_getaffinity(0))   # every host core this process may use (torchrun sets OMP_NUM_THREADS=1)
    oracle.set_threads(threads)
    rng = np.random.default_rng(cfg.seed)
    kc, vc, ic, pool = oracle.cache_arrays(d)
    chunk = 16384
    for pos in range(0, n_past, chunk):
        n = min(chunk, n_past - pos)
        oracle.append(d, kc, vc, ic, pos, (rng.standard_normal((n, 512), np.float32) * K_SCALE),
                      rng.standard_normal((n, 512), np.float32), rng.standard_normal((n, 128), np.float32) * IDX_STD)
    _, p16 = oracle.pool_blocks(d, ic, 0, n_past // 64)
    pool[: n_past // 64] = p16
    S = 8
    qf = rng.standard_normal((S, 16, 256), np.float32)
    qh = (qf.view(np.uint32) >> 16).astype(np.uint16)           # bf16 bits (truncated draw)
    qi = rng.standard_normal((S, 1, 128), np.float32) * IDX_STD
    kn = rng.standard_normal((S, 512), np.float32) * K_SCALE
    vn = rng.standard_normal((S, 512), np.float32)
    kin = rng.standard_normal((S, 128), np.float32) * IDX_STD
    flags = oracle.DEFAULT_FLAGS | oracle.GGML_FA | oracle.GGML_V_F16

    def step(s):
        oracle.append(d, kc, vc, ic, n_past, kn[s:s + 1], vn[s:s + 1], kin[s:s + 1])
        b = n_past // 64
        _, p = oracle.pool_blocks(d, ic, b, 1)
        pool[b] = p[0]
        oracle.node(d, kc, vc, pool, [n_past], qh[s:s + 1], qi[s:s + 1], q_type=TYPE_BF16, flags=flags)

    for i in range(args.warmup):
        step(i % S)
    times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        step(i % S)
        times.append(time.perf_counter() - t0)
    us = statistics.mean(times) * 1e6
    return {
        "impl": "reference", "metric": METRIC, "value": round(us, 1), "unit": "us/layer-token",
        "n_gpus": args.gpus,                   # the N of the launch (rank 0 runs the CPU arm alone)
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(us / 1e3, 4), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "q8_0 KV, f16-rounded K/V and Q, f32 softmax", "data": "synthetic",
        "config": {"workload": "config2: decode 1 token, 1 layer, ctx 163840, q8_0 KV, top-64 + 128-token window",
                   "global_batch": 1, "seq_len": n_past + 1, "parallelism": f"CPU, {threads} threads"},
        "cpu_baseline": {"value": round(us, 1), "unit": "us/layer-token", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} decode steps (append + pooled key + scores + top-k + ggml-mode "
                                   f"attention), oracle port of the reference node"},
        "e2e": {"value": round(us, 1), "unit": "us/layer-token", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def _sub(res):
    """A configuration's line as a sub-object of the headline line (its own timing, roofline, e2e
    and clocks; the keys the headline already states are dropped)."""
    return {k: v for k, v in res.items() if k not in ("n_gpus", "steps", "warmup", "vs_baseline", "data", "dtype")}


def run_sub_benches(args, ws, rank, local):
    """Configs 3, 4 and 5 beside the headline (every rank runs the same sequence of them)."""
    import torch
    sub = argparse.Namespace(**vars(args))
    sub.steps = max(5, min(args.steps, 20))
    out = {}
    runs = (("batched", run_ours_config3, {}), ("prefill", run_ours_config4, {}),
            ("sharded.layer_after_layer", run_ours_config5, {"layer_batch": False}),
            ("sharded.layer_batched", run_ours_config5, {"layer_batch": True}))
    for key, fn, over in runs:
        a = argparse.Namespace(**{**vars(sub), **over})
        r = _sub(fn(a, ws, rank, local))
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        if "." in key:
            k0, k1 = key.split(".")
            out.setdefault(k0, {})[k1] = r
        else:
            out[key] = r
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=2, choices=[2, 3, 4, 5])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--headline-only", action="store_true",
                    help="config 2 only, without the batched / prefill / sharded sub-objects")
    ap.add_argument("--layer-batch", action="store_true",
                    help="config 5: issue the 12 independent layers as one batch of 12 items (2 exchanges per token)")
    ap.add_argument("--index", default="replicated", choices=["sharded", "replicated"],
                    help="config 5: the indexer caches replicated on every rank (one state exchange per layer) or "
                         "sharded with the K/V (candidates exchanged too)")
    ap.add_argument("--exchange", default="peer", choices=["peer", "peer_push", "nccl"],
                    help="config 5 with N > 1: the shards' exchanges over NVLink peer memory or NCCL")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        if args.config != 2:
            print(json.dumps({"impl": "reference", "unavailable": f"the CPU reference arm times config 2 only"}))
            return
        res = run_reference_config2(args)
        print(json.dumps(res), flush=True)
        return

    ws, rank, local = dist_setup("nccl")
    if args.config == 2:
        res = run_ours_config2(args, ws, rank, local)
        if not args.headline_only:
            res.update(run_sub_benches(args, ws, rank, local))
    elif args.config == 3:
        res = run_ours_config3(args, ws, rank, local)
    elif args.config == 4:
        res = run_ours_config4(args, ws, rank, local)
    else:
        res = run_ours_config5(args, ws, rank, local)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
