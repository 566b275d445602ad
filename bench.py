#!/usr/bin/env python
"""Benchmark of the quantized decode hot path.

Workload: the full 24-layer LFM2.5-8B-A1B-shaped model (random init, INT4
G=128 weights, fp16 tied lm_head; the real checkpoint is absent), batch 1,
greedy decode at context 4096: a 64-token random prompt is fed, the model
decodes until position 4096, then W warm-up and K timed steps follow.  One
step = one token through all layers + lm_head + argmax.

  python bench.py [--gpus N] [--steps K] [--warmup W]
                  [--impl ours|reference|reference-engine]

Under torchrun each rank decodes its own independent sequence on its GPU
(bs1 decode does not shard: replicas, weak scaling); value = total tokens/s
over the max per-rank time.  The same line carries config 5 (batched,
expert-parallel decode over the ranks), 5b (prefill), 1-3 (kernel
measurements) and a compact `summary` as its last key.

--impl reference: the reference has no CPU implementation of this path (all
of src/engine.cu's math is CUDA), so its arm is the CPU restatement of the
same decode step (oracle.c built as the fp32 baseline, -O3, all host threads)
at context 4096 on weights synthesized without this library; rank 0 only.
Its line also reports the reference's own CUDA engine (src/engine.cu rebuilt
unmodified for sm_100a) on the same GPU as `reference_engine_gpu`.
--impl reference-engine: only that GPU engine run.
"""
import argparse
import json
import os
import re
import shutil
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (bs1, context 4096)"
PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM = 6650.0
REF_BUDGET_S = 150.0  # the CPU reference arm's timed steps stop after about this long
FALLBACK_TFLOPS, FALLBACK_TFLOPS_SUSTAINED = 1590.0, 1400.0
PUBLISHED = {"value": 97.3, "unit": "tok/s", "hardware": "RTX 3060 (sm_86)",
             "source": "kb/03_status.md:21-24 (decode at 1.9k context)"}


def hbm_peak():
    try:
        p = json.load(open(PEAKS))
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM, "fallback"


def tensor_peak(sustained):
    """Dense bf16 TFLOP/s: the burst figure for a kernel timed alone, the
    sustained one (power cap) for work timed over a long run."""
    try:
        p = json.load(open(PEAKS))
        return float(p["bf16_tflops_sustained" if sustained else "bf16_tflops"]), "measured"
    except Exception:
        return (FALLBACK_TFLOPS_SUSTAINED if sustained else FALLBACK_TFLOPS), "fallback"


def linear_macs_per_token(cfg):
    """Multiply-adds of one token's linear layers (projections, router and
    the top-k experts' FFN; not attention's QK/PV or the lm_head)."""
    H, hd = cfg.hidden, cfg.head_dim
    macs = 0
    for L in range(cfg.n_layers):
        if cfg.attn_layer[L]:
            macs += (cfg.n_heads + 2 * cfg.n_kv_heads) * hd * H + H * cfg.n_heads * hd
        else:
            macs += 3 * H * H + H * H
        if L < cfg.n_dense:
            macs += 3 * cfg.dense_inter * H
        else:
            macs += cfg.n_experts * H + cfg.top_k * 3 * cfg.moe_inter * H
    return macs


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.Q,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            time.sleep(0.25)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([x.strip() for x in line.split(",")])

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(2)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if len(r) > 8 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 8 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            if len(r) > 8:
                for n, v in zip(names, r[5:9]):
                    if v.strip().lower() == "active":
                        reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(self.rows)}


def step_bytes(cfg, ctx):
    """Algorithmic bytes of one decode step at context ctx (weights read once,
    KV cache of the attention layers, activations): the roofline numerator."""
    from cuda_inf_b200 import weights as W
    H = cfg.hidden
    q4 = lambda n, k: n * k // 2 + n * (k // 128) * 2
    b = 0
    for L in range(cfg.n_layers):
        b += 2 * H * 2  # norms
        if cfg.attn_layer[L]:
            b += q4((cfg.n_heads + 2 * cfg.n_kv_heads) * 64, H) + q4(H, cfg.n_heads * 64) + 256
            cm = (ctx // 64) * 64
            b += cm * cfg.n_kv_heads * 128 + (cm // 64) * cfg.n_kv_heads * 4
            b += (ctx - cm) * cfg.n_kv_heads * 256
        else:
            b += q4(3 * H, H) + q4(H, H) + H * 3 * 2 + 2 * H * 2
        if L < cfg.n_dense:
            b += 3 * q4(cfg.dense_inter, H)
        else:
            b += cfg.n_experts * H * 2 + cfg.n_experts * 2
            b += cfg.top_k * (2 * q4(cfg.moe_inter, H) + q4(H, cfg.moe_inter))
    b += cfg.vocab * H * 2 + H * 2 + H * 2  # lm_head, final norm, embedding row
    return b


def dist_setup(ngpus):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        torch.distributed.barrier()


def max_over_ranks(x, ws):
    if ws == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def prompt_ids(seed, n, vocab, rank=0):
    return np.random.default_rng(seed + 7919 * rank).integers(0, vocab, n).tolist()


def gemv_config1(copies=24, graphs=10):
    """Config 1: y[7168] = W[7168x2048] . x[2048] through cuinf_gemv_int4, one
    launch per call, rotating `copies` distinct weight copies (24 x 7.57 MB >
    the 126 MB L2, so every call streams its weights from HBM).  The launches
    are captured once in a CUDA graph and replayed; CUDA events on the stream.
    Algorithmic bytes per call: 7,340,032 packed + 229,376 scales + 4,096 x +
    28,672 y = 7,602,176."""
    from cuda_inf_b200 import ops
    N, K = 7168, 2048
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    packed = [torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=g)
              for _ in range(copies)]
    scales = [torch.exp(torch.empty(N, K // 128, device="cuda").uniform_(np.log(0.005), np.log(0.05),
                                                                          generator=g)).half()
              for _ in range(copies)]
    x = torch.randn(K, device="cuda", generator=g).half()
    y = torch.empty(N, dtype=torch.float32, device="cuda")
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for i in range(copies):  # warm-up (also loads the kernel)
            ops.gemv_int4(x, packed[i], scales[i], y)
        st.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            for i in range(copies):
                ops.gemv_int4(x, packed[i], scales[i], y)
        graph.replay()
        st.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(graphs):
            graph.replay()
        e1.record(st)
        st.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (graphs * copies)
    bpc = N * K // 2 + N * (K // 128) * 2 + K * 2 + N * 4
    peak, kind = hbm_peak()
    gbps = bpc / (us * 1e-6) / 1e9
    del graph
    return {"kernel": "k_gemv_int4", "shape": "7168x2048 INT4 G=128, batch 1", "us_per_call": round(us, 3),
            "bytes_per_call": bpc, "achieved": round(gbps, 1), "peak": peak, "unit": "GB/s",
            "frac": round(gbps / peak, 4), "peak_source": kind, "weight_copies": copies,
            "calls_timed": graphs * copies}


def gemm_tc_batch(M=64, copies=24, graphs=10):
    """The tensor-core INT4 GEMM (cuinf_gemm_int4_tc, tcgen05) on the config-1
    weight shape at M activation rows (a config-5 batch): rotating `copies`
    weight copies (> L2), launches captured in a CUDA graph.  Algorithmic
    bytes per call: packed + scales + x (M x 2048 fp16) + y (M x 7168 fp32)."""
    from cuda_inf_b200 import ops
    N, K = 7168, 2048
    g = torch.Generator(device="cuda")
    g.manual_seed(13)
    packed = [torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=g)
              for _ in range(copies)]
    scales = [torch.exp(torch.empty(N, K // 128, device="cuda").uniform_(np.log(0.005), np.log(0.05),
                                                                          generator=g)).half()
              for _ in range(copies)]
    x = torch.randn(M, K, device="cuda", generator=g).half()
    y = torch.empty(M, N, dtype=torch.float32, device="cuda")
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        for i in range(copies):  # warm-up: kernel load, split-K workspace
            ops.gemm_int4_tc(x, packed[i], scales[i], y)
        st.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            for i in range(copies):
                ops.gemm_int4_tc(x, packed[i], scales[i], y)
        graph.replay()
        st.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(graphs):
            graph.replay()
        e1.record(st)
        st.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (graphs * copies)
    bpc = N * K // 2 + N * (K // 128) * 2 + M * K * 2 + M * N * 4
    flops = 2 * M * N * K
    peak, kind = hbm_peak()
    tpeak, tkind = tensor_peak(sustained=False)
    gbps = bpc / (us * 1e-6) / 1e9
    tflops = flops / (us * 1e-6) / 1e12
    del graph
    return {"kernel": "k_tc_gemm", "shape": f"7168x2048 INT4 G=128, {M} activation rows", "us_per_call": round(us, 3),
            "bytes_per_call": bpc, "achieved": round(gbps, 1), "peak": peak, "unit": "GB/s",
            "frac": round(gbps / peak, 4), "peak_source": kind, "tflops": round(tflops, 2),
            "tensor_peak_tflops": tpeak, "tensor_frac": round(tflops / tpeak, 4), "tensor_peak_source": tkind,
            "weight_copies": copies, "calls_timed": graphs * copies}


def _graph_time(fn, n_inner, graphs=10):
    """Capture fn() (n_inner launches) in a CUDA graph after a warm-up call,
    replay it `graphs` times; returns us per inner launch (CUDA events)."""
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        fn()
        st.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=st):
            fn()
        graph.replay()
        st.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(graphs):
            graph.replay()
        e1.record(st)
        st.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (graphs * n_inner)
    del graph
    return us


def moe_config2(layers=8):
    """Config 2: one MoE FFN decode layer, batch 1 (cuinf_moe_ffn: router,
    sigmoid + bias top-4, norm_topk_prob, 4 x SwiGLU experts, weighted sum and
    residual), over `layers` distinct layers of 32 random INT4 experts (the
    selected experts' weights, 8 x 22.7 MB, exceed L2).  Algorithmic bytes
    per call: 4 experts x 5,677,056 + gate 131,072 + bias 64 + x 4,096 +
    h read/write 8,192."""
    from cuda_inf_b200 import ops
    H, I, E, K = 2048, 1792, 32, 4
    g = torch.Generator(device="cuda")
    g.manual_seed(21)

    def q4(n, k):
        p = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, device="cuda", generator=g)
        sc = torch.exp(torch.empty(n, k // 128, device="cuda").uniform_(np.log(0.005), np.log(0.05),
                                                                        generator=g)).half()
        return p, sc
    keep, tables, gates, biases = [], [], [], []
    for _ in range(layers):
        experts = [q4(I, H) + q4(I, H) + q4(H, I) for _ in range(E)]
        keep.append(experts)
        tables.append(ops.expert_table([(a, b, c, d, e, f) for a, b, c, d, e, f in experts]))
        gates.append((0.02 * torch.randn(E, H, device="cuda", generator=g)).half())
        biases.append((0.1 * torch.randn(E, device="cuda", generator=g)).half())
    xs = [torch.randn(H, device="cuda", generator=g).half() for _ in range(layers)]
    h = torch.zeros(H, device="cuda").half()

    def run():
        for i in range(layers):
            ops.moe_ffn(xs[i], gates[i], biases[i], tables[i], h, K, I)
    us = _graph_time(run, layers)
    bpc = 4 * 5_677_056 + 131_072 + 64 + 4_096 + 8_192
    peak, kind = hbm_peak()
    gbps = bpc / (us * 1e-6) / 1e9
    return {"kernels": "k_moe_fused (cuinf_moe_ffn)", "shape": "H 2048, 32 experts, I 1792, top-4, batch 1",
            "us_per_layer": round(us, 3), "bytes_per_layer": bpc, "achieved": round(gbps, 1), "peak": peak,
            "unit": "GB/s", "frac": round(gbps / peak, 4), "peak_source": kind, "layers_rotated": layers}


def attn_config3(ctxs=(2048, 8192, 32768)):
    """Config 3: FP8 E4M3 KV flash-decoding attention for one GQA layer (32 q /
    8 kv heads, head_dim 64) at each context, over enough distinct caches to
    exceed L2; tail = ctx mod 64 (0 here).  QK-norm and RoPE of the query run
    in the engine's q/k/v kernel, not here.  Algorithmic bytes per call:
    1024*C + (C/64)*32 + 2048*(ctx - C) + q/out 8,192."""
    from cuda_inf_b200 import ops
    nh, nkv = 32, 8
    out = {}
    peak, kind = hbm_peak()
    for ctx in ctxs:
        C = (ctx // 64) * 64
        per = 1024 * C + (C // 64) * 32 + 2048 * (ctx - C) + 8192
        copies = max(2, int(np.ceil(160e6 / per)))
        g = torch.Generator(device="cuda")
        g.manual_seed(ctx)
        caches = []
        for _ in range(copies):
            kc = (torch.randint(0, 256, (ctx, nkv, 64), dtype=torch.uint8, device="cuda", generator=g) & 0x77)
            vc = (torch.randint(0, 256, (ctx, nkv, 64), dtype=torch.uint8, device="cuda", generator=g) & 0x77)
            ks = torch.full((C // 64 + 1, nkv), 1.0 / 64, dtype=torch.float16, device="cuda")
            vs = torch.full((C // 64 + 1, nkv), 1.0 / 64, dtype=torch.float16, device="cuda")
            kt = torch.randn(64, nkv, 64, device="cuda", generator=g).half()
            vt = torch.randn(64, nkv, 64, device="cuda", generator=g).half()
            caches.append((kc, vc, ks, vs, kt, vt))
        q = torch.randn(nh, 64, device="cuda", generator=g).half()
        o = torch.empty_like(q)

        def run():
            for kc, vc, ks, vs, kt, vt in caches:
                ops.attn_decode(q, kc, vc, ks, vs, kt, vt, C, ctx - 1, 0.125, o)
        us = _graph_time(run, copies)
        gbps = per / (us * 1e-6) / 1e9
        out[str(ctx)] = {"us_per_call": round(us, 3), "bytes_per_call": per, "achieved": round(gbps, 1),
                         "frac": round(gbps / peak, 4), "caches_rotated": copies}
        del caches
        torch.cuda.empty_cache()
    return {"kernel": "k_attn_decode", "shape": "32 q / 8 kv heads, hd 64, FP8 groups of 64 + fp16 tail",
            "peak": peak, "unit": "GB/s", "peak_source": kind, "by_context": out}


def _baseline_oracle():
    """pyoracle bound to the timed CPU baseline build of oracle.c (fp32
    accumulation, -O3, this host's ISA)."""
    import oracle
    from oracle import pyoracle as orc
    orc.use_library(oracle.baseline_library())
    return orc


def _time_cpu_steps(orc, om, snap, threads, warm, max_steps, budget_s, seed):
    """Decode steps of the CPU baseline from a state snapshot: `warm` untimed,
    then up to max_steps timed ones, stopped once budget_s is spent.
    Returns (steps, seconds)."""
    orc.set_threads(threads)
    st = om.state(4096 + 64 + warm + max_steps)
    st.load_state(snap)
    toks = np.random.default_rng(seed).integers(0, om.cfg.vocab, warm + max_steps)
    for i in range(warm):
        st.forward(int(toks[i]), want_logits=False)
    t0 = time.perf_counter()
    n = 0
    while n < max_steps:
        st.forward(int(toks[warm + n]), want_logits=False)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    return n, time.perf_counter() - t0


def cpu_baseline(cfg, host_blob, idx, ctx, budget_s=20.0):
    """The CPU baseline (oracle.c restatement of the decode step, fp32, -O3,
    OpenMP over output rows and heads) on this host, from a state snapshot at
    context ctx - 6: single-threaded and on all host threads, each over a
    bounded sample of the same workload."""
    from cuda_inf_b200 import weights as W
    from oracle.snapshot import random_snapshot
    orc = _baseline_oracle()
    om = orc.Model(W.config_dict(cfg), host_blob, idx)
    snap = random_snapshot(cfg, ctx - 6, seed=ctx)
    threads = len(os.sched_getaffinity(0))
    n1, t1 = _time_cpu_steps(orc, om, snap, 1, 1, 64, budget_s * 0.4, 3)
    nN, tN = _time_cpu_steps(orc, om, snap, threads, 1, 256, budget_s * 0.6, 4)
    return {"value": round(nN / tN, 3), "unit": "tok/s", "cores": threads, "kind": "port",
            "single_thread": {"value": round(n1 / t1, 3), "unit": "tok/s", "cores": 1, "steps": n1,
                              "seconds": round(t1, 2)},
            "sample": f"{nN} decode steps from position {ctx - 5} on {threads} threads ({tN:.1f} s) and {n1} "
                      f"on 1 thread ({t1:.1f} s): oracle.c built as the fp32 baseline (-O3, native ISA, "
                      f"OpenMP), from a random KV/conv state snapshot at position {ctx - 6}"}


def run_ours(a, ws, rank):
    from cuda_inf_b200 import weights as W
    from cuda_inf_b200.engine import Model, Session
    if a.profile_small:
        # every stage kind on ~1.3 GB of weights: for ncu captures, which must
        # stay a few GB on the device; its numbers are not bench values
        cfg = W.make_config(n_layers=6, n_dense=1, vocab=32000, attn_layers=(2, 5))
    else:
        cfg = W.default_config()
    t0 = time.time()
    blob, idx = W.synth_device_blob(cfg, seed=a.seed)
    t_synth = time.time() - t0
    model = Model.from_device_blob(blob, idx, cfg)
    stream = torch.cuda.Stream()
    max_ctx = a.ctx + a.warmup + 2 * a.steps + 8
    sess = Session(model, max_ctx=max_ctx, stream=stream)
    kps = sess.kernels_per_step
    prompt = prompt_ids(a.seed, a.prompt_len, cfg.vocab, rank)
    with torch.cuda.stream(stream):
        for t in prompt:
            sess.step(t, want=False)
        while sess.pos < a.ctx:
            sess.step(-1, want=False)
        for _ in range(a.warmup):
            sess.step(-1, want=False)
    stream.synchronize()
    ctx0 = sess.pos
    # ---- device-timed: K steps back to back, token fed back on the device ----
    barrier(ws)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        ev0.record(stream)
        for _ in range(a.steps):
            sess.step(-1, want=False)
        ev1.record(stream)
        stream.synchronize()
    torch.cuda.synchronize()
    barrier(ws)
    ms = ev0.elapsed_time(ev1)
    ms_max = max_over_ranks(ms, ws)
    value = a.steps * ws / (ms_max / 1e3)
    # ---- end to end: public API per step, H2D token in + D2H argmax out ----
    tok = sess.step(-1, want=True)
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk2:
        e0.record(stream)
        for _ in range(a.steps):
            tok = sess.step(tok, want=True)
        e1.record(stream)
        stream.synchronize()
    barrier(ws)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), ws)
    e2e = a.steps * ws / (e2e_ms / 1e3)
    # ---- per-kernel roofline: one step launched kernel by kernel ----
    prof = sess.profile_step(-1)
    agg = {}
    for name, kms, kb in prof:
        d = agg.setdefault(name, [0, 0.0, 0.0])
        d[0] += 1
        d[1] += kms
        d[2] += kb
    tot = sum(v[1] for v in agg.values())
    top = max(agg.items(), key=lambda kv: kv[1][1])
    peak, peak_kind = hbm_peak()
    n_l, k_ms, k_b = top[1]
    k_ach = (k_b / n_l) / (k_ms / n_l / 1e3) / 1e9
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if os.path.exists(tpath):
        try:
            traffic = json.load(open(tpath)).get(top[0])
        except Exception:
            traffic = None
    sb = step_bytes(cfg, ctx0 + a.steps // 2)
    step_ach = sb / (ms_max / a.steps / 1e3) / 1e9 if ws == 1 else sb * ws / (ms_max / a.steps / 1e3) / 1e9 / ws
    out = {
        "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": ws,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms_max / a.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int4xfp16->fp32", "data": "synthetic (seeded random-init weights and prompt)",
        "config": {"workload": "config 4: full 24-layer decode, batch 1, context 4096",
                   "model": "LFM2.5-8B-A1B-shaped random init (INT4 G=128, fp16 tied lm_head)",
                   "global_batch": ws, "seq_len": a.ctx, "prompt_len": a.prompt_len,
                   "context_at_timing": ctx0, "parallelism": f"replicas x{ws}" if ws > 1 else "single GPU",
                   "l2": "no flush needed: each step streams 1.29 GB of weights (> 126 MB L2)"},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4},
        "roofline": {"bound": "hbm", "kernel": top[0], "achieved": round(k_ach, 1),
                     "peak": peak, "unit": "GB/s", "frac": round(k_ach / peak, 4),
                     "peak_source": peak_kind, "traffic": traffic,
                     "bytes_per_launch": int(k_b / n_l), "launches_per_step": n_l,
                     "share_of_step": round(k_ms / tot, 3)},
        "roofline_step": {"bound": "hbm", "bytes_per_step": sb, "achieved": round(step_ach, 1),
                          "peak": peak, "unit": "GB/s", "frac": round(step_ach / peak, 4),
                          "peak_source": peak_kind},
        "kernel_breakdown": {k: {"launches": v[0], "ms": round(v[1], 4),
                                 "GBps": round(v[2] / (v[1] / 1e3) / 1e9, 1) if v[1] > 0 else None}
                             for k, v in sorted(agg.items(), key=lambda kv: -kv[1][1])},
        "gpu_launches": kps * a.steps,
        "clocks": clk.summary(), "clocks_e2e": clk2.summary(),
        "published_reference": PUBLISHED,
        "setup_s": round(t_synth, 1),
    }
    if rank == 0 and ws == 1 and not a.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(cfg, blob.cpu().numpy(), idx, a.ctx, a.cpu_budget)
    sess.close()
    if a.batch > 0 and not a.profile_small:
        out["batched_ep"] = run_batched(a, ws, rank, model, cfg)
    if a.prefill_len > 0 and not a.profile_small:
        try:
            out["prefill_config5b"] = run_prefill(a, model, cfg)
        except Exception as e:  # a side measurement never takes the headline line down
            out["prefill_config5b"] = {"error": str(e)[:300]}
    model.close()
    return out


def run_prefill(a, model, cfg):
    """Config 5b: one prompt of a.prefill_len random ids through cuinf_prefill
    (the reference's batched prefill: every layer on all tokens, keys/values
    placed and FP8-committed before attention).  Projections on the
    tensor-core GEMM, experts grouped per chunk of 256 tokens.  Timed with CUDA
    events around the (synchronous) call, after one untimed run."""
    from cuda_inf_b200.engine import Session
    S = a.prefill_len
    stream = torch.cuda.Stream()
    sess = Session(model, max_ctx=S + 64, stream=stream)
    ids = prompt_ids(a.seed + 17, S, cfg.vocab)
    sess.prefill(ids)  # warm-up: kernels, scratch, tensor maps
    times = []
    for _ in range(2):
        sess.reset()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        tok = sess.prefill(ids)
        e1.record(stream)
        stream.synchronize()
        times.append(e0.elapsed_time(e1))
    sess.close()
    ms = min(times)
    flops = 2.0 * S * linear_macs_per_token(cfg)
    tflops = flops / (ms / 1e3) / 1e12
    tpeak, tkind = tensor_peak(sustained=True)
    return {"workload": f"config 5b: prefill of {S} prompt tokens, batch 1", "value": round(S / (ms / 1e3), 1),
            "unit": "tok/s", "ms": round(ms, 3), "runs": len(times), "next_token": tok,
            "linear_tflop": round(flops / 1e12, 3), "tflops": round(tflops, 2),
            "tensor_peak_tflops": tpeak, "tensor_frac": round(tflops / tpeak, 4), "tensor_peak_source": tkind,
            "data": "synthetic random prompt ids, random-init weights"}


def run_batched(a, ws, rank, model, cfg):
    """Config 5: a.batch sequences at context 2048 decoding together, split
    over the ranks with the experts sharded (E/ws per GPU) and the (token,
    slot) rows exchanged over NCCL each MoE layer; one GPU runs them all with
    every expert local.  value = all sequences' tokens / max-over-ranks time."""
    from cuda_inf_b200.engine import Batch, ep_unique_id_shared
    if a.batch % ws or cfg.n_experts % ws:
        return {"skipped": f"batch {a.batch} or {cfg.n_experts} experts not divisible by {ws} GPUs"}
    B = a.batch // ws
    ctx = 2048
    stream = torch.cuda.Stream()
    ep = (ep_unique_id_shared(), rank, ws) if ws > 1 else None
    bt = Batch(model, B, max_ctx=ctx + a.batch_warmup + 2 * a.batch_steps + 64, stream=stream, ep=ep)
    bt.fill_synthetic(ctx, seed=a.seed + rank)
    toks = prompt_ids(a.seed, B, cfg.vocab, rank)
    bt.step(toks)
    for _ in range(a.batch_warmup):
        bt.step(None, want=False)
    torch.cuda.synchronize()
    barrier(ws)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(torch.cuda.current_device()) as clk:
        ev0.record(stream)
        for _ in range(a.batch_steps):
            bt.step(None, want=False)
        ev1.record(stream)
        stream.synchronize()
    barrier(ws)
    ms = max_over_ranks(ev0.elapsed_time(ev1), ws)
    # end to end through the public API: tokens in from the host, argmaxes out
    cur = bt.step(None, want=True)
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(a.batch_steps):
        cur = bt.step(cur, want=True)
    e1.record(stream)
    stream.synchronize()
    barrier(ws)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), ws)
    # one step launched kernel by kernel (CUDA events between launches)
    agg = {}
    for name, kms in bt.profile_step():
        d = agg.setdefault(name, [0, 0.0])
        d[0] += 1
        d[1] += kms
    tot = sum(v[1] for v in agg.values())
    err = Batch.error()
    kps = bt.kernels_per_step
    exch = bt.exchange
    bt.close()  # its step graph holds NCCL calls: released before the process group
    step_flops = 2.0 * a.batch * (linear_macs_per_token(cfg) + cfg.vocab * cfg.hidden)
    tf_gpu = step_flops / (ms / a.batch_steps / 1e3) / 1e12 / ws
    tpeak, tkind = tensor_peak(sustained=True)
    return {
        "workload": f"config 5: {a.batch} sequences at context {ctx}, batched decode",
        "parallelism": f"expert-parallel x{ws} ({cfg.n_experts // ws} experts per GPU, rows exchanged by "
                       f"{'peer-memory stores over NVLink' if exch == 'peer_memory' else 'NCCL send/recv'})"
                       if ws > 1 else "single GPU, all experts local",
        "value": round(a.batch * a.batch_steps / (ms / 1e3), 1), "unit": "tok/s",
        "ms_per_step": round(ms / a.batch_steps, 4), "steps": a.batch_steps, "warmup": a.batch_warmup,
        "scaling": "strong", "sequences_per_gpu": B,
        "e2e": {"value": round(a.batch * a.batch_steps / (e2e_ms / 1e3), 1), "unit": "tok/s",
                "h2d_bytes_per_step": 4 * B, "d2h_bytes_per_step": 4 * B},
        "gpu_launches": kps * a.batch_steps, "device_errors": err,
        # all ranks' linear layers + lm_head per step over the step time (per GPU)
        "tflops_per_gpu": round(tf_gpu, 2), "tensor_peak_tflops": tpeak,
        "tensor_frac": round(tf_gpu / tpeak, 4), "tensor_peak_source": tkind,
        "kernel_breakdown_eager": {k: {"launches": v[0], "ms": round(v[1], 4), "share": round(v[1] / tot, 3)}
                                   for k, v in sorted(agg.items(), key=lambda kv: -kv[1][1])},
        "data": "synthetic FP8 caches at context 2048 (seeded), random-init weights",
        "clocks": clk.summary(),
    }


def synth_host_blob(cfg, seed):
    """The seeded random-init model of weights.synth_device_blob without this
    library: the same torch generator draws (on the GPU when there is one),
    quantized on the host by oracle.c's restatement of the exporter's
    quantizer (tools/export_weights.py:64-79), so the reference arm never
    loads libcuinf.  Returns (host uint8 blob, index bytes)."""
    import concurrent.futures as cf
    from cuda_inf_b200 import weights as W
    from oracle import pyoracle as orc
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    ents = W.layout(cfg)
    blob = np.empty(ents[-1].offset + ents[-1].nbytes, np.uint8)

    def quant(e, w):
        p, sc = orc.quant_int4_group(w)
        blob[e.offset:e.offset + e.packed] = p.reshape(-1)
        blob[e.offset + e.packed:e.offset + e.nbytes] = sc.view(np.uint8).reshape(-1)

    with cf.ThreadPoolExecutor(len(os.sched_getaffinity(0))) as ex:
        futs = []
        for e in ents:
            w = W.synth_tensor_torch(e.name, e.shape, seed, dev).cpu().numpy()
            if e.kind == W.FP16:
                blob[e.offset:e.offset + e.nbytes] = w.reshape(-1).astype(np.float16).view(np.uint8)
            else:
                futs.append(ex.submit(quant, e, w))
        for f in futs:
            f.result()
    return blob, W.index_bytes(ents)


def run_reference(a, ws, rank):
    """Reference arm: the reference has no CPU implementation of this path
    (all of src/engine.cu's math is CUDA), so it is the CPU restatement of
    the same decode step (oracle.c built as the fp32 baseline) on all host
    threads, at context 4096 (from a random KV/conv snapshot at a.ctx - 6),
    on the same seeded model synthesized without this library: W untimed
    steps, then up to K timed steps, stopped early after about REF_BUDGET_S
    seconds.  Then the reference's own CUDA engine on the same weights."""
    from cuda_inf_b200 import weights as W
    from oracle.snapshot import random_snapshot
    cfg = W.make_config()  # the default LFM2.5-8B-A1B shape (no library call)
    orc = _baseline_oracle()
    t0 = time.time()
    host, idx = synth_host_blob(cfg, a.seed)
    t_synth = time.time() - t0
    threads = len(os.sched_getaffinity(0))
    om = orc.Model(W.config_dict(cfg), host, idx)
    snap = random_snapshot(cfg, a.ctx - 6, seed=a.ctx)
    n, dt = _time_cpu_steps(orc, om, snap, threads, min(a.warmup, 3), a.steps, REF_BUDGET_S, a.seed)
    tps = n / dt
    sample = (f"{n} decode steps from position {a.ctx - 6 + min(a.warmup, 3)} after {min(a.warmup, 3)} untimed "
              f"(oracle.c fp32 baseline, -O3 native ISA, OpenMP, {threads} threads, {dt:.1f} s), from a random "
              f"KV/conv state snapshot at position {a.ctx - 6}")
    del om
    out = {
        "metric": METRIC, "value": round(tps, 3), "unit": "tok/s", "n_gpus": ws, "steps": n,
        "warmup": a.warmup, "ms_per_step": round(dt / n * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4xfp16->fp32",
        "data": "synthetic (the ours arm's seeded weights, synthesized and quantized on the host)",
        "impl": "reference",
        "config": {"workload": "config 4: full 24-layer decode, batch 1, context 4096",
                   "model": "LFM2.5-8B-A1B-shaped random init (INT4 G=128, fp16 tied lm_head)",
                   "global_batch": 1, "seq_len": a.ctx, "prompt_len": a.prompt_len,
                   "parallelism": "host cores of rank 0 (the other ranks exit without work)"},
        "cpu_baseline": {"kind": "port", "value": round(tps, 3), "unit": "tok/s", "cores": threads,
                         "sample": sample},
        "e2e": {"value": round(tps, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "setup_s": round(t_synth, 1),
    }
    if not a.no_reference_engine:
        try:
            eng = run_reference_engine(a, ws, rank, host=(host, idx))
            out["reference_engine_gpu"] = {k: eng.get(k) for k in ("value", "unit", "ms_per_step", "steps",
                                                                   "unavailable", "clocks")
                                           if k in eng}
            if "config" in eng:
                out["reference_engine_gpu"]["timed"] = eng["config"]["timed"]
        except Exception as e:  # the GPU side run never takes the CPU arm's line down
            out["reference_engine_gpu"] = {"unavailable": str(e)[:300]}
    return out


def run_reference_engine(a, ws, rank, host=None):
    """The reference's own engine (src/engine.cu, built unmodified for sm_100a
    into oracle/_ref/ref_engine) on the GPU, same weights and prompt, timed by
    its own decode-loop clock: the GPU-to-GPU comparison.  host = (blob,
    index) of run_reference's host-synthesized model, else synthesized here."""
    eng = os.path.join(ROOT, "oracle", "_ref", "ref_engine")
    if not os.path.exists(eng):
        return {"impl": "reference-engine", "unavailable": "oracle/_ref/ref_engine not built (reference tree absent at build time)"}
    from cuda_inf_b200 import weights as W
    cfg = W.make_config()
    if host is None:
        _baseline_oracle()
        host = synth_host_blob(cfg, a.seed)
    blob, idx = host
    base = "/dev/shm" if shutil.disk_usage("/dev/shm").free > 6e9 else None
    with tempfile.TemporaryDirectory(dir=base) as d:
        with open(os.path.join(d, "weights.bin"), "wb") as f:
            f.write(memoryview(blob))
        with open(os.path.join(d, "index.bin"), "wb") as f:
            f.write(idx)
        ids = np.array(prompt_ids(a.seed, a.prompt_len, cfg.vocab, rank), np.int32)
        ids.tofile(os.path.join(d, "ids.i32"))
        os.makedirs(os.path.join(d, "scratch"), exist_ok=True)
        n_new = a.ctx - a.prompt_len + a.warmup + a.steps
        cmd = [eng, "--dir", d, "--ids", os.path.join(d, "ids.i32"), "--n", str(n_new), "--no-stream"]
        with ClockSampler(torch.cuda.current_device()) as clk:
            r = subprocess.run(cmd, cwd=d, capture_output=True, text=True, timeout=900)
        m = re.search(r"generated (\d+) tokens in ([\d.]+)s \(([\d.]+) tok/s\)", r.stdout)
        if r.returncode != 0 or not m:
            return {"impl": "reference-engine", "unavailable": f"reference engine failed rc={r.returncode}: "
                    + (r.stderr or r.stdout)[-300:].replace("\n", " ")}
        n, secs, tps = int(m.group(1)), float(m.group(2)), float(m.group(3))
    return {
        "metric": METRIC, "value": tps, "unit": "tok/s", "n_gpus": 1, "steps": n,
        "warmup": 0, "ms_per_step": round(secs / n * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4xfp16->fp32",
        "data": "synthetic (same seeded weights and prompt as the ours arm)",
        "impl": "reference-engine",
        "config": {"workload": "config 4: full 24-layer decode, batch 1, context 4096",
                   "model": "LFM2.5-8B-A1B-shaped random init (INT4 G=128, fp16 tied lm_head)",
                   "global_batch": 1, "seq_len": a.ctx, "prompt_len": a.prompt_len,
                   "timed": f"the reference's own decode-loop clock over {n} greedy tokens "
                            f"from position {a.prompt_len} (engine.cu:942-969)"},
        "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": None, "clocks": clk.summary(),
    }


PHASES = {  # kernel id (csrc/common.cuh PH_*) -> (name, {slot: phase reached})
    0: ("k_attn_qkv", {0: "start", 1: "dependency wait done", 2: "norm done", 4: "dot done",
                       5: "head gathered (rank 0)", 9: "end (rank 0 of k/v heads)"}),
    1: ("k_gemv_residual", {0: "start", 1: "dependency wait done", 2: "x staged", 4: "dot done", 9: "end"}),
    2: ("k_conv_in", {0: "start", 1: "dependency wait done", 2: "norm done", 4: "dot done", 9: "end"}),
    3: ("k_ffn_up", {0: "start", 1: "dependency wait done", 2: "norm done", 4: "dot done", 9: "end"}),
    4: ("k_moe_fused", {0: "start", 1: "dependency wait done", 2: "norm done", 3: "logits exchanged",
                        10: "sigmoids done (warp 0)", 4: "experts selected", 5: "expert weights requested", 6: "w1/w3 dot done",
                        7: "SwiGLU values gathered (cluster)", 8: "w2 partial added, ticket taken",
                        9: "eighth finalized (last cluster)"}),
    5: ("k_moe_down", {0: "start", 1: "dependency wait done", 2: "mid staged", 4: "cluster sum done",
                       9: "end"}),
    6: ("k_lmhead", {0: "start", 1: "dependency wait done", 2: "norm done", 3: "rows done",
                     9: "token published (last CTA)"}),
    7: ("k_attn_decode", {0: "start", 1: "dependency wait done", 2: "keys done (warp 0)",
                          3: "splits merged (cluster) / combining CTA elected (global)",
                          4: "cluster released / combine done (global)"}),
}


def phase_trace(a):
    """Diagnostic: run the decode step built with phase timestamps
    (libcuinf_trace.so, `python -m cuda_inf_b200.build --trace`) to context
    a.ctx and report, for the latest launch of each kernel, when its CTAs
    reached each phase (microseconds after the earliest kernel start of the
    last step's traced launches; min / median / max over CTAs)."""
    import ctypes
    import cuda_inf_b200._lib as L
    L.LIB_PATH = os.path.join(ROOT, "cuda_inf_b200", "libcuinf_trace.so")
    from cuda_inf_b200 import weights as W
    from cuda_inf_b200.engine import Model, Session
    cfg = W.default_config()
    blob, idx = W.synth_device_blob(cfg, seed=a.seed)
    model = Model.from_device_blob(blob, idx, cfg)
    stream = torch.cuda.Stream()
    sess = Session(model, max_ctx=a.ctx + a.warmup + 16, stream=stream)
    with torch.cuda.stream(stream):
        for t in prompt_ids(a.seed, a.prompt_len, cfg.vocab, 0):
            sess.step(t, want=False)
        while sess.pos < a.ctx + a.warmup:
            sess.step(-1, want=False)
    stream.synchronize()
    buf = np.zeros((8, 1024, 12), dtype=np.uint64)
    rc = L.lib().cuinf_phase_trace_read(buf.ctypes.data_as(ctypes.c_void_p), ctypes.c_size_t(buf.nbytes))
    if rc != 0:
        raise RuntimeError(f"cuinf_phase_trace_read failed ({rc})")
    t = buf.astype(np.int64)
    starts = [t[k][t[k][:, 0] > 0, 0] for k in range(8)]
    t0 = min(int(x.min()) for x in starts if len(x))
    out = {}
    for k, (name, slots) in PHASES.items():
        live = t[k][:, 0] > 0
        if not live.any():
            continue
        rows = t[k][live]
        ent = {"ctas": int(live.sum()), "sms": int(len(np.unique(rows[:, 11]))), "phases": {}}
        for sl, what in slots.items():
            # a mark older than its CTA's start is from an earlier launch (the
            # CTA did not reach that phase this time): dropped
            col = rows[:, sl]
            col = col[col >= rows[:, 0]] - t0
            if len(col):
                ent["phases"][f"{sl} {what}"] = [round(float(col.min()) / 1e3, 2),
                                                  round(float(np.median(col)) / 1e3, 2),
                                                  round(float(col.max()) / 1e3, 2)]
        out[name] = ent
    return {"profiling_only": True, "phase_trace_us_min_med_max": out,
            "context": int(sess.pos), "note": "latest launch of each kernel in the last step"}


def summary(out):
    """The headline figures of every configuration in one short object, put
    last on the line (a record that keeps only the line's tail still shows
    them)."""
    def g(*path):
        d = out
        for k in path:
            if not isinstance(d, dict) or k not in d:
                return None
            d = d[k]
        return d
    return {
        "bs1_tok_s": g("value"), "bs1_e2e_tok_s": g("e2e", "value"), "bs1_ms_per_step": g("ms_per_step"),
        "bs1_step_frac": g("roofline_step", "frac"), "top_kernel": g("roofline", "kernel"),
        "top_kernel_frac": g("roofline", "frac"),
        "batched_tok_s": g("batched_ep", "value"), "batched_e2e_tok_s": g("batched_ep", "e2e", "value"),
        "batched_ms_per_step": g("batched_ep", "ms_per_step"), "batched_parallelism": g("batched_ep", "parallelism"),
        "batched_clocks_mhz": g("batched_ep", "clocks", "sm_mhz"),
        "prefill_tok_s": g("prefill_config5b", "value"), "prefill_tensor_frac": g("prefill_config5b", "tensor_frac"),
        "gemv_int4_frac": g("gemv_int4_config1", "frac"), "tc_gemm_frac": g("gemm_int4_tc_batch64", "frac"),
        "moe_ffn_frac": g("moe_ffn_config2", "frac"),
        "attn_frac_2k_8k_32k": [g("attention_config3", "by_context", c, "frac") for c in ("2048", "8192", "32768")],
        "cpu_baseline_tok_s": g("cpu_baseline", "value"),
        "cpu_baseline_1thread_tok_s": g("cpu_baseline", "single_thread", "value"),
        "clocks_mhz": g("clocks", "sm_mhz"), "clock_reasons": g("clocks", "reasons"),
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-engine"],
                    help="reference: the CPU restatement on the host cores (the reference has no CPU "
                         "path); reference-engine: the reference's own CUDA engine on the GPU")
    ap.add_argument("--ctx", type=int, default=4096)
    ap.add_argument("--prompt-len", type=int, default=64)
    ap.add_argument("--seed", type=int, default=1234)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--no-reference-engine", action="store_true",
                    help="reference arm: skip the reference's CUDA engine run")
    ap.add_argument("--gemv-only", action="store_true",
                    help="only the config-1 INT4 GEMV measurement (for profiler captures)")
    ap.add_argument("--kernels-only", action="store_true",
                    help="only the config-2 MoE layer and config-3 attention measurements")
    ap.add_argument("--tc-gemm-only", action="store_true",
                    help="only the tensor-core INT4 GEMM at 64 rows (for profiler captures)")
    ap.add_argument("--batch", type=int, default=64,
                    help="config 5 batched decode: total sequences (0 = skip)")
    ap.add_argument("--batch-steps", type=int, default=20)
    ap.add_argument("--prefill-len", type=int, default=4096,
                    help="config 5b prefill length (0 = skip)")
    ap.add_argument("--batch-warmup", type=int, default=3)
    ap.add_argument("--phase-trace", action="store_true",
                    help="diagnostic: per-phase timestamps of the decode kernels (needs build --trace)")
    ap.add_argument("--prefill-only", action="store_true",
                    help="only the config-5b prefill of --prefill-len tokens (with --profile-small: on the 6-layer "
                         "model, for profiler captures)")
    ap.add_argument("--batch-only", action="store_true",
                    help="only the config-5 batched decode (with --profile-small: on the 6-layer model, for "
                         "profiler captures)")
    ap.add_argument("--profile-small", action="store_true",
                    help="6-layer, 32k-vocab model of the same shapes, for profiler captures only")
    a = ap.parse_args()
    a.warmup = max(a.warmup, 3)
    ws, rank, local = dist_setup(a.gpus)
    if a.impl in ("reference", "reference-engine"):
        if rank == 0:
            fn = run_reference if a.impl == "reference" else run_reference_engine
            print(json.dumps(fn(a, ws, rank)), flush=True)
        if ws > 1:
            torch.distributed.destroy_process_group()
        return
    if a.phase_trace:
        if rank == 0:
            print(json.dumps(phase_trace(a)), flush=True)
        if ws > 1:
            torch.distributed.destroy_process_group()
        return
    if a.gemv_only:
        if rank == 0:
            print(json.dumps({"profiling_only": True, "gemv_int4_config1": gemv_config1()}), flush=True)
        if ws > 1:
            torch.distributed.destroy_process_group()
        return
    if a.kernels_only:
        if rank == 0:
            print(json.dumps({"profiling_only": True, "moe_ffn_config2": moe_config2(),
                              "attention_config3": attn_config3()}), flush=True)
        if ws > 1:
            torch.distributed.destroy_process_group()
        return
    if a.tc_gemm_only:
        if rank == 0:
            print(json.dumps({"profiling_only": True, "gemm_int4_tc_batch64": gemm_tc_batch()}), flush=True)
        if ws > 1:
            torch.distributed.destroy_process_group()
        return
    if a.prefill_only:
        from cuda_inf_b200 import weights as W
        from cuda_inf_b200.engine import Model
        cfg = (W.make_config(n_layers=6, n_dense=1, vocab=32000, attn_layers=(2, 5)) if a.profile_small
               else W.default_config())
        blob, idx = W.synth_device_blob(cfg, seed=a.seed)
        res = run_prefill(a, Model.from_device_blob(blob, idx, cfg), cfg)
        if rank == 0:
            print(json.dumps({"profiling_only": a.profile_small, "prefill_config5b": res}), flush=True)
        if ws > 1:
            torch.distributed.destroy_process_group()
        return
    if a.batch_only:
        from cuda_inf_b200 import weights as W
        from cuda_inf_b200.engine import Model
        cfg = (W.make_config(n_layers=6, n_dense=1, vocab=32000, attn_layers=(2, 5)) if a.profile_small
               else W.default_config())
        blob, idx = W.synth_device_blob(cfg, seed=a.seed)
        res = run_batched(a, ws, rank, Model.from_device_blob(blob, idx, cfg), cfg)
        if rank == 0:
            print(json.dumps({"profiling_only": a.profile_small, "batched_ep": res}), flush=True)
        if ws > 1:
            torch.distributed.destroy_process_group()
        return
    if a.profile_small:
        a.no_cpu_baseline = True
    out = run_ours(a, ws, rank)
    if not a.profile_small:
        out["gemv_int4_config1"] = gemv_config1()
        out["gemm_int4_tc_batch64"] = gemm_tc_batch()
        for key, fn in (("moe_ffn_config2", moe_config2), ("attention_config3", attn_config3)):
            try:
                out[key] = fn()
            except Exception as e:  # a side measurement never takes the headline line down
                out[key] = {"error": str(e)[:300]}
    if a.profile_small:
        out = {"profiling_only": True, "ms_per_step": out["ms_per_step"],
               "kernel_breakdown": out["kernel_breakdown"]}
    else:
        out["summary"] = summary(out)
    if rank == 0:
        print(json.dumps(out), flush=True)
    if ws > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
