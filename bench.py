"""Benchmark of the attention hot path (prologue + attention, 28 layers).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

One step = one pass of the hot path over one micro-batch: for each of the 28
layers, the fused Q/K RMSNorm + RoPE prologue and the causal/sparse GQA
attention (the two runs Qwen3ExecutionPlan encodes per layer,
src/webgpu/model.ts:94-95), each layer with its own seeded inputs.

Multi-GPU (torchrun, one process per GPU): requests are independent, so the
workload's requests are split across the ranks (LPT on kept pairs; strong
scaling), each rank runs its share as one packed micro-batch, and the e2e leg
gathers every rank's output rows into one shared host buffer in request
order. No collective is on the hot path; the barrier and the max-over-ranks
timing only frame the measurement. ``value`` = the workload's tokens / max
step time. ``--weak-scaling`` gives every rank the whole workload instead.

``--impl reference``: the reference's hot path exists only as WGSL for a
browser WebGPU (unavailable on this box), so this arm times the CPU oracle
(a C/OpenMP restatement of the same math) on the host cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

PKG = "qwen3-embedding-webgpu-prepacked_b200"
DEFAULT_WORKLOAD = "c5_16x5000_sparse"
METRIC = "prefill attention tokens/s (GQA 16/8x128, 28 layers)"
UNIT = "tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=DEFAULT_WORKLOAD)
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--weak-scaling", action="store_true",
                    help="every rank runs the whole workload (default: the workload's requests "
                         "are split across the ranks)")
    ap.add_argument("--gemm", action="store_true",
                    help="time the projection GEMM against cuBLAS and the fused QKV projection")
    ap.add_argument("--gemm-rows", type=int, default=0,
                    help="with --gemm: one M (rows) instead of the default shapes; small runs "
                         "for profiling")
    ap.add_argument("--engine", action="store_true",
                    help="time the micro-batch engine, padded vs varlen packing (one GPU)")
    ap.add_argument("--model", action="store_true",
                    help="time the whole 28-layer embedding model (FFN included) through the "
                         "engine, padded vs varlen packing (one GPU)")
    # profiling aids: shrink the workload (never used for the reported line)
    ap.add_argument("--requests", type=int, default=0, help="override request count")
    ap.add_argument("--layers", type=int, default=0, help="override layer count")
    return ap.parse_args()


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons, sampled every 50 ms from before
    the warm-up on. mark_start() / mark_end() bracket the timed region, and
    summary() uses the samples taken inside it (±50 ms), or all samples,
    flagged, if the region was too short to catch one."""
    Q = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    INTERVAL_MS = 50

    def __init__(self, index: int):
        self.index = index
        self.rows = []  # (datetime or None, [fields after the timestamp])
        self.window = [None, None]
        self._stop = threading.Event()
        self._t = None

    @staticmethod
    def _time(text):
        import datetime
        try:
            return datetime.datetime.strptime(text.strip(), "%Y/%m/%d %H:%M:%S.%f")
        except ValueError:
            return None

    def _run(self):
        try:
            p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.Q}",
                                  "--format=csv,noheader,nounits", "-lms", str(self.INTERVAL_MS)],
                                 stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            return
        while not self._stop.is_set():
            line = p.stdout.readline()
            if not line:
                break
            f = [x.strip() for x in line.split(",")]
            self.rows.append((self._time(f[0]), f[1:]))
        p.terminate()
        try:
            p.wait(timeout=5)
        except subprocess.TimeoutExpired:
            p.kill()

    def mark_start(self):
        import datetime
        self.window[0] = datetime.datetime.now()

    def mark_end(self):
        import datetime
        self.window[1] = datetime.datetime.now()

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)

    def summary(self):
        import datetime
        rows, scope = [r for _, r in self.rows], "whole run"
        if self.window[0] and self.window[1]:
            pad = datetime.timedelta(milliseconds=self.INTERVAL_MS)
            inside = [r for t, r in self.rows
                      if t is not None and self.window[0] - pad <= t <= self.window[1] + pad]
            if inside:
                rows, scope = inside, "timed region"
            else:
                scope = "whole run (no sample inside the timed region)"
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"],
                    "samples": 0, "scope": scope}
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4)
                          if len(r) > 3 + i and r[3 + i] == "Active"})
        loaded = sorted(sm)[len(sm) // 4:] if sm else []
        return {"sm_mhz": float(np.median(loaded)) if loaded else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows), "scope": scope}


def dist_setup(gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        import torch
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, rank, local


def cpu_baseline(pkg, workload, seconds_budget=20.0):
    """The CPU oracle (C/OpenMP restatement, all host threads) on a bounded
    sample of the workload: one request of the workload through one layer
    (prologue + attention over all its rows), scaled to tokens/s through 28
    layers."""
    from oracle import oracle
    oracle.set_threads(os.cpu_count() or 1)  # torchrun sets OMP_NUM_THREADS=1
    L = int(max(workload.lengths))
    cu = [0, L]
    qkv, qw, kw = pkg.workloads.host_layer_inputs(L, seed=1)
    sparse_mode = workload.mode
    reps, elapsed = 0, 0.0
    t0 = time.perf_counter()
    while True:
        q, k = oracle.c_qk_norm_rope(qkv, qw, kw, cu)
        oracle.c_attention(q.astype(np.float16), k.astype(np.float16), qkv, 4096, 3072, cu,
                           sparse_mode if sparse_mode else 0)
        reps += 1
        elapsed = time.perf_counter() - t0
        if elapsed > seconds_budget / 4 or reps >= 3:
            break
    per_layer = elapsed / reps
    value = L / (per_layer * workload.layers)
    return {"value": value, "unit": UNIT, "cores": oracle.threads(), "kind": "port",
            "sample": f"1 request x {L} tokens x 1 layer (prologue + attention, all rows), "
                      f"{reps} rep(s), scaled to {workload.layers} layers"}


def run_reference(args, world, rank):
    """--impl reference: the CPU oracle on the host cores (rank 0 only)."""
    if rank != 0:
        return
    pkg = importlib.import_module(PKG)
    from oracle import oracle
    oracle.set_threads(os.cpu_count() or 1)  # all host threads (torchrun sets OMP_NUM_THREADS=1)
    w = pkg.workloads.WORKLOADS[args.workload]
    # a bounded sample per step: one request through one layer, all rows
    L = int(max(w.lengths))
    qkv, qw, kw = pkg.workloads.host_layer_inputs(L, seed=1)
    cu = [0, L]

    def step():
        q, k = oracle.c_qk_norm_rope(qkv, qw, kw, cu)
        oracle.c_attention(q.astype(np.float16), k.astype(np.float16), qkv, 4096, 3072, cu,
                           w.mode)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = L / (dt * w.layers)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": w.name, "requests": len(w.lengths), "seq_len": L,
                   "layers": w.layers, "mode": w.mode,
                   "note": "reference WGSL/WebGPU path unavailable on this box; CPU oracle "
                           "(C/OpenMP restatement of src/webgpu/ops.ts) timed instead"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": oracle.threads(), "kind": "port",
                         "sample": f"1 request x {L} tokens x 1 layer per step, scaled to "
                                   f"{w.layers} layers"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_engine(args, full_model=False):
    """Micro-batch engine: 16 requests of 15..5000 tokens through the 28-layer
    attention stack (or, with full_model, the whole embedding model: token
    lookup, attention and FFN halves, output norm, pool), packed (varlen) vs
    padded to the longest request as the reference does. Each step is one
    whole micro-batch through the engine's public call (ids host->device,
    embeddings device->host included)."""
    import asyncio
    import torch
    pkg = importlib.import_module(PKG)
    eng_mod = importlib.import_module(PKG + ".engine")
    pool = importlib.import_module(PKG + ".pooling")
    torch.cuda.set_device(0)
    L = args.layers or pkg.workloads.LAYERS
    lengths = pkg.workloads.ragged_lengths(args.requests or 16, 15, 5000, 2025)
    if full_model:
        # seeded weights of the model's shapes (no checkpoint), full vocabulary
        data = pkg.model.synthetic_model_file(L, eng_mod.EOS_TOKEN + 1, seed=7)
        weights = pkg.prepacked.PrepackedWeights(pkg.prepacked.parse_prepacked_model(data), 0)
        rt = pkg.model.Qwen3EmbeddingModel(weights)
        del data
    else:
        rt = eng_mod.AttentionStackRuntime(layers=L, seed=7)
    rng = np.random.default_rng(3)
    reqs = [list(rng.integers(0, eng_mod.EOS_TOKEN, size=n - 1)) + [eng_mod.EOS_TOKEN]
            for n in lengths]
    results, embs = {}, {}
    with ClockSampler(0) as clocks:
        for packing in ("padded", "varlen"):
            eng = eng_mod.EmbeddingEngine(rt, None, 16, 0, packing=packing)

            async def batch():
                return await asyncio.gather(*[eng.submit_tokens(r) for r in reqs])

            for _ in range(args.warmup):
                asyncio.run(batch())
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(args.steps):
                out = asyncio.run(batch())
            torch.cuda.synchronize()
            sec = (time.perf_counter() - t0) / args.steps
            embs[packing] = np.stack(out)
            computed = (len(reqs) * max(lengths) if packing == "padded" else sum(lengths))
            results[packing] = {"ms_per_step": sec * 1e3, "requests_per_s": len(reqs) / sec,
                                "tokens_per_s": sum(lengths) / sec,
                                "tokens_computed_per_layer": computed}
    cos = np.sum(embs["padded"] * embs["varlen"], axis=1)
    # the pool kernel alone, on the packed final hidden state (eager, events)
    cu = [0] + list(np.cumsum(lengths).astype(int).tolist())
    hidden = torch.randn(cu[-1], 1024, device="cuda").half()
    outp = torch.empty(len(lengths), 1024, device="cuda")
    run = pool.LastTokenPoolKernel(0).create_run_varlen(hidden, cu, outp)
    for _ in range(10):
        pkg.attention.encode_run(None, run)
    # 200 launches captured in one CUDA graph, so the host's submission rate
    # does not set the time
    n = 200
    gs = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=gs):
        for _ in range(n):
            pkg.attention.encode_run(None, run)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(gs):  # replay on the stream the events are recorded on
        graph.replay()
        torch.cuda.synchronize()
        e0.record(gs)
        graph.replay()
        e1.record(gs)
    torch.cuda.synchronize()
    pool_ms = e0.elapsed_time(e1) / n
    pool_bytes = len(lengths) * 1024 * (2 + 4)
    # residual + RMSNorm over the packed batch: reads x and the residual, writes
    # x and normalized (8 KB per 1024-wide row; 429 MB per launch, > L2)
    normm = importlib.import_module(PKG + ".norm")
    xs = torch.randn(cu[-1], 1024, device="cuda").half()
    delta = (0.01 * torch.randn(cu[-1], 1024, device="cuda")).half()
    nw = torch.ones(1024, device="cuda")
    nout = torch.empty_like(xs)
    nrun = normm.RmsNormKernel(0).create_run(xs, delta, nw, nout, cu[-1], 1024, 1e-6, True)
    for _ in range(5):
        pkg.attention.encode_run(None, nrun)
    nn = 20
    ng = torch.cuda.CUDAGraph()
    with torch.cuda.graph(ng, stream=gs):
        for _ in range(nn):
            pkg.attention.encode_run(None, nrun)
    with torch.cuda.stream(gs):
        ng.replay()
        torch.cuda.synchronize()
        e0.record(gs)
        ng.replay()
        e1.record(gs)
    torch.cuda.synchronize()
    norm_ms = e0.elapsed_time(e1) / nn
    norm_bytes = cu[-1] * 1024 * 2 * 4
    peaks, psrc = measured_peaks()
    v = results["varlen"]
    line = {
        "metric": ("embedding micro-batch requests/s (engine, whole model)" if full_model
                   else "embedding micro-batch requests/s (engine, attention stack)"),
        "value": v["requests_per_s"], "unit": "requests/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": v["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic token ids; seeded random Q4_0 tile32 weights",
        "config": {"workload": "engine_mixed16", "lengths": list(lengths), "layers": L,
                   "per_layer": ("Q4_0 QKV projection with fused Q/K norm + RoPE (tcgen05), "
                                 "attention, Q4_0 O projection, residual + RMSNorm, Q4_0 "
                                 "gate_up projection, SwiGLU, Q4_0 down projection, residual + "
                                 "RMSNorm; Q6_K token lookup before, last-token pool after"
                                 if full_model else
                                 "Q4_0 QKV projection with fused Q/K norm + RoPE (tcgen05), "
                                 "attention, Q4_0 O projection, residual + RMSNorm; then "
                                 "last-token pool"),
                   "packing": "varlen"},
        "packing": results,
        "varlen_speedup_over_padded": results["padded"]["ms_per_step"] / v["ms_per_step"],
        "padded_vs_varlen_min_cosine": float(cos.min()),
        "pool_kernel": {"avg_launch_ms": pool_ms, "bytes_per_launch": pool_bytes,
                        "achieved_gbs": pool_bytes / (pool_ms * 1e-3) / 1e9,
                        "bound": "launch latency (96 KB per launch)",
                        "timing": "CUDA graph of 200 back-to-back launches, events"},
        "rms_norm_kernel": {"avg_launch_ms": norm_ms, "rows": cu[-1], "width": 1024,
                            "bytes_per_launch": norm_bytes,
                            "achieved_gbs": norm_bytes / (norm_ms * 1e-3) / 1e9,
                            "peak_gbs": peaks["hbm_gbs"], "peak_source": f"{psrc} hbm_gbs",
                            "frac": norm_bytes / (norm_ms * 1e-3) / 1e9 / peaks["hbm_gbs"],
                            "timing": "CUDA graph of 20 launches, events; with residual"},
        "timing": "wall clock around each whole micro-batch through EmbeddingEngine, "
                  "synchronised; pool kernel by CUDA events",
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def _graph_ms(torch, fn, reps=10):
    """Mean ms of fn over a CUDA graph of `reps` calls (events on its stream)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for _ in range(reps):
            fn()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        g.replay()
        torch.cuda.synchronize()
        e0.record(s)
        g.replay()
        e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def run_gemm(args):
    """Projection GEMM (tcgen05) against cuBLAS on the engine's shapes, the
    fused attn_qkv projection + Q/K norm + RoPE against GEMM + prologue, and
    the gate_up projection with the SwiGLU in its epilogue against GEMM +
    SwiGLU kernel. Inputs
    are larger than L2 except where stated; each number is a CUDA graph of 10
    launches timed with events."""
    import torch
    pkg = importlib.import_module(PKG)
    mm, attn = pkg.matmul, pkg.attention
    torch.cuda.set_device(0)
    peaks, psrc = measured_peaks()
    lengths = pkg.workloads.ragged_lengths(16, 15, 5000, 2025)  # the engine's micro-batch
    T = int(sum(lengths))
    shapes = ([(args.gemm_rows, 4096, 1024)] if args.gemm_rows else
              [(T, 4096, 1024), (T, 1024, 2048), (80000, 4096, 1024), (8192, 4096, 1024),
               (16384, 16384, 1024)])
    lines = []
    with ClockSampler(0) as clocks:
        for m, n, k in shapes:
            a = torch.randn(m, k, device="cuda").half()
            w = (torch.randn(n, k, device="cuda") * k ** -0.5).half()
            out = torch.empty(m, n, device="cuda", dtype=torch.float16)
            ours = _graph_ms(torch, lambda: mm.matmul(a, w, out))
            cub = _graph_ms(torch, lambda: torch.matmul(a, w.t(), out=out))
            flop = 2.0 * m * n * k
            lines.append({"shape": [m, n, k], "ours_ms": ours, "ours_tflops": flop / ours / 1e9,
                          "cublas_ms": cub, "cublas_tflops": flop / cub / 1e9,
                          "cta_pairs": m >= 4096})
        rows = args.gemm_rows or T
        cu = [0] + list(np.cumsum(lengths if not args.gemm_rows else [rows]).astype(int).tolist())
        x = torch.randn(rows, 1024, device="cuda").half()
        w = (torch.randn(4096, 1024, device="cuda") * 1024 ** -0.5).half()
        qw = torch.ones(128, device="cuda")
        kw = torch.ones(128, device="cuda")
        q = torch.empty(rows, 16, 128, device="cuda", dtype=torch.half)
        kk = torch.empty(rows, 8, 128, device="cuda", dtype=torch.half)
        v = torch.empty(rows, 1024, device="cuda", dtype=torch.half)
        qkv = torch.empty(rows, 4096, device="cuda", dtype=torch.half)
        fused = _graph_ms(torch, lambda: mm.qkv_projection(x, w, qw, kw, cu, q_out=q, k_out=kk,
                                                          v_out=v))
        gemm = _graph_ms(torch, lambda: mm.matmul(x, w, qkv))
        pro = _graph_ms(torch, lambda: attn.qk_norm_rope(qkv, qw, kw, cu, q_out=q, k_out=kk))
        # ffn_gate_up with the SwiGLU in the epilogue against GEMM + SwiGLU kernel
        wg = (torch.randn(6144, 1024, device="cuda") * 1024 ** -0.5).half()
        wg_il = mm.interleave_gate_up(wg)
        gu = torch.empty(rows, 6144, device="cuda", dtype=torch.half)
        hid = torch.empty(rows, 3072, device="cuda", dtype=torch.half)
        glu_fused = _graph_ms(torch, lambda: mm.matmul_swiglu(x, wg_il, hid))
        glu_gemm = _graph_ms(torch, lambda: mm.matmul(x, wg, gu))
        glu_act = _graph_ms(torch, lambda: pkg.ffn.swiglu(gu, 3072, hid))
    line = {
        "metric": "projection GEMM TFLOP/s (f16 in, f32 accumulate)", "unit": "TFLOP/s",
        "value": lines[0]["ours_tflops"], "n_gpus": 1, "dtype": "f16",
        "peak_tflops": peaks["bf16_tflops"], "peak_source": f"{psrc} bf16_tflops (burst)",
        "shapes": lines,
        "qkv_projection": {"rows": rows, "fused_ms": fused, "gemm_ms": gemm, "prologue_ms": pro,
                           "unfused_ms": gemm + pro, "speedup": (gemm + pro) / fused},
        "gate_up_swiglu": {"rows": rows, "fused_ms": glu_fused, "gemm_ms": glu_gemm,
                           "swiglu_ms": glu_act, "unfused_ms": glu_gemm + glu_act,
                           "fused_tflops": 2.0 * rows * 6144 * 1024 / glu_fused / 1e9,
                           "speedup": (glu_gemm + glu_act) / glu_fused},
        "timing": "CUDA graph of 10 launches per number, events", "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.gemm:
        run_gemm(args)
        return
    if args.engine or args.model:
        run_engine(args, full_model=args.model)
        return
    world, rank, local = dist_setup(args.gpus)
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            import torch.distributed as dist
            dist.barrier()
            dist.destroy_process_group()
        return
    import torch
    pkg = importlib.import_module(PKG)
    attn = pkg.attention
    ex = pkg.executor
    lib = pkg._lib.load()
    w = pkg.workloads.WORKLOADS[args.workload]
    if args.requests or args.layers:
        import dataclasses
        w = dataclasses.replace(
            w, name=w.name + "_reduced",
            lengths=(w.lengths * 64)[:args.requests] if args.requests else w.lengths,
            layers=args.layers or w.layers)
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    ctx = attn.Context.for_device(local)
    # Strong scaling (default): the workload's requests are split across the
    # ranks (LPT on kept pairs), each rank runs its share as one packed
    # micro-batch. --weak-scaling: every rank runs the whole workload.
    plan = ex.ShardPlan(w.lengths, 1 if args.weak_scaling else world, w.mode)
    me = 0 if args.weak_scaling else rank
    cu = plan.local_cu(me)
    cu_c = pkg._lib.cu_array(cu)
    T = plan.local_tokens(me)
    T_all = plan.total_tokens * (world if args.weak_scaling else 1)
    mode = plan.resolved_mode  # AUTO resolved on the whole micro-batch
    L = w.layers
    idle = T == 0

    # inputs resident in HBM: one qkv activation per layer (each > L2 at the
    # default workload, so consecutive layers never hit in L2), per-layer
    # norm weights
    layers = [pkg.workloads.device_layer_inputs(max(T, 1), seed=1000 * rank + l, device=dev)
              for l in range(L)]
    Tb = max(T, 1)
    q_buf = torch.empty(Tb, 16, 128, dtype=torch.float16, device=dev)
    k_buf = torch.empty(Tb, 8, 128, dtype=torch.float16, device=dev)
    out = torch.empty(Tb, 16, 128, dtype=torch.float16, device=dev)
    stream = torch.cuda.Stream(dev)
    s = stream.cuda_stream
    P = attn._ptr

    def layer_calls(qkv, qw, kw, ev=None, out_buf=None):
        o = out if out_buf is None else out_buf
        st = lib.qwa_qk_norm_rope(ctx.handle, P(qkv), 4096, P(qw), P(kw), P(q_buf), P(k_buf),
                                  cu_c, len(cu) - 1, 1e-6, 1e6, None, s)
        if st:
            pkg._lib.check(st, ctx.handle)
        if ev is not None:
            ev[0].record(stream)
        st = lib.qwa_attention(ctx.handle, P(q_buf), P(k_buf), P(qkv), 4096, 3072, P(o), cu_c,
                               len(cu) - 1, mode, 176, 432, s)
        if st:
            pkg._lib.check(st, ctx.handle)
        if ev is not None:
            ev[1].record(stream)

    def step(evs=None):
        if idle:
            return
        for l, (qkv, qw, kw) in enumerate(layers):
            layer_calls(qkv, qw, kw, evs[l] if evs is not None else None)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    ctx.check(stream)

    def barrier():
        if world > 1:
            import torch.distributed as dist
            dist.barrier()

    # The step (2 launches x L layers) is captured once in a CUDA graph and
    # replayed: the timed region then measures the device, not Python/ctypes
    # launch overhead (which dominates the small configurations). After the
    # warm-up every call is capture-safe: plans are cached and tensor maps are
    # encoded on the host.
    graph = torch.cuda.CUDAGraph()
    if not idle:
        with torch.cuda.graph(graph, stream=stream):
            step()
        with torch.cuda.stream(stream):
            graph.replay()
    torch.cuda.synchronize()
    ctx.check(stream)

    def replay():
        if not idle:
            graph.replay()

    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        # the sampler is up (and the clocks settled under load) before timing
        with torch.cuda.stream(stream):
            for _ in range(max(1, args.warmup)):
                replay()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        clocks.mark_start()
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(args.steps):
                replay()
            end.record(stream)
        torch.cuda.synchronize()
        clocks.mark_end()
    barrier()
    ctx.check(stream)
    ms = start.elapsed_time(end) / args.steps

    # Per-kernel device times for the roofline: the same K steps launched
    # eagerly with CUDA events around each prologue and attention launch.
    ev_layer = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(L)]
                for _ in range(args.steps)]
    ev_pro_start = [[torch.cuda.Event(enable_timing=True) for _ in range(L)]
                    for _ in range(args.steps)]
    attn_ms, pro_ms = [0.0], [0.0]
    if not idle:
        for kstep in range(args.steps):
            for l, (qkv, qw, kw) in enumerate(layers):
                ev_pro_start[kstep][l].record(stream)
                layer_calls(qkv, qw, kw, ev_layer[kstep][l])
        torch.cuda.synchronize()
        ctx.check(stream)
        attn_ms = [ev_layer[k][l][0].elapsed_time(ev_layer[k][l][1])
                   for k in range(args.steps) for l in range(L)]
        pro_ms = [ev_pro_start[k][l].elapsed_time(ev_layer[k][l][0])
                  for k in range(args.steps) for l in range(L)]
    rank_ms = [ms]
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev)
        gathered = [torch.zeros(1, device=dev) for _ in range(world)]
        dist.all_gather(gathered, t)
        rank_ms = [float(x.item()) for x in gathered]
        ms = max(rank_ms)

    # End to end through the package's request-sharded executor, with host
    # buffers: every layer's qkv rows of this rank's requests cross
    # host->device from page-locked memory, and the layer's output rows come
    # back into one host output buffer at their requests' rows (the host
    # gather; with several ranks the buffers are shared memory that every
    # rank maps). Uploads, kernels and downloads of consecutive layers
    # overlap (double-buffered, ordered by events; PCIe is full duplex).
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e(args, torch, ex, plan, me, world, rank, local, dev, layers, ctx, barrier,
                      T, T_all, L)

    if rank != 0:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    peaks, src = measured_peaks()
    pairs, tiles = attn.attention_work(cu, mode) if not idle else (0, 0)
    flop_per_launch = 8192.0 * pairs
    attn_avg = float(np.mean(attn_ms))
    pro_avg = float(np.mean(pro_ms))
    achieved_tflops = flop_per_launch / (attn_avg * 1e-3) / 1e12 if attn_avg else 0.0
    peak = peaks.get("bf16_tflops_sustained") or peaks["bf16_tflops"]
    # attention kernel bytes: read q, k, v (4096 + 2048 + 2048 B), write out (4096 B)
    attn_kernel_bytes = T * 12288
    ridge = peak * 1e12 / (peaks["hbm_gbs"] * 1e9)
    intensity = flop_per_launch / attn_kernel_bytes if T else 0.0
    hbm_bound = intensity < ridge
    pro_bytes = T * (2048 + 1024) * 2 * 2  # read q,k columns; write q,k
    attn_bytes = T * 12288  # algorithmic bytes of the hot path per token
    traffic, traffic_src = None, None
    tfile = os.path.join(ROOT, "profiles", "attention_traffic.json")
    if os.path.exists(tfile):
        with open(tfile) as f:
            tinfo = json.load(f).get(w.name)
        if tinfo:
            # DRAM traffic grows with the tokens of a launch (requests of one
            # length), so a capture is scaled to this rank's share
            traffic = tinfo["bytes_per_launch"] * T / plan.total_tokens
            traffic_src = ("not measured by this run: scaled from a smaller ncu capture ("
                           + tinfo["source"] + ")")
    ms_safe = ms if ms > 0 else float("nan")
    strong = not args.weak_scaling
    line = {
        "metric": METRIC, "value": T_all / (ms_safe / 1e3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong" if strong else "weak",
        "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded N(0,1) qkv per layer, weights 1+N(0,0.02))",
        "config": {"workload": w.name, "requests": len(w.lengths) * (1 if strong else world),
                   "seq_len": int(max(w.lengths)), "tokens": T_all, "layers": L,
                   "mode": ["auto(sparse<=8192)", "full", "sparse"][w.mode]
                           + (" -> sparse" if mode == 2 else " -> full"),
                   "global_batch": len(w.lengths) * (1 if strong else world),
                   "parallelism": (f"requests split over {world} GPU(s) (LPT on kept pairs), "
                                   "host gather, no collective" if strong else
                                   f"dp{world}: every rank runs the whole workload"),
                   "requests_per_rank": ([len(r) for r in plan.assignment] if strong
                                         else [len(w.lengths)] * world),
                   "tokens_per_rank": ([plan.local_tokens(r) for r in range(world)] if strong
                                       else [T] * world),
                   "l2": "inputs larger than L2 (one qkv of >= 82 MB per layer per rank)"
                         if T * 8192 > 126e6 else
                         "qkv per layer smaller than L2; each of the 28 layers reads its own "
                         "buffer, so the 28 x qkv working set exceeds L2"},
        "rank_ms_per_step": rank_ms,
        "roofline": ({"bound": "hbm", "achieved": attn_kernel_bytes / (attn_avg * 1e-3) / 1e9,
                      "peak": peaks["hbm_gbs"], "unit": "GB/s",
                      "frac": attn_kernel_bytes / (attn_avg * 1e-3) / 1e9 / peaks["hbm_gbs"],
                      "peak_source": f"{src} hbm_gbs (copy bandwidth)",
                      "achieved_tflops": achieved_tflops}
                     if hbm_bound else
                     {"bound": "tensor", "achieved": achieved_tflops, "peak": peak,
                      "unit": "TFLOP/s", "frac": achieved_tflops / peak,
                      "frac_burst": achieved_tflops / peaks["bf16_tflops"],
                      "peak_burst": peaks["bf16_tflops"],
                      "peak_source": f"{src} bf16_tflops_sustained (kernel timed inside a "
                                     f"{L}-layer step); frac_burst against {src} bf16_tflops"})
                    if attn_avg else {"bound": None, "achieved": None, "note": "rank 0 idle"},
        "prologue": {"avg_launch_ms": pro_avg, "bytes_per_launch": pro_bytes,
                     "achieved_gbs": pro_bytes / (pro_avg * 1e-3) / 1e9 if pro_avg else None,
                     "peak_gbs": peaks["hbm_gbs"],
                     "frac": pro_bytes / (pro_avg * 1e-3) / 1e9 / peaks["hbm_gbs"]
                     if pro_avg else None},
        "attention_share_of_step": float(np.sum(attn_ms) / args.steps / rank_ms[0])
        if rank_ms[0] else None,
        "algorithmic_bytes_per_token_layer": 12288, "hot_path_bytes_per_step": attn_bytes * L,
        "gpu_launches": 0 if idle else 2 * L * args.steps,  # rank 0's launches in the region
        "timing": "CUDA graph of one step replayed K times (max over ranks); per-kernel times "
                  "(rank 0) from an eager event-instrumented pass of the same K steps",
        "clocks": clocks.summary(),
    }
    if attn_avg:
        line["roofline"].update({"traffic": traffic, "traffic_source": traffic_src,
                                 "kernel": "attention_kernel",
                                 "flop_per_launch": flop_per_launch,
                                 "bytes_per_launch": attn_kernel_bytes,
                                 "arithmetic_intensity": intensity, "ridge": ridge,
                                 "avg_launch_ms": attn_avg})
    if e2e:
        line["e2e"] = e2e
    if not args.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(pkg, w)
    print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def run_e2e(args, torch, ex, plan, me, world, rank, local, dev, layers, ctx, barrier, T, T_all,
            L):
    """The e2e leg (see main): returns the e2e dict (on every rank)."""
    Tg = plan.total_tokens
    shared = world > 1 and not args.weak_scaling
    in_shape, out_shape = (Tg, 4096), (Tg, 16, 128)
    nbytes = 2 * (Tg * 4096 * 2 + Tg * 2048 * 2)
    bufs = None
    gather = "one page-locked host buffer"
    if shared:
        if ex.SharedHostBuffer.fits(nbytes):
            tag = os.environ.get("MASTER_PORT", "0")
            names = [f"/dev/shm/qwa_bench_{tag}_{n}" for n in ("in0", "in1", "out0", "out1")]
            shapes = [in_shape, in_shape, out_shape, out_shape]
            if rank == 0:
                bufs = [ex.SharedHostBuffer(n, sh, create=True) for n, sh in zip(names, shapes)]
            barrier()
            if rank != 0:
                bufs = [ex.SharedHostBuffer(n, sh) for n, sh in zip(names, shapes)]
            host_in = [b.tensor for b in bufs[:2]]
            host_out = [b.tensor for b in bufs[2:]]
            gather = ("host buffers in shared memory mapped by every rank: each rank copies its "
                      "requests' output rows to their place")
        else:
            shared = False
            gather = "per-rank page-locked buffers (shared memory too small for the gather)"
    if not shared:
        host_in = [torch.empty(in_shape, dtype=torch.float16).pin_memory() for _ in range(2)]
        host_out = [torch.empty(out_shape, dtype=torch.float16).pin_memory() for _ in range(2)]
    # each rank writes its own requests' rows of the host input
    ranges = plan.row_ranges(me)
    for h in host_in:
        for g, l0, n in ranges:
            h[g:g + n].copy_(layers[0][0][l0:l0 + n])
    barrier()
    backend = ex.DeviceBackend(local, T, buffers=2, ctx=ctx)
    shard = ex.ShardExecutor(plan, me, backend)
    ins = [host_in[l % 2] for l in range(L)]
    outs = [host_out[l % 2] for l in range(L)]
    ws = [(qw, kw) for _, qw, kw in layers]
    shard.run(ins, outs, ws)
    torch.cuda.synchronize()
    backend.check()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(backend.stream)
    for _ in range(args.e2e_steps):
        shard.run(ins, outs, ws)
    e1.record(backend.stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = e0.elapsed_time(e1) / args.e2e_steps if T else 0.0
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    if bufs:
        barrier()
        for b in bufs:
            b.close(unlink=rank == 0)
    return {"value": T_all / (e2e_ms / 1e3), "unit": UNIT,
            "h2d_bytes_per_step": T * 4096 * 2 * L, "d2h_bytes_per_step": T * 2048 * 2 * L,
            "bytes_scope": "per rank (rank 0)" if world > 1 else "whole job",
            "ms_per_step": e2e_ms, "gather": gather,
            "path": "executor.ShardExecutor + DeviceBackend (qwa_prefill_attention_layer)"}


if __name__ == "__main__":
    main()
