#!/usr/bin/env python
"""Benchmark of the Q2_K mul_mat hot path on B200 (one JSON line per run; the metric is defined below).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload decode|gemv|prefill] [--quant program|separate|fused|mixed]

Workloads (one "step" each):
  decode  (default)  one token through the Llama-2-7B-shape Q2_K linear stack:
                     32 layers x {Wq,Wk,Wv,Wo 4096x4096; Wg,Wu 11008x4096;
                     Wd 4096x11008} + lm_head 32000x4096, batch 1, every linear's
                     input re-quantized to Q8_K (RMSNorm fused before the qkv,
                     gate/up and lm_head inputs).  On one GPU the whole step is
                     one persistent kernel (q2k_program_kernel); on N GPUs the
                     weights are row-sharded and each linear is one GEMV launch
                     whose finishers also store their rows into every rank's
                     copy of the next input over NVLink (CUDA-IPC peer memory)
                     and signal it; the next GEMV waits for all ranks' rows
                     (--quant separate: NCCL all-gathers instead).
  gemv               one Q2_K x Q8_K GEMV W[4096,4096] x x[4096], rotating
                     over 64 distinct weight copies (352 MB > L2).
  prefill            activations [512,4096] (Q8_K per row) x W[11008,4096] Q2_K
                     on the tcgen05 tensor cores.
  attention          sme_ai_self_attention packed, causal: 2048 tokens,
                     model_dim 4096, 32 heads (fp16 weights, fp32 projections,
                     scores, softmax and weighted sum); its own metric, tokens/s.

Metric: "Q2_K mul_mat HBM GB/s": algorithmic bytes of every GEMV in the step
(Q2_K weights + Q8_K activations + fp32 outputs), summed over ranks, per
second of the step time (max over ranks, CUDA events).  The line also gives
tokens/s.  Weights are seeded N(0, 0.02) draws quantized to Q2_K on the device
(synthetic; no checkpoint).  The 2.17 GB of weights per token exceed the
126 MB L2, so no L2 flush is needed between steps.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "sme-ai-ops_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "Q2_K mul_mat HBM GB/s (% of peak) and 7B-shape linear-layer tokens/s"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["decode", "gemv", "prefill", "prefill-stack", "attention"],
                    default="decode")
    ap.add_argument("--attn-seq", type=int, default=2048, help="attention workload: tokens")
    ap.add_argument("--attn-dim", type=int, default=4096, help="attention workload: model_dim")
    ap.add_argument("--attn-heads", type=int, default=32, help="attention workload: heads")
    ap.add_argument("--prefill-tokens", type=int, default=512, help="prefill workload: activation rows")
    ap.add_argument("--prefill-shard", choices=["tokens", "rows"], default="tokens",
                    help="prefill-stack on N > 1 GPUs: split the tokens over the ranks (full weights on every rank, no data-path collective) or the weight rows (NCCL all-gathers of every output)")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--decode-batch", type=int, default=1, choices=[1, 2, 4, 8],
                    help="decode workload: tokens per step (the batch of a decode step)")
    ap.add_argument("--quant", choices=["fused", "separate", "mixed", "program"], default="program",
                    help="decode: 'program' (default) runs the whole step as one persistent kernel on one GPU; "
                         "the others launch one GEMV per linear with the Q8_K quantization fused, separate or "
                         "mixed (all give identical results; N > 1 GPUs always launch per linear)")
    ap.add_argument("--gemv-rows", type=int, default=4096, help="gemv workload: weight rows")
    ap.add_argument("--gemv-k", type=int, default=4096, help="gemv workload: row length")
    ap.add_argument("--gemv-epilogue", type=int, default=0, help="gemv workload: 0 store, 1 residual, 2 silu*mul")
    ap.add_argument("--gemv-fmt", choices=["q2k", "q3k", "q6k"], default="q2k", help="gemv workload: weight format")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="decode on one GPU: skip the per-configuration measurements (configs 1-4)")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="bounded CPU sample length")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def hbm_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def traffic_ratio(name="q2k_gemv_decode.txt"):
    """DRAM bytes per algorithmic byte of a kernel, from its committed ncu
    summary under profiles/ (line 'traffic_ratio=<x>')."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(path):
            if line.startswith("traffic_ratio="):
                return float(line.split("=", 1)[1].split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------- CPU side
class CpuLayerSample:
    """The oracle (ggml generic-C restatement) on one full layer of the stack:
    qkv, o, gate+up and down GEMVs at full shape, batch 1, rows split over
    the host's cores with OpenMP.  Weights are random Q2_K blocks with the
    magnitudes of quantized N(0, 0.02) draws, not the GPU run's seeded
    weights: the generic dot's work does not depend on the values.
    Activations are Q8_K of N(0, 1)."""

    def __init__(self, hidden=4096, ffn=11008, n_threads=1, seed=0):
        import numpy as np
        from oracle import oracle as O
        from smeai_b200.stack import gemv_bytes
        self.O, self.threads = O, n_threads
        rng = np.random.default_rng(seed)

        def rand_q2k(rows, k):
            nb = k // 256
            b = rng.integers(0, 256, size=(rows * nb, 84), dtype=np.uint8)
            d = (np.abs(rng.standard_normal(rows * nb)) * 0.002 + 1e-4).astype(np.float16)
            dm = (np.abs(rng.standard_normal(rows * nb)) * 0.004 + 1e-4).astype(np.float16)
            b[:, 80:82] = d.view(np.uint8).reshape(-1, 2)
            b[:, 82:84] = dm.view(np.uint8).reshape(-1, 2)
            return b.reshape(-1).view(O.BLOCK_Q2_K)

        self.mats = [(3 * hidden, hidden), (hidden, hidden), (2 * ffn, hidden), (hidden, ffn)]
        self.ws = [rand_q2k(r, k) for r, k in self.mats]
        self.xs = {k: O.quantize_q8_K(rng.standard_normal(k).astype(np.float32)) for k in (hidden, ffn)}
        self.layer_bytes = sum(gemv_bytes(r, k, 1) for r, k in self.mats)

    def run_once(self, threads=None):
        for (r, k), w in zip(self.mats, self.ws):
            self.O.q2k_mul_mat(w, r, k, self.xs[k], 1, n_threads=self.threads if threads is None else threads)

    def timed(self, seconds):
        """Repeat the layer until `seconds` elapsed (at least once): (GB/s, s per layer, reps)."""
        reps, t0 = 0, time.perf_counter()
        while True:
            self.run_once()
            reps += 1
            el = time.perf_counter() - t0
            if el >= seconds:
                break
        per_layer = el / reps
        return self.layer_bytes / per_layer / 1e9, per_layer, reps


def cpu_rate(unit_fn, seconds, threads):
    """Repeat unit_fn(threads) until `seconds` elapsed (at least twice):
    seconds per unit, units run."""
    unit_fn(threads)
    reps, t0 = 0, time.perf_counter()
    while True:
        unit_fn(threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds and reps >= 2:
            return el / reps, reps


def cpu_baseline_pair(unit_fn, seconds, per_unit, unit, sample, single_only=False):
    """CPU baseline of the oracle (-march=native build) on this host: one
    thread and every host thread (OpenMP rows).  per_unit converts seconds
    per unit into the metric's unit.  value = the all-cores figure."""
    from oracle import oracle as O
    O.select(native=True)
    try:
        threads = os.cpu_count() or 1
        s1, r1 = cpu_rate(unit_fn, seconds, 1)
        out = {"unit": unit, "kind": "port", "cpu_model": O.cpu_model(), "nproc": threads,
               "build": "gcc -O3 -march=native -ffp-contract=off -fopenmp",
               "single_thread": {"value": per_unit(s1), "cores": 1, "reps": r1}}
        if single_only:
            out.update(value=per_unit(s1), cores=1, sample=sample + " (a scalar loop: one thread)")
        else:
            sa, ra = cpu_rate(unit_fn, seconds, threads)
            out["all_cores"] = {"value": per_unit(sa), "cores": threads, "reps": ra}
            out.update(value=per_unit(sa), cores=threads, sample=sample)
        return out
    finally:
        O.select(native=False)


def graph_time(step, stream, calls, replays, warmup):
    """Capture `calls` back-to-back calls of step() in a CUDA graph, replay it
    `warmup` times, then time `replays` replays with CUDA events on the stream:
    device ms per call."""
    import torch
    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(calls):
            step()
    for _ in range(max(3, warmup)):
        with torch.cuda.stream(stream):
            g.replay()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(replays):
            g.replay()
    e1.record(stream)
    e1.synchronize()
    ms = e0.elapsed_time(e1) / (replays * calls)
    del g
    return ms


def per_launch_ms(launch, stream, n):
    """Median device time of n single launches, each bracketed by events on
    the stream and queued behind a sleep kernel (launch gaps do not count)."""
    import torch
    evs = []
    with torch.cuda.stream(stream):
        torch.cuda._sleep(20_000_000)
        for i in range(n):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            launch(i)
            b.record(stream)
            evs.append((a, b))
    stream.synchronize()
    return statistics.median(a.elapsed_time(b) for a, b in evs)


def run_configs(dev, stream, args, peak, peak_kind):
    """Configurations 1-4 of the workload list, each with its own value,
    roofline and CPU baseline (the headline is configuration 5)."""
    import ctypes

    import numpy as np
    import torch

    import smeai_b200 as S
    from oracle import oracle as O
    from smeai_b200 import q2k as Q
    from smeai_b200.stack import gemv_bytes
    L = S.lib()
    P = ctypes.c_void_p
    cpu_s = max(1.5, args.cpu_seconds / 5)
    steps, warm = max(args.steps, 10), args.warmup
    fp32_peak = 148 * 128 * 2 * 1.965e9 / 1e12
    out = {}

    # ---- 1: fp16-ABI packed Linear X[128,512] . W[512,512]^T + b
    B, K, N = 128, 512, 512
    rng = np.random.default_rng(0)
    x16 = rng.standard_normal((B, K)).astype(np.float16)
    w = rng.uniform(-1 / np.sqrt(K), 1 / np.sqrt(K), (N, K)).astype(np.float32)
    wt16 = np.ascontiguousarray(w.T).astype(np.float16)          # the ABI's W[in][out]
    bias = (rng.standard_normal(N) * 0.02).astype(np.float32)
    ws, pw = S.Workspace(), S.PackedWeight()
    S.check(L.sme_ai_workspace_init(ctypes.byref(ws), B, K, N), "workspace_init")
    S.check(L.sme_ai_packed_linear_weight_init(ctypes.byref(pw), P(wt16.ctypes.data), K, N), "packed_init")
    xd = torch.from_numpy(x16.view(np.int16)).to(dev)
    bd = torch.from_numpy(bias).to(dev)
    yd = torch.empty((B, N), device=dev)
    st = P(stream.cuda_stream)
    lin = lambda: L.sme_ai_linear_packed_f16f32_device(P(xd.data_ptr()), B, ctypes.byref(pw), P(bd.data_ptr()), 0,
                                                      P(yd.data_ptr()), st)
    ms = graph_time(lin, stream, 50, steps, warm)
    flops = 2 * B * K * N
    exp = O.linear_f16f32(x16.view(np.uint16), B, K, wt16.view(np.uint16), N, bias)
    exact = bool(np.array_equal(yd.cpu().numpy().view(np.uint32), exp.view(np.uint32)))
    yh = np.zeros((B, N), np.float32)
    host = lambda: L.sme_ai_linear_sme_packed_f16f32(ctypes.byref(ws), P(x16.ctypes.data), B, ctypes.byref(pw),
                                                     P(bias.ctypes.data), P(yh.ctypes.data))
    host()
    t0, reps = time.perf_counter(), 0
    while reps < 200:
        host()
        reps += 1
    e2e_ms = (time.perf_counter() - t0) / reps * 1e3
    one = lambda n: O.linear_f16f32(x16.view(np.uint16), B, K, wt16.view(np.uint16), N, bias)
    out["config1_fp_linear"] = {
        "workload": "fp16-ABI packed Linear X[128,512] ~N(0,1) . W[512,512]^T ~U(+-1/sqrt(512)) + b ~N(0,0.02) "
                    "-> fp32 (sme_ai_linear_packed_f16f32_device)",
        "value": flops / (ms / 1e3) / 1e9, "unit": "GFLOP/s", "us_per_call": ms * 1e3,
        "bit_exact_vs_oracle": exact,
        "e2e": {"value": flops / (e2e_ms / 1e3) / 1e9, "unit": "GFLOP/s", "us_per_call": e2e_ms * 1e3,
                "entry": "sme_ai_linear_sme_packed_f16f32 (host buffers, synchronous)",
                "h2d_bytes_per_call": B * K * 2 + N * 4, "d2h_bytes_per_call": B * N * 4},
        "roofline": {"bound": "fp32 FFMA (latency at this size)", "achieved": flops / (ms / 1e3) / 1e12,
                     "peak": fp32_peak, "unit": "TFLOP/s", "frac": flops / (ms / 1e3) / 1e12 / fp32_peak,
                     "peak_kind": "nominal FP32 CUDA-core rate (no measured fp32 peak on this pool)",
                     "traffic": None, "flops_per_launch": flops},
        "cpu_baseline": cpu_baseline_pair(one, cpu_s, lambda sec: flops / sec / 1e9, "GFLOP/s",
                                          "the oracle's scalar_matmul_f16f16_f32 restatement on the same inputs",
                                          single_only=True),
    }
    L.sme_ai_packed_linear_weight_destroy(ctypes.byref(pw))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))

    # ---- 2: Q2_K x Q8_K GEMV W[4096,4096]
    rows, k = 4096, 4096
    nb = k // 256
    mbytes = rows * nb * 84
    copies = max(4, -(-4 * 126 * 2**20 // mbytes))
    g = torch.Generator(device=dev).manual_seed(0)
    blocks = [Q.quantize_q2k(torch.randn((rows, k), generator=g, device=dev) * 0.02) for _ in range(copies)]
    mats = [Q.Q2KMatrix(b, rows, k) for b in blocks]
    x = torch.randn((1, k), generator=g, device=dev)
    xq = Q.quantize_q8k(x)
    y = torch.empty((1, rows), device=dev)
    it = {"i": 0}

    def gemv_step():
        m = mats[it["i"] % copies]
        it["i"] += 1
        m.mul_mat(xq, 1, out=y)

    ms = graph_time(gemv_step, stream, copies, steps, warm)
    nbytes = gemv_bytes(rows, k, 1)
    lms = per_launch_ms(lambda i: mats[i % copies].mul_mat(xq, 1, out=y), stream, 16)
    w0 = blocks[0].cpu().numpy().reshape(-1).view(O.BLOCK_Q2_K)
    xq0 = xq.cpu().numpy().reshape(-1).view(O.BLOCK_Q8_K)
    exact = bool(np.array_equal(mats[0].mul_mat(xq, 1).cpu().numpy().view(np.uint32),
                                O.q2k_mul_mat(w0, rows, k, xq0, 1, n_threads=os.cpu_count()).view(np.uint32)))
    ratio = traffic_ratio()
    out["config2_gemv"] = {
        "workload": f"Q2_K x Q8_K GEMV W[4096,4096] ~N(0,0.02) -> Q2_K, x[4096] ~N(0,1) -> Q8_K, y[4096]; "
                    f"{copies} rotating weight copies ({copies * mbytes / 2**20:.0f} MB > L2)",
        "value": nbytes / (ms / 1e3) / 1e9, "unit": "GB/s", "us_per_call": ms * 1e3, "bit_exact_vs_oracle": exact,
        "roofline": {"bound": "hbm", "kernel": "q2k_gemv_kernel", "achieved": nbytes / (lms / 1e3) / 1e9,
                     "peak": peak, "unit": "GB/s", "frac": nbytes / (lms / 1e3) / 1e9 / peak, "peak_kind": peak_kind,
                     "traffic": ratio * nbytes if ratio else None, "algorithmic_bytes_per_launch": nbytes,
                     "median_launch_us": lms * 1e3},
        "cpu_baseline": cpu_baseline_pair(lambda n: O.q2k_mul_mat(w0, rows, k, xq0, 1, n_threads=n), cpu_s,
                                          lambda sec: nbytes / sec / 1e9, "GB/s",
                                          "the oracle's generic-C Q2_K x Q8_K dot over the same W and x"),
    }
    del mats, blocks

    # ---- 3: SwiGLU MLP decode, batch 1 and 8 (the two phases as one program launch)
    H, F = 4096, 11008
    per_copy = (2 * F * (H // 256) + H * (F // 256)) * 84
    copies = max(3, -(-4 * 126 * 2**20 // per_copy))
    gu_m, dn_m, blk = [], [], None
    for c in range(copies):
        wg = Q.quantize_q2k(torch.randn((F, H), generator=g, device=dev) * 0.02)
        wu = Q.quantize_q2k(torch.randn((F, H), generator=g, device=dev) * 0.02)
        wd = Q.quantize_q2k(torch.randn((H, F), generator=g, device=dev) * 0.02)
        gu_m.append(Q.Q2KMatrix(torch.stack([wg, wu], 1).reshape(2 * F, -1), 2 * F, H))
        dn_m.append(Q.Q2KMatrix(wd, H, F))
        if c == 0:
            blk = [t.cpu().numpy().reshape(-1).view(O.BLOCK_Q2_K) for t in (wg, wu, wd)]
        del wg, wu, wd
    for B in (1, 8):
        xb = torch.randn((B, H), generator=g, device=dev)
        hb = torch.empty((B, F), device=dev)
        yb = torch.empty((B, H), device=dev)
        progs = [Q.Q2KProgram([dict(w=gu_m[c], x=xb, input=S.IN_F32, y=hb, epilogue=S.EPI_SILU_MUL),
                               dict(w=dn_m[c], x=hb, input=S.IN_F32, y=yb)], B) for c in range(copies)]
        it = {"i": 0}

        def mlp_step():
            progs[it["i"] % copies].run()
            it["i"] += 1

        ms = graph_time(mlp_step, stream, copies, steps, warm)
        nbytes = gemv_bytes(2 * F, H, B, F) + gemv_bytes(H, F, B)
        lms = per_launch_ms(lambda i: progs[i % copies].run(), stream, 12)
        progs[0].run()
        torch.cuda.synchronize()
        y_gpu, h_gpu = yb.cpu().numpy(), hb.cpu().numpy()
        xq_o = O.quantize_q8_K(xb.cpu().numpy().reshape(-1))
        gg = O.q2k_mul_mat(blk[0], F, H, xq_o, B, n_threads=os.cpu_count())
        uu = O.q2k_mul_mat(blk[1], F, H, xq_o, B, n_threads=os.cpu_count())
        h_o = O.silu_mul(gg.reshape(-1), uu.reshape(-1)).reshape(B, F)
        hq_o = O.quantize_q8_K(h_gpu.reshape(-1))
        y_o = O.q2k_mul_mat(blk[2], H, F, hq_o, B, n_threads=os.cpu_count())
        ok = bool(np.all(np.abs(h_gpu - h_o) <= 1e-5 * np.abs(h_o) + 1e-30) and
                  np.array_equal(y_gpu.view(np.uint32), y_o.view(np.uint32)))

        def mlp_cpu(n, B=B, xq_o=xq_o):
            g_ = O.q2k_mul_mat(blk[0], F, H, xq_o, B, n_threads=n)
            u_ = O.q2k_mul_mat(blk[1], F, H, xq_o, B, n_threads=n)
            h_ = O.silu_mul(g_.reshape(-1), u_.reshape(-1))
            O.q2k_mul_mat(blk[2], H, F, O.quantize_q8_K(h_), B, n_threads=n)

        out[f"config3_swiglu_b{B}"] = {
            "workload": f"SwiGLU MLP decode, batch {B}: hidden 4096, ffn 11008, W_gate/W_up[11008,4096] and "
                        f"W_down[4096,11008] ~N(0,0.02) Q2_K, x ~N(0,1); gate/up (silu*mul) and down as one "
                        f"q2k_program launch; {copies} rotating weight copies ({copies * per_copy / 2**20:.0f} MB)",
            "value": nbytes / (ms / 1e3) / 1e9, "unit": "GB/s", "us_per_call": ms * 1e3,
            "tokens_per_s": B / (ms / 1e3), "matches_oracle": ok,
            "roofline": {"bound": "hbm", "kernel": "q2k_program_kernel", "achieved": nbytes / (lms / 1e3) / 1e9,
                         "peak": peak, "unit": "GB/s", "frac": nbytes / (lms / 1e3) / 1e9 / peak,
                         "peak_kind": peak_kind, "traffic": None, "algorithmic_bytes_per_launch": nbytes,
                         "median_launch_us": lms * 1e3},
            "cpu_baseline": cpu_baseline_pair(mlp_cpu, cpu_s, lambda sec: nbytes / sec / 1e9, "GB/s",
                                              f"the oracle's generic-C dots of the same MLP, batch {B}"),
        }
        for pr in progs:
            pr.free()
    del gu_m, dn_m

    # ---- 4: prefill mul_mat [512,4096] x W[11008,4096] on tcgen05
    rows, k, cols = 11008, 4096, 512
    copies = max(2, -(-4 * 126 * 2**20 // (rows * (k // 256) * 84)))
    wblocks0 = Q.quantize_q2k(torch.randn((rows, k), generator=g, device=dev) * 0.02)
    mats = [Q.Q2KMatrix(wblocks0, rows, k)] + [
        Q.Q2KMatrix(Q.quantize_q2k(torch.randn((rows, k), generator=g, device=dev) * 0.02), rows, k)
        for _ in range(copies - 1)]
    xa = torch.randn((cols, k), generator=g, device=dev)
    xqa = Q.quantize_q8k(xa)
    ya = torch.empty((cols, rows), device=dev)
    it = {"i": 0}

    def gemm_step():
        mats[it["i"] % copies].mul_mat_tc(xqa, cols, out=ya)
        it["i"] += 1

    ms = graph_time(gemm_step, stream, copies, steps, warm)
    ops = 2 * rows * k * cols
    lms = per_launch_ms(lambda i: mats[i % copies].mul_mat_tc(xqa, cols, out=ya), stream, 8)
    tpeak, tkind = tensor_peak()
    i8peak = 2 * tpeak
    mats[0].mul_mat_tc(xqa, cols, out=ya)
    torch.cuda.synchronize()
    w0 = wblocks0.cpu().numpy().reshape(-1).view(O.BLOCK_Q2_K)
    xq_all = xqa.cpu().numpy().reshape(cols, -1)
    sample_rows = [0, 1, 137, 255, 256, 511]
    exp = O.q2k_mul_mat(w0, rows, k, np.ascontiguousarray(xq_all[sample_rows]).reshape(-1).view(O.BLOCK_Q8_K),
                        len(sample_rows), n_threads=os.cpu_count())
    exact = bool(np.array_equal(ya.cpu().numpy()[sample_rows].view(np.uint32), exp.view(np.uint32)))
    cs = 16                                      # CPU sample: 16 of the 512 activation rows
    xq_s = np.ascontiguousarray(xq_all[:cs]).reshape(-1).view(O.BLOCK_Q8_K)
    s_ops = 2 * rows * k * cs
    out["config4_prefill"] = {
        "workload": "Q2_K prefill mul_mat: activations [512,4096] ~N(0,1) (Q8_K per row) x W[11008,4096] "
                    f"~N(0,0.02) Q2_K -> fp32 [512,11008] on tcgen05 (kind::i8 + kind::f16); {copies} rotating "
                    "weight copies",
        "value": ops / (ms / 1e3) / 1e12, "unit": "TOPS", "us_per_call": ms * 1e3,
        "bit_exact_vs_oracle_sampled_rows": exact,
        "roofline": {"bound": "tensor", "kernel": "q2k_gemm_tc_kernel (+ operand prepass)",
                     "achieved": ops / (lms / 1e3) / 1e12, "peak": i8peak, "unit": "TOPS",
                     "frac": ops / (lms / 1e3) / 1e12 / i8peak,
                     "peak_kind": f"int8 dense taken as 2 x the {tkind} bf16 GEMM rate ({tpeak:.1f} TFLOP/s)",
                     "frac_of_bf16_peak": ops / (lms / 1e3) / 1e12 / tpeak,
                     "traffic": None, "ops_per_launch": ops, "median_launch_us": lms * 1e3},
        "cpu_baseline": cpu_baseline_pair(lambda n: O.q2k_mul_mat(w0, rows, k, xq_s, cs, n_threads=n), cpu_s,
                                          lambda sec: s_ops / sec / 1e12, "TOPS",
                                          f"the oracle's generic-C dot on {cs} of the 512 activation rows "
                                          "(same W), scaled per op"),
    }
    del mats
    torch.cuda.synchronize()
    return out


def stack_bytes_per_token(L, H, F, V):
    from smeai_b200.stack import gemv_bytes
    per_layer = gemv_bytes(3 * H, H, 1) + gemv_bytes(H, H, 1) + gemv_bytes(2 * F, H, 1, F) + gemv_bytes(H, F, 1)
    return L * per_layer + gemv_bytes(V, H, 1)


def run_reference(args):
    """The reference's CPU implementation of the path (the generic-C Q2_K x
    Q8_K dot, restated in oracle/) with every host thread, on bounded samples
    of the decode workload: each step times one full layer's GEMVs."""
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    from oracle import oracle as O
    O.build()
    O.select(native=True)            # the -march=native build of this host
    threads = os.cpu_count() or 1
    dims = dict(hidden=4096, ffn=11008, vocab=32000, n_layers=32)
    tok_bytes = stack_bytes_per_token(32, 4096, 11008, 32000)
    sample = CpuLayerSample(dims["hidden"], dims["ffn"], threads)
    for _ in range(args.warmup):
        sample.run_once()
    gbs = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        g, _, _ = sample.timed(1.0)
        gbs.append(g)
    wall = time.perf_counter() - t0
    value = statistics.median(gbs)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall / args.steps * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8xu2",
        "data": "synthetic", "tokens_per_s": value * 1e9 / tok_bytes,
        "config": {"workload": "llama2-7b-shape Q2_K linear stack decode, batch 1 (one layer per step)",
                   "global_batch": 1, "parallelism": f"cpu threads {threads}"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port",
                         "cpu_model": O.cpu_model(), "nproc": threads,
                         "build": "gcc -O3 -march=native -ffp-contract=off -fopenmp",
                         "sample": "each step: whole layers (qkv 12288x4096, o 4096x4096, gate+up 22016x4096, "
                                   "down 4096x11008 GEMVs, batch 1) repeated for ~1 s, generic-C Q2_KxQ8_K "
                                   "dot, OpenMP rows; random Q2_K blocks of the same shapes (the dot's work "
                                   "does not depend on the values)"},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def tensor_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def gemv_roofline(gemvs, stream, dev, peak, peak_kind):
    """Every GEMV of a step timed alone: events around each launch, queued
    behind a sleep kernel so launch gaps do not count; consecutive GEMVs read
    distinct weights, so nothing sits in L2."""
    import torch
    from smeai_b200 import q2k as Q
    from smeai_b200.stack import gemv_bytes
    per = {}
    with torch.cuda.stream(stream):
        xq_by_k = {}
        for name, m in gemvs:
            if m.k not in xq_by_k:
                xq_by_k[m.k] = Q.quantize_q8k(torch.randn((1, m.k), device=dev))
        outs = {name: torch.empty((1, m.n_rows), device=dev) for name, m in gemvs}
        evs = []
        torch.cuda._sleep(20_000_000)
        for name, m in gemvs:
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            m.mul_mat(xq_by_k[m.k], 1, out=outs[name])
            b.record(stream)
            evs.append((name, m, a, b))
    stream.synchronize()
    tot_b, tot_ms = 0, 0.0
    for name, m, a, b in evs:
        d = a.elapsed_time(b)
        extra = 110 - 84 if isinstance(m, Q.Q3KMatrix) else (210 - 84 if isinstance(m, Q.Q6KMatrix) else 0)
        nbytes = gemv_bytes(m.n_rows, m.k, 1) + m.n_rows * m.nb * extra
        agg = per.setdefault(name, [0, 0.0, 0])
        agg[0] += nbytes
        agg[1] += d
        agg[2] += 1
        tot_b += nbytes
        tot_ms += d
    achieved = tot_b / (tot_ms / 1e3) / 1e9
    ratio = traffic_ratio()
    launch_avg_bytes = tot_b / len(evs)
    return {"bound": "hbm", "kernel": "q2k_gemv_kernel", "achieved": achieved, "peak": peak,
            "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind,
            "traffic": (ratio * launch_avg_bytes) if ratio else None,
            "algorithmic_bytes_per_launch": launch_avg_bytes,
            "avg_launch_us": tot_ms / len(evs) * 1e3,
            "per_matrix": {n: {"GB/s": v[0] / (v[1] / 1e3) / 1e9, "us": v[1] / v[2] * 1e3, "launches": v[2]}
                           for n, v in per.items()}}


def program_roofline(stack, stream, peak, peak_kind, launches=8):
    """The persistent decode kernel timed per launch (events around each
    launch, queued behind a sleep kernel; one launch = one token, 2.17 GB of
    distinct weights, far more than L2)."""
    import torch
    evs = []
    with torch.cuda.stream(stream):
        stack.prog.run()
        torch.cuda._sleep(20_000_000)
        for _ in range(launches):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            stack.prog.run()
            b.record(stream)
            evs.append((a, b))
    stream.synchronize()
    ms = statistics.median(a.elapsed_time(b) for a, b in evs)
    nbytes = stack.algorithmic_bytes()
    achieved = nbytes / (ms / 1e3) / 1e9
    ratio = traffic_ratio("q2k_program_decode.txt")
    return {"bound": "hbm", "kernel": "q2k_program_kernel", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_kind": peak_kind,
            "traffic": (ratio * nbytes) if ratio else None, "algorithmic_bytes_per_launch": nbytes,
            "median_launch_us": ms * 1e3, "launches_timed": launches}


# ---------------------------------------------------------------------------- GPU side
def run_ours(args):
    import torch
    import torch.distributed as dist

    import smeai_b200 as S
    from smeai_b200 import q2k as Q
    from smeai_b200.stack import Q2KDecodeStack, gemv_bytes

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    S.lib()
    assert S.device_ready(), S.last_error()
    peak, peak_kind = hbm_peak()
    stream = torch.cuda.Stream(device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stack = None
    if args.workload in ("decode", "prefill-stack"):
        L, H, F, V = args.layers, 4096, 11008, 32000
        prefill_stack = args.workload == "prefill-stack"
        seq_shard = prefill_stack and world > 1 and args.prefill_shard == "tokens"
        if seq_shard:   # every rank: the full weights and its own tokens of the prefill
            from smeai_b200.stack import token_range
            tok = token_range(args.prefill_tokens, rank, world)
            stack = Q2KDecodeStack(n_layers=L, hidden=H, ffn=F, vocab=V, batch=args.prefill_tokens, tokens=tok,
                                   device=dev, seed=0, quant="tc")
        else:
            stack = Q2KDecodeStack(n_layers=L, hidden=H, ffn=F, vocab=V, batch=args.prefill_tokens if prefill_stack
                                   else args.decode_batch, rank=rank, world=world, device=dev, seed=0,
                                   quant="tc" if prefill_stack else args.quant)
        x_in = torch.empty_like(stack.x0)
        x_in.copy_(stack.x0)

        def step():
            return stack.step(x_in)

        launches_per_step = stack.launches_per_step()
        local_bytes = stack.algorithmic_bytes()
        h2d, d2h = x_in.numel() * 4, stack.logits.numel() * 4
        out_buf = stack.logits
        workload = (f"llama2-7b-shape Q2_K linear stack decode, batch {args.decode_batch}: {L} layers x "
                    "(qkv, o, gate+up, down)"
                    " + lm_head 32000x4096, RMSNorm+Q8_K re-quantization between linears")
        if prefill_stack:
            workload = (f"llama2-7b-shape Q2_K linear stack prefill, {args.prefill_tokens} tokens: {L} layers x "
                        "(qkv, o, gate+up, down) + lm_head 32000x4096 on the tcgen05 GEMM (residual and silu*mul "
                        "in its epilogue), RMSNorm+Q8_K between linears")
        gemvs = stack.gemv_list()
    else:
        rows, k, epi = args.gemv_rows, args.gemv_k, args.gemv_epilogue
        q3 = args.gemv_fmt in ("q3k", "q6k")          # the generic-path formats (store epilogue)
        blk_bytes = {"q2k": 84, "q3k": 110, "q6k": 210}[args.gemv_fmt]
        mbytes = rows * (k // 256) * blk_bytes
        copies = max(4, min(64, -(-4 * 126 * 2**20 // mbytes)))   # > 4x L2 of distinct weights
        g = torch.Generator(device=dev).manual_seed(0)
        if q3:
            # blocks of random bits with a small positive fp16 d (this library has no Q3_K /
            # Q6_K quantizer; the GEMV's work does not depend on the values)
            import numpy as np
            rng = np.random.default_rng(0)
            cls = Q.Q3KMatrix if args.gemv_fmt == "q3k" else Q.Q6KMatrix
            def q_blocks():
                b = rng.integers(0, 256, size=(rows * (k // 256), blk_bytes), dtype=np.uint8)
                d = (np.abs(rng.standard_normal(b.shape[0])) * 0.0005 + 1e-5).astype(np.float16)
                b[:, blk_bytes - 2:] = d.view(np.uint8).reshape(-1, 2)
                return torch.from_numpy(b.reshape(-1)).to(dev)
            mats = [cls(q_blocks(), rows, k) for _ in range(copies)]
            if epi != 0:
                raise SystemExit("--gemv-fmt q3k/q6k run the store epilogue only")
        else:
            mats = [Q.Q2KMatrix(Q.quantize_q2k(torch.randn((rows, k), generator=g, device=dev) * 0.02), rows, k)
                    for _ in range(copies)]
        x_in = torch.randn((1, k), generator=g, device=dev)
        xq = torch.empty((1, k // 256 * 292), dtype=torch.uint8, device=dev)
        out_rows = rows // 2 if epi == 2 else rows
        y = torch.zeros((1, out_rows), device=dev)
        it = {"i": 0}

        def step():
            m = mats[it["i"] % copies]
            it["i"] += 1
            Q.quantize_q8k(x_in, out=xq)
            if q3:
                m.mul_mat(xq, 1, out=y)
            else:
                m.mul_mat(xq, 1, out=y, epilogue=epi, resid=y if epi == 1 else None)
            return y

        launches_per_step = 2
        local_bytes = gemv_bytes(rows, k, 1, out_rows) + rows * (k // 256) * (blk_bytes - 84)
        h2d, d2h = k * 4, out_rows * 4
        out_buf = y
        workload = (f"{args.gemv_fmt.upper().replace('K', '_K')} x Q8_K GEMV W[{rows},{k}], x[{k}] ~N(0,1), epilogue {epi}, "
                    f"{copies} rotating weight copies ({copies * mbytes / 2**20:.0f} MB > L2)")
        gemvs = [("gemv", m) for m in mats]

    if args.workload == "prefill":
        # config 4: activations [512, 4096] (Q8_K per row) x W[11008, 4096] Q2_K -> [512, 11008]
        rows, k, cols = 11008, 4096, args.prefill_tokens
        mbytes = rows * (k // 256) * 84
        copies = max(2, min(48, -(-4 * 126 * 2**20 // mbytes)))
        g = torch.Generator(device=dev).manual_seed(0)
        mats = [Q.Q2KMatrix(Q.quantize_q2k(torch.randn((rows, k), generator=g, device=dev) * 0.02), rows, k)
                for _ in range(copies)]
        x_in = torch.randn((cols, k), generator=g, device=dev)
        xq = Q.quantize_q8k(x_in)
        y = torch.empty((cols, rows), device=dev)
        it = {"i": 0}

        def step():
            m = mats[it["i"] % copies]
            it["i"] += 1
            Q.quantize_q8k(x_in, out=xq)
            m.mul_mat_tc(xq, cols, out=y)
            return y

        launches_per_step = 4   # quantizer, operand prepass, GEMM (+ a memset of the operand padding)
        local_bytes = gemv_bytes(rows, k, cols)
        h2d, d2h = cols * k * 4, cols * rows * 4
        out_buf = y
        workload = (f"Q2_K prefill mul_mat: activations [{cols},{k}] ~N(0,1) (Q8_K per row) x W[{rows},{k}] "
                    f"~N(0,0.02) Q2_K -> fp32 [{cols},{rows}] on tcgen05; {copies} rotating weight copies")
        gemvs = []
        prefill_ops = 2 * rows * k * cols

    total_bytes = local_bytes * world

    # ---- warm-up, then capture into a CUDA graph: one step (decode) or one
    # pass over every rotating weight copy (gemv; a step is then one GEMV)
    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    barrier()
    steps_per_replay = {"decode": 1, "prefill-stack": 1, "gemv": len(gemvs),
                        "prefill": len(mats) if args.workload == "prefill" else 0}[args.workload]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(steps_per_replay):
            step()
    torch.cuda.synchronize()

    def run():
        with torch.cuda.stream(stream):
            graph.replay()

    use_graph = True
    for _ in range(max(3, args.warmup)):
        run()
    torch.cuda.synchronize()
    barrier()

    # ---- timed region: K steps, device time with CUDA events
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            run()
    e1.record(stream)
    e1.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / (args.steps * steps_per_replay)
    clocks = sampler.stop()
    ms = max_over_ranks(ms)
    value = total_bytes / (ms / 1e3) / 1e9
    code = S.take_device_error()
    if code:  # a bounded wait gave up (a kernel or a peer never arrived): the timing is void
        raise S.SmeaiError(f"device error word {code:#x} set during the timed steps")

    # ---- end to end: pinned host input -> H2D -> step -> D2H of the result
    host_x = torch.empty(x_in.shape, dtype=torch.float32, pin_memory=True)
    host_x.copy_(x_in.cpu())
    host_out = torch.empty(out_buf.shape, dtype=torch.float32, pin_memory=True)
    # one CUDA graph per step holding the H2D copy of the input, the step and
    # the D2H copy of the result (the copies stay inside the timed region;
    # only their separate launches go); three separate enqueues if capture fails
    e2e_graph = None
    nccl_in_step = world > 1 and not (stack is not None and (stack.quant == "mgprog" or stack.world == 1))
    if use_graph and not nccl_in_step:
        try:
            g2 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g2, stream=stream):
                x_in.copy_(host_x, non_blocking=True)
                for _ in range(steps_per_replay):
                    step()
                host_out.copy_(out_buf, non_blocking=True)
            e2e_graph = g2
        except Exception:
            torch.cuda.synchronize()
            e2e_graph = None

    def e2e_step():
        with torch.cuda.stream(stream):
            if e2e_graph is not None:
                e2e_graph.replay()
            else:
                x_in.copy_(host_x, non_blocking=True)
                run()
                host_out.copy_(out_buf, non_blocking=True)
        stream.synchronize()

    for _ in range(2):
        e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_ms = (time.perf_counter() - t0) / (args.steps * steps_per_replay) * 1e3
    barrier()
    e2e_ms = max_over_ranks(e2e_ms)
    e2e_value = total_bytes / (e2e_ms / 1e3) / 1e9

    if args.workload == "prefill":
        # roofline of the GEMM kernel: events around each launch (distinct weights)
        evs = []
        with torch.cuda.stream(stream):
            torch.cuda._sleep(20_000_000)
            for m in mats[:8]:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                m.mul_mat_tc(xq, cols, out=y)
                b.record(stream)
                evs.append((a, b))
        stream.synchronize()
        gemm_ms = sorted(a.elapsed_time(b) for a, b in evs)[len(evs) // 2]
        tpeak, tkind = tensor_peak()
        achieved = prefill_ops / (gemm_ms / 1e3) / 1e12
        roofline = {"bound": "tensor", "kernel": "q2k_gemm_tc_kernel (+ operand prepass)", "achieved": achieved,
                    "peak": tpeak, "unit": "TFLOP/s", "frac": achieved / tpeak, "peak_kind": tkind,
                    "traffic": None, "ops_per_launch": prefill_ops, "median_launch_us": gemm_ms * 1e3,
                    "note": "fp16 tensor-core MMAs on exact integer operands; peak is the measured dense bf16 "
                            "GEMM rate (same tensor throughput as fp16)"}
    # ---- roofline of the dominant kernel: every GEMV of a step timed alone
    # (events around each launch, queued behind a sleep so launch gaps do not
    # count; consecutive GEMVs read distinct weights, so nothing sits in L2)
    if args.workload == "prefill-stack":
        # every GEMM of the step on the tensor cores: this rank's ops per step
        # over the device step time, against the int8 dense rate (2 x the
        # measured bf16 GEMM rate)
        tpeak, tkind = tensor_peak()
        rank_ops = stack.ops_per_step()
        achieved = rank_ops / (ms / 1e3) / 1e12
        roofline = {"bound": "tensor", "kernel": "q2k_gemm_tc_kernel (the step's GEMMs)", "achieved": achieved,
                    "peak": 2 * tpeak, "unit": "TOPS", "frac": achieved / (2 * tpeak),
                    "peak_kind": f"int8 dense taken as 2 x the {tkind} bf16 GEMM rate ({tpeak:.1f} TFLOP/s)",
                    "traffic": None, "ops_per_step_per_rank": rank_ops}
    elif args.workload == "decode" and stack.quant in ("program", "mgprog"):
        roofline = program_roofline(stack, stream, peak, peak_kind)
        roofline["gemv_per_launch"] = gemv_roofline(gemvs, stream, dev, peak, peak_kind)
    elif gemvs:
        roofline = gemv_roofline(gemvs, stream, dev, peak, peak_kind)

    # ---- CPU baseline (rank 0, one GPU only): one thread and every host
    # thread, the oracle built with -march=native on this host
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sample = CpuLayerSample(4096, 11008, 1)
        cpu = cpu_baseline_pair(lambda n: sample.run_once(n), args.cpu_seconds / 2,
                                lambda sec: sample.layer_bytes / sec / 1e9, "GB/s",
                                "whole decode layers (qkv 12288x4096, o 4096x4096, gate+up 22016x4096, down "
                                "4096x11008 GEMVs, batch 1) repeated for the sample time through the oracle's "
                                "generic-C Q2_KxQ8_K dot; random Q2_K blocks of the same shapes (the dot's work "
                                "does not depend on the values)")
    configs = None
    if rank == 0 and world == 1 and args.workload == "decode" and not args.no_configs:
        configs = run_configs(dev, stream, args, peak, peak_kind)

    unit = "GB/s"
    if args.workload == "prefill-stack":   # tokens of the (row-sharded) prefill per second
        value, e2e_value, unit = args.prefill_tokens / (ms / 1e3), args.prefill_tokens / (e2e_ms / 1e3), "tokens/s"
    if rank == 0:
        if args.workload == "prefill-stack":
            parallel = ("single GPU" if world == 1 else
                        f"sequence-shard sp{world}: each rank runs {stack.B} of the {args.prefill_tokens} tokens "
                        "through the full weights, no data-path collective (tokens are independent through this "
                        "linear stack; an attention layer would add a K/V all-gather)" if seq_shard else
                        f"row-shard tp{world}, NCCL all-gathers of the output slices")
        elif args.workload == "decode":
            parallel = (f"row-shard tp{world}, " + {
                "peer": "all-gather fused into each GEMV (NVLink peer stores + signals)",
                "mgprog": "one persistent kernel per rank; every finished row stored into every rank's copy of the "
                          "phase's output over NVLink peer memory (tagged words, no collective library)"}.get(
                stack.quant, "NCCL all-gathers")) if world > 1 else "single GPU"
        else:
            parallel = f"{world} independent replicas (each GPU runs the whole workload)" if world > 1 \
                else "single GPU"
        line = {
            "metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if args.workload in ("decode", "prefill-stack") else "weak",
            "vs_baseline": None, "dtype": "int8xu2", "data": "synthetic",
            "tokens_per_s": (args.decode_batch * 1e3 / ms) if args.workload == "decode" else
            ((args.prefill_tokens * 1e3 / ms) if args.workload in ("prefill", "prefill-stack") else None),
            "pct_of_hbm_peak": (value / (peak * world) * 100) if unit == "GB/s" else None,
            "config": {"workload": workload,
                       "global_batch": args.prefill_tokens if args.workload in ("prefill", "prefill-stack")
                       else (args.decode_batch if args.workload == "decode" else 1),
                       "seq_len": 1, "parallelism": parallel,
                       "l2": "inputs larger than L2 (2.17 GB of weights per step)"
                       if args.workload in ("decode", "prefill-stack")
                       else "inputs larger than L2 (rotating distinct weight copies)",
                       **({"tops": stack.ops_per_step() * world / (ms / 1e3) / 1e12}
                          if args.workload == "prefill-stack" else {}),
                       **({"prefill_ops_per_step": prefill_ops, "tops": prefill_ops / (ms / 1e3) / 1e12}
                          if args.workload == "prefill" else {}),
                       "cuda_graph": use_graph, "pdl": os.environ.get("SMEAI_PDL", "1") != "0",
                       "q8k_placement": stack.quant if stack is not None else args.quant},
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms,
                    "copies": "pinned host -> device input and device -> pinned host result every step, "
                              + ("captured with the step in one CUDA graph" if e2e_graph is not None
                                 else "enqueued around the step's graph")},
            "gpu_launches": launches_per_step * args.steps * steps_per_replay,
            "roofline": roofline,
            "cpu_baseline": cpu,
        }
        if configs:
            line["configs"] = configs
        print(json.dumps(line), flush=True)
    if graph is not None:
        del graph
    if e2e_graph is not None:
        del e2e_graph
    barrier()
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_attention(args):
    """--workload attention: one step = one causal self-attention of
    args.attn_seq tokens through sme_ai_self_attention_packed_f16f32_device
    (four packed projections + the score/softmax/weighted-sum kernel) on
    device-resident data; e2e = the reference-facing synchronous entry point
    with host buffers.  N GPUs run N independent replicas."""
    import ctypes

    import numpy as np
    import torch
    import torch.distributed as dist

    import smeai_b200 as S

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    L = S.lib()
    assert S.device_ready(), S.last_error()
    Sq, D, H = args.attn_seq, args.attn_dim, args.attn_heads
    hd = D // H
    P = ctypes.c_void_p
    rng = np.random.default_rng(1234)
    f16 = lambda n, sc: (rng.standard_normal(n) * sc).astype(np.float16).view(np.uint16)
    x16 = f16(Sq * D, 1.0)
    w16 = [f16(D * D, D ** -0.5) for _ in range(4)]
    b32 = [(rng.standard_normal(D) * 0.02).astype(np.float32) for _ in range(4)]
    ws = S.Workspace()
    assert L.sme_ai_workspace_init(ctypes.byref(ws), Sq, D, D) == 0, S.last_error()
    pws = []
    for w in w16:
        pw = S.PackedWeight()
        assert L.sme_ai_packed_linear_weight_init(ctypes.byref(pw), P(w.ctypes.data), D, D) == 0, S.last_error()
        pws.append(pw)
    xd = torch.from_numpy(x16).to(dev)
    bd = [torch.from_numpy(b).to(dev) for b in b32]
    od = torch.empty(Sq * D, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    d = lambda t: P(t.data_ptr())

    def step():
        r = L.sme_ai_self_attention_packed_f16f32_device(
            ctypes.byref(ws), d(xd), Sq, D, H, ctypes.byref(pws[0]), d(bd[0]), ctypes.byref(pws[1]), d(bd[1]),
            ctypes.byref(pws[2]), d(bd[2]), ctypes.byref(pws[3]), d(bd[3]), 1, d(od), P(stream.cuda_stream))
        assert r == 0, S.last_error()

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(max(3, args.warmup)):
        step()
    stream.synchronize()
    barrier()
    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.3)
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    e1.synchronize()
    barrier()
    ms = e0.elapsed_time(e1) / args.steps
    clocks = sampler.stop()
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * Sq / (ms / 1e3)

    # the core kernel alone (events on its stream; Q/K/V from the last step)
    qd = torch.empty(Sq * D, dtype=torch.float32, device=dev)
    kd, vd = torch.empty_like(qd), torch.empty_like(qd)
    for t in (qd, kd, vd):
        t.normal_()
    cd = torch.empty(Sq * D, dtype=torch.float16, device=dev)
    evs = []
    with torch.cuda.stream(stream):
        torch.cuda._sleep(20_000_000)
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            assert L.sme_ai_self_attention_core_f32_device(d(qd), d(kd), d(vd), Sq, D, H, 1, d(cd),
                                                           P(stream.cuda_stream)) == 0, S.last_error()
            b.record(stream)
            evs.append((a, b))
    stream.synchronize()
    core_ms = sorted(a.elapsed_time(b) for a, b in evs)[len(evs) // 2]
    pairs = Sq * (Sq + 1) // 2                    # (i, j <= i) score / weight pairs per head
    core_flops = 4 * hd * pairs * H               # QK^T fma + (mul, add) of the weighted sum
    proj_flops = 4 * 2 * Sq * D * D
    fp32_peak = 148 * 128 * 2 * 1.965e9 / 1e12   # nominal FP32 CUDA-core rate at the max clock
    achieved = core_flops / (core_ms / 1e3) / 1e12
    roofline = {"bound": "fp32", "kernel": "attention_kernel (scores + softmax + weighted sum)",
                "achieved": achieved, "peak": fp32_peak, "unit": "TFLOP/s", "frac": achieved / fp32_peak,
                "peak_kind": "nominal (no measured fp32 CUDA-core peak on this pool)", "traffic": None,
                "flops_per_launch": core_flops, "median_launch_us": core_ms * 1e3,
                "core_share_of_step": core_ms / ms, "projection_flops_per_step": proj_flops}

    # e2e: the synchronous reference-facing call with host buffers
    out_h = np.zeros(Sq * D, np.float32)
    pp = lambda a: P(a.ctypes.data)

    def e2e_step():
        r = L.sme_ai_self_attention_sme_packed_f16f32(
            ctypes.byref(ws), pp(x16), Sq, D, H, ctypes.byref(pws[0]), pp(b32[0]), ctypes.byref(pws[1]),
            pp(b32[1]), ctypes.byref(pws[2]), pp(b32[2]), ctypes.byref(pws[3]), pp(b32[3]), 1, pp(out_h))
        assert r == 0, S.last_error()

    e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_ms = (time.perf_counter() - t0) / args.steps * 1e3
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        O.build()
        cs = 8
        t0, reps = time.perf_counter(), 0
        while True:
            O.self_attention_f16f32(x16[:cs * D], cs, D, H, *[a for pair in zip(w16, b32) for a in pair], 1)
            reps += 1
            if time.perf_counter() - t0 >= min(args.cpu_seconds, 30.0):
                break
        per = (time.perf_counter() - t0) / reps
        cpu = {"value": cs / per, "unit": "tokens/s", "cores": 1, "kind": "port",
               "sample": f"{reps} x the oracle's self-attention (the reference's ref path restated in scalar C, "
                         f"its Linear's column-strided weight reads included) on the first {cs} tokens at "
                         f"model_dim {D}, {H} heads, causal; {per * 1e3:.0f} ms each"}
    for pw in pws:
        L.sme_ai_packed_linear_weight_destroy(ctypes.byref(pw))
    L.sme_ai_workspace_destroy(ctypes.byref(ws))
    if rank == 0:
        line = {
            "metric": "self-attention (packed, causal) tokens/s", "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16xf32",
            "data": "synthetic",
            "config": {"workload": f"causal self-attention, {Sq} tokens, model_dim {D}, {H} heads (head_dim {hd}); "
                                   "fp16 packed weights ~N(0, 1/D), fp16 input ~N(0,1)",
                       "global_batch": world * Sq, "seq_len": Sq, "parallelism": f"{world} replicas",
                       "l2": "inputs larger than L2: a step touches 4 x 32 MB of fp16 weights, the 16 MB input "
                             "and 3 x 32 MB of fp32 Q/K/V plus the output (~270 MB > 126 MB)"},
            "clocks": clocks,
            "e2e": {"value": world * Sq / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": Sq * D * 2 + 4 * D * 4,
                    "d2h_bytes_per_step": Sq * D * 4, "ms_per_step": e2e_ms},
            "gpu_launches": 5 * args.steps,
            "roofline": roofline,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    barrier()
    if world > 1:
        dist.destroy_process_group()
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.workload == "attention":
        return run_attention(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
