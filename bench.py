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
    ap.add_argument("--workload", choices=["decode", "gemv", "prefill", "attention"], default="decode")
    ap.add_argument("--attn-seq", type=int, default=2048, help="attention workload: tokens")
    ap.add_argument("--attn-dim", type=int, default=4096, help="attention workload: model_dim")
    ap.add_argument("--attn-heads", type=int, default=32, help="attention workload: heads")
    ap.add_argument("--prefill-tokens", type=int, default=512, help="prefill workload: activation rows")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--quant", choices=["fused", "separate", "mixed", "program"], default="program",
                    help="decode: 'program' (default) runs the whole step as one persistent kernel on one GPU; "
                         "the others launch one GEMV per linear with the Q8_K quantization fused, separate or "
                         "mixed (all give identical results; N > 1 GPUs always launch per linear)")
    ap.add_argument("--gemv-rows", type=int, default=4096, help="gemv workload: weight rows")
    ap.add_argument("--gemv-k", type=int, default=4096, help="gemv workload: row length")
    ap.add_argument("--gemv-epilogue", type=int, default=0, help="gemv workload: 0 store, 1 residual, 2 silu*mul")
    ap.add_argument("--gemv-fmt", choices=["q2k", "q3k", "q6k"], default="q2k", help="gemv workload: weight format")
    ap.add_argument("--no-cpu-baseline", action="store_true")
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
    the host's cores with OpenMP.  Weights are valid random Q2_K blocks with
    the magnitudes of quantized N(0, 0.02) draws (the CPU work does not
    depend on the values); activations are Q8_K of N(0, 1)."""

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

    def run_once(self):
        for (r, k), w in zip(self.mats, self.ws):
            self.O.q2k_mul_mat(w, r, k, self.xs[k], 1, n_threads=self.threads)

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
                         "sample": "each step: whole layers (qkv 12288x4096, o 4096x4096, gate+up 22016x4096, "
                                   "down 4096x11008 GEMVs, batch 1) repeated for ~1 s, generic-C Q2_KxQ8_K "
                                   "dot, OpenMP rows"},
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

    if args.workload == "decode":
        L, H, F, V = args.layers, 4096, 11008, 32000
        stack = Q2KDecodeStack(n_layers=L, hidden=H, ffn=F, vocab=V, batch=1, rank=rank, world=world,
                               device=dev, seed=0, quant=args.quant)
        x_in = torch.empty_like(stack.x0)
        x_in.copy_(stack.x0)

        def step():
            return stack.step(x_in)

        launches_per_step = stack.launches_per_step()
        local_bytes = stack.algorithmic_bytes()
        h2d, d2h = x_in.numel() * 4, stack.logits.numel() * 4
        out_buf = stack.logits
        workload = (f"llama2-7b-shape Q2_K linear stack decode, batch 1: {L} layers x (qkv, o, gate+up, down)"
                    " + lm_head 32000x4096, RMSNorm+Q8_K re-quantization between linears")
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
    steps_per_replay = {"decode": 1, "gemv": len(gemvs), "prefill": len(mats) if args.workload == "prefill"
                        else 0}[args.workload]
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
    def e2e_step():
        with torch.cuda.stream(stream):
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
    if args.workload == "decode" and stack.quant == "program":
        roofline = program_roofline(stack, stream, peak, peak_kind)
        roofline["gemv_per_launch"] = gemv_roofline(gemvs, stream, dev, peak, peak_kind)
    elif gemvs:
        roofline = gemv_roofline(gemvs, stream, dev, peak, peak_kind)

    # ---- CPU baseline (rank 0, one GPU only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        sample = CpuLayerSample(4096, 11008, threads)
        sample.run_once()
        gbs, per_layer, reps = sample.timed(args.cpu_seconds)
        cpu = {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{reps} x one full decode layer (qkv, o, gate+up, down GEMVs, batch 1) through the "
                         f"oracle's generic-C Q2_KxQ8_K dot, {per_layer * 1e3:.1f} ms per layer"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8xu2", "data": "synthetic",
            "tokens_per_s": (1e3 / ms) if args.workload == "decode" else
            ((args.prefill_tokens * 1e3 / ms) if args.workload == "prefill" else None),
            "pct_of_hbm_peak": value / (peak * world) * 100,
            "config": {"workload": workload,
                       "global_batch": args.prefill_tokens if args.workload == "prefill" else 1, "seq_len": 1,
                       "parallelism": (f"row-shard tp{world}, " + ("all-gather fused into each GEMV (NVLink "
                                       "peer stores + signals)" if stack.quant == "peer" else "NCCL all-gather")
                                       if args.workload == "decode" else f"row-shard tp{world}")
                       if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (2.17 GB of weights per step)" if args.workload == "decode"
                       else "inputs larger than L2 (rotating distinct weight copies)",
                       **({"prefill_ops_per_step": prefill_ops, "tops": prefill_ops / (ms / 1e3) / 1e12}
                          if args.workload == "prefill" else {}),
                       "cuda_graph": use_graph, "pdl": os.environ.get("SMEAI_PDL", "1") != "0",
                       "q8k_placement": stack.quant if args.workload == "decode" else args.quant},
            "clocks": clocks,
            "e2e": {"value": e2e_value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": e2e_ms},
            "gpu_launches": launches_per_step * args.steps * steps_per_replay,
            "roofline": roofline,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if graph is not None:
        del graph
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
