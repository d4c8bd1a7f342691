#!/usr/bin/env python
"""Throughput benchmark of the Q8 greedy translation path on B200.

Metric: target tokens/s (greedy, EOS masked until round(1.2 x src) so the work
is fixed), whole job over all GPUs.  Workload per step (BASELINE config 4 as
a capacity measurement): 20,000 requests with lognormal(ln 24, 0.8) source
lengths clipped to 4..256 tokens (EOS included), Zipf(1.1) ids, all queued at
once and served by the continuous batcher (1024 decode slots, 16-token KV
pages) on the benchmark model shape (d=512, 8 heads, 6 encoder layers, 2
self+cross-attention decoder layers, FFN 2048, vocabulary 32000, random
init, seed 0).  Each rank owns a full model replica and its own request
stream (request-sharded; no collective on the data path).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl cuda|reference]

The same JSON line also carries, unless --no-configs:
  * config3_encoder -- config 3: packed encoder passes over 256 lognormal
    sentences each (mc_encode_token_ids): source tokens/s, encoder attention
    GB/s and GEMM TOP/s against the measured peaks, and the CPU port's
    encoder rate;
  * config5_longtext -- config 5 as strong scaling: one fixed global set of
    --longtext-docs documents of 200..2,000 Zipf(1.1) tokens with a
    pseudo-sentence end every 8..64 tokens, split by the library's
    segment_text into segments of at most 128 tokens with EOS, sorted by
    length and dealt round-robin over the N replicas;
  * config2_gemm -- config 2: the Q8 GEMM operator over (K, N) in
    {(512, 1536), (512, 2048), (2048, 512), (512, 32000)} x M in
    {1, 7, 64, 333, 1024, 4096}, microseconds per launch back to back with
    operands from HBM, against the int8 tensor rate (M >= 64) or the HBM
    copy rate (weight streaming, M <= 7);
  * latency_ms -- config 4's latency: 20,000 requests replayed with Poisson
    arrivals at 2,000 req/s, and again near capacity, by the library's own
    arrival loop (mc_replay), p50/p99 from arrival to last token.

`--workload longtext` makes the long-text stream the step workload instead
(weak scaling: --docs documents per GPU).

The reference arm times the CPU restatement of marian-edge's Q8 engine (the
Rust reference cannot be built on this image) on the host cores.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "marian-edge_b200"))

from marian_cuda import workloads as W  # noqa: E402

METRIC = "target tokens/sec per box (greedy)"
UNIT = "tokens/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="cuda", choices=["cuda", "reference"])
    p.add_argument("--model", default="graph_b", choices=list(W.SHAPES))
    p.add_argument("--requests", type=int, default=20000, help="requests per step per GPU")
    p.add_argument("--max-inflight", type=int, default=1024)
    p.add_argument("--lanes", type=int, default=0, help="decode lanes (0: library default)")
    p.add_argument("--cpu-seconds", type=float, default=15.0, help="CPU baseline sample budget")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-latency", action="store_true")
    p.add_argument("--no-configs", action="store_true", help="skip the config 2, 3 and 5 lines")
    p.add_argument("--workload", default="stream", choices=["stream", "longtext"])
    p.add_argument("--docs", type=int, default=500, help="longtext workload: documents per GPU per step")
    p.add_argument("--longtext-docs", type=int, default=400, help="config 5: global documents")
    p.add_argument("--encoder-batches", type=int, default=16, help="config 3: timed 256-sentence passes")
    p.add_argument("--capacity-rate", type=float, default=40000.0, help="near-capacity arrival rate")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def config_dict(args, world):
    if args.workload == "longtext":
        workload = ("long-text stream: %d documents/GPU/step of 200..2000 Zipf(1.1) tokens, pseudo-sentence "
                    "every 8..64 tokens, split by segment_text into segments <= 128 tokens, dealt round-robin "
                    "by length over %d replica(s), out=round(1.2*src) EOS-masked" % (args.docs, world))
    else:
        workload = ("continuous-batching stream: %d requests/GPU/step, lognormal(ln24,0.8) src "
                    "4..256 tok, Zipf(1.1) ids, out=round(1.2*src) EOS-masked; value is capacity with "
                    "every request queued at the step's start (config 4's Poisson arrivals are replayed "
                    "separately in latency_ms)" % args.requests)
    return {"workload": workload,
            "model_shape": args.model, "d_model": W.SHAPES[args.model].dim,
            "decoder": W.SHAPES[args.model].decoder_kind, "max_inflight": args.max_inflight,
            "page_tokens": 16, "parallelism": "replica x%d (request-sharded)" % world,
            "l2": "no flush: each step streams > 1 GB of KV-cache pages and activations (L2 is 126 MB)"}


def step_batches(args, rank, count, base_seed, world=1):
    vocab = W.SHAPES[args.model].vocab
    if args.workload == "longtext":
        # one document set per call, dealt over the replicas; every step
        # repeats it (the engine keeps nothing between steps)
        b = W.longtext_batch(args.docs * world, vocab=vocab, seed=base_seed, rank=rank, world=world)
        return [b] * count
    return [W.stream_batch(n=args.requests, vocab=vocab, seed=base_seed + 7919 * rank + s) for s in range(count)]


# ---- clocks sampler ------------------------------------------------------------
class Clocks:
    def __init__(self, device):
        self.device = device
        self.samples = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), "--query-gpu=clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            for line in out.strip().splitlines():
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 7:
                    self.samples.append(parts)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4) if s[3 + i].lower() == "active"})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


# ---- CPU side (oracle) ---------------------------------------------------------
def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def host_cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    return O


def cpu_sample(model_bytes, batches, seconds, threads, encoder_only=False):
    """Time the CPU restatement of the reference's Q8 engine on host threads.

    Each thread is one engine worker (the reference's worker pool,
    marian-core/src/scheduler.rs:179-226) translating reference-legal batches
    (B <= 256, B*Lmax^2 <= 65536, first fit, marian-cpu/src/backend.rs:223-243)
    of the same request distribution until the time budget is spent.  With
    encoder_only, every row stops after one token (the encoder pass and one
    decode step); the rate counted is then source tokens.
    Returns (rate, requests, counted tokens, seconds).
    """
    O = _oracle()
    om = O.OracleModel(model_bytes)
    work = []
    for b in batches:
        for g in W.legal_cpu_batches(b):
            sb = W.subset(b, g)
            if encoder_only:
                sb.max_out[:] = 1
                sb.force_len[:] = 1
            work.append(sb)
    lock = threading.Lock()
    state = {"next": 0, "tokens": 0, "requests": 0}
    deadline = time.perf_counter() + seconds

    def worker():
        while time.perf_counter() < deadline:
            with lock:
                i = state["next"]
                state["next"] += 1
            if i >= len(work):
                return
            sb = work[i]
            toks, offs = om.translate(sb.tokens, sb.offsets, sb.max_out, sb.force_len)
            n = int(sb.offsets[-1]) if encoder_only else int(offs[-1])
            with lock:
                state["tokens"] += n
                state["requests"] += sb.size
    t0 = time.perf_counter()
    ts = [threading.Thread(target=worker) for _ in range(threads)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    el = time.perf_counter() - t0
    return state["tokens"] / el, state["requests"], state["tokens"], el


def cpu_baseline_obj(rate, reqs, toks, secs, threads, what, unit=UNIT):
    return {"value": rate, "unit": unit, "cores": threads, "cpu_model": host_cpu_model(), "kind": "port",
            "sample": f"{reqs} requests ({toks} {what}) in {secs:.1f} s, reference-legal CPU batches "
                      f"(B<=256, B*Lmax^2<=65536), {threads} worker threads, AVX2 integer GEMM"}


# ---- reference arm ---------------------------------------------------------------
def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    model_bytes = W.synthetic_model(W.SHAPES[args.model], seed=0)
    threads = host_threads()
    per_step = max(2.0, args.cpu_seconds / max(1, args.steps))
    batches = step_batches(args, 0, 1, 1000)
    for _ in range(args.warmup):
        cpu_sample(model_bytes, batches, 0.5, threads)
    reqs, toks, secs = 0, 0, 0.0
    for _ in range(args.steps):
        _, r, t, s = cpu_sample(model_bytes, batches, per_step, threads)
        reqs += r
        toks += t
        secs += s
    value = toks / secs if secs else 0.0
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * secs / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "s8xs8->s32, f32",
            "data": "synthetic (seeded random-init model and token streams)",
            "config": config_dict(args, 1),
            "cpu_baseline": cpu_baseline_obj(value, reqs, toks, secs, threads, "target tokens"),
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---- CUDA arm --------------------------------------------------------------------
def reduce_job(tokens, dev_ms, wall_s, world, device):
    """Whole-job totals over the ranks: tokens summed, device time and wall
    time as the max over ranks (the job ends when its slowest rank does)."""
    if world == 1:
        return float(tokens), float(dev_ms), float(wall_s)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(tokens)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    m = torch.tensor([float(dev_ms), float(wall_s)], dtype=torch.float64, device=device)
    dist.all_reduce(m, op=dist.ReduceOp.MAX)
    return float(t.item()), float(m[0].item()), float(m[1].item())


# DRAM traffic per algorithmic byte, from one ncu --set full capture of each
# kernel class on the benchmark stream (2,048-request run; launches and
# figures in profiles/: dram__bytes_read.sum + dram__bytes_write.sum divided
# by the engine's algorithmic byte count for the same launch).  The bench
# scales it to its own launches; classes without a capture report null.
DRAM_PER_ALGO_BYTE = {
    "attn_cross": 231.5 / 223.8,   # 1,024 rows, 54,009 keys, tail boxes of 4/2/1 rows
    "attn_self": 231.5 / 223.8,    # same kernel and page layout
    "gemm_vocab": 17.12 / 17.17,   # M=1,024, N=32,000, K=512, weight-stationary
    "gemm_ln": 12.54 / 24.43,      # one layer's three fused launches, 1,024 rows, d=512
    "layernorm": 4.24 / 6.82,      # 1,024 rows; outputs still in L2 at exit
}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def read_profile(lib, eng, L):
    prof = {}
    for k, name in enumerate(L.KERNEL_KINDS):
        n, ms, fl, by = C.c_uint64(), C.c_double(), C.c_double(), C.c_double()
        lib.mc_profile_read(eng.handle, k, C.byref(n), C.byref(ms), C.byref(fl), C.byref(by))
        if n.value:
            prof[name] = {"launches": n.value, "ms": ms.value, "flops": fl.value, "bytes": by.value}
    return prof


def class_roofline(name, r, peaks, peak_kind):
    """Roofline object of one kernel class from its profile record."""
    per_launch_s = r["ms"] / 1000.0 / r["launches"]
    if name.startswith("gemm"):
        peak = 2.0 * peaks["bf16_tflops"]  # dense int8 tensor rate = 2 x bf16
        achieved = r["flops"] / r["launches"] / per_launch_s / 1e12
        out = {"kernel": name, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TOP/s",
               "frac": achieved / peak, "peak_source": f"2 x {peak_kind} bf16 dense TFLOP/s (int8 rate is twice bf16)"}
    else:
        peak = peaks["hbm_gbs"]
        achieved = r["bytes"] / r["launches"] / per_launch_s / 1e9
        out = {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
               "frac": achieved / peak, "peak_source": f"{peak_kind} HBM copy GB/s"}
    ratio = DRAM_PER_ALGO_BYTE.get(name)
    out["traffic"] = (ratio * r["bytes"] / r["launches"]) if ratio else None
    out["traffic_unit"] = "bytes per launch (ncu DRAM bytes per algorithmic byte x algorithmic bytes)"
    out["algorithmic_bytes_per_launch"] = r["bytes"] / r["launches"]
    out["avg_launch_us"] = per_launch_s * 1e6
    return out


def measure_encoder(args, eng, lib, L, model_bytes, peaks, peak_kind, rank, world):
    """Config 3: packed encoder passes over 256 lognormal sentences."""
    vocab = W.SHAPES[args.model].vocab
    batches = [W.stream_batch(n=256, vocab=vocab, seed=31000 + 101 * rank + i)
               for i in range(args.encoder_batches + 3)]
    for b in batches[:3]:
        eng.encode_token_ids(b.tokens, b.offsets)
    lib.mc_profile(eng.handle, 1)
    eng.encode_token_ids(batches[0].tokens, batches[0].offsets)
    prof = read_profile(lib, eng, L)
    lib.mc_profile(eng.handle, 0)
    timed = batches[3:]
    src = sum(int(b.offsets[-1]) for b in timed)
    t0 = time.perf_counter()
    for b in timed:
        eng.encode_token_ids(b.tokens, b.offsets)
    wall = time.perf_counter() - t0
    out = {"workload": "config 3: %d packed encoder passes of 256 sentences, lognormal(ln24,0.8) src 4..256 "
                       "tok, Zipf(1.1) ids (mc_encode_token_ids, host buffers in, cross K/V written)"
                       % len(timed),
           "value": src / wall, "unit": "source tokens/s", "ms_per_pass": 1000.0 * wall / len(timed),
           "mean_source_tokens_per_pass": src / len(timed),
           "device_ms_per_pass_profiled": sum(v["ms"] for v in prof.values()),
           "kernel_profile": prof}
    if prof:
        dom = max(prof.items(), key=lambda kv: kv[1]["ms"])
        out["roofline"] = class_roofline(dom[0], dom[1], peaks, peak_kind)
        if "attn_enc" in prof:
            out["attn_enc"] = class_roofline("attn_enc", prof["attn_enc"], peaks, peak_kind)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        v, reqs, toks, secs = cpu_sample(model_bytes, timed[:2], 6.0, threads, encoder_only=True)
        out["cpu_baseline"] = cpu_baseline_obj(v, reqs, toks, secs, threads,
                                               "source tokens, encoder + one decode step",
                                               unit="source tokens/s")
    return out


GEMM_SHAPES = [(512, 1536), (512, 2048), (2048, 512), (512, 32000)]  # (K, N)
GEMM_ROWS = [1, 7, 64, 333, 1024, 4096]
L2_BYTES = 126 << 20


def measure_gemm(lib, peaks, peak_kind, iters=20):
    """Config 2: the Q8 GEMM operator (mc_q8_gemm, f32 epilogue with per-row
    and per-column scales and a bias) over the (K, N) x M grid.  Weights and
    activations cycle through copies totalling more than twice the L2, so
    every timed launch reads its operands from HBM.  A spin kernel ahead of
    the timed launches keeps the stream busy while the host enqueues them,
    so CUDA events around `iters` launches time them back to back on the
    device rather than the host's call rate."""
    import torch
    dev = torch.device("cuda")
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    gen = torch.Generator(device=dev)
    gen.manual_seed(2)
    points = []
    for k, n in GEMM_SHAPES:
        nw = max(2, -(-2 * L2_BYTES // (n * k)))
        w = torch.randint(-127, 128, (nw, n, k), dtype=torch.int8, device=dev, generator=gen)
        col_scale = torch.rand(n, device=dev, generator=gen) * 0.019 + 0.001
        bias = torch.rand(n, device=dev, generator=gen) * 0.2 - 0.1
        for m in GEMM_ROWS:
            na = max(2, -(-2 * L2_BYTES // (m * k)))
            a = torch.randint(-127, 128, (na, m, k), dtype=torch.int8, device=dev, generator=gen)
            row_scale = torch.rand(m, device=dev, generator=gen) * 0.019 + 0.001
            out = torch.empty((m, n), dtype=torch.float32, device=dev)

            a0, w0, rs, cs, bs, o = (a.data_ptr(), w.data_ptr(), row_scale.data_ptr(), col_scale.data_ptr(),
                                     bias.data_ptr(), out.data_ptr())

            def launch(i):
                st = lib.mc_q8_gemm(a0 + (i % na) * m * k, w0 + (i % nw) * n * k, m, n, k, rs, cs, bs, None, 0, 1,
                                    o, sp)
                if st != 0:
                    raise RuntimeError(f"mc_q8_gemm failed ({st}) at M={m} K={k} N={n}")

            for i in range(3):
                launch(i)
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            torch.cuda._sleep(4_000_000)  # ~2 ms of device time: longer than enqueueing the launches
            start.record(stream)
            for i in range(3, 3 + iters):
                launch(i)
            end.record(stream)
            torch.cuda.synchronize()
            sec = start.elapsed_time(end) / 1000.0 / iters
            ops = 2.0 * m * n * k
            nbytes = m * k + n * k + 8 * n + 4 * m + 4 * m * n
            tensor = m >= 64  # the configuration's own rule: weight streaming below 64 rows
            tensor_frac = ops / sec / 1e12 / (2.0 * peaks["bf16_tflops"])
            hbm_frac = nbytes / sec / 1e9 / peaks["hbm_gbs"]
            # frac follows the rule; both are given, since at large M x N the
            # f32 output's bytes, not the MMAs, set the floor
            points.append({"k": k, "n": n, "m": m, "us": sec * 1e6, "tops": ops / sec / 1e12,
                           "gbs": nbytes / sec / 1e9, "bound": "tensor" if tensor else "hbm",
                           "frac": tensor_frac if tensor else hbm_frac, "tensor_frac": tensor_frac,
                           "hbm_frac": hbm_frac})
            del a, row_scale, out
        del w
    torch.cuda.empty_cache()
    return {"workload": "config 2: mc_q8_gemm, int8 A [M,K] x int8 W [N,K], f32 out with per-row and "
                        "per-column scales and bias; operands cycled through > 2 x L2 of copies",
            "unit": "us per launch", "peak_source": f"{peak_kind}: 2 x bf16 dense TFLOP/s (int8) for M >= 64, "
                                                    "HBM copy GB/s below", "points": points}


def measure_longtext(args, eng, stream, model_bytes, rank, world, barrier):
    """Config 5 as strong scaling: a fixed global document set dealt over
    the replicas by length bucket."""
    import torch
    vocab = W.SHAPES[args.model].vocab
    batch = W.longtext_batch(args.longtext_docs, vocab=vocab, seed=555, rank=rank, world=world)
    eng.translate_token_ids(batch.tokens, batch.offsets, batch.max_out, batch.force_len)  # warm
    torch.cuda.synchronize()
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    t0 = time.perf_counter()
    out, off = eng.translate_token_ids(batch.tokens, batch.offsets, batch.max_out, batch.force_len)
    end.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    barrier()
    tokens, max_ms, max_wall = reduce_job(int(off[-1]), start.elapsed_time(end), wall, world, "cuda")
    res = {"workload": "config 5: %d documents of 200..2000 Zipf(1.1) tokens split by segment_text into "
                       "segments <= 128 tokens, sorted by length and dealt round-robin over %d replica(s)"
                       % (args.longtext_docs, world),
           "scaling": "strong", "value": tokens / (max_ms / 1000.0), "unit": UNIT,
           "e2e_value": tokens / max_wall, "target_tokens": int(tokens),
           "segments_this_rank": int(batch.size), "ms": max_ms}
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = host_threads()
        v, reqs, toks, secs = cpu_sample(model_bytes, [batch], 6.0, threads)
        res["cpu_baseline"] = cpu_baseline_obj(v, reqs, toks, secs, threads, "target tokens")
    return res


def measure_latency(args, eng, n=20000):
    """Config 4's latency: Poisson arrivals replayed by mc_replay."""
    vocab = W.SHAPES[args.model].vocab
    batch = W.stream_batch(n=n, vocab=vocab, seed=4242)
    out = []
    for rate in (2000.0, args.capacity_rate):
        arrivals = W.poisson_arrivals(n, rate, seed=4242)
        t0 = time.perf_counter()
        lat = eng.replay(batch.tokens, batch.offsets, batch.max_out, batch.force_len, arrivals) * 1000.0
        wall = time.perf_counter() - t0
        lens = np.diff(batch.offsets.astype(np.int64))
        tokens = int(np.minimum(np.minimum(np.minimum(batch.force_len, batch.max_out), 3 * lens), 256).sum())
        out.append({"arrival_rate_per_s": rate, "requests": n, "p50": float(np.percentile(lat, 50)),
                    "p99": float(np.percentile(lat, 99)), "mean": float(lat.mean()),
                    "served_tokens_per_s": tokens / wall, "wall_s": wall,
                    "loop": "mc_replay (C++ arrival loop, host clock)"})
    return out


def run_cuda(args):
    import torch
    import torch.distributed as dist
    from marian_cuda import _lib as L
    from marian_cuda.backend import CudaEngine

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    model_bytes = W.synthetic_model(W.SHAPES[args.model], seed=0)
    eng = CudaEngine(model_bytes, device=local, max_inflight=args.max_inflight, max_encode_tokens=65536,
                     lanes=args.lanes)
    lib = L.load()
    stream = torch.cuda.ExternalStream(eng.stream(), device=torch.device("cuda", local))
    warm = step_batches(args, rank, max(1, args.warmup), 100, world)
    timed = step_batches(args, rank, args.steps, 1000, world)

    def run(batch):
        out, off = eng.translate_token_ids(batch.tokens, batch.offsets, batch.max_out, batch.force_len)
        return int(off[-1])

    for i in range(args.warmup):
        run(warm[i % len(warm)])

    # kernel-class profile on one extra (untimed) step of the same stream
    lib.mc_profile(eng.handle, 1)
    run(warm[0])
    prof = read_profile(lib, eng, L)
    lib.mc_profile(eng.handle, 0)

    # decode-stream timeline on one more (untimed) step: each decode step's
    # device time and the stream's idle time between steps
    lib.mc_timeline(eng.handle, 1)
    run(warm[0])
    tl_n, tl_busy, tl_idle = C.c_uint64(), C.c_double(), C.c_double()
    lib.mc_timeline_read(eng.handle, C.byref(tl_n), C.byref(tl_busy), C.byref(tl_idle))
    lib.mc_timeline(eng.handle, 0)
    timeline = {"decode_steps": tl_n.value, "busy_ms": tl_busy.value, "idle_ms": tl_idle.value,
                "idle_frac": tl_idle.value / max(1e-9, tl_busy.value + tl_idle.value)}

    torch.cuda.synchronize()
    barrier()
    launches0 = lib.mc_launch_count(eng.handle)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    tokens = 0
    h2d = d2h = 0
    with Clocks(local) as clocks:
        torch.cuda.synchronize()
        start.record(stream)
        t0 = time.perf_counter()
        for b in timed:
            n = run(b)
            tokens += n
            h2d += b.tokens.nbytes + b.offsets.nbytes + b.max_out.nbytes + b.force_len.nbytes
            d2h += 4 * n + 4 * (b.size + 1)
        end.record(stream)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
    barrier()
    launches = lib.mc_launch_count(eng.handle) - launches0
    dev_ms = start.elapsed_time(end)
    all_tokens, max_ms, max_wall = reduce_job(tokens, dev_ms, wall, world, "cuda")
    peaks, peak_kind = load_peaks()

    extra = {}
    if not args.no_configs and args.workload == "stream":
        # every rank takes part (config 5 is a whole-job measurement)
        extra["config5_longtext"] = measure_longtext(args, eng, stream, model_bytes, rank, world, barrier)
        extra["config3_encoder"] = measure_encoder(args, eng, lib, L, model_bytes, peaks, peak_kind, rank,
                                                   world)
    if not args.no_latency and rank == 0 and args.workload == "stream":
        extra["latency_ms"] = measure_latency(args, eng)
    if not args.no_configs and rank == 0 and args.workload == "stream":
        extra["config2_gemm"] = measure_gemm(lib, peaks, peak_kind)

    if rank == 0:
        roofline = None
        if prof:
            name, r = max(prof.items(), key=lambda kv: kv[1]["ms"])
            roofline = class_roofline(name, r, peaks, peak_kind)
            roofline["share_of_profiled_time"] = r["ms"] / sum(v["ms"] for v in prof.values())
            # every class beside the dominant one: the HBM-bound attention
            # and the tensor-bound vocabulary GEMM next to the latency-bound
            # fused linear + LayerNorm
            roofline["classes"] = {
                k: {key: c[key] for key in ("bound", "frac", "achieved", "unit", "avg_launch_us")}
                for k, c in ((k, class_roofline(k, v, peaks, peak_kind)) for k, v in prof.items() if v["launches"])}
        cpu = None
        if not args.no_cpu_baseline and world == 1:
            threads = host_threads()
            v, reqs, toks, secs = cpu_sample(model_bytes, timed[:1], args.cpu_seconds, threads)
            cpu = cpu_baseline_obj(v, reqs, toks, secs, threads, "target tokens of step 0's stream")
        whole = None
        if prof:  # whole-step fraction: all algorithmic bytes of the profiled step over the timed step time
            step_bytes = sum(v["bytes"] for v in prof.values())
            whole = {"algorithmic_bytes_per_step": step_bytes,
                     "hbm_frac_of_timed_step": step_bytes / (max_ms / args.steps / 1000.0) / 1e9 / peaks["hbm_gbs"]}
        line = {"metric": METRIC, "value": all_tokens / (max_ms / 1000.0), "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": max_ms / args.steps,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "s8xs8->s32 GEMMs, f32 activations/attention/KV",
                "data": "synthetic (seeded random-init model weights and token streams)",
                "config": config_dict(args, world),
                "e2e": {"value": all_tokens / max_wall, "unit": UNIT, "h2d_bytes_per_step": h2d // args.steps,
                        "d2h_bytes_per_step": d2h // args.steps,
                        "path": "mc_translate_token_ids from host numpy buffers, host wall clock"},
                "gpu_launches": int(launches), "roofline": roofline, "whole_step": whole, "cpu_baseline": cpu,
                "clocks": clocks.summary(), "kernel_profile": prof, "decode_stream": timeline,
                "target_tokens": int(all_tokens)}
        line.update(extra)
        print(json.dumps(line), flush=True)
    eng.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_cuda(args)


if __name__ == "__main__":
    main()
