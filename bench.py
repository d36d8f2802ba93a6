"""Benchmark of the GGUF quantized matvec (decode hot path) on B200.

Workload (one step): the per-type matvec sweep -- W [4096 x 11008] and
[11008 x 4096] ([n_out x k]) in each of Q8_0, Q4_K, Q5_K and Q6_K, weights fp32
N(0, 0.02) quantized from fixed seeds, activations fp32 N(0, 1), batch 1:
eight matvecs, 282 MB of packed weights per step. The weight set is larger
than the 126 MB L2, so consecutive launches stream from HBM (no flush).

Metric: algorithmic bytes (packed W + x + y) per second, whole job.
  value      device time of exactly K steps replayed from a CUDA graph, inputs
             resident in HBM (CUDA events, max over ranks).
  e2e        the same steps through the public API (hesa_cuda.qmatvec ->
             C ABI) with x copied from pinned host memory and y read back
             every step.
  roofline   achieved GB/s of the streaming kernels vs the measured HBM copy
             peak (MEASURED_PEAKS.json).
  cpu_baseline  the reference's own scalar matmul (cpu_matmul_f32,
             oracle/_ref) on the dequantized weights of a bounded row sample,
             on all host threads, rank 0 at N=1 only.

N > 1 GPUs (torchrun): weak scaling with row-sharded weights -- rank r holds
rows [r*n, (r+1)*n) of an N-times taller matrix (its shard has the N=1 shape)
and every rank ends each step holding the full outputs: the matvec kernels
store their rows straight into every rank's gathered buffer over NVLink as
tagged 64-bit words (hesa_cuda_qmatvec_gather_tagged) and one collector kernel
per step waits until every word of this rank's buffer carries the step's tag
(hesa_cuda_peer_collect). The same step with an NCCL all-gather instead is
timed beside it ("nccl_allgather").

--impl reference: times the reference CPU path (above) on rank 0 only.
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

import numpy as np

# stdout carries the one JSON line. NCCL writes its log (the version banner
# included, at every level but NONE) to stdout; the line goes out through a
# duplicate of the original stdout (RESULT) and file descriptor 1 is pointed at
# stderr, so whatever a library prints lands there.
os.environ.setdefault("NCCL_DEBUG", "WARN")
RESULT = None


def _route_stdout():
    global RESULT
    if RESULT is None:
        sys.stdout.flush()
        RESULT = os.fdopen(os.dup(1), "w")
        os.dup2(2, 1)


def emit(obj) -> None:
    """Print the bench's JSON line on the original stdout."""
    out = RESULT if RESULT is not None else sys.stdout
    print(json.dumps(obj), file=out, flush=True)

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "hesa-llm_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

SWEEP = [(name, n, k) for name in ("Q8_0", "Q4_K", "Q5_K", "Q6_K") for (n, k) in ((4096, 11008), (11008, 4096))]
QT = {"Q4_0": 2, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14}
BE = {2: 32, 8: 32, 12: 256, 13: 256, 14: 256}
BB = {2: 18, 8: 34, 12: 144, 13: 176, 14: 210}
METRIC = "quant matvec HBM GB/s (algorithmic bytes: packed W + x + y)"
L2_NOTE = "inputs larger than L2: 282 MB weight set per step vs 126 MB L2, no flush"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def row_bytes(qt, k):
    return (k // BE[qt]) * BB[qt]


def step_bytes(world=1):
    """Algorithmic bytes of one step for ONE rank's shards."""
    tot = 0
    for name, n, k in SWEEP:
        tot += n * row_bytes(QT[name], k) + 4 * k + 4 * n
    return tot


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def committed_traffic():
    """Per-step DRAM bytes of the batch-1 matvec kernels from the committed ncu
    summary (profiles/qmv_strip_sweep_traffic.json), or None."""
    p = os.path.join(ROOT, "profiles", "qmv_strip_sweep_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        d = json.load(f)
    return d.get("dram_bytes_per_step")


# --------------------------------------------------------------------------
# clocks sampled with nvidia-smi while the GPU is under this workload
# --------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [s.strip() for s in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for nm, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# --------------------------------------------------------------------------
# inputs
# --------------------------------------------------------------------------

def make_inputs(rank: int, dev):
    """The sweep's matrices on the device: seeded fp32 N(0, 0.02) weights
    quantized by this library's GPU quantizer, N(0, 1) activations."""
    import torch
    import hesa_cuda as H
    g = torch.Generator(device=dev)
    mats = []
    for i, (name, n, k) in enumerate(SWEEP):
        qt = QT[name]
        g.manual_seed(1000 * (rank + 1) + i)
        w = H.quantize(qt, torch.randn((n, k), generator=g, device=dev).mul_(0.02))
        g.manual_seed(500 + i)
        x = torch.randn(k, generator=g, device=dev)
        mats.append((name, qt, n, k, w, x))
    torch.cuda.synchronize(dev)
    return mats


def cpu_model() -> str:
    """The host CPU's model name (from /proc/cpuinfo)."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_inputs(rows_cap: int = 1024):
    """A row sample of each sweep matrix for the CPU legs: the first rows_cap
    rows of W, fp32 N(0, 0.02) quantized by the oracle's codec (byte-identical
    to the GPU quantizer), the same rows dequantized to fp32 (the reference
    stores F32 weights: it has no quantized path), and x ~ N(0, 1)."""
    from oracle import oracle as O
    out = []
    for i, (name, n, k) in enumerate(SWEEP):
        qt = QT[name]
        rows = min(rows_cap, n)
        packed = O.quantize(qt, O.gaussian((rows, k), 0.02, 3000 + i))
        deq = O.dequantize(qt, packed, k)
        x = O.gaussian((k,), 1.0, 3100 + i)
        out.append((name, qt, rows, k, packed, deq, x))
    return out


def _timed_passes(one_pass, target_seconds: float, passes: int | None):
    one_pass()   # warm
    if passes is None:
        t0 = time.perf_counter()
        one_pass()
        passes = max(1, int(target_seconds / max(time.perf_counter() - t0, 1e-9)))
    t0 = time.perf_counter()
    for _ in range(passes):
        one_pass()
    return passes, time.perf_counter() - t0


def cpu_reference_rate(samples, threads: int, target_seconds: float = 10.0, passes: int | None = None):
    """GB/s of the reference's scalar matmul (hesa::cpu_matmul_f32, compiled
    from the reference's sources into oracle/_ref) over the sample's
    dequantized rows, in the bench's metric (packed bytes of the rows + x + y),
    rows split over `threads` host threads (1 = as the reference runs it)."""
    import ctypes
    from oracle import oracle as O
    ref = O.ref_lib()
    if ref is None:
        return None
    f32p = ctypes.POINTER(ctypes.c_float)
    bufs = [(deq, np.ascontiguousarray(x), np.empty(rows, np.float32), rows, k)
            for _, _, rows, k, _, deq, x in samples]

    def one_pass():
        for deq, x, y, rows, k in bufs:
            ref.ref_cpu_matvec_mt(deq.ctypes.data_as(f32p), x.ctypes.data_as(f32p), y.ctypes.data_as(f32p),
                                  rows, k, ctypes.c_float(1.0), threads)

    qbytes = sum(rows * row_bytes(qt, k) + 4 * k + 4 * rows for _, qt, rows, k, _, _, _ in samples)
    passes, dt = _timed_passes(one_pass, target_seconds, passes)
    rows = samples[0][2]
    return {"value": qbytes * passes / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "reference",
            "sample": f"hesa::cpu_matmul_f32 (the reference's scalar kernel, compiled from its sources) on the "
                      f"dequantized fp32 weights of the first {rows} rows of each of the 8 sweep matrices, "
                      f"{passes} pass(es), rows split over {threads} host thread(s), {dt:.1f} s; credited with "
                      f"the packed bytes of those rows",
            "seconds": dt, "passes": passes}


def cpu_oracle_rate(samples, threads: int, target_seconds: float = 5.0):
    """GB/s of this build's oracle (fused dequantize + dot in C, OpenMP over
    rows) on the packed sample rows: plan (ii) of the CPU baseline, labelled
    as the build's oracle, not the reference."""
    from oracle import oracle as O

    def one_pass():
        for _, qt, rows, k, packed, _, x in samples:
            O.qmatvec(qt, packed, x, n_threads=threads)

    qbytes = sum(rows * row_bytes(qt, k) + 4 * k + 4 * rows for _, qt, rows, k, _, _, _ in samples)
    passes, dt = _timed_passes(one_pass, target_seconds, None)
    return {"value": round(qbytes * passes / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"oracle_qmatvec (this build's C restatement: fused dequantize + fp32 dot, OpenMP) on the "
                      f"packed rows of the same sample, {passes} pass(es), {dt:.1f} s"}


def cpu_decode_rate(dev, threads: int):
    """tokens/s of the oracle's decode step at the 7B shape on the host cores:
    the step is timed with one and with two layers (the same layer twice:
    its weights quantized on the GPU and copied to the host), and a 32-layer
    token is extrapolated as t(1) + 31 (t(2) - t(1))."""
    import torch
    from oracle import oracle as O
    cfg = dict(DECODE_7B, n_layer=1)
    d = build_decoder(cfg, dev, seed=91)
    L0 = d["layers"][0]
    host = {n: (L0[n].cpu().numpy().view(np.uint16).copy() if n in ("k_cache", "v_cache")
                else np.ascontiguousarray(L0[n].cpu().numpy()))
            for n in ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down", "attn_norm", "ffn_norm", "k_cache",
                      "v_cache")}
    w_out = d["w_out"].cpu().numpy()
    out_norm = d["out_norm"].cpu().numpy()
    x = O.dequantize(cfg["qtype"], d["emb"][1234:1235].cpu().numpy(), cfg["d_model"])[0]
    del d
    torch.cuda.empty_cache()
    times = {}
    for nl in (1, 2):
        c = dict(cfg, n_layer=nl)
        O.decode_step(c, [host] * nl, out_norm, w_out, x, DECODE_POS, n_threads=threads)   # warm
        t0 = time.perf_counter()
        reps = 2
        for _ in range(reps):
            O.decode_step(c, [host] * nl, out_norm, w_out, x, DECODE_POS, n_threads=threads)
        times[nl] = (time.perf_counter() - t0) / reps
    per_layer = max(times[2] - times[1], 1e-9)
    token_s = times[1] + (DECODE_7B["n_layer"] - 1) * per_layer
    return {"tokens_per_s": round(1.0 / token_s, 3), "s_per_token": round(token_s, 3), "cores": threads,
            "kind": "port",
            "sample": f"oracle_decode_step at the 7B shape (Q4_K, ctx 2048, pos 2047) timed with 1 and 2 layers "
                      f"({times[1]:.3f} s, {times[2]:.3f} s), 32 layers extrapolated"}


def cpu_baselines(dev):
    """The CPU legs of the bench line, on the GPU box's host cores (rank 0,
    N = 1): the reference's own scalar matmul on all host threads (the
    reported baseline) and on one thread (as the reference runs it), the
    build's oracle, and the oracle's 7B decode step."""
    from oracle import oracle as O
    threads = O.n_threads_default()
    samples = cpu_inputs()
    base = cpu_reference_rate(samples, threads, target_seconds=8.0)
    if base is None:
        return None
    out = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")}
    out["value"] = round(out["value"], 3)
    one = cpu_reference_rate(samples, 1, target_seconds=6.0)
    out["single_thread"] = {"value": round(one["value"], 3), "unit": "GB/s", "cores": 1, "kind": "reference",
                            "sample": one["sample"]}
    out["oracle"] = cpu_oracle_rate(samples, threads)
    out["decode_7b"] = cpu_decode_rate(dev, threads)
    out["cpu_model"] = cpu_model()
    out["host_threads"] = threads
    return out


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return 0
    from oracle import oracle as O
    threads = O.n_threads_default()
    samples = cpu_inputs()
    # one step = one pass of the reference kernel over the row sample on all
    # host threads (about 0.1 s), so the K timed steps stay within minutes
    base = cpu_reference_rate(samples, threads, passes=args.steps)
    if base is None:
        emit({"impl": "reference", "unavailable": "reference CPU library (oracle/_ref) not built"})
        return 0
    per_step_ms = base["seconds"] / args.steps * 1e3
    out = {"metric": METRIC, "value": round(base["value"], 3), "unit": "GB/s", "impl": "reference",
           "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step_ms, 3),
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic (seeded N(0,0.02) weights quantized to GGUF blocks, N(0,1) activations)",
           "config": {"workload": "per-type matvec sweep Q8_0/Q4_K/Q5_K/Q6_K x {4096x11008, 11008x4096} "
                                  "([n_out x k]), batch 1", "cpu_model": cpu_model()},
           "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
           "e2e": {"value": round(base["value"], 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                   "d2h_bytes_per_step": 0}}
    emit(out)
    return 0


# --------------------------------------------------------------------------
# 7B-shaped decode step (tokens/s)
# --------------------------------------------------------------------------

DECODE_7B = dict(n_layer=32, d_model=4096, n_head=32, n_kv_head=32, head_dim=128, d_ff=11008, vocab=32000,
                 ctx=2048, rms_eps=1e-6, rope_base=10000.0, qtype=12)
DECODE_POS = 2047   # decode at the last position: attention spans the full 2048-slot cache


def build_decoder(cfg, dev, seed):
    """Random-init Llama-shaped decoder on the device: weights N(0, 0.02)
    quantized by the GPU quantizer (Q, K, V rows joined, gate and up rows
    joined), RMSNorm weights 1, fp16 KV caches N(0, 1), embedding N(0, 1)."""
    import torch
    import hesa_cuda as H
    qt = cfg["qtype"]
    D, HD = cfg["d_model"], cfg["head_dim"]
    QD, KD, F, V, C = cfg["n_head"] * HD, cfg["n_kv_head"] * HD, cfg["d_ff"], cfg["vocab"], cfg["ctx"]
    g = torch.Generator(device=dev)

    def qrand(rows, k, sd, std=0.02):
        g.manual_seed(sd)
        out = torch.empty((rows, H.row_bytes(qt, k)), dtype=torch.uint8, device=dev)
        step = max(1, (1 << 26) // k)          # bounded fp32 temporary (256 MB)
        for r0 in range(0, rows, step):
            r1 = min(rows, r0 + step)
            H.quantize(qt, torch.randn((r1 - r0, k), generator=g, device=dev).mul_(std), out=out[r0:r1])
        return out

    layers, wbytes = [], 0
    for l in range(cfg["n_layer"]):
        sd = seed + 100 * l
        qkv, wo, gu, down = qrand(QD + 2 * KD, D, sd), qrand(D, QD, sd + 1), qrand(2 * F, D, sd + 2), \
            qrand(D, F, sd + 3)
        wbytes += qkv.numel() + wo.numel() + gu.numel() + down.numel()
        g.manual_seed(sd + 4)
        kc = torch.randn((C, KD), generator=g, device=dev).half()
        vc = torch.randn((C, KD), generator=g, device=dev).half()
        ones = torch.ones(D, dtype=torch.float32, device=dev)
        layers.append(dict(wq=qkv[:QD], wk=qkv[QD:QD + KD], wv=qkv[QD + KD:], wo=wo, w_gate=gu[:F], w_up=gu[F:],
                           w_down=down, attn_norm=ones, ffn_norm=ones.clone(), k_cache=kc, v_cache=vc))
    w_out = qrand(V, D, seed + 7)
    emb = qrand(V, D, seed + 8, std=1.0)
    wbytes += w_out.numel()
    m = H.Model(cfg["n_layer"], D, cfg["n_head"], cfg["n_kv_head"], HD, F, V, C, cfg["rms_eps"], cfg["rope_base"], qt)
    table = torch.from_numpy(H.rope_table(C, HD, cfg["rope_base"])).to(dev)
    n_ctx = min(DECODE_POS + 1, C)
    kv_bytes = cfg["n_layer"] * (2 * n_ctx * KD * 2 + 2 * KD * 2)   # caches read + the new slot written
    bytes_token = wbytes + emb.shape[1] + kv_bytes
    torch.cuda.synchronize(dev)
    return dict(model=m, layers=layers, arr=H.make_layers(layers), w_out=w_out, emb=emb,
                out_norm=torch.ones(D, dtype=torch.float32, device=dev), table=table,
                ws=H.decode_workspace(m, dev), bytes_token=bytes_token, weight_bytes=wbytes, kv_bytes=kv_bytes)


BATCHED_SHAPES = ((4096, 11008), (11008, 4096))
BATCHED_B = (1, 2, 4, 8, 16)


def run_batched(dev, stream, reps: int = 20, qname: str = "Q4_K", shapes=BATCHED_SHAPES, batches=BATCHED_B):
    """Batched-decode matvec: `qname` [n_out x k] against B activation rows,
    for the two FFN shapes of the 7B model and B in BATCHED_B. Eight weight
    copies (more than L2) rotate inside one CUDA graph; device-timed.
    Returns {shape: {B: (us per matvec, algorithmic GB/s)}}, bytes = W + 4 B (k + n_out)."""
    import torch
    import hesa_cuda as H
    qt, nw = QT[qname], 8
    out = {}
    g = torch.Generator(device=dev)
    g.manual_seed(4321)
    for (n, k) in shapes:
        w0 = H.quantize(qt, torch.randn((n, k), generator=g, device=dev) * 0.02)
        ws_list = [w0.clone() for _ in range(nw)]
        del w0
        res = {}
        for B in batches:
            x = torch.randn((B, k), generator=g, device=dev)
            y = torch.empty((B, n), device=dev)
            wsp = H.make_workspace(qt, n, k, B, device=dev)
            with torch.cuda.stream(stream):
                for w in ws_list:
                    H.qmatvec(qt, w, x, y=y, workspace=wsp, stream=stream)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    for w in ws_list:
                        H.qmatvec(qt, w, x, y=y, workspace=wsp, stream=stream)
                for _ in range(3):
                    graph.replay()
                stream.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e0.record(stream)
                for _ in range(reps):
                    graph.replay()
                e1.record(stream)
                e1.synchronize()
            us = e0.elapsed_time(e1) * 1000.0 / (reps * nw)
            byts = n * row_bytes(qt, k) + 4 * B * (k + n)
            res[B] = (round(us, 2), round(byts / us / 1e3, 1))
            del graph
        out[f"{n}x{k}"] = res
        del ws_list
    return out


PROJ70B = (("wq", 8192, 8192), ("wk", 1024, 8192), ("wv", 1024, 8192), ("wo", 8192, 8192),
           ("gate", 28672, 8192), ("up", 28672, 8192), ("down", 8192, 28672))


def proj70b_bytes(world: int) -> int:
    """Algorithmic bytes of one pass over the 70B projection set, all ranks
    together: every packed row once, x once per rank, every output once."""
    qt = QT["Q4_K"]
    return sum(n * row_bytes(qt, k) + 4 * k * world + 4 * n for _, n, k in PROJ70B)


def run_proj70b(dev, stream, rank: int, world: int, pg=None, reps: int = 20):
    """70B-shaped Q4_K projections (d_model 8192, FFN 28672, 8 KV heads of
    128), batch 1, row-sharded: this rank holds rows [r0, r1) of each of the
    seven matrices (sharding.row_range) and one pass is its seven matvecs,
    replayed from a CUDA graph (443 MB of weights at N = 1, more than L2). At
    N > 1 every pass also gathers the seven outputs on every rank (tagged peer
    stores from the matvecs, one collector per pass). Returns (ms per pass with
    the gather, ms per pass of the local matvecs alone) on this rank (device
    time)."""
    import torch
    import hesa_cuda as H
    import sharding
    qt = QT["Q4_K"]
    g = torch.Generator(device=dev)
    g.manual_seed(7070 + rank)
    tg = sharding.TaggedGather(sum(n for _, n, _ in PROJ70B), rank, world, device=dev) if world > 1 else None
    mats = []
    off = 0
    for name, n, k in PROJ70B:
        r0, r1 = sharding.row_range(n, rank, world)
        w = H.quantize(qt, torch.randn((r1 - r0, k), generator=g, device=dev) * 0.02)
        x = torch.randn(k, generator=g, device=dev)
        y = torch.empty(r1 - r0, device=dev)
        # the gather's workspace: only the down projection (k = 28672, longer
        # rows than the strip kernel takes) needs one
        gws = H.gather_tagged_workspace(qt, r1 - r0, k, device=dev) if tg else None
        mats.append((w, x, y, H.make_workspace(qt, r1 - r0, k, device=dev), off + r0, gws))
        off += n

    def local():
        for w, x, y, ws, row0, gws in mats:
            H.qmatvec(qt, w, x, y=y, workspace=ws, stream=stream)

    def gathered():
        for w, x, y, ws, row0, gws in mats:
            H.qmatvec_gather_tagged(qt, w, x, tg.targets(), row0, world, tg.sync, workspace=gws, stream=stream)
        tg.collect(stream=stream)

    def timed(body):
        body()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            body()
        for _ in range(3):
            graph.replay()
        stream.synchronize()
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            graph.replay()
        e1.record(stream)
        e1.synchronize()
        del graph
        return e0.elapsed_time(e1) / reps

    with torch.cuda.stream(stream):
        ms_local = timed(local)
        ms = timed(gathered) if tg is not None else ms_local
    if tg is not None:
        torch.cuda.synchronize(dev)
        pg.barrier()
        tg.close()
    del mats
    return ms, ms_local


def run_decode(dev, stream, steps: int, warmup: int, pg=None, rank: int = 0, world: int = 1):
    """tokens/s of the 7B-shaped Q4_K decode step (embedding lookup + every
    layer + LM head) of ONE sequence, one CUDA graph per token, device-timed.
    At N > 1 the sequence is decoded on all N GPUs together: heads, KV caches
    and row shares of gate|up and the LM head per rank, Wo and W_down whole on
    every rank (sharding.ShardedDecoder)."""
    import torch
    import hesa_cuda as H
    cfg = DECODE_7B
    d = build_decoder(cfg, dev, seed=77)
    x = torch.empty(cfg["d_model"], dtype=torch.float32, device=dev)
    logits = torch.empty(cfg["vocab"], dtype=torch.float32, device=dev)
    pos_dev = torch.tensor([DECODE_POS], dtype=torch.int32, device=dev)
    tok_dev = torch.tensor([1234], dtype=torch.int32, device=dev)
    dec = None
    want = None
    replica_ms = None
    if world > 1:
        import sharding
        # the unsharded step on this rank's full copy: the sharded step computes
        # every row with the same summation order, so its logits must equal
        # these bit for bit; timed too (one independent sequence per GPU)
        want = torch.empty_like(logits)

        def replica():
            H.embed(cfg["qtype"], d["emb"], cfg["d_model"], tok_dev, out=x, stream=stream)
            H.decode_step(d["model"], d["arr"], d["out_norm"], d["w_out"], d["table"], x, pos_dev, want, d["ws"],
                          stream=stream)

        with torch.cuda.stream(stream):
            replica()
            stream.synchronize()
            g_rep = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_rep, stream=stream):
                replica()
            for _ in range(3):
                g_rep.replay()
            stream.synchronize()
            r0 = torch.cuda.Event(enable_timing=True)
            r1 = torch.cuda.Event(enable_timing=True)
            r0.record(stream)
            for _ in range(steps):
                g_rep.replay()
            r1.record(stream)
            r1.synchronize()
            replica_ms = r0.elapsed_time(r1) / steps
            del g_rep
        dec = sharding.ShardedDecoder(cfg, d, rank, world, device=dev)
        logits = dec.logits()
        del d["layers"], d["arr"]   # the full model's weights: every rank keeps its shards only
        torch.cuda.empty_cache()
        torch.cuda.synchronize(dev)
        pg.barrier()   # the ranks start their first step within the peer wait limit of one another

    def step():
        H.embed(cfg["qtype"], d["emb"], cfg["d_model"], tok_dev, out=x, stream=stream)
        if dec is not None:
            dec.step(x, pos_dev, stream=stream)
        else:
            H.decode_step(d["model"], d["arr"], d["out_norm"], d["w_out"], d["table"], x, pos_dev, logits, d["ws"],
                          stream=stream)

    with torch.cuda.stream(stream):
        for _ in range(2):
            step()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        for _ in range(max(warmup, 3)):
            graph.replay()
        stream.synchronize()
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1) / steps
    ok = bool(torch.isfinite(logits).all().item()) and H.device_status(stream) == 0
    same = None if want is None else bool(torch.equal(logits, want))
    del graph
    if dec is not None:
        torch.cuda.synchronize(dev)
        pg.barrier()
        dec.close()
        pg.barrier()
    return dict(ms=ms, finite=ok, equal_unsharded=same, replica_ms=replica_ms, bytes_token=d["bytes_token"], weight_bytes=d["weight_bytes"],
                kv_bytes=d["kv_bytes"])


def profile_decode(steps: int):
    """A few eager decode steps of a 2-layer model with the 7B shapes (per-layer
    launches as in the full model, small enough for an ncu launch list)."""
    import torch
    import hesa_cuda as H
    cfg = dict(DECODE_7B, n_layer=2)
    dev = torch.device("cuda", 0)
    d = build_decoder(cfg, dev, seed=5)
    x = torch.empty(cfg["d_model"], dtype=torch.float32, device=dev)
    logits = torch.empty(cfg["vocab"], dtype=torch.float32, device=dev)
    pos = torch.tensor([DECODE_POS], dtype=torch.int32, device=dev)
    tok = torch.tensor([3], dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for _ in range(max(steps, 1)):
            H.embed(cfg["qtype"], d["emb"], cfg["d_model"], tok, out=x, stream=stream)
            H.decode_step(d["model"], d["arr"], d["out_norm"], d["w_out"], d["table"], x, pos, logits, d["ws"],
                          stream=stream)
        stream.synchronize()
    log(f"profile decode done: {steps} step(s), logits finite: {bool(torch.isfinite(logits).all())}")
    return 0


def profile_batched(steps: int, batch: int, qname: str = "Q4_K"):
    """A few eager batched matvecs (`qname` 4096 x 11008, `batch` activation
    rows) on one weight copy, small enough for an ncu capture of one launch."""
    import torch
    import hesa_cuda as H
    dev = torch.device("cuda", 0)
    n, k = BATCHED_SHAPES[0]
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    qt = QT[qname]
    w = H.quantize(qt, torch.randn((n, k), generator=g, device=dev) * 0.02)
    x = torch.randn((batch, k), generator=g, device=dev)
    y = torch.empty((batch, n), device=dev)
    ws = H.make_workspace(qt, n, k, batch, device=dev)
    for _ in range(max(steps, 1)):
        H.qmatvec(qt, w, x, y=y, workspace=ws)
    torch.cuda.synchronize()
    log(f"profile batched done: {steps} launch(es) of B={batch}, outputs finite: {bool(torch.isfinite(y).all())}")
    return 0


def profile_sharded(steps: int):
    """A 2-layer model of the 7B decode shapes: `steps` eager unsharded decode
    steps, then `steps` of the sharded step on one rank (world 1), for an ncu
    launch list that compares the two forms kernel by kernel."""
    import torch
    import hesa_cuda as H
    import sharding
    dev = torch.device("cuda", 0)
    cfg = dict(DECODE_7B, n_layer=2)
    d = build_decoder(cfg, dev, seed=77)
    x = torch.empty(cfg["d_model"], device=dev)
    pos = torch.tensor([DECODE_POS], dtype=torch.int32, device=dev)
    tok = torch.tensor([1234], dtype=torch.int32, device=dev)
    lg = torch.empty(cfg["vocab"], device=dev)
    dec = sharding.ShardedDecoder(cfg, d, 0, 1, device=dev)
    for _ in range(max(steps, 1)):
        H.embed(cfg["qtype"], d["emb"], cfg["d_model"], tok, out=x)
        H.decode_step(d["model"], d["arr"], d["out_norm"], d["w_out"], d["table"], x, pos, lg, d["ws"])
    torch.cuda.synchronize()
    for _ in range(max(steps, 1)):
        H.embed(cfg["qtype"], d["emb"], cfg["d_model"], tok, out=x)
        dec.step(x, pos)
    torch.cuda.synchronize()
    same = bool(torch.equal(dec.logits(), lg))
    dec.close()
    log(f"profile sharded done: {steps} step(s) of each form, logits equal: {same}")
    return 0


def profile_shapes(steps: int):
    """A few eager launches of the shapes outside the sweep, for ncu: the
    Q4_0 4096 x 4096 matvec (batch 1, row-strip kernel) and the 70B down
    projection, Q4_K 8192 x 28672 (rows longer than the strip kernel takes:
    the split-row streaming kernel). One weight copy of each (9.4 + 132 MB)."""
    import torch
    import hesa_cuda as H
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(4040)
    out = []
    for qt, n, k in ((QT["Q4_0"], 4096, 4096), (QT["Q4_K"], 8192, 28672)):
        w = H.quantize(qt, torch.randn((n, k), generator=g, device=dev).mul_(0.02))
        x = torch.randn(k, generator=g, device=dev)
        y = torch.empty(n, device=dev)
        ws = H.make_workspace(qt, n, k, device=dev)
        for _ in range(max(steps, 1)):
            H.qmatvec(qt, w, x, y=y, workspace=ws)
        out.append(y)
    torch.cuda.synchronize()
    log(f"profile shapes done: {steps} launch(es) each, outputs finite: "
        f"{all(bool(torch.isfinite(y).all()) for y in out)}")
    return 0


# --------------------------------------------------------------------------
# GPU arm
# --------------------------------------------------------------------------

def run_gpu(args, rank: int, world: int, local_rank: int):
    import torch
    import hesa_cuda as H

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pg = None
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        pg = dist

    H.lib()
    mats = make_inputs(rank, dev)
    # all activations of a step in one device buffer (each k is a multiple of
    # 4, so every view stays 16-byte aligned), as a serving loop keeps them
    x_all = torch.empty(sum(k for _, _, _, k, _, _ in mats), dtype=torch.float32, device=dev)
    dmats = []
    xoff = 0
    for name, qt, n, k, w, x in mats:
        wt = w
        xt = x_all[xoff:xoff + k]
        xt.copy_(x)
        xoff += k
        yt = torch.empty(n, dtype=torch.float32, device=dev)
        ws = H.make_workspace(qt, n, k, device=dev)
        dmats.append((name, qt, n, k, wt, xt, yt, ws))
    # the full (all-gathered) outputs of one step
    y_local = torch.empty(sum(n for _, _, n, _, _, _, _, _ in dmats), dtype=torch.float32, device=dev)
    y_all = torch.empty(world * y_local.numel(), dtype=torch.float32, device=dev)
    peers, targets = None, []
    if world > 1:
        # gathered buffers shared over NVLink, laid out as NCCL's all-gather of
        # y_local lays them out: rank r's block of all eight outputs at r * rows
        import sharding
        peers = sharding.TaggedGather(y_all.numel(), rank, world, device=dev)
        off = rank * y_local.numel()
        for name, qt, n, k, wt, xt, yt, ws in dmats:
            targets.append(off)
            off += n
        pg.barrier()

    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):
        for name, qt, n, k, wt, xt, yt, ws in dmats:
            H.qmatvec(qt, wt, xt, y=yt, workspace=ws)
        stream.synchronize()

    def one_step_nccl():
        off = 0
        for name, qt, n, k, wt, xt, yt, ws in dmats:
            H.qmatvec(qt, wt, xt, y=y_local[off:off + n], workspace=ws, stream=stream)
            off += n
        if pg is not None:
            pg.all_gather_into_tensor(y_all, y_local)

    def one_step():
        if peers is None:
            return one_step_nccl()
        for (name, qt, n, k, wt, xt, yt, ws), row0 in zip(dmats, targets):
            H.qmatvec_gather_tagged(qt, wt, xt, peers.targets(), row0, world, peers.sync, stream=stream)
        peers.collect(stream=stream)

    if args.profile:
        # a short, untimed run for ncu: K plain steps (8 launches each), no graphs
        with torch.cuda.stream(stream):
            for _ in range(args.steps):
                one_step()
            stream.synchronize()
        if pg is not None:
            pg.destroy_process_group()
        log(f"profile run done: {args.steps} step(s), {len(SWEEP) * args.steps} matvec launches")
        return 0

    # capture one step in a CUDA graph; replaying it removes host launch gaps
    with torch.cuda.stream(stream):
        for _ in range(3):
            one_step()
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            one_step()
        stream.synchronize()

        for _ in range(max(args.warmup, 3)):
            graph.replay()
        stream.synchronize()

        # clocks: sampled over a ~2 s load window of the same replay and the timed region
        sampler = ClockSampler(local_rank) if rank == 0 else None
        if sampler:
            sampler.start()
        # the same number of replays on every rank (each step ends waiting for
        # every rank's rows), sized to ~2 s from a short timed run
        t0 = time.time()
        for _ in range(50):
            graph.replay()
        stream.synchronize()
        n_load = torch.tensor([int(2.0 / max((time.time() - t0) / 50, 1e-6))], device=dev)
        if pg is not None:
            pg.all_reduce(n_load, op=pg.ReduceOp.MAX)
        for _ in range(min(int(n_load.item()), 100000)):
            graph.replay()
        stream.synchronize()

        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize(dev)
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        ev1.record(stream)
        ev1.synchronize()
        torch.cuda.synchronize(dev)
        dt_ms = ev0.elapsed_time(ev1)
        clocks = sampler.stop() if sampler else None

        # the same step with NCCL's all-gather instead of the fused one
        nccl_ms = None
        if pg is not None:
            gn = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gn, stream=stream):
                one_step_nccl()
            for _ in range(3):
                gn.replay()
            stream.synchronize()
            pg.barrier()
            torch.cuda.synchronize(dev)
            en0 = torch.cuda.Event(enable_timing=True)
            en1 = torch.cuda.Event(enable_timing=True)
            en0.record(stream)
            for _ in range(args.steps):
                gn.replay()
            en1.record(stream)
            en1.synchronize()
            nccl_ms = en0.elapsed_time(en1)
            del gn

        # kernel-only time of the same step without the collective (roofline)
        if pg is not None:
            kgraph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(kgraph, stream=stream):
                off = 0
                for name, qt, n, k, wt, xt, yt, ws in dmats:
                    H.qmatvec(qt, wt, xt, y=y_local[off:off + n], workspace=ws, stream=stream)
                    off += n
            for _ in range(3):
                kgraph.replay()
            stream.synchronize()
            ek0 = torch.cuda.Event(enable_timing=True)
            ek1 = torch.cuda.Event(enable_timing=True)
            ek0.record(stream)
            for _ in range(args.steps):
                kgraph.replay()
            ek1.record(stream)
            ek1.synchronize()
            kernel_ms = ek0.elapsed_time(ek1)
        else:
            kernel_ms = dt_ms

        # per-type breakdown (kernel only): each type's two matrices are
        # cloned until the rotated set exceeds 300 MB, so every launch streams
        # its weights from HBM rather than L2
        per_type = {}
        if rank == 0:
            # the Q4_0 4096 x 4096 matvec (batch 1) is measured here only: it
            # is not part of the sweep step
            g40 = torch.Generator(device=dev)
            g40.manual_seed(4040)
            w40 = H.quantize(QT["Q4_0"], torch.randn((4096, 4096), generator=g40, device=dev).mul_(0.02))
            x40 = torch.randn(4096, generator=g40, device=dev)
            q40 = [("Q4_0", QT["Q4_0"], 4096, 4096, w40, x40, torch.empty(4096, device=dev),
                    H.make_workspace(QT["Q4_0"], 4096, 4096, device=dev))]
            for tname in ("Q4_0", "Q8_0", "Q4_K", "Q5_K", "Q6_K"):
                sel = [m for m in dmats + q40 if m[0] == tname]
                pair = sum(m[4].numel() for m in sel)
                copies = max(2, -(-300_000_000 // pair))
                rot = [(qt, n, k, wt.clone(), xt, yt, ws) for _ in range(copies)
                       for (name, qt, n, k, wt, xt, yt, ws) in sel]
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for qt, n, k, wt, xt, yt, ws in rot:
                        H.qmatvec(qt, wt, xt, y=yt, workspace=ws, stream=stream)
                for _ in range(3):
                    g.replay()
                stream.synchronize()
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                reps = 20
                e0.record(stream)
                for _ in range(reps):
                    g.replay()
                e1.record(stream)
                e1.synchronize()
                by = sum(n * row_bytes(qt, k) + 4 * k + 4 * n for qt, n, k, _, _, _, _ in rot) * reps
                per_type[tname] = round(by / (e0.elapsed_time(e1) * 1e-3) / 1e9, 1)
                del g, rot

        # e2e through the public API with host buffers: every step copies all
        # activations in from pinned host memory (one copy) and the full
        # output back (one copy), then waits for it on the host
        x_host = x_all.cpu().pin_memory()
        y_out = y_all if pg is not None else y_local
        y_host = torch.empty(y_out.numel(), dtype=torch.float32).pin_memory()
        h2d = x_host.numel() * 4
        d2h = y_host.numel() * 4

        def e2e_body():
            x_all.copy_(x_host, non_blocking=True)
            if peers is None:
                off = 0
                for name, qt, n, k, wt, xt, yt, ws in dmats:
                    H.qmatvec(qt, wt, xt, y=y_local[off:off + n], workspace=ws, stream=stream)
                    off += n
                y_host.copy_(y_out, non_blocking=True)
            else:
                one_step()
                y_host.copy_(peers.out, non_blocking=True)

        def e2e_step():
            e2e_body()
            stream.synchronize()

        # eager: every call from Python, as a notebook user would make them
        for _ in range(3):
            e2e_step()
        if pg is not None:
            pg.barrier()
        ee0 = torch.cuda.Event(enable_timing=True)
        ee1 = torch.cuda.Event(enable_timing=True)
        ee0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        ee1.record(stream)
        ee1.synchronize()
        e2e_eager_ms = ee0.elapsed_time(ee1)

        # graphed: the same public-API calls and copies captured once, as a
        # serving loop runs its decode step; each replay copies x in from
        # pinned host memory and y back out, and the host waits for it
        per_replay = 1
        g_e2e = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_e2e, stream=stream):
            e2e_body()
        for _ in range(3):
            g_e2e.replay()
            stream.synchronize()
        if pg is not None:
            pg.barrier()
        replays = max(1, args.steps // per_replay)
        ee0.record(stream)
        for _ in range(replays):
            g_e2e.replay()
            stream.synchronize()
        ee1.record(stream)
        ee1.synchronize()
        e2e_ms = ee0.elapsed_time(ee1) * args.steps / (replays * per_replay)
        if peers is not None:
            # the gathered outputs equal the NCCL-gathered ones
            one_step()
            one_step_nccl()
            stream.synchronize()
            gathered_ok = bool(torch.equal(peers.out, y_all))

    # the 7B-shaped Q4_K decode step of one sequence (sharded over the ranks at N > 1)
    dec = run_decode(dev, stream, steps=max(args.steps, 20), warmup=args.warmup, pg=pg, rank=rank, world=world)
    batched = run_batched(dev, stream) if rank == 0 else None
    # eight activation rows per block type (4096 x 11008): Q4_K / Q5_K scale-split
    # kernel, Q8_0 / Q4_0 one MMA per 32-weight block, Q6_K one strip pass per row
    batched_types = ({t: run_batched(dev, stream, qname=t, shapes=BATCHED_SHAPES[:1], batches=(8,))
                      ["%dx%d" % BATCHED_SHAPES[0]][8] for t in ("Q4_0", "Q8_0", "Q4_K", "Q5_K", "Q6_K")}
                     if rank == 0 else None)
    p70_ms, p70_local_ms = run_proj70b(dev, stream, rank, world, pg=pg)

    # max over ranks
    times = torch.tensor([dt_ms, kernel_ms, e2e_ms, e2e_eager_ms, dec["ms"], nccl_ms or 0.0,
                          0.0 if peers is None or gathered_ok else 1.0, p70_ms,
                          0.0 if dec["equal_unsharded"] in (None, True) else 1.0, p70_local_ms,
                          dec["replica_ms"] or 0.0],
                         dtype=torch.float64, device=dev)
    if pg is not None:
        pg.all_reduce(times, op=pg.ReduceOp.MAX)
    (dt_ms, kernel_ms, e2e_ms, e2e_eager_ms, dec_ms, nccl_ms, gather_bad, p70_ms, dec_bad, p70_local_ms,
     replica_ms) = (float(v) for v in times.cpu())

    if rank == 0:
        bytes_step = step_bytes() * world
        value = bytes_step * args.steps / (dt_ms * 1e-3) / 1e9
        achieved = step_bytes() * args.steps / (kernel_ms * 1e-3) / 1e9
        peak, peak_kind = measured_peaks()
        traffic = committed_traffic()
        cpu_base = cpu_baselines(dev) if world == 1 else None
        out = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights quantized to GGUF blocks, N(0,1) activations)",
            "config": {"workload": "per-type matvec sweep Q8_0/Q4_K/Q5_K/Q6_K x {4096x11008, 11008x4096} "
                                   "([n_out x k]), batch 1",
                       "bytes_per_step_per_gpu": step_bytes(), "l2": L2_NOTE,
                       "parallelism": (f"row-sharded weights x{world}, all-gather of y fused into the matvec "
                                       "(tagged peer stores over NVLink + one collector kernel per step)"
                                       if world > 1
                                       else "single GPU"),
                       "timing": "CUDA graph of one step, replayed K times between CUDA events"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)",
                         "traffic": traffic,
                         "kernel": "qmv_strip_kernel (8 launches per step)"},
            "per_type_gbs": per_type,
            "nccl_allgather": ({"value": round(bytes_step * args.steps / (nccl_ms * 1e-3) / 1e9, 1),
                                "ms_per_step": round(nccl_ms / args.steps, 4),
                                "how": "the same step with local outputs and NCCL all_gather_into_tensor",
                                "gathered_outputs_equal": gather_bad == 0.0}
                               if world > 1 else None),
            "pct_of_8tbs": round(achieved / 8000.0, 4),
            "e2e": {"value": round(bytes_step * args.steps / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d * world, "d2h_bytes_per_step": d2h * world,
                    "how": "hesa_cuda.qmatvec per matrix (hesa_cuda.qmatvec_gather_tagged + peer_collect at "
                           "N > 1); "
                           "every step one copy of all activations from pinned host memory and one copy of "
                           "all outputs back, captured once in a CUDA graph and replayed with a host "
                           "synchronize per replay",
                    "eager_value": round(bytes_step * args.steps / (e2e_eager_ms * 1e-3) / 1e9, 1)},
            "gpu_launches": (len(SWEEP) + (1 if world > 1 else 0)) * args.steps,
            "decode": {"model": "Llama-shaped 7B (32 layers, d_model 4096, 32 heads x 128, FFN 11008 SwiGLU, "
                                "vocab 32000, RMSNorm, RoPE 10000), Q4_K, random init N(0, 0.02)",
                       "ctx": DECODE_7B["ctx"], "pos": DECODE_POS,
                       "tokens_per_s": round(1000.0 / dec_ms, 1), "ms_per_token": round(dec_ms, 4),
                       "bytes_per_token": dec["bytes_token"],
                       "gbs": round(dec["bytes_token"] / (dec_ms * 1e-3) / 1e9, 1),
                       "frac_of_hbm": round(dec["bytes_token"] / (dec_ms * 1e-3) / 1e9 / (peak * world), 4),
                       "parallelism": (f"one sequence on {world} GPUs: heads, KV caches and row shares of gate|up and "
                                       "the LM head per rank, Wo and W_down whole on every rank; the two exchanges "
                                       "per layer fused into the producing kernels (tagged 64-bit peer stores, "
                                       "waited for per word by the next kernel)"
                                       if world > 1 else "single GPU"),
                       "timing": "embedding lookup + 32 layers + LM head captured as one CUDA graph per token, "
                                 "replayed between CUDA events",
                       "logits_finite": dec["finite"],
                       "logits_equal_unsharded_step": (dec_bad == 0.0) if world > 1 else None,
                       "independent_sequences": ({"tokens_per_s": round(world * 1000.0 / replica_ms, 1),
                                                  "ms_per_token": round(replica_ms, 4),
                                                  "how": f"the unsharded step of one sequence on each of the {world} "
                                                         "GPUs at once (max over ranks)"}
                                                 if world > 1 else None)},
            "batched": {"workload": "Q4_K [n_out x k] times B activation rows (batched decode), "
                                    "one launch per 16 rows on the tensor cores (B >= 3; B = 2 as two batch-1 passes)",
                        "us_and_gbs": batched,
                        "b8_by_type_4096x11008": batched_types,
                        "b8_by_type_paths": "Q4_K/Q5_K: tcgen05, scale folded into two weight operands; Q8_0/Q4_0: "
                                            "tcgen05, one MMA per 32-weight block; Q6_K: eight batch-1 strip passes",
                        "timing": "8 rotating weight copies (203 MB > L2) in one CUDA graph, CUDA events, rank 0"},
            "proj70b": {"workload": "70B-shaped Q4_K projections, batch 1: Wq, Wo 8192x8192; Wk, Wv 1024x8192; "
                                   "gate, up 28672x8192; down 8192x28672 ([n_out x k])",
                        "parallelism": (f"rows split over {world} GPUs (each rank its shards; time = max over "
                                        "ranks), every rank ends each pass with all seven full outputs (tagged "
                                        "peer stores from the matvecs + one collector per pass)"
                                        if world > 1 else "single GPU"),
                        "scaling": "strong",
                        "ms_per_pass": round(p70_ms, 4),
                        "ms_per_pass_without_gather": round(p70_local_ms, 4),
                        "gbs": round(proj70b_bytes(world) / (p70_ms * 1e-3) / 1e9, 1),
                        "bytes_per_pass": proj70b_bytes(world),
                        "timing": "the seven matvecs in one CUDA graph, 20 replays between CUDA events"},
            "clocks": clocks,
            "cpu_baseline": cpu_base,
        }
        emit(out)

    del graph, g_e2e   # graphs that hold NCCL calls go before the process group
    if pg is not None:
        torch.cuda.synchronize(dev)
        pg.barrier()
        if peers is not None:
            peers.close()
        pg.barrier()
        pg.destroy_process_group()
    return 0


def main():
    _route_stdout()
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="hesa", choices=["hesa", "reference"])
    ap.add_argument("--profile", action="store_true",
                    help="untimed: build inputs, run --steps plain steps, exit (for ncu captures)")
    ap.add_argument("--profile-batched", type=int, default=0, metavar="B",
                    help="run --steps eager batched matvecs with B activation rows (for an ncu capture) and exit")
    ap.add_argument("--profile-type", default="Q4_K", choices=sorted(QT),
                    help="block type of the --profile-batched matrix")
    ap.add_argument("--profile-decode", action="store_true",
                    help="untimed: a 2-layer model of the 7B decode shapes, --steps eager decode steps "
                         "(for ncu launch lists of one step)")
    ap.add_argument("--profile-sharded", action="store_true",
                    help="untimed: a 2-layer model of the 7B decode shapes, --steps eager unsharded steps then "
                         "--steps sharded steps on one rank (for an ncu launch list comparing the two)")
    ap.add_argument("--profile-shapes", action="store_true",
                    help="untimed: --steps eager launches each of Q4_0 4096x4096 and Q4_K 8192x28672 "
                         "(for ncu captures of the shapes outside the sweep)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus if args.gpus else 1)))
    if "WORLD_SIZE" not in os.environ:
        world = 1
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.profile_decode:
        return profile_decode(args.steps)
    if args.profile_shapes:
        return profile_shapes(args.steps)
    if args.profile_sharded:
        return profile_sharded(args.steps)
    if args.profile_batched:
        return profile_batched(args.steps, args.profile_batched, args.profile_type)
    return run_gpu(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
