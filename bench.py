#!/usr/bin/env python
"""Benchmark of the mzoo attention hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl mzb|reference]

Configs (BASELINE.json ``configs``; synthetic seeded inputs with the stated shapes and
distributions -- there is no dataset):

- ``indexer`` (default, configs[1]): lightning indexer + top-512 over FP8 q/k, B=2,
  4096 queries at absolute positions 12288..16383 x 4096 compressed keys (ratio 4),
  Hi=64, Di=128.  Metric: indexer Mq/s (queries per second, whole job).
- ``prefill``: sparse latent MQA over FP8 576/512 rows, 16384 tokens x 128
  heads, top-2048 compressed entries + a 128-token window.  Metric: TFLOP/s.
- ``decode``: paged decode of 128 sequences (lengths 8k..131k), decode indexer
  + top-2048 + window 128.  Metric: algorithmic HBM GB/s.
- ``train``: window attention training step, B=4, S=8192, 64 heads, D=128,
  window 512, MXFP4 / FP8 fake quant of q, k, v.  Metric: TFLOP/s.
- ``candidates`` (next row F1, not a BASELINE config): two-level indexer selection, 2048
  queries x 65536 compressed positions.  Metric: Mq/s.
- ``compressor`` (next row F3, not a BASELINE config): compressor pool + RMSNorm + RoPE +
  MXFP4 cache entry, 8 x 16384 tokens at ratio 4, 576 channels.  Metric: algorithmic HBM GB/s.

A "step" is one pass of the hot path over one batch.  ``value`` times the device path with
inputs resident in HBM (L2 flushed with a 256 MB write before every timed step);
``e2e`` times the public API call with pinned host inputs, host->device copies, the
kernels and the device->host copy of the result inside the timed region.  Multi-GPU:
one process per GPU (torchrun); the indexer, prefill, decode, candidates and compressor
configs split one workload's independent units (query chunks, token chunks, sequences,
query rows, sequences) over the ranks with no data-path collective (strong scaling), the training config runs one instance per rank
(weak scaling); timing is the max over ranks of CUDA-event time.

``--impl reference`` times the reference's CPU path (the numpy restatement in
``oracle/``; the reference itself is Python and cannot travel to the GPU host) on a
bounded sample of the same workload, with all host threads, and prints the same metric.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        d["_source"] = "measured"
        return d
    d = dict(FALLBACK_PEAKS)
    d["_source"] = "fallback"
    return d


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi sampling (200 ms) of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def _rows(self) -> list:
        rows = []
        try:
            for line in open(self.path):
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except OSError:
            pass
        return rows

    def ready(self, timeout: float = 5.0) -> None:
        """Block until nvidia-smi has written its first sample (it takes ~0.1-1 s to start),
        and remember how many rows precede the timed region."""
        t0 = time.time()
        while self.proc is not None and not self._rows() and time.time() - t0 < timeout:
            time.sleep(0.02)
        self.n0 = len(self._rows()) if self.proc is not None else 0

    def stop(self, busy=None, min_samples: int = 2, timeout: float = 3.0) -> dict:
        """Stop sampling.  A timed region of a few milliseconds is shorter than the 200 ms
        sampling period, so ``busy`` (one more step of the same workload) keeps the GPU
        under that load until ``min_samples`` rows were taken after the region started."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        t0 = time.time()
        n0 = getattr(self, "n0", 0)
        while busy is not None and len(self._rows()) < n0 + min_samples and time.time() - t0 < timeout:
            busy()
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = self._rows()[n0:]
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        load = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# DRAM bytes (read + write) of one full-size launch of each config's roofline kernel, from a
# one-pass ncu capture of this build (dram__bytes_read.sum + dram__bytes_write.sum).
TRAFFIC = {
    "indexer": 72764928 + 69933824,
    "prefill": 2535907584 + 2112252416,
    "decode": 313127680 + 10324480,
    "train": (4376674816 + 94292736) + (1107655936 + 505236480),  # dkv_kernel + dq_kernel
    "candidates": 381950464 + 3411200,  # level two (gathered): 32-byte blocks cost ~2.8x in DRAM bursts
    "compressor": 612400896 + 68001536,
}


# ----------------------------------------------------------------------------- timing helpers

class Timer:
    """Per-step CUDA-event timing on the current stream with an L2 flush before each step."""

    def __init__(self, torch, device):
        self.torch = torch
        self.flush_buf = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    def flush(self):
        self.flush_buf.zero_()

    def run(self, fn, steps: int, flush: bool = True) -> list:
        torch = self.torch
        times = []
        for _ in range(steps):
            if flush:
                self.flush()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            times.append((s, e))
        torch.cuda.synchronize()
        return [s.elapsed_time(e) for s, e in times]


def max_over_ranks(torch, dist, value: float, device) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- indexer (C2)

C2 = dict(B=2, S=4096, T=4096, Hi=64, Di=128, ratio=4, topk=512, q_offset=12288)


def c2_pairs(cfg=C2) -> int:
    """Visible (query, key) pairs per batch element: sum_s min(T, (q_offset + s + 1) // ratio)."""
    return sum(min(cfg["T"], (cfg["q_offset"] + s + 1) // cfg["ratio"]) for s in range(cfg["S"]))


def c2_inputs(torch, seed: int):
    g = torch.Generator(device="cpu").manual_seed(seed)
    B, S, T, Hi, Di = (C2[k] for k in ("B", "S", "T", "Hi", "Di"))
    q = torch.randn(B, S, Hi, Di, generator=g)
    k = torch.randn(B, T, Di, generator=g)
    w = torch.randn(B, S, Hi, generator=g) / 8
    return q, k, w


def bench_indexer(args, torch, dist, rank, world, device) -> dict:
    from mzoo_b200 import indexer, _lib

    from mzoo_b200.sharding import shard_tokens
    q, k, w = c2_inputs(torch, seed=0)  # the same workload on every rank
    q8, sq = indexer.quantize_fp8(q.to(device))
    k8, sk = indexer.quantize_fp8(k.to(device))
    w = w.to(device)
    B, S, T, Hi, Di = (C2[x] for x in ("B", "S", "T", "Hi", "Di"))
    kw = dict(compress_ratio=C2["ratio"], topk=C2["topk"], q_offset=C2["q_offset"], scales=(sq, sk), check=False)
    toks = list(range(S))
    if world > 1:  # (batch x 128-query chunk) units, cyclic over ranks: the same chunks of every batch
        toks = shard_tokens(S, world, 128)[rank]
        tk = torch.tensor(toks, device=device)
        q8, sq, w = q8[:, tk].contiguous(), sq[:, tk].contiguous(), w[:, tk].contiguous()
        kw.update(scales=(sq, sk), q_pos=(tk + C2["q_offset"]).to(torch.int32).view(1, -1).expand(B, -1))
    step = lambda: indexer.attn(q8, k8, w, **kw)  # noqa: E731
    timer = Timer(torch, device)
    sampler = ClockSampler(device.index)
    sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler.ready()
    if dist:
        dist.barrier()
    t_steps = timer.run(step, args.steps)
    # the dominant kernel alone (score GEMM), for the roofline
    qp, kp, wp, sqp, skp, scale, dt = indexer._prep(q8, k8, w, (sq, sk), None)
    qpos = kw.get("q_pos")
    qpos = qpos.contiguous() if qpos is not None else None
    t_score = timer.run(lambda: indexer._scores(qp, kp, wp, sqp, skp, C2["ratio"], C2["q_offset"], scale, dt,
                                                False, False, qpos), args.steps)
    # end to end through the public API from pinned host memory
    hq8 = q8.view(torch.uint8).cpu().pin_memory()
    hk8 = k8.view(torch.uint8).cpu().pin_memory()
    hsq, hsk, hw = (x.cpu().pin_memory() for x in (sq, sk, w))
    dq8, dk8 = torch.empty_like(hq8, device=device), torch.empty_like(hk8, device=device)
    dsq, dsk, dw = (torch.empty_like(x, device=device) for x in (hsq, hsk, hw))
    hout = torch.empty(B, len(toks), C2["topk"], dtype=torch.int32).pin_memory()

    def e2e():
        for d, h in ((dq8, hq8), (dk8, hk8), (dsq, hsq), (dsk, hsk), (dw, hw)):
            d.copy_(h, non_blocking=True)
        idx = indexer.attn(dq8.view(torch.float8_e4m3fn), dk8.view(torch.float8_e4m3fn), dw,
                           **dict(kw, scales=(dsq, dsk)))
        hout.copy_(idx, non_blocking=True)

    for _ in range(2):
        e2e()
    t_e2e = timer.run(e2e, args.steps, flush=False)
    clocks = sampler.stop(busy=step)
    torch.cuda.synchronize()
    indexer.attn(q8, k8, w, **dict(kw, check=True))  # one checked call: raises on a device error word
    h2d = sum(x.numel() * x.element_size() for x in (hq8, hk8, hsq, hsk, hw))
    d2h = hout.numel() * hout.element_size()

    ms = max_over_ranks(torch, dist, sum(t_steps) / len(t_steps), device)
    ms_e2e = max_over_ranks(torch, dist, sum(t_e2e) / len(t_e2e), device)
    ms_score = sum(t_score) / len(t_score)
    queries = B * S  # the whole job: every rank does its share of one workload
    pairs_local = sum(min(T, (C2["q_offset"] + s + 1) // C2["ratio"]) for s in toks)
    flops = 2.0 * B * pairs_local * Hi * Di
    pk = peaks()
    fp8_peak = 2.0 * pk["bf16_tflops"]
    achieved = flops / (ms_score * 1e-3) / 1e12
    out = {
        "metric": "indexer Mq/s", "value": queries / (ms * 1e-3) / 1e6, "unit": "Mq/s",
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e4m3 (fp32 accumulate)", "data": "synthetic (seeded N(0,1), absmax fp8)",
        "config": {"workload": "C2 lightning indexer + top-k", "B": B, "queries": S, "keys": T, "Hi": Hi, "Di": Di,
                   "compress_ratio": C2["ratio"], "topk": C2["topk"], "q_offset": C2["q_offset"],
                   "parallelism": (f"(batch x 128-query chunk) units cyclic over {world} GPUs, keys replicated, no "
                                   "collective in the step" if world > 1 else "1 GPU"),
                   "l2": "flushed (256 MB write) per step"},
        "e2e": {"value": queries / (ms_e2e * 1e-3) / 1e6, "unit": "Mq/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "tensor", "kernel": "mzb::idx::score_kernel<fp8,128,2>", "achieved": achieved,
                     "peak": fp8_peak, "unit": "TFLOP/s", "frac": achieved / fp8_peak,
                     "peak_note": f"dense FP8 = 2 x {pk['_source']} bf16 burst {pk['bf16_tflops']} TFLOP/s",
                     "algorithmic_flops_per_launch": flops, "ms_per_launch": ms_score,
                     "traffic": TRAFFIC["indexer"], "traffic_unit": "bytes per launch (ncu)"},
        "gpu_launches": 3 * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_indexer(torch, q, k, w, sample=args.cpu_sample)
    return out


def cpu_indexer(torch, q, k, w, sample: int) -> dict:
    """Oracle port on the host: canonical fp64 scores + exact top-k for `sample` queries
    (the last ones of batch 0, every key visible to most of them)."""
    import numpy as np
    from oracle import indexer as I
    from oracle import quant as Q
    qn = q[0:1, -sample:].numpy()
    kn = k[0:1].numpy()
    wn = w[0:1, -sample:].cpu().numpy()
    qv, sq = Q.quantize_fp8_rows(qn, C2["Di"])
    kv, sk = Q.quantize_fp8_rows(kn, C2["Di"])
    off = C2["q_offset"] + C2["S"] - sample
    t0 = time.perf_counter()
    sc = I.canonical_scores(qv, kv, wn, sq[..., 0], sk[..., 0], C2["ratio"], off)
    I.canonical_topk(sc, C2["topk"], C2["ratio"], off)
    dt = time.perf_counter() - t0
    return {"value": sample / dt / 1e6, "unit": "Mq/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{sample} queries of batch 0 (positions {off}..{off + sample - 1}), numpy fp64 canonical "
                      f"scores + top-{C2['topk']}, {dt:.2f} s"}


def reference_indexer(args, rank, world) -> dict:
    import torch
    if rank != 0:
        return None
    q, k, w = c2_inputs(torch, seed=0)
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_indexer(torch, q, k, w, sample=min(args.cpu_sample // 4, 1024))
        if i >= args.warmup:
            vals.append(r["value"])
    v = statistics.mean(vals)
    r["value"] = v
    return {"metric": "indexer Mq/s", "value": v, "unit": "Mq/s", "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": C2["B"] * C2["S"] / (v * 1e6) * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64 (oracle port)",
            "data": "synthetic (seeded N(0,1), absmax fp8)",
            "config": {"workload": "C2 lightning indexer + top-k", "B": C2["B"], "queries": C2["S"], "keys": C2["T"],
                       "Hi": C2["Hi"], "Di": C2["Di"], "compress_ratio": C2["ratio"], "topk": C2["topk"],
                       "q_offset": C2["q_offset"]},
            "cpu_baseline": r,
            "e2e": {"value": v, "unit": "Mq/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ----------------------------------------------------------------------------- sparse MLA prefill (C3)

C3 = dict(B=1, S=16384, H=128, G=4096, ratio=4, topk=2048, window=128)


def sorted_causal_indices(torch, S, G, topk, ratio, gen, device, q_offset=0, chunk=2048):
    """Per query t: seeded random distinct compressed indices from [0, (t+q_offset+1)//ratio),
    the first topk of a random permutation, sorted ascending, -1 padded."""
    out = torch.empty(S, topk, dtype=torch.int32, device=device)
    cols = torch.arange(G, device=device)
    for s0 in range(0, S, chunk):
        s1 = min(S, s0 + chunk)
        r = torch.rand(s1 - s0, G, generator=gen, device=device)
        vis = (torch.arange(s0, s1, device=device) + q_offset + 1) // ratio
        r.masked_fill_(cols[None, :] >= vis[:, None], 2.0)
        vals, ind = r.topk(topk, dim=1, largest=False)
        ind = torch.where(vals < 2.0, ind, torch.full_like(ind, 1 << 30)).sort(dim=1).values
        out[s0:s1] = torch.where(ind == (1 << 30), torch.full_like(ind, -1), ind).to(torch.int32)
    return out


def c3_inputs(torch, device, seed: int):
    from mzoo_b200 import sparse_mla
    S, G = C3["S"], C3["G"]
    g = torch.Generator(device=device).manual_seed(seed)
    q = torch.randn(1, S, C3["H"], 576, generator=g, device=device, dtype=torch.bfloat16)
    raw = sparse_mla.pack_kv(torch.randn(1, S, 576, generator=g, device=device))
    cmp = sparse_mla.pack_kv(torch.randn(1, G, 576, generator=g, device=device))
    g1 = torch.Generator(device=device).manual_seed(seed + 1)
    idx = sorted_causal_indices(torch, S, G, C3["topk"], C3["ratio"], g1, device).view(1, S, C3["topk"])
    return q, raw, cmp, idx


def c3_pairs(torch, idx, positions=None) -> int:
    """Selected (query, key) pairs: valid compressed indices + window keys of each query
    (query i sits at positions[i], default i)."""
    positions = range(idx.shape[1]) if positions is None else positions
    win = sum(min(C3["window"], t + 1) for t in positions)
    return int((idx >= 0).sum().item()) + win


def bench_prefill(args, torch, dist, rank, world, device) -> dict:
    from mzoo_b200 import sparse_mla
    from mzoo_b200.sharding import shard_tokens
    q, raw, cmp, idx = c3_inputs(torch, device, seed=0)  # the same workload on every rank
    total_flops = sparse_mla.pair_flops(c3_pairs(torch, idx))
    pos, toks = None, None
    if world > 1:  # this rank's cyclic 128-token chunks of the query axis; KV replicated
        toks = shard_tokens(C3["S"], world, 128)[rank]
        tk = torch.tensor(toks, device=device)
        q, idx = q[:, tk].contiguous(), idx[:, tk].contiguous()
        pos = tk.to(torch.int32).view(1, -1)
    flops = sparse_mla.pair_flops(c3_pairs(torch, idx, toks))
    n_q = q.shape[1]
    step = lambda: sparse_mla.prefill(q, raw, cmp, idx, window=C3["window"], q_pos=pos, check=False)  # noqa: E731
    timer = Timer(torch, device)
    sampler = ClockSampler(device.index)
    sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler.ready()
    if dist:
        dist.barrier()
    t_steps = timer.run(step, args.steps)
    clocks = sampler.stop(busy=step)
    # end to end from pinned host buffers
    hq, hraw, hcmp, hidx = (x.cpu().pin_memory() for x in (q, raw, cmp, idx))
    dq, draw, dcmp, didx = (torch.empty_like(x, device=device) for x in (hq, hraw, hcmp, hidx))
    ho = torch.empty(1, n_q, C3["H"], 512, dtype=torch.bfloat16).pin_memory()
    hl = torch.empty(1, C3["H"], n_q, dtype=torch.float32).pin_memory()

    def e2e():
        for d, h in ((dq, hq), (draw, hraw), (dcmp, hcmp), (didx, hidx)):
            d.copy_(h, non_blocking=True)
        o, lse = sparse_mla.prefill(dq, draw, dcmp, didx, window=C3["window"], q_pos=pos, check=False)
        ho.copy_(o, non_blocking=True)
        hl.copy_(lse, non_blocking=True)

    e2e()
    t_e2e = timer.run(e2e, max(2, args.steps // 4), flush=False)
    h2d = sum(x.numel() * x.element_size() for x in (hq, hraw, hcmp, hidx))
    d2h = ho.numel() * ho.element_size() + hl.numel() * hl.element_size()
    ms = max_over_ranks(torch, dist, sum(t_steps) / len(t_steps), device)
    ms_e2e = max_over_ranks(torch, dist, sum(t_e2e) / len(t_e2e), device)
    gather_ms = None
    if dist:  # optional output gather (o of every rank's shard to every rank), timed on its own
        o_loc, _ = step()
        width = max(len(p) for p in shard_tokens(C3["S"], world, 128))
        pad = o_loc.new_zeros((width,) + tuple(o_loc.shape[2:]))
        pad[:n_q] = o_loc[0]
        buf = o_loc.new_empty((world * width,) + tuple(o_loc.shape[2:]))
        dist.all_gather_into_tensor(buf, pad)  # untimed: the collective's lazy setup
        t_g = timer.run(lambda: dist.all_gather_into_tensor(buf, pad), 3, flush=False)
        gather_ms = max_over_ranks(torch, dist, sum(t_g) / len(t_g), device)
    pk = peaks()
    tflops = total_flops / (ms * 1e-3) / 1e12
    achieved = flops / (ms * 1e-3) / 1e12
    out = {
        "metric": "sparse-MLA prefill TFLOP/s", "value": tflops, "unit": "TFLOP/s", "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 (fp8 KV dequant, fp32 acc)",
        "data": "synthetic (seeded N(0,1); FP8 no-rope rows with per-64 absmax scales)",
        "config": {"workload": "C3 sparse latent-MQA prefill", "B": 1, "S": C3["S"], "heads": C3["H"],
                   "d_qk": 576, "d_v": 512, "topk": C3["topk"], "window": C3["window"], "compressed": C3["G"],
                   "total_flops": total_flops,
                   "parallelism": (f"query tokens sharded over {world} GPUs (cyclic 128-token chunks, KV replicated,"
                                   " no collective in the step)" if world > 1 else "1 GPU"),
                   "o_gather_ms": gather_ms,
                   "l2": "inputs (2.4 GB q) larger than L2; 256 MB flush per step"},
        "e2e": {"value": total_flops / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "tensor", "kernel": "mzb::mla::mla_fwd_kernel", "achieved": achieved,
                     "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": achieved / pk["bf16_tflops"],
                     "peak_note": f"{pk['_source']} bf16 burst", "algorithmic_flops_per_launch": flops,
                     "ms_per_launch": ms, "traffic": TRAFFIC["prefill"],
                     "traffic_unit": "bytes per launch (ncu)"},
        "gpu_launches": 2 * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        toks = _prefill_sample(C3["S"], max(8, args.cpu_sample // 9))
        out["cpu_baseline"] = cpu_prefill(q[0, toks].float().cpu().numpy(), toks, raw[0].cpu().numpy(),
                                          cmp[0].cpu().numpy(), idx[0, toks].cpu().numpy())
    return out


def cpu_prefill(q_rows, toks, raw_rows, cmp_rows, idx_rows) -> dict:
    """Oracle port: sparse attention for the sampled query tokens (all 128 heads), reported
    as TFLOP/s of the sample's selected pairs (extrapolation to the full config is by
    selected-pair count)."""
    from oracle import mla as M
    t0 = time.perf_counter()
    pairs = 0
    for i, t in enumerate(toks):
        keys = M.unpack_rows(M.token_keys(raw_rows, cmp_rows, idx_rows[i], int(t), C3["window"]))
        pairs += keys.shape[0]
        M.attend_rows(q_rows[i], keys, 576**-0.5)
    dt = time.perf_counter() - t0
    flops = 2.0 * 128 * 1088 * pairs
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{len(toks)} evenly spaced query tokens x 128 heads ({pairs} selected pairs), numpy fp64, "
                      f"{dt:.2f} s, extrapolated by selected-pair count"}


def _prefill_sample(S, n_tok):
    import numpy as np
    return [int(t) for t in np.linspace(S // n_tok, S - 1, n_tok)]


def reference_prefill(args, rank, world) -> dict:
    import torch
    from oracle import mla as M
    if rank != 0:
        return None
    S = C3["S"]
    n_tok = max(8, args.cpu_sample // 256)
    toks = _prefill_sample(S, n_tok)
    g = torch.Generator().manual_seed(0)
    q_rows = torch.randn(n_tok, 128, 576, generator=g).to(torch.bfloat16).float().numpy()
    raw = M.pack_rows(torch.randn(S, 576, generator=g).numpy())
    cmp = M.pack_rows(torch.randn(C3["G"], 576, generator=g).numpy())
    idx = sorted_causal_indices(torch, S, C3["G"], C3["topk"], C3["ratio"], torch.Generator().manual_seed(1),
                                torch.device("cpu"))[toks].numpy()
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_prefill(q_rows, toks, raw, cmp, idx)
        if i >= args.warmup:
            vals.append(r["value"])
    v = statistics.mean(vals)
    r["value"] = v
    return {"metric": "sparse-MLA prefill TFLOP/s", "value": v, "unit": "TFLOP/s", "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f64 (oracle port)", "data": "synthetic",
            "config": {"workload": "C3 sparse latent-MQA prefill", "B": 1, "S": S, "heads": 128, "topk": C3["topk"],
                       "window": C3["window"]},
            "cpu_baseline": r, "e2e": {"value": v, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}

# ----------------------------------------------------------------------------- SWA train + fake quant (C5)

C5 = dict(B=4, S=8192, H=64, D=128, window=512)


def c5_band(cfg=C5) -> int:
    """Visible (query, key) pairs per (batch, head): sum_t min(t + 1, window)."""
    return sum(min(t + 1, cfg["window"]) for t in range(cfg["S"]))


def c5_flops(cfg=C5) -> tuple:
    fwd = 4.0 * cfg["B"] * cfg["H"] * cfg["D"] * c5_band(cfg)
    return fwd, 2.5 * fwd


def c5_step(q, k, v, do):
    """One training step of the path: fake quant (Q, K: OCP MXFP4 block 32; V: FP8 per-128
    absmax), window attention forward, backward; straight-through gradients."""
    from mzoo_b200 import quant, swa_attn
    qf = quant.fake_quant_fp4_block(q, 32, rule="ocp")
    kf = quant.fake_quant_fp4_block(k, 32, rule="ocp")
    vf = quant.fake_quant_fp8_block(v, 128, rule="absmax")
    o, lse = swa_attn.fwd(qf, kf, window=C5["window"], v=vf)
    dq, dk, _, dv = swa_attn.bwd(qf, kf, o, lse, do, window=C5["window"], v=vf)
    return dq, dk, dv  # STE: gradients w.r.t. the pre-quant inputs


def bench_train(args, torch, dist, rank, world, device) -> dict:
    from mzoo_b200 import quant, swa_attn
    B, S, H, D, W = (C5[x] for x in ("B", "S", "H", "D", "window"))
    g = torch.Generator(device=device).manual_seed(10 + rank)
    q = torch.randn(B, S, H, D, generator=g, device=device, dtype=torch.bfloat16)
    k = torch.randn(B, S, 1, D, generator=g, device=device, dtype=torch.bfloat16)
    v = torch.randn(B, S, 1, D, generator=g, device=device, dtype=torch.bfloat16)
    do = torch.randn(B, S, H, D, generator=g, device=device, dtype=torch.bfloat16)
    fwd_flops, bwd_flops = c5_flops()
    timer = Timer(torch, device)
    step = lambda: c5_step(q, k, v, do)  # noqa: E731
    sampler = ClockSampler(device.index)
    sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler.ready()
    if dist:
        dist.barrier()
    t_steps = timer.run(step, args.steps)
    clocks = sampler.stop(busy=step)
    # per-kernel legs for the roofline
    qf = quant.fake_quant_fp4_block(q, 32, rule="ocp")
    kf = quant.fake_quant_fp4_block(k, 32, rule="ocp")
    vf = quant.fake_quant_fp8_block(v, 128, rule="absmax")
    o, lse = swa_attn.fwd(qf, kf, window=W, v=vf)
    t_fwd = timer.run(lambda: swa_attn.fwd(qf, kf, window=W, v=vf), args.steps)
    t_bwd = timer.run(lambda: swa_attn.bwd(qf, kf, o, lse, do, window=W, v=vf), args.steps)
    t_fq = timer.run(lambda: quant.fake_quant_fp4_block(q, 32, rule="ocp"), args.steps)
    # end to end from pinned host memory
    hq, hk, hv, hdo = (x.cpu().pin_memory() for x in (q, k, v, do))
    dq_, dk_, dv_, ddo = (torch.empty_like(x, device=device) for x in (hq, hk, hv, hdo))
    hdq, hdk, hdv = (torch.empty_like(x).pin_memory() for x in (hq, hk, hv))

    def e2e():
        for d, h in ((dq_, hq), (dk_, hk), (dv_, hv), (ddo, hdo)):
            d.copy_(h, non_blocking=True)
        gq, gk, gv = c5_step(dq_, dk_, dv_, ddo)
        hdq.copy_(gq, non_blocking=True)
        hdk.copy_(gk, non_blocking=True)
        hdv.copy_(gv, non_blocking=True)

    e2e()
    t_e2e = timer.run(e2e, max(2, args.steps // 2), flush=False)
    h2d = sum(x.numel() * x.element_size() for x in (hq, hk, hv, hdo))
    d2h = sum(x.numel() * x.element_size() for x in (hdq, hdk, hdv))
    ms = max_over_ranks(torch, dist, sum(t_steps) / len(t_steps), device)
    ms_e2e = max_over_ranks(torch, dist, sum(t_e2e) / len(t_e2e), device)
    ms_fwd, ms_bwd, ms_fq = (sum(t) / len(t) for t in (t_fwd, t_bwd, t_fq))
    pk = peaks()
    total = fwd_flops + bwd_flops
    ach_bwd = bwd_flops / (ms_bwd * 1e-3) / 1e12
    fq_bytes = 2 * q.numel() * 2
    out = {
        "metric": "SWA train fwd+bwd TFLOP/s (fake-quant Q/K MXFP4, V FP8)", "value": total * world / (ms * 1e-3) / 1e12,
        "unit": "TFLOP/s", "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 (fp32 acc)", "data": "synthetic (seeded N(0,1) bf16 inputs and dO)",
        "config": {"workload": "C5 SWA train + fake quant", "B": B, "S": S, "heads": H, "head_dim": D, "window": W,
                   "fq": "Q,K OCP MXFP4 block 32; V FP8 absmax per 128; STE", "parallelism": f"x{world} independent",
                   "l2": "256 MB flush per step"},
        "e2e": {"value": total * world / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "tensor", "kernel": "mzb::attnb::dkv_kernel + dq_kernel (backward)",
                     "achieved": ach_bwd, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": ach_bwd / pk["bf16_tflops"], "peak_note": f"{pk['_source']} bf16 burst",
                     "algorithmic_flops_per_launch": bwd_flops, "ms_per_launch": ms_bwd,
                     "traffic": TRAFFIC["train"], "traffic_unit": "bytes per launch (ncu, dkv + dq kernels)"},
        "legs": {"fwd_ms": ms_fwd, "fwd_tflops": fwd_flops / (ms_fwd * 1e-3) / 1e12, "bwd_ms": ms_bwd,
                 "fq_q_ms": ms_fq, "fq_q_gbs": fq_bytes / (ms_fq * 1e-3) / 1e9},
        "gpu_launches": 7 * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_train(q, k, v, do, n_tok=max(16, args.cpu_sample // 2))
    return out


def cpu_train(q, k, v, do, n_tok: int) -> dict:
    """Oracle port: fake quant + window attention fwd/bwd (fp64 numpy) for n_tok query tokens
    of batch 0 (all 64 heads, full 512-key window each), as TFLOP/s of their band pairs."""
    import numpy as np
    from oracle import quant as Q
    S, W, D = C5["S"], C5["window"], C5["D"]
    toks = [int(t) for t in np.linspace(W, S - 1, n_tok)]
    qs = q[0].float().cpu().numpy()
    ks = k[0, :, 0].float().cpu().numpy()
    vs = v[0, :, 0].float().cpu().numpy()
    dos = do[0].float().cpu().numpy().astype(np.float64)
    t0 = time.perf_counter()
    pairs = 0
    for t in toks:
        lo = t - W + 1
        qq = Q.fake_quant_fp4(qs[t], 32, "ocp").astype(np.float64)
        kk = Q.fake_quant_fp4(ks[lo:t + 1], 32, "ocp").astype(np.float64)
        vv = Q.fake_quant_fp8(vs[lo:t + 1], 128, "absmax").astype(np.float64)
        z = qq @ kk.T * D**-0.5
        p = np.exp(z - z.max(1, keepdims=True))
        p /= p.sum(1, keepdims=True)
        o = p @ vv
        dp = dos[t] @ vv.T
        ds = p * (dp - (dos[t] * o).sum(1, keepdims=True))
        _ = (ds @ kk * D**-0.5, ds.T @ qq * D**-0.5, p.T @ dos[t])
        pairs += 64 * W
    dt = time.perf_counter() - t0
    flops = 4.0 * D * pairs * 3.5
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n_tok} query tokens x 64 heads x {W}-key window, numpy fp64 fake quant + fwd + bwd, "
                      f"{dt:.2f} s, extrapolated by band pairs"}


def reference_train(args, rank, world) -> dict:
    import torch
    if rank != 0:
        return None
    g = torch.Generator().manual_seed(10)
    S = C5["S"]
    q = torch.randn(1, S, 64, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(1, S, 1, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(1, S, 1, 128, generator=g).to(torch.bfloat16)
    do = torch.randn(1, S, 64, 128, generator=g).to(torch.bfloat16)
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_train(q, k, v, do, n_tok=max(16, args.cpu_sample // 128))
        if i >= args.warmup:
            vals.append(r["value"])
    val = statistics.mean(vals)
    r["value"] = val
    return {"metric": "SWA train fwd+bwd TFLOP/s (fake-quant Q/K MXFP4, V FP8)", "value": val, "unit": "TFLOP/s",
            "impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64 (oracle port)",
            "data": "synthetic", "config": {"workload": "C5 SWA train + fake quant", **C5},
            "cpu_baseline": r, "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ----------------------------------------------------------------------------- paged decode + indexer (C4)

C4 = dict(B=128, L_lo=8192, L_hi=131072, ratio=4, topk=2048, window=128, Hi=64, Di=128, page=64)


def c4_lens(torch, n=None):
    g = torch.Generator().manual_seed(1)
    return torch.randint(C4["L_lo"], C4["L_hi"] + 1, (C4["B"] if n is None else n,), generator=g)


def _random_rows(torch, n_rows: int, device, gen, chunk: int = 1 << 20):
    """n_rows KV rows of 672 B with valid e4m3 codes (no NaN), scales in [1/448, 4/448] and
    N(0,1) bf16 rope channels."""
    rows = torch.empty(n_rows, 672, dtype=torch.uint8, device=device)
    for r0 in range(0, n_rows, chunk):
        r1 = min(n_rows, r0 + chunk)
        n = r1 - r0
        codes = torch.randint(0, 255, (n, 512), generator=gen, device=device, dtype=torch.int32)
        codes = torch.where((codes & 0x7F) == 0x7F, codes - 1, codes).to(torch.uint8)
        rows[r0:r1, :512] = codes
        sc = (torch.rand(n, 8, generator=gen, device=device) * 3 + 1) / 448.0
        rows[r0:r1, 512:544] = sc.view(torch.uint8).view(n, 32)
        rope = torch.randn(n, 64, generator=gen, device=device).to(torch.bfloat16)
        rows[r0:r1, 544:] = rope.view(torch.uint8).view(n, 128)
    return rows


def c4_inputs(torch, device, seqs, lens):
    """Device inputs for the sequences `seqs` (global ids): paged raw / compressed latent
    caches with random page tables, dense per-sequence FP8 index keys, queries."""
    B = len(seqs)
    L = torch.tensor([int(lens[b]) for b in seqs], dtype=torch.int32)
    pages = (L + 63) // 64
    cl = L // C4["ratio"]
    cpages = (cl + 63) // 64
    g = torch.Generator(device=device).manual_seed(100 + seqs[0])
    gc = torch.Generator().manual_seed(200 + seqs[0])
    n_raw, n_cmp = int(pages.sum()), int(cpages.sum())
    pt = torch.full((B, int(pages.max())), 0, dtype=torch.int32)
    perm = torch.randperm(n_raw, generator=gc).to(torch.int32)
    o = 0
    for i in range(B):
        pt[i, :pages[i]] = perm[o:o + pages[i]]
        o += int(pages[i])
    cpt = torch.full((B, int(cpages.max())), 0, dtype=torch.int32)
    cperm = torch.randperm(n_cmp, generator=gc).to(torch.int32)
    o = 0
    for i in range(B):
        cpt[i, :cpages[i]] = cperm[o:o + cpages[i]]
        o += int(cpages[i])
    raw = _random_rows(torch, n_raw * 64, device, g).view(n_raw, 64, 672)
    cmp = _random_rows(torch, n_cmp * 64, device, g).view(n_cmp, 64, 672)
    T = int(cl.max())
    kcodes = torch.randint(0, 255, (B, T, C4["Di"]), generator=g, device=device, dtype=torch.int32)
    k8 = torch.where((kcodes & 0x7F) == 0x7F, kcodes - 1, kcodes).to(torch.uint8).view(torch.float8_e4m3fn)
    sk = (torch.rand(B, T, generator=g, device=device) * 3 + 1) / 448.0
    qcodes = torch.randint(0, 255, (B, 1, C4["Hi"], C4["Di"]), generator=g, device=device, dtype=torch.int32)
    q8 = torch.where((qcodes & 0x7F) == 0x7F, qcodes - 1, qcodes).to(torch.uint8).view(torch.float8_e4m3fn)
    sq = (torch.rand(B, 1, C4["Hi"], generator=g, device=device) * 3 + 1) / 448.0
    w = torch.randn(B, 1, C4["Hi"], generator=g, device=device) / 8
    q = torch.randn(B, 128, 576, generator=g, device=device, dtype=torch.bfloat16)
    dev = lambda t: t.to(device)  # noqa: E731
    return dict(q=q, raw=raw, pt=dev(pt), lens=dev(L), cmp=cmp, cpt=dev(cpt), cmp_lens=dev(cl.to(torch.int32)),
                q8=q8, sq=sq, k8=k8, sk=sk, w=w, pos=dev((L - 1).view(B, 1)))


def c4_step(x):
    from mzoo_b200 import indexer, sparse_mla
    idx = indexer.attn(x["q8"], x["k8"], x["w"], compress_ratio=C4["ratio"], topk=C4["topk"], scales=(x["sq"], x["sk"]),
                       q_pos=x["pos"], check=False)
    return sparse_mla.decode(x["q"], x["raw"], x["pt"], x["lens"], x["cmp"], x["cpt"], x["cmp_lens"], idx[:, 0],
                             window=C4["window"], check=False)


def c4_bytes(lens_sub) -> float:
    """Algorithmic HBM bytes of one decode step for these sequences."""
    tot = 0.0
    for L in lens_sub:
        L = int(L)
        tot += (L // C4["ratio"]) * (C4["Di"] + 4)                 # index keys + scales
        tot += min(L, C4["window"]) * 672 + min(C4["topk"], L // C4["ratio"]) * 672  # selected latent rows
        tot += 128 * 576 * 2 + 128 * 512 * 2 + 128 * 4             # q, o, lse
        tot += C4["Hi"] * (C4["Di"] + 8) + C4["topk"] * 4          # indexer q / scales / w, indices
    return tot


def bench_decode(args, torch, dist, rank, world, device) -> dict:
    lens = c4_lens(torch)
    from mzoo_b200.sharding import shard_sequences
    parts = shard_sequences(lens.tolist(), world)
    mine = parts[rank]
    x = c4_inputs(torch, device, mine, lens)
    nbytes = c4_bytes([lens[b] for b in mine])
    total_bytes = c4_bytes(lens.tolist())
    n_mine = len(mine)
    shard = max(len(p) for p in parts)  # greedy-by-length shards differ in count
    gather_buf = torch.empty(world * shard, 128, 512, dtype=torch.bfloat16, device=device) if dist else None

    def step():  # no collective: every sequence is independent
        o, lse = c4_step(x)
        return o

    timer = Timer(torch, device)
    sampler = ClockSampler(device.index)
    sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler.ready()
    if dist:
        dist.barrier()
    t_steps = timer.run(step, args.steps)
    clocks = sampler.stop(busy=step)
    gather_ms = None
    if dist:  # the optional output gather (every rank's o to every rank, padded shards), timed alone
        part = torch.zeros(shard, 128, 512, dtype=torch.bfloat16, device=device)
        part[:n_mine] = step()
        dist.all_gather_into_tensor(gather_buf, part)  # untimed: the collective's lazy setup
        t_g = timer.run(lambda: dist.all_gather_into_tensor(gather_buf, part), 3, flush=False)
        gather_ms = max_over_ranks(torch, dist, sum(t_g) / len(t_g), device)
    # dominant kernel legs
    from mzoo_b200 import indexer
    qp, kp, wp, sqp, skp, scale, dt = indexer._prep(x["q8"], x["k8"], x["w"], (x["sq"], x["sk"]), None)
    qpos = x["pos"].to(torch.int32).contiguous()
    t_score = timer.run(lambda: indexer._scores(qp, kp, wp, sqp, skp, C4["ratio"], 0, scale, dt, False, False, qpos),
                        args.steps)
    # e2e: queries / indexer queries / weights from pinned host memory, o back to the host
    hq, hq8, hw = x["q"].cpu().pin_memory(), x["q8"].view(torch.uint8).cpu().pin_memory(), x["w"].cpu().pin_memory()
    ho = torch.empty(n_mine, 128, 512, dtype=torch.bfloat16).pin_memory()

    def e2e():
        x["q"].copy_(hq, non_blocking=True)
        x["q8"].view(torch.uint8).copy_(hq8, non_blocking=True)
        x["w"].copy_(hw, non_blocking=True)
        o = step()
        ho.copy_(o, non_blocking=True)

    e2e()
    t_e2e = timer.run(e2e, args.steps, flush=False)
    ms = max_over_ranks(torch, dist, sum(t_steps) / len(t_steps), device)
    ms_e2e = max_over_ranks(torch, dist, sum(t_e2e) / len(t_e2e), device)
    ms_score = sum(t_score) / len(t_score)
    pk = peaks()
    score_bytes = sum((int(lens[b]) // 4) * (C4["Di"] + 4) + C4["Hi"] * (C4["Di"] + 8) for b in mine)
    ach = score_bytes / (ms_score * 1e-3) / 1e9
    out = {
        "metric": "paged sparse-MLA decode HBM GB/s (indexer + attention)", "value": total_bytes / (ms * 1e-3) / 1e9,
        "unit": "GB/s", "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e4m3 KV / bf16 q (fp32 acc)", "data": "synthetic (seeded lengths, random page tables, random FP8 rows)",
        "config": {"workload": "C4 paged decode + indexer", "sequences": C4["B"], "context": "U[8192,131072] seed 1",
                   "mean_context": float(lens.float().mean()), "heads": 128, "topk": C4["topk"],
                   "window": C4["window"], "page": 64, "algorithmic_bytes_per_step": total_bytes,
                   "parallelism": (f"sequences sharded over {world} GPUs (greedy by length), no collective in the "
                                   "step" if world > 1 else "1 GPU"),
                   "o_gather_ms": gather_ms,
                   "l2": "caches (~8 GB) larger than L2; 256 MB flush per step"},
        "e2e": {"value": total_bytes / (ms_e2e * 1e-3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": hq.numel() * 2 + hq8.numel() + hw.numel() * 4,
                "d2h_bytes_per_step": ho.numel() * 2},
        "roofline": {"bound": "hbm", "kernel": "mzb::idx::score_kernel<fp8,128,1> (decode indexer)", "achieved": ach,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": ach / pk["hbm_gbs"],
                     "peak_note": f"{pk['_source']} HBM copy", "algorithmic_bytes_per_launch": score_bytes,
                     "ms_per_launch": ms_score, "traffic": TRAFFIC["decode"], "traffic_unit": "bytes per launch (ncu)"},
        "gpu_launches": 6 * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_decode(min(C4["B"], max(1, args.cpu_sample // 32)))
    return out


def cpu_decode(n_seq: int) -> dict:
    """Oracle port of one decode step for n_seq sequences (the first of the seeded lengths):
    canonical fp64 indexer scores over L/4 FP8 keys -> exact top-2048 -> sparse attention
    over window + selected latent rows (numpy fp64), as GB/s of their algorithmic bytes."""
    import numpy as np
    import torch
    from oracle import indexer as I
    from oracle import mla as M
    lens = c4_lens(torch)[:n_seq].tolist()
    rng = np.random.default_rng(5)
    t_total = 0.0
    for L in lens:
        T = L // C4["ratio"]
        codes = rng.integers(0, 255, (T, C4["Di"]), dtype=np.uint8)
        codes[(codes & 0x7F) == 0x7F] -= 1
        kv = M.e4m3_values(codes)[None]
        qc = rng.integers(0, 255, (1, 1, C4["Hi"], C4["Di"]), dtype=np.uint8)
        qc[(qc & 0x7F) == 0x7F] -= 1
        qv = M.e4m3_values(qc)
        sk = ((rng.random((1, T)) * 3 + 1) / 448).astype(np.float32)
        sq = ((rng.random((1, 1, C4["Hi"])) * 3 + 1) / 448).astype(np.float32)
        w = (rng.standard_normal((1, 1, C4["Hi"])) / 8).astype(np.float32)
        raw_rows = M.pack_rows(rng.standard_normal((C4["window"], 576)).astype(np.float32))
        cmp_rows = M.pack_rows(rng.standard_normal((min(T, C4["topk"]), 576)).astype(np.float32))
        q = rng.standard_normal((128, 576)).astype(np.float32)
        t0 = time.perf_counter()
        sc = I.canonical_scores(qv, kv, w, sq, sk, C4["ratio"], L - 1)
        sel = I.canonical_topk(sc, C4["topk"], C4["ratio"], L - 1)[0, 0]
        keys = M.unpack_rows(np.concatenate([raw_rows, cmp_rows[:int((sel >= 0).sum())]], 0))
        M.attend_rows(q, keys, 576**-0.5)
        t_total += time.perf_counter() - t0
    nbytes = c4_bytes(lens)
    return {"value": nbytes / t_total / 1e9, "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
            "sample": f"{n_seq} sequences (L = {lens}), numpy fp64 canonical indexer + exact top-2048 + sparse "
                      f"attention, {t_total:.2f} s"}


def reference_decode(args, rank, world) -> dict:
    if rank != 0:
        return None
    n = max(1, args.cpu_sample // 2048)
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_decode(n)
        if i >= args.warmup:
            vals.append(r["value"])
    v = statistics.mean(vals)
    r["value"] = v
    return {"metric": "paged sparse-MLA decode HBM GB/s (indexer + attention)", "value": v, "unit": "GB/s",
            "impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f64 (oracle port)",
            "data": "synthetic", "config": {"workload": "C4 paged decode + indexer", "sequences": C4["B"]},
            "cpu_baseline": r, "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ----------------------------------------------------------------------------- two-level selection

# Level one over a candidate source's scores and level two over a later index source's, for
# the model's defaults (blocks of 8 compressed positions, top-2048 blocks, top-512 positions)
# at a context long enough for the block selection to bite: 65536 compressed positions
# (262144 tokens at ratio 4), the last 2048 queries of the sequence.
CF = dict(rows=2048, T=65536, block=8, topk_blocks=2048, topk=512)


def cf_inputs(torch, seed: int, rows=None):
    """Two score matrices [rows, T] ~ N(0,1), -inf past each query's compressed length, and
    the lengths (query r sees T - rows + r + 1 positions)."""
    rows = rows or CF["rows"]
    g = torch.Generator().manual_seed(seed)
    T = CF["T"]
    clen = torch.arange(T - CF["rows"] + 1, T - CF["rows"] + 1 + rows, dtype=torch.int32)
    vis = torch.arange(T).view(1, -1) < clen.view(-1, 1)
    mats = [torch.randn(rows, T, generator=g).masked_fill_(~vis, float("-inf")) for _ in range(2)]
    return mats[0], mats[1], clen


def bench_candidates(args, torch, dist, rank, world, device) -> dict:
    from mzoo_b200 import candidates as K
    lg_h, sc_h, cl_h = cf_inputs(torch, seed=0)
    mine = torch.arange(rank, CF["rows"], world)  # rows cyclic over ranks, no collective
    lg, sc, cl = (x[mine].contiguous().to(device) for x in (lg_h, sc_h, cl_h))
    rows = lg.shape[0]
    bs, tb, topk = CF["block"], CF["topk_blocks"], CF["topk"]

    def step():
        blocks = K.candidate_blocks(lg, cl, tb, bs)
        return K.candidate_topk(sc, blocks, topk, block_size=bs)

    timer = Timer(torch, device)
    sampler = ClockSampler(device.index)
    sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler.ready()
    if dist:
        dist.barrier()
    t_steps = timer.run(step, args.steps)
    blocks = K.candidate_blocks(lg, cl, tb, bs)
    t_l1 = timer.run(lambda: K.candidate_blocks(lg, cl, tb, bs), args.steps)
    t_l2 = timer.run(lambda: K.candidate_topk(sc, blocks, topk, block_size=bs), args.steps)
    # end to end through the public API from pinned host memory
    hlg, hsc, hcl = (x[mine].contiguous().pin_memory() for x in (lg_h, sc_h, cl_h))
    dlg, dsc, dcl = (torch.empty_like(x, device=device) for x in (hlg, hsc, hcl))
    hout = torch.empty(rows, topk, dtype=torch.int32).pin_memory()

    def e2e():
        for d, h in ((dlg, hlg), (dsc, hsc), (dcl, hcl)):
            d.copy_(h, non_blocking=True)
        b = K.candidate_blocks(dlg, dcl, tb, bs)
        hout.copy_(K.candidate_topk(dsc, b, topk, block_size=bs), non_blocking=True)

    for _ in range(2):
        e2e()
    t_e2e = timer.run(e2e, args.steps, flush=False)
    clocks = sampler.stop(busy=step)
    torch.cuda.synchronize()
    h2d = sum(x.numel() * x.element_size() for x in (hlg, hsc, hcl))
    d2h = hout.numel() * hout.element_size()

    ms = max_over_ranks(torch, dist, sum(t_steps) / len(t_steps), device)
    ms_e2e = max_over_ranks(torch, dist, sum(t_e2e) / len(t_e2e), device)
    ms_l1, ms_l2 = sum(t_l1) / len(t_l1), sum(t_l2) / len(t_l2)
    pk = peaks()
    # dominant kernel: the level-two top-k, which reads only the listed blocks' scores (plus the
    # block list) and writes the indices
    alg2 = rows * (CF["topk_blocks"] * CF["block"] * 4 + CF["topk_blocks"] * 4 + CF["topk"] * 4)
    achieved = alg2 / (ms_l2 * 1e-3) / 1e9
    out = {
        "metric": "two-level indexer selection Mq/s", "value": CF["rows"] / (ms * 1e-3) / 1e6, "unit": "Mq/s",
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32 keys (radix select on order-preserving uint32)",
        "data": "synthetic (seeded N(0,1) scores, -inf past each query's compressed length)",
        "config": {"workload": "F1 two-level selection: level-one candidate blocks + level-two top-k",
                   "queries": CF["rows"], "positions": CF["T"], "block_size": bs, "topk_blocks": tb, "topk": topk,
                   "parallelism": (f"query rows cyclic over {world} GPUs, no collective" if world > 1 else "1 GPU"),
                   "l2": "flushed (256 MB write) per step; inputs (2 x 512 MB) larger than L2"},
        "legs": {"level_one_ms": ms_l1, "level_two_ms": ms_l2,
                 "level_one_gbs": rows * CF["T"] * 4 / (ms_l1 * 1e-3) / 1e9},
        "e2e": {"value": CF["rows"] / (ms_e2e * 1e-3) / 1e6, "unit": "Mq/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "kernel": "mzb::cand::topk_gather_kernel (level two)", "achieved": achieved,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "peak_note": f"{pk['_source']} copy bandwidth", "algorithmic_bytes_per_launch": alg2,
                     "ms_per_launch": ms_l2, "traffic": TRAFFIC.get("candidates"),
                     "traffic_unit": "bytes per launch (ncu)"},
        "gpu_launches": 2 * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_candidates(lg_h, sc_h, cl_h, sample=max(1, min(CF["rows"], args.cpu_sample // 2)))
    return out


def cpu_candidates(lg, sc, cl, sample: int) -> dict:
    """Oracle port on the host: both levels for the first `sample` query rows."""
    from oracle import candidates as C
    lgn, scn, cln = lg[:sample].numpy(), sc[:sample].numpy(), cl[:sample].numpy()
    t0 = time.perf_counter()
    mask = C.candidate_mask_ref(lgn, cln, CF["topk_blocks"], CF["block"])
    C.candidate_topk_ref(scn, mask, CF["topk"])
    dt = time.perf_counter() - t0
    return {"value": sample / dt / 1e6, "unit": "Mq/s", "cores": 1, "kind": "port",
            "sample": f"{sample} query rows of {CF['T']} positions, numpy (lexsort per row), {dt:.2f} s"}


def reference_candidates(args, rank, world) -> dict:
    import torch
    if rank != 0:
        return None
    n = max(1, args.cpu_sample // 16)
    lg, sc, cl = cf_inputs(torch, seed=0, rows=n)
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_candidates(lg, sc, cl, sample=n)
        if i >= args.warmup:
            vals.append(r["value"])
    v = statistics.mean(vals)
    r["value"] = v
    return {"metric": "two-level indexer selection Mq/s", "value": v, "unit": "Mq/s", "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": CF["rows"] / (v * 1e6) * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64 (oracle port)", "data": "synthetic",
            "config": {"workload": "F1 two-level selection: level-one candidate blocks + level-two top-k",
                       "queries": CF["rows"], "positions": CF["T"], "block_size": CF["block"],
                       "topk_blocks": CF["topk_blocks"], "topk": CF["topk"]},
            "cpu_baseline": r, "e2e": {"value": v, "unit": "Mq/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ----------------------------------------------------------------------------- compressor producer step

# The compressor after its two fp32 projections, for a prefill batch: 8 sequences of 16384
# tokens at ratio 4 (4096 groups each), the V4.1 latent (576 channels, 64 of them rope),
# writing the pre-RoPE latent and the MXFP4 compressed-cache entry.
CP = dict(B=8, S=16384, ratio=4, D=576, rope=64)


def cp_inputs(torch, seed: int, B=None):
    B = B or CP["B"]
    g = torch.Generator().manual_seed(seed)
    G = CP["S"] // CP["ratio"]
    kv = torch.randn(B, CP["S"], CP["D"], generator=g)
    gate = torch.randn(B, CP["S"], CP["D"], generator=g) * 2
    w = (1 + 0.25 * torch.randn(CP["D"], generator=g)).to(torch.bfloat16)
    ang = torch.rand(B, G, CP["rope"] // 2, generator=g) * 6
    return kv, gate, w, ang.cos(), ang.sin()


def cp_bytes(B: int) -> float:
    """Algorithmic HBM bytes of one step: kv and gate read once, cos / sin read, two bf16 outputs."""
    G = CP["S"] // CP["ratio"]
    return B * (2 * CP["S"] * CP["D"] * 4 + 2 * G * (CP["rope"] // 2) * 4 + 2 * G * CP["D"] * 2)


def bench_compressor(args, torch, dist, rank, world, device) -> dict:
    from mzoo_b200 import compressor as K
    h = cp_inputs(torch, seed=0)
    mine = torch.arange(rank, CP["B"], world)  # sequences cyclic over ranks, no collective
    kv, gate, w, cos, sin = (x[mine].contiguous().to(device) if x.dim() > 1 else x.to(device) for x in h)
    B = kv.shape[0]
    step = lambda: K.compress(kv, gate, w, CP["ratio"], 1e-6, cos, sin)  # noqa: E731
    timer = Timer(torch, device)
    sampler = ClockSampler(device.index)
    sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler.ready()
    if dist:
        dist.barrier()
    t_steps = timer.run(step, args.steps)
    hkv, hgate, hcos, hsin = (x[mine].contiguous().pin_memory() for x in (h[0], h[1], h[3], h[4]))
    dkv, dgate, dcos, dsin = (torch.empty_like(x, device=device) for x in (hkv, hgate, hcos, hsin))
    G = CP["S"] // CP["ratio"]
    hlat = torch.empty(B, G, CP["D"], dtype=torch.bfloat16).pin_memory()
    hcache = torch.empty_like(hlat).pin_memory()

    def e2e():
        for d, x in ((dkv, hkv), (dgate, hgate), (dcos, hcos), (dsin, hsin)):
            d.copy_(x, non_blocking=True)
        lat, cache = K.compress(dkv, dgate, w, CP["ratio"], 1e-6, dcos, dsin)
        hlat.copy_(lat, non_blocking=True)
        hcache.copy_(cache, non_blocking=True)

    for _ in range(2):
        e2e()
    t_e2e = timer.run(e2e, args.steps, flush=False)
    clocks = sampler.stop(busy=step)
    torch.cuda.synchronize()
    h2d = sum(x.numel() * x.element_size() for x in (hkv, hgate, hcos, hsin))
    d2h = 2 * hlat.numel() * hlat.element_size()
    ms = max_over_ranks(torch, dist, sum(t_steps) / len(t_steps), device)
    ms_e2e = max_over_ranks(torch, dist, sum(t_e2e) / len(t_e2e), device)
    total = cp_bytes(CP["B"])  # the whole job
    local = cp_bytes(B)
    achieved = local / ((sum(t_steps) / len(t_steps)) * 1e-3) / 1e9
    pk = peaks()
    out = {
        "metric": "compressor producer step HBM GB/s (algorithmic bytes)", "value": total / (ms * 1e-3) / 1e9,
        "unit": "GB/s", "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32 pool, bf16 latent / cache", "data": "synthetic (seeded N(0,1) projections, random angles)",
        "config": {"workload": "F3 compressor: gated softmax pool + RMSNorm + RoPE + MXFP4 cache entry",
                   "B": CP["B"], "tokens": CP["S"], "compress_ratio": CP["ratio"], "head_dim": CP["D"],
                   "rope_dim": CP["rope"],
                   "parallelism": (f"sequences cyclic over {world} GPUs, no collective" if world > 1 else "1 GPU"),
                   "l2": "flushed (256 MB write) per step; inputs (604 MB) larger than L2"},
        "e2e": {"value": total / (ms_e2e * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "kernel": "mzb::comp::compress_kernel", "achieved": achieved,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "peak_note": f"{pk['_source']} copy bandwidth", "algorithmic_bytes_per_launch": local,
                     "ms_per_launch": sum(t_steps) / len(t_steps), "traffic": TRAFFIC.get("compressor"),
                     "traffic_unit": "bytes per launch (ncu)"},
        "gpu_launches": args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_compressor(h, n_groups=max(1, args.cpu_sample))
    return out


def cpu_compressor(h, n_groups: int) -> dict:
    """Oracle port on the host: latent + cache entry for the first n_groups groups of sequence 0."""
    import numpy as np
    import torch
    from oracle import compressor as Cm
    r = CP["ratio"]
    n = min(n_groups, CP["S"] // r)
    kv, gate = h[0][0:1, :n * r].numpy(), h[1][0:1, :n * r].numpy()
    w = h[2].view(torch.int16).numpy().view(np.uint16)
    cos, sin = h[3][0:1, :n].numpy(), h[4][0:1, :n].numpy()
    t0 = time.perf_counter()
    lat = Cm.latent_ref(kv, gate, w, 1e-6, r)
    Cm.cache_ref(lat, cos, sin)
    dt = time.perf_counter() - t0
    return {"value": cp_bytes(1) * n / (CP["S"] // r) / dt / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{n} groups of sequence 0, numpy, {dt:.2f} s"}


def reference_compressor(args, rank, world) -> dict:
    import torch
    if rank != 0:
        return None
    h = cp_inputs(torch, seed=0, B=1)
    vals = []
    for i in range(args.warmup + args.steps):
        r = cpu_compressor(h, n_groups=max(1, args.cpu_sample))
        if i >= args.warmup:
            vals.append(r["value"])
    v = statistics.mean(vals)
    r["value"] = v
    return {"metric": "compressor producer step HBM GB/s (algorithmic bytes)", "value": v, "unit": "GB/s",
            "impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cp_bytes(CP["B"]) / (v * 1e9) * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64 (oracle port)", "data": "synthetic",
            "config": {"workload": "F3 compressor: gated softmax pool + RMSNorm + RoPE + MXFP4 cache entry",
                       "B": CP["B"], "tokens": CP["S"], "compress_ratio": CP["ratio"], "head_dim": CP["D"],
                       "rope_dim": CP["rope"]},
            "cpu_baseline": r, "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


BENCHES = {"indexer": (bench_indexer, reference_indexer), "prefill": (bench_prefill, reference_prefill),
           "train": (bench_train, reference_train), "decode": (bench_decode, reference_decode),
           "candidates": (bench_candidates, reference_candidates),
           "compressor": (bench_compressor, reference_compressor)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="indexer", choices=sorted(BENCHES))
    ap.add_argument("--impl", default="mzb", choices=["mzb", "reference"])
    ap.add_argument("--cpu-sample", type=int, default=4096,
                    help="size of the timed CPU baseline sample (about 10 s of host work at the default)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--small", action="store_true",
                    help="shrunken workload (profiling captures only; not a bench number)")
    args = ap.parse_args()
    if args.small:  # a few hundred MB on the device: safe for multi-pass ncu captures
        C2.update(S=1024, q_offset=4096 - 1024)
        C3.update(S=2048)
        C5.update(B=1, S=2048)
        C4.update(B=8)
        CF.update(rows=256)
        CP.update(B=1, S=4096)
        args.no_cpu_baseline = True
    assert args.warmup >= 3 or args.impl == "reference", "at least 3 warm-up steps"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        res = BENCHES[args.config][1](args, rank, world)
        if res is not None:
            print(json.dumps(res), flush=True)
        return

    import torch
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    res = BENCHES[args.config][0](args, torch, dist, rank, world, device)
    res.update({"n_gpus": world, "steps": args.steps, "warmup": args.warmup})
    if rank == 0:
        print(json.dumps(res), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
