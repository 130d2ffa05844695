#!/usr/bin/env python
"""Benchmark of the mzoo attention hot path on B200 (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl mzb|reference]

Configs (BASELINE.json ``configs``; synthetic seeded inputs with the stated shapes and
distributions -- there is no dataset):

- ``prefill`` (default, configs[2]): sparse latent MQA over FP8 576/512 rows, 16384 tokens x
  128 heads, top-2048 compressed entries + a 128-token window.  Metric: TFLOP/s.
- ``window``: sliding-window MQA forward, B=1, S=2048, 16 heads, D=128,
  window 128, fp32 inputs and outputs.  Metric: TFLOP/s.
- ``indexer``: lightning indexer + top-512 over FP8 q/k, B=2, 4096 queries at
  absolute positions 12288..16383 x 4096 compressed keys (ratio 4), Hi=64, Di=128.
  Metric: indexer Mq/s (queries per second, whole job).
- ``decode``: paged decode of 128 sequences (lengths 8k..131k), decode indexer
  + top-2048 + window 128.  Metric: algorithmic HBM GB/s.
- ``train``: window attention training step, B=4, S=8192, 64 heads, D=128,
  window 512, MXFP4 / FP8 fake quant of q, k, v.  Metric: TFLOP/s.
- ``candidates`` (next row F1, not a BASELINE config): two-level indexer selection, 2048
  queries x 65536 compressed positions.  Metric: Mq/s.
- ``compressor`` (next row F3, not a BASELINE config): compressor pool + RMSNorm + RoPE +
  MXFP4 cache entry, 8 x 16384 tokens at ratio 4, 576 channels.  Metric: algorithmic HBM GB/s.
- ``normrope`` (next row F3, not a BASELINE config): the fused RMSNorm + RoPE prologue of q,
  forward + backward, at the reference's own benchmark shape (B1 S4096 H64 D128, rope 64).
  Metric: algorithmic HBM GB/s.

A "step" is one pass of the hot path over one batch.  ``value`` times the device path with
inputs resident in HBM (L2 flushed with a 256 MB write before every timed step);
``e2e`` times the public API call with pinned host inputs, host->device copies, the
kernels and the device->host copy of the result inside the timed region.  Multi-GPU:
one process per GPU (torchrun); the indexer, prefill, decode, candidates and compressor
configs split one workload's independent units (query chunks, token chunks, sequences,
query rows, sequences) over the ranks with no data-path collective (strong scaling), the
window and training configs run one instance per rank (weak scaling); timing is the max
over ranks of CUDA-event time.

``--impl reference`` times the reference's CPU arithmetic -- its float32 PyTorch path
(``golden_ref.py``, ``quant.py``) as restated in ``oracle/torch_ref.py``; the reference
itself is Python and cannot travel to the GPU host -- on the host cores (all threads), one
bounded sample of the same workload per step (stated in ``cpu_baseline.sample``; the
printed ``ms_per_step`` is the time of that sample, ``value`` the metric over it), with the
same ``config`` as this build's line.  The ``cpu_baseline`` of this build's line (rank 0,
one GPU) times the same sample once and compares the GPU's rows for it with the CPU result
(``cpu_baseline.parity``).
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


# DRAM bytes (read + write) of one full-size launch of each config's roofline kernel at one
# GPU, from a one-pass ncu capture of this build (dram__bytes_read.sum + dram__bytes_write.sum).
# A rank of a multi-GPU run reports it scaled by its share of the work (``traffic_for``).
TRAFFIC_N1 = {
    "indexer": 72764928 + 69933824,
    "prefill": 2533523200 + 2108656128,
    "decode": 313127680 + 10324480,
    "train": (1469937152 + 86258176) + (1107655936 + 505236480),  # dkv_kernel + dq_kernel
    "candidates": 381950464 + 3411200,  # level two (gathered): 32-byte blocks cost ~2.8x in DRAM bursts
    "compressor": 612400896 + 68001536,
}


def traffic_for(name: str, share: float) -> dict:
    """The roofline's ``traffic`` fields: the N=1 capture scaled by this rank's share of the
    job's algorithmic work (1.0 at one GPU)."""
    t = TRAFFIC_N1.get(name)
    if t is None:
        return {"traffic": None}
    note = "bytes per launch (ncu one-pass capture, full-size workload, 1 GPU)"
    if abs(share - 1.0) > 1e-9:
        note += f", scaled by this rank's {share:.4f} share of the work"
    return {"traffic": t * share, "traffic_unit": note}


def cpu_threads(torch) -> int:
    """All host threads for the CPU arms."""
    torch.set_num_threads(os.cpu_count() or 1)
    return torch.get_num_threads()


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


class Pipeline:
    """End-to-end step in chunks on three streams: chunk c's host-to-device copies (copy
    stream in), its kernels (the current stream) and its device-to-host copies (copy stream
    out) overlap with the neighbouring chunks' -- PCIe runs both directions at once, so the
    step costs about its larger transfer instead of the sum.  Every copy and launch of the
    step is enqueued between the timer's events: the streams join the current stream at both
    ends of `run`."""

    def __init__(self, torch, device):
        self.torch = torch
        self.s_in = torch.cuda.Stream(device)
        self.s_out = torch.cuda.Stream(device)

    def run(self, n: int, h2d, compute, d2h, prologue=None):
        """h2d(c) enqueues chunk c's input copies, compute(c) its kernels (returns tensors),
        d2h(c, result) its output copies; prologue() copies inputs every chunk shares."""
        torch = self.torch
        cur = torch.cuda.current_stream()
        start = torch.cuda.Event()
        start.record(cur)
        self.s_in.wait_event(start)
        ev_in, ev_done = [], []
        with torch.cuda.stream(self.s_in):
            if prologue is not None:
                prologue()
            for c in range(n):
                h2d(c)
                ev = torch.cuda.Event()
                ev.record(self.s_in)
                ev_in.append(ev)
        for c in range(n):
            cur.wait_event(ev_in[c])
            res = compute(c)
            ev = torch.cuda.Event()
            ev.record(cur)
            self.s_out.wait_event(ev)
            with torch.cuda.stream(self.s_out):
                for t in res:  # the caching allocator must not hand these out before the copy
                    t.record_stream(self.s_out)
                d2h(c, res)
        end = torch.cuda.Event()
        end.record(self.s_out)
        cur.wait_event(end)


def _graph(torch, device, fn):
    """A CUDA graph of fn's launches (captured on a side stream after one eager call)."""
    g = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(device)
    cap.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(cap):
        fn()
        with torch.cuda.graph(g, stream=cap):
            fn()
    torch.cuda.current_stream(device).wait_stream(cap)
    g.replay()
    torch.cuda.synchronize()
    return g


def max_over_ranks(torch, dist, value: float, device) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- window attention (C1)

C1 = dict(B=1, S=2048, H=16, D=128, window=128)


def c1_flops() -> float:
    """Algorithmic forward FLOPs: 4 * B * H * D * sum_t min(t + 1, window)."""
    band = sum(min(t + 1, C1["window"]) for t in range(C1["S"]))
    return 4.0 * C1["B"] * C1["H"] * C1["D"] * band


def c1_inputs(torch, seed: int = 0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(C1["B"], C1["S"], C1["H"], C1["D"], generator=g)
    kv = torch.randn(C1["B"], C1["S"], 1, C1["D"], generator=g)
    return q, kv


def c1_config(world: int) -> dict:
    return {"workload": "C1 sliding-window MQA forward", "B": C1["B"], "S": C1["S"], "heads": C1["H"],
            "head_dim": C1["D"], "window": C1["window"], "inputs": "fp32 q / kv, fp32 o + lse out",
            "parallelism": f"x{world} independent" if world > 1 else "1 GPU",
            "l2": "256 MB flush per step"}


def bench_window(args, torch, dist, rank, world, device) -> dict:
    from mzoo_b200 import swa_attn
    qh, kvh = c1_inputs(torch)
    q, kv = qh.to(device), kvh.to(device)
    W = C1["window"]

    def step():  # fp32 in, bf16 kernel, fp32 out (o; lse is fp32 already)
        o, lse = swa_attn.fwd(q.to(torch.bfloat16), kv.to(torch.bfloat16), window=W)
        return o.float(), lse

    timer = Timer(torch, device)
    sampler = ClockSampler(device.index)
    sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # A step is ~2 GFLOP: launched one op at a time it is bound by the host's launch rate,
    # so the timed step replays a CUDA graph of the same launches (captured after warm-up).
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(device)
    cap.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(cap):
        step()
        with torch.cuda.graph(graph, stream=cap):
            o_graph, lse_graph = step()
    torch.cuda.current_stream(device).wait_stream(cap)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    sampler.ready()
    if dist:
        dist.barrier()
    t_steps = timer.run(graph.replay, args.steps)
    clocks = sampler.stop(busy=graph.replay, min_samples=2)
    qb, kvb = q.to(torch.bfloat16), kv.to(torch.bfloat16)
    kgraph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(cap):
        swa_attn.fwd(qb, kvb, window=W)
        with torch.cuda.graph(kgraph, stream=cap):
            swa_attn.fwd(qb, kvb, window=W)
    torch.cuda.current_stream(device).wait_stream(cap)
    kgraph.replay()
    t_k = timer.run(kgraph.replay, args.steps)
    hq, hkv = qh.pin_memory(), kvh.pin_memory()
    dq, dkv = torch.empty_like(q), torch.empty_like(kv)
    ho = torch.empty(qh.shape, dtype=torch.float32).pin_memory()
    hl = torch.empty(C1["B"], C1["H"], C1["S"], dtype=torch.float32).pin_memory()

    def e2e():
        dq.copy_(hq, non_blocking=True)
        dkv.copy_(hkv, non_blocking=True)
        o, lse = swa_attn.fwd(dq.to(torch.bfloat16), dkv.to(torch.bfloat16), window=W)
        ho.copy_(o, non_blocking=True)  # bf16 -> fp32 on the copy
        hl.copy_(lse, non_blocking=True)

    for _ in range(2):
        e2e()
    t_e2e = timer.run(e2e, args.steps, flush=False)
    o_gpu, lse_gpu = step()
    torch.cuda.synchronize()
    assert torch.equal(o_gpu, o_graph) and torch.equal(lse_gpu, lse_graph), "graph replay differs from the step"
    ms = max_over_ranks(torch, dist, sum(t_steps) / len(t_steps), device)
    ms_e2e = max_over_ranks(torch, dist, sum(t_e2e) / len(t_e2e), device)
    ms_k = sum(t_k) / len(t_k)
    flops = c1_flops()
    pk = peaks()
    ach = flops / (ms_k * 1e-3) / 1e12
    out = {
        "metric": "sliding-window MQA forward TFLOP/s", "value": flops * world / (ms * 1e-3) / 1e12,
        "unit": "TFLOP/s", "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 (fp32 inputs cast on the device, fp32 acc)", "data": "synthetic (seeded N(0,1) fp32)",
        "config": c1_config(world),
        "timing": "value: CUDA-graph replay of the step's launches (casts, window kernel, cast back); e2e: the "
                  "public API called op by op with host copies",
        "e2e": {"value": flops * world / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
                "h2d_bytes_per_step": (hq.numel() + hkv.numel()) * 4,
                "d2h_bytes_per_step": (ho.numel() + hl.numel()) * 4},
        "roofline": {"bound": "tensor", "kernel": "mzb::attn::attn_fwd_kernel<128>", "achieved": ach,
                     "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": ach / pk["bf16_tflops"],
                     "peak_note": f"{pk['_source']} bf16 burst; 2 GFLOP per launch is latency-bound, not "
                                  "tensor-bound", "algorithmic_flops_per_launch": flops, "ms_per_launch": ms_k,
                     "traffic": None},
        "gpu_launches": 4 * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = cpu_window(torch, qh, kvh)
        ro, rl = r.pop("result")
        eo = (o_gpu.cpu() - ro).abs().max().item()
        el = (lse_gpu.cpu() - rl).abs().max().item()
        r["parity"] = {"rows": "all", "max_abs_err_o": eo, "max_abs_err_lse": el, "atol": 2e-2,
                       "ok": bool(eo <= 2e-2 and el <= 2e-2),
                       "note": "GPU output (bf16 kernel) vs the CPU float32 reference on the whole config"}
        out["cpu_baseline"] = r
    return out


def cpu_window(torch, q, kv) -> dict:
    """The reference's CPU path for this config, ``golden(q, kv, level="window", window=128)``
    (its float32 ``_attend`` with the band mask), on the whole config, all host threads."""
    from oracle import torch_ref as R
    cores = cpu_threads(torch)
    t0 = time.perf_counter()
    o, lse = R.window_attention(q, kv, C1["window"])
    dt = time.perf_counter() - t0
    return {"value": c1_flops() / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port", "ms": dt * 1e3,
            "sample": f"the whole config: torch float32 golden(level='window') arithmetic (dense masked "
                      f"_attend), {dt:.3f} s; FLOPs counted for the visible band only",
            "result": (o, lse)}


def reference_window(args, rank, world) -> dict:
    import torch
    if rank != 0:
        return None
    q, kv = c1_inputs(torch)
    runs = []
    for _ in range(args.warmup + args.steps):
        r = cpu_window(torch, q, kv)
        r.pop("result")
        runs.append(r)
    return _reference_line(args, world, "sliding-window MQA forward TFLOP/s", "TFLOP/s", c1_config(world), runs,
                           "f32 (reference CPU path)", "synthetic (seeded N(0,1) fp32)", scaling="weak")


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


def c2_config(world: int) -> dict:
    return {"workload": "C2 lightning indexer + top-k", "B": C2["B"], "queries": C2["S"], "keys": C2["T"],
            "Hi": C2["Hi"], "Di": C2["Di"], "compress_ratio": C2["ratio"], "topk": C2["topk"],
            "q_offset": C2["q_offset"],
            "parallelism": (f"(batch x 128-query chunk) units cyclic over {world} GPUs, keys replicated, no "
                            "collective in the step; the optional index gather timed on its own (legs)"
                            if world > 1 else "1 GPU"),
            "l2": "flushed (256 MB write) per step"}


def bench_indexer(args, torch, dist, rank, world, device) -> dict:
    from mzoo_b200 import indexer

    from mzoo_b200.sharding import shard_tokens
    q, k, w_host = c2_inputs(torch, seed=0)  # the same workload on every rank
    q8, sq = indexer.quantize_fp8(q.to(device))
    k8, sk = indexer.quantize_fp8(k.to(device))
    w = w_host.to(device)
    B, S, T, Hi, Di = (C2[x] for x in ("B", "S", "T", "Hi", "Di"))
    kw = dict(compress_ratio=C2["ratio"], topk=C2["topk"], q_offset=C2["q_offset"], scales=(sq, sk))
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
    g_step = _graph(torch, device, step)  # the step's launches replayed: no host launch gaps
    sampler.ready()
    if dist:
        dist.barrier()
    t_steps = timer.run(g_step.replay, args.steps)
    # the dominant kernel alone (score GEMM), for the roofline
    qp, kp, wp, sqp, skp, scale, dt = indexer._prep(q8, k8, w, (sq, sk), None)
    qpos = kw.get("q_pos")
    qpos = qpos.contiguous() if qpos is not None else None
    g_score = _graph(torch, device, lambda: indexer._scores(qp, kp, wp, sqp, skp, C2["ratio"], C2["q_offset"],
                                                             scale, dt, False, False, qpos))
    t_score = timer.run(g_score.replay, args.steps)  # graph replay: the kernel's time, no host launch gap
    # end to end through the public API from pinned host memory
    hq8 = q8.view(torch.uint8).cpu().pin_memory()
    hk8 = k8.view(torch.uint8).cpu().pin_memory()
    hsq, hsk, hw = (x.cpu().pin_memory() for x in (sq, sk, w))
    dq8, dk8 = torch.empty_like(hq8, device=device), torch.empty_like(hk8, device=device)
    dsq, dsk, dw = (torch.empty_like(x, device=device) for x in (hsq, hsk, hw))
    hout = torch.empty(B, len(toks), C2["topk"], dtype=torch.int32).pin_memory()

    # the step in chunks (batch x halves of the query axis) through the public API, each
    # chunk's copies overlapping the neighbouring chunks' kernels and copies
    n_loc = len(toks)
    halves = 2 if n_loc >= 256 else 1
    chunks = [(b, n_loc * h // halves, n_loc * (h + 1) // halves) for b in range(B) for h in range(halves)]
    qpos_all = kw.get("q_pos")
    if qpos_all is None:
        qpos_all = (torch.arange(n_loc, device=device, dtype=torch.int32) + C2["q_offset"]).view(1, -1).expand(B, -1)
    qpos_ch = [qpos_all[b:b + 1, a:e].contiguous() for b, a, e in chunks]
    pipe = Pipeline(torch, device)

    def e2e():
        def prologue():
            dk8.copy_(hk8, non_blocking=True)
            dsk.copy_(hsk, non_blocking=True)

        def h2d(c):
            b, a, e = chunks[c]
            dq8[b, a:e].copy_(hq8[b, a:e], non_blocking=True)
            dsq[b, a:e].copy_(hsq[b, a:e], non_blocking=True)
            dw[b, a:e].copy_(hw[b, a:e], non_blocking=True)

        def compute(c):
            b, a, e = chunks[c]
            return (indexer.attn(dq8[b:b + 1, a:e].view(torch.float8_e4m3fn), dk8[b:b + 1].view(torch.float8_e4m3fn),
                                 dw[b:b + 1, a:e], compress_ratio=C2["ratio"], topk=C2["topk"],
                                 scales=(dsq[b:b + 1, a:e], dsk[b:b + 1]), q_pos=qpos_ch[c]),)

        def d2h(c, res):
            b, a, e = chunks[c]
            hout[b, a:e].copy_(res[0][0], non_blocking=True)

        pipe.run(len(chunks), h2d, compute, d2h, prologue)

    for _ in range(2):
        e2e()
    t_e2e = timer.run(e2e, args.steps, flush=False)
    clocks = sampler.stop(busy=step)
    torch.cuda.synchronize()
    out_idx = indexer.attn(q8, k8, w, **dict(kw, check=True))  # one checked call: raises on a device error word
    assert torch.equal(hout, out_idx.cpu()), "e2e index sets differ from the device step"
    gather_ms = None
    if dist:  # the optional index gather (every rank's rows to every rank, padded shards), timed alone
        width = max(len(p) for p in shard_tokens(S, world, 128))
        pad = out_idx.new_full((B, width, C2["topk"]), -1)
        pad[:, :len(toks)] = out_idx
        gbuf = out_idx.new_empty((world, B, width, C2["topk"]))
        dist.all_gather_into_tensor(gbuf, pad)  # untimed: the collective's lazy setup
        t_g = timer.run(lambda: dist.all_gather_into_tensor(gbuf, pad), 3, flush=False)
        gather_ms = max_over_ranks(torch, dist, sum(t_g) / len(t_g), device)
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
        "config": c2_config(world),
        "timing": "value: CUDA-graph replay of the step's launches; e2e: the public API op by op",
        "legs": {"idx_gather_ms": gather_ms},
        "e2e": {"value": queries / (ms_e2e * 1e-3) / 1e6, "unit": "Mq/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "note": f"indexer.attn on {len(chunks)} chunks (batch x query halves), each chunk's H2D / kernels / "
                        "D2H overlapped with its neighbours' on three streams"},
        "roofline": {"bound": "tensor", "kernel": "mzb::idx::score_kernel<fp8,128,2>", "achieved": achieved,
                     "peak": fp8_peak, "unit": "TFLOP/s", "frac": achieved / fp8_peak,
                     "peak_note": f"dense FP8 = 2 x {pk['_source']} bf16 burst {pk['bf16_tflops']} TFLOP/s",
                     "algorithmic_flops_per_launch": flops, "ms_per_launch": ms_score,
                     **traffic_for("indexer", len(toks) / S)},
        "gpu_launches": 3 * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = cpu_indexer(torch, q, k, w_host)
        got = out_idx[0, C2["S"] - r.pop("n"):].cpu()
        ref = r.pop("result")
        r["parity"] = {"rows": int(got.shape[0]), "equal_sets": int(_set_equal_rows(torch, got, ref)),
                       "note": "GPU index sets vs the CPU float32 reference's top-k sets on the sample rows"}
        out["cpu_baseline"] = r
    return out


def _set_equal_rows(torch, a, b) -> int:
    """Rows of two [rows, topk] index lists that hold the same set (-1 = empty)."""
    big = 1 << 30
    sa = torch.where(a < 0, big, a.long()).sort(-1).values
    sb = torch.where(b < 0, big, b.long()).sort(-1).values
    return int((sa == sb).all(-1).sum())


def cpu_indexer(torch, q, k, w, n: int = 512) -> dict:
    """The reference's float32 CPU path (``indexer_scores`` + ``topk_indices``) on the last
    ``n`` queries of batch 0, with the FP8 inputs dequantised (q * s_q, k * s_k), all host
    threads.  Returns the metric over the sample and the sample's index sets."""
    from oracle import torch_ref as R
    cores = cpu_threads(torch)
    q8, sq = _fp8_absmax_cpu(torch, q[0:1, -n:])
    k8, sk = _fp8_absmax_cpu(torch, k[0:1])
    off = C2["q_offset"] + C2["S"] - n
    t0 = time.perf_counter()
    qd = q8.float() * sq.unsqueeze(-1)
    kd = k8.float() * sk.unsqueeze(-1)
    sc = R.indexer_scores(qd, kd, w[0:1, -n:], C2["ratio"], off, scale=1.0)
    idx = R.topk_indices(sc, C2["topk"])
    dt = time.perf_counter() - t0
    return {"value": n / dt / 1e6, "unit": "Mq/s", "cores": cores, "kind": "port", "ms": dt * 1e3,
            "sample": f"{n} queries of batch 0 (positions {off}..{off + n - 1}) x {C2['T']} keys: torch float32 "
                      f"indexer_scores + topk_indices (the reference's CPU arithmetic), {dt:.2f} s",
            "n": n, "result": idx[0]}


def _fp8_absmax_cpu(torch, x):
    """Absmax e4m3 codes and fp32 scales per row of the last dim (the synthetic inputs' rule)."""
    xf = x.float()
    amax = xf.abs().amax(-1)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    return (xf / scale.unsqueeze(-1)).clamp(-448, 448).to(torch.float8_e4m3fn), scale


def _reference_line(args, world, metric, unit, cfg, runs, dtype, data, scaling="strong") -> dict:
    """The reference arm's JSON line from per-step CPU-sample results ``runs`` (the last
    ``args.steps`` are timed; ``ms_per_step`` is the sample's own time)."""
    timed = runs[args.warmup:]
    v = statistics.mean(r["value"] for r in timed)
    ms = statistics.mean(r["ms"] for r in timed)
    cb = {k: timed[-1][k] for k in ("unit", "cores", "kind", "sample")}
    cb["value"] = v
    return {"metric": metric, "value": v, "unit": unit, "impl": "reference", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": scaling,
            "vs_baseline": None,
            "dtype": dtype, "data": data, "config": cfg, "cpu_baseline": cb,
            "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def reference_indexer(args, rank, world) -> dict:
    import torch
    if rank != 0:
        return None
    q, k, w = c2_inputs(torch, seed=0)
    runs = []
    for _ in range(args.warmup + args.steps):
        r = cpu_indexer(torch, q, k, w)
        r.pop("result")
        runs.append(r)
    return _reference_line(args, world, "indexer Mq/s", "Mq/s", c2_config(world), runs,
                           "f32 (reference CPU arithmetic, FP8 inputs dequantised)",
                           "synthetic (seeded N(0,1), absmax fp8)")


# ----------------------------------------------------------------------------- sparse MLA prefill (C3)

C3 = dict(B=1, S=16384, H=128, G=4096, ratio=4, topk=2048, window=128)


def sorted_causal_indices(torch, S, G, topk, ratio, gen, device, q_offset=0, chunk=2048, positions=None):
    """Per query t: seeded random distinct compressed indices from [0, (t+q_offset+1)//ratio),
    the first topk of a random permutation, sorted ascending, -1 padded.  ``positions``
    (a list) gives the query positions explicitly instead of q_offset..q_offset+S-1."""
    pos_all = (torch.arange(S, device=device) + q_offset if positions is None
               else torch.tensor(positions, device=device))
    S = pos_all.shape[0]
    out = torch.empty(S, topk, dtype=torch.int32, device=device)
    cols = torch.arange(G, device=device)
    for s0 in range(0, S, chunk):
        s1 = min(S, s0 + chunk)
        r = torch.rand(s1 - s0, G, generator=gen, device=device)
        vis = (pos_all[s0:s1] + 1) // ratio
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


def c3_config(world: int) -> dict:
    return {"workload": "C3 sparse latent-MQA prefill", "B": 1, "S": C3["S"], "heads": C3["H"], "d_qk": 576,
            "d_v": 512, "topk": C3["topk"], "window": C3["window"], "compressed": C3["G"],
            "parallelism": (f"query tokens sharded over {world} GPUs (cyclic 128-token chunks, KV replicated,"
                            " no collective in the step)" if world > 1 else "1 GPU"),
            "l2": "inputs (2.4 GB q) larger than L2; 256 MB flush per step"}


def bench_prefill(args, torch, dist, rank, world, device) -> dict:
    from mzoo_b200 import sparse_mla
    from mzoo_b200.sharding import shard_tokens
    q, raw, cmp, idx = c3_inputs(torch, device, seed=0)  # the same workload on every rank
    total_flops = sparse_mla.pair_flops(c3_pairs(torch, idx))
    pos, toks = None, None
    q_full, idx_full = q, idx
    if world > 1:  # this rank's cyclic 128-token chunks of the query axis; KV replicated
        toks = shard_tokens(C3["S"], world, 128)[rank]
        tk = torch.tensor(toks, device=device)
        q, idx = q[:, tk].contiguous(), idx[:, tk].contiguous()
        pos = tk.to(torch.int32).view(1, -1)
    flops = sparse_mla.pair_flops(c3_pairs(torch, idx, toks))
    n_q = q.shape[1]
    step = lambda: sparse_mla.prefill(q, raw, cmp, idx, window=C3["window"], q_pos=pos)  # noqa: E731
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

    # the step in chunks of the query axis through the public API (explicit positions), the
    # copies of one chunk overlapping the kernels and copies of its neighbours
    n_ch = 8 if n_q >= 8 * 128 else 1
    bounds = [n_q * c // n_ch for c in range(n_ch + 1)]
    pos_all = pos if pos is not None else torch.arange(n_q, device=device, dtype=torch.int32).view(1, -1)
    pos_ch = [pos_all[:, bounds[c]:bounds[c + 1]].contiguous() for c in range(n_ch)]
    hl_ch = [torch.empty(1, C3["H"], bounds[c + 1] - bounds[c], dtype=torch.float32).pin_memory()
             for c in range(n_ch)]
    pipe = Pipeline(torch, device)

    def e2e():
        def prologue():
            draw.copy_(hraw, non_blocking=True)
            dcmp.copy_(hcmp, non_blocking=True)

        def h2d(c):
            a, b = bounds[c], bounds[c + 1]
            dq[:, a:b].copy_(hq[:, a:b], non_blocking=True)
            didx[:, a:b].copy_(hidx[:, a:b], non_blocking=True)

        def compute(c):
            a, b = bounds[c], bounds[c + 1]
            return sparse_mla.prefill(dq[:, a:b], draw, dcmp, didx[:, a:b], window=C3["window"], q_pos=pos_ch[c])

        def d2h(c, res):
            a, b = bounds[c], bounds[c + 1]
            ho[:, a:b].copy_(res[0], non_blocking=True)
            hl_ch[c].copy_(res[1], non_blocking=True)

        pipe.run(n_ch, h2d, compute, d2h, prologue)

    e2e()
    t_e2e = timer.run(e2e, max(2, args.steps // 4), flush=False)
    h2d = sum(x.numel() * x.element_size() for x in (hq, hraw, hcmp, hidx))
    d2h = ho.numel() * ho.element_size() + sum(x.numel() * x.element_size() for x in hl_ch)
    ms = max_over_ranks(torch, dist, sum(t_steps) / len(t_steps), device)
    ms_e2e = max_over_ranks(torch, dist, sum(t_e2e) / len(t_e2e), device)
    o_loc, lse_loc = sparse_mla.prefill(q, raw, cmp, idx, window=C3["window"], q_pos=pos, check=True)
    torch.cuda.synchronize()
    for c in (0, n_ch - 1):  # the chunked end-to-end path computed the same rows, bit for bit
        a, b = bounds[c], min(bounds[c] + 64, bounds[c + 1])
        assert torch.equal(ho[0, a:b], o_loc[0, a:b].cpu()), "e2e output differs from the device step"
        assert torch.equal(hl_ch[c][0, :, :b - a], lse_loc[0, :, a:b].cpu()), "e2e lse differs"
    gather_ms = None
    if dist:  # optional output gather (o of every rank's shard to every rank), timed on its own
        width = max(len(p) for p in shard_tokens(C3["S"], world, 128))
        pad = o_loc.new_zeros((width,) + tuple(o_loc.shape[2:]))
        pad[:n_q] = o_loc[0]
        buf = o_loc.new_empty((world * width,) + tuple(o_loc.shape[2:]))
        dist.all_gather_into_tensor(buf, pad)  # untimed: the collective's lazy setup
        t_g = timer.run(lambda: dist.all_gather_into_tensor(buf, pad), 3, flush=False)
        gather_ms = max_over_ranks(torch, dist, sum(t_g) / len(t_g), device)
    pk = peaks()
    tflops = total_flops / (ms * 1e-3) / 1e12
    ms_local = sum(t_steps) / len(t_steps)
    achieved = flops / (ms_local * 1e-3) / 1e12
    out = {
        "metric": "sparse-MLA prefill TFLOP/s", "value": tflops, "unit": "TFLOP/s", "ms_per_step": ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 (fp8 KV dequant, fp32 acc)",
        "data": "synthetic (seeded N(0,1); FP8 no-rope rows with per-64 absmax scales)",
        "config": c3_config(world),
        "legs": {"total_flops": total_flops, "o_gather_ms": gather_ms},
        "e2e": {"value": total_flops / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "note": f"sparse_mla.prefill on {n_ch} query chunks, each chunk's H2D / kernels / D2H overlapped "
                        "with its neighbours' on three streams"},
        "roofline": {"bound": "tensor", "kernel": "mzb::mla::mla_fwd_kernel", "achieved": achieved,
                     "peak": pk["bf16_tflops"], "unit": "TFLOP/s", "frac": achieved / pk["bf16_tflops"],
                     "peak_note": f"{pk['_source']} bf16 burst", "algorithmic_flops_per_launch": flops,
                     "ms_per_launch": ms_local, **traffic_for("prefill", flops / total_flops),
                     # the launch runs for ~10 ms back to back, in the power-capped regime the
                     # sustained GEMM figure was measured in: given beside the burst fraction
                     **({"frac_of_sustained": achieved / pk["bf16_tflops_sustained"],
                         "sustained_peak": pk["bf16_tflops_sustained"]} if "bf16_tflops_sustained" in pk else {})},
        "gpu_launches": 2 * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        toks_s = _prefill_sample(C3["S"], 256)
        tk = torch.tensor(toks_s, device=device)
        r = cpu_prefill(torch, q_full[0, tk].cpu(), toks_s, raw[0].cpu(), cmp[0].cpu(), idx_full[0, tk].cpu())
        ro, rl = r.pop("result")
        eo = (o_loc[0, tk].float().cpu() - ro).abs().max().item()
        el = (lse_loc[0, :, tk].cpu().T - rl).abs().max().item()
        r["parity"] = {"tokens": len(toks_s), "max_abs_err_o": eo, "max_abs_err_lse": el, "atol": 2e-2,
                       "ok": bool(eo <= 2e-2 and el <= 2e-2),
                       "note": "GPU rows vs the CPU float32 reference on the sampled tokens"}
        out["cpu_baseline"] = r
    return out


def cpu_prefill(torch, q_rows, toks, raw_rows, cmp_rows, idx_rows, chunk: int = 32) -> dict:
    """The reference's float32 CPU arithmetic (``_attend`` over each token's gathered rows:
    the 128-token window then the listed compressed entries, rows dequantised from FP8) for
    the sampled query tokens, all 128 heads, all host threads.  Metric: TFLOP/s of the
    sample's selected pairs.  q_rows [n,128,576] bf16, raw_rows [S,672], cmp_rows [G,672],
    idx_rows [n,topk] (CPU tensors)."""
    from oracle import torch_ref as R
    cores = cpu_threads(torch)
    n, W = len(toks), C3["window"]
    S, G = raw_rows.shape[0], cmp_rows.shape[0]
    t0 = time.perf_counter()
    table = torch.cat([raw_rows, cmp_rows])           # compressed entry g is row S + g
    pos = torch.tensor(toks).view(-1, 1)
    wrow = pos - W + 1 + torch.arange(W).view(1, -1)   # window rows, -ve = empty
    ci = idx_rows.long()
    crow = torch.where((ci >= 0) & (ci < G), ci + S, torch.full_like(ci, -1))
    rows = torch.cat([wrow.masked_fill(wrow < 0, -1), crow], 1)
    counts = (rows >= 0).sum(1)
    order = torch.sort((rows < 0).to(torch.int8), dim=1, stable=True).indices  # valid rows first, in order
    rows = torch.gather(rows, 1, order)
    o = torch.empty(n, 128, 512)
    lse = torch.empty(n, 128)
    for c0 in range(0, n, chunk):
        c1 = min(n, c0 + chunk)
        tmax = int(counts[c0:c1].max())
        keys = R.unpack_rows(table[rows[c0:c1, :tmax].clamp_min(0)])
        o[c0:c1], lse[c0:c1] = R.gathered_attention(q_rows[c0:c1].float(), keys, counts[c0:c1], 576 ** -0.5)
    dt = time.perf_counter() - t0
    pairs = int(counts.sum())
    flops = 2.0 * 128 * 1088 * pairs
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port", "ms": dt * 1e3,
            "sample": f"{n} evenly spaced query tokens x 128 heads ({pairs} selected pairs): torch float32 "
                      f"_attend over the gathered, dequantised rows (the reference's CPU arithmetic), {dt:.2f} s",
            "result": (o, lse)}


def _prefill_sample(S, n_tok):
    import numpy as np
    return [int(t) for t in np.linspace(0, S - 1, n_tok)]


def reference_prefill(args, rank, world) -> dict:
    import torch
    from oracle import torch_ref as R
    if rank != 0:
        return None
    S, G = C3["S"], C3["G"]
    toks = _prefill_sample(S, 256)
    g = torch.Generator().manual_seed(0)
    q_rows = torch.randn(len(toks), 128, 576, generator=g).to(torch.bfloat16)
    raw = R.pack_rows(torch.randn(S, 576, generator=g))
    cmp = R.pack_rows(torch.randn(G, 576, generator=g))
    idx = sorted_causal_indices(torch, 0, G, C3["topk"], C3["ratio"], torch.Generator().manual_seed(1),
                                torch.device("cpu"), positions=toks)
    runs = []
    for _ in range(args.warmup + args.steps):
        r = cpu_prefill(torch, q_rows, toks, raw, cmp, idx)
        r.pop("result")
        runs.append(r)
    return _reference_line(args, world, "sparse-MLA prefill TFLOP/s", "TFLOP/s", c3_config(world), runs,
                           "f32 (reference CPU arithmetic, FP8 KV dequantised)",
                           "synthetic (seeded N(0,1); FP8 no-rope rows with per-64 absmax scales)")

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


def c5_config(world: int) -> dict:
    return {"workload": "C5 SWA train + fake quant", "B": C5["B"], "S": C5["S"], "heads": C5["H"],
            "head_dim": C5["D"], "window": C5["window"], "fq": "Q,K OCP MXFP4 block 32; V FP8 absmax per 128; STE",
            "parallelism": f"x{world} independent" if world > 1 else "1 GPU", "l2": "256 MB flush per step"}


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

    # the step one sequence (batch element) at a time through the public API: each
    # sequence's copies overlap the neighbouring sequences' kernels and copies
    pipe = Pipeline(torch, device)

    def e2e():
        def h2d(b):
            for d, h in ((dq_, hq), (dk_, hk), (dv_, hv), (ddo, hdo)):
                d[b].copy_(h[b], non_blocking=True)

        def compute(b):
            return c5_step(dq_[b:b + 1], dk_[b:b + 1], dv_[b:b + 1], ddo[b:b + 1])

        def d2h(b, res):
            for h, g_ in zip((hdq, hdk, hdv), res):
                h[b].copy_(g_[0], non_blocking=True)

        pipe.run(B, h2d, compute, d2h)

    e2e()
    t_e2e = timer.run(e2e, max(2, args.steps // 2), flush=False)
    torch.cuda.synchronize()
    ref_g = c5_step(q, k, v, do)
    e2e_err = max(((h.float() - r_.float().cpu()).abs().max() / (1.0 + r_.float().abs().max().cpu())).item()
                  for h, r_ in zip((hdq, hdk, hdv), ref_g))
    assert e2e_err <= 1e-2, f"e2e gradients differ from the device step (relative {e2e_err})"
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
        "config": c5_config(world),
        "e2e": {"value": total * world / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "note": f"the step per sequence ({B} chunks), each chunk's H2D / kernels / D2H overlapped with its "
                        f"neighbours' on three streams; gradients within {e2e_err:.1e} (relative) of the one-launch "
                        "step"},
        "roofline": {"bound": "tensor", "kernel": "mzb::attnb::dkv_kernel + dq_kernel (backward)",
                     "achieved": ach_bwd, "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": ach_bwd / pk["bf16_tflops"], "peak_note": f"{pk['_source']} bf16 burst",
                     "algorithmic_flops_per_launch": bwd_flops, "ms_per_launch": ms_bwd, **traffic_for("train", 1.0)},
        "legs": {"fwd_ms": ms_fwd, "fwd_tflops": fwd_flops / (ms_fwd * 1e-3) / 1e12, "bwd_ms": ms_bwd,
                 "fq_q_ms": ms_fq, "fq_q_gbs": fq_bytes / (ms_fq * 1e-3) / 1e9},
        "gpu_launches": 7 * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        toks = _train_sample()
        dq_gpu = c5_step(q, k, v, do)[0][0, torch.tensor(toks, device=device)].float().cpu()
        r = cpu_train(torch, q[0, toks].cpu(), k[0, :, 0].cpu(), v[0, :, 0].cpu(), do[0, toks].cpu(), toks)
        dq_ref = r.pop("result")
        err = (dq_gpu - dq_ref).abs().max().item()
        tol = 2e-2 + 1e-2 * dq_ref.abs().max().item()
        r["parity"] = {"tokens": len(toks), "max_abs_err_dq": err, "tol": tol, "ok": bool(err <= tol),
                       "note": "GPU dq rows vs the CPU float32 reference (STE fake quant + autograd) on the "
                               "sampled tokens"}
        out["cpu_baseline"] = r
    return out


def _train_sample(n: int = 512):
    import numpy as np
    return [int(t) for t in np.linspace(0, C5["S"] - 1, n)]


def cpu_train(torch, q_rows, k_seq, v_seq, do_rows, toks) -> dict:
    """The reference's float32 CPU arithmetic for the sampled query tokens of one sequence:
    STE fake quant (``x - x.detach() + fq(x)``, ``indexer/attn.py:29-34``; Q, K OCP MXFP4 per
    32, V FP8 absmax per 128), ``_attend`` over each token's window with autograd, backward
    from dO.  q_rows / do_rows [n,H,D], k_seq / v_seq [S,D].  Metric: TFLOP/s of the sample's
    band pairs (forward + 2.5x backward)."""
    from oracle import torch_ref as R
    cores = cpu_threads(torch)
    W, D = C5["window"], C5["D"]
    n = len(toks)
    t0 = time.perf_counter()
    qx = q_rows.float().requires_grad_()
    kx = k_seq.float().requires_grad_()
    vx = v_seq.float().requires_grad_()
    qf = qx - qx.detach() + R.fake_quant_fp4_ocp(qx.detach(), 32)
    kf = kx - kx.detach() + R.fake_quant_fp4_ocp(kx.detach(), 32)
    vf = vx - vx.detach() + R.fake_quant_fp8_absmax(vx.detach(), 128)
    pos = torch.tensor(toks).view(-1, 1)
    rows = pos - W + 1 + torch.arange(W).view(1, -1)             # [n, W] window positions
    valid = rows >= 0
    rc = rows.clamp_min(0)
    bias = torch.zeros(n, W).masked_fill_(~valid, float("-inf")).view(n, 1, 1, W)
    o, _ = R.attend(qf.unsqueeze(1), kf[rc].unsqueeze(1), vf[rc].unsqueeze(1), bias, D ** -0.5)
    o.backward(do_rows.float().unsqueeze(2))        # o is [n, H, 1, D]
    dt = time.perf_counter() - t0
    pairs = int(valid.sum()) * q_rows.shape[1]
    flops = 4.0 * D * pairs * 3.5
    return {"value": flops / dt / 1e12, "unit": "TFLOP/s", "cores": cores, "kind": "port", "ms": dt * 1e3,
            "sample": f"{n} evenly spaced query tokens of one sequence x {q_rows.shape[1]} heads x their {W}-key "
                      f"windows: torch float32 STE fake quant + _attend forward + autograd backward (the "
                      f"reference's CPU arithmetic), {dt:.2f} s",
            "result": qx.grad}


def reference_train(args, rank, world) -> dict:
    import torch
    if rank != 0:
        return None
    g = torch.Generator().manual_seed(10)
    toks = _train_sample()
    H, D = C5["H"], C5["D"]
    q = torch.randn(len(toks), H, D, generator=g).to(torch.bfloat16)
    k = torch.randn(C5["S"], D, generator=g).to(torch.bfloat16)
    v = torch.randn(C5["S"], D, generator=g).to(torch.bfloat16)
    do = torch.randn(len(toks), H, D, generator=g).to(torch.bfloat16)
    runs = []
    for _ in range(args.warmup + args.steps):
        r = cpu_train(torch, q, k, v, do, toks)
        r.pop("result")
        runs.append(r)
    return _reference_line(args, world, "SWA train fwd+bwd TFLOP/s (fake-quant Q/K MXFP4, V FP8)", "TFLOP/s",
                           c5_config(world), runs, "f32 (reference CPU arithmetic)",
                           "synthetic (seeded N(0,1) bf16 inputs and dO)", scaling="weak")


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
    caches with random page tables, the FP8 index keys in 64-key pages under the compressed
    cache's page table, queries."""
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
    kcodes = torch.randint(0, 255, (n_cmp, 64, C4["Di"]), generator=g, device=device, dtype=torch.int32)
    k8 = torch.where((kcodes & 0x7F) == 0x7F, kcodes - 1, kcodes).to(torch.uint8).view(torch.float8_e4m3fn)
    sk = (torch.rand(n_cmp, 64, generator=g, device=device) * 3 + 1) / 448.0
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
                       q_pos=x["pos"], k_page_table=x["cpt"])
    return sparse_mla.decode(x["q"], x["raw"], x["pt"], x["lens"], x["cmp"], x["cpt"], x["cmp_lens"], idx[:, 0],
                             window=C4["window"])


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


def c4_config(world: int) -> dict:
    return {"workload": "C4 paged decode + indexer", "sequences": C4["B"], "context": "U[8192,131072] seed 1",
            "heads": 128, "topk": C4["topk"], "window": C4["window"], "page": 64,
            "parallelism": (f"sequences sharded over {world} GPUs (greedy by length), no collective in the "
                            "step" if world > 1 else "1 GPU"),
            "l2": "caches (~8 GB) larger than L2; 256 MB flush per step"}


def bench_decode(args, torch, dist, rank, world, device) -> dict:
    lens = c4_lens(torch)
    from mzoo_b200.sharding import shard_sequences
    parts = shard_sequences(lens.tolist(), world)
    mine = parts[rank]
    x = c4_inputs(torch, device, mine, lens)
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
    g_step = _graph(torch, device, step)  # a decode step as a serving engine runs it: one graph
    sampler.ready()
    if dist:
        dist.barrier()
    t_steps = timer.run(g_step.replay, args.steps)
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
    qp, kp, wp, sqp, skp, scale, dt = indexer._prep(x["q8"], x["k8"], x["w"], (x["sq"], x["sk"]), None, x["cpt"])
    qpos = x["pos"].to(torch.int32).contiguous()
    g_score = _graph(torch, device, lambda: indexer._scores(qp, kp, wp, sqp, skp, C4["ratio"], 0, scale, dt, False,
                                                             False, qpos, x["cpt"]))
    t_score = timer.run(g_score.replay, args.steps)  # graph replay: the kernel's time, no host launch gap
    # e2e: queries / indexer queries / weights from pinned host memory, o back to the host
    hq, hq8, hw = x["q"].cpu().pin_memory(), x["q8"].view(torch.uint8).cpu().pin_memory(), x["w"].cpu().pin_memory()
    ho = torch.empty(n_mine, 128, 512, dtype=torch.bfloat16).pin_memory()

    # one step through the public API (chunking the step here measured slower: each chunk
    # pays the wrappers' host launch work, which a decode step cannot hide)
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
    score_bytes_all = sum((int(L) // 4) * (C4["Di"] + 4) + C4["Hi"] * (C4["Di"] + 8) for L in lens.tolist())
    ach = score_bytes / (ms_score * 1e-3) / 1e9
    out = {
        "metric": "paged sparse-MLA decode HBM GB/s (indexer + attention)", "value": total_bytes / (ms * 1e-3) / 1e9,
        "unit": "GB/s", "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "e4m3 KV / bf16 q (fp32 acc)", "data": "synthetic (seeded lengths, random page tables, random FP8 rows)",
        "config": c4_config(world),
        "timing": "value: CUDA-graph replay of the step's launches; e2e: the public API op by op",
        "legs": {"algorithmic_bytes_per_step": total_bytes, "mean_context": float(lens.float().mean()),
                 "o_gather_ms": gather_ms},
        "e2e": {"value": total_bytes / (ms_e2e * 1e-3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": hq.numel() * 2 + hq8.numel() + hw.numel() * 4,
                "d2h_bytes_per_step": ho.numel() * 2},
        "roofline": {"bound": "hbm", "kernel": "mzb::idx::score_kernel<fp8,128,1> (decode indexer)", "achieved": ach,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": ach / pk["hbm_gbs"],
                     "peak_note": f"{pk['_source']} HBM copy", "algorithmic_bytes_per_launch": score_bytes,
                     "ms_per_launch": ms_score, **traffic_for("decode", score_bytes / score_bytes_all)},
        "gpu_launches": 6 * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        from mzoo_b200 import sparse_mla
        idx = indexer.attn(x["q8"], x["k8"], x["w"], compress_ratio=C4["ratio"], topk=C4["topk"],
                           scales=(x["sq"], x["sk"]), q_pos=x["pos"], k_page_table=x["cpt"], check=True)
        o, lse = sparse_mla.decode(x["q"], x["raw"], x["pt"], x["lens"], x["cmp"], x["cpt"], x["cmp_lens"],
                                   idx[:, 0], window=C4["window"], check=True)
        sample = _decode_sample(lens)
        items = [_decode_item_from_device(torch, x, b, int(lens[b])) for b in sample]
        r = cpu_decode(torch, items)
        res = r.pop("result")
        same = sum(_set_equal_rows(torch, idx[b, 0:1].cpu(), ri.view(1, -1)) for b, (ri, _, _) in zip(sample, res))
        eo = max((o[b].float().cpu() - ro).abs().max().item() for b, (_, ro, _) in zip(sample, res))
        el = max((lse[b].cpu() - rl).abs().max().item() for b, (_, _, rl) in zip(sample, res))
        r["parity"] = {"sequences": len(sample), "equal_index_sets": int(same), "max_abs_err_o": eo,
                       "max_abs_err_lse": el, "atol": 2e-2,
                       "note": "GPU index sets and rows vs the CPU float32 reference on the sampled sequences (the "
                               "attention check holds where the sets agree)"}
        out["cpu_baseline"] = r
    return out


def _decode_sample(lens, n: int = 32) -> list:
    """n sequences spread over the length distribution (every len/n-th in length order)."""
    order = sorted(range(len(lens)), key=lambda b: int(lens[b]))
    step = max(1, len(order) // n)
    return [order[i] for i in range(step // 2, len(order), step)][:n]


def _window_pages(L: int):
    """Raw pages the 128-token window of a query at position L-1 reads."""
    return range(max(0, L - C4["window"]) // 64, (L - 1) // 64 + 1)


def _decode_item_from_device(torch, x, b: int, L: int) -> dict:
    """One sequence's decode inputs moved to the host: indexer tensors, its compressed pages
    (compacted, page table 0..n-1) and the raw pages its window reads (other entries of the
    raw page table are never read)."""
    T = L // C4["ratio"]
    ncp = -(-T // 64)
    wp = list(_window_pages(L))
    raw_pt = torch.zeros(-(-L // 64), dtype=torch.int64)
    raw_pt[wp] = torch.arange(len(wp))
    cpages = x["cpt"][b, :ncp].long()
    return {"L": L, "q8": x["q8"][b, 0].cpu(), "sq": x["sq"][b, 0].cpu(), "w": x["w"][b, 0].cpu(),
            "k8": x["k8"][cpages].reshape(-1, C4["Di"])[:T].cpu(), "sk": x["sk"][cpages].reshape(-1)[:T].cpu(),
            "q": x["q"][b].cpu(),
            "cmp": x["cmp"][x["cpt"][b, :ncp].long()].cpu(), "cpt": torch.arange(ncp),
            "raw": x["raw"][x["pt"][b, wp].long()].cpu(), "pt": raw_pt}


def _decode_item_cpu(torch, L: int, gen) -> dict:
    """One sequence's decode inputs generated on the host with the bench's distributions."""
    T = L // C4["ratio"]
    ncp = -(-T // 64)
    wp = list(_window_pages(L))
    raw_pt = torch.zeros(-(-L // 64), dtype=torch.int64)
    raw_pt[wp] = torch.arange(len(wp))

    def codes(*shape):
        c = torch.randint(0, 255, shape, generator=gen, dtype=torch.int32)
        return torch.where((c & 0x7F) == 0x7F, c - 1, c).to(torch.uint8).view(torch.float8_e4m3fn)
    return {"L": L, "q8": codes(C4["Hi"], C4["Di"]), "sq": (torch.rand(C4["Hi"], generator=gen) * 3 + 1) / 448.0,
            "w": torch.randn(C4["Hi"], generator=gen) / 8, "k8": codes(T, C4["Di"]),
            "sk": (torch.rand(T, generator=gen) * 3 + 1) / 448.0,
            "q": torch.randn(128, 576, generator=gen).to(torch.bfloat16),
            "cmp": _random_rows(torch, ncp * 64, torch.device("cpu"), gen).view(ncp, 64, 672), "cpt": torch.arange(ncp),
            "raw": _random_rows(torch, len(wp) * 64, torch.device("cpu"), gen).view(len(wp), 64, 672), "pt": raw_pt}


def cpu_decode(torch, items) -> dict:
    """The reference's float32 CPU arithmetic for one decode step of the given sequences:
    ``indexer_scores`` of the one query over the sequence's L/4 dequantised FP8 keys
    (position L-1), ``topk_indices`` (top-2048), then ``_attend`` over the window and the
    selected compressed rows, read through the page tables and dequantised.  Metric: GB/s
    of the sequences' algorithmic bytes."""
    from oracle import torch_ref as R
    cores = cpu_threads(torch)
    W = C4["window"]
    res = []
    t0 = time.perf_counter()
    for it in items:
        L = it["L"]
        qd = (it["q8"].float() * it["sq"].view(-1, 1)).view(1, 1, C4["Hi"], C4["Di"])
        kd = (it["k8"].float() * it["sk"].view(-1, 1)).unsqueeze(0)
        sc = R.indexer_scores(qd, kd, it["w"].view(1, 1, -1), C4["ratio"], L - 1, scale=1.0)
        idx = R.topk_indices(sc, C4["topk"])[0, 0]
        sel = idx[idx >= 0]
        pos = torch.arange(max(0, L - W), L)
        rows = torch.cat([it["raw"][it["pt"][pos // 64], pos % 64], it["cmp"][it["cpt"][sel // 64], sel % 64]])
        keys = R.unpack_rows(rows).unsqueeze(0)
        o, lse = R.gathered_attention(it["q"].float().unsqueeze(0), keys, torch.tensor([rows.shape[0]]),
                                      576 ** -0.5)
        res.append((idx, o[0], lse[0]))
    dt = time.perf_counter() - t0
    lens = [it["L"] for it in items]
    nbytes = c4_bytes(lens)
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": cores, "kind": "port", "ms": dt * 1e3,
            "sample": f"{len(items)} of the 128 sequences ({sum(lens)} tokens of context): torch float32 indexer_scores + topk_indices + _attend over the paged, dequantised "
                      f"rows (the reference's CPU arithmetic), {dt:.2f} s",
            "result": res}


def reference_decode(args, rank, world) -> dict:
    import torch
    if rank != 0:
        return None
    lens = c4_lens(torch)
    g = torch.Generator().manual_seed(5)
    items = [_decode_item_cpu(torch, int(lens[b]), g) for b in range(C4["B"])]  # the whole config
    runs = []
    for _ in range(args.warmup + args.steps):
        r = cpu_decode(torch, items)
        r.pop("result")
        runs.append(r)
    return _reference_line(args, world, "paged sparse-MLA decode HBM GB/s (indexer + attention)", "GB/s",
                           c4_config(world), runs, "f32 (reference CPU arithmetic, FP8 dequantised)",
                           "synthetic (seeded lengths, random page tables, random FP8 rows)")


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


def cf_config(world: int) -> dict:
    return {"workload": "F1 two-level selection: level-one candidate blocks + level-two top-k",
            "queries": CF["rows"], "positions": CF["T"], "block_size": CF["block"], "topk_blocks": CF["topk_blocks"],
            "topk": CF["topk"],
            "parallelism": (f"query rows cyclic over {world} GPUs, no collective" if world > 1 else "1 GPU"),
            "l2": "flushed (256 MB write) per step; inputs (2 x 512 MB) larger than L2"}


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
        "config": cf_config(world),
        "legs": {"level_one_ms": ms_l1, "level_two_ms": ms_l2,
                 "level_one_gbs": rows * CF["T"] * 4 / (ms_l1 * 1e-3) / 1e9},
        "e2e": {"value": CF["rows"] / (ms_e2e * 1e-3) / 1e6, "unit": "Mq/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "kernel": "mzb::cand::topk_gather_kernel (level two)", "achieved": achieved,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "peak_note": f"{pk['_source']} copy bandwidth", "algorithmic_bytes_per_launch": alg2,
                     "ms_per_launch": ms_l2, **traffic_for("candidates", rows / CF["rows"])},
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
    return {"value": sample / dt / 1e6, "unit": "Mq/s", "cores": 1, "kind": "port", "ms": dt * 1e3,
            "sample": f"{sample} query rows of {CF['T']} positions, numpy (lexsort per row), {dt:.2f} s"}


def reference_candidates(args, rank, world) -> dict:
    import torch
    if rank != 0:
        return None
    n = max(1, args.cpu_sample // 16)
    lg, sc, cl = cf_inputs(torch, seed=0, rows=n)
    runs = [cpu_candidates(lg, sc, cl, sample=n) for _ in range(args.warmup + args.steps)]
    return _reference_line(args, world, "two-level indexer selection Mq/s", "Mq/s", cf_config(world), runs,
                           "f32 keys (oracle port, numpy)", "synthetic")


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


def cp_config(world: int) -> dict:
    return {"workload": "F3 compressor: gated softmax pool + RMSNorm + RoPE + MXFP4 cache entry",
            "B": CP["B"], "tokens": CP["S"], "compress_ratio": CP["ratio"], "head_dim": CP["D"],
            "rope_dim": CP["rope"],
            "parallelism": (f"sequences cyclic over {world} GPUs, no collective" if world > 1 else "1 GPU"),
            "l2": "flushed (256 MB write) per step; inputs (604 MB) larger than L2"}


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
        "config": cp_config(world),
        "e2e": {"value": total / (ms_e2e * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h},
        "roofline": {"bound": "hbm", "kernel": "mzb::comp::compress_kernel", "achieved": achieved,
                     "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                     "peak_note": f"{pk['_source']} copy bandwidth", "algorithmic_bytes_per_launch": local,
                     "ms_per_launch": sum(t_steps) / len(t_steps), **traffic_for("compressor", B / CP["B"])},
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
            "ms": dt * 1e3, "sample": f"{n} groups of sequence 0, numpy, {dt:.2f} s"}


def reference_compressor(args, rank, world) -> dict:
    import torch
    if rank != 0:
        return None
    h = cp_inputs(torch, seed=0, B=1)
    runs = [cpu_compressor(h, n_groups=max(1, args.cpu_sample)) for _ in range(args.warmup + args.steps)]
    return _reference_line(args, world, "compressor producer step HBM GB/s (algorithmic bytes)", "GB/s",
                           cp_config(world), runs, "f32 (oracle port, numpy)", "synthetic")


# ----------------------------------------------------------------------------- RMSNorm + RoPE prologue

# The reference's own benchmark shape for its fused prologue (norm_rope_bench.py: q of
# B1 S4096 H64 D128, rope_dim 64); a step is the forward and the backward.
NR = dict(B=1, S=4096, H=64, D=128, rope=64)


def nr_config(world: int) -> dict:
    return {"workload": "F3 QK prologue: fused RMSNorm + RoPE forward + backward", "B": NR["B"], "S": NR["S"],
            "heads": NR["H"], "head_dim": NR["D"], "rope_dim": NR["rope"],
            "parallelism": f"x{world} independent" if world > 1 else "1 GPU",
            "l2": "flushed (256 MB write) per step"}


def nr_bytes() -> float:
    """Algorithmic HBM bytes of a step: forward reads x, writes out and rstd; backward reads
    x, dy and rstd, writes dx; cos / sin read by both."""
    rows = NR["B"] * NR["S"] * NR["H"]
    xb = rows * NR["D"] * 2
    cs = 2 * NR["B"] * NR["S"] * (NR["rope"] // 2) * 4
    return (2 * xb + rows * 4 + cs) + (3 * xb + rows * 4 + cs)


def nr_inputs(torch, seed: int = 0):
    g = torch.Generator().manual_seed(seed)
    B, S, H, D, rd = (NR[k] for k in ("B", "S", "H", "D", "rope"))
    x = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16)
    w = torch.randn(D, generator=g).to(torch.bfloat16)
    pos = torch.arange(S, dtype=torch.float32)
    freqs = pos[:, None] / (10000.0 ** (torch.arange(0, rd, 2, dtype=torch.float32) / rd))
    dy = torch.randn(B, S, H, D, generator=g).to(torch.bfloat16)
    return x, w, freqs.cos()[None].expand(B, -1, -1).contiguous(), freqs.sin()[None].expand(B, -1, -1).contiguous(), dy


def bench_normrope(args, torch, dist, rank, world, device) -> dict:
    from mzoo_b200 import norm_rope
    xh, wh, ch, sh, dyh = nr_inputs(torch, seed=rank)
    x, w, cos, sin, dy = (t.to(device) for t in (xh, wh, ch, sh, dyh))

    def step():
        out, rstd = norm_rope.fwd(x, w, cos, sin)
        return out, norm_rope.bwd(x, w, cos, sin, rstd, dy)

    timer = Timer(torch, device)
    sampler = ClockSampler(device.index)
    sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # A step is ~0.1 ms of device work: launched op by op its timing would include the host's
    # launch overhead, so the timed step (and each leg) replays a CUDA graph of its launches.
    out, rstd = norm_rope.fwd(x, w, cos, sin)
    g_step, g_fwd, g_bwd = (_graph(torch, device, f) for f in (
        step, lambda: norm_rope.fwd(x, w, cos, sin), lambda: norm_rope.bwd(x, w, cos, sin, rstd, dy)))
    sampler.ready()
    if dist:
        dist.barrier()
    t_steps = timer.run(g_step.replay, args.steps)
    clocks = sampler.stop(busy=g_step.replay)
    t_fwd = timer.run(g_fwd.replay, args.steps)
    t_bwd = timer.run(g_bwd.replay, args.steps)
    hx, hdy = xh.pin_memory(), dyh.pin_memory()
    dx_, ddy = torch.empty_like(x), torch.empty_like(dy)
    hout, hdx = torch.empty_like(hx).pin_memory(), torch.empty_like(hx).pin_memory()

    def e2e():  # through the public, differentiable API
        dx_.copy_(hx, non_blocking=True)
        ddy.copy_(hdy, non_blocking=True)
        xg = dx_.detach().requires_grad_()
        o = norm_rope.qk_norm_rope(xg, w, cos, sin)
        o.backward(ddy)
        hout.copy_(o.detach(), non_blocking=True)
        hdx.copy_(xg.grad, non_blocking=True)

    for _ in range(2):
        e2e()
    t_e2e = timer.run(e2e, args.steps, flush=False)
    ms = max_over_ranks(torch, dist, sum(t_steps) / len(t_steps), device)
    ms_e2e = max_over_ranks(torch, dist, sum(t_e2e) / len(t_e2e), device)
    ms_f, ms_b = sum(t_fwd) / len(t_fwd), sum(t_bwd) / len(t_bwd)
    rows = NR["B"] * NR["S"] * NR["H"]
    xb = rows * NR["D"] * 2
    cs = 2 * NR["B"] * NR["S"] * (NR["rope"] // 2) * 4
    bwd_bytes = 3 * xb + rows * 4 + cs
    pk = peaks()
    ach = bwd_bytes / (ms_b * 1e-3) / 1e9
    total = nr_bytes()
    res = {
        "metric": "QK prologue (RMSNorm + RoPE fwd + bwd) HBM GB/s (algorithmic bytes)",
        "value": total * world / (ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (fp32 statistics)",
        "data": "synthetic (seeded N(0,1) bf16 q, dy and weight; RoPE angles of positions 0..S-1)",
        "config": nr_config(world),
        "timing": "value and legs: CUDA-graph replay of the step's launches; e2e: the public API op by op",
        "legs": {"fwd_ms": ms_f, "fwd_gbs": (2 * xb + rows * 4 + cs) / (ms_f * 1e-3) / 1e9, "bwd_ms": ms_b},
        "e2e": {"value": total * world / (ms_e2e * 1e-3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": 2 * hx.numel() * 2, "d2h_bytes_per_step": 2 * hx.numel() * 2},
        "roofline": {"bound": "hbm", "kernel": "mzb::nr::bwd_kernel<128>", "achieved": ach, "peak": pk["hbm_gbs"],
                     "unit": "GB/s", "frac": ach / pk["hbm_gbs"], "peak_note": f"{pk['_source']} copy bandwidth",
                     "algorithmic_bytes_per_launch": bwd_bytes, "ms_per_launch": ms_b, "traffic": None},
        "gpu_launches": 3 * args.steps,
        "clocks": clocks,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = cpu_normrope(torch, xh, wh, ch, sh, dyh)
        ro, rdx = r.pop("result")
        n = ro.shape[1]
        eo = (out[:, :n].float().cpu() - ro.float()).abs().max().item()
        r["parity"] = {"tokens": n, "max_abs_err_out": eo, "note": "GPU forward rows vs the CPU reference "
                       "composition in bf16 on the sampled tokens (same rounding points: expected 0 or one bf16 step)"}
        res["cpu_baseline"] = r
    return res


def cpu_normrope(torch, x, w, cos, sin, dy, n_tok: int = 1024) -> dict:
    """The reference's CPU path (the model's RMSNorm + RoPE in torch, bf16, with autograd for
    the backward) on the first ``n_tok`` tokens (all heads), all host threads."""
    from oracle import torch_ref as R
    cores = cpu_threads(torch)
    xs = x[:, :n_tok].clone().requires_grad_()
    ws = w.clone().requires_grad_()
    t0 = time.perf_counter()
    o = R.qk_norm_rope(xs, ws, cos[:, :n_tok], sin[:, :n_tok])
    o.backward(dy[:, :n_tok])
    dt = time.perf_counter() - t0
    frac = n_tok / NR["S"]
    return {"value": nr_bytes() * frac / dt / 1e9, "unit": "GB/s", "cores": cores, "kind": "port", "ms": dt * 1e3,
            "sample": f"{n_tok} of {NR['S']} tokens x {NR['H']} heads: torch bf16 RMSNorm + RoPE forward + autograd "
                      f"backward (the reference's eager composition), {dt:.2f} s",
            "result": (o.detach(), xs.grad)}


def reference_normrope(args, rank, world) -> dict:
    import torch
    if rank != 0:
        return None
    x, w, cos, sin, dy = nr_inputs(torch)
    runs = []
    for _ in range(args.warmup + args.steps):
        r = cpu_normrope(torch, x, w, cos, sin, dy)
        r.pop("result")
        runs.append(r)
    return _reference_line(args, world, "QK prologue (RMSNorm + RoPE fwd + bwd) HBM GB/s (algorithmic bytes)",
                           "GB/s", nr_config(world), runs, "bf16 (reference CPU composition)", "synthetic",
                           scaling="weak")


CONFIGS = {"window": c1_config, "indexer": c2_config, "prefill": c3_config, "decode": c4_config,
           "train": c5_config, "candidates": cf_config, "compressor": cp_config, "normrope": nr_config}

BENCHES = {"window": (bench_window, reference_window),
           "indexer": (bench_indexer, reference_indexer), "prefill": (bench_prefill, reference_prefill),
           "train": (bench_train, reference_train), "decode": (bench_decode, reference_decode),
           "candidates": (bench_candidates, reference_candidates),
           "compressor": (bench_compressor, reference_compressor),
           "normrope": (bench_normrope, reference_normrope)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="prefill", choices=sorted(BENCHES))
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
        C4.update(L_hi=16384)  # all 128 sequences (the latent kernel's full item count), short contexts
        CF.update(rows=256)
        CP.update(B=1, S=4096)
        NR.update(S=1024)
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
