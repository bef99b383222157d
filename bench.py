"""Benchmark of the B200 DSA sparse-MLA decode (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

A step is one decode call (the reference's `kernel(...)`, solution/triton/fused.py:150)
over one batch of the workload: 64 decode rows x 16 heads x topk 2048 by default, the
production decode config.  Every rank holds its own rows and its own paged pool (the
batch is sharded; there is no collective on the timed path), so the scaling is weak.

Reported numbers:
  value      algorithmic HBM GB/s of the whole job (all ranks' bytes / max rank time),
             device-timed with CUDA events over K steps replayed from a CUDA graph, inputs
             resident in HBM.  Four independent input sets (4 x ~154 MB, more than the
             126 MB L2) rotate so that a step never finds its rows in L2.
  e2e        the same metric through the public entry point with host buffers: per step
             the step's q_nope, q_pe and sparse_indices are copied from pinned host memory,
             the decode runs, and output + lse are copied back (the paged KV pool is
             device-resident state, like a serving engine's cache).  Also reported: the
             host time spent issuing a step and the time of the step's copies alone.
  roofline   achieved GB/s of the decode call vs the measured HBM peak; `traffic` is the
             DRAM bytes of one call from the ncu capture recorded in
             profiles/dram_traffic.json, reported only while the kernel sources still
             match the capture's digest.
  workloads  (one GPU) the other single-GPU configurations: b32_h128 (128 heads, with its
             tensor-pipe rate) and ragged_b256 (-1 padding), timed like `value`.
  index_production  the step before the decode (each row's top-2048 positions of index
             scores, as slot ids) alone and chained with the decode.
  b2048      (every N) the batch-sharded decode of a global batch of 2048 rows: each rank
             decodes its 2048/N rows against its own page pool, at most 1024 rows per
             call (a rank with more runs its rows as consecutive calls); per-GPU and
             aggregate us per global batch and HBM fraction (strong scaling).
  cpu_baseline  the CPU oracle (C restatement of solution/triton/baseline.py) on a
             bounded sample of the same workload, all host cores.
  torch_gpu_restatement  (one GPU) the same decode math as unfused PyTorch ops on the GPU,
             timed beside the kernel as a bar, with its difference from the kernel.

With --impl reference the line reports the reference's CPU path instead (the oracle port;
the reference itself is PyTorch code that cannot travel to the GPU host).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

# The end-to-end leg keeps four buffer-slot streams in flight.  CUDA maps streams onto a
# few hardware queues (8 by default); when two slot streams share one, a step's copy waits
# behind the previous slot's decode and the step time doubles (measured 104-131 against
# 46 us per step, decided per process).  More queues, set before CUDA starts.
os.environ.setdefault("CUDA_DEVICE_MAX_CONNECTIONS", "32")

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sparse MLA decode µs/call and HBM GB/s (% of B200 peak) at 1/2/4/8 GPUs"
N_SETS = 4


def _peaks():
    """Measured HBM copy bandwidth (GB/s) and dense bf16 rate (TFLOP/s, burst) of this pool."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm": float(d["hbm_gbs"]), "bf16": float(d["bf16_tflops"]), "source": "measured"}
    except Exception:
        return {"hbm": 6650.0, "bf16": 1590.0, "source": "fallback"}


DECODE_SOURCES = ("dsa_decode.cu", "dsa_decode_h16.cuh", "dsa_decode_hm.cuh", "dsa_pipeline.cuh",
                  "sm100_ptx.cuh")


def kernel_digest() -> str:
    """SHA-256 (16 hex digits) of the CUDA sources the decode kernels are built from."""
    import hashlib

    csrc = os.path.join(ROOT, "flashinfer_mlsys2026_dsa_b200", "csrc")
    h = hashlib.sha256()
    for name in DECODE_SOURCES:
        with open(os.path.join(csrc, name), "rb") as f:
            h.update(name.encode() + b"\0" + f.read())
    return h.hexdigest()[:16]


def measured_traffic(workload: str):
    """DRAM bytes (read + write) of one call of `workload` from the committed ncu capture.

    profiles/dram_traffic.json records, per workload, the bytes of one captured launch and
    the digest of the kernel sources it was captured on; a capture of other sources is not
    this kernel's traffic, so it is reported as None with the reason.
    """
    try:
        with open(os.path.join(ROOT, "profiles", "dram_traffic.json")) as f:
            rec = json.load(f)["workloads"][workload]
    except (OSError, KeyError, ValueError):
        return None, "no ncu capture of this workload"
    if rec.get("kernel_digest") != kernel_digest():
        return None, "the ncu capture predates the current kernel sources"
    return int(rec["bytes_per_call"]), rec.get("profile", "")


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.idx = device_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sms, maxs, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                maxs.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxs),
                "reasons": sorted(reasons), "samples": len(sms)}


def _dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    return world, rank, local


def cpu_baseline(workload: str, rows: int, seed: int):
    """Oracle timing on `rows` decode rows of the workload (compacted pool), all host cores."""
    import numpy as np
    import torch

    from flashinfer_mlsys2026_dsa_b200 import workloads
    from oracle import oracle

    w = workloads.make(workload, device="cpu", seed=seed, batch=rows)
    u16 = lambda t: t.contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    idx = w.sparse_indices
    valid = idx >= 0
    slots = torch.unique(idx[valid].long())
    remap = torch.searchsorted(slots, idx.clamp(min=0).long()).to(torch.int32)
    remap = torch.where(valid, remap, torch.full_like(remap, -1)).numpy()
    ckv = u16(w.ckv_cache.view(-1, 512)[slots])
    kpe = u16(w.kpe_cache.view(-1, 64)[slots])
    qn, qp = u16(w.q_nope), u16(w.q_pe)
    cores = os.cpu_count() or 1
    oracle.decode(qn, qp, ckv, kpe, remap, w.sm_scale, nthreads=cores)  # warm-up
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.decode(qn, qp, ckv, kpe, remap, w.sm_scale, nthreads=cores)
        reps += 1
        if time.perf_counter() - t0 > 10.0 and reps >= 2:
            break
    dt = (time.perf_counter() - t0) / reps
    gbs = w.algorithmic_bytes() / dt / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{rows} of the {workload} rows (all heads, topk {w.topk}), compacted pool, "
                      f"{reps} calls, {dt * 1e3:.1f} ms/call",
            "ms_per_call": dt * 1e3}


def run_reference(args):
    world, rank, _ = _dist_setup(args.gpus)
    if rank != 0:
        return
    base = cpu_baseline(args.workload, args.cpu_rows, args.seed)
    from flashinfer_mlsys2026_dsa_b200 import workloads
    # The whole job of the GPU arm: `rows_per_rank` rows on each of the N ranks (b2048: the
    # global 2048 rows).  The host's cores run it all, so its time is the per-row time of
    # the sample times every row of the job; GB/s stays per byte, as in the GPU arm.
    rows_per_rank = (workloads.CONFIGS[args.workload]["B"] if args.workload != "b2048"
                     else 2048 // args.gpus)
    job_rows = rows_per_rank * world
    ms_full = base["ms_per_call"] * job_rows / args.cpu_rows  # rows are independent
    line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_full, 3), "higher_is_better": True,
            "scaling": "weak" if args.workload != "b2048" else "strong",
            "vs_baseline": None, "dtype": "bf16 in, fp32 math", "data": "synthetic",
            "config": {"workload": args.workload, "rows_per_rank": rows_per_rank,
                       "job_rows": job_rows, "heads": workloads.CONFIGS[args.workload]["H"],
                       "topk": workloads.CONFIGS[args.workload]["topk"], "page_size": 64,
                       "sample_rows": args.cpu_rows,
                       "basis": "whole job on all host cores: value is job bytes / job time, "
                                "the same basis as the GPU arm's value; the host's cores do "
                                "not grow with N"},
            "cpu_baseline": {k: v for k, v in base.items() if k != "ms_per_call"},
            "gpu_reference": "unmeasured: the reference's Triton kernel (solution/triton/"
                             "fused.py) needs its sources, which are not present on the GPU "
                             "host",
            "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def max_over_ranks(values, world, device):
    """Element-wise max of per-rank timings (ms) over all ranks of the default group."""
    import torch
    import torch.distributed as dist

    t = torch.tensor(values, dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def sum_over_ranks(values, world, device):
    """Element-wise sum of per-rank values over all ranks of the default group."""
    import torch
    import torch.distributed as dist

    t = torch.tensor(values, dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return t.tolist()


def job_gbs(bytes_per_step, steps, world, max_ms):
    """Whole-job throughput: the bytes of every rank's steps over the slowest rank's time."""
    return bytes_per_step * steps * world / (max_ms * 1e-3) / 1e9


def graph_ms(calls, reps, warmup, stream, barrier=lambda: None):
    """Device ms per call: CUDA-graph replays of `calls` (each replay runs each call once),
    timed with CUDA events on the launching stream after `warmup` replays."""
    import torch

    with torch.cuda.stream(stream):
        for c in calls:
            c()  # eager first: allocates the stream's workspace outside the capture
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for c in calls:
                c()
        for _ in range(warmup):
            g.replay()
        stream.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            g.replay()
        e1.record(stream)
        stream.synchronize()
    ms = e0.elapsed_time(e1) / (reps * len(calls))
    del g
    return ms


def roofline_record(nbytes, nflops, ms, peaks, traffic_of):
    """HBM (and tensor-pipe) roofline of one call of `nbytes` / `nflops` taking `ms`."""
    gbs = nbytes / (ms * 1e-3) / 1e9
    traffic, note = traffic_of
    rec = {"bound": "hbm", "achieved": round(gbs, 1), "peak": peaks["hbm"], "unit": "GB/s",
           "frac": round(gbs / peaks["hbm"], 4), "traffic": traffic,
           "peak_source": peaks["source"], "algorithmic_bytes_per_call": int(nbytes)}
    if traffic is None:
        rec["traffic_note"] = note
    tflops = nflops / (ms * 1e-3) / 1e12
    tensor = {"achieved_tflops": round(tflops, 1), "peak_tflops": peaks["bf16"],
              "frac": round(tflops / peaks["bf16"], 4), "algorithmic_flops_per_call": int(nflops)}
    return rec, tensor


def workload_record(name, dev, stream, args, peaks, kernel, read_device_errors):
    """One GPU, one configuration: four rotating input sets, graph-replayed like `value`."""
    import torch

    from flashinfer_mlsys2026_dsa_b200 import workloads

    sets = [workloads.make(name, device=dev, seed=args.seed * 97 + s) for s in range(N_SETS)]
    B, H = sets[0].num_tokens, sets[0].num_heads
    out = torch.empty(B, H, 512, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B, H, dtype=torch.float32, device=dev)
    calls = [lambda w=w: kernel(*w.args(), out, lse) for w in sets]
    reps = max(1, math.ceil(args.steps / N_SETS))
    ms = graph_ms(calls, reps, max(1, math.ceil(args.warmup / N_SETS)), stream)
    nbytes = sum(w.algorithmic_bytes() for w in sets) / N_SETS
    nflops = sum(w.algorithmic_flops() for w in sets) / N_SETS
    roof, tensor = roofline_record(nbytes, nflops, ms, peaks, measured_traffic(name))
    rec = {"us_per_call": round(ms * 1e3, 2), "value": roof["achieved"], "unit": "GB/s",
           "rows": B, "heads": H, "topk": sets[0].topk, "roofline": roof, "tensor": tensor,
           "tokens_per_s": round(B / (ms * 1e-3), 1),
           "l2": f"{N_SETS} rotating input sets of {nbytes / 1e6:.0f} MB each"}
    with torch.cuda.stream(stream):
        rec["device_errors"] = read_device_errors(dev)
    del sets, calls, out, lse
    torch.cuda.empty_cache()
    return rec


def torch_restatement(w):
    """The decode of solution/triton/baseline.py:17-45 as plain PyTorch ops on the tensors'
    device: gather the selected rows of the flattened pools, fp32 logits over the 576-d key
    scaled by sm_scale, -inf where the index is -1, base-2 log-sum-exp, softmax, PV, bf16
    output.  An unfused GPU program of the same math, timed beside the kernel as a bar; it
    is a restatement, not the reference's own code, whose sources are not on the GPU host."""
    import torch

    ckv = w.ckv_cache.reshape(-1, 512)
    kpe = w.kpe_cache.reshape(-1, 64)
    valid = w.sparse_indices != -1
    safe = torch.where(valid, w.sparse_indices, torch.zeros_like(w.sparse_indices)).long()
    kc = ckv[safe].float()  # [B, topk, 512]
    kp = kpe[safe].float()  # [B, topk, 64]
    logits = (torch.matmul(w.q_nope.float(), kc.transpose(1, 2)) +
              torch.matmul(w.q_pe.float(), kp.transpose(1, 2))) * w.sm_scale
    logits = logits.masked_fill(~valid[:, None, :], float("-inf"))
    lse = torch.logsumexp(logits, dim=-1) * (1.0 / math.log(2.0))
    out = torch.matmul(torch.softmax(logits, dim=-1), kc).to(torch.bfloat16)
    return out, lse


def torch_restatement_record(names, dev, stream, args, kernel):
    """us per call of torch_restatement on each workload (one GPU, four rotating input sets,
    eager calls timed with CUDA events on the launching stream), and its largest difference
    from the kernel's output on the same inputs."""
    import torch

    from flashinfer_mlsys2026_dsa_b200 import workloads

    rec = {}
    for name in names:
        sets = [workloads.make(name, device=dev, seed=args.seed * 97 + s) for s in range(N_SETS)]
        B, H = sets[0].num_tokens, sets[0].num_heads
        out = torch.empty(B, H, 512, dtype=torch.bfloat16, device=dev)
        lse = torch.empty(B, H, dtype=torch.float32, device=dev)
        reps = 3
        with torch.cuda.stream(stream):
            for w in sets:
                torch_restatement(w)
            stream.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                for w in sets:
                    torch_restatement(w)
            e1.record(stream)
            e1.synchronize()
            us = e0.elapsed_time(e1) / (reps * len(sets)) * 1e3
            ref_out, ref_lse = torch_restatement(sets[0])
            kernel(*sets[0].args(), out, lse)
            stream.synchronize()
        ok = torch.isfinite(ref_lse)
        rec[name] = {"us_per_call": round(us, 1),
                     "max_abs_out_diff_vs_kernel": float((ref_out.float() - out.float()).abs().max()),
                     "max_abs_lse_diff_vs_kernel": float((ref_lse[ok] - lse[ok]).abs().max())}
        del sets, out, lse, ref_out, ref_lse
        torch.cuda.empty_cache()
    rec["method"] = ("the decode math of solution/triton/baseline.py:17-45 as unfused PyTorch ops "
                     "on the GPU (gather, fp32 matmuls, masked softmax, base-2 LSE), eager, "
                     "CUDA events; a restatement timed as a bar, not the reference's own code")
    return rec


# Multi-token rows: the last 128 tokens of 8 sequences (1024 rows of 16 heads), decoded per
# token (kernel() on each token's selection) and in groups of 8 tokens (union_groups +
# kernel_grouped).  "all": 2048-token sequences, every token selects all its causal
# positions (full overlap); "random": 32768-token sequences, 2048 positions per token drawn
# independently (the least overlap).
MULTI_TOKEN_CASES = {"prefill_all": dict(seq_len=2048, mode="all"),
                     "prefill_random": dict(seq_len=32768, mode="random")}


def multi_token_record(dev, stream, args, kernel, kernel_grouped, union_groups,
                       read_device_errors):
    """Per-token against grouped decode of prefill chunks (one GPU, four rotating sets)."""
    import torch

    from flashinfer_mlsys2026_dsa_b200 import workloads

    recs = {}
    for name, cfg in MULTI_TOKEN_CASES.items():
        sets = [workloads.make_prefill(8, 128, cfg["seq_len"], heads=16, topk=2048,
                                       mode=cfg["mode"], device=dev, seed=args.seed * 13 + s)
                for s in range(N_SETS)]
        B, H = sets[0].num_tokens, sets[0].num_heads
        G = 128 // H
        out = torch.empty(B, H, 512, dtype=torch.bfloat16, device=dev)
        lse = torch.empty(B, H, dtype=torch.float32, device=dev)
        tables = [w.page_table[::G].contiguous() for w in sets]
        with torch.cuda.stream(stream):
            unions = [union_groups(w.positions, t, G) for w, t in zip(sets, tables)]
        stream.synchronize()
        reps = max(1, math.ceil(args.steps / N_SETS))
        wu = max(1, math.ceil(args.warmup / N_SETS))
        per_token = graph_ms([lambda w=w: kernel(*w.args(), out, lse) for w in sets], reps, wu,
                             stream)
        grouped = graph_ms([lambda w=w, u=u: kernel_grouped(w.q_nope, w.q_pe, w.ckv_cache,
                                                            w.kpe_cache, u[0], u[1], w.sm_scale,
                                                            out, lse)
                            for w, u in zip(sets, unions)], reps, wu, stream)
        union_ms = graph_ms([lambda w=w, t=t: union_groups(w.positions, t, G)
                             for w, t in zip(sets, tables)], reps, wu, stream)
        sel = sum(float((w.positions >= 0).sum().item()) for w in sets) / N_SETS
        uni = sum(float(u[2].sum().item()) for u in unions) / N_SETS
        rec = {"tokens": B, "heads": H, "group": G, "seq_len": cfg["seq_len"],
               "selection": cfg["mode"], "topk": 2048,
               "union_over_selections": round(uni / sel, 4),
               "per_token_us_per_call": round(per_token * 1e3, 2),
               "grouped_us_per_call": round(grouped * 1e3, 2),
               "union_us_per_call": round(union_ms * 1e3, 2),
               "per_token_us_per_token": round(per_token * 1e3 / B, 4),
               "grouped_us_per_token": round((grouped + union_ms) * 1e3 / B, 4),
               "gain": round(per_token / (grouped + union_ms), 3)}
        with torch.cuda.stream(stream):
            rec["device_errors"] = read_device_errors(dev)
        recs[name] = rec
        del sets, unions, tables, out, lse
        torch.cuda.empty_cache()
    recs["method"] = ("per token: kernel() over each token's own selection; grouped: "
                      "union_groups (union of 8 tokens' selections + membership bytes) then "
                      "kernel_grouped (one 128-head row per group), both CUDA-graph replayed "
                      "over 4 rotating input sets; gain = per-token time / (union + grouped)")
    return recs


B2048_MAX_ROWS_PER_CALL = 1024  # a 1024-row shard's page pool is about 82 GB


def b2048_record(dev, stream, args, peaks, kernel, world, rank, barrier):
    """The global 2048-row batch sharded over the ranks (strong scaling).

    Rank r decodes rows [r * 2048/N, (r + 1) * 2048/N), each rank with its own page pool,
    in calls of at most 1024 rows: one call per rank from 2 GPUs up, two consecutive calls
    on one GPU (whose single pool would not fit beside the other buffers).  Rows are
    independent, so a rank's time for the global batch is the sum of its calls' times.
    The generator's piece index is rank * calls + call, so the same seed splits the same
    2048 rows across ranks and calls.
    """
    import torch

    from flashinfer_mlsys2026_dsa_b200 import workloads

    rows = 2048 // world
    calls = max(1, -(-rows // B2048_MAX_ROWS_PER_CALL))
    reps = max(3, args.steps)
    t_ms, nbytes, nflops = 0.0, 0.0, 0.0
    for c in range(calls):
        w = workloads.make("b2048", device=dev, seed=args.seed, rank=rank * calls + c,
                           world_size=world * calls)
        out = torch.empty(w.num_tokens, 16, 512, dtype=torch.bfloat16, device=dev)
        lse = torch.empty(w.num_tokens, 16, dtype=torch.float32, device=dev)
        t_ms += graph_ms([lambda: kernel(*w.args(), out, lse)], reps, args.warmup, stream,
                         barrier)
        nbytes += w.algorithmic_bytes()
        nflops += w.algorithmic_flops()
        del w, out, lse
        torch.cuda.empty_cache()
    t_max, = max_over_ranks([t_ms], world, dev)
    job_bytes, = sum_over_ranks([nbytes], world, dev)
    per_gpu_gbs = job_bytes / world / (t_max * 1e-3) / 1e9
    return {
        "global_batch": 2048, "rows_per_rank": rows, "calls_per_rank": calls,
        "us_per_global_batch": round(t_max * 1e3, 2),
        "per_gpu": {"us": round(t_max * 1e3, 2), "value": round(per_gpu_gbs, 1), "unit": "GB/s",
                    "hbm_frac": round(per_gpu_gbs / peaks["hbm"], 4),
                    "basis": "the slowest rank's time for its rows; bytes per rank"},
        "aggregate": {"value": round(job_bytes / (t_max * 1e-3) / 1e9, 1), "unit": "GB/s",
                      "tokens_per_s": round(2048 / (t_max * 1e-3), 1),
                      "algorithmic_bytes": int(job_bytes)},
        "scaling": "strong", "n_gpus": world,
        "timing": f"per call: CUDA-graph replay x{reps}, CUDA events, max over ranks",
    }


def run_ours(args):
    import torch
    import torch.distributed as dist

    from flashinfer_mlsys2026_dsa_b200 import (kernel, kernel_grouped, kernel_paged,
                                               read_device_errors, topk_slots, union_groups,
                                               workloads)

    world, rank, local = _dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # The end-to-end leg's buffer-slot streams are the process's first streams, so that
    # each gets a hardware queue of its own (created later, after the other legs' streams,
    # two of them shared one in some runs and a step waited behind the previous slot).
    NSLOT = 4
    slot_stream = [torch.cuda.Stream(device=dev) for _ in range(NSLOT)]
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    peaks = _peaks()
    wl_world = world if args.workload == "b2048" else 1
    sets = [workloads.make(args.workload, device=dev, seed=args.seed * 97 + s, rank=rank,
                           world_size=wl_world) for s in range(N_SETS)]
    B, H = sets[0].num_tokens, sets[0].num_heads
    # kernels of this library per call: one (the cluster kernel merges split rows itself)
    launches_per_call = 1
    bytes_per_step = sum(w.algorithmic_bytes() for w in sets) / N_SETS
    flops_per_step = sum(w.algorithmic_flops() for w in sets) / N_SETS
    out = torch.empty(B, H, 512, dtype=torch.bfloat16, device=dev)
    lse = torch.empty(B, H, dtype=torch.float32, device=dev)
    stream = torch.cuda.Stream(device=dev)

    # ---------------- device-resident timing (graph replay of the 4 rotating steps)
    with torch.cuda.stream(stream):
        for w in sets:
            kernel(*w.args(), out, lse)
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for w in sets:
                kernel(*w.args(), out, lse)
        reps = max(1, math.ceil(args.steps / N_SETS))
        steps = reps * N_SETS
        for _ in range(max(1, math.ceil(args.warmup / N_SETS))):
            graph.replay()
        stream.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            # keep the GPU busy long enough for the clock sampler to see it under load
            busy_until = time.perf_counter() + 0.5
            while time.perf_counter() < busy_until:
                graph.replay()
                stream.synchronize()
            torch.cuda.synchronize(dev)
            barrier()
            e0.record(stream)
            for _ in range(reps):
                graph.replay()
            e1.record(stream)
            stream.synchronize()
        torch.cuda.synchronize(dev)
        err = read_device_errors(dev)
    dev_ms = e0.elapsed_time(e1)
    del graph

    # ---------------- the same steps through the paged entry (positions + page tables;
    # the slot ids are formed inside the kernel), device-timed the same way
    pargs = [(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, w.page_table, w.positions,
              w.sm_scale) for w in sets]
    paged_ms = graph_ms([lambda a=a: kernel_paged(*a, out, lse) for a in pargs], reps,
                        max(1, math.ceil(args.warmup / N_SETS)), stream, barrier) * N_SETS * reps
    with torch.cuda.stream(stream):
        err |= read_device_errors(dev)

    # ---------------- end to end through the public API, host buffers
    # Every step copies its query and index rows from pinned host memory, runs the public
    # kernel() and copies out/lse back.  Steps are pipelined the way a server runs them: a
    # step runs wholly on the stream of its buffer slot (host-to-device copy, decode,
    # device-to-host copy, in stream order), and four slots rotate, so one step's copies
    # overlap the decodes of its neighbours.  No event crosses streams: on this platform
    # cross-stream event chains between copy and compute streams measured 50-140 us per
    # step for the same work, against 47 us for this layout.  A step's inputs (q_nope, q_pe,
    # indices) sit in one pinned host buffer and cross in one copy; out and lse sit in one
    # device buffer and come back in one copy.
    def packed(parts, device=None, pinned=False):
        sizes = [t.numel() * t.element_size() for t in parts]
        offs = [0]
        for n in sizes[:-1]:
            offs.append(offs[-1] + (n + 255) // 256 * 256)
        buf = torch.empty(offs[-1] + sizes[-1], dtype=torch.uint8, device=device,
                          pin_memory=pinned)
        views = [buf[o:o + n].view(t.dtype).view(t.shape) for o, n, t in zip(offs, sizes, parts)]
        return buf, views

    host_in = []
    for w in sets:
        buf, views = packed([w.q_nope, w.q_pe, w.sparse_indices], pinned=True)
        for v, t in zip(views, (w.q_nope, w.q_pe, w.sparse_indices)):
            v.copy_(t.cpu())
        host_in.append(buf)
    dev_in = [packed([sets[0].q_nope, sets[0].q_pe, sets[0].sparse_indices], device=dev)
              for _ in range(NSLOT)]
    out_proto = [torch.empty(B, H, 512, dtype=torch.bfloat16), torch.empty(B, H, dtype=torch.float32)]
    dev_out = [packed(out_proto, device=dev) for _ in range(NSLOT)]
    host_out = [packed(out_proto, pinned=True) for _ in range(NSLOT)]
    h2d = host_in[0].numel()
    d2h = host_out[0][0].numel()
    home = torch.cuda.current_stream(dev)

    assert NSLOT == N_SETS  # slot sl always carries input set sl

    def slot_body(sl):
        w = sets[sl]
        ibuf, (qn, qp, idx) = dev_in[sl]
        obuf, (o, l) = dev_out[sl]
        ibuf.copy_(host_in[sl], non_blocking=True)
        kernel(qn, qp, w.ckv_cache, w.kpe_cache, idx, w.sm_scale, o, l)
        host_out[sl][0].copy_(obuf, non_blocking=True)

    # A slot's step (H2D copy, the public kernel() call, D2H copy) is captured once into a
    # CUDA graph on the slot's stream, after eager warm-up steps, and replayed per step: the
    # host then issues one launch per step (about 6 us instead of 18-25 us of Python), so
    # host jitter no longer reaches the device timeline.
    for k in range(max(3, args.warmup) + NSLOT):
        with torch.cuda.stream(slot_stream[k % NSLOT]):
            slot_body(k % NSLOT)
    torch.cuda.synchronize(dev)
    slot_graph = []
    for sl in range(NSLOT):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=slot_stream[sl]):
            slot_body(sl)
        slot_graph.append(g)
    torch.cuda.synchronize(dev)

    def e2e_step(k):
        sl = k % NSLOT
        torch.cuda.set_stream(slot_stream[sl])  # a graph replays on the current stream
        slot_graph[sl].replay()
        torch.cuda.set_stream(home)

    for k in range(NSLOT):
        e2e_step(k)
    def e2e_trial():
        torch.cuda.synchronize(dev)
        barrier()
        f0 = torch.cuda.Event(enable_timing=True)
        f1 = torch.cuda.Event(enable_timing=True)
        f0.record(home)
        for st in slot_stream:
            st.wait_event(f0)
        h0 = time.perf_counter()
        for k in range(steps):
            e2e_step(k)
        h_us = (time.perf_counter() - h0) / steps * 1e6
        for st in slot_stream:
            done = torch.cuda.Event()
            done.record(st)
            home.wait_event(done)
        f1.record(home)
        f1.synchronize()
        return f0.elapsed_time(f1), h_us

    # Untimed warm-up trials first: after the device-only region above, the first ~0.3 s of
    # host<->device copies ran at about half speed (four slots: ~100 us per step, then a
    # steady 44-45 us with the same graphs), so about 1.2 s of steps bring the link to its
    # steady state. Every rank runs the same number of trials (each trial has a barrier).
    first_ms = max_over_ranks([e2e_trial()[0]], world, dev)[0]
    warm_trials = 1 + int(min(200, max(2, math.ceil(1200.0 / max(first_ms, 1e-3)))))
    for _ in range(warm_trials - 1):
        e2e_trial()
    # Three timed trials of `steps` steps each; the median trial is reported, all three
    # beside it (concurrent slots make a trial's copy-engine overlap vary between runs).
    trials = sorted(e2e_trial() for _ in range(3))
    e2e_ms, host_us = trials[1]
    e2e_trials_us = [round(t[0] / steps * 1e3, 1) for t in trials]
    # the last step's results really are on the host
    assert torch.isfinite(host_out[(steps - 1) % NSLOT][1][1]).any()
    for st in slot_stream:  # each slot stream has a workspace of its own
        with torch.cuda.stream(st):
            err |= read_device_errors(dev)
    # the step's copies alone, back to back on one stream (what bounds e2e when the decode
    # is hidden under them)
    copy_us = {}
    for name, (dst, src) in {"h2d": (dev_in[0][0], host_in[0]),
                             "d2h": (host_out[0][0], dev_out[0][0])}.items():
        torch.cuda.synchronize(dev)
        c0 = torch.cuda.Event(enable_timing=True)
        c1 = torch.cuda.Event(enable_timing=True)
        c0.record(slot_stream[0])
        with torch.cuda.stream(slot_stream[0]):
            for _ in range(steps):
                dst.copy_(src, non_blocking=True)
        c1.record(slot_stream[0])
        c1.synchronize()
        copy_us[name] = c0.elapsed_time(c1) / steps * 1e3

    # ---------------- index production, the step before the decode: each row's top-k
    # positions of index scores over its whole sequence, as slot ids, alone and chained
    # with the decode (the ids cross HBM once, 8 KB per row)
    index_rec = None
    if not args.no_extra:
        gsc = torch.Generator(device=dev).manual_seed(args.seed + 5)
        topk_in = []
        for w in sets:
            sc = torch.randn(B, int(max(w.seq_lens)), generator=gsc, device=dev)
            ln = torch.tensor(w.seq_lens, dtype=torch.int32, device=dev)
            ids = torch.empty(B, w.topk, dtype=torch.int32, device=dev)
            topk_in.append((sc, ln, ids, w))

        def chained(a):
            topk_slots(a[0], a[1], a[3].page_table, a[3].topk, out=a[2])
            kernel(a[3].q_nope, a[3].q_pe, a[3].ckv_cache, a[3].kpe_cache, a[2], a[3].sm_scale,
                   out, lse)

        warm = max(1, math.ceil(args.warmup / N_SETS))
        t_ms = graph_ms([lambda a=a: topk_slots(a[0], a[1], a[3].page_table, a[3].topk, out=a[2])
                         for a in topk_in], reps, warm, stream, barrier)
        c_ms = graph_ms([lambda a=a: chained(a) for a in topk_in], reps, warm, stream, barrier)
        t_ms, c_ms = max_over_ranks([t_ms, c_ms], world, dev)
        n_scores = sum(sum(a[3].seq_lens) for a in topk_in) / N_SETS
        index_rec = {"topk_us_per_call": round(t_ms * 1e3, 2),
                     "topk_then_decode_us_per_call": round(c_ms * 1e3, 2),
                     "scores_per_call": int(n_scores),
                     "scores_per_s": round(n_scores / (t_ms * 1e-3), 1),
                     "method": "topk_slots(): fp32 index scores of every position of each row "
                               "(seq_len 4k-32k) -> the 2048 best as slot ids, exact, one "
                               "launch; then kernel() on those ids; CUDA-graph replay over "
                               "the same 4 input sets as value"}
        with torch.cuda.stream(stream):
            err |= read_device_errors(dev)
        del topk_in

    dev_ms, e2e_ms, paged_ms = max_over_ranks([dev_ms, e2e_ms, paged_ms], world, dev)
    ms_per_step = dev_ms / steps
    value, e2e_value = job_gbs(bytes_per_step, steps, world, dev_ms), job_gbs(
        bytes_per_step, steps, world, e2e_ms)
    per_call_gbs = bytes_per_step / (ms_per_step * 1e-3) / 1e9
    roof, tensor = roofline_record(bytes_per_step, flops_per_step, ms_per_step, peaks,
                                   measured_traffic(args.workload))
    del sets, host_in, dev_in, dev_out, host_out, out, lse
    torch.cuda.empty_cache()

    # ---------------- the other configurations (one GPU) and the global 2048-row batch
    extra = {}
    if world == 1 and not args.no_extra:
        for name in ("b32_h128", "ragged_b256"):
            if name != args.workload:
                extra[name] = workload_record(name, dev, stream, args, peaks, kernel,
                                              read_device_errors)
    b2048 = None if args.no_extra else b2048_record(dev, stream, args, peaks, kernel, world,
                                                    rank, barrier)
    multi = None
    torch_bar = None
    if world == 1 and not args.no_extra:
        multi = multi_token_record(dev, stream, args, kernel, kernel_grouped, union_groups,
                                   read_device_errors)
        torch_bar = torch_restatement_record(tuple(dict.fromkeys((args.workload, "b32_h128"))),
                                             dev, stream, args, kernel)

    base = None
    if rank == 0 and not args.no_cpu_baseline:
        base = cpu_baseline(args.workload, args.cpu_rows, args.seed)
        base.pop("ms_per_call", None)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "us_per_call": round(ms_per_step * 1e3, 2),
        "tokens_per_s": round(B * world / (ms_per_step * 1e-3), 1),
        "hbm_frac_of_measured": round(per_call_gbs / peaks["hbm"], 4),
        "hbm_frac_of_nominal_8tbs": round(per_call_gbs / 8000.0, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 (fp32 accumulate)", "data": "synthetic",
        "config": {"workload": args.workload, "rows_per_rank": B, "heads": H,
                   "topk": workloads.CONFIGS[args.workload]["topk"],
                   "page_size": 64, "parallelism": f"batch-sharded x{world}",
                   "l2": f"{N_SETS} rotating input sets of {bytes_per_step / 1e6:.0f} MB each "
                         f"(> 126 MB L2)", "timing": "CUDA graph replay, CUDA events"},
        "roofline": roof,
        "tensor": tensor,
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms / steps, 4),
                "host_us_per_step": round(host_us, 1),
                "trials_us_per_step": e2e_trials_us, "warmup_trials": warm_trials,
                "h2d_copy_us": round(copy_us["h2d"], 1), "d2h_copy_us": round(copy_us["d2h"], 1),
                "method": "public kernel() per step; one pinned H2D copy of the step's q_nope, "
                          "q_pe, indices and one D2H copy of its out, lse inside the timed "
                          "region; each step wholly on its buffer slot's stream (copy in, "
                          "decode, copy out), four slots rotating, no cross-stream events; "
                          "a slot's step (both copies and the kernel() call) captured once "
                          "as a CUDA graph and replayed per step; after ~1.2 s of untimed "
                          "trials (the host link's steady state), median of 3 trials"},
        "paged_entry": {"us_per_call": round(paged_ms / steps * 1e3, 2),
                        "value": round(job_gbs(bytes_per_step, steps, world, paged_ms), 1),
                        "unit": "GB/s",
                        "method": "kernel_paged(): token positions + page tables in, slot ids "
                                  "formed in the kernel; same steps, bytes and timing as value"},
        "gpu_launches": steps * launches_per_call,
        "clocks": clk.summary(),
        "device_errors": err,
    }
    if index_rec is not None:
        line["index_production"] = index_rec
    if extra:
        line["workloads"] = extra
    if b2048 is not None:
        line["b2048"] = b2048
    if multi is not None:
        line["multi_token"] = multi
    if torch_bar is not None:
        line["torch_gpu_restatement"] = torch_bar
    if base is not None:
        line["cpu_baseline"] = base
    print(json.dumps(line), flush=True)


def main():
    global N_SETS
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--workload", default="b64_h16",
                    choices=["b64_h16", "b32_h128", "ragged_b256", "b2048", "tiny"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-rows", type=int, default=0,
                    help="decode rows in the CPU-baseline sample (default: one per host core, "
                         "at most the workload's rows)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the other configurations and the 2048-row batch")
    ap.add_argument("--sets", type=int, default=N_SETS,
                    help="rotating input sets of the main workload (fewer keep an ncu capture "
                         "small; the bytes of one set must still exceed the L2 for DRAM figures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    N_SETS = max(1, args.sets)
    if args.cpu_rows <= 0:
        from flashinfer_mlsys2026_dsa_b200.workloads import CONFIGS
        args.cpu_rows = max(1, min(CONFIGS[args.workload]["B"], os.cpu_count() or 1))
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
