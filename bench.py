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
             device-resident state, like a serving engine's cache).
  roofline   achieved GB/s of the decode call vs the measured HBM peak.
  cpu_baseline  the CPU oracle (C restatement of solution/triton/baseline.py) on a
             bounded sample of the same workload, all host cores.

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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sparse MLA decode µs/call and HBM GB/s (% of B200 peak) at 1/2/4/8 GPUs"
N_SETS = 4


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


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
    B = workloads.CONFIGS[args.workload]["B"] if args.workload != "b2048" else 2048 // args.gpus
    ms_full = base["ms_per_call"] * B / args.cpu_rows  # rows are independent
    line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms_full, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16 in, fp32 math", "data": "synthetic",
            "config": {"workload": args.workload, "rows_per_rank": B, "heads": 16, "topk": 2048,
                       "page_size": 64, "sample_rows": args.cpu_rows},
            "cpu_baseline": {k: v for k, v in base.items() if k != "ms_per_call"},
            "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# DRAM bytes (read + write) of one decode launch, from the ncu capture summarised in
# profiles/dsa_decode_h16_b64_h16_metrics.md (dram__bytes_read.sum + dram__bytes_write.sum).
MEASURED_TRAFFIC = {"b64_h16": 160330496}


def max_over_ranks(values, world, device):
    """Element-wise max of per-rank timings (ms) over all ranks of the default group."""
    import torch
    import torch.distributed as dist

    t = torch.tensor(values, dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def job_gbs(bytes_per_step, steps, world, max_ms):
    """Whole-job throughput: the bytes of every rank's steps over the slowest rank's time."""
    return bytes_per_step * steps * world / (max_ms * 1e-3) / 1e9


def run_ours(args):
    import torch
    import torch.distributed as dist

    from flashinfer_mlsys2026_dsa_b200 import kernel, kernel_paged, read_device_errors, workloads

    world, rank, local = _dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    wl_world = world if args.workload == "b2048" else 1
    sets = [workloads.make(args.workload, device=dev, seed=args.seed * 97 + s, rank=rank,
                           world_size=wl_world) for s in range(N_SETS)]
    B, H = sets[0].num_tokens, sets[0].num_heads
    # kernels of this library per call: one (the cluster kernel merges split rows itself)
    launches_per_call = 1
    bytes_per_step = sum(w.algorithmic_bytes() for w in sets) / N_SETS
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
    dev_ms = e0.elapsed_time(e1)
    err = read_device_errors(dev)

    # ---------------- the same steps through the paged entry (positions + page tables;
    # the slot ids are formed inside the kernel), device-timed the same way
    with torch.cuda.stream(stream):
        pargs = [(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, w.page_table, w.positions,
                  w.sm_scale) for w in sets]
        for a in pargs:
            kernel_paged(*a, out, lse)
        stream.synchronize()
        pgraph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(pgraph, stream=stream):
            for a in pargs:
                kernel_paged(*a, out, lse)
        for _ in range(max(1, math.ceil(args.warmup / N_SETS))):
            pgraph.replay()
        stream.synchronize()
        barrier()
        p0 = torch.cuda.Event(enable_timing=True)
        p1 = torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        for _ in range(reps):
            pgraph.replay()
        p1.record(stream)
        stream.synchronize()
    paged_ms = p0.elapsed_time(p1)
    err |= read_device_errors(dev)
    del pgraph

    # ---------------- end to end through the public API, host buffers
    # Every step copies its query and index rows from pinned host memory, runs the public
    # kernel() and copies out/lse back.  Steps are pipelined the way a server runs them:
    # host-to-device copies, decode and device-to-host copies go on three streams, with
    # two device buffer slots, so step k's copies overlap the decode of step k-1.
    # A step's inputs (q_nope, q_pe, indices) sit in one pinned host buffer and cross in
    # one copy; out and lse sit in one device buffer and come back in one copy.
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
    NSLOT = 2
    dev_in = [packed([sets[0].q_nope, sets[0].q_pe, sets[0].sparse_indices], device=dev)
              for _ in range(NSLOT)]
    out_proto = [torch.empty(B, H, 512, dtype=torch.bfloat16), torch.empty(B, H, dtype=torch.float32)]
    dev_out = [packed(out_proto, device=dev) for _ in range(NSLOT)]
    host_out = [packed(out_proto, pinned=True) for _ in range(NSLOT)]
    h2d = host_in[0].numel()
    d2h = host_out[0][0].numel()
    s_in, s_run, s_out = (torch.cuda.Stream(device=dev) for _ in range(3))
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_done = [ev() for _ in range(NSLOT)]
    run_done = [ev() for _ in range(NSLOT)]
    out_done = [ev() for _ in range(NSLOT)]
    started = [False] * NSLOT
    home = torch.cuda.current_stream(dev)

    def e2e_step(k):
        w = sets[k % N_SETS]
        sl = k % NSLOT
        ibuf, (qn, qp, idx) = dev_in[sl]
        obuf, (o, l) = dev_out[sl]
        torch.cuda.set_stream(s_in)
        if started[sl]:
            s_in.wait_event(run_done[sl])          # the decode of step k-2 read this slot
        ibuf.copy_(host_in[k % N_SETS], non_blocking=True)
        in_done[sl].record(s_in)
        torch.cuda.set_stream(s_run)
        s_run.wait_event(in_done[sl])
        if started[sl]:
            s_run.wait_event(out_done[sl])         # step k-2's outputs have been copied out
        kernel(qn, qp, w.ckv_cache, w.kpe_cache, idx, w.sm_scale, o, l)
        run_done[sl].record(s_run)
        torch.cuda.set_stream(s_out)
        s_out.wait_event(run_done[sl])
        host_out[sl][0].copy_(obuf, non_blocking=True)
        out_done[sl].record(s_out)
        torch.cuda.set_stream(home)
        started[sl] = True

    for k in range(max(3, args.warmup)):
        e2e_step(k)
    torch.cuda.synchronize(dev)
    barrier()
    f0 = torch.cuda.Event(enable_timing=True)
    f1 = torch.cuda.Event(enable_timing=True)
    f0.record(s_in)
    s_run.wait_event(f0)
    s_out.wait_event(f0)
    for k in range(steps):
        e2e_step(k)
    s_in.wait_event(out_done[(steps - 1) % NSLOT])
    f1.record(s_in)
    f1.synchronize()
    e2e_ms = f0.elapsed_time(f1)
    # the last step's results really are on the host
    assert torch.isfinite(host_out[(steps - 1) % NSLOT][1][1]).any()

    dev_ms, e2e_ms, paged_ms = max_over_ranks([dev_ms, e2e_ms, paged_ms], world, dev)
    ms_per_step = dev_ms / steps
    value, e2e_value = job_gbs(bytes_per_step, steps, world, dev_ms), job_gbs(
        bytes_per_step, steps, world, e2e_ms)
    peak, peak_kind = _peaks()
    per_call_gbs = bytes_per_step / (ms_per_step * 1e-3) / 1e9

    base = None
    if rank == 0 and not args.no_cpu_baseline:
        base = cpu_baseline(args.workload, args.cpu_rows, args.seed)
        base.pop("ms_per_call", None)
    if world > 1:
        dist.barrier()
        del graph
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 5),
        "us_per_call": round(ms_per_step * 1e3, 2),
        "tokens_per_s": round(B * world / (ms_per_step * 1e-3), 1),
        "hbm_frac_of_measured": round(per_call_gbs / peak, 4),
        "hbm_frac_of_nominal_8tbs": round(per_call_gbs / 8000.0, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16 (fp32 accumulate)", "data": "synthetic",
        "config": {"workload": args.workload, "rows_per_rank": B, "heads": H,
                   "topk": sets[0].topk, "page_size": 64, "parallelism": f"batch-sharded x{world}",
                   "l2": f"{N_SETS} rotating input sets of {bytes_per_step / 1e6:.0f} MB each "
                         f"(> 126 MB L2)", "timing": "CUDA graph replay, CUDA events"},
        "roofline": {"bound": "hbm", "achieved": round(per_call_gbs, 1), "peak": peak,
                     "unit": "GB/s", "frac": round(per_call_gbs / peak, 4),
                     "traffic": MEASURED_TRAFFIC.get(args.workload), "peak_source": peak_kind,
                     "algorithmic_bytes_per_call": int(bytes_per_step)},
        "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms / steps, 4),
                "method": "public kernel() per step; one pinned H2D copy of the step's q_nope, "
                          "q_pe, indices and one D2H copy of its out, lse inside the timed "
                          "region; copies and decode on three streams with two buffer slots "
                          "(step k's copies overlap step k-1's decode)"},
        "paged_entry": {"us_per_call": round(paged_ms / steps * 1e3, 2),
                        "value": round(job_gbs(bytes_per_step, steps, world, paged_ms), 1),
                        "unit": "GB/s",
                        "method": "kernel_paged(): token positions + page tables in, slot ids "
                                  "formed in the kernel; same steps, bytes and timing as value"},
        "gpu_launches": steps * launches_per_call,
        "clocks": clk.summary(),
        "device_errors": err,
    }
    if base is not None:
        line["cpu_baseline"] = base
    print(json.dumps(line), flush=True)


def main():
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
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.cpu_rows <= 0:
        from flashinfer_mlsys2026_dsa_b200.workloads import CONFIGS
        args.cpu_rows = max(1, min(CONFIGS[args.workload]["B"], os.cpu_count() or 1))
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
