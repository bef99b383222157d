"""Multi-rank host logic on CPU (gloo, world size 2).

The decode path shards by rows with no collective on the data path; what the ranks share
is the timing reduction of the benchmark (max over ranks) and the per-rank workload
construction.  A rank that leaves early must surface as an error on the other rank within
the process group's timeout, not as a hang.
"""
import os
import socket
import subprocess
import sys
import textwrap

import pytest
import torch

import bench
from flashinfer_mlsys2026_dsa_b200 import workloads

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_ranks(body: str, world: int = 2, timeout: float = 120.0):
    """Run `body` in `world` fresh interpreters as gloo ranks; return their outputs."""
    script = textwrap.dedent("""
        import os, sys, datetime
        sys.path.insert(0, {repo!r})
        import torch, torch.distributed as dist
        rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=5))
    """).format(repo=REPO) + textwrap.dedent(body)
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), CUDA_VISIBLE_DEVICES="")
        procs.append(subprocess.Popen([sys.executable, "-c", script], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT,
                                      text=True))
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=timeout)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
            raise AssertionError("rank did not finish:\n" + out)
        outs.append((p.returncode, out))
    return outs


def test_max_over_ranks_and_job_throughput():
    outs = _run_ranks("""
        import bench
        mine = [10.0 + rank, 30.0 - rank]          # device ms, e2e ms
        dev_ms, e2e_ms = bench.max_over_ranks(mine, world, "cpu")
        print("RESULT", dev_ms, e2e_ms, bench.job_gbs(1e9, 4, world, dev_ms))
        dist.destroy_process_group()
    """)
    for rc, out in outs:
        assert rc == 0, out
        line = [l for l in out.splitlines() if l.startswith("RESULT")][0].split()
        assert float(line[1]) == 11.0 and float(line[2]) == 30.0
        assert abs(float(line[3]) - 1e9 * 4 * 2 / 11e-3 / 1e9) < 1e-6


def test_job_throughput_is_all_ranks_bytes_over_the_slowest_rank():
    assert bench.job_gbs(2e8, 10, 4, 100.0) == pytest.approx(2e8 * 10 * 4 / 0.1 / 1e9)
    assert bench.max_over_ranks([3.0, 4.0], 1, "cpu") == [3.0, 4.0]


def test_row_shards_are_disjoint_deterministic_and_self_contained():
    a0 = workloads.make("tiny", device="cpu", seed=3, rank=0, world_size=2, batch=4)
    a1 = workloads.make("tiny", device="cpu", seed=3, rank=1, world_size=2, batch=4)
    b0 = workloads.make("tiny", device="cpu", seed=3, rank=0, world_size=2, batch=4)
    assert a0.num_tokens == a1.num_tokens == 2
    # the same (seed, rank) gives the same shard; different ranks get different rows
    assert torch.equal(a0.sparse_indices, b0.sparse_indices)
    assert torch.equal(a0.q_nope, b0.q_nope)
    assert not torch.equal(a0.q_nope, a1.q_nope)
    for w in (a0, a1):
        slots = w.ckv_cache.shape[0] * w.ckv_cache.shape[1]
        idx = w.sparse_indices
        assert int(idx.max()) < slots and int(idx.min()) >= -1
        # each row's valid slots are distinct (topk of distinct positions)
        for r in range(idx.shape[0]):
            v = idx[r][idx[r] >= 0]
            assert v.unique().numel() == v.numel()
    with pytest.raises(ValueError):
        workloads.make("tiny", device="cpu", rank=0, world_size=3, batch=4)


def test_a_rank_that_leaves_early_fails_the_other_rank_promptly():
    outs = _run_ranks("""
        import time
        dist.barrier()
        if rank == 1:
            os._exit(0)          # leaves between steps, before the next collective
        t = time.time()
        try:
            dist.barrier()
            print("NO-ERROR")
        except Exception as e:   # gloo reports the lost peer
            print("ERROR after %.1f s: %s" % (time.time() - t, type(e).__name__))
    """, timeout=60.0)
    rc0, out0 = outs[0]
    assert "ERROR after" in out0, out0
    assert outs[1][0] == 0
