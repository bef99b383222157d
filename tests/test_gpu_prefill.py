"""Multi-token rows: prefill and multi-token decode as rows of the same operator.

The operator's definition counts tokens, not sequences (num_tokens rows, each with its own
top-k selection): a prefill chunk or a multi-token decode step of one sequence is several
rows that share the sequence's page table. These tests build two sequences, take their
last 128 tokens each as rows, give every token a causal selection (positions <= its own;
early tokens select fewer than topk and are padded with -1), and run them through the flat
entry (slot ids) and the paged entry (positions + the sequence's page table): bit-identical
to each other, within tolerance of the oracle.
"""
import math

import numpy as np
import pytest
import torch

from flashinfer_mlsys2026_dsa_b200 import kernel, kernel_paged, read_device_errors, workloads
from oracle import oracle

pytestmark = pytest.mark.gpu

PAGE = 64


def _prefill_rows(seq_lens, tokens_per_seq, topk, H, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    gc = torch.Generator().manual_seed(seed)
    npages = [-(-L // PAGE) for L in seq_lens]
    P = sum(npages)
    perm = torch.randperm(P, generator=gc).to("cuda")
    maxp = max(npages)
    tables, positions = [], []
    off = 0
    for L, n in zip(seq_lens, npages):
        table = torch.full((maxp,), -1, dtype=torch.int64, device="cuda")
        table[:n] = perm[off:off + n]
        off += n
        for p in range(L - tokens_per_seq, L):  # causal: token p sees positions 0..p
            k = min(topk, p + 1)
            pos = torch.randperm(p + 1, generator=g, device="cuda")[:k]
            row = torch.full((topk,), -1, dtype=torch.int64, device="cuda")
            row[:k] = pos
            tables.append(table)
            positions.append(row)
    pt = torch.stack(tables).to(torch.int32).contiguous()
    pos = torch.stack(positions).to(torch.int32).contiguous()
    B = pos.shape[0]
    q_nope = torch.randn(B, H, 512, generator=g, device="cuda", dtype=torch.bfloat16)
    q_pe = torch.randn(B, H, 64, generator=g, device="cuda", dtype=torch.bfloat16)
    ckv = (torch.randn(P, PAGE, 512, generator=g, device="cuda", dtype=torch.bfloat16) * 0.5)
    kpe = (torch.randn(P, PAGE, 64, generator=g, device="cuda", dtype=torch.bfloat16) * 0.5)
    ids = torch.from_numpy(oracle.slots_from_positions(pt.cpu().numpy(), pos.cpu().numpy(), PAGE))
    w = workloads.Workload("prefill", q_nope, q_pe, ckv, kpe, ids.cuda().contiguous(),
                           1.0 / math.sqrt(192.0), list(seq_lens), pt, pos)
    return w


def _run(fn, w, *extra):
    B, H = w.num_tokens, w.num_heads
    out = torch.full((B, H, 512), float("nan"), dtype=torch.bfloat16, device="cuda")
    lse = torch.full((B, H), float("nan"), dtype=torch.float32, device="cuda")
    fn(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, *extra, w.sm_scale, out, lse)
    torch.cuda.synchronize()
    return out, lse


@pytest.mark.parametrize("seq_lens,heads", [((3000, 1500), 16), ((2200, 700), 64)])
def test_prefill_rows_match_oracle_and_paged_entry(seq_lens, heads):
    from test_gpu_parity import assert_close, oracle_on_workload

    read_device_errors(clear=True)
    w = _prefill_rows(seq_lens, 128, 2048, heads, seed=11)
    assert (w.sparse_indices == -1).any()  # early tokens of the short sequence are padded
    flat = _run(kernel, w, w.sparse_indices)
    paged = _run(kernel_paged, w, w.page_table, w.positions)
    assert torch.equal(flat[0].view(torch.int16), paged[0].view(torch.int16))
    assert torch.equal(flat[1], paged[1])
    ref_out, ref_lse = oracle_on_workload(w)
    assert_close(flat[0].float().cpu().numpy(), flat[1].cpu().numpy(), ref_out, ref_lse)
    assert read_device_errors() == 0


def test_tokens_sharing_a_selection_give_identical_rows():
    """Two rows with the same q and the same selection (in different orders) are equal."""
    w = _prefill_rows((2500,), 2, 2048, 16, seed=5)
    w.q_nope[1] = w.q_nope[0]
    w.q_pe[1] = w.q_pe[0]
    perm = torch.randperm(2048, device="cuda")
    w.sparse_indices[1] = w.sparse_indices[0][perm]
    out, lse = _run(kernel, w, w.sparse_indices)
    np.testing.assert_allclose(out[1].float().cpu().numpy(), out[0].float().cpu().numpy(),
                               atol=1e-2, rtol=1e-2)
    np.testing.assert_allclose(lse[1].cpu().numpy(), lse[0].cpu().numpy(), atol=1e-4)
