"""Multi-token rows decoded in token groups: union kernel, top-k positions, grouped decode.

A group of G = 128 / H consecutive tokens of one sequence is decoded as one 128-head row
over the union of the tokens' selections (each union slot gathered once for the group;
a membership byte per entry masks the other tokens' heads).  Checked here: the union
kernel bit for bit against the numpy oracle; top-k without a page table (positions)
against the C oracle; the grouped decode against the oracle's per-token decode of each
token's own selection, and against the per-token CUDA path, at 16, 32 and 64 heads,
with full overlap (short-context prefill), independent random selections, tokens with
no selection and a cut union.
"""
import numpy as np
import pytest
import torch

from flashinfer_mlsys2026_dsa_b200 import (kernel, kernel_grouped, read_device_errors,
                                           topk_slots, union_groups, workloads)
from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _clear_errors():
    read_device_errors(clear=True)
    yield


def _np(t):
    return t.cpu().numpy()


@pytest.mark.parametrize("group,k,page_size", [(8, 2048, 64), (4, 300, 16), (2, 1000, 1), (1, 64, 64)])
def test_union_kernel_matches_oracle(group, k, page_size):
    g = torch.Generator(device="cuda").manual_seed(group * 31 + k)
    groups, seq = 13, 70000
    tokens = groups * group
    pos = torch.full((tokens, k), -1, dtype=torch.int32, device="cuda")
    for t in range(tokens):
        n = int(torch.randint(0, k + 1, (1,), generator=g, device="cuda").item())
        pos[t, :n] = torch.randperm(seq + 500, generator=g, device="cuda")[:n].to(torch.int32)
    cols = -(-seq // page_size)
    pt = torch.stack([torch.randperm(3 * cols, generator=g, device="cuda")[:cols]
                      for _ in range(groups)]).to(torch.int32)
    pt[2, cols // 3] = -1
    for out_cols in (None, max(1, group * k // 4)):
        s, m, c = union_groups(pos, pt, group, out_cols=out_cols, page_size=page_size)
        torch.cuda.synchronize()
        oc = s.shape[1]
        rs, rm, rc = oracle.union_groups_numpy(_np(pos), _np(pt), group, page_size, oc)
        np.testing.assert_array_equal(_np(c), rc)
        np.testing.assert_array_equal(_np(s), rs)
        np.testing.assert_array_equal(_np(m), rm)


def test_topk_positions_without_page_table():
    g = torch.Generator(device="cuda").manual_seed(3)
    rows, L, k = 9, 20000, 2048
    sc = torch.randn(rows, L, generator=g, device="cuda")
    sc[1] = torch.round(sc[1] * 2)  # ties
    lengths = torch.tensor([L, L, 5000, 100, L, 2048, 2049, 0, 17], dtype=torch.int32, device="cuda")
    out = topk_slots(sc, lengths, None, k)
    ident = np.arange(L, dtype=np.int32)[None, :].repeat(rows, 0)
    ref = oracle.topk_slots(_np(sc), _np(lengths), ident, k, 1)
    np.testing.assert_array_equal(_np(out), ref)


def _group_table(w, group):
    return w.page_table[::group].contiguous()


def _check_grouped(w, group, out_cols=None):
    s, m, c = union_groups(w.positions, _group_table(w, group), group, out_cols=out_cols)
    B, H = w.num_tokens, w.num_heads
    out = torch.full((B, H, 512), float("nan"), dtype=torch.bfloat16, device="cuda")
    lse = torch.full((B, H), float("nan"), dtype=torch.float32, device="cuda")
    kernel_grouped(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, s, m, w.sm_scale, out, lse)
    ref = torch.empty_like(out)
    ref_lse = torch.empty_like(lse)
    kernel(*w.args(), ref, ref_lse)
    torch.cuda.synchronize()
    assert read_device_errors() == 0
    from test_gpu_parity import assert_close, oracle_on_workload
    o_out, o_lse = oracle_on_workload(w)
    assert_close(out.float().cpu().numpy(), lse.cpu().numpy(), o_out, o_lse)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.float().cpu().numpy(), atol=1e-2, rtol=1e-2)
    return s, m, c


@pytest.mark.parametrize("heads", [16, 32, 64])
def test_grouped_decode_full_overlap(heads):
    group = 128 // heads
    w = workloads.make_prefill(5, 32, 2000, heads=heads, topk=2048, mode="all", seed=heads)
    s, m, c = _check_grouped(w, group)
    # every group's union is its last token's selection
    last = (w.positions[group - 1::group] >= 0).sum(1).to(torch.int32)
    assert torch.equal(c, last)


@pytest.mark.parametrize("heads", [16, 64])
def test_grouped_decode_random_selections(heads):
    group = 128 // heads
    w = workloads.make_prefill(3, 16, 9000, heads=heads, topk=512, mode="random", seed=7)
    _check_grouped(w, group)


def test_grouped_decode_tokens_without_selection_and_split_rows():
    # 160 groups of 8 tokens: more rows than cluster pairs, so rows are split between
    # pairs and merged; two tokens select nothing (output 0, lse -inf)
    w = workloads.make_prefill(10, 128, 1500, heads=16, topk=2048, mode="all", seed=2)
    w.positions[3] = -1
    w.positions[600] = -1
    w.sparse_indices[3] = -1
    w.sparse_indices[600] = -1
    s, m, c = union_groups(w.positions, _group_table(w, 8), 8)
    out = torch.empty(w.num_tokens, 16, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(w.num_tokens, 16, dtype=torch.float32, device="cuda")
    kernel_grouped(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, s, m, w.sm_scale, out, lse)
    torch.cuda.synchronize()
    assert read_device_errors() == 0
    for t in (3, 600):
        assert (out[t].float() == 0).all()
        assert torch.isneginf(lse[t]).all()
    from test_gpu_parity import assert_close, oracle_on_workload
    keep = [t for t in range(w.num_tokens) if t not in (3, 600)]
    o_out, o_lse = oracle_on_workload(w, rows=keep)
    assert_close(out[keep].float().cpu().numpy(), lse[keep].cpu().numpy(), o_out, o_lse)


def test_grouped_argument_errors():
    w = workloads.make_prefill(1, 8, 500, heads=16, topk=512, mode="all")
    s, m, c = union_groups(w.positions, _group_table(w, 8), 8)
    out = torch.empty(8, 16, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(8, 16, dtype=torch.float32, device="cuda")
    with pytest.raises(ValueError):  # token count not a multiple of the group
        kernel_grouped(w.q_nope[:7], w.q_pe[:7], w.ckv_cache, w.kpe_cache, s, m, w.sm_scale,
                       out[:7], lse[:7])
    with pytest.raises(ValueError):  # membership of another shape
        kernel_grouped(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, s, m[:, :10], w.sm_scale,
                       out, lse)
    with pytest.raises(ValueError):  # group does not divide the tokens
        union_groups(w.positions[:6], _group_table(w, 8), 8)
