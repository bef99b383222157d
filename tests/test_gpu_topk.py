"""The index-production kernel (dsa_topk_slots) against the C oracle, bit-exact.

Every case compares the whole [rows, k] slot array: the same selected set (ties at the
k-th score to the smaller positions), the same ascending order, the same -1 padding.
"""
import numpy as np
import pytest
import torch

from flashinfer_mlsys2026_dsa_b200 import kernel, read_device_errors, topk_slots, workloads
from oracle import oracle

pytestmark = pytest.mark.gpu


def _run(sc, lengths, pt, k, page_size):
    got = topk_slots(torch.from_numpy(sc).cuda(), torch.from_numpy(lengths).cuda(),
                     torch.from_numpy(pt).cuda(), k, page_size)
    torch.cuda.synchronize()
    return got.cpu().numpy()


def _case(seed, rows, max_len, ties=False, special=False, page_size=64):
    rng = np.random.default_rng(seed)
    sc = rng.standard_normal((rows, max_len)).astype(np.float32)
    if ties:
        sc = np.round(sc * 2).astype(np.float32)
    if special:
        for r in range(rows):
            sc[r, rng.integers(0, max_len, 50)] = -0.0
            sc[r, rng.integers(0, max_len, 50)] = 0.0
            sc[r, rng.integers(0, max_len, 5)] = np.inf
            sc[r, rng.integers(0, max_len, 5)] = -np.inf
            sc[r, rng.integers(0, max_len, 20)] = np.nan
    lengths = rng.integers(0, max_len + 1, size=rows).astype(np.int32)
    lengths[0] = max_len
    lengths[1] = 0
    pages = (max_len + page_size - 1) // page_size
    pt = np.stack([rng.permutation(4 * pages)[:pages] for _ in range(rows)]).astype(np.int32)
    return sc, lengths, pt


@pytest.mark.parametrize("max_len", [9000, 13000])  # one CTA per row; two (past 12k positions)
@pytest.mark.parametrize("k", [1, 64, 2048])
@pytest.mark.parametrize("ties,special", [(False, False), (True, False), (False, True)])
def test_topk_slots_match_oracle(k, ties, special, max_len):
    sc, lengths, pt = _case(k + 3 * ties + 5 * special + max_len, 12, max_len, ties, special)
    np.testing.assert_array_equal(_run(sc, lengths, pt, k, 64),
                                  oracle.topk_slots(sc, lengths, pt, k, 64))


def _sm_count():
    return torch.cuda.get_device_properties(0).multi_processor_count


@pytest.mark.parametrize("max_len", [3000, 60000])
def test_topk_slots_one_cta_per_row(max_len):
    """More rows than half the SMs: one CTA per row (keys cached in shared memory at 3000
    positions, read from global memory at 60000)."""
    rows = _sm_count() // 2 + 9
    sc, lengths, pt = _case(21 + max_len, rows, max_len, ties=max_len == 3000)
    np.testing.assert_array_equal(_run(sc, lengths, pt, 256, 64),
                                  oracle.topk_slots(sc, lengths, pt, 256, 64))


@pytest.mark.parametrize("ties", [False, True])
def test_topk_slots_same_result_for_one_and_two_ctas_per_row(ties):
    """The first rows of a call small enough for two CTAs per row (rows past 12k
    positions), padded with copies of them to a call that runs one CTA per row: the same
    slots."""
    few = 16
    sc, lengths, pt = _case(31 + ties, few, 20000, ties=ties)
    lengths[2:6] = [20000, 19999, 2049, 4097]  # halves that are not multiples of 4
    reps = (_sm_count() // 2) // few + 1
    got_few = _run(sc, lengths, pt, 2048, 64)
    got_many = _run(np.tile(sc, (reps, 1)), np.tile(lengths, reps), np.tile(pt, (reps, 1)), 2048, 64)
    assert reps * few * 2 > _sm_count()
    np.testing.assert_array_equal(got_few, got_many[:few])
    np.testing.assert_array_equal(got_few, oracle.topk_slots(sc, lengths, pt, 2048, 64))


def test_topk_slots_long_rows_and_token_granular_table():
    sc, lengths, pt = _case(11, 4, 131072)
    lengths[:] = [131072, 131071, 2049, 2048]
    np.testing.assert_array_equal(_run(sc, lengths, pt, 2048, 64),
                                  oracle.topk_slots(sc, lengths, pt, 2048, 64))
    sc, lengths, pt = _case(12, 6, 5000, ties=True, page_size=1)
    np.testing.assert_array_equal(_run(sc, lengths, pt, 300, 1),
                                  oracle.topk_slots(sc, lengths, pt, 300, 1))


def test_topk_then_decode_equals_decode_of_oracle_slots():
    """Chained: the kernel's slot ids feed the decode, which gives what the oracle ids give."""
    w = workloads.make("b64_h16", device="cuda", seed=9, batch=16)
    rows = w.num_tokens
    max_len = int(max(w.seq_lens))
    g = torch.Generator(device="cuda").manual_seed(3)
    scores = torch.randn(rows, max_len, generator=g, device="cuda")
    lengths = torch.tensor(w.seq_lens, dtype=torch.int32, device="cuda")
    slots = topk_slots(scores, lengths, w.page_table, 2048)
    want = oracle.topk_slots(scores.cpu().numpy(), lengths.cpu().numpy(),
                             w.page_table.cpu().numpy(), 2048, 64)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(slots.cpu().numpy(), want)
    out = torch.empty(rows, 16, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(rows, 16, dtype=torch.float32, device="cuda")
    kernel(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, slots, w.sm_scale, out, lse)
    out2, lse2 = torch.empty_like(out), torch.empty_like(lse)
    kernel(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, torch.from_numpy(want).cuda(), w.sm_scale,
           out2, lse2)
    torch.cuda.synchronize()
    assert read_device_errors() == 0
    assert torch.equal(out, out2) and torch.equal(lse, lse2)


def test_topk_slots_argument_errors():
    sc = torch.zeros(2, 10, device="cuda")
    ln = torch.zeros(2, dtype=torch.int32, device="cuda")
    pt = torch.zeros(2, 1, dtype=torch.int32, device="cuda")
    with pytest.raises(TypeError):
        topk_slots(sc.half(), ln, pt, 4)
    with pytest.raises(ValueError):
        topk_slots(sc, ln, pt, 0)
    with pytest.raises(ValueError):
        topk_slots(sc.cpu(), ln, pt, 4)
