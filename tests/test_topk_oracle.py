"""The index-production oracle (top-k of index scores -> slot ids), checked on the CPU.

The C restatement (oracle/dsa_oracle.c) against an independent numpy one, on ties, signed
zeros, infinities, NaN, short rows and table misses; and against flashinfer's published
reference of the step (top_k_page_table_transform) on tie-free scores, as sets.
"""
import numpy as np
import pytest

from oracle import oracle


def _case(seed, rows, max_len, ties=False, special=False):
    rng = np.random.default_rng(seed)
    sc = rng.standard_normal((rows, max_len)).astype(np.float32)
    if ties:
        sc = np.round(sc * 2).astype(np.float32)
    if special:
        sc[0, 5:15] = -0.0
        sc[0, 15:25] = 0.0
        sc[0, 25] = np.inf
        sc[0, 26] = -np.inf
        sc[0, 27:40] = np.nan
    lengths = rng.integers(0, max_len + 100, size=rows).astype(np.int32)
    lengths[0] = max_len
    pages = (max_len + 63) // 64
    pt = np.stack([rng.permutation(10 * pages)[:pages] for _ in range(rows)]).astype(np.int32)
    pt[-1, pages // 2:] = -1  # a row whose later pages are missing
    return sc, lengths, pt


@pytest.mark.parametrize("k", [1, 100, 512, 2048])
@pytest.mark.parametrize("ties,special", [(False, False), (True, False), (False, True)])
def test_c_oracle_matches_numpy_restatement(k, ties, special):
    sc, lengths, pt = _case(k, 6, 4000, ties, special)
    a = oracle.topk_slots(sc, lengths, pt, k, 64)
    b = oracle.topk_slots_numpy(sc, lengths, pt, k, 64)
    np.testing.assert_array_equal(a, b)


def test_selection_order_and_padding():
    sc = np.array([[0.5, 3.0, 3.0, -1.0, 3.0, 2.0, -0.0, 0.0]], dtype=np.float32)
    pt = np.array([[7]], dtype=np.int32)
    # the three 3.0s tie for the top; k = 2 takes positions 1 and 2 (smaller positions)
    np.testing.assert_array_equal(oracle.topk_slots(sc, [8], pt, 2, 64), [[7 * 64 + 1, 7 * 64 + 2]])
    # +0.0 ranks above -0.0: the top 6 leave out -1.0 and -0.0
    np.testing.assert_array_equal(oracle.topk_slots(sc, [8], pt, 6, 64),
                                  [[448, 449, 450, 452, 453, 455]])
    # a row shorter than k: every position in order, then -1
    np.testing.assert_array_equal(oracle.topk_slots(sc, [3], pt, 5, 64), [[448, 449, 450, -1, -1]])


def test_matches_flashinfer_published_reference():
    torch = pytest.importorskip("torch")
    try:
        from flashinfer.trace.templates.sampling import \
            _top_k_page_table_transform_reference as ref
    except Exception as e:  # pragma: no cover - the library is part of the image
        pytest.skip(f"flashinfer reference unavailable: {e}")
    rng = np.random.default_rng(7)
    rows, L, k = 5, 6000, 512
    sc = rng.standard_normal((rows, L)).astype(np.float32)  # continuous scores: no ties
    lengths = np.array([6000, 4097, 700, 512, 100], np.int32)
    table = rng.integers(0, 1 << 20, size=(rows, L)).astype(np.int32)  # one entry per token
    want = ref(torch.from_numpy(sc), torch.from_numpy(table), torch.from_numpy(lengths), k).numpy()
    got = oracle.topk_slots(sc, lengths, table, k, 1)  # page size 1: a token-granular table
    for r in range(rows):
        n = min(k, int(lengths[r]))
        assert sorted(got[r, :n].tolist()) == sorted(want[r, :n].tolist())
        assert (got[r, n:] == -1).all()
