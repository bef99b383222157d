"""The token-group union oracle (input of the grouped decode), checked on the CPU.

oracle.union_groups_numpy against an independent vectorised restatement (np.unique over
position * 8 + token) on random selections with cross-token duplicates, -1 entries,
positions past the table, a missing page and a cut union.
"""
import numpy as np
import pytest

from oracle import oracle


def _union_vectorised(pos, pt, group, page_size, out_cols):
    pos = np.asarray(pos, np.int64)
    groups = pos.shape[0] // group
    max_pos = pt.shape[1] * page_size
    slots = np.full((groups, out_cols), -1, np.int32)
    member = np.zeros((groups, out_cols), np.uint8)
    counts = np.zeros(groups, np.int32)
    for g in range(groups):
        p = pos[g * group:(g + 1) * group]
        tok = np.repeat(np.arange(group), p.shape[1]).reshape(p.shape)
        ok = (p >= 0) & (p < max_pos)
        q, t = p[ok], tok[ok]
        u, inv = np.unique(q, return_inverse=True)
        bits = np.zeros(len(u), np.int64)
        np.bitwise_or.at(bits, inv, 1 << t)
        counts[g] = len(u)
        n = min(len(u), out_cols)
        page = pt[g, u[:n] // page_size].astype(np.int64)
        s = np.where(page >= 0, page * page_size + u[:n] % page_size, -1)
        slots[g, :n] = s
        member[g, :n] = np.where(s >= 0, bits[:n], 0)
    return slots, member, counts


@pytest.mark.parametrize("group,k,page_size", [(8, 64, 64), (4, 100, 16), (2, 257, 1), (1, 32, 64)])
def test_union_oracle_matches_vectorised_restatement(group, k, page_size):
    rng = np.random.default_rng(group * 1000 + k)
    groups, seq = 5, 900
    pos = np.full((groups * group, k), -1, np.int32)
    for t in range(groups * group):
        n = int(rng.integers(0, k + 1))
        pos[t, :n] = rng.choice(seq + 40, n, replace=False)  # some past the table
    cols = -(-seq // page_size)
    pt = np.stack([rng.permutation(4 * cols)[:cols] for _ in range(groups)]).astype(np.int32)
    pt[1, cols // 2] = -1  # a missing page
    for out_cols in (group * k, max(1, group * k // 3)):
        a = oracle.union_groups_numpy(pos, pt, group, page_size, out_cols)
        b = _union_vectorised(pos, pt, group, page_size, out_cols)
        for x, y in zip(a, b):
            np.testing.assert_array_equal(x, y)


def test_union_of_causal_prefill_selections_is_the_longest():
    # short context: every token selects all positions up to its own, so a group's union
    # is the last token's selection and every earlier token is a member of a prefix
    group, k = 8, 2048
    L = 1000
    pos = np.full((group, k), -1, np.int32)
    for j in range(group):
        p = L - group + j
        pos[j, :p + 1] = np.arange(p + 1)
    pt = np.arange(16, dtype=np.int32)[None, :]
    slots, member, counts = oracle.union_groups_numpy(pos, pt, group, 64, group * k)
    assert counts[0] == L
    np.testing.assert_array_equal(slots[0, :L], np.arange(L))
    assert (member[0, :L - group + 1] == 0xFF).all()
    assert member[0, L - 1] == 0x80
