"""The CPU oracle against the reference's own outputs (tests/golden/golden.npz).

golden.npz was written by tests/golden/make_golden.py, which runs the
reference implementation (solution/triton/baseline.py) on the seeded inputs of
cases.py.  Passing here pins the oracle before it is used to check the GPU.
"""
import json
import os

import numpy as np
import pytest

import cases
from oracle import oracle

GOLDEN = np.load(os.path.join(os.path.dirname(cases.__file__), "golden.npz"))
META = json.load(open(os.path.join(os.path.dirname(cases.__file__), "golden.json")))


@pytest.fixture(scope="module", autouse=True)
def _built():
    oracle.build()


@pytest.mark.parametrize("name", sorted(cases.CASES))
def test_inputs_match_fixture_digest(name):
    c = cases.make_case(name)
    assert cases.input_digest(c) == META["cases"][name]["digest"], \
        "input generator changed: regenerate the fixtures with make_golden.py"


@pytest.mark.parametrize("name", sorted(cases.CASES))
def test_c_oracle_matches_reference(name):
    c = cases.make_case(name)
    out, lse = oracle.decode(c["q_nope"], c["q_pe"], c["ckv_cache"], c["kpe_cache"],
                             c["sparse_indices"], c["sm_scale"], nthreads=4)
    ref_out = oracle.bf16_bits_to_f32(GOLDEN[f"{name}.out"])
    ref_lse = GOLDEN[f"{name}.lse"]
    got = oracle.bf16_bits_to_f32(out)
    # same NaN / inf pattern as the reference (all-padding rows)
    np.testing.assert_array_equal(np.isnan(got), np.isnan(ref_out))
    np.testing.assert_array_equal(np.isneginf(lse), np.isneginf(ref_lse))
    fin = np.isfinite(ref_out)
    # summation order differs from torch's fp32 bmm: at most one bf16 ulp apart
    np.testing.assert_allclose(got[fin], ref_out[fin], atol=2e-3, rtol=8e-3)
    fl = np.isfinite(ref_lse)
    np.testing.assert_allclose(lse[fl], ref_lse[fl], atol=1e-5, rtol=0)
    assert np.mean(out[fin] == GOLDEN[f"{name}.out"][fin]) > 0.99


@pytest.mark.parametrize("name", ["tiny_b2_h16_k256", "ragged_pad", "mid_pad", "h128_k256"])
def test_numpy_restatement_agrees_with_c(name):
    c = cases.make_case(name)
    a_out, a_lse = oracle.decode(*[c[k] for k in ("q_nope", "q_pe", "ckv_cache", "kpe_cache",
                                                  "sparse_indices", "sm_scale")])
    b_out, b_lse = oracle.decode_numpy(*[c[k] for k in ("q_nope", "q_pe", "ckv_cache",
                                                        "kpe_cache", "sparse_indices", "sm_scale")])
    np.testing.assert_allclose(oracle.bf16_bits_to_f32(a_out), oracle.bf16_bits_to_f32(b_out),
                               atol=2e-3, rtol=8e-3)
    np.testing.assert_allclose(a_lse, b_lse, atol=1e-5)


def _tiny():
    return cases.make_case("tiny_b2_h16_k256")


def test_kat_single_valid_index():
    """One valid slot: out = that ckv row, lse = its scaled score in base 2."""
    c = _tiny()
    idx = np.full_like(c["sparse_indices"], -1)
    idx[:, 7] = c["sparse_indices"][:, 7]
    out, lse = oracle.decode(c["q_nope"], c["q_pe"], c["ckv_cache"], c["kpe_cache"], idx, c["sm_scale"])
    kc = oracle.bf16_bits_to_f32(c["ckv_cache"].reshape(-1, 512))
    kp = oracle.bf16_bits_to_f32(c["kpe_cache"].reshape(-1, 64))
    qn = oracle.bf16_bits_to_f32(c["q_nope"])
    qp = oracle.bf16_bits_to_f32(c["q_pe"])
    for b in range(idx.shape[0]):
        s = idx[b, 7]
        np.testing.assert_array_equal(out[b], np.broadcast_to(oracle.f32_to_bf16_bits(kc[s]), (16, 512)))
        score = (qn[b] @ kc[s] + qp[b] @ kp[s]) * c["sm_scale"] / np.log(2.0)
        np.testing.assert_allclose(lse[b], score, atol=1e-4)


def test_kat_zero_query_is_mean_of_values():
    """q = 0: uniform attention, out = mean of the valid rows, lse = log2(n_valid)."""
    c = _tiny()
    zq = np.zeros_like(c["q_nope"])
    zp = np.zeros_like(c["q_pe"])
    idx = c["sparse_indices"].copy()
    idx[1, 100:] = -1
    out, lse = oracle.decode(zq, zp, c["ckv_cache"], c["kpe_cache"], idx, c["sm_scale"])
    kc = oracle.bf16_bits_to_f32(c["ckv_cache"].reshape(-1, 512))
    for b in range(2):
        v = idx[b][idx[b] >= 0]
        np.testing.assert_allclose(oracle.bf16_bits_to_f32(out[b, 0]), kc[v].mean(0), atol=4e-3, rtol=8e-3)
        np.testing.assert_allclose(lse[b], np.log2(len(v)), atol=1e-5)


def test_permutation_and_padding_invariance():
    c = _tiny()
    base_out, base_lse = oracle.decode(c["q_nope"], c["q_pe"], c["ckv_cache"], c["kpe_cache"],
                                       c["sparse_indices"], c["sm_scale"])
    rng = np.random.default_rng(5)
    perm = c["sparse_indices"][:, rng.permutation(256)]
    padded = np.concatenate([perm, np.full((2, 64), -1, np.int32)], axis=1)
    out, lse = oracle.decode(c["q_nope"], c["q_pe"], c["ckv_cache"], c["kpe_cache"], padded, c["sm_scale"])
    np.testing.assert_allclose(oracle.bf16_bits_to_f32(out), oracle.bf16_bits_to_f32(base_out), atol=2e-3, rtol=8e-3)
    np.testing.assert_allclose(lse, base_lse, atol=1e-5)


def test_out_of_range_index_raises_like_reference():
    c = _tiny()
    idx = c["sparse_indices"].copy()
    idx[0, 3] = 32 * 64  # one past the last slot
    with pytest.raises(IndexError):
        oracle.decode(c["q_nope"], c["q_pe"], c["ckv_cache"], c["kpe_cache"], idx, c["sm_scale"])
