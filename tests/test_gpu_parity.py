"""Parity of the CUDA path (through the C ABI) with the reference and the oracle.

Tolerances (the operator's contract): output within atol = rtol = 1e-2 of the
reference, lse within 1e-3 absolute (base 2), padded slots contribute exactly
zero.  Small cases compare against the reference's own outputs (golden.npz);
the benchmark-size configs compare against the C oracle run on the compacted
pool of the slots they reference.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import cases
from flashinfer_mlsys2026_dsa_b200 import _native, kernel, ops, read_device_errors, workloads
from oracle import oracle

pytestmark = pytest.mark.gpu

OUT_TOL = dict(atol=1e-2, rtol=1e-2)
LSE_ATOL = 1e-3
GOLDEN = np.load(os.path.join(os.path.dirname(cases.__file__), "golden.npz"))


def to_dev(c):
    dev = "cuda"
    t = lambda a: torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16).to(dev)  # noqa: E731
    return (t(c["q_nope"]), t(c["q_pe"]), t(c["ckv_cache"]), t(c["kpe_cache"]),
            torch.from_numpy(c["sparse_indices"]).to(dev), c["sm_scale"])


def run(args):
    q_nope = args[0]
    B, H, _ = q_nope.shape
    out = torch.full((B, H, 512), float("nan"), dtype=torch.bfloat16, device=q_nope.device)
    lse = torch.full((B, H), float("nan"), dtype=torch.float32, device=q_nope.device)
    kernel(*args, out, lse)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), lse.cpu().numpy()


def assert_close(out, lse, ref_out, ref_lse):
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out, ref_out, **OUT_TOL)
    fin = np.isfinite(ref_lse)
    np.testing.assert_array_equal(np.isneginf(lse), np.isneginf(ref_lse))
    np.testing.assert_allclose(lse[fin], ref_lse[fin], atol=LSE_ATOL, rtol=0)


@pytest.fixture(autouse=True)
def _clear_errors():
    read_device_errors(clear=True)
    yield


@pytest.mark.parametrize("name", sorted(set(cases.CASES) - cases.REFERENCE_ONLY))
def test_golden_cases_match_reference(name):
    c = cases.make_case(name)
    out, lse = run(to_dev(c))
    ref_out = oracle.bf16_bits_to_f32(GOLDEN[f"{name}.out"])
    assert_close(out, lse, ref_out, GOLDEN[f"{name}.lse"])
    assert read_device_errors() == 0


def test_all_padding_row_writes_zero_and_neg_inf():
    """The reference gives NaN / -inf for a row with no valid slot; this path gives 0 / -inf."""
    c = cases.make_case("all_pad_row")
    out, lse = run(to_dev(c))
    ref_out = oracle.bf16_bits_to_f32(GOLDEN["all_pad_row.out"])
    assert_close(out[:1], lse[:1], ref_out[:1], GOLDEN["all_pad_row.lse"][:1])
    assert (out[1] == 0).all() and np.isneginf(lse[1]).all()


def test_bad_index_is_flagged_and_treated_as_padding():
    c = cases.make_case("neg_index")
    out, lse = run(to_dev(c))
    assert read_device_errors() & _native.DEVERR_BAD_INDEX
    idx = c["sparse_indices"].copy()
    idx[idx < -1] = -1
    ref_out, ref_lse = oracle.decode(c["q_nope"], c["q_pe"], c["ckv_cache"], c["kpe_cache"], idx,
                                     c["sm_scale"])
    assert_close(out, lse, oracle.bf16_bits_to_f32(ref_out), ref_lse)
    # an index past the end of the pool is flagged too, and reads nothing
    c["sparse_indices"][0, 3] = c["ckv_cache"].shape[0] * 64
    run(to_dev(c))
    assert read_device_errors() & _native.DEVERR_BAD_INDEX


def oracle_on_workload(w, rows=None):
    """C oracle on the compacted pool of the slots ``w`` references."""
    idx = w.sparse_indices if rows is None else w.sparse_indices[rows]
    qn = w.q_nope if rows is None else w.q_nope[rows]
    qp = w.q_pe if rows is None else w.q_pe[rows]
    flat_ckv = w.ckv_cache.view(-1, 512)
    flat_kpe = w.kpe_cache.view(-1, 64)
    valid = idx >= 0
    slots = torch.unique(idx[valid].long())
    remap = torch.searchsorted(slots, idx.clamp(min=0).long()).to(torch.int32)
    remap = torch.where(valid, remap, torch.full_like(remap, -1))
    u16 = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    out, lse = oracle.decode(u16(qn), u16(qp), u16(flat_ckv[slots]), u16(flat_kpe[slots]),
                             remap.cpu().numpy(), w.sm_scale)
    return oracle.bf16_bits_to_f32(out), lse


# b2048 at world sizes 8, 4 and 2: the rank-0 shard of the global 2048-row batch (256, 512
# and 1024 rows with sequences of 8k-131k tokens, page pools of about 20, 41 and 82 GB);
# the 512- and 1024-row shards run every row split between cluster pairs (stream-K).
@pytest.mark.parametrize("name,world", [("b64_h16", 1), ("b32_h128", 1), ("ragged_b256", 1),
                                        ("b2048", 8), ("b2048", 4), ("b2048", 2)])
def test_benchmark_configs_match_oracle(name, world):
    torch.cuda.empty_cache()
    w = workloads.make(name, device="cuda", seed=0, rank=0, world_size=world)
    out, lse = run(w.args())
    ref_out, ref_lse = oracle_on_workload(w)
    assert_close(out, lse, ref_out, ref_lse)
    assert read_device_errors() == 0
    # deterministic: a second call gives identical bits
    out2, lse2 = run(w.args())
    np.testing.assert_array_equal(out, out2)
    np.testing.assert_array_equal(lse, lse2)
    del w
    torch.cuda.empty_cache()


def test_strided_query_and_concatenated_cache_through_c_abi():
    """q_nope / q_pe as views of one [B,H,576] tensor; ckv/kpe as one [P,64,576] cache."""
    c = cases.make_case("h16_k2048")
    qn, qp, ckv, kpe, idx, scale = to_dev(c)
    B, H, _ = qn.shape
    qcat = torch.cat([qn, qp], dim=-1)
    kvcat = torch.cat([ckv, kpe], dim=-1)
    out = torch.empty(B, H, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, H, dtype=torch.float32, device="cuda")
    lib = _native.load()
    stream = torch.cuda.current_stream()
    ws = ops.workspace_for(qn.device, stream.cuda_stream, B, H, idx.shape[1])
    rc = lib.dsa_sparse_mla_decode(
        qcat.data_ptr(), qcat.stride(0), qcat.stride(1),
        qcat.data_ptr() + 512 * 2, qcat.stride(0), qcat.stride(1),
        kvcat.data_ptr(), 576, kvcat.data_ptr() + 512 * 2, 576, kvcat.shape[0] * 64,
        idx.data_ptr(), idx.stride(0), scale,
        out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), lse.stride(0), lse.stride(1),
        B, H, idx.shape[1], ws.data_ptr(), ws.numel(), stream.cuda_stream)
    assert rc == 0, _native.status_text(rc)
    torch.cuda.synchronize()
    assert_close(out.float().cpu().numpy(), lse.cpu().numpy(),
                 oracle.bf16_bits_to_f32(GOLDEN["h16_k2048.out"]), GOLDEN["h16_k2048.lse"])


def test_padding_and_permutation_properties():
    w = workloads.make("b64_h16", device="cuda", seed=3)
    base_out, base_lse = run(w.args())
    g = torch.Generator(device="cuda").manual_seed(1)
    perm = torch.randperm(w.topk, device="cuda", generator=g)
    idx = w.sparse_indices[:, perm]
    padded = torch.cat([torch.full((w.num_tokens, 100), -1, dtype=torch.int32, device="cuda"), idx,
                        torch.full((w.num_tokens, 28), -1, dtype=torch.int32, device="cuda")], 1)
    out, lse = run((w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, padded.contiguous(), w.sm_scale))
    np.testing.assert_allclose(out, base_out, atol=1e-2, rtol=1e-2)
    np.testing.assert_allclose(lse, base_lse, atol=1e-4)


def test_cuda_graph_replay_matches_eager():
    w = workloads.make("b64_h16", device="cuda", seed=4)
    B, H = w.num_tokens, w.num_heads
    out = torch.empty(B, H, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, H, dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        kernel(*w.args(), out, lse)  # warm-up: allocates the stream's workspace
        s.synchronize()
        ref_out, ref_lse = out.clone(), lse.clone()
        out.zero_()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            kernel(*w.args(), out, lse)
        graph.replay()
        graph.replay()
        s.synchronize()
    torch.testing.assert_close(out, ref_out, atol=0, rtol=0)
    torch.testing.assert_close(lse, ref_lse, atol=0, rtol=0)


def test_input_validation_errors():
    c = cases.make_case("tiny_b2_h16_k256")
    args = list(to_dev(c))
    out = torch.empty(2, 16, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(2, 16, dtype=torch.float32, device="cuda")
    with pytest.raises(TypeError):
        kernel(args[0].float(), *args[1:], out, lse)
    with pytest.raises(TypeError):
        kernel(*args[:4], args[4].long(), args[5], out, lse)
    with pytest.raises(ValueError):
        kernel(args[0].cpu(), *args[1:], out, lse)
    with pytest.raises(ValueError):
        kernel(args[0][:, :8], args[1][:, :8], *args[2:], out[:, :8], lse[:, :8])


def test_bounded_wait_reports_timeout_without_hanging():
    """A wait no one satisfies gives up after its bound and sets the timeout bit."""
    lib = _native.load()
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()
    assert lib.dsa_selftest_bounded_wait(2_000_000, ws.data_ptr(), stream.cuda_stream) == 0
    word = ctypes.c_uint32(0)
    assert lib.dsa_read_error_word(ws.data_ptr(), stream.cuda_stream, 1, ctypes.byref(word)) == 0
    assert word.value & _native.DEVERR_TIMEOUT
    # the context is still usable afterwards
    c = cases.make_case("tiny_b2_h16_k256")
    out, lse = run(to_dev(c))
    assert_close(out, lse, oracle.bf16_bits_to_f32(GOLDEN["tiny_b2_h16_k256.out"]),
                 GOLDEN["tiny_b2_h16_k256.lse"])


def test_shared_workspace_across_batch_sizes():
    """Calls of different batch sizes share one workspace; each must start from clean counters."""
    w = workloads.make("b64_h16", device="cuda", seed=7, batch=256)
    sizes = [64, 256, 128, 160, 20, 256]
    refs = {}
    for b in sizes:
        args = (w.q_nope[:b].contiguous(), w.q_pe[:b].contiguous(), w.ckv_cache, w.kpe_cache,
                w.sparse_indices[:b].contiguous(), w.sm_scale)
        out, lse = run(args)
        assert np.isfinite(out).all() and np.isfinite(lse).all(), f"batch {b}"
        if b in refs:  # same shape again: bit-identical
            np.testing.assert_array_equal(out, refs[b][0])
        refs.setdefault(b, (out, lse))
    ref_out, ref_lse = oracle_on_workload(w, rows=slice(0, 20))
    assert_close(refs[20][0], refs[20][1], ref_out, ref_lse)
