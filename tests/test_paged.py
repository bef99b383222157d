"""Index production fused into the gather: ``kernel_paged`` / ``dsa_sparse_mla_decode_paged``.

The caller passes token positions and each row's page table; the kernel forms the slot ids
(page_table[b, pos // page_size] * page_size + pos % page_size) the reference's callers
build for ``sparse_indices`` (its pools flattened as page * 64 + offset, fused.py:155-156).

CPU: the oracle's translation against a plain loop, and against the ids the synthetic
workloads build.  GPU: the paged entry gives bit-identical results to the flat entry on the
translated ids (both run the same kernel after the translation), including split-K rows,
128 heads, a page size of 1, and invalid positions (flagged, treated as padding).
"""
import numpy as np
import pytest
import torch

from flashinfer_mlsys2026_dsa_b200 import workloads
from oracle import oracle


def _loop_translate(pt, pos, ps):
    out = np.empty(pos.shape, dtype=np.int64)
    for b in range(pos.shape[0]):
        for k in range(pos.shape[1]):
            q = int(pos[b, k])
            if q == -1:
                out[b, k] = -1
            elif q < -1 or q // ps >= pt.shape[1] or pt[b, q // ps] < 0:
                out[b, k] = -2
            else:
                out[b, k] = int(pt[b, q // ps]) * ps + q % ps
    return out


@pytest.mark.parametrize("ps", [1, 16, 64])
def test_oracle_translation_matches_loop(ps):
    rng = np.random.default_rng(ps)
    B, cols, topk = 5, 9, 40
    pt = rng.integers(-1, 50, size=(B, cols)).astype(np.int32)
    pos = rng.integers(-3, cols * ps + 5, size=(B, topk)).astype(np.int32)
    pos[:, :3] = -1
    got = oracle.slots_from_positions(pt, pos, ps)
    np.testing.assert_array_equal(got, _loop_translate(pt, pos, ps))


def test_workload_ids_are_the_translation_of_its_positions():
    for name, batch in (("tiny", None), ("b64_h16", 4), ("ragged_b256", 8)):
        w = workloads.make(name, device="cpu", seed=2, batch=batch)
        ids = oracle.slots_from_positions(w.page_table.numpy(), w.positions.numpy(), 64)
        np.testing.assert_array_equal(ids, w.sparse_indices.numpy())


# ---------------------------------------------------------------------------- GPU

def _run(fn, w, *extra, **kw):
    B, H = w.num_tokens, w.num_heads
    out = torch.full((B, H, 512), float("nan"), dtype=torch.bfloat16, device="cuda")
    lse = torch.full((B, H), float("nan"), dtype=torch.float32, device="cuda")
    fn(w.q_nope, w.q_pe, w.ckv_cache, w.kpe_cache, *extra, w.sm_scale, out, lse, **kw)
    torch.cuda.synchronize()
    return out, lse


def _same(a, b):
    assert torch.equal(a[0].view(torch.int16), b[0].view(torch.int16))
    assert torch.equal(a[1], b[1])


@pytest.mark.gpu
@pytest.mark.parametrize("name,batch", [("b64_h16", None), ("b64_h16", 256), ("b32_h128", 4),
                                        ("ragged_b256", 64)])
def test_paged_matches_flat_ids(name, batch):
    from flashinfer_mlsys2026_dsa_b200 import kernel, kernel_paged, read_device_errors

    read_device_errors(clear=True)
    w = workloads.make(name, device="cuda", seed=5, batch=batch)
    flat = _run(kernel, w, w.sparse_indices)
    paged = _run(kernel_paged, w, w.page_table, w.positions)
    _same(paged, flat)
    assert read_device_errors() == 0


@pytest.mark.gpu
def test_paged_against_oracle_small():
    from flashinfer_mlsys2026_dsa_b200 import kernel_paged

    w = workloads.make("tiny", device="cuda", seed=9)
    out, lse = _run(kernel_paged, w, w.page_table, w.positions)
    ids = oracle.slots_from_positions(w.page_table.cpu().numpy(), w.positions.cpu().numpy(), 64)
    bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    ref_out, ref_lse = oracle.decode(bits(w.q_nope), bits(w.q_pe), bits(w.ckv_cache.reshape(-1, 512)),
                                     bits(w.kpe_cache.reshape(-1, 64)), ids, w.sm_scale)
    np.testing.assert_allclose(out.float().cpu().numpy(), oracle.bf16_bits_to_f32(ref_out),
                               atol=1e-2, rtol=1e-2)
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse, atol=1e-3, rtol=0)


@pytest.mark.gpu
def test_page_size_one_pool():
    """The same memory as a [slots, 1, D] pool with a per-slot page table."""
    from flashinfer_mlsys2026_dsa_b200 import kernel, kernel_paged

    w = workloads.make("b64_h16", device="cuda", seed=6, batch=8)
    flat = _run(kernel, w, w.sparse_indices)
    pt = w.page_table.long()
    j = torch.arange(pt.shape[1] * 64, device="cuda")
    pt1 = torch.where(pt[:, j // 64] >= 0, pt[:, j // 64] * 64 + j % 64, -1).to(torch.int32)
    w1 = workloads.Workload(w.name, w.q_nope, w.q_pe, w.ckv_cache.reshape(-1, 1, 512),
                            w.kpe_cache.reshape(-1, 1, 64), w.sparse_indices, w.sm_scale)
    paged = _run(kernel_paged, w1, pt1.contiguous(), w.positions)
    _same(paged, flat)


@pytest.mark.gpu
def test_invalid_positions_are_flagged_and_treated_as_padding():
    from flashinfer_mlsys2026_dsa_b200 import _native, kernel, kernel_paged, read_device_errors

    w = workloads.make("b64_h16", device="cuda", seed=8, batch=16)
    pos = w.positions.clone()
    pt = w.page_table.clone()
    pos[0, 5] = -7                          # negative, not the padding value
    pos[1, 100] = pt.shape[1] * 64 + 3      # past the row's table
    pt[2, :] = -1                           # every page of row 2 unmapped
    want = torch.from_numpy(oracle.slots_from_positions(pt.cpu().numpy(), pos.cpu().numpy(), 64))
    flat_ids = torch.where(want < 0, -1, want).to(torch.int32).cuda()
    read_device_errors(clear=True)
    flat = _run(kernel, w, flat_ids)
    assert read_device_errors() == 0
    paged = _run(kernel_paged, w, pt, pos.contiguous())
    assert read_device_errors() & _native.DEVERR_BAD_INDEX
    _same(paged, flat)
    assert (paged[0][2] == 0).all() and torch.isneginf(paged[1][2]).all()


@pytest.mark.gpu
def test_paged_argument_errors():
    from flashinfer_mlsys2026_dsa_b200 import kernel_paged

    w = workloads.make("tiny", device="cuda", seed=1)
    with pytest.raises(TypeError):
        _run(kernel_paged, w, w.page_table.long(), w.positions)
    with pytest.raises(ValueError):
        _run(kernel_paged, w, w.page_table[:1], w.positions)
    with pytest.raises(ValueError):
        _run(kernel_paged, w, w.page_table, w.positions, page_size=48)
