"""dsa_sparse_mla_decode_noalloc: the decode with the library's built-in scratch array.

Callers that cannot allocate device memory while they decode (a plugin inside a host
application that forbids cudaMalloc on its decode path, code running under another
framework's allocator) use this entry point: it takes no workspace and allocates nothing.
It must give exactly what dsa_sparse_mla_decode gives with a caller workspace (same
kernel, same work split), call after call, although every call reuses the array the
previous one left behind.  This file is collected last so that it also runs after the
rest of the GPU suite has used the device.
"""
import numpy as np
import pytest
import torch

from flashinfer_mlsys2026_dsa_b200 import _native, ops, workloads

pytestmark = pytest.mark.gpu


def _args(w, out, lse):
    B, H, _ = w.q_nope.shape
    return (w.q_nope.data_ptr(), w.q_nope.stride(0), w.q_nope.stride(1),
            w.q_pe.data_ptr(), w.q_pe.stride(0), w.q_pe.stride(1),
            w.ckv_cache.data_ptr(), w.ckv_cache.stride(-2),
            w.kpe_cache.data_ptr(), w.kpe_cache.stride(-2),
            w.ckv_cache.numel() // 512,
            w.sparse_indices.data_ptr(), w.sparse_indices.stride(0), w.sm_scale,
            out.data_ptr(), out.stride(0), out.stride(1),
            lse.data_ptr(), lse.stride(0), lse.stride(1),
            B, H, w.sparse_indices.shape[1])


def _outputs(w):
    B, H, _ = w.q_nope.shape
    out = torch.full((B, H, 512), float("nan"), dtype=torch.bfloat16, device="cuda")
    lse = torch.full((B, H), float("nan"), dtype=torch.float32, device="cuda")
    return out, lse


def _with_workspace(lib, w, stream):
    out, lse = _outputs(w)
    B, H, _ = w.q_nope.shape
    ws = ops.workspace_for(w.q_nope.device, stream.cuda_stream, B, H, w.sparse_indices.shape[1])
    rc = lib.dsa_sparse_mla_decode(*_args(w, out, lse), ws.data_ptr(), ws.numel(),
                                   stream.cuda_stream)
    assert rc == 0, _native.status_text(rc)
    return out, lse


def _no_alloc(lib, w, stream):
    out, lse = _outputs(w)
    rc = lib.dsa_sparse_mla_decode_noalloc(*_args(w, out, lse), stream.cuda_stream)
    assert rc == 0, _native.status_text(rc)
    return out, lse


def test_no_alloc_matches_workspace_entry_on_consecutive_calls():
    lib = _native.load()
    stream = torch.cuda.current_stream()
    # Two different problems back to back, both with fewer (row, head group) units than
    # the persistent grid has cluster pairs, so neither splits a row (the only calls the
    # array serves on a 148-SM B200): a full-size H=16 batch, then a smaller ragged batch
    # with -1 padding that finds the first call's error word and counters in the array.
    first = workloads.make("b64_h16", device="cuda", seed=11)
    second = workloads.make("ragged_b256", device="cuda", seed=12, batch=40)
    got = [_no_alloc(lib, first, stream), _no_alloc(lib, second, stream)]
    want = [_with_workspace(lib, first, stream), _with_workspace(lib, second, stream)]
    torch.cuda.synchronize()
    for (o, l), (wo, wl) in zip(got, want):
        assert torch.isfinite(o.float()).all()
        assert torch.equal(o, wo)
        assert torch.equal(l, wl)
    # The same problem again gives the same bits (nothing carried over between calls).
    again = _no_alloc(lib, first, stream)
    torch.cuda.synchronize()
    assert torch.equal(again[0], got[0][0]) and torch.equal(again[1], got[0][1])


def test_no_alloc_limit_is_the_persistent_grid():
    """Calls up to one 16-head row per cluster pair fit; one more row needs split-K partials."""
    lib = _native.load()
    stream = torch.cuda.current_stream()
    pairs = torch.cuda.get_device_properties(0).multi_processor_count // 2
    w = workloads.make("b64_h16", device="cuda", seed=5, batch=pairs + 1)
    fit = workloads.Workload("fit", w.q_nope[:pairs].contiguous(), w.q_pe[:pairs].contiguous(),
                             w.ckv_cache, w.kpe_cache, w.sparse_indices[:pairs].contiguous(),
                             w.sm_scale)
    got = _no_alloc(lib, fit, stream)
    want = _with_workspace(lib, fit, stream)
    torch.cuda.synchronize()
    assert torch.equal(got[0], want[0]) and torch.equal(got[1], want[1])
    out, lse = _outputs(w)
    rc = lib.dsa_sparse_mla_decode_noalloc(*_args(w, out, lse), stream.cuda_stream)
    assert rc == _native.ERR_SCRATCH_LIMIT, _native.status_text(rc)
    torch.cuda.synchronize()
    assert torch.isnan(lse).all()  # nothing was launched


def test_no_alloc_rejects_problems_beyond_its_scratch():
    lib = _native.load()
    stream = torch.cuda.current_stream()
    w = workloads.make("b32_h128", device="cuda", seed=3)
    out, lse = _outputs(w)
    rc = lib.dsa_sparse_mla_decode_noalloc(*_args(w, out, lse), stream.cuda_stream)
    assert rc == _native.ERR_SCRATCH_LIMIT
    assert "scratch" in _native.status_text(rc)
    torch.cuda.synchronize()
    assert torch.isnan(lse).all()  # nothing was launched
    np.testing.assert_equal(rc, 7)
