"""A split-K merge that gives up waiting is visible: timeout bit, NaN rows, strict-mode error.

The kernel's waits are bounded (dsa_set_wait_limit); here the bound is shortened to about
a millisecond and the workspace's split-K arrival counters are pre-set so that the other
parts' arrivals can never add up to the count a merge waits for.  Every split row's merge
then runs out of time: the row must come back as NaN (output and lse) with the timeout
bit set, the rows no merge touched must be unaffected, and the context must stay usable.
No GPU fault or hang is involved: the wait returns by itself.
"""
import numpy as np
import pytest
import torch

from flashinfer_mlsys2026_dsa_b200 import (DSAError, _native, kernel, ops, read_device_errors,
                                           set_strict, workloads)

pytestmark = pytest.mark.gpu

COUNTERS = slice(256, 8448)  # split-K arrival counters in the workspace (dsa_decode.cu layout)
TILE_SLOTS = 112             # slots per tile of a 16-head work unit


def split_rows(rows, tiles_per_row, pairs):
    """Rows cut between cluster pairs by the stream-K split (equal tile shares per pair)."""
    units = rows * tiles_per_row
    cut = set()
    for c in range(1, pairs):
        u = c * units // pairs
        if u % tiles_per_row:
            cut.add(u // tiles_per_row)
    return cut


def _run(w):
    B, H = w.num_tokens, w.num_heads
    out = torch.empty(B, H, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, H, dtype=torch.float32, device="cuda")
    kernel(*w.args(), out, lse)
    torch.cuda.synchronize()
    return out, lse


def test_merge_that_runs_out_of_time_writes_nan_and_sets_the_bit():
    pairs = torch.cuda.get_device_properties(0).multi_processor_count // 2
    rows = pairs + 54  # more rows than pairs: stream-K, rows cut between pairs
    w = workloads.make("b64_h16", device="cuda", seed=21, batch=rows)
    ref_out, ref_lse = _run(w)
    assert read_device_errors() == 0
    stream = torch.cuda.current_stream()
    ws = ops.workspace_for(w.q_nope.device, stream.cuda_stream, rows, 16, w.topk)
    lib = _native.load()
    prev = lib.dsa_set_wait_limit(2_000_000)  # about 1 ms at 2 GHz
    try:
        ws[COUNTERS].view(torch.int32).fill_(1 << 30)
        out, lse = _run(w)
        word = read_device_errors(clear=True)
        # strict mode turns the same outcome into an exception
        ws[COUNTERS].view(torch.int32).fill_(1 << 30)
        was = set_strict(True)
        try:
            with pytest.raises(DSAError, match="ran out"):
                _run(w)
        finally:
            set_strict(was)
    finally:
        lib.dsa_set_wait_limit(prev)
        ws[COUNTERS].zero_()
        read_device_errors(clear=True)
    assert word & _native.DEVERR_TIMEOUT
    cut = split_rows(rows, -(-w.topk // TILE_SLOTS), pairs)
    assert cut, "the workload must split rows"
    nan_rows = set(torch.nonzero(torch.isnan(lse).any(dim=1)).flatten().tolist())
    assert nan_rows == cut
    for r in cut:
        assert torch.isnan(lse[r]).all() and torch.isnan(out[r].float()).all()
    keep = sorted(set(range(rows)) - cut)
    assert torch.equal(out[keep], ref_out[keep]) and torch.equal(lse[keep], ref_lse[keep])
    # the context is usable and the next call is whole again
    again_out, again_lse = _run(w)
    assert read_device_errors() == 0
    assert torch.equal(again_out, ref_out) and torch.equal(again_lse, ref_lse)
    np.testing.assert_array_equal(np.isnan(again_lse.cpu().numpy()), False)
