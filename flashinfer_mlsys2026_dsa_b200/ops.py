"""Python entry points of the DSA sparse-MLA decode (PyTorch tensors in, CUDA out).

``kernel`` mirrors the reference solution's destination-passing entry point
``kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output,
lse)`` (solution/triton/fused.py:150-180; same signature as
solution/triton/baseline.py:12): same argument names, order and meaning, the
outputs written in place, nothing returned.  ``decode`` is the value-returning
form (``destination_passing_style: false`` in the reference README).

Both call the native library through its C ABI (include/dsa_b200.h) on the
current CUDA stream.  There is no CPU path: CPU tensors raise.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import _native

D_CKV = 512
D_KPE = 64
PAGE_SIZE = 64
SUPPORTED_HEADS = (16, 32, 64, 128)

_ws_lock = threading.Lock()
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


class DSAError(RuntimeError):
    """A non-zero status from the native library, or (strict mode) device error bits."""


# Strict mode: every call synchronises its stream and raises DSAError when the kernel set
# a device error bit (an out-of-range index treated as padding, or a wait that ran out, in
# which case a split row was written as NaN).  Off by default, since the check costs a
# stream synchronisation per call; DSA_STRICT=1 in the environment turns it on.
_strict = os.environ.get("DSA_STRICT", "0") not in ("", "0")


def set_strict(enabled: bool) -> bool:
    """Turn strict mode on or off; returns the previous setting."""
    global _strict
    prev, _strict = _strict, bool(enabled)
    return prev


def _strict_check(device: torch.device, what: str) -> None:
    word = read_device_errors(device, clear=True)
    if word:
        bits = []
        if word & _native.DEVERR_BAD_INDEX:
            bits.append("an index outside [-1, num_slots) was treated as padding")
        if word & _native.DEVERR_TIMEOUT:
            bits.append("a wait in the kernel ran out (rows whose split-K merge gave up are NaN)")
        raise DSAError(f"{what}: device error word {word:#x}: " + "; ".join(bits))


def _check(code: int, what: str) -> None:
    if code != _native.DSA_OK:
        raise DSAError(f"{what}: {_native.status_text(code)} (status {code})")


def workspace_for(device: torch.device, stream_handle: int, num_tokens: int, num_heads: int,
                  topk: int) -> torch.Tensor:
    """The cached, zero-initialised workspace of (device, stream), grown on demand."""
    key = (device.index or 0, stream_handle)
    ws = _workspaces.get(key)
    if ws is not None:
        return ws  # its size depends only on the device
    lib = _native.load()
    need = int(lib.dsa_sparse_mla_decode_workspace_size(num_tokens, num_heads, topk,
                                                        device.index or 0))
    if need == 0:
        raise ValueError(f"unsupported problem: num_heads={num_heads}, topk={topk}")
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < need:
            ws = torch.zeros(max(need, 1 << 20), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
    return ws


_BF16 = torch.bfloat16
# native statuses about the arguments: the general route re-validates and raises the
# precise TypeError / ValueError (-1: the binding did not handle the argument form)
_REVALIDATE = (-1, 1, 2)


def _validate(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, output, lse,
              check_index_rows=True):
    tensors = (("q_nope", q_nope), ("q_pe", q_pe), ("ckv_cache", ckv_cache),
               ("kpe_cache", kpe_cache), ("sparse_indices", sparse_indices), ("output", output),
               ("lse", lse))
    for name, t in tensors:
        if not isinstance(t, torch.Tensor):
            raise TypeError(f"{name} must be a torch.Tensor")
        if not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor (this operator has no CPU path)")
    dev = q_nope.device
    for name, t in tensors[1:]:
        if t.device != dev:
            raise ValueError(f"{name} is on {t.device}, expected {dev}")
    for name, t in tensors[:4] + tensors[5:6]:
        if t.dtype != _BF16:
            raise TypeError(f"{name} must be bfloat16, got {t.dtype}")
    if sparse_indices.dtype != torch.int32:
        raise TypeError(f"sparse_indices must be int32, got {sparse_indices.dtype}")
    if lse.dtype != torch.float32:
        raise TypeError(f"lse must be float32, got {lse.dtype}")
    qs = q_nope.shape
    if len(qs) != 3 or qs[2] != D_CKV:
        raise ValueError(f"q_nope must be [num_tokens, num_heads, {D_CKV}], got {tuple(qs)}")
    B, H = qs[0], qs[1]
    if q_pe.shape != (B, H, D_KPE):
        raise ValueError(f"q_pe must be [{B}, {H}, {D_KPE}], got {tuple(q_pe.shape)}")
    if ckv_cache.shape[-1] != D_CKV or kpe_cache.shape[-1] != D_KPE:
        raise ValueError("ckv_cache / kpe_cache last dims must be 512 / 64")
    if sparse_indices.dim() != 2 or (check_index_rows and sparse_indices.shape[0] != B):
        raise ValueError(f"sparse_indices must be [{B}, topk], got {tuple(sparse_indices.shape)}")
    if output.shape != (B, H, D_CKV):
        raise ValueError(f"output must be [{B}, {H}, {D_CKV}], got {tuple(output.shape)}")
    if lse.shape != (B, H):
        raise ValueError(f"lse must be [{B}, {H}], got {tuple(lse.shape)}")
    if H not in SUPPORTED_HEADS:
        raise ValueError(f"num_heads={H} is not supported (supported: {SUPPORTED_HEADS})")


def _slot_view(cache: torch.Tensor, width: int, name: str) -> torch.Tensor:
    """[..., page, width] cache as a [num_slots, width] slot table, always a view.

    The pools are flattened the way fused.py:155-156 does (``reshape(-1, D)``), but a pool
    that is not a uniform slot table (inner stride not 1, or pages not evenly spaced)
    raises instead of being copied: a copy of a 1.5-20 GB pool per call would dwarf the
    decode.
    """
    if cache.stride(-1) != 1:
        raise ValueError(f"{name} must have a unit inner stride (got strides {cache.stride()})")
    try:
        return cache.view(-1, width)
    except RuntimeError:
        pass
    if cache.dim() == 3 and cache.stride(0) == cache.stride(1) * cache.shape[1]:
        return cache.as_strided((cache.shape[0] * cache.shape[1], width), (cache.stride(1), 1))
    raise ValueError(f"{name} is not a uniform slot table: pages of shape {tuple(cache.shape)} "
                     f"with strides {cache.stride()} cannot be addressed with one slot stride")


def kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output, lse) -> None:
    """DSA sparse-MLA decode, destination-passing (writes ``output`` and ``lse``).

    q_nope [B,H,512] bf16, q_pe [B,H,64] bf16, ckv_cache [P,64,512] bf16,
    kpe_cache [P,64,64] bf16, sparse_indices [B,topk] int32 flat slot ids
    (page*64 + offset; -1 = padding), sm_scale float, output [B,H,512] bf16,
    lse [B,H] fp32 (base-2 log-sum-exp).  Runs on the current CUDA stream
    and does not synchronise.
    """
    ext = _native._ext if _native._ext_tried else _native.ext()
    if ext is not None and type(q_nope) is torch.Tensor and q_nope.is_cuda:
        # Fast route: the binding reads the tensors in C++; -1 means "not the plain form",
        # and the general route below validates, raises or re-lays-out.
        dev_index = q_nope.get_device()
        stream = torch._C._cuda_getCurrentRawStream(dev_index)
        ws = _workspaces.get((dev_index, stream))
        if ws is not None and q_nope.shape[0] > 0:
            rc = ext.decode(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, float(sm_scale),
                            output, lse, ws, stream)
            if rc == _native.DSA_OK:
                if _strict:
                    _strict_check(q_nope.device, "dsa_sparse_mla_decode")
                return
            if rc not in _REVALIDATE:
                _check(rc, "dsa_sparse_mla_decode")
    _validate(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, output, lse)
    lib = _native._lib or _native.load()
    B, H, _ = q_nope.shape
    topk = sparse_indices.shape[1]
    if B == 0:
        return
    if q_nope.stride(-1) != 1:
        q_nope = q_nope.contiguous()
    if q_pe.stride(-1) != 1:
        q_pe = q_pe.contiguous()
    if sparse_indices.stride(-1) != 1:
        sparse_indices = sparse_indices.contiguous()
    ckv = _slot_view(ckv_cache, D_CKV, "ckv_cache")
    kpe = _slot_view(kpe_cache, D_KPE, "kpe_cache")
    if ckv.shape[0] != kpe.shape[0]:
        raise ValueError("ckv_cache and kpe_cache hold different slot counts")
    out_t = output if output.stride(-1) == 1 else torch.empty_like(output, memory_format=torch.contiguous_format)
    dev_index = q_nope.get_device()
    stream = torch._C._cuda_getCurrentRawStream(dev_index)
    ws = workspace_for(q_nope.device, stream, B, H, topk)
    rc = lib.dsa_sparse_mla_decode(
        q_nope.data_ptr(), q_nope.stride(0), q_nope.stride(1),
        q_pe.data_ptr(), q_pe.stride(0), q_pe.stride(1),
        ckv.data_ptr(), ckv.stride(0),
        kpe.data_ptr(), kpe.stride(0), ckv.shape[0],
        sparse_indices.data_ptr(), sparse_indices.stride(0),
        float(sm_scale),
        out_t.data_ptr(), out_t.stride(0), out_t.stride(1),
        lse.data_ptr(), lse.stride(0), lse.stride(1),
        B, H, topk, ws.data_ptr(), ws.numel(), stream)
    _check(rc, "dsa_sparse_mla_decode")
    if out_t is not output:
        output.copy_(out_t)
    if _strict:
        _strict_check(q_nope.device, "dsa_sparse_mla_decode")


def kernel_paged(q_nope, q_pe, ckv_cache, kpe_cache, page_table, positions, sm_scale, output,
                 lse, page_size=None) -> None:
    """:func:`kernel` with the slot ids formed in the kernel from a page table.

    ``positions`` [B, topk] int32 are token positions in each row's sequence (-1 =
    padding) and ``page_table`` [B, max_pages] int32 lists each row's pool pages; the
    kernel gathers slot ``page_table[b, pos // page_size] * page_size + pos % page_size``,
    the flat id the reference's callers build for ``sparse_indices`` (its pools are
    flattened as page * 64 + offset, fused.py:155-156).  ``page_size`` defaults to the
    pools' page dimension (``ckv_cache.shape[-2]`` of a [P, page_size, 512] pool).  A
    position past the row's table or on a negative page is treated as padding and
    flagged in :func:`read_device_errors`.
    """
    _validate(q_nope, q_pe, ckv_cache, kpe_cache, positions, output, lse)
    if not isinstance(page_table, torch.Tensor) or not page_table.is_cuda:
        raise ValueError("page_table must be a CUDA tensor")
    if page_table.device != q_nope.device:
        raise ValueError(f"page_table is on {page_table.device}, expected {q_nope.device}")
    if page_table.dtype != torch.int32:
        raise TypeError(f"page_table must be int32, got {page_table.dtype}")
    B, H, _ = q_nope.shape
    if page_table.dim() != 2 or page_table.shape[0] != B or page_table.shape[1] < 1:
        raise ValueError(f"page_table must be [{B}, max_pages], got {tuple(page_table.shape)}")
    if page_size is None:
        if ckv_cache.dim() != 3:
            raise ValueError("page_size is required for a pool that is not [pages, page_size, 512]")
        page_size = ckv_cache.shape[-2]
    page_size = int(page_size)
    if page_size < 1 or page_size & (page_size - 1):
        raise ValueError(f"page_size must be a power of two, got {page_size}")
    if B == 0:
        return
    lib = _native._lib or _native.load()
    topk = positions.shape[1]
    if q_nope.stride(-1) != 1:
        q_nope = q_nope.contiguous()
    if q_pe.stride(-1) != 1:
        q_pe = q_pe.contiguous()
    if positions.stride(-1) != 1:
        positions = positions.contiguous()
    if page_table.stride(-1) != 1:
        page_table = page_table.contiguous()
    ckv = _slot_view(ckv_cache, D_CKV, "ckv_cache")
    kpe = _slot_view(kpe_cache, D_KPE, "kpe_cache")
    if ckv.shape[0] != kpe.shape[0]:
        raise ValueError("ckv_cache and kpe_cache hold different slot counts")
    out_t = output if output.stride(-1) == 1 else torch.empty_like(output, memory_format=torch.contiguous_format)
    dev_index = q_nope.get_device()
    stream = torch._C._cuda_getCurrentRawStream(dev_index)
    ws = workspace_for(q_nope.device, stream, B, H, topk)
    rc = lib.dsa_sparse_mla_decode_paged(
        q_nope.data_ptr(), q_nope.stride(0), q_nope.stride(1),
        q_pe.data_ptr(), q_pe.stride(0), q_pe.stride(1),
        ckv.data_ptr(), ckv.stride(0),
        kpe.data_ptr(), kpe.stride(0), ckv.shape[0],
        page_table.data_ptr(), page_table.stride(0), page_table.shape[1], page_size,
        positions.data_ptr(), positions.stride(0),
        float(sm_scale),
        out_t.data_ptr(), out_t.stride(0), out_t.stride(1),
        lse.data_ptr(), lse.stride(0), lse.stride(1),
        B, H, topk, ws.data_ptr(), ws.numel(), stream)
    _check(rc, "dsa_sparse_mla_decode_paged")
    if out_t is not output:
        output.copy_(out_t)
    if _strict:
        _strict_check(q_nope.device, "dsa_sparse_mla_decode_paged")


def topk_slots(scores, lengths, page_table, k, page_size=PAGE_SIZE, out=None):
    """Index production: the decode's ``sparse_indices`` from index scores.

    ``scores`` [rows, max_len] float32 CUDA tensor of the rows' token positions, ``lengths``
    [rows] int32 (row b chooses among positions ``[0, lengths[b])``), ``page_table``
    [rows, max_pages] int32 (the row's pool pages in order).  Returns (or writes into
    ``out``) [rows, k] int32 slot ids ``page_table[b, pos // page_size] * page_size +
    pos % page_size`` of each row's k highest-scoring positions, in ascending position
    order, -1 after a row's positions when it has fewer than k (the decode's padding);
    ties at the k-th score go to the smaller positions.  One launch on the current stream;
    the result feeds :func:`kernel` directly.  The reference forms these ids on the caller
    side (solution/triton/baseline.py:17-23); flashinfer names the step
    ``top_k_page_table_transform``.
    """
    tensors = (("scores", scores), ("lengths", lengths))
    if page_table is not None:
        tensors += (("page_table", page_table),)
    for name, t in tensors:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
    if scores.dtype != torch.float32:
        raise TypeError(f"scores must be float32, got {scores.dtype}")
    if lengths.dtype != torch.int32 or (page_table is not None and page_table.dtype != torch.int32):
        raise TypeError("lengths and page_table must be int32")
    if scores.dim() != 2 or (page_table is not None and page_table.dim() != 2):
        raise ValueError("scores and page_table must be 2-D")
    rows, max_len = scores.shape
    if lengths.shape != (rows,) or (page_table is not None and page_table.shape[0] != rows):
        raise ValueError("lengths must be [rows] and page_table [rows, max_pages]")
    k = int(k)
    page_size = int(page_size)
    if k < 1 or page_size < 1 or page_size & (page_size - 1):
        raise ValueError("k must be >= 1 and page_size a power of two")
    if scores.stride(-1) != 1:
        scores = scores.contiguous()
    if page_table is not None and page_table.stride(-1) != 1:
        page_table = page_table.contiguous()
    lengths = lengths.contiguous()
    if out is None:
        out = torch.empty(rows, k, dtype=torch.int32, device=scores.device)
    elif out.shape != (rows, k) or out.dtype != torch.int32 or out.stride(-1) != 1:
        raise ValueError(f"out must be an int32 [{rows}, {k}] tensor with a unit inner stride")
    stream = torch._C._cuda_getCurrentRawStream(scores.get_device())
    lib = _native._lib or _native.load()
    pt_ptr, pt_sb, pt_cols = ((page_table.data_ptr(), page_table.stride(0), page_table.shape[1])
                              if page_table is not None else (None, 0, 0))
    _check(lib.dsa_topk_slots(scores.data_ptr(), scores.stride(0), lengths.data_ptr(),
                              pt_ptr, pt_sb, pt_cols, page_size, rows, max_len, k,
                              out.data_ptr(), out.stride(0), stream),
           "dsa_topk_slots")
    return out


def union_groups(positions, page_table, group, out_cols=None, page_size=PAGE_SIZE):
    """Union of the selections of token groups, for :func:`kernel_grouped`.

    ``positions`` [tokens, k] int32 CUDA tensor: each token's selected positions (distinct;
    -1 = none), e.g. :func:`topk_slots` with ``page_table=None``. Tokens ``[g * group,
    (g + 1) * group)`` form group g and share the sequence's ``page_table`` row g
    ([tokens // group, max_pages] int32). Returns ``(slots, member, counts)``: per group
    the union's slot ids in ascending position order then -1 ([groups, out_cols] int32),
    the membership bytes (bit j: token j of the group selected the entry; uint8, same
    shape) and the union sizes ([groups] int32). ``out_cols`` defaults to ``min(group * k,
    max_pages * page_size)``, which always holds the union; a smaller value cuts it
    (``counts`` shows by how much). One launch on the current stream.
    """
    for name, t in (("positions", positions), ("page_table", page_table)):
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError(f"{name} must be a CUDA tensor")
        if t.dtype != torch.int32:
            raise TypeError(f"{name} must be int32, got {t.dtype}")
        if t.dim() != 2:
            raise ValueError(f"{name} must be 2-D")
    group = int(group)
    tokens, k = positions.shape
    if group < 1 or group > 8 or tokens % group:
        raise ValueError(f"group must be in [1, 8] and divide the token count {tokens}")
    groups = tokens // group
    if page_table.shape[0] != groups:
        raise ValueError(f"page_table must be [{groups}, max_pages], got {tuple(page_table.shape)}")
    page_size = int(page_size)
    if page_size < 1 or page_size & (page_size - 1):
        raise ValueError(f"page_size must be a power of two, got {page_size}")
    if out_cols is None:
        out_cols = min(group * k, page_table.shape[1] * page_size)
    out_cols = int(out_cols)
    if out_cols < 1:
        raise ValueError("out_cols must be >= 1")
    positions = positions.contiguous()
    page_table = page_table.contiguous()
    dev = positions.device
    slots = torch.empty(groups, out_cols, dtype=torch.int32, device=dev)
    member = torch.empty(groups, out_cols, dtype=torch.uint8, device=dev)
    counts = torch.empty(groups, dtype=torch.int32, device=dev)
    if groups == 0:
        return slots, member, counts
    stream = torch._C._cuda_getCurrentRawStream(positions.get_device())
    lib = _native._lib or _native.load()
    _check(lib.dsa_union_groups(positions.data_ptr(), positions.stride(0), tokens, k, group,
                                page_table.data_ptr(), page_table.stride(0), page_table.shape[1],
                                page_size, slots.data_ptr(), member.data_ptr(), slots.stride(0),
                                out_cols, counts.data_ptr(), stream),
           "dsa_union_groups")
    return slots, member, counts


def kernel_grouped(q_nope, q_pe, ckv_cache, kpe_cache, union_indices, member, sm_scale,
                   output, lse):
    """Multi-token rows decoded in token groups (prefill chunks, multi-token decode).

    The same result as :func:`kernel` on each token's own selection, computed for groups of
    ``G = 128 // num_heads`` consecutive tokens of one sequence at once: ``union_indices``
    and ``member`` [tokens // G, U] (from :func:`union_groups`) hold the union of the
    group's selections and which token selected each entry, so every union slot is
    gathered once for the whole group and decoded as one 128-head row. The tokens' heads
    must be consecutive in ``q_nope``, ``q_pe``, ``output`` and ``lse`` (contiguous
    [tokens, H, ...] tensors). Pays when the group's selections overlap: the union of G
    tokens costs about as much as G / 3 separate tokens' selections per slot.
    """
    _validate(q_nope, q_pe, ckv_cache, kpe_cache, union_indices, output, lse,
              check_index_rows=False)
    B, H, _ = q_nope.shape
    if H not in (16, 32, 64):
        raise ValueError(f"grouped decode takes 16, 32 or 64 heads per token, got {H}")
    G = 128 // H
    if B % G:
        raise ValueError(f"the token count {B} is not a multiple of the group size {G}")
    if not isinstance(member, torch.Tensor) or member.dtype != torch.uint8 or \
            member.shape != union_indices.shape or member.device != union_indices.device:
        raise ValueError("member must be a uint8 tensor shaped like union_indices, on its device")
    if union_indices.shape[0] != B // G:
        raise ValueError(f"union_indices must be [{B // G}, U], got {tuple(union_indices.shape)}")
    if B == 0:
        return
    union_indices = union_indices.contiguous()
    member = member.contiguous()
    for name, t in (("q_nope", q_nope), ("q_pe", q_pe), ("output", output), ("lse", lse)):
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous for the grouped decode")
    ckv = _slot_view(ckv_cache, D_CKV, "ckv_cache")
    kpe = _slot_view(kpe_cache, D_KPE, "kpe_cache")
    if ckv.shape[0] != kpe.shape[0]:
        raise ValueError("ckv_cache and kpe_cache hold different slot counts")
    lib = _native._lib or _native.load()
    stream = torch._C._cuda_getCurrentRawStream(q_nope.get_device())
    U = union_indices.shape[1]
    ws = workspace_for(q_nope.device, stream, B // G, 128, U)
    rc = lib.dsa_sparse_mla_decode_grouped(
        q_nope.data_ptr(), q_nope.stride(0), q_nope.stride(1),
        q_pe.data_ptr(), q_pe.stride(0), q_pe.stride(1),
        ckv.data_ptr(), ckv.stride(0), kpe.data_ptr(), kpe.stride(0), ckv.shape[0],
        union_indices.data_ptr(), member.data_ptr(), union_indices.stride(0), U,
        float(sm_scale), output.data_ptr(), output.stride(0), output.stride(1),
        lse.data_ptr(), lse.stride(0), lse.stride(1), B, H,
        ws.data_ptr(), ws.numel(), stream)
    _check(rc, "dsa_sparse_mla_decode_grouped")
    if _strict:
        _strict_check(q_nope.device, "dsa_sparse_mla_decode_grouped")


def decode(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale):
    """Value-returning form of :func:`kernel`: returns (output, lse)."""
    B, H, _ = q_nope.shape
    output = torch.empty(B, H, D_CKV, dtype=torch.bfloat16, device=q_nope.device)
    lse = torch.empty(B, H, dtype=torch.float32, device=q_nope.device)
    kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output, lse)
    return output, lse


def read_device_errors(device=None, clear: bool = True) -> int:
    """Sticky device error bits (bad index, timeout) of the current stream's workspace."""
    device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    stream = torch.cuda.current_stream(device)
    ws = _workspaces.get((device.index or 0, stream.cuda_stream))
    if ws is None:
        return 0
    word = ctypes.c_uint32(0)
    _check(_native.load().dsa_read_error_word(ws.data_ptr(), stream.cuda_stream, int(clear),
                                              ctypes.byref(word)), "dsa_read_error_word")
    return int(word.value)
