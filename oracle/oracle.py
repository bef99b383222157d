"""CPU oracle for the DSA sparse-MLA decode operator (test infrastructure).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module.  It checks the product and is never part of it:
the product path (``flashinfer_mlsys2026_dsa_b200``) has no CPU fallback and
never imports it.

``decode`` runs the C restatement in ``dsa_oracle.c`` of the reference PyTorch
path ``kernel`` in solution/triton/baseline.py:12-45 (see the C file for the
line-by-line mapping).  ``decode_numpy`` is a second, independent restatement
in numpy used to cross-check the C file on small cases.

Inputs are numpy arrays: bf16 tensors are passed as ``uint16`` bit patterns.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_BUILD_DIR = os.path.join(_HERE, "_build")
_LIB_PATH = os.path.join(_BUILD_DIR, "libdsa_oracle.so")
_SRC = os.path.join(_HERE, "dsa_oracle.c")
_lock = threading.Lock()
_lib = None

D_CKV = 512
D_KPE = 64


def build(force: bool = False) -> str:
    """Compile ``dsa_oracle.c`` into ``oracle/_build/libdsa_oracle.so``."""
    if (not force and os.path.exists(_LIB_PATH)
            and os.path.getmtime(_LIB_PATH) >= os.path.getmtime(_SRC)):
        return _LIB_PATH
    os.makedirs(_BUILD_DIR, exist_ok=True)
    tmp = _LIB_PATH + f".tmp{os.getpid()}"
    cmd = ["gcc", "-O3", "-mavx2", "-mfma", "-fopenmp", "-shared", "-fPIC",
           "-o", tmp, _SRC, "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(tmp, _LIB_PATH)
    return _LIB_PATH


def _load():
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(_LIB_PATH):
                build()
            lib = ctypes.CDLL(_LIB_PATH)
            lib.dsa_oracle_decode.restype = ctypes.c_int
            lib.dsa_oracle_decode.argtypes = [
                ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32,
                ctypes.c_int32, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p,
                ctypes.c_int32]
            lib.dsa_oracle_max_threads.restype = ctypes.c_int
            lib.dsa_oracle_topk_slots.restype = ctypes.c_int
            lib.dsa_oracle_topk_slots.argtypes = [
                ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                ctypes.c_int32, ctypes.c_int32, ctypes.c_int64, ctypes.c_int32, ctypes.c_int32,
                ctypes.c_void_p, ctypes.c_int64]
            _lib = lib
    return _lib


def max_threads() -> int:
    return int(_load().dsa_oracle_max_threads())


def decode(q_nope, q_pe, ckv, kpe, sparse_indices, sm_scale, nthreads: int | None = None):
    """Run the C oracle.

    Shapes: q_nope [B,H,512] u16, q_pe [B,H,64] u16, ckv [..., 512] u16 (any
    leading dims, flattened to slots), kpe [..., 64] u16, sparse_indices
    [B,topk] int32.  Returns (out [B,H,512] uint16 bf16 bits, lse [B,H] f32).
    Raises IndexError where the reference's gather would raise.
    """
    lib = _load()
    q_nope = np.ascontiguousarray(q_nope, dtype=np.uint16)
    q_pe = np.ascontiguousarray(q_pe, dtype=np.uint16)
    ckv = np.ascontiguousarray(ckv, dtype=np.uint16).reshape(-1, D_CKV)
    kpe = np.ascontiguousarray(kpe, dtype=np.uint16).reshape(-1, D_KPE)
    idx = np.ascontiguousarray(sparse_indices, dtype=np.int32)
    B, H, _ = q_nope.shape
    topk = idx.shape[-1]
    assert ckv.shape[0] == kpe.shape[0]
    out = np.empty((B, H, D_CKV), dtype=np.uint16)
    lse = np.empty((B, H), dtype=np.float32)
    if nthreads is None:
        nthreads = os.cpu_count() or 1
    rc = lib.dsa_oracle_decode(
        q_nope.ctypes.data, q_pe.ctypes.data, ckv.ctypes.data, kpe.ctypes.data,
        ckv.shape[0], idx.ctypes.data, B, H, topk, float(sm_scale),
        out.ctypes.data, lse.ctypes.data, int(nthreads))
    if rc != 0:
        raise IndexError("sparse_indices holds a slot id >= num_slots")
    return out, lse


def bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (NaN -> 0x7FC0)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(a, dtype=np.float32))
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FC0
    return r


def decode_numpy(q_nope, q_pe, ckv, kpe, sparse_indices, sm_scale):
    """Independent numpy restatement of baseline.py:12-45 (small cases only)."""
    qn = bf16_bits_to_f32(q_nope)
    qp = bf16_bits_to_f32(q_pe)
    kc_all = bf16_bits_to_f32(np.asarray(ckv).reshape(-1, D_CKV))
    kp_all = bf16_bits_to_f32(np.asarray(kpe).reshape(-1, D_KPE))
    idx = np.asarray(sparse_indices, dtype=np.int64)
    valid = idx != -1                                   # baseline.py:22
    safe = np.clip(idx, 0, None)                        # baseline.py:23
    if safe.size and safe.max() >= kc_all.shape[0]:
        raise IndexError("sparse_indices holds a slot id >= num_slots")
    kc = kc_all[safe]                                   # baseline.py:27  [B,topk,512]
    kp = kp_all[safe]                                   # baseline.py:28  [B,topk,64]
    logits = (np.einsum("bhd,bkd->bhk", qn, kc, dtype=np.float32)
              + np.einsum("bhd,bkd->bhk", qp, kp, dtype=np.float32))   # baseline.py:34
    z = (logits * np.float32(sm_scale)).astype(np.float32)              # baseline.py:35
    z = np.where(valid[:, None, :], z, np.float32(-np.inf))             # baseline.py:38
    m = z.max(axis=-1, keepdims=True)
    with np.errstate(invalid="ignore", divide="ignore"):
        e = np.exp(z.astype(np.float64) - m)
        s = e.sum(axis=-1, keepdims=True)
        lse = ((m[..., 0] + np.log(s[..., 0])) / np.log(2.0)).astype(np.float32)  # :41
        lse = np.where(np.isneginf(m[..., 0]), np.float32(-np.inf), lse)
        attn = (e / s).astype(np.float32)                               # baseline.py:44
    out = np.einsum("bhk,bkd->bhd", attn, kc, dtype=np.float32)         # baseline.py:45
    return f32_to_bf16_bits(out), lse


def slots_from_positions(page_table: np.ndarray, positions: np.ndarray, page_size: int):
    """Index production: token positions + page table -> flat slot ids.

    slot = page_table[b, pos // page_size] * page_size + pos % page_size, the flat slot
    of a [pages, page_size, D] pool flattened to rows (baseline.py:17-23 and
    fused.py:155-156 flatten the pools; the reference's callers pass such ids as
    ``sparse_indices``).  -1 stays padding; a position < -1, past the row's table, or
    on a negative page gives -2 (an invalid id: padding plus a bad-index flag in the
    CUDA path).  Pure numpy, any size.
    """
    pt = np.asarray(page_table, dtype=np.int64)
    pos = np.asarray(positions, dtype=np.int64)
    cols = pt.shape[1]
    page_idx = np.where(pos >= 0, pos // page_size, 0)
    in_table = (pos >= 0) & (page_idx < cols)
    page = np.take_along_axis(pt, np.where(in_table, page_idx, 0), axis=1)
    slot = page * page_size + np.where(pos >= 0, pos % page_size, 0)
    ok = in_table & (page >= 0) & (slot <= np.iinfo(np.int32).max)
    out = np.where(ok, slot, np.where(pos == -1, -1, -2))
    return out.astype(np.int32)


def compact_pool(ckv_rows_fn, kpe_rows_fn, sparse_indices: np.ndarray):
    """Gather only the referenced slots so the oracle runs on a small pool.

    ``ckv_rows_fn(slots)`` / ``kpe_rows_fn(slots)`` return the uint16 rows of
    the given (sorted, unique, int64) slot ids.  Returns (ckv_small,
    kpe_small, remapped_indices).  Rows are independent, so the math is the
    same as on the full pool.  ``-1`` stays ``-1``; other negatives map to
    slot 0 of the full pool, as the reference's clamp does.
    """
    idx = np.asarray(sparse_indices, dtype=np.int64)
    safe = np.where(idx == -1, -1, np.clip(idx, 0, None))
    slots = np.unique(safe[safe >= 0])
    if slots.size == 0:
        slots = np.zeros(1, dtype=np.int64)
    remap = np.searchsorted(slots, np.clip(safe, 0, None)).astype(np.int32)
    remap = np.where(safe == -1, -1, remap).astype(np.int32)
    return ckv_rows_fn(slots), kpe_rows_fn(slots), remap


def topk_slots(scores, lengths, page_table, k: int, page_size: int):
    """Index production in C: per-row top-k of ``scores`` [rows, max_len] (float32) over
    the first ``lengths[row]`` entries, ties to the smaller position, selected positions in
    ascending order translated through ``page_table`` [rows, cols] (int32), -1 up to k.
    See ``dsa_oracle_topk_slots`` in dsa_oracle.c for the order of scores."""
    lib = _load()
    sc = np.ascontiguousarray(scores, dtype=np.float32)
    ln = np.ascontiguousarray(lengths, dtype=np.int32)
    pt = np.ascontiguousarray(page_table, dtype=np.int32)
    rows, max_len = sc.shape
    out = np.empty((rows, k), dtype=np.int32)
    rc = lib.dsa_oracle_topk_slots(sc.ctypes.data, max_len, ln.ctypes.data, pt.ctypes.data,
                                   pt.shape[1], pt.shape[1], int(page_size), rows, max_len,
                                   int(k), out.ctypes.data, k)
    if rc != 0:
        raise MemoryError("oracle top-k: allocation failed")
    return out


def score_keys(scores) -> np.ndarray:
    """Order-preserving uint32 keys of float32 scores (NaN lowest, -0.0 below +0.0)."""
    u = np.ascontiguousarray(scores, dtype=np.float32).view(np.uint32)
    nan = ((u & 0x7F800000) == 0x7F800000) & ((u & 0x007FFFFF) != 0)
    key = np.where(u & 0x80000000, ~u, u | 0x80000000).astype(np.uint32)
    return np.where(nan, np.uint32(0), key)


def topk_slots_numpy(scores, lengths, page_table, k: int, page_size: int):
    """Independent numpy restatement of :func:`topk_slots` (stable sort per row)."""
    sc = np.asarray(scores, dtype=np.float32)
    rows, max_len = sc.shape
    out = np.full((rows, k), -1, dtype=np.int32)
    for r in range(rows):
        L = int(min(max(int(lengths[r]), 0), max_len))
        if L <= k:
            pos = np.arange(L)
        else:
            keys = score_keys(sc[r, :L]).astype(np.int64)
            order = np.argsort(-keys, kind="stable")      # larger key first, ties by position
            pos = np.sort(order[:k])
        out[r, :len(pos)] = slots_from_positions(page_table[r:r + 1], pos[None, :].astype(np.int64),
                                                 page_size)[0].clip(min=-1)
    return out


def union_groups_numpy(positions, page_table, group: int, page_size: int, out_cols: int):
    """Union of the selections of token groups (the input of the grouped decode).

    ``positions`` [tokens, k] (each token's selected positions, -1 = none); tokens
    ``[g * group, (g + 1) * group)`` form group g with ``page_table`` row g. Per group: the
    positions any token selected (0 <= pos < cols * page_size), ascending, as slot ids
    through the group's table (-1 where the table has no page), with a membership byte
    (bit j: token j of the group selected the position; 0 for a -1 slot); -1 / 0 after the
    union up to ``out_cols``; and the union sizes. The grouped decode of token t equals
    the decode of t's own selection (baseline.py:17-45), so the decode oracle for a group
    is :func:`decode` per token. Pure numpy.
    """
    pos = np.asarray(positions, dtype=np.int64)
    pt = np.asarray(page_table, dtype=np.int64)
    tokens, _ = pos.shape
    groups = tokens // group
    max_pos = pt.shape[1] * page_size
    slots = np.full((groups, out_cols), -1, dtype=np.int32)
    member = np.zeros((groups, out_cols), dtype=np.uint8)
    counts = np.zeros(groups, dtype=np.int32)
    for g in range(groups):
        bits = {}
        for j in range(group):
            for q in pos[g * group + j]:
                if 0 <= q < max_pos:
                    bits[int(q)] = bits.get(int(q), 0) | (1 << j)
        u = np.array(sorted(bits), dtype=np.int64)
        counts[g] = len(u)
        u = u[:out_cols]
        if len(u):
            s = slots_from_positions(pt[g:g + 1], u[None, :], page_size)[0]
            ok = s >= 0
            slots[g, :len(u)] = np.where(ok, s, -1)
            member[g, :len(u)] = np.where(ok, [bits[int(q)] for q in u], 0).astype(np.uint8)
    return slots, member, counts
