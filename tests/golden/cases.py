"""Seeded small input cases for the golden fixtures and the parity tests.

Every case is rebuilt from its spec with numpy's PCG64 generator, so the
fixtures only store the outputs the reference produced plus a SHA-256 of the
inputs (a changed generator is caught instead of silently compared).

bf16 tensors are held as uint16 bit patterns (round-to-nearest-even from the
float32 draws).  Shapes follow the operator definition
dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64 (reference config.toml:3):
q_nope [B,H,512], q_pe [B,H,64], ckv_cache [P,64,512], kpe_cache [P,64,64],
sparse_indices [B,topk] int32 flat slot ids (page*64 + offset), -1 = padding.
"""
from __future__ import annotations

import hashlib
import math

import numpy as np

PAGE = 64
D_CKV = 512
D_KPE = 64


def _bf16(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _normal(rng, shape, scale=1.0):
    return _bf16(rng.standard_normal(size=shape, dtype=np.float32) * np.float32(scale))


def _paged_indices(rng, seq_lens, topk, num_pages, pad_short=True, mode="uniform"):
    """Shuffled global page pool; topk distinct positions per row -> flat slots."""
    perm = rng.permutation(num_pages)
    idx = np.full((len(seq_lens), topk), -1, dtype=np.int32)
    off = 0
    for r, L in enumerate(seq_lens):
        npg = -(-L // PAGE)
        table = perm[off:off + npg]
        off += npg
        if L <= topk and pad_short:
            pos = rng.permutation(L)
        elif mode == "recent_half":
            recent = min(4096, L // 2)
            a = rng.choice(recent, size=topk // 2, replace=False) + (L - recent)
            b = rng.choice(L - recent, size=topk - topk // 2, replace=False)
            pos = np.concatenate([a, b])
        else:
            pos = rng.choice(L, size=topk, replace=False)
        slots = table[pos // PAGE] * PAGE + pos % PAGE
        idx[r, :len(slots)] = slots.astype(np.int32)
    assert off <= num_pages
    return idx


CASES = {
    # the CPU-runnable tiny decode (B=2, H=16, topk=256, 32-page pool)
    "tiny_b2_h16_k256": dict(B=2, H=16, topk=256, pages=32, seq=[1024, 1000], kv_scale=1.0),
    "h16_k2048": dict(B=2, H=16, topk=2048, pages=80, seq=[2500, 2100], kv_scale=0.5),
    "h128_k256": dict(B=2, H=128, topk=256, pages=24, seq=[700, 600], kv_scale=0.5),
    "h64_k128": dict(B=2, H=64, topk=128, pages=10, seq=[300, 200], kv_scale=0.5),
    "h32_k192": dict(B=3, H=32, topk=192, pages=16, seq=[300, 200, 400], kv_scale=0.5),
    "ragged_pad": dict(B=4, H=16, topk=512, pages=40, seq=[1500, 100, 512, 7], kv_scale=0.5),
    "topk100": dict(B=3, H=16, topk=100, pages=12, seq=[300, 80, 250], kv_scale=0.5),
    "mid_pad": dict(B=2, H=16, topk=256, pages=16, seq=[500, 400], kv_scale=0.5,
                    extra="mid_pad"),
    "duplicates": dict(B=2, H=16, topk=256, pages=16, seq=[500, 400], kv_scale=0.5,
                       extra="duplicates"),
    "recent_half_h128": dict(B=1, H=128, topk=512, pages=40, seq=[2560], kv_scale=0.5,
                             mode="recent_half"),
    "many_rows": dict(B=40, H=16, topk=128, pages=160, seq=[256] * 40, kv_scale=0.5),
    # Reference corner cases: an all-padding row (NaN output, lse=-inf in the
    # reference) and an index < -1 (the reference clamps it to slot 0).
    "all_pad_row": dict(B=2, H=16, topk=128, pages=8, seq=[200, 0], kv_scale=0.5),
    "neg_index": dict(B=1, H=16, topk=128, pages=8, seq=[300], kv_scale=0.5, extra="neg"),
}

# Cases whose reference result the CUDA path deliberately does not reproduce
# (it writes zeros / flags the index instead); the oracle is still pinned on them.
REFERENCE_ONLY = {"all_pad_row", "neg_index"}


def make_case(name: str, seed: int = 1234):
    spec = CASES[name]
    rng = np.random.Generator(np.random.PCG64(seed + sum(map(ord, name))))
    B, H, topk, P = spec["B"], spec["H"], spec["topk"], spec["pages"]
    q_nope = _normal(rng, (B, H, D_CKV))
    q_pe = _normal(rng, (B, H, D_KPE))
    ckv = _normal(rng, (P, PAGE, D_CKV), spec["kv_scale"])
    kpe = _normal(rng, (P, PAGE, D_KPE), spec["kv_scale"])
    idx = _paged_indices(rng, spec["seq"], topk, P, mode=spec.get("mode", "uniform"))
    extra = spec.get("extra")
    if extra == "mid_pad":
        idx[0, 10:40] = -1
        idx[0, 200:256] = -1
        idx[1, ::3] = -1
    elif extra == "duplicates":
        idx[0, 100:200] = idx[0, 0]
        idx[1, 1::2] = idx[1, 0::2]
    elif extra == "neg":
        idx[0, 5] = -7
        idx[0, 9] = -2
    sm_scale = 1.0 / math.sqrt(192.0)
    return dict(q_nope=q_nope, q_pe=q_pe, ckv_cache=ckv, kpe_cache=kpe,
                sparse_indices=idx, sm_scale=sm_scale)


def input_digest(case: dict) -> str:
    h = hashlib.sha256()
    for k in ("q_nope", "q_pe", "ckv_cache", "kpe_cache", "sparse_indices"):
        h.update(np.ascontiguousarray(case[k]).tobytes())
    h.update(np.float64(case["sm_scale"]).tobytes())
    return h.hexdigest()
