"""Seeded synthetic decode workloads with the shapes of the benchmark configs.

The reference is evaluated on the FlashInfer ``mlsys26-contest`` trace set
(reference README.md:25,53-66), which is not available here; these generators
stand in for it with the shapes, sizes and value distributions of the five
benchmark configurations:

  tiny        B=2,    H=16,  topk=256,  32-page pool, seq_len 1024 / 1000, N(0,1) values
  b64_h16     B=64,   H=16,  topk=2048, seq_len ~ U[4096, 32768], kv ~ 0.5 N(0,1)
  b32_h128    B=32,   H=128, topk=2048, seq_len 65536, half the positions from the
              last 4096 tokens and half from the rest
  ragged_b256 B=256,  H=16,  topk=2048, seq_len log-uniform in [128, 131072]; rows
              shorter than topk take every position and pad with -1
  b2048       global B=2048, H=16, topk=2048, seq_len ~ U[8192, 131072]; each rank
              of a world of size W builds its own B/W rows and its own page pool

Every row's pages come from a shuffled global pool sized to sum(ceil(seq_len/64));
``sparse_indices`` holds flat slot ids page*64 + offset of distinct positions.
Large pools are generated directly on the GPU.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

PAGE = 64
D_CKV = 512
D_KPE = 64

CONFIGS = {
    "tiny": dict(B=2, H=16, topk=256, kv_scale=1.0),
    "b64_h16": dict(B=64, H=16, topk=2048, kv_scale=0.5),
    "b32_h128": dict(B=32, H=128, topk=2048, kv_scale=0.5),
    "ragged_b256": dict(B=256, H=16, topk=2048, kv_scale=0.5),
    "b2048": dict(B=2048, H=16, topk=2048, kv_scale=0.5),
}


@dataclass
class Workload:
    name: str
    q_nope: torch.Tensor
    q_pe: torch.Tensor
    ckv_cache: torch.Tensor
    kpe_cache: torch.Tensor
    sparse_indices: torch.Tensor
    sm_scale: float
    seq_lens: list = field(default_factory=list)
    # the inputs the slot ids were built from: each row's pool pages (-1 past the row's
    # pages) and the selected token positions (-1 = padding)
    page_table: torch.Tensor | None = None
    positions: torch.Tensor | None = None

    @property
    def num_tokens(self) -> int:
        return self.q_nope.shape[0]

    @property
    def num_heads(self) -> int:
        return self.q_nope.shape[1]

    @property
    def topk(self) -> int:
        return self.sparse_indices.shape[1]

    def n_valid(self) -> int:
        return int((self.sparse_indices != -1).sum().item())

    def algorithmic_bytes(self) -> int:
        """HBM bytes a call must move: selected rows, indices, q, out and lse.

        sum over rows of n_valid*(512+64)*2 + topk*4 + H*(576*2 + 512*2 + 4);
        padded slots and untouched pool pages count zero.
        """
        B, H, k = self.num_tokens, self.num_heads, self.topk
        return self.n_valid() * (D_CKV + D_KPE) * 2 + B * k * 4 + B * H * ((D_CKV + D_KPE) * 2 + D_CKV * 2 + 4)

    def algorithmic_flops(self) -> int:
        """2*H*n_valid*(576+512): the QK^T and PV contractions over valid slots."""
        return 2 * self.num_heads * self.n_valid() * ((D_CKV + D_KPE) + D_CKV)

    def args(self):
        return (self.q_nope, self.q_pe, self.ckv_cache, self.kpe_cache, self.sparse_indices,
                self.sm_scale)


def _seq_lens(name: str, B: int, gen: torch.Generator) -> list:
    if name == "tiny":
        return [1024, 1000][:B]
    if name == "b64_h16":
        return torch.randint(4096, 32768 + 1, (B,), generator=gen).tolist()
    if name == "b32_h128":
        return [65536] * B
    if name == "ragged_b256":
        u = torch.rand(B, generator=gen, dtype=torch.float64)
        return [int(round(math.exp(math.log(128) + x * (math.log(131072) - math.log(128))))) for x in u.tolist()]
    if name == "b2048":
        return torch.randint(8192, 131072 + 1, (B,), generator=gen).tolist()
    raise KeyError(name)


def _positions(name: str, seq: torch.Tensor, topk: int, device, gen_dev) -> torch.Tensor:
    """Distinct positions per row (random order), -1 after a short row's positions."""
    B = seq.numel()
    Lmax = int(seq.max().item())
    out = torch.empty(B, topk, dtype=torch.int64, device=device)
    chunk = max(1, (1 << 26) // max(Lmax, 1))
    ar = torch.arange(Lmax, device=device)
    for r0 in range(0, B, chunk):
        r1 = min(B, r0 + chunk)
        L = seq[r0:r1].to(device)[:, None]
        keys = torch.rand(r1 - r0, Lmax, generator=gen_dev, device=device)
        if name == "b32_h128":
            # half from the most recent 4096 tokens, half from the rest
            recent = torch.clamp(L - 4096, min=0)
            in_recent = (ar[None, :] >= recent) & (ar[None, :] < L)
            in_rest = ar[None, :] < recent
            k_recent = torch.where(in_recent, keys, torch.full_like(keys, 2.0))
            k_rest = torch.where(in_rest, keys, torch.full_like(keys, 2.0))
            a = torch.topk(k_recent, topk // 2, dim=1, largest=False).indices
            b = torch.topk(k_rest, topk - topk // 2, dim=1, largest=False).indices
            pos = torch.cat([a, b], dim=1)
        else:
            keys = torch.where(ar[None, :] < L, keys, torch.full_like(keys, 2.0))
            k = min(topk, Lmax)
            sel = torch.topk(keys, k, dim=1, largest=False)
            pos = torch.where(sel.values < 2.0, sel.indices, torch.full_like(sel.indices, -1))
            if k < topk:
                pos = torch.cat([pos, torch.full((r1 - r0, topk - k), -1, dtype=pos.dtype, device=device)], 1)
        out[r0:r1] = pos
    return out


def make(name: str, device="cuda", seed: int = 0, rank: int = 0, world_size: int = 1,
         batch: int | None = None) -> Workload:
    """Build config ``name`` for ``rank`` of ``world_size`` (rows split evenly)."""
    cfg = CONFIGS[name]
    device = torch.device(device)
    B_total = cfg["B"] if batch is None else batch
    if B_total % world_size:
        raise ValueError(f"batch {B_total} does not split over {world_size} ranks")
    B, H, topk = B_total // world_size, cfg["H"], cfg["topk"]
    gen = torch.Generator().manual_seed(seed * 1000003 + rank)
    gen_dev = torch.Generator(device=device).manual_seed(seed * 1000003 + rank + 17)
    seq = _seq_lens(name, B, gen)
    npages = [-(-L // PAGE) for L in seq]
    P = 32 if name == "tiny" else sum(npages)
    perm = torch.randperm(P, generator=gen).to(device)
    offs = torch.tensor([0] + npages[:-1], dtype=torch.int64).cumsum(0).to(device)
    pos = _positions(name, torch.tensor(seq, dtype=torch.int64), topk, device, gen_dev)
    valid = pos >= 0
    posc = pos.clamp(min=0)
    page = perm[offs[:, None] + posc // PAGE]
    slots = torch.where(valid, page * PAGE + posc % PAGE, torch.full_like(posc, -1)).to(torch.int32)

    def normal(shape, scale):
        t = torch.randn(shape, generator=gen_dev, device=device, dtype=torch.bfloat16)
        if scale != 1.0:
            t.mul_(scale)
        return t

    q_nope = normal((B, H, D_CKV), 1.0)
    q_pe = normal((B, H, D_KPE), 1.0)
    ckv = normal((P, PAGE, D_CKV), cfg["kv_scale"])
    kpe = normal((P, PAGE, D_KPE), cfg["kv_scale"])
    maxp = max(npages)
    j = torch.arange(maxp, device=device)
    np_t = torch.tensor(npages, dtype=torch.int64, device=device)
    page_table = torch.where(j[None, :] < np_t[:, None],
                             perm[(offs[:, None] + j[None, :]).clamp(max=P - 1)],
                             torch.full((B, maxp), -1, dtype=perm.dtype, device=device))
    return Workload(name, q_nope, q_pe, ckv, kpe, slots.contiguous(), 1.0 / math.sqrt(192.0), seq,
                    page_table.to(torch.int32).contiguous(), pos.to(torch.int32).contiguous())


def make_prefill(num_seqs: int, chunk: int, seq_len: int, heads: int = 16, topk: int = 2048,
                 mode: str = "all", device="cuda", seed: int = 0) -> Workload:
    """Multi-token rows: the last ``chunk`` tokens of ``num_seqs`` sequences of ``seq_len``.

    Token j of a sequence sits at position p = seq_len - chunk + j and selects among the
    positions <= p (causal): every one of them (``mode="all"``, the indexer's choice when
    the sequence is no longer than topk, so seq_len <= topk), or ``min(topk, p + 1)``
    distinct ones drawn uniformly and independently per token (``mode="random"``: the
    least overlap between tokens). Positions are ascending with -1 after them, as the
    top-k step writes them. Rows are the tokens, sequence by sequence; ``page_table`` has
    one row per token (equal rows within a sequence).
    """
    if mode == "all" and seq_len > topk:
        raise ValueError("mode 'all' needs seq_len <= topk")
    device = torch.device(device)
    gen = torch.Generator().manual_seed(seed * 7919 + 3)
    gen_dev = torch.Generator(device=device).manual_seed(seed * 7919 + 5)
    B = num_seqs * chunk
    npg = -(-seq_len // PAGE)
    P = num_seqs * npg
    perm = torch.randperm(P, generator=gen).to(device)
    seq_pt = perm.view(num_seqs, npg)
    page_table = seq_pt.repeat_interleave(chunk, dim=0).to(torch.int32).contiguous()
    p_tok = (seq_len - chunk + torch.arange(chunk, device=device)).repeat(num_seqs)  # [B]
    ar = torch.arange(seq_len, device=device)
    pos = torch.full((B, topk), -1, dtype=torch.int64, device=device)
    rows_per = max(1, (1 << 25) // seq_len)
    for r0 in range(0, B, rows_per):
        r1 = min(B, r0 + rows_per)
        live = ar[None, :] <= p_tok[r0:r1, None]
        if mode == "all":
            cand = torch.where(live, ar[None, :].expand(r1 - r0, -1), torch.full_like(ar, seq_len)[None, :])
            sel = torch.sort(cand, dim=1).values[:, :topk]
        elif mode == "random":
            keys = torch.rand(r1 - r0, seq_len, generator=gen_dev, device=device)
            keys = torch.where(live, keys, torch.full_like(keys, 2.0))
            k = min(topk, seq_len)
            v, i = torch.topk(keys, k, dim=1, largest=False)
            cand = torch.where(v < 2.0, i, torch.full_like(i, seq_len))
            sel = torch.sort(cand, dim=1).values
        else:
            raise ValueError(f"unknown mode {mode!r}")
        sel = torch.where(sel < seq_len, sel, torch.full_like(sel, -1))
        pos[r0:r1, :sel.shape[1]] = sel
    seq_of = torch.arange(B, device=device) // chunk
    valid = pos >= 0
    posc = pos.clamp(min=0)
    page = seq_pt[seq_of[:, None], posc // PAGE]
    slots = torch.where(valid, page * PAGE + posc % PAGE, torch.full_like(posc, -1)).to(torch.int32)

    def normal(shape, scale):
        t = torch.randn(shape, generator=gen_dev, device=device, dtype=torch.bfloat16)
        return t.mul_(scale) if scale != 1.0 else t

    q_nope = normal((B, heads, D_CKV), 1.0)
    q_pe = normal((B, heads, D_KPE), 1.0)
    ckv = normal((P, PAGE, D_CKV), 0.5)
    kpe = normal((P, PAGE, D_KPE), 0.5)
    return Workload(f"prefill_{mode}", q_nope, q_pe, ckv, kpe, slots.contiguous(),
                    1.0 / math.sqrt(192.0), [seq_len] * num_seqs, page_table,
                    pos.to(torch.int32).contiguous())
