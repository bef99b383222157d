// Pieces of the decode pipeline that every kernel instance shares: the UMMA shared-memory
// descriptor, the per-tile index fetch (flat slot ids or paged token positions), the gather
// producers that fill a stage with this CTA's half of every selected slot, and the Q loader.
//
// Both CTAs of a cluster pair gather the same slots: rank r keeps ckv columns
// [256r, 256r + 256) as four 64-wide d-blocks (128-byte swizzle, [kTS slots x 128 B] each)
// and kpe columns [32r, 32r + 32) as one block (64-byte swizzle, [kTS x 64 B]).
#pragma once

namespace dsa {
namespace pipe {

constexpr int kBlk = 4;                   // 64-wide ckv d-blocks per CTA
constexpr int kProdWarps = kBlk + 1;      // one gather producer warp per d-block + the kpe half
constexpr int kMaskAny = 7;               // mask word of a stage: nonzero when any slot is valid
constexpr uint32_t kSw128 = 2, kSw64 = 4;  // UMMA descriptor layout types

// UMMA shared-memory descriptor (sm_100, version 1): start, leading and stride byte offsets.
__device__ __forceinline__ uint64_t desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                         uint32_t layout) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46) |
         ((uint64_t)layout << 61);
}

// Index entries of tile t of (row, head group) rh for a producer lane's group g: slot
// ids, or token positions in a paged call; -1 past topk.
template <int kTS>
__device__ __forceinline__ void tile_entries(const Params& p, int64_t rh, int t, bool has, int g,
                                             int (&r)[4]) {
  const int32_t* ir = p.idx + (rh >> p.hg_shift) * p.idx_sb;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int k = t * kTS + 4 * g + e;
    r[e] = (has && k < p.topk) ? __ldg(ir + k) : -1;
  }
}

// Slot ids of a paged call's token positions: slot = page_table[row][pos >> pg_shift] *
// page_size + (pos & (page_size - 1)), the flat slot the pool's [pages, page_size, D] layout
// gives (fused.py:155-156).  -1 stays padding; a position past the row's table, a negative
// page or a slot beyond int32 becomes -2, which the producer flags as a bad index.
__device__ __forceinline__ void translate(const Params& p, int64_t rh, const int (&pos)[4],
                                          int (&r)[4]) {
  const int32_t* pr = p.pt + (rh >> p.hg_shift) * p.pt_sb;
  const int mask = (1 << p.pg_shift) - 1;
  int page[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int q = pos[e];
    const bool in_table = q >= 0 && (q >> p.pg_shift) < p.pt_cols;
    page[e] = in_table ? __ldg(pr + (q >> p.pg_shift)) : (q == -1 ? -1 : -2);
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int q = pos[e];
    if (q < 0 || page[e] < 0) {
      r[e] = (q == -1) ? -1 : -2;
    } else {
      const int64_t slot = ((int64_t)page[e] << p.pg_shift) | (int64_t)(q & mask);
      r[e] = slot > (int64_t)INT32_MAX ? -2 : (int)slot;
    }
  }
}

// One gather producer warp (d-block `blk` of this CTA's half; blk == kBlk: the kpe half)
// over the units [u_lo, u_hi) of this pair.  Lane g issues one tile::gather4 (slots
// 4g..4g+3 of the tile) per tile into stage st = i % kStages, after the stage's region is
// free again (barrier kve0 + 8 (5 st + blk)); the stage's full barrier (kvf0 + 8 st) counts
// one arrive with the expected bytes per producer warp.  d-block 0's warp also writes the
// tile's slot-validity mask (one bit per slot, word kMaskAny nonzero when any slot is
// valid) and flags bad indices.  kPaged: the entries are token positions, fetched two tiles
// ahead and translated through the row's page table one tile ahead, so the dependent
// page-table load is off the producer's path.
//
// kMember (token groups): d-block 0's warp also loads the entries' membership bytes one
// tile ahead, like the ids, and stores them per stage into `memb` ([kStages][kTS / 4]
// words, byte e of word g = entry 4g + e, zero for padding and bad entries) before the
// stage's full barrier is armed.
template <int kTS, int kStageB, int kStages, int kMaskStride, bool kPaged, bool kMember = false>
__device__ __forceinline__ void gather_producer(const Params& p, const CUtensorMap* tm_ckv,
                                                const CUtensorMap* tm_kpe, int blk, int lane,
                                                uint32_t rank, uint32_t stage0,
                                                volatile uint32_t* masks, uint32_t kvf0,
                                                uint32_t kve0, int64_t u_lo, int64_t u_hi,
                                                const Waiter& wait, volatile uint32_t* drain_flag,
                                                volatile uint32_t* memb = nullptr) {
  static_assert(!(kMember && kPaged), "membership bytes come with flat slot ids");
  constexpr int kRB = kTS * 128;  // one ckv d-block region of a stage
  constexpr int kGroups = kTS / 4;
  static_assert(kGroups <= 32 && kTS <= 128, "one gather4 group per lane, four mask words");
  const int g = lane;
  const bool has = g < kGroups;
  const bool is_kpe = blk == kBlk;
  const uint32_t dst_off =
      is_kpe ? (uint32_t)(kBlk * kRB + g * 256) : (uint32_t)(blk * kRB + g * 512);
  const int col = is_kpe ? (int)(32 * rank) : (int)(256 * rank) + 64 * blk;
  const uint32_t req_bytes = is_kpe ? 256u : 512u;
  const CUtensorMap* map = is_kpe ? tm_kpe : tm_ckv;
  const uint64_t policy = ptx::policy_evict_first();
  bool ok = true;
  int64_t n_issued = 0;
  int cur[4], nxt[4], ahead[4];
  // (rh, t) of the tile whose entries are fetched next, stepped without divisions
  int64_t n_rh = u_lo / p.tpr;
  int n_t = (int)(u_lo - n_rh * p.tpr);
  int64_t a_rh = n_rh;  // paged: row of the positions held in `ahead`
  // paged: pull a row's page table into L2 when the producers reach the row (d-block 0's
  // warp; 128-byte lines), so the translations read it from L2
  auto pf_row = [&](int64_t rh) {
    if constexpr (kPaged) {
      if (blk != 0) return;
      const int32_t* pr = p.pt + (rh >> p.hg_shift) * p.pt_sb;
      for (int c = lane * 32; c < p.pt_cols; c += 32 * 32)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(pr + c));
    }
  };
  // membership bytes of a lane's four entries (d-block 0's warp of a grouped call)
  auto tile_member = [&](int64_t rh, int t) -> uint32_t {
    uint32_t m = 0;
    if constexpr (kMember) {
      if (blk == 0 && has) {
        const uint8_t* mr = p.member + rh * p.member_sb;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int k = t * kTS + 4 * g + e;
          if (k < p.topk) m |= (uint32_t)__ldg(mr + k) << (8 * e);
        }
      }
    }
    return m;
  };
  uint32_t mcur = 0, mnxt = 0;
  if (u_lo < u_hi) pf_row(n_rh);
  if (u_lo < u_hi) {
    if constexpr (kMember) mcur = tile_member(n_rh, n_t);
    tile_entries<kTS>(p, n_rh, n_t, has, g, kPaged ? ahead : cur);
    if constexpr (kPaged) translate(p, n_rh, ahead, cur);
  }
  if constexpr (kPaged) {
    if (++n_t == p.tpr) {
      n_t = 0;
      ++n_rh;
    }
    a_rh = n_rh;
    if (u_lo + 1 < u_hi) tile_entries<kTS>(p, n_rh, n_t, has, g, ahead);
  }
  int st = 0;
  uint32_t phase = 0;
  for (int64_t uu = u_lo, i = 0; uu < u_hi; ++uu, ++i) {
    if constexpr (kPaged) {
      // slot ids of tile uu + 1 from the positions fetched one tile earlier, then the
      // positions of tile uu + 2
      if (uu + 1 < u_hi) translate(p, a_rh, ahead, nxt);
    }
    if (++n_t == p.tpr) {
      n_t = 0;
      ++n_rh;
      if (uu + 2 < u_hi) pf_row(n_rh);
    }
    if constexpr (kPaged) {
      a_rh = n_rh;
      if (uu + 2 < u_hi) tile_entries<kTS>(p, n_rh, n_t, has, g, ahead);
    } else {
      if (uu + 1 < u_hi) {
        if constexpr (kMember) mnxt = tile_member(n_rh, n_t);
        tile_entries<kTS>(p, n_rh, n_t, has, g, nxt);
      }
    }
    uint32_t nib = 0;
    bool bad = false;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (cur[e] < -1 || (int64_t)cur[e] >= p.num_slots) {
        bad = true;
        cur[e] = -1;
      }
      nib |= (cur[e] >= 0 ? 1u : 0u) << e;
    }
    // In a tile with any valid slot every group is requested: a padding slot's id is out
    // of range, so the copy fills its row with zeros, and PV reads 0 * 0 there instead of
    // stale bytes.  An all-padding tile is not requested at all (its score and PV are
    // skipped).  Every producer warp sees the same ids, so the same tiles.
    const bool tile_live = __ballot_sync(0xffffffffu, nib != 0u) != 0u;
    const bool issue = has && tile_live;
    const uint32_t n_req = (uint32_t)__popc(__ballot_sync(0xffffffffu, issue));
    uint32_t w0 = 0, w1 = 0, w2 = 0, w3 = 0;
    if (blk == 0) {
      if (bad) atomicOr(p.err, (uint32_t)DSA_DEVERR_BAD_INDEX);
      const uint32_t sh = nib << (4 * (g & 7));
      w0 = __reduce_or_sync(0xffffffffu, (g >> 3) == 0 ? sh : 0u);
      w1 = __reduce_or_sync(0xffffffffu, (g >> 3) == 1 ? sh : 0u);
      w2 = __reduce_or_sync(0xffffffffu, (g >> 3) == 2 ? sh : 0u);
      w3 = __reduce_or_sync(0xffffffffu, (g >> 3) == 3 ? sh : 0u);
    }
    if constexpr (kMember) {
      // the stage's region must be free before its membership words are rewritten: the
      // whole warp learns the outcome of the wait first
      if (lane == 0) ok = wait(kve0 + 8u * (uint32_t)(5 * st + blk), phase ^ 1u);
      ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
      if (!ok) break;
      if (blk == 0 && has) {
        uint32_t mw = 0;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (cur[e] >= 0) mw |= mcur & (0xFFu << (8 * e));
        memb[st * (kTS / 4) + g] = mw;
      }
      __syncwarp();
      if (lane == 0) {
        if (blk == 0) {
          masks[st * kMaskStride + 0] = w0;
          masks[st * kMaskStride + 1] = w1;
          masks[st * kMaskStride + 2] = w2;
          masks[st * kMaskStride + 3] = w3;
          masks[st * kMaskStride + kMaskAny] = w0 | w1 | w2 | w3;
        }
        ptx::mbar_arrive_expect_tx(kvf0 + 8u * (uint32_t)st, n_req * req_bytes);
      }
      mcur = mnxt;
    } else {
      if (lane == 0) {
        ok = wait(kve0 + 8u * (uint32_t)(5 * st + blk), phase ^ 1u);
        if (ok) {
          if (blk == 0) {
            masks[st * kMaskStride + 0] = w0;
            masks[st * kMaskStride + 1] = w1;
            masks[st * kMaskStride + 2] = w2;
            masks[st * kMaskStride + 3] = w3;
            masks[st * kMaskStride + kMaskAny] = w0 | w1 | w2 | w3;  // nonzero: a valid slot
          }
          ptx::mbar_arrive_expect_tx(kvf0 + 8u * (uint32_t)st, n_req * req_bytes);
        }
      }
      ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
      if (!ok) break;
    }
    n_issued = i + 1;
    if (issue)
      ptx::tma_gather4(stage0 + (uint32_t)(st * kStageB) + dst_off, map, col,
                       make_int4(cur[0], cur[1], cur[2], cur[3]), kvf0 + 8u * (uint32_t)st, policy);
#pragma unroll
    for (int e = 0; e < 4; ++e) cur[e] = nxt[e];
    if (++st == kStages) {
      st = 0;
      phase ^= 1u;
    }
  }
  if (!ok && lane == 0) {
    const Waiter drain{drain_flag, p.err, p.wait_cycles};
    for (int64_t li = n_issued - 1; li >= 0 && li >= n_issued - kStages; --li)
      drain(kvf0 + 8u * (uint32_t)(li % kStages), (uint32_t)((li / kStages) & 1));
  }
}

// The Q loader (one thread): per segment of this pair's units, once the previous segment's
// last score is done (qe), the unit's Q half into one buffer at qdst: kBlk boxes of
// [NH heads x 64] (128-byte swizzle, NH * 128 bytes apart) and one [NH x 32] box of q_pe.
template <int NH>
__device__ __forceinline__ void q_loader(const Params& p, const CUtensorMap* tm_qn,
                                         const CUtensorMap* tm_qp, uint32_t rank, uint32_t qdst,
                                         uint32_t qf, uint32_t qe, int64_t u_lo, int64_t u_hi,
                                         const Waiter& wait, volatile uint32_t* drain_flag) {
  constexpr int kQBlk = NH * 128;
  constexpr uint32_t kQB = kBlk * kQBlk + NH * 64;
  int seg = 0;
  int64_t u = u_lo;
  Segment s;
  while (next_segment(u, u_hi, p.tpr, s)) {
    if (!wait(qe, (uint32_t)((seg & 1) ^ 1))) break;
    ptx::mbar_arrive_expect_tx(qf, kQB);
    const int b = (int)(s.rh >> p.hg_shift);
    const int h0 = NH * (int)(s.rh & ((1 << p.hg_shift) - 1));
    for (int j = 0; j < kBlk; ++j)
      ptx::tma_load_3d(qdst + (uint32_t)(j * kQBlk), tm_qn, (int)(256 * rank) + 64 * j, h0, b, qf);
    ptx::tma_load_3d(qdst + (uint32_t)(kBlk * kQBlk), tm_qp, (int)(32 * rank), h0, b, qf);
    ++seg;
  }
  if (seg > 0) {
    const Waiter drain{drain_flag, p.err, p.wait_cycles};
    drain(qf, (uint32_t)((seg - 1) & 1));
  }
}

}  // namespace pipe
}  // namespace dsa
