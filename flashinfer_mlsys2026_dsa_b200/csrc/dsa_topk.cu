// Index production for the sparse decode: per-row top-k selection over index scores and
// translation of the selected token positions to pool slot ids.
//
// This is the step that builds the decode's `sparse_indices` (the reference's callers form
// them as page * 64 + offset of the selected positions, solution/triton/baseline.py:17-23;
// flashinfer publishes the step as `top_k_page_table_transform`: per row, the top k of
// input[i, :lengths[i]], translated through the row's page table).  Selection is exact:
// the k largest scores of the row, and among scores equal to the k-th largest the smallest
// positions.  The output lists the selected slots in ascending position order, -1 after
// the row's positions when the row has fewer than k (the decode's padding), so that the
// result is one deterministic array.
//
// Without a page table the output is the selected positions themselves (the input of the
// token-group union below).
//
// One CTA per row (1024 threads), or two (a cluster) when the call has at most half as many
// rows as the GPU has SMs and long rows.  Scores are mapped to order-preserving 32-bit keys; a
// radix select finds the k-th largest key T in three histogram passes, high bits first: the
// top byte (one 256-bin histogram per warp, as score bytes crowd into few bins there), then
// two 12-bit digits in one 4096-bin histogram per pass (each over the keys that share the
// bits already fixed, which spread over the bins); a counting pass
// and an ordered compaction pass then write every position with key > T and the first
// ones with key == T.  Each warp owns one contiguous segment of the row and reads it
// coalesced, so positions come out in order without a sort.
//
// The first pass reads the row from global memory once, 16 bytes per load, and keeps the
// keys in shared memory when every row of the call fits (up to kCapKeys positions per CTA),
// so the other four passes read shared memory; otherwise every pass reads global memory.
// The ordered compaction writes positions; a last pass translates them through the page
// table, so that the page-table loads of a thread are in flight together.
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

#include "dsa_b200.h"

namespace dsa {
namespace topk {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kBins = 256;     // the first pass: the key's top byte
constexpr int kBins12 = 4096;  // the second and third passes: 12 key bits each
constexpr int kCapKeys = 48 * 1024;  // positions whose keys stay in shared memory (192 KB)
// The same per CTA of a two-CTA row, whose static shared memory is 1 KB larger.
constexpr int kCapKeysPart = 47 * 1024;
// Rows split between two CTAs only past this length: the split adds a cluster barrier per
// pass and one for the counts (about 0.5 us each), which the halved passes repay on longer
// rows (measured on B200 with 64 rows, four-pass select: 4k positions 11.3 us split against
// 9.2 whole, 32k positions 17.4 against 22.5).
constexpr int kPartsMinLen = 12 * 1024;

struct Params {
  const float* scores;
  int64_t scores_sb;
  const int32_t* lengths;
  const int32_t* pt;  // page table rows
  int64_t pt_sb;
  int32_t pt_cols;
  int32_t pg_shift;   // log2(page_size)
  int32_t max_len;
  int32_t k;
  int32_t* slots;
  int64_t slots_sb;
};

// Order-preserving key: a larger float has a larger key; NaN maps below every number.
__device__ __forceinline__ uint32_t score_key(float f) {
  const uint32_t u = __float_as_uint(f);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu)) return 0u;  // NaN
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ int32_t slot_of(const Params& p, const int32_t* pr, int pos) {
  if (pr == nullptr) return pos;  // no page table: the positions themselves
  const int pg = pos >> p.pg_shift;
  if (pg >= p.pt_cols) return -1;
  const int32_t page = __ldg(pr + pg);
  if (page < 0) return -1;
  const int64_t slot = ((int64_t)page << p.pg_shift) | (int64_t)(pos & ((1 << p.pg_shift) - 1));
  return slot > (int64_t)INT32_MAX ? -1 : (int32_t)slot;
}

// Inclusive prefix sum over the block of one value per thread (warp shuffles + one smem pass).
__device__ __forceinline__ uint32_t block_inclusive_scan(uint32_t v, uint32_t* wsum) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) wsum[warp] = v;
  __syncthreads();
  if (warp == 0) {
    uint32_t w = wsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    wsum[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const uint32_t r = v + (warp > 0 ? wsum[warp - 1] : 0u);
  __syncthreads();  // wsum may be reused by the caller's next scan
  return r;
}

// Given the histogram `hist[kBins]` of the candidate keys' current byte and `need` (>= 1,
// at most the candidates' count) elements still to take from the top: the bin holding the
// need-th largest candidate into *bin_out, and how many candidates lie in higher bins into
// *above.  Threads t < kBins (eight warps) own bin kBins - 1 - t: a warp scan over each
// warp's 32 bins, the eight warp totals through `wtot` and one block barrier.  (One warp
// walking eight bins per lane took ~1,800 cycles per pass, mostly its serial scan.)
__device__ __forceinline__ void select_bin(const uint32_t* hist, uint32_t need, uint32_t* wtot,
                                           uint32_t* above, int* bin_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int kSelWarps = kBins / 32;
  uint32_t incl = 0, mine = 0;
  if (warp < kSelWarps) {
    mine = hist[kBins - 1 - (int)threadIdx.x];
    incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) wtot[warp] = incl;
  }
  __syncthreads();
  if (warp < kSelWarps) {
#pragma unroll
    for (int w = 0; w < kSelWarps; ++w) incl += w < warp ? wtot[w] : 0u;
    const uint32_t excl = incl - mine;  // candidates in bins above this thread's
    if (excl < need && incl >= need) {
      *bin_out = kBins - 1 - (int)threadIdx.x;
      *above = excl;
    }
  }
}

// The same over kBins12 bins, from the four counts `cnt` of this thread's bins 4095 - 4t down
// to 4092 - 4t (thread t of the block, highest first): a block scan of the per-thread sums
// (warp shuffles, the 32 warp totals through `wtot32`, one block barrier), then the thread
// whose range holds the need-th candidate walks its four bins.
__device__ __forceinline__ void select_bin12(const uint32_t (&cnt)[4], uint32_t need,
                                             uint32_t* wtot32, uint32_t* above, int* bin_out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t mine = cnt[0] + cnt[1] + cnt[2] + cnt[3];
  uint32_t incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) wtot32[warp] = incl;
  __syncthreads();
  uint32_t wt = wtot32[lane];  // inclusive scan of the warp totals, in every warp
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t n = __shfl_up_sync(0xffffffffu, wt, o);
    if (lane >= o) wt += n;
  }
  const uint32_t before = __shfl_sync(0xffffffffu, wt, (warp + 31) & 31);
  incl += warp > 0 ? before : 0u;
  const uint32_t excl = incl - mine;  // candidates in bins above this thread's four
  if (excl < need && incl >= need) {
    uint32_t acc = excl;
    int b = kBins12 - 4 - 4 * (int)threadIdx.x;
    bool done = false;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (!done) {
        if (acc + cnt[j] >= need) {
          b = kBins12 - 1 - 4 * (int)threadIdx.x - j;
          done = true;
        } else {
          acc += cnt[j];
        }
      }
    }
    *bin_out = b;
    *above = acc;
  }
}

// ---- programmatic dependent launch: the kernel is launched so that it may start while the
// previous grid of the stream drains, and waits for that grid (griddepcontrol.wait) before
// it reads global memory; once its threshold key is known it lets the next grid (the
// decode) start its set-up, which itself waits for this grid before it reads the slot ids.
__device__ __forceinline__ void wait_prior_grid() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_next_grid() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- the two CTAs of a row (a cluster of two): every thread of both takes part
__device__ __forceinline__ uint32_t cta_rank_in_cluster() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Full cluster barrier: this CTA's earlier shared-memory writes are visible to the other
// CTA, and the other CTA's to this one, once it returns.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}
// Split form: the arrive says this thread's reads of the other CTA's shared memory are
// complete; the wait (before exit) keeps the CTA, and so its shared memory, alive until the
// other CTA has arrived too.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The 32-bit word at the same shared-memory address in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t ld_peer_u32(const uint32_t* local, uint32_t rank) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(local);
  uint32_t ra, v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(ra) : "memory");
  return v;
}

// The 16 bytes at the same (16-byte aligned) shared-memory address in CTA `rank`.
__device__ __forceinline__ uint4 ld_peer_v4(const uint32_t* local, uint32_t rank) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(local);
  uint32_t ra;
  uint4 v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(a), "r"(rank));
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(ra)
               : "memory");
  return v;
}

// kCached: the keys of a CTA's positions are kept in dynamic shared memory (every row of the
// call fits); otherwise each pass reads the scores from global memory.  Two instances per
// kParts, because only the cached one raises the function's shared-memory limit (the full
// carve-out leaves L1 too small for the uncached passes' re-reads).
//
// kParts == 2: a row is split between the two CTAs of a cluster (used when the call has at
// most half as many rows as the GPU has SMs, so that the other SMs are not left idle, and
// rows longer than kPartsMinLen).  CTA
// r holds the positions [lo_r, hi_r) (rank 0 the first half, rounded to 4 positions so that
// both halves start 16-byte aligned); each pass adds the other CTA's histogram, read through
// distributed shared memory after a cluster barrier, so that both CTAs pick the same bin and
// end with the same T; rank 1's compaction then starts after rank 0's keys.  The output is
// the same array as with one CTA per row.
template <bool kCached, int kParts>
__global__ void __launch_bounds__(kThreads, 1) topk_slots_kernel(const Params p) {
  static_assert(kParts == 1 || kParts == 2, "one or two CTAs per row");
  extern __shared__ uint32_t skey[];         // kCached: the keys of this CTA's positions
  // the first pass's per-warp histograms of the top key byte; then (same memory) the
  // 4096-bin histograms of the second and third passes, [pass - 1][bin]
  __shared__ __align__(16) uint32_t whist[kWarps][kBins];
  static_assert(kWarps * kBins == 2 * kBins12, "two 12-bit histograms in the first pass's memory");
  __shared__ uint32_t hist[kBins];           // the first pass's row histogram (both CTAs' added)
  __shared__ uint32_t hpart[kBins];          // kParts == 2: this CTA's first-pass histogram
  __shared__ uint32_t wtot[kWarps];          // bin selection: per-warp totals
  __shared__ uint32_t above_s;
  __shared__ int bin_s;
  __shared__ uint32_t wcount[2][kWarps];  // per warp: keys > T, keys == T
  __shared__ uint32_t ccount[2];          // kParts == 2: this CTA's keys > T, keys == T
  wait_prior_grid();
  const int row = blockIdx.x / kParts;
  const uint32_t part = kParts == 1 ? 0u : cta_rank_in_cluster();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* sr = p.scores + (int64_t)row * p.scores_sb;
  const int32_t* pr = p.pt ? p.pt + (int64_t)row * p.pt_sb : nullptr;
  int32_t* out = p.slots + (int64_t)row * p.slots_sb;
  int L = __ldg(p.lengths + row);
  L = L < 0 ? 0 : (L > p.max_len ? p.max_len : L);
  const int k = p.k;

  if (L <= k) {  // every position, in order, then padding (both CTAs return here together)
    for (int i = (int)part * kThreads + threadIdx.x; i < k; i += kParts * kThreads)
      out[i] = i < L ? slot_of(p, pr, i) : -1;
    return;
  }

  // this CTA's positions [lo, hi)
  const int half = kParts == 1 ? L : min(L, ((L >> 1) + 3) & ~3);
  const int lo = part == 0 ? 0 : half, hi = part == 0 ? half : L;
  const int n = hi - lo;
  const float* sl = sr + lo;

  constexpr bool cached = kCached;
  auto key_at = [&](int j) -> uint32_t {  // j: index into [lo, hi)
    if constexpr (kCached) return skey[j];
    else return score_key(__ldg(sl + j));
  };

  // ---- radix select of the k-th largest key: the top byte (bits 31..24), then bits 23..12,
  // then bits 11..0, each later pass over the keys that share the bits already fixed
  uint32_t prefix = 0, need = (uint32_t)k;
  {
    uint32_t* wh = whist[warp];
    for (int j = lane; j < kBins; j += 32) wh[j] = 0u;
    __syncwarp();
    // every key: 16-byte loads where the row is 16-byte aligned, keys kept if cached
    const int nv = (reinterpret_cast<uintptr_t>(sl) & 15u) == 0 ? (n >> 2) : 0;
    const float4* sr4 = reinterpret_cast<const float4*>(sl);
#pragma unroll 2
    for (int v = threadIdx.x; v < nv; v += kThreads) {
      const float4 f = __ldg(sr4 + v);
      const uint32_t k0 = score_key(f.x), k1 = score_key(f.y), k2 = score_key(f.z),
                     k3 = score_key(f.w);
      if constexpr (cached) reinterpret_cast<uint4*>(skey)[v] = make_uint4(k0, k1, k2, k3);
      atomicAdd(&wh[k0 >> 24], 1u);
      atomicAdd(&wh[k1 >> 24], 1u);
      atomicAdd(&wh[k2 >> 24], 1u);
      atomicAdd(&wh[k3 >> 24], 1u);
    }
    for (int i = 4 * nv + threadIdx.x; i < n; i += kThreads) {
      const uint32_t key = score_key(__ldg(sl + i));
      if constexpr (cached) skey[i] = key;
      atomicAdd(&wh[key >> 24], 1u);
    }
    __syncthreads();
    uint32_t c = 0;
    if (threadIdx.x < kBins) {
#pragma unroll 8
      for (int w = 0; w < kWarps; ++w) c += whist[w][threadIdx.x];
      if constexpr (kParts == 1) hist[threadIdx.x] = c;
      else hpart[threadIdx.x] = c;
    }
    if constexpr (kParts == 2) {
      // both CTAs' first-pass histograms are complete; hpart is not written again
      cluster_sync();
      if (threadIdx.x < kBins) hist[threadIdx.x] = c + ld_peer_u32(&hpart[threadIdx.x], part ^ 1u);
    }
    __syncthreads();  // hist complete; every read of whist is done
    // the two 12-bit histograms (whist's memory) start at zero; the barrier below orders
    // this before the second pass's counts
    reinterpret_cast<uint4*>(&whist[0][0])[threadIdx.x] = make_uint4(0u, 0u, 0u, 0u);
    reinterpret_cast<uint4*>(&whist[0][0])[threadIdx.x + kThreads] = make_uint4(0u, 0u, 0u, 0u);
    select_bin(hist, need, wtot, &above_s, &bin_s);
    __syncthreads();
    need -= above_s;
    prefix = (uint32_t)bin_s;
  }
  for (int pass = 1; pass < 3; ++pass) {
    uint32_t* h12 = &whist[0][0] + (pass - 1) * kBins12;
    const int sh = pass == 1 ? 12 : 0;  // the pass's 12 bits are key bits [sh, sh + 12)
#pragma unroll 4
    for (int i = threadIdx.x; i < n; i += kThreads) {
      const uint32_t key = key_at(i);
      if ((key >> (sh + 12)) == prefix) atomicAdd(&h12[(key >> sh) & (kBins12 - 1)], 1u);
    }
    // this thread's bins 4095 - 4t .. 4092 - 4t, highest first (both CTAs' added); each
    // 12-bit histogram is written in its pass only, so the other CTA may read it any time
    // after the cluster barrier
    const uint32_t* mine = h12 + (kBins12 - 4 - 4 * (int)threadIdx.x);
    if constexpr (kParts == 2) cluster_sync();
    else __syncthreads();
    uint4 v = *reinterpret_cast<const uint4*>(mine);
    if constexpr (kParts == 2) {
      const uint4 r = ld_peer_v4(mine, part ^ 1u);
      v.x += r.x;
      v.y += r.y;
      v.z += r.z;
      v.w += r.w;
    }
    const uint32_t cnt[4] = {v.w, v.z, v.y, v.x};
    select_bin12(cnt, need, wtot, &above_s, &bin_s);
    // bin_s / above_s and wtot are written again only after two more barriers
    __syncthreads();
    need -= above_s;
    prefix = (prefix << 12) | (uint32_t)bin_s;
  }
  const uint32_t T = prefix;  // the k-th largest key; `need` keys equal to T are taken
  allow_next_grid();

  // ---- counting pass: each warp owns a contiguous segment of this CTA's positions
  const int seg = (n + kWarps - 1) / kWarps;
  const int s0 = warp * seg, s1 = min(n, s0 + seg);
  uint32_t gt = 0, eq = 0;
#pragma unroll 4
  for (int i = s0 + lane; i < s1; i += 32) {
    const uint32_t key = key_at(i);
    gt += key > T;
    eq += key == T;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    gt += __shfl_xor_sync(0xffffffffu, gt, o);
    eq += __shfl_xor_sync(0xffffffffu, eq, o);
  }
  if (lane == 0) {
    wcount[0][warp] = gt;
    wcount[1][warp] = eq;
  }
  __syncthreads();
  // keys > T and == T at positions before this CTA's (rank 0's counts, for rank 1)
  uint32_t gt_base = 0, eq_base = 0;
  if constexpr (kParts == 2) {
    if (threadIdx.x == 0) {
      uint32_t g = 0, e = 0;
      for (int w = 0; w < kWarps; ++w) {
        g += wcount[0][w];
        e += wcount[1][w];
      }
      ccount[0] = g;
      ccount[1] = e;
    }
    cluster_sync();
    if (part == 1) {
      gt_base = ld_peer_u32(&ccount[0], 0);
      eq_base = ld_peer_u32(&ccount[1], 0);
    }
    cluster_arrive();  // no read of the other CTA's shared memory follows
  }
  uint32_t gt_before = gt_base, eq_before = eq_base;
  for (int w = 0; w < warp; ++w) {
    gt_before += wcount[0][w];
    eq_before += wcount[1][w];
  }
  // ---- ordered compaction: keys > T, and keys == T while fewer than `need` were taken
  uint32_t pos_out = gt_before + min(eq_before, need);
  uint32_t eq_seen = eq_before;
  const uint32_t below = (1u << lane) - 1u;  // lanes before this one
  constexpr int kU = 4;
  int base = s0;
  for (; base + 32 * kU <= s1; base += 32 * kU) {
    uint32_t key[kU], em[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) key[u] = key_at(base + 32 * u + lane);
#pragma unroll
    for (int u = 0; u < kU; ++u) em[u] = __ballot_sync(0xffffffffu, key[u] == T);
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const uint32_t eq_rank = eq_seen + __popc(em[u] & below);
      const bool take = key[u] > T || (key[u] == T && eq_rank < need);
      const uint32_t take_mask = __ballot_sync(0xffffffffu, take);
      if (take) out[pos_out + __popc(take_mask & below)] = lo + base + 32 * u + lane;
      pos_out += __popc(take_mask);
      eq_seen += __popc(em[u]);
    }
  }
  for (; base < s1; base += 32) {
    const int i = base + lane;
    const uint32_t key = i < s1 ? key_at(i) : 0u;
    const bool is_eq = i < s1 && key == T;
    const uint32_t eq_mask = __ballot_sync(0xffffffffu, is_eq);
    const uint32_t eq_rank = eq_seen + __popc(eq_mask & ((1u << lane) - 1u));
    const bool take = i < s1 && (key > T || (is_eq && eq_rank < need));
    const uint32_t take_mask = __ballot_sync(0xffffffffu, take);
    if (take) out[pos_out + __popc(take_mask & ((1u << lane) - 1u))] = lo + i;
    pos_out += __popc(take_mask);
    eq_seen += __popc(eq_mask);
  }
  // ---- positions to slot ids: a separate pass over the entries this CTA wrote, so that
  // the page-table loads of a thread's entries are in flight together instead of one per
  // compaction step
  if (pr != nullptr) {
    int j0 = 0, j1 = k;
    if constexpr (kParts == 2) {
      // rank 0 wrote [0, m0), rank 1 [m0, k), m0 = rank 0's keys > T and taken keys == T
      const uint32_t m0 = part == 0 ? ccount[0] + min(ccount[1], need) : gt_base + min(eq_base, need);
      (part == 0 ? j1 : j0) = (int)m0;
    }
    __syncthreads();
#pragma unroll 4
    for (int j = j0 + threadIdx.x; j < j1; j += kThreads) out[j] = slot_of(p, pr, out[j]);
  }
  if constexpr (kParts == 2) cluster_wait();
}

// ---------------------------------------------------------------------------------------
// Union of the selections of a token group, for the grouped decode.
//
// G consecutive tokens of one sequence (G * heads = 128) are decoded as one 128-head row
// over the union of their selected positions: each union entry is gathered once for all
// G tokens and carries a membership byte (bit j: token j of the group selected it), which
// masks the other tokens' heads in the softmax.  One CTA per group: the positions of the
// group's tokens are scattered into a membership byte per position in shared memory (one
// window of kWin positions at a time), then an ordered compaction writes the positions
// that any token selected, ascending, translated through the group's page table (a
// position past the table or on a negative page becomes a -1 entry with no member), -1 /
// 0 after the last entry.  counts[g] receives the union size; entries past out_cols are
// dropped (counts[g] > out_cols tells the caller).

constexpr int kWin = 65536;            // positions per shared-memory window (64 KB)
constexpr int kWinWords = kWin / 4;    // membership bytes packed four to a word
constexpr int kWordsPerThread = kWinWords / kThreads;

struct UnionParams {
  const int32_t* pos;
  int64_t pos_sb;
  int32_t k;
  int32_t group;
  const int32_t* pt;
  int64_t pt_sb;
  int32_t pt_cols;
  int32_t pg_shift;
  int64_t max_pos;  // pt_cols * page_size
  int32_t* slots;
  uint8_t* member;
  int64_t out_sb;
  int32_t out_cols;
  int32_t* counts;
};

// Nonzero bytes of a word, as a 4-bit mask (bit b: byte b is nonzero).
__device__ __forceinline__ uint32_t nonzero_bytes(uint32_t v) {
  return (v & 0xFFu ? 1u : 0u) | (v & 0xFF00u ? 2u : 0u) | (v & 0xFF0000u ? 4u : 0u) |
         (v & 0xFF000000u ? 8u : 0u);
}

__global__ void __launch_bounds__(kThreads, 1) union_groups_kernel(const UnionParams p) {
  extern __shared__ uint32_t win[];  // kWinWords membership words
  __shared__ uint32_t wsum[32];
  __shared__ uint32_t total_s;
  const int g = blockIdx.x;
  const int32_t* pr = p.pt + (int64_t)g * p.pt_sb;
  int32_t* so = p.slots + (int64_t)g * p.out_sb;
  uint8_t* mo = p.member + (int64_t)g * p.out_sb;
  const int mask = (1 << p.pg_shift) - 1;
  int64_t n_out = 0;  // union entries so far (block-uniform)
  for (int64_t w0 = 0; w0 < p.max_pos; w0 += kWin) {
    for (int i = threadIdx.x; i < kWinWords; i += kThreads) win[i] = 0u;
    __syncthreads();
    for (int j = 0; j < p.group; ++j) {
      const int32_t* pj = p.pos + ((int64_t)g * p.group + j) * p.pos_sb;
      for (int i = threadIdx.x; i < p.k; i += kThreads) {
        const int64_t q = (int64_t)__ldg(pj + i) - w0;
        if (q >= 0 && q < kWin && q + w0 < p.max_pos)
          atomicOr(&win[q >> 2], (1u << j) << (8 * (int)(q & 3)));
      }
    }
    __syncthreads();
    // thread t owns words [t * kWordsPerThread, (t + 1) * kWordsPerThread) of the window
    const int wbase = threadIdx.x * kWordsPerThread;
    uint32_t cnt = 0;
#pragma unroll 8
    for (int i = 0; i < kWordsPerThread; ++i) cnt += __popc(nonzero_bytes(win[wbase + i]));
    const uint32_t incl = block_inclusive_scan(cnt, wsum);
    if (threadIdx.x == kThreads - 1) total_s = incl;
    int64_t o = n_out + (int64_t)(incl - cnt);
    for (int i = 0; i < kWordsPerThread; ++i) {
      const uint32_t v = win[wbase + i];
      if (v == 0u) continue;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint32_t m = (v >> (8 * b)) & 0xFFu;
        if (m == 0u) continue;
        if (o < p.out_cols) {
          const int64_t q = w0 + 4 * (int64_t)(wbase + i) + b;
          const int pg = (int)(q >> p.pg_shift);
          const int32_t page = pg < p.pt_cols ? __ldg(pr + pg) : -1;
          const int64_t slot = page < 0 ? -1 : (((int64_t)page << p.pg_shift) | (q & mask));
          const bool ok = slot >= 0 && slot <= (int64_t)INT32_MAX;
          so[o] = ok ? (int32_t)slot : -1;
          mo[o] = ok ? (uint8_t)m : (uint8_t)0;
        }
        ++o;
      }
    }
    __syncthreads();
    n_out += total_s;
    __syncthreads();  // total_s and win are rewritten by the next window
  }
  for (int64_t i = n_out + threadIdx.x; i < p.out_cols; i += kThreads) {
    so[i] = -1;
    mo[i] = 0;
  }
  if (threadIdx.x == 0 && p.counts) p.counts[g] = (int32_t)(n_out < INT32_MAX ? n_out : INT32_MAX);
}

// Launch with kParts CTAs per row (a cluster of that size), as a programmatic dependent of
// the stream's previous grid.
template <bool kCached, int kParts>
int launch(const Params& p, int64_t rows, size_t smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(rows * kParts));
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = kParts;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = kParts > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, topk_slots_kernel<kCached, kParts>, p) == cudaSuccess ? DSA_OK
                                                                                         : DSA_ERR_CUDA;
}

}  // namespace topk
}  // namespace dsa

extern "C" int dsa_topk_slots(const float* scores, int64_t scores_stride_b, const int32_t* lengths,
                              const int32_t* page_table, int64_t page_table_stride_b,
                              int32_t page_table_cols, int32_t page_size, int64_t num_rows,
                              int32_t max_len, int32_t k, int32_t* slots,
                              int64_t slots_stride_b, void* stream) {
  if (num_rows < 0 || max_len < 0 || k < 1 || num_rows > INT32_MAX) return DSA_ERR_INVALID_ARGUMENT;
  if (num_rows == 0) return DSA_OK;
  if (!scores || !lengths || !slots) return DSA_ERR_INVALID_ARGUMENT;
  if (scores_stride_b < max_len || slots_stride_b < k) return DSA_ERR_INVALID_ARGUMENT;
  if (page_table != nullptr &&
      (page_table_cols < 1 || page_table_stride_b < page_table_cols || page_size < 1 ||
       page_size > (1 << 20) || (page_size & (page_size - 1)) != 0))
    return DSA_ERR_INVALID_ARGUMENT;
  dsa::topk::Params p;
  p.scores = scores;
  p.scores_sb = scores_stride_b;
  p.lengths = lengths;
  p.pt = page_table;
  p.pt_sb = page_table_stride_b;
  p.pt_cols = page_table_cols;
  p.pg_shift = 0;
  while (page_table != nullptr && (1 << p.pg_shift) < page_size) ++p.pg_shift;
  p.max_len = max_len;
  p.k = k;
  p.slots = slots;
  p.slots_sb = slots_stride_b;
  // Two CTAs per row (a cluster) when the call has at most half as many rows as the GPU has
  // SMs and rows longer than kPartsMinLen.  When every row's keys fit (kCapKeys per CTA)
  // they stay in dynamic shared memory, a per-device function attribute of the cached
  // instances, set once per device (not inside a stream capture when the first call ran
  // eagerly).
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DSA_ERR_CUDA;
  static std::atomic<int> sm_count[64];
  static std::atomic<bool> attr_set[64];
  int sms = sm_count[dev].load(std::memory_order_acquire);
  if (sms == 0) {
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1)
      return DSA_ERR_CUDA;
    sm_count[dev].store(sms, std::memory_order_release);
  }
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(dsa::topk::topk_slots_kernel<true, 1>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             dsa::topk::kCapKeys * 4) != cudaSuccess ||
        cudaFuncSetAttribute(dsa::topk::topk_slots_kernel<true, 2>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             dsa::topk::kCapKeysPart * 4) != cudaSuccess)
      return DSA_ERR_CUDA;
    attr_set[dev].store(true, std::memory_order_release);
  }
  if (num_rows * 2 <= sms && max_len > dsa::topk::kPartsMinLen) {
    const int per_cta = (max_len >> 1) + 4;  // the larger half of a row, rounded up
    return per_cta <= dsa::topk::kCapKeysPart
               ? dsa::topk::launch<true, 2>(p, num_rows, (size_t)per_cta * 4, st)
               : dsa::topk::launch<false, 2>(p, num_rows, 0, st);
  }
  return max_len <= dsa::topk::kCapKeys
             ? dsa::topk::launch<true, 1>(p, num_rows, (size_t)max_len * 4, st)
             : dsa::topk::launch<false, 1>(p, num_rows, 0, st);
}

extern "C" int dsa_union_groups(const int32_t* positions, int64_t positions_stride_b,
                                int64_t num_tokens, int32_t k, int32_t group,
                                const int32_t* page_table, int64_t page_table_stride_g,
                                int32_t page_table_cols, int32_t page_size, int32_t* slots,
                                uint8_t* member, int64_t out_stride_g, int32_t out_cols,
                                int32_t* counts, void* stream) {
  if (num_tokens < 0 || k < 1 || group < 1 || group > 8 || out_cols < 1 ||
      num_tokens % group != 0 || num_tokens / group > INT32_MAX)
    return DSA_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return DSA_OK;
  if (!positions || !page_table || !slots || !member) return DSA_ERR_INVALID_ARGUMENT;
  if (positions_stride_b < k || out_stride_g < out_cols || page_table_cols < 1 ||
      page_table_stride_g < page_table_cols || page_size < 1 || page_size > (1 << 20) ||
      (page_size & (page_size - 1)) != 0)
    return DSA_ERR_INVALID_ARGUMENT;
  dsa::topk::UnionParams p;
  p.pos = positions;
  p.pos_sb = positions_stride_b;
  p.k = k;
  p.group = group;
  p.pt = page_table;
  p.pt_sb = page_table_stride_g;
  p.pt_cols = page_table_cols;
  p.pg_shift = 0;
  while ((1 << p.pg_shift) < page_size) ++p.pg_shift;
  p.max_pos = (int64_t)page_table_cols * page_size;
  p.slots = slots;
  p.member = member;
  p.out_sb = out_stride_g;
  p.out_cols = out_cols;
  p.counts = counts;
  constexpr int kSmem = dsa::topk::kWinWords * 4;
  // the shared-memory limit is a per-device function attribute: set once per device (not
  // inside a stream capture when the first call ran eagerly)
  static std::atomic<bool> attr_set[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return DSA_ERR_CUDA;
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    if (cudaFuncSetAttribute(dsa::topk::union_groups_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
      return DSA_ERR_CUDA;
    attr_set[dev].store(true, std::memory_order_release);
  }
  dsa::topk::union_groups_kernel<<<(unsigned)(num_tokens / group), dsa::topk::kThreads, kSmem,
                                   static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}
