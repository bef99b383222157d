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
// One CTA per row (1024 threads).  Scores are mapped to order-preserving 32-bit keys; a
// radix select finds the k-th largest key T in three histogram passes over 12, 12 and 8 key
// bits (each later pass only over the keys that share the bits already fixed); a counting
// pass and an ordered compaction pass then write every position with key > T and the
// first ones with key == T.  Each warp owns one contiguous segment of the row and reads it
// coalesced, so positions come out in order without a sort.
#include <cuda_runtime.h>
#include <stdint.h>

#include "dsa_b200.h"

namespace dsa {
namespace topk {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kBins = 4096;

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

// Given the histogram `hist[nbins]` of the candidate keys and `need` (>= 1) elements still to
// take from the top, the bin holding the need-th largest candidate and how many of the
// candidates in higher bins are taken (through *above).  Thread t owns bins
// [nbins - (t + 1) * per, nbins - t * per), scanned from the top.
__device__ __forceinline__ int select_bin(const uint32_t* hist, int nbins, uint32_t need,
                                          uint32_t* wsum, uint32_t* above, int* bin_out) {
  const int per = nbins / kThreads > 0 ? nbins / kThreads : 1;
  const int hi = nbins - threadIdx.x * per;  // exclusive
  uint32_t mine = 0;
  if (hi > 0)
    for (int b = hi - 1; b >= hi - per && b >= 0; --b) mine += hist[b];
  const uint32_t incl = block_inclusive_scan(mine, wsum);  // count in bins >= hi - per
  const uint32_t excl = incl - mine;                       // count in bins >= hi
  if (hi > 0 && excl < need && incl >= need) {
    uint32_t acc = excl;
    for (int b = hi - 1; b >= hi - per; --b) {
      if (acc + hist[b] >= need) {
        *bin_out = b;
        *above = acc;
        break;
      }
      acc += hist[b];
    }
  }
  __syncthreads();
  return *bin_out;
}

__global__ void __launch_bounds__(kThreads, 1) topk_slots_kernel(const Params p) {
  __shared__ uint32_t hist[kBins];
  __shared__ uint32_t wsum[32];
  __shared__ uint32_t above_s;
  __shared__ int bin_s;
  __shared__ uint32_t wcount[2][kWarps];  // per warp: keys > T, keys == T
  const int row = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* sr = p.scores + (int64_t)row * p.scores_sb;
  const int32_t* pr = p.pt + (int64_t)row * p.pt_sb;
  int32_t* out = p.slots + (int64_t)row * p.slots_sb;
  int L = __ldg(p.lengths + row);
  L = L < 0 ? 0 : (L > p.max_len ? p.max_len : L);
  const int k = p.k;

  if (L <= k) {  // every position, in order, then padding
    for (int i = threadIdx.x; i < k; i += kThreads) out[i] = i < L ? slot_of(p, pr, i) : -1;
    return;
  }

  // ---- radix select of the k-th largest key: bits [31:20], [19:8], [7:0]
  uint32_t prefix = 0, need = (uint32_t)k;
  const int shifts[3] = {20, 8, 0};
  const int nbins[3] = {4096, 4096, 256};
  for (int pass = 0; pass < 3; ++pass) {
    for (int b = threadIdx.x; b < kBins; b += kThreads) hist[b] = 0u;
    __syncthreads();
    const int sh = shifts[pass];
    const uint32_t bmask = (uint32_t)nbins[pass] - 1u;
    const int hsh = sh + (pass == 0 ? 12 : (pass == 1 ? 12 : 8));  // bits above this digit
    // every lane of a warp runs every iteration (the loop bound is uniform), so the match
    // below always has the full warp; lanes past the row or outside the prefix take no bin
    for (int base = 0; base < L; base += kThreads) {
      const int i = base + threadIdx.x;
      uint32_t bin = 0xFFFFFFFFu;
      if (i < L) {
        const uint32_t key = score_key(__ldg(sr + i));
        if (pass == 0 || (key >> hsh) == prefix) bin = (key >> sh) & bmask;
      }
      // one atomic per distinct bin of the warp
      const uint32_t peers = __match_any_sync(0xffffffffu, bin);
      if (bin != 0xFFFFFFFFu && (__ffs(peers) - 1) == lane)
        atomicAdd(&hist[bin], (uint32_t)__popc(peers));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      bin_s = -1;
      above_s = 0u;
    }
    __syncthreads();
    const int b = select_bin(hist, nbins[pass], need, wsum, &above_s, &bin_s);
    need -= above_s;
    prefix = (prefix << (pass == 2 ? 8 : 12)) | (uint32_t)b;
    __syncthreads();
  }
  const uint32_t T = prefix;  // the k-th largest key; `need` keys equal to T are taken

  // ---- counting pass: each warp owns a contiguous segment of the row
  const int seg = (L + kWarps - 1) / kWarps;
  const int s0 = warp * seg, s1 = min(L, s0 + seg);
  uint32_t gt = 0, eq = 0;
  for (int i = s0 + lane; i < s1; i += 32) {
    const uint32_t key = score_key(__ldg(sr + i));
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
  uint32_t gt_before = 0, eq_before = 0;
  for (int w = 0; w < warp; ++w) {
    gt_before += wcount[0][w];
    eq_before += wcount[1][w];
  }
  // ---- ordered compaction: keys > T, and keys == T while fewer than `need` were taken
  uint32_t pos_out = gt_before + min(eq_before, need);
  uint32_t eq_seen = eq_before;
  for (int base = s0; base < s1; base += 32) {
    const int i = base + lane;
    const uint32_t key = i < s1 ? score_key(__ldg(sr + i)) : 0u;
    const bool is_eq = i < s1 && key == T;
    const uint32_t eq_mask = __ballot_sync(0xffffffffu, is_eq);
    const uint32_t eq_rank = eq_seen + __popc(eq_mask & ((1u << lane) - 1u));
    const bool take = i < s1 && (key > T || (is_eq && eq_rank < need));
    const uint32_t take_mask = __ballot_sync(0xffffffffu, take);
    if (take) out[pos_out + __popc(take_mask & ((1u << lane) - 1u))] = slot_of(p, pr, i);
    pos_out += __popc(take_mask);
    eq_seen += __popc(eq_mask);
  }
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
  if (!scores || !lengths || !page_table || !slots) return DSA_ERR_INVALID_ARGUMENT;
  if (scores_stride_b < max_len || slots_stride_b < k || page_table_cols < 1 ||
      page_table_stride_b < page_table_cols)
    return DSA_ERR_INVALID_ARGUMENT;
  if (page_size < 1 || page_size > (1 << 20) || (page_size & (page_size - 1)) != 0)
    return DSA_ERR_INVALID_ARGUMENT;
  dsa::topk::Params p;
  p.scores = scores;
  p.scores_sb = scores_stride_b;
  p.lengths = lengths;
  p.pt = page_table;
  p.pt_sb = page_table_stride_b;
  p.pt_cols = page_table_cols;
  p.pg_shift = 0;
  while ((1 << p.pg_shift) < page_size) ++p.pg_shift;
  p.max_len = max_len;
  p.k = k;
  p.slots = slots;
  p.slots_sb = slots_stride_b;
  dsa::topk::topk_slots_kernel<<<(unsigned)num_rows, dsa::topk::kThreads, 0,
                                 static_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}
