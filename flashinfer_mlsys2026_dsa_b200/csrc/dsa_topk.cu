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
// radix select finds the k-th largest key T in four histogram passes over the key's bytes,
// high to low (each later pass only over the keys that share the bytes already fixed), with
// one 256-bin histogram per warp so that warps never contend for a counter; a counting pass
// and an ordered compaction pass then write every position with key > T and the first
// ones with key == T.  Each warp owns one contiguous segment of the row and reads it
// coalesced, so positions come out in order without a sort.
#include <cuda_runtime.h>
#include <stdint.h>

#include "dsa_b200.h"

namespace dsa {
namespace topk {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kBins = 256;  // one key byte per pass

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

// Given the histogram `hist[kBins]` of the candidate keys' current byte and `need` (>= 1)
// elements still to take from the top, the bin holding the need-th largest candidate, and
// through *above how many candidates lie in higher bins.  Thread t < kBins owns bin
// kBins - 1 - t (so the scan runs from the top bin down).
__device__ __forceinline__ int select_bin(const uint32_t* hist, uint32_t need, uint32_t* wsum,
                                          uint32_t* above, int* bin_out) {
  const int b = kBins - 1 - (int)threadIdx.x;
  const uint32_t mine = b >= 0 ? hist[b] : 0u;
  const uint32_t incl = block_inclusive_scan(mine, wsum);  // candidates in bins >= b
  const uint32_t excl = incl - mine;                       // candidates in bins > b
  if (b >= 0 && excl < need && incl >= need) {
    *bin_out = b;
    *above = excl;
  }
  __syncthreads();
  return *bin_out;
}

__global__ void __launch_bounds__(kThreads, 1) topk_slots_kernel(const Params p) {
  __shared__ uint32_t whist[kWarps][kBins];  // per-warp histograms of the current key byte
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

  // ---- radix select of the k-th largest key, one key byte per pass (bits 31..24 first)
  uint32_t prefix = 0, need = (uint32_t)k;
  uint32_t* wh = whist[warp];
  for (int pass = 0; pass < 4; ++pass) {
    const int sh = 24 - 8 * pass;
    for (int j = lane; j < kBins; j += 32) wh[j] = 0u;
    __syncwarp();
    for (int i = threadIdx.x; i < L; i += kThreads) {
      const uint32_t key = score_key(__ldg(sr + i));
      // pass 0 takes every key; later passes the keys whose higher bytes equal the prefix
      if (pass == 0 || (key >> (sh + 8)) == prefix) atomicAdd(&wh[(key >> sh) & 0xFFu], 1u);
    }
    __syncthreads();
    if (threadIdx.x < kBins) {
      uint32_t c = 0;
#pragma unroll 8
      for (int w = 0; w < kWarps; ++w) c += whist[w][threadIdx.x];
      hist[threadIdx.x] = c;
    }
    if (threadIdx.x == 0) {
      bin_s = -1;
      above_s = 0u;
    }
    __syncthreads();
    const int b = select_bin(hist, need, wsum, &above_s, &bin_s);
    need -= above_s;
    prefix = (prefix << 8) | (uint32_t)b;
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
