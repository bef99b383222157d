/*
 * dsa_b200.h -- C ABI of the B200 (sm_100a) DeepSeek sparse-attention (DSA)
 * sparse-MLA decode operator.
 *
 * This ABI is the native slot the reference leaves empty: the reference's CUDA
 * solution directory holds only an empty `__global__ void kernel()` template
 * (solution/cuda/kernel.cu:13) and an empty TVM-FFI binding registered as
 * "flashinfer.kernel" (solution/cuda/binding.py:11-25).  The Python entry point
 * the reference actually runs is the destination-passing
 *     kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale,
 *            output, lse)
 * of solution/triton/fused.py:150-180 (same signature in
 * solution/triton/baseline.py:12 and solution/cutedsl/kernel.py:148).
 * dsa_sparse_mla_decode() below is that call with the tensors lowered to
 * plain device pointers, element strides and sizes.
 *
 * Conventions (all functions):
 *   - pointers are CUDA device pointers on the current device unless noted;
 *   - strides are in ELEMENTS; the innermost dimension is contiguous;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *   - calls are asynchronous with respect to the host and return a status code
 *     (DSA_OK == 0); no function traps or asserts on the device.
 */
#ifndef DSA_B200_H_
#define DSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes returned by every entry point. */
enum {
  DSA_OK = 0,
  DSA_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad stride */
  DSA_ERR_UNSUPPORTED = 2,      /* head count / shape this build does not support */
  DSA_ERR_MISALIGNED = 3,       /* pointer or stride violates the 16-byte TMA rule */
  DSA_ERR_WORKSPACE = 4,        /* workspace missing or smaller than required */
  DSA_ERR_CUDA = 5,             /* a CUDA runtime call or the launch failed */
  DSA_ERR_DRIVER = 6,           /* cuTensorMapEncodeTiled unavailable / rejected */
  DSA_ERR_SCRATCH_LIMIT = 7     /* dsa_sparse_mla_decode_noalloc: over its fixed scratch */
};

/* Bits of the sticky device error word kept in the workspace. */
enum {
  DSA_DEVERR_BAD_INDEX = 1u, /* an index < -1 or >= num_slots was seen; treated as padding */
  DSA_DEVERR_TIMEOUT = 2u    /* a wait ran past its bound; the CTA stopped early, and a
                                split row whose merge gave up was written as NaN */
};

/*
 * Sparse-MLA decode, destination-passing style.
 * Replaces: fused.py:150-180 `kernel(...)` (and baseline.py:12 for any head count).
 *
 *   q_nope     [num_tokens, num_heads, 512] bf16, strides (q_nope_stride_b, q_nope_stride_h, 1)
 *   q_pe       [num_tokens, num_heads, 64]  bf16, strides (q_pe_stride_b,   q_pe_stride_h,   1)
 *   ckv_cache  [num_slots, 512] bf16, row stride ckv_slot_stride  (the paged
 *              [num_pages, 64, 512] cache viewed as slots, fused.py:155)
 *   kpe_cache  [num_slots, 64]  bf16, row stride kpe_slot_stride  (fused.py:156)
 *   sparse_indices [num_tokens, topk] int32, row stride indices_stride_b;
 *              flat slot id = page * 64 + offset, -1 = padding (contributes 0)
 *   output     [num_tokens, num_heads, 512] bf16 (written)
 *   lse        [num_tokens, num_heads] fp32, base-2 log-sum-exp (written)
 *   workspace  device buffer of at least dsa_sparse_mla_decode_workspace_size()
 *              bytes (split-K partials and the error word); zero-fill it once
 *              before first use so that the error word starts clear.  Calls
 *              sharing a workspace must be ordered on one stream.
 *
 * num_heads must be 16, 32, 64 or 128; topk >= 1.  Base addresses and the
 * byte value of every row stride must be multiples of 16.  A concatenated
 * [num_slots, 576] cache is accepted by passing kpe_cache = ckv_cache + 512
 * with both slot strides 576.  A row whose indices are all -1 gets output 0
 * and lse -inf.
 */
int dsa_sparse_mla_decode(const void* q_nope, int64_t q_nope_stride_b, int64_t q_nope_stride_h,
                          const void* q_pe, int64_t q_pe_stride_b, int64_t q_pe_stride_h,
                          const void* ckv_cache, int64_t ckv_slot_stride,
                          const void* kpe_cache, int64_t kpe_slot_stride, int64_t num_slots,
                          const int32_t* sparse_indices, int64_t indices_stride_b,
                          float sm_scale, void* output, int64_t output_stride_b,
                          int64_t output_stride_h, float* lse, int64_t lse_stride_b,
                          int64_t lse_stride_h, int64_t num_tokens, int32_t num_heads,
                          int32_t topk, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The same decode with the index production step fused into the gather: the caller
 * passes each row's token positions and page table instead of flat slot ids, and the
 * kernel forms slot = page_table[row][pos / page_size] * page_size + pos % page_size
 * as it fetches the slots, so the slot ids never travel through HBM.  Replaces the
 * caller-side step that builds `sparse_indices` for the reference's entry point
 * (fused.py:150; its pools are flattened as page * 64 + offset at fused.py:155-156 and
 * baseline.py:17-23); the reference has no such entry point.
 *
 *   page_table [num_tokens, >= page_table_cols] int32, row stride page_table_stride_b:
 *              row b lists the pool pages of row b's sequence in order
 *   positions  [num_tokens, topk] int32, row stride positions_stride_b: token
 *              positions within the row's sequence, -1 = padding
 *   page_size  the pool's page size (a power of two; 64 for the reference's pools)
 *
 * A position < -1 or past the row's table (pos / page_size >= page_table_cols), or one
 * whose page id is negative, is treated as padding and sets DSA_DEVERR_BAD_INDEX, like
 * an out-of-range slot id.  Other arguments as for dsa_sparse_mla_decode().
 */
int dsa_sparse_mla_decode_paged(
    const void* q_nope, int64_t q_nope_stride_b, int64_t q_nope_stride_h, const void* q_pe,
    int64_t q_pe_stride_b, int64_t q_pe_stride_h, const void* ckv_cache, int64_t ckv_slot_stride,
    const void* kpe_cache, int64_t kpe_slot_stride, int64_t num_slots, const int32_t* page_table,
    int64_t page_table_stride_b, int32_t page_table_cols, int32_t page_size,
    const int32_t* positions, int64_t positions_stride_b, float sm_scale, void* output,
    int64_t output_stride_b, int64_t output_stride_h, float* lse, int64_t lse_stride_b,
    int64_t lse_stride_h, int64_t num_tokens, int32_t num_heads, int32_t topk, void* workspace,
    size_t workspace_bytes, void* stream);

/*
 * Index production: per-row top-k of index scores, written as the slot ids the decode takes.
 * Replaces the caller-side step that builds `sparse_indices` for the reference's entry
 * point (fused.py:150; its callers pass slot = page * 64 + offset of the selected token
 * positions, baseline.py:17-23); the reference has no such kernel, and the published
 * definition of the step is flashinfer's top_k_page_table_transform (top k of
 * input[i, :lengths[i]], translated through the row's page table).
 *
 *   scores     [num_rows, >= max_len] fp32, row stride scores_stride_b: index scores of
 *              the row's token positions
 *   lengths    [num_rows] int32: row b selects among positions [0, min(lengths[b], max_len))
 *   page_table [num_rows, >= page_table_cols] int32 as for dsa_sparse_mla_decode_paged
 *   slots      [num_rows, >= k] int32 (written), row stride slots_stride_b
 *
 * Row b gets the slots of its k largest scores (ties at the k-th largest go to the smaller
 * positions; scores are ordered by their IEEE-754 bit pattern: -0.0 below +0.0, NaN below
 * every number), in ascending position order, then -1 up to k when the row has fewer than
 * k positions.  A position past the row's table or on a negative page gives -1.  With
 * page_table NULL the selected positions themselves are written (page_table_cols and
 * page_size are then ignored).  The result is exact and deterministic.  One launch on
 * `stream`; nothing is allocated.
 */
int dsa_topk_slots(const float* scores, int64_t scores_stride_b, const int32_t* lengths,
                   const int32_t* page_table, int64_t page_table_stride_b,
                   int32_t page_table_cols, int32_t page_size, int64_t num_rows,
                   int32_t max_len, int32_t k, int32_t* slots, int64_t slots_stride_b,
                   void* stream);

/*
 * Multi-token rows (prefill chunks, multi-token decode) decoded in token groups.
 *
 * The reference's operator takes one row per token (fused.py:150; the definition counts
 * num_tokens, each with its own selection), so consecutive tokens of one sequence gather
 * the slots they both selected once each.  A token group of G = 128 / num_heads
 * consecutive tokens of one sequence is decoded here as one 128-head row over the union
 * of the tokens' selections: each union entry is gathered once for all G tokens, and a
 * membership byte per entry (bit j: token j of the group selected it) masks the other
 * tokens' heads.  Every token's output equals the decode of its own selection
 * (baseline.py:17-45) up to floating-point summation order.
 *
 * dsa_union_groups builds the union: positions [num_tokens, >= k] int32 (row stride
 * positions_stride_b; each token's selected positions, distinct, -1 = none; the output of
 * dsa_topk_slots with page_table NULL) -> per group g = tokens [g G, (g + 1) G):
 *   slots  [num_tokens / G, >= out_cols] int32 (row stride out_stride_g): the slot ids of
 *          the union's positions, ascending by position, translated through the group's
 *          page table row (page_table [num_tokens / G, >= page_table_cols], page_size a
 *          power of two; a position past the table or on a negative page becomes -1),
 *          then -1;
 *   member [num_tokens / G, >= out_cols] uint8 (same row stride): the membership bytes,
 *          0 after the union;
 *   counts [num_tokens / G] int32 (optional, may be NULL): the union sizes.  A union
 *          larger than out_cols is cut at out_cols (counts shows it); out_cols =
 *          min(G * k, page_table_cols * page_size) always suffices.
 * 1 <= G <= 8.  Positions < 0 or >= page_table_cols * page_size are not part of the union.
 * One launch (one CTA per group) on `stream`; nothing is allocated.
 *
 * dsa_sparse_mla_decode_grouped decodes num_tokens tokens of num_heads (16, 32 or 64)
 * heads as num_tokens / G rows of 128 heads: union_indices and member as written by
 * dsa_union_groups (union_cols entries per group, row stride union_stride_g for both).
 * Arguments otherwise as dsa_sparse_mla_decode, with every token's heads consecutive in
 * q_nope, q_pe, output and lse (stride_b = num_heads * stride_h; output and its strides
 * 16-byte aligned); num_tokens a multiple of G.  A token with no member entry gets
 * output 0 and lse -inf, like an all-padding row.
 */
int dsa_union_groups(const int32_t* positions, int64_t positions_stride_b, int64_t num_tokens,
                     int32_t k, int32_t group, const int32_t* page_table,
                     int64_t page_table_stride_g, int32_t page_table_cols, int32_t page_size,
                     int32_t* slots, uint8_t* member, int64_t out_stride_g, int32_t out_cols,
                     int32_t* counts, void* stream);

int dsa_sparse_mla_decode_grouped(
    const void* q_nope, int64_t q_nope_stride_b, int64_t q_nope_stride_h, const void* q_pe,
    int64_t q_pe_stride_b, int64_t q_pe_stride_h, const void* ckv_cache, int64_t ckv_slot_stride,
    const void* kpe_cache, int64_t kpe_slot_stride, int64_t num_slots,
    const int32_t* union_indices, const uint8_t* member, int64_t union_stride_g,
    int32_t union_cols, float sm_scale, void* output, int64_t output_stride_b,
    int64_t output_stride_h, float* lse, int64_t lse_stride_b, int64_t lse_stride_h,
    int64_t num_tokens, int32_t num_heads, void* workspace, size_t workspace_bytes,
    void* stream);

/*
 * Bytes of workspace dsa_sparse_mla_decode() needs for this problem on
 * `device` (split-K partials and the error word; the size depends only on
 * the device's SM count, so one workspace serves every shape).
 * Returns 0 for an unsupported shape.  No counterpart in the reference (its
 * kernels hold no split-K state); fused.py:148 documents that it allocates
 * nothing per call, which the caller-owned workspace preserves.
 */
size_t dsa_sparse_mla_decode_workspace_size(int64_t num_tokens, int32_t num_heads, int32_t topk,
                                            int32_t device);

/*
 * Reads the sticky device error word (DSA_DEVERR_* bits) of `workspace` after
 * synchronizing `stream`; clears it when `clear` is non-zero.  Host pointer
 * `word` receives the value.  No counterpart in the reference (its kernels do
 * no index checking: fused.py:89-91 only maps -1 to slot 0).
 */
int dsa_read_error_word(void* workspace, void* stream, int clear, uint32_t* word);

/*
 * Sets the bound of every wait inside the decode kernels (pipeline barriers and the
 * split-K merge's wait for the other parts of a row) to `cycles` SM clock cycles for
 * launches that follow; 0 restores the default of 4e9 cycles (about 2 s at the B200's
 * ~2 GHz clock).  Returns the previous bound.  A wait that runs out sets
 * DSA_DEVERR_TIMEOUT, and a split row whose merge gave up is written as NaN (output and
 * lse).  Process-wide; a diagnostic for tests of the timeout path, which shorten the
 * bound.  No counterpart in the reference (its kernels do not wait on one another).
 */
uint64_t dsa_set_wait_limit(uint64_t cycles);

/*
 * Failure-detection self test: launches one CTA that waits on an mbarrier no
 * one arrives at, bounded by `timeout_ns` (counted as 2 SM clock cycles per ns,
 * i.e. about `timeout_ns` at the B200's ~2 GHz clock; the decode kernels bound
 * every wait the same way, at about 2 s), then records DSA_DEVERR_TIMEOUT in
 * the workspace error word and returns.  Lets a test check the bounded-wait
 * path without faulting or hanging the GPU.  No counterpart in the reference.
 */
int dsa_selftest_bounded_wait(int64_t timeout_ns, void* workspace, void* stream);

/*
 * The same decode for callers that cannot allocate device memory (code running under
 * another framework's allocator, a host application that forbids cudaMalloc on its
 * decode path, a process whose device footprint must not grow after start-up).  No
 * counterpart in the reference: its entry point (fused.py:150) is called with outputs
 * preallocated and needs no scratch; this library's split-K partials normally live in
 * the caller's workspace.
 *
 * Arguments are those of dsa_sparse_mla_decode() without the workspace.  Instead of a
 * workspace the call uses a fixed 2 MiB array that the library's CUDA module holds on
 * every device that loads it, until the process exits; the call itself allocates
 * nothing (no cudaMalloc, cudaFree or allocating library routine).
 *   - The first call on a device resolves the array's device address (once per device,
 *     with that device current) and keeps it for later calls.  Do not use this entry
 *     point across cudaDeviceReset() on that device: the module may be reloaded at
 *     another address.
 *   - Limit: 8448 bytes of header and split-K counters, plus, when rows are split
 *     between cluster pairs of the persistent grid, one partial per pair (32,896 bytes
 *     for 16-head rows, 65,792 bytes for wider rows, which run as 32-head groups).  A
 *     call whose (row, head group) count is at most the number of two-CTA clusters the
 *     device runs at once (its persistent grid: half the SM count on a B200, 74 pairs on
 *     148 SMs, e.g. 74 rows of 16 heads or 64 rows of 32 heads) splits no row and always
 *     fits; a larger call runs split rows on every pair and needs 2.4 MB or more, beyond
 *     the array: it returns DSA_ERR_SCRATCH_LIMIT (use dsa_sparse_mla_decode).  The
 *     split path of this entry point is therefore reachable only on devices with fewer
 *     cluster pairs.
 *   - Every call on a device shares the array and finds the previous call's bytes there:
 *     the call clears the first 8448 bytes (error word and split-K arrival counters;
 *     device error bits are not reported by this entry point) and always writes the
 *     partials before reading them.  Calls that
 *     overlap on the GPU (different streams, or concurrent host threads) race on the
 *     array; order them on one stream.
 */
int dsa_sparse_mla_decode_noalloc(const void* q_nope, int64_t q_nope_stride_b,
                                  int64_t q_nope_stride_h, const void* q_pe,
                                  int64_t q_pe_stride_b, int64_t q_pe_stride_h,
                                  const void* ckv_cache, int64_t ckv_slot_stride,
                                  const void* kpe_cache, int64_t kpe_slot_stride,
                                  int64_t num_slots, const int32_t* sparse_indices,
                                  int64_t indices_stride_b, float sm_scale, void* output,
                                  int64_t output_stride_b, int64_t output_stride_h, float* lse,
                                  int64_t lse_stride_b, int64_t lse_stride_h, int64_t num_tokens,
                                  int32_t num_heads, int32_t topk, void* stream);

/* Human-readable text of a status code (static storage). */
const char* dsa_status_string(int status);

/* ABI version: bumped when a signature above changes. */
int dsa_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* DSA_B200_H_ */
