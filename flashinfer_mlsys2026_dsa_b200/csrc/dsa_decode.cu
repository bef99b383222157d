// B200 (sm_100a) DeepSeek sparse-attention decode: one persistent kernel per call.
//
// Math (the reference PyTorch path, solution/triton/baseline.py:12-45):
//   for each decode row b and head h over the topk selected slots k:
//     z[h,k]  = sm_scale * (q_nope[b,h] . ckv[idx[b,k]] + q_pe[b,h] . kpe[idx[b,k]])
//     z[h,k]  = -inf where idx[b,k] == -1
//     lse[b,h] = log2(sum_k exp(z[h,k]))
//     out[b,h] = bf16(sum_k softmax(z)[h,k] * ckv[idx[b,k]])
//
// Design (B200-first, not a translation of the Triton kernel fused.py:26-144):
//   * Work = (row, head-group, 64-slot tile) units laid out row-major; each CTA of a
//     persistent grid (one CTA per SM) takes a contiguous, equal share of units
//     (stream-K).  A row cut between CTAs leaves one partial (unnormalised O, running
//     max, sum) per CTA; a second small kernel merges them (LSE-weighted).  Merging
//     inside the decode kernel would put several dependent global round trips on
//     the tail of the merging CTA while the gathers of the others load the memory
//     system.
//   * Warp 0 loads each segment's Q.  Warps 1-3, 5-7, 9-11 (producers): per 64-slot
//     tile, read the slot ids and issue 144 TMA tile::gather4 loads (4 slots x 128 B each) of the 512-d ckv rows and the
//     64-d kpe rows into a 128-byte-swizzled shared-memory stage, the loads dealt
//     over all nine warps (one warp issues them too slowly) and completing on one
//     mbarrier per d-block; a -1 slot is requested as an
//     out-of-range row, which reads nothing from HBM.  Tiles with no valid slot skip
//     both MMAs; in other tiles the softmax warps clear a padded slot's value row so
//     that its P == 0 contributes exactly zero.
//   * Warp 4 (MMA issuer, one thread): score S^T[slots x NHC heads] = K . Q^T with
//     tcgen05.mma (M=64, K=576 as 36 k-steps, each d-block as soon as it lands) into
//     TMEM, then after softmax the
//     output O^T[512 d x NHC heads] += V^T . P^T (M=128 x 4 d-tiles, V read from the
//     same stage as an MN-major operand) into TMEM.
//   * Warps 12-15 (softmax + epilogue, given most of the register file): tcgen05.ld the scores, base-2 online softmax
//     with a lazily-updated running max (the accumulator is rescaled only when a
//     score exceeds the running max by more than kTau), write bf16 P^T to shared
//     memory, and at a segment's end read O from TMEM and write the output or a
//     partial.
//   * Heads are split into groups of NHC = min(H, 64) per unit (H = 128 -> 2 groups).
//
// Every mbarrier wait is bounded (Waiter); on timeout the CTA records
// DSA_DEVERR_TIMEOUT, stops issuing work and exits after its copies land.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>
#include <utility>

#include "dsa_b200.h"
#include "sm100_ptx.cuh"

namespace dsa {

constexpr int kDCkv = 512;            // latent (value) width
constexpr int kDKpe = 64;             // rope key width
constexpr int kBK = 56;               // slots per tile (the score MMA is M=64; its last 8
                                      // rows read the next 1 KB and are never used)
constexpr int kMRows = 64;            // M of the score MMA = rows of P per tile
constexpr int kGroups = kBK / 4;      // gather4 groups per d-block
constexpr int kNDB = 9;               // 64-element d-blocks: 8 ckv + 1 kpe
constexpr int kRegion = kBK * 128;    // bytes of one d-block of a stage
constexpr int kStageBytes = kNDB * kRegion;
constexpr int kUnits = kGroups * kNDB;    // gather4 copies per tile
constexpr int kPVSteps = kMRows / 16;     // K steps of the PV MMA (rows >= kBK carry P == 0)
constexpr int kPVSplit = 5;               // d-block of score(i) before which PV(i-1) is issued
constexpr int kThreads = 512;         // four warpgroups
constexpr int kQWarp = 0;             // loads Q (one TMA box per d-block and segment)
constexpr int kProducerWarps = 9;     // warps 1-3, 5-7 and 9-11 issue the gathers
constexpr int kMmaWarp = 4;           // sub-partition 0 (warps 0, 4, 8, 12) issues no gathers
constexpr int kIdleWarp = 8;
constexpr int kSmWarp0 = 12;          // warps 12-15: softmax / epilogue
constexpr int kSmThreads = 128;
constexpr uint32_t kNamedBar = 1;
constexpr uint32_t kRegsLow = 80;     // producer / MMA warpgroups after the split
constexpr uint32_t kRegsHigh = 248;   // softmax warpgroup after the split
constexpr float kTau = 8.0f;          // lazy-rescale threshold (log2 units)
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint64_t kWaitCycles = 4000000000ull;  // ~2 s at the B200's ~2 GHz SM clock
static_assert(kProducerWarps * 32 >= kUnits, "one gather per producer lane per tile");
static_assert(kBK % 8 == 0 && kBK <= 64, "tile rows: whole 8-row swizzle atoms, 64-bit masks");

template <int NHC>
struct Cfg {
  static constexpr int STAGES = (NHC == 16) ? 3 : 2;
  static constexpr int QBUF = (NHC == 32) ? 2 : 1;
  static constexpr int PBUF = 2;
  // With three stages the MMA issuer runs score(i+1) before PV(i) so that the tensor
  // core is not idle during softmax(i); with two, PV(i) follows score(i) at once so that
  // each stage is handed back as early as possible.
  static constexpr bool OVERLAP = STAGES >= 3;
  static constexpr int Q_REGION = NHC * 128;
  static constexpr int Q_BYTES = kNDB * Q_REGION;
  static constexpr int P_BYTES = NHC * 128;  // P^T [NHC x 64] bf16
  static constexpr int OFF_KV = 0;
  static constexpr int OFF_Q = OFF_KV + STAGES * kStageBytes;
  static constexpr int OFF_P = OFF_Q + QBUF * Q_BYTES;
  static constexpr int OFF_BAR = OFF_P + PBUF * P_BYTES;
  static constexpr int OFF_MASK = OFF_BAR + 512;
  static constexpr int OFF_MISC = OFF_MASK + 256;
  static constexpr int OFF_RED = OFF_MISC + 64;
  static constexpr int SMEM_USED = OFF_RED + 4 * NHC * 4;
  static constexpr int SMEM_BYTES = SMEM_USED + 1024;  // slack to 1024-align the base
  static constexpr int O_COL = 0;                        // 4 d-tiles x NHC columns
  static constexpr int S_COL = 4 * NHC;                  // 2 score buffers x NHC columns
  static constexpr int TMEM_COLS = (6 * NHC <= 32)    ? 32
                                   : (6 * NHC <= 64)  ? 64
                                   : (6 * NHC <= 128) ? 128
                                   : (6 * NHC <= 256) ? 256
                                                      : 512;
  static constexpr int SLOT_FLOATS = NHC * kDCkv + 2 * NHC;  // partial O, m, l
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(STAGES * kProducerWarps * 8 <= 256, "mask words");
  static_assert(OFF_Q % 1024 == 0 && OFF_P % 1024 == 0, "swizzle atoms need 1024-B alignment");
};

// Barrier slots (8 bytes each) inside the OFF_BAR block.
// Per stage: B_META (the producers' slot masks are written) and one B_KVF per d-block,
// so that the score MMAs of d-block j can start as soon as its 8 KB have landed.
enum : int {
  B_META = 0, B_KVF = 4, B_KVE = 40, B_QF = 44, B_QE = 46, B_SF = 48, B_SE = 50, B_PF = 52,
  B_PD = 54,
  B_DRAIN = 56  // used only when the MMA issuer stops early
};
__host__ __device__ constexpr int kvf(int stage, int j) { return B_KVF + stage * kNDB + j; }

struct Params {
  const int32_t* idx;
  int64_t idx_sb;
  __nv_bfloat16* out;
  int64_t out_sb, out_sh;
  float* lse;
  int64_t lse_sb, lse_sh;
  int64_t num_slots;
  int64_t units;  // num_rh * tpr
  int32_t hg_count;
  int32_t topk;
  int32_t tpr;    // tiles per (row, head-group)
  float scale_log2;
  uint32_t* err;
  float* parts;
  uint32_t* counters;  // split-K arrival counters (16-head kernel), zero between calls
};

// UMMA shared-memory descriptor, 128-byte swizzle, sm_100 (version 1).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16: bf16 A/B, fp32 D.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Byte offset of element (row h, column k) in a [rows x 64] bf16 tile stored
// K-major with the 128-byte swizzle (the UMMA canonical SW128 K-major layout).
__device__ __forceinline__ uint32_t sw128_off(int h, int k) {
  return (uint32_t)((h >> 3) * 1024 + (h & 7) * 128 + ((((k >> 3) ^ (h & 7))) << 4) + (k & 7) * 2);
}

// Bounded mbarrier wait.  `spin` polls without letting the hardware suspend the thread
// (for the latency-critical MMA issuer); otherwise try_wait may suspend it briefly.
struct Waiter {
  volatile uint32_t* abort_flag;
  uint32_t* err;
  bool spin = false;
  __device__ __forceinline__ bool poll(uint32_t bar, uint32_t parity) const {
    return spin ? ptx::mbar_test_wait(bar, parity) : ptx::mbar_try_wait(bar, parity);
  }
  __device__ __forceinline__ bool operator()(uint32_t bar, uint32_t parity) const {
    if (poll(bar, parity)) return true;
    const uint64_t t0 = ptx::cycles();
    for (uint32_t it = 1;; ++it) {
      if (poll(bar, parity)) return true;
      if ((it & 63u) == 0) {
        if (*abort_flag) return false;
        if (ptx::cycles() - t0 > kWaitCycles) {
          *abort_flag = 1;
          atomicOr(err, (uint32_t)DSA_DEVERR_TIMEOUT);
          return false;
        }
      }
    }
  }
};

// CTA c owns units [u_begin(c), u_begin(c+1)).
__device__ __forceinline__ int64_t u_begin(int64_t c, int64_t units, int64_t G) {
  return (c * units) / G;
}
// The CTA whose range holds unit u.
__device__ __forceinline__ int64_t cta_of(int64_t u, int64_t units, int64_t G) {
  return ((u + 1) * G - 1) / units;
}

// Slot ids of tile `uu` (unit index) for a producer lane's group g; -1 past topk.
__device__ __forceinline__ void load_slot_ids(const Params& p, int64_t uu, bool has_unit, int g,
                                              int (&r)[4]) {
  const int64_t rh = uu / p.tpr;
  const int t = (int)(uu % p.tpr);
  const int32_t* idx_row = p.idx + (rh / p.hg_count) * p.idx_sb;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int k = t * kBK + 4 * g + q;
    r[q] = (has_unit && k < p.topk) ? __ldg(idx_row + k) : -1;
  }
}

struct Segment {
  int64_t rh;  // row * hg_count + head-group
  int t0, t1;  // tile range [t0, t1) within the row
};

__device__ __forceinline__ bool next_segment(int64_t& u, int64_t u1, int tpr, Segment& s) {
  if (u >= u1) return false;
  s.rh = u / tpr;
  s.t0 = (int)(u % tpr);
  const int64_t room = u1 - u;
  s.t1 = (int)((int64_t)s.t0 + room < (int64_t)tpr ? (int64_t)s.t0 + room : (int64_t)tpr);
  u += s.t1 - s.t0;
  return true;
}


// PV of tile `pi` (held in stage `pst`): O^T[512 x NHC] (+)= V^T . P^T, then hand the stage
// back and signal pv_done.  An all-padding tile (live == false) has P == 0 and skips the
// MMAs.  o_init tracks whether O already holds this segment's sum.
template <int NHC>
__device__ __forceinline__ bool issue_pv(const Waiter& wait, uint32_t bar0, uint32_t sbase,
                                         uint32_t tmem, int64_t pi, int pst, bool first,
                                         bool live, bool& o_init) {
  using C = Cfg<NHC>;
  constexpr uint32_t kIdescPV = idesc_bf16(128, NHC, true);
  if (!wait(bar0 + 8u * (uint32_t)(B_PF + (int)(pi & 1)), (uint32_t)((pi >> 1) & 1))) return false;
  ptx::tc_fence_after();
  if (first) o_init = false;
  if (live) {
    const uint32_t kv = sbase + (uint32_t)(C::OFF_KV + pst * kStageBytes);
    const uint32_t pb = sbase + (uint32_t)(C::OFF_P + (int)(pi % C::PBUF) * C::P_BYTES);
#pragma unroll
    for (int mt = 0; mt < 4; ++mt)
#pragma unroll
      for (int ks = 0; ks < kPVSteps; ++ks)
        ptx::umma_bf16(tmem + (uint32_t)(C::O_COL + mt * NHC),
                       sdesc(kv + (uint32_t)(2 * mt * kRegion + ks * 2048), kRegion, 1024),
                       sdesc(pb + (uint32_t)(ks * 32), 16, 1024), kIdescPV,
                       (o_init || ks > 0) ? 1u : 0u);
    o_init = true;
  }
  ptx::umma_commit(bar0 + 8u * (uint32_t)(B_KVE + pst));
  ptx::umma_commit(bar0 + 8u * (uint32_t)(B_PD + (int)(pi & 1)));
  return true;
}

template <int NHC>
__global__ void __launch_bounds__(kThreads, 1)
    dsa_decode_kernel(const __grid_constant__ CUtensorMap tm_ckv,
                      const __grid_constant__ CUtensorMap tm_kpe,
                      const __grid_constant__ CUtensorMap tm_qn,
                      const __grid_constant__ CUtensorMap tm_qp, const __grid_constant__ Params p) {
  using C = Cfg<NHC>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  const uint32_t sbase = (raw_addr + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - raw_addr);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(sgen + C::OFF_MISC);
  uint64_t* masks = reinterpret_cast<uint64_t*>(sgen + C::OFF_MASK);  // [STAGES][producer warp]
  float* red = reinterpret_cast<float*>(sgen + C::OFF_RED);
  const uint32_t bar0 = sbase + (uint32_t)C::OFF_BAR;
#define bar(k) (bar0 + 8u * (uint32_t)(k))

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      ptx::mbar_init(bar(B_META + s), kProducerWarps);
      for (int j = 0; j < kNDB; ++j) ptx::mbar_init(bar(kvf(s, j)), 1);
      ptx::mbar_init(bar(B_KVE + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar(B_QF + b), 1);
      ptx::mbar_init(bar(B_QE + b), 1);
      ptx::mbar_init(bar(B_SF + b), 1);
      ptx::mbar_init(bar(B_SE + b), kSmThreads);
      ptx::mbar_init(bar(B_PF + b), kSmThreads);
      ptx::mbar_init(bar(B_PD + b), 1);
    }
    ptx::mbar_init(bar(B_DRAIN), 1);
    misc[1] = 0;
    misc[2] = 0;
    misc[3] = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kQWarp && lane == 0) {
    ptx::prefetch_tmap(&tm_ckv);
    ptx::prefetch_tmap(&tm_kpe);
    ptx::prefetch_tmap(&tm_qn);
    ptx::prefetch_tmap(&tm_qp);
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(sbase + (uint32_t)C::OFF_MISC, (uint32_t)C::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = misc[0];
  // Launched with programmatic stream serialization: the set-up above overlapped the
  // previous grid's tail; nothing in global memory is touched before that grid is done.
  ptx::grid_dep_wait();
  ptx::launch_dependents();

  const int64_t G = gridDim.x;
  const int64_t u_lo = u_begin(blockIdx.x, p.units, G);
  const int64_t u_hi = u_begin((int64_t)blockIdx.x + 1, p.units, G);
  const Waiter wait{misc + 2, p.err};

  if (warp == kQWarp) {
    // ------------------------------------------------------------------ Q loader
    ptx::regs_dec<kRegsLow>();
    if (lane == 0) {
      int seg = 0;
      int64_t u = u_lo;
      Segment s;
      while (next_segment(u, u_hi, p.tpr, s)) {
        const int64_t b = s.rh / p.hg_count;
        const int hg = (int)(s.rh % p.hg_count);
        const int qb = seg % C::QBUF;
        if (!wait(bar(B_QE + qb), (uint32_t)(((seg / C::QBUF) & 1) ^ 1))) break;
        ptx::mbar_arrive_expect_tx(bar(B_QF + qb), (uint32_t)C::Q_BYTES);
        const uint32_t qdst = sbase + (uint32_t)(C::OFF_Q + qb * C::Q_BYTES);
        for (int jj = 0; jj < 8; ++jj)
          ptx::tma_load_3d(qdst + (uint32_t)(jj * C::Q_REGION), &tm_qn, 64 * jj, hg * NHC, (int)b,
                           bar(B_QF + qb));
        ptx::tma_load_3d(qdst + (uint32_t)(8 * C::Q_REGION), &tm_qp, 0, hg * NHC, (int)b,
                         bar(B_QF + qb));
        ++seg;
      }
      // Let the last Q copy land before the CTA can exit.
      if (seg > 0) {
        const Waiter drain{misc + 3, p.err};
        const int qb = (seg - 1) % C::QBUF;
        drain(bar(B_QF + qb), (uint32_t)(((seg - 1) / C::QBUF) & 1));
      }
    }
    __syncwarp();
  } else if (warp == kIdleWarp) {
    ptx::regs_dec<kRegsLow>();
  } else if (warp < kSmWarp0 && warp != kMmaWarp) {
    // ------------------------------------------------------------------ gather producers
    // Each tile is kUnits gather4 copies (kGroups groups of 4 slots x 9 d-blocks), ordered
    // d-block first and dealt round-robin over the producer warps, so that all warps
    // issue in parallel and d-block 0 lands first.
    ptx::regs_dec<kRegsLow>();
    const int pw = warp - 1 - (warp >> 2);
    const int unit = lane * kProducerWarps + pw;
    const bool has_unit = unit < kUnits;
    const int j = has_unit ? unit / kGroups : 0;  // d-block
    const int g = has_unit ? unit % kGroups : 0;  // slots 4g .. 4g+3 of the tile
    const uint64_t policy = ptx::policy_evict_first();
    bool ok = true;
    int64_t n_issued = 0;  // tiles whose copies this warp has issued
    int cur[4], nxt[4];
    if (u_lo < u_hi) load_slot_ids(p, u_lo, has_unit, g, cur);
    for (int64_t uu = u_lo, i = 0; uu < u_hi; ++uu, ++i) {
      // The next tile's ids are requested before this tile waits for its stage, so
      // their load latency overlaps the wait instead of adding to it.
      if (uu + 1 < u_hi) load_slot_ids(p, uu + 1, has_unit, g, nxt);
      const int stage = (int)(i % C::STAGES);
      uint64_t vbits = 0;
      bool bad = false;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (cur[q] < -1 || (int64_t)cur[q] >= p.num_slots) {
          bad = true;
          cur[q] = -1;
        }
        vbits |= (uint64_t)(cur[q] >= 0 ? 1u : 0u) << (4 * g + q);
      }
      if (bad) atomicOr(p.err, (uint32_t)DSA_DEVERR_BAD_INDEX);
      const uint64_t wmask =
          ((uint64_t)__reduce_or_sync(0xffffffffu, (uint32_t)(vbits >> 32)) << 32) |
          __reduce_or_sync(0xffffffffu, (uint32_t)vbits);
      if (lane == 0) {
        ok = wait(bar(B_KVE + stage), (uint32_t)(((i / C::STAGES) & 1) ^ 1));
        if (ok) {
          masks[stage * kProducerWarps + pw] = wmask;
          ptx::mbar_arrive(bar(B_META + stage));
          if (pw == 0)
            for (int jj = 0; jj < kNDB; ++jj)
              ptx::mbar_arrive_expect_tx(bar(kvf(stage, jj)), (uint32_t)kGroups * 512u);
        }
      }
      ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
      if (!ok) break;
      n_issued = i + 1;
      if (has_unit) {
        const uint32_t dst = sbase + (uint32_t)(C::OFF_KV + stage * kStageBytes + j * kRegion + g * 512);
        const int4 rows = make_int4(cur[0], cur[1], cur[2], cur[3]);
        if (j < 8)
          ptx::tma_gather4(dst, &tm_ckv, 64 * j, rows, bar(kvf(stage, j)), policy);
        else
          ptx::tma_gather4(dst, &tm_kpe, 0, rows, bar(kvf(stage, j)), policy);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) cur[q] = nxt[q];
    }
    if (!ok && lane == 0) {
      // Stop early: let every copy this warp issued land before the CTA exits.
      const Waiter drain{misc + 3, p.err};
      for (int64_t li = n_issued - 1; li >= 0 && li >= n_issued - C::STAGES; --li)
        for (int jj = 0; jj < kNDB; ++jj)
          drain(bar(kvf((int)(li % C::STAGES), jj)), (uint32_t)((li / C::STAGES) & 1));
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ MMA issuer
    ptx::regs_dec<kRegsLow>();
    if (lane == 0) {
      const Waiter wait{misc + 2, p.err, true};
      constexpr uint32_t kIdescS = idesc_bf16(64, NHC, false);
      constexpr uint32_t kIdescPV = idesc_bf16(128, NHC, true);
      int64_t i = 0;
      int seg = 0;
      bool ok = true;
      int64_t u = u_lo;
      Segment s;
      bool o_init = false;  // O holds this segment's sum (a live tile's PV was issued)
      int64_t prev_i = -1;
      int prev_stage = 0;
      bool prev_first = false, prev_live = false;
      while (ok && next_segment(u, u_hi, p.tpr, s)) {
        const int qb = seg % C::QBUF;
        const uint32_t qbase = sbase + (uint32_t)(C::OFF_Q + qb * C::Q_BYTES);
        for (int t = s.t0; t < s.t1; ++t, ++i) {
          const int stage = (int)(i % C::STAGES);
          const int sb = (int)(i & 1);
          const uint32_t kpar = (uint32_t)((i / C::STAGES) & 1);
          if (t == s.t0) ok = wait(bar(B_QF + qb), (uint32_t)((seg / C::QBUF) & 1));
          ok = ok && wait(bar(B_META + stage), kpar);
          ok = ok && wait(bar(B_SE + sb), (uint32_t)(((i >> 1) & 1) ^ 1));
          if (!ok) break;
          uint64_t m = 0;
#pragma unroll
          for (int w = 0; w < kProducerWarps; ++w) m |= masks[stage * kProducerWarps + w];
          const bool live = m != 0ull;
          ptx::tc_fence_after();  // S(i & 1) was read by softmax(i - 2) before s_empty
          // S^T[64 x NHC] = K[64 x 576] . Q[NHC x 576]^T, d-block by d-block as they land
          // (a TMA full barrier orders the copy before the MMA; no tcgen05 fence needed).
          // An all-padding tile's scores are all masked: its MMAs are skipped, but its
          // copies are still waited for before the stage is handed back.  With OVERLAP,
          // the previous tile's PV is issued half-way through this score, so that the
          // tensor core works on this tile while softmax(i-1) runs, without holding the
          // previous stage for a whole extra score.
          const uint32_t kv = sbase + (uint32_t)(C::OFF_KV + stage * kStageBytes);
          const uint32_t d_s = tmem + (uint32_t)(C::S_COL + sb * NHC);
#pragma unroll 1
          for (int jj = 0; jj < kNDB; ++jj) {
            if (C::OVERLAP && jj == kPVSplit && prev_i >= 0) {
              ok = issue_pv<NHC>(wait, bar0, sbase, tmem, prev_i, prev_stage, prev_first,
                                 prev_live, o_init);
              prev_i = -1;
              if (!ok) break;
            }
            ok = wait(bar(kvf(stage, jj)), kpar);
            if (!ok) break;
            if (live) {
#pragma unroll
              for (int ks = 0; ks < 4; ++ks)
                ptx::umma_bf16(d_s, sdesc(kv + (uint32_t)(jj * kRegion + ks * 32), 16, 1024),
                               sdesc(qbase + (uint32_t)(jj * C::Q_REGION + ks * 32), 16, 1024),
                               kIdescS, (jj | ks) ? 1u : 0u);
            }
          }
          if (!ok) break;
          ptx::umma_commit(bar(B_SF + sb));
          if (t == s.t1 - 1) ptx::umma_commit(bar(B_QE + qb));
          if (C::OVERLAP) {
            prev_i = i;
            prev_stage = stage;
            prev_first = (t == s.t0);
            prev_live = live;
            if (t == s.t1 - 1) {
              // The segment's last PV is not deferred behind the next segment's first
              // score (which waits for the next Q): the epilogue needs it now.
              ok = issue_pv<NHC>(wait, bar0, sbase, tmem, prev_i, prev_stage, prev_first,
                                 prev_live, o_init);
              prev_i = -1;
              if (!ok) break;
            }
          } else {
            // PV(i) right behind score(i), so that the stage is handed back early.
            ok = issue_pv<NHC>(wait, bar0, sbase, tmem, i, stage, t == s.t0, live, o_init);
            if (!ok) break;
          }
        }
        ++seg;
      }
      if (ok && C::OVERLAP && prev_i >= 0)
        ok = issue_pv<NHC>(wait, bar0, sbase, tmem, prev_i, prev_stage, prev_first, prev_live,
                           o_init);
      if (!ok) {
        // Stop early: wait (bounded) until every MMA issued so far has retired.
        const Waiter drain{misc + 3, p.err};
        ptx::umma_commit(bar(B_DRAIN));
        drain(bar(B_DRAIN), 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax / epilogue
    ptx::regs_inc<kRegsHigh>();
    const int sp = warp & 3;                 // TMEM sub-partition of this warp
    const int tid = threadIdx.x - kSmWarp0 * 32;  // 0..127
    const uint32_t lane_base = (uint32_t)(32 * sp) << 16;
    // Score row (slot within the tile) of this lane: the M=64 accumulator keeps
    // rows 16*sp .. 16*sp+15 in lanes 0-15 of sub-partition sp.
    const int kv_row = 16 * sp + lane;
    const bool row_lane = lane < 16;                  // holds a score row (0..63)
    const bool slot_lane = row_lane && kv_row < kBK;  // ... that is a slot of the tile
    int64_t i = 0;
    bool aborted = false;
    int64_t u = u_lo;
    Segment s;
    const int64_t first_rh = u_lo / p.tpr;
    float m_run[NHC], l_part[NHC];
    while (!aborted && next_segment(u, u_hi, p.tpr, s)) {
#pragma unroll
      for (int h = 0; h < NHC; ++h) {
        m_run[h] = -INFINITY;
        l_part[h] = 0.f;
      }
      bool o_valid = false;
      for (int t = s.t0; t < s.t1; ++t, ++i) {
        const int stage = (int)(i % C::STAGES);
        const int sb = (int)(i & 1);
        const bool ok = !aborted && wait(bar(B_META + stage), (uint32_t)((i / C::STAGES) & 1)) &&
                        wait(bar(B_SF + sb), (uint32_t)((i >> 1) & 1));
        uint64_t vmask = 0;
#pragma unroll
        for (int w = 0; w < kProducerWarps; ++w) vmask |= masks[stage * kProducerWarps + w];
        ptx::tc_fence_after();
        uint32_t sr[NHC];
#pragma unroll
        for (int c = 0; c < NHC / 16; ++c) {
          uint32_t chunk[16];
          ptx::tmem_ld16(tmem + lane_base + (uint32_t)(C::S_COL + sb * NHC + 16 * c), chunk);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) sr[16 * c + jj] = chunk[jj];
        }
        ptx::tc_fence_before();
        if (ok) ptx::mbar_arrive(bar(B_SE + sb));
        const bool rv = slot_lane && ((vmask >> kv_row) & 1ull);
        float x[NHC];
        bool need = false;
#pragma unroll
        for (int h = 0; h < NHC; ++h) {
          x[h] = rv ? __uint_as_float(sr[h]) * p.scale_log2 : -INFINITY;
          need |= x[h] > m_run[h] + kTau;
        }
        // One vote per tile: "some score needs a new running max, or a wait failed".
        // The rare second vote tells the two apart, so every thread agrees on both.
        bool rescale = false;
        if (ptx::bar_red_or(kNamedBar, kSmThreads, need || aborted || !ok)) {
          if (ptx::bar_red_or(kNamedBar, kSmThreads, aborted || !ok)) {
            aborted = true;
            break;
          }
          rescale = true;
        }
        if (rescale) {
#pragma unroll
          for (int h = 0; h < NHC; ++h) {
            float v = x[h];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
            if (lane == 0) red[sp * NHC + h] = v;
          }
          ptx::bar_sync(kNamedBar, kSmThreads);
          float alpha[NHC];
#pragma unroll
          for (int h = 0; h < NHC; ++h) {
            const float mt = fmaxf(fmaxf(red[h], red[NHC + h]), fmaxf(red[2 * NHC + h], red[3 * NHC + h]));
            const float mn = fmaxf(m_run[h], mt);
            alpha[h] = (m_run[h] == -INFINITY) ? 0.f : ptx::ex2(m_run[h] - mn);
            l_part[h] *= alpha[h];
            m_run[h] = mn;
          }
          if (o_valid) {
            if (!wait(bar(B_PD + (int)((i - 1) & 1)), (uint32_t)(((i - 1) >> 1) & 1))) {
              aborted = true;
            } else {
              ptx::tc_fence_after();
#pragma unroll
              for (int mt = 0; mt < 4; ++mt)
#pragma unroll
                for (int c = 0; c < NHC / 16; ++c) {
                  const uint32_t ta = tmem + lane_base + (uint32_t)(C::O_COL + mt * NHC + 16 * c);
                  uint32_t rr[16];
                  ptx::tmem_ld16(ta, rr);
                  ptx::tmem_wait_ld();
#pragma unroll
                  for (int jj = 0; jj < 16; ++jj)
                    rr[jj] = __float_as_uint(__uint_as_float(rr[jj]) * alpha[16 * c + jj]);
                  ptx::tmem_st16(ta, rr);
                }
              ptx::tmem_wait_st();
            }
          }
        }
        if (aborted) continue;  // the next vote ends the loop for every thread
        // The P buffer is free once the PV that read it (tile i - PBUF) has retired.
        if (i >= C::PBUF &&
            !wait(bar(B_PD + (int)((i - C::PBUF) & 1)), (uint32_t)(((i - C::PBUF) >> 1) & 1))) {
          aborted = true;
          continue;
        }
        uint8_t* pbuf = sgen + C::OFF_P + (int)(i % C::PBUF) * C::P_BYTES;
#pragma unroll
        for (int h = 0; h < NHC; ++h) {
          const float me = (m_run[h] == -INFINITY) ? 0.f : m_run[h];
          const float pv = ptx::ex2(x[h] - me);
          l_part[h] += pv;
          if (row_lane)
            *reinterpret_cast<__nv_bfloat16*>(pbuf + sw128_off(h, kv_row)) = __float2bfloat16_rn(pv);
        }
        if (vmask != 0ull && slot_lane && !rv) {
          // A padded slot of a live tile: its P is 0, but 0 * (non-finite stale bytes)
          // would poison the PV sum, so clear its row in every d-block (the PV's last K
          // step also reads rows kBK..63 of a d-block, i.e. rows 0..7 of the next one).
          uint8_t* row = sgen + C::OFF_KV + stage * kStageBytes + kv_row * 128;
#pragma unroll
          for (int jj = 0; jj < kNDB; ++jj)
#pragma unroll
            for (int q = 0; q < 8; ++q)
              *reinterpret_cast<uint4*>(row + jj * kRegion + q * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        ptx::fence_proxy_async_smem();
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(B_PF + (int)(i & 1)));
        o_valid = o_valid || (vmask != 0ull);
      }
      // ---------------------------------------------------------------- epilogue
      const int64_t il = i - 1;
      const bool okw = !aborted && wait(bar(B_PD + (int)(il & 1)), (uint32_t)((il >> 1) & 1));
      if (ptx::bar_red_or(kNamedBar, kSmThreads, aborted || !okw)) {
        aborted = true;
        break;
      }
      ptx::tc_fence_after();
#pragma unroll
      for (int h = 0; h < NHC; ++h) {
        float v = l_part[h];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) red[sp * NHC + h] = v;
      }
      ptx::bar_sync(kNamedBar, kSmThreads);
      float L[NHC];
#pragma unroll
      for (int h = 0; h < NHC; ++h) L[h] = (red[h] + red[NHC + h]) + (red[2 * NHC + h] + red[3 * NHC + h]);
      const int64_t b = s.rh / p.hg_count;
      const int head0 = (int)(s.rh % p.hg_count) * NHC;
      const bool full = (s.t0 == 0 && s.t1 == p.tpr);
      const int64_t slot = 2 * (int64_t)blockIdx.x + (s.rh == first_rh ? 0 : 1);
      float* part = p.parts + slot * C::SLOT_FLOATS;
#pragma unroll
      for (int mt = 0; mt < 4; ++mt) {
        const int d = 128 * mt + 32 * sp + lane;
#pragma unroll
        for (int c = 0; c < NHC / 16; ++c) {
          uint32_t rr[16];
          ptx::tmem_ld16(tmem + lane_base + (uint32_t)(C::O_COL + mt * NHC + 16 * c), rr);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int h = 16 * c + jj;
            const float o = __uint_as_float(rr[jj]);
            if (full) {
              const float y = L[h] > 0.f ? o / L[h] : 0.f;
              p.out[b * p.out_sb + (int64_t)(head0 + h) * p.out_sh + d] = __float2bfloat16_rn(y);
            } else {
              part[h * kDCkv + d] = o;
            }
          }
        }
      }
      if (tid < NHC) {
        // Thread tid writes head tid's scalars.  The element is picked with an unrolled
        // select: indexing the register arrays by a run-time value would move them (and
        // every access to them in the softmax loop) to local memory.
        float mh = 0.f, lh = 0.f;
#pragma unroll
        for (int h = 0; h < NHC; ++h)
          if (h == tid) {
            mh = m_run[h];
            lh = L[h];
          }
        if (full) {
          p.lse[b * p.lse_sb + (int64_t)(head0 + tid) * p.lse_sh] =
              lh > 0.f ? mh + ptx::lg2(lh) : -INFINITY;
        } else {
          part[NHC * kDCkv + tid] = mh;
          part[NHC * kDCkv + NHC + tid] = lh;
        }
      }
      ptx::tc_fence_before();
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, (uint32_t)C::TMEM_COLS);
  }
#undef bar
}


// Split-K merge.  CTA x of this grid looks at the boundary between decode CTAs x and x+1;
// if that boundary cuts a (row, head-group) and it is the first boundary that does, this
// CTA combines the row's partials (LSE-weighted, running max) for 16 heads (blockIdx.y).
// Rows that one decode CTA finished were written directly and are not touched here.
template <int NHC>
__global__ void __launch_bounds__(kDCkv) dsa_merge_kernel(const __grid_constant__ Params p,
                                                          int grid_main) {
  using C = Cfg<NHC>;
  ptx::grid_dep_wait();  // launched early (programmatic serialization): wait for the decode
  const int64_t G = grid_main;
  const int64_t c = (int64_t)blockIdx.x + 1;
  if (c >= G) return;
  const int64_t ub = u_begin(c, p.units, G);
  if (ub % p.tpr == 0) return;
  const int64_t rh = ub / p.tpr;
  const int64_t c_lo = cta_of(rh * p.tpr, p.units, G);
  if (c_lo != c - 1) return;
  const int64_t c_hi = cta_of((rh + 1) * p.tpr - 1, p.units, G);
  const int h0 = 16 * (int)blockIdx.y;
  const int d = threadIdx.x;
  float M[16], Lt[16], acc[16];
#pragma unroll
  for (int h = 0; h < 16; ++h) {
    M[h] = -INFINITY;
    Lt[h] = 0.f;
    acc[h] = 0.f;
  }
  for (int64_t cc = c_lo; cc <= c_hi; ++cc) {
    const int64_t sl = 2 * cc + ((u_begin(cc, p.units, G) / p.tpr) == rh ? 0 : 1);
    const float* pp = p.parts + sl * C::SLOT_FLOATS;
    float pm[16], pl[16], po[16];
#pragma unroll
    for (int h = 0; h < 16; ++h) {
      pm[h] = __ldg(pp + NHC * kDCkv + h0 + h);
      pl[h] = __ldg(pp + NHC * kDCkv + NHC + h0 + h);
      po[h] = __ldg(pp + (h0 + h) * kDCkv + d);
    }
#pragma unroll
    for (int h = 0; h < 16; ++h) {
      // A part with l == 0 saw only padding; its O is never read (it may be stale).
      const bool live = pl[h] > 0.f;
      const float mn = live ? fmaxf(M[h], pm[h]) : M[h];
      const float keep = (M[h] == -INFINITY) ? 0.f : ptx::ex2(M[h] - mn);
      const float w = live ? ptx::ex2(pm[h] - mn) : 0.f;
      Lt[h] = Lt[h] * keep + (live ? w * pl[h] : 0.f);
      acc[h] = acc[h] * keep + (live ? w * po[h] : 0.f);
      M[h] = mn;
    }
  }
  const int64_t b = rh / p.hg_count;
  const int head0 = (int)(rh % p.hg_count) * NHC + h0;
#pragma unroll
  for (int h = 0; h < 16; ++h) {
    const float y = Lt[h] > 0.f ? acc[h] / Lt[h] : 0.f;
    p.out[b * p.out_sb + (int64_t)(head0 + h) * p.out_sh + d] = __float2bfloat16_rn(y);
  }
  if (d < 16) {
    float mh = 0.f, lh = 0.f;  // unrolled select keeps M / Lt in registers
#pragma unroll
    for (int h = 0; h < 16; ++h)
      if (h == d) {
        mh = M[h];
        lh = Lt[h];
      }
    p.lse[b * p.lse_sb + (int64_t)(head0 + d) * p.lse_sh] = lh > 0.f ? mh + ptx::lg2(lh) : -INFINITY;
  }
}

__global__ void selftest_wait_kernel(uint32_t* err, int64_t timeout_ns) {
  __shared__ __align__(8) uint64_t mbar;
  const uint32_t b = ptx::smem_u32(&mbar);
  if (threadIdx.x == 0) {
    ptx::mbar_init(b, 1);
    ptx::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Nothing ever arrives on this barrier: the wait must give up by itself.
    // The bound counts SM cycles, two per requested nanosecond (~2 GHz clock).
    const uint64_t t0 = ptx::cycles();
    while (!ptx::mbar_try_wait(b, 0)) {
      if ((int64_t)(ptx::cycles() - t0) > 2 * timeout_ns) {
        atomicOr(err, (uint32_t)DSA_DEVERR_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
}

}  // namespace dsa

#include "dsa_decode_h16.cuh"

namespace dsa {
// ====================================================================== host side
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

constexpr int kMaxDevices = 64;

struct DeviceState {
  int sms = 0;
  int pairs = 0;  // co-resident two-CTA clusters of the 16-head kernel
  bool attr_done[4] = {false, false, false, false};
};
std::mutex g_mu;
DeviceState g_dev[kMaxDevices];

int device_sms(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (dev < 0 || dev >= kMaxDevices) return 0;
  if (g_dev[dev].sms == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
    g_dev[dev].sms = v;
  }
  return g_dev[dev].sms;
}

// Sets the 16-head kernel's shared-memory attribute and returns how many of its
// clusters fit on the device at once (the persistent grid's size), 0 on error.
int device_pairs(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (dev < 0 || dev >= kMaxDevices) return 0;
  DeviceState& d = g_dev[dev];
  if (d.pairs == 0) {
    // The kernel re-splits its register pool per warpgroup (setmaxnreg); refuse a build
    // whose pool is too small for that split, which would stall.
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, h16::dsa_decode_h16_kernel) != cudaSuccess) return 0;
    if ((int64_t)fa.numRegs * h16::kThreads < 256 * (int64_t)(h16::kRegsLow + h16::kRegsHigh))
      return 0;
    if (cudaFuncSetAttribute(h16::dsa_decode_h16_kernel,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             h16::SMEM_BYTES) != cudaSuccess)
      return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (unsigned)(d.sms > 0 ? d.sms : 148), 1, 1);
    cfg.blockDim = dim3(h16::kThreads, 1, 1);
    cfg.dynamicSmemBytes = h16::SMEM_BYTES;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, h16::dsa_decode_h16_kernel, &cfg) != cudaSuccess ||
        n <= 0)
      return 0;
    d.pairs = n;
  }
  return d.pairs;
}

int nhc_for(int heads) {
  switch (heads) {
    case 16: return 16;
    case 32: return 32;
    case 64: return 64;
    case 128: return 64;
    default: return 0;
  }
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Workspace layout, fixed for a device so that calls of any shape can share it:
//   [0, 256)            header (word 0: sticky device error bits)
//   [256, 8448)         split-K arrival counters of the 16-head kernel, 2 per CTA pair
//                       (each returns to zero when its row is merged)
//   [8448, ...)         split-K partials: 2 slots per decode CTA (or CTA pair), each
//                       sized for the widest head group (64 heads)
constexpr size_t kCountersOff = 256;
constexpr size_t kPartsOff = 8448;
constexpr int kMaxPairs = (int)((kPartsOff - kCountersOff) / 8);

struct WsLayout {
  size_t parts_off, total;
};

WsLayout ws_layout(int sms) {
  WsLayout w;
  w.parts_off = kPartsOff;
  w.total = align_up(w.parts_off + (size_t)(2 * sms) * (size_t)Cfg<64>::SLOT_FLOATS * 4, 256);
  return w;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Encoded tensor maps of recent calls (per host thread): a decode loop reuses its pools and
// usually its query buffers, and encoding costs microseconds of host time per map.
struct MapKey {
  const void* base;
  int rank;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
  int swz;
  bool operator==(const MapKey& o) const { return memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapCache {
  static constexpr int kWays = 16;
  MapKey key[kWays];
  CUtensorMap map[kWays];
  bool used[kWays] = {};
  int next = 0;
};
thread_local MapCache t_maps;

int encode(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
           const cuuint64_t* strides_bytes, const cuuint32_t* box, CUtensorMapSwizzle swz) {
  MapKey k;
  memset(&k, 0, sizeof(k));  // padding bytes take part in the comparison
  k.base = base;
  k.rank = rank;
  for (int i = 0; i < rank; ++i) {
    k.dims[i] = dims[i];
    k.box[i] = box[i];
  }
  for (int i = 0; i + 1 < rank; ++i) k.strides[i] = strides_bytes[i];
  k.swz = (int)swz;
  MapCache& c = t_maps;
  for (int w = 0; w < MapCache::kWays; ++w)
    if (c.used[w] && c.key[w] == k) {
      *m = c.map[w];
      return DSA_OK;
    }
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return DSA_ERR_DRIVER;
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base),
                  dims, strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return DSA_ERR_DRIVER;
  const int w = c.next;
  c.next = (c.next + 1) % MapCache::kWays;
  c.key[w] = k;
  c.map[w] = *m;
  c.used[w] = true;
  return DSA_OK;
}

// Every kernel of a call is launched with programmatic stream serialization: it may be
// scheduled while the grid before it drains, runs its set-up, and waits for that grid
// (griddepcontrol.wait) before it touches global memory.
cudaLaunchAttribute g_pdl_attr = [] {
  cudaLaunchAttribute a;
  a.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  a.val.programmaticStreamSerializationAllowed = 1;
  return a;
}();

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1] = {g_pdl_attr};
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) == cudaSuccess
             ? DSA_OK
             : DSA_ERR_CUDA;
}

// The split-K merge for a decode grid of `grid` CTAs.
template <int NHC>
int launch_merge(const Params& prm, int grid, cudaStream_t stream) {
  if (grid <= 1) return DSA_OK;
  return launch_pdl(dsa_merge_kernel<NHC>, dim3((unsigned)(grid - 1), NHC / 16, 1),
                    dim3(kDCkv, 1, 1), 0, stream, prm, grid);
}

template <int NHC>
int launch(const CUtensorMap& ckv, const CUtensorMap& kpe, const CUtensorMap& qn,
           const CUtensorMap& qp, const Params& prm, int grid, int dev, cudaStream_t stream) {
  using C = Cfg<NHC>;
  const int ai = NHC == 16 ? 0 : NHC == 32 ? 1 : 2;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_dev[dev].attr_done[ai]) {
      // The kernel re-splits its register pool per warpgroup (setmaxnreg); refuse to
      // launch a build whose pool is too small for that split, which would stall.
      cudaFuncAttributes fa;
      if (cudaFuncGetAttributes(&fa, dsa_decode_kernel<NHC>) != cudaSuccess) return DSA_ERR_CUDA;
      if ((int64_t)fa.numRegs * kThreads < 128 * (int64_t)(3 * kRegsLow + kRegsHigh))
        return DSA_ERR_CUDA;
      if (cudaFuncSetAttribute(dsa_decode_kernel<NHC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               C::SMEM_BYTES) != cudaSuccess)
        return DSA_ERR_CUDA;
      g_dev[dev].attr_done[ai] = true;
    }
  }
  int rc = launch_pdl(dsa_decode_kernel<NHC>, dim3((unsigned)grid), dim3(kThreads),
                      (size_t)C::SMEM_BYTES, stream, ckv, kpe, qn, qp, prm);
  if (rc != DSA_OK) return rc;
  return launch_merge<NHC>(prm, grid, stream);
}

// One decode call: the C-ABI arguments without the workspace.
struct DecodeArgs {
  const void* q_nope;
  int64_t qn_sb, qn_sh;
  const void* q_pe;
  int64_t qp_sb, qp_sh;
  const void* ckv;
  int64_t ckv_ss;
  const void* kpe;
  int64_t kpe_ss;
  int64_t num_slots;
  const int32_t* idx;
  int64_t idx_sb;
  float sm_scale;
  void* out;
  int64_t out_sb, out_sh;
  float* lse;
  int64_t lse_sb, lse_sh;
  int64_t num_tokens;
  int32_t num_heads;
  int32_t topk;
};

int check_args(const DecodeArgs& a) {
  if (a.num_tokens < 0 || a.topk < 1 || a.num_slots < 1 || a.num_slots > INT32_MAX ||
      a.num_tokens > INT32_MAX)
    return DSA_ERR_INVALID_ARGUMENT;
  if (nhc_for(a.num_heads) == 0) return DSA_ERR_UNSUPPORTED;
  if (a.num_tokens == 0) return DSA_OK;
  if (!a.q_nope || !a.q_pe || !a.ckv || !a.kpe || !a.idx || !a.out || !a.lse)
    return DSA_ERR_INVALID_ARGUMENT;
  if (a.ckv_ss < kDCkv || a.kpe_ss < kDKpe || a.qn_sh < kDCkv || a.qp_sh < kDKpe || a.qn_sb < 1 ||
      a.qp_sb < 1 || a.idx_sb < a.topk)
    return DSA_ERR_INVALID_ARGUMENT;
  if (!aligned16(a.q_nope) || !aligned16(a.q_pe) || !aligned16(a.ckv) || !aligned16(a.kpe) ||
      (a.qn_sb * 2) % 16 || (a.qn_sh * 2) % 16 || (a.qp_sb * 2) % 16 || (a.qp_sh * 2) % 16 ||
      (a.ckv_ss * 2) % 16 || (a.kpe_ss * 2) % 16)
    return DSA_ERR_MISALIGNED;
  return DSA_OK;
}

// Which kernel a call runs, its persistent grid and the scratch it needs.
struct Plan {
  bool pair = false;  // the 16-head two-CTA-cluster kernel
  int nhc = 0;
  int tpr = 0;
  int64_t units = 0;
  int grid = 0;       // CTAs (generic kernel) or clusters (pair kernel)
  size_t need = 0;    // bytes of error header + partials
};

int make_plan(const DecodeArgs& a, int dev, Plan& pl) {
  const int sms = device_sms(dev);
  if (sms <= 0) return DSA_ERR_CUDA;
  pl.nhc = nhc_for(a.num_heads);
  pl.pair = (pl.nhc == 16);
  const int hg = a.num_heads / pl.nhc;
  const int tile = pl.pair ? h16::kTS : kBK;
  pl.tpr = (a.topk + tile - 1) / tile;
  pl.units = a.num_tokens * hg * (int64_t)pl.tpr;
  int cap = sms;
  if (pl.pair) {
    cap = device_pairs(dev);
    if (cap <= 0) return DSA_ERR_CUDA;
  }
  // 16 heads: with no more rows than the grid can hold, each row gets a whole CTA pair and
  // none is split: a split-K merge costs a few dependent global round trips on the tail,
  // each slow while the other SMs saturate HBM, which outweighs the idle SMs.  Otherwise
  // (and for the generic kernel) stream-K over the tiles with an equal share per CTA.
  const int64_t num_rh = a.num_tokens * hg;
  pl.grid = (int)(pl.pair && num_rh <= cap ? num_rh : (pl.units < cap ? pl.units : cap));
  const size_t slot_bytes = (size_t)(pl.nhc * kDCkv + 2 * pl.nhc) * 4;
  if (pl.pair && pl.grid > kMaxPairs) pl.grid = kMaxPairs;
  pl.need = kPartsOff + (size_t)(2 * pl.grid) * slot_bytes;
  return DSA_OK;
}

int run_plan(const DecodeArgs& a, const Plan& pl, uint8_t* ws, int dev, cudaStream_t st) {
  const int nhc = pl.nhc;
  CUtensorMap m_ckv, m_kpe, m_qn, m_qp;
  const cuuint32_t kpe_w = pl.pair ? 32 : 64;  // the pair kernel loads 32-wide kpe halves
  const CUtensorMapSwizzle kpe_swz = pl.pair ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  int rc;
  {
    cuuint64_t dims[2] = {(cuuint64_t)kDCkv, (cuuint64_t)a.num_slots};
    cuuint64_t str[1] = {(cuuint64_t)a.ckv_ss * 2};
    cuuint32_t box[2] = {64, 1};
    if ((rc = encode(&m_ckv, a.ckv, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) != DSA_OK)
      return rc;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)kDKpe, (cuuint64_t)a.num_slots};
    cuuint64_t str[1] = {(cuuint64_t)a.kpe_ss * 2};
    cuuint32_t box[2] = {kpe_w, 1};
    if ((rc = encode(&m_kpe, a.kpe, 2, dims, str, box, kpe_swz)) != DSA_OK) return rc;
  }
  {
    cuuint64_t dims[3] = {(cuuint64_t)kDCkv, (cuuint64_t)a.num_heads, (cuuint64_t)a.num_tokens};
    cuuint64_t str[2] = {(cuuint64_t)a.qn_sh * 2, (cuuint64_t)a.qn_sb * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)nhc, 1};
    if ((rc = encode(&m_qn, a.q_nope, 3, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) != DSA_OK)
      return rc;
  }
  {
    cuuint64_t dims[3] = {(cuuint64_t)kDKpe, (cuuint64_t)a.num_heads, (cuuint64_t)a.num_tokens};
    cuuint64_t str[2] = {(cuuint64_t)a.qp_sh * 2, (cuuint64_t)a.qp_sb * 2};
    cuuint32_t box[3] = {kpe_w, (cuuint32_t)nhc, 1};
    if ((rc = encode(&m_qp, a.q_pe, 3, dims, str, box, kpe_swz)) != DSA_OK) return rc;
  }
  Params prm;
  prm.idx = a.idx;
  prm.idx_sb = a.idx_sb;
  prm.out = static_cast<__nv_bfloat16*>(a.out);
  prm.out_sb = a.out_sb;
  prm.out_sh = a.out_sh;
  prm.lse = a.lse;
  prm.lse_sb = a.lse_sb;
  prm.lse_sh = a.lse_sh;
  prm.num_slots = a.num_slots;
  prm.units = pl.units;
  prm.hg_count = a.num_heads / nhc;
  prm.topk = a.topk;
  prm.tpr = pl.tpr;
  prm.scale_log2 = a.sm_scale * kLog2e;
  prm.err = reinterpret_cast<uint32_t*>(ws);
  prm.parts = reinterpret_cast<float*>(ws + kPartsOff);
  prm.counters = reinterpret_cast<uint32_t*>(ws + kCountersOff);
  if (pl.pair) {
    return launch_pdl(h16::dsa_decode_h16_kernel, dim3((unsigned)(2 * pl.grid)),
                      dim3(h16::kThreads), (size_t)h16::SMEM_BYTES, st, m_ckv, m_kpe, m_qn, m_qp,
                      prm);
  }
  switch (nhc) {
    case 32: return launch<32>(m_ckv, m_kpe, m_qn, m_qp, prm, pl.grid, dev, st);
    default: return launch<64>(m_ckv, m_kpe, m_qn, m_qp, prm, pl.grid, dev, st);
  }
}

int current_device(int& dev) {
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DSA_ERR_CUDA;
  return DSA_OK;
}

}  // namespace
}  // namespace dsa

using namespace dsa;

extern "C" {

int dsa_abi_version(void) { return 1; }

const char* dsa_status_string(int status) {
  switch (status) {
    case DSA_OK: return "ok";
    case DSA_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DSA_ERR_UNSUPPORTED: return "unsupported shape (num_heads must be 16, 32, 64 or 128)";
    case DSA_ERR_MISALIGNED: return "pointer or row stride is not a multiple of 16 bytes";
    case DSA_ERR_WORKSPACE: return "workspace missing or too small";
    case DSA_ERR_CUDA: return "CUDA runtime error";
    case DSA_ERR_DRIVER: return "cuTensorMapEncodeTiled unavailable or rejected the tensor";
    case DSA_ERR_SCRATCH_LIMIT:
      return "problem needs more scratch than the built-in no-allocation array holds "
             "(use dsa_sparse_mla_decode with a caller workspace)";
    default: return "unknown status";
  }
}

size_t dsa_sparse_mla_decode_workspace_size(int64_t num_tokens, int32_t num_heads, int32_t topk,
                                            int32_t device) {
  const int nhc = nhc_for(num_heads);
  if (nhc == 0 || num_tokens < 0 || topk < 1) return 0;
  const int sms = device_sms(device);
  if (sms <= 0) return 0;
  return ws_layout(sms).total;
}

int dsa_sparse_mla_decode(const void* q_nope, int64_t q_nope_stride_b, int64_t q_nope_stride_h,
                          const void* q_pe, int64_t q_pe_stride_b, int64_t q_pe_stride_h,
                          const void* ckv_cache, int64_t ckv_slot_stride,
                          const void* kpe_cache, int64_t kpe_slot_stride, int64_t num_slots,
                          const int32_t* sparse_indices, int64_t indices_stride_b,
                          float sm_scale, void* output, int64_t output_stride_b,
                          int64_t output_stride_h, float* lse, int64_t lse_stride_b,
                          int64_t lse_stride_h, int64_t num_tokens, int32_t num_heads,
                          int32_t topk, void* workspace, size_t workspace_bytes, void* stream) {
  const DecodeArgs a{q_nope,          q_nope_stride_b, q_nope_stride_h, q_pe,
                     q_pe_stride_b,   q_pe_stride_h,   ckv_cache,       ckv_slot_stride,
                     kpe_cache,       kpe_slot_stride, num_slots,       sparse_indices,
                     indices_stride_b, sm_scale,       output,          output_stride_b,
                     output_stride_h, lse,             lse_stride_b,    lse_stride_h,
                     num_tokens,      num_heads,       topk};
  int rc = check_args(a);
  if (rc != DSA_OK || num_tokens == 0) return rc;
  int dev = 0;
  if ((rc = current_device(dev)) != DSA_OK) return rc;
  const int sms = device_sms(dev);
  if (sms <= 0) return DSA_ERR_CUDA;
  if (!workspace || workspace_bytes < ws_layout(sms).total) return DSA_ERR_WORKSPACE;
  Plan pl;
  if ((rc = make_plan(a, dev, pl)) != DSA_OK) return rc;
  return run_plan(a, pl, static_cast<uint8_t*>(workspace), dev, static_cast<cudaStream_t>(stream));
}

int dsa_read_error_word(void* workspace, void* stream, int clear, uint32_t* word) {
  if (!workspace || !word) return DSA_ERR_INVALID_ARGUMENT;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t v = 0;
  if (cudaMemcpyAsync(&v, workspace, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return DSA_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return DSA_ERR_CUDA;
  *word = v;
  if (clear) {
    if (cudaMemsetAsync(workspace, 0, 4, st) != cudaSuccess) return DSA_ERR_CUDA;
    if (cudaStreamSynchronize(st) != cudaSuccess) return DSA_ERR_CUDA;
  }
  return DSA_OK;
}

int dsa_selftest_bounded_wait(int64_t timeout_ns, void* workspace, void* stream) {
  if (!workspace || timeout_ns < 0) return DSA_ERR_INVALID_ARGUMENT;
  selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint32_t*>(workspace), timeout_ns);
  return cudaGetLastError() == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
}

}  // extern "C"

// ============================================================ no-allocation entry point
// Some callers cannot allocate device memory at the point where they decode: code that
// runs inside another framework's allocator-controlled region, a plugin whose host
// application forbids cudaMalloc on its hot path, or a process that must not grow its
// device footprint after start-up.  dsa_sparse_mla_decode_noalloc() serves them: instead of
// a caller-provided workspace it uses the fixed array below, which the CUDA module holds on
// every device that loads this library until the process exits.
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;  // error word + split-K partials
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
std::mutex g_noalloc_mu;
void* g_noalloc_addr[kMaxDevices] = {};
}  // namespace

extern "C" int dsa_sparse_mla_decode_noalloc(
    const void* q_nope, int64_t q_nope_stride_b, int64_t q_nope_stride_h, const void* q_pe,
    int64_t q_pe_stride_b, int64_t q_pe_stride_h, const void* ckv_cache, int64_t ckv_slot_stride,
    const void* kpe_cache, int64_t kpe_slot_stride, int64_t num_slots,
    const int32_t* sparse_indices, int64_t indices_stride_b, float sm_scale, void* output,
    int64_t output_stride_b, int64_t output_stride_h, float* lse, int64_t lse_stride_b,
    int64_t lse_stride_h, int64_t num_tokens, int32_t num_heads, int32_t topk, void* stream) {
  const DecodeArgs a{q_nope,          q_nope_stride_b, q_nope_stride_h, q_pe,
                     q_pe_stride_b,   q_pe_stride_h,   ckv_cache,       ckv_slot_stride,
                     kpe_cache,       kpe_slot_stride, num_slots,       sparse_indices,
                     indices_stride_b, sm_scale,       output,          output_stride_b,
                     output_stride_h, lse,             lse_stride_b,    lse_stride_h,
                     num_tokens,      num_heads,       topk};
  int rc = check_args(a);
  if (rc != DSA_OK || num_tokens == 0) return rc;
  int dev = 0;
  if ((rc = current_device(dev)) != DSA_OK) return rc;
  Plan pl;
  if ((rc = make_plan(a, dev, pl)) != DSA_OK) return rc;
  if (pl.need > kNoAllocScratchBytes) return DSA_ERR_SCRATCH_LIMIT;

  // The host cannot use g_noalloc_scratch as a device address: resolve the array's address
  // on this device once (with this device current) and reuse it.
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_addr[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return DSA_ERR_CUDA;
      g_noalloc_addr[dev] = p;
    }
    scratch = g_noalloc_addr[dev];
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The array keeps the previous call's bytes: the error word and the split-K counters
  // must start at zero; the partials are always written before they are read.
  if (cudaMemsetAsync(scratch, 0, kPartsOff, st) != cudaSuccess) return DSA_ERR_CUDA;
  return run_plan(a, pl, static_cast<uint8_t*>(scratch), dev, st);
}
