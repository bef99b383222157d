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
//     (stream-K).  A row cut between CTAs is finished by the CTA that arrives last at
//     the row's counter, which merges the LSE-weighted partials (split-K merge fused
//     into the same launch).
//   * Warp 0 (producer): per tile, reads 64 slot ids and issues TMA tile::gather4
//     loads (4 slots x 128 B each) of the 512-d ckv row and the 64-d kpe row into a
//     128-byte-swizzled shared-memory stage; a -1 slot is requested as an
//     out-of-range row, which reads nothing from HBM.  Tiles with no valid slot skip
//     both MMAs; in other tiles the softmax warps clear a padded slot's value row so
//     that its P == 0 contributes exactly zero.
//   * Warp 1 (MMA issuer, one thread): score S^T[64 slots x NHC heads] = K . Q^T with
//     tcgen05.mma (M=64, K=576 as 36 k-steps) into TMEM, then after softmax the
//     output O^T[512 d x NHC heads] += V^T . P^T (M=128 x 4 d-tiles, V read from the
//     same stage as an MN-major operand) into TMEM.
//   * Warps 2-5 (softmax + epilogue): tcgen05.ld the scores, base-2 online softmax
//     with a lazily-updated running max (the accumulator is rescaled only when a
//     score exceeds the running max by more than kTau), write bf16 P^T to shared
//     memory, and at a segment's end read O from TMEM and write the output or a
//     partial.
//   * Heads are split into groups of NHC = min(H, 64) per unit (H = 128 -> 2 groups).
//
// Every mbarrier wait is bounded (wait_bounded); on timeout the CTA records
// DSA_DEVERR_TIMEOUT, stops issuing work and exits after its copies land.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <mutex>

#include "dsa_b200.h"
#include "sm100_ptx.cuh"

namespace dsa {

constexpr int kDCkv = 512;            // latent (value) width
constexpr int kDKpe = 64;             // rope key width
constexpr int kBK = 64;               // slots per tile (MMA M of the score)
constexpr int kNDB = 9;               // 64-element d-blocks: 8 ckv + 1 kpe
constexpr int kRegion = kBK * 128;    // bytes of one d-block of a stage
constexpr int kStageBytes = kNDB * kRegion;
constexpr int kThreads = 192;
constexpr int kSmThreads = 128;       // softmax / epilogue warpgroup
constexpr uint32_t kNamedBar = 1;
constexpr float kTau = 8.0f;          // lazy-rescale threshold (log2 units)
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;

template <int NHC>
struct Cfg {
  static constexpr int STAGES = 2;
  static constexpr int QBUF = (NHC <= 32) ? 2 : 1;
  static constexpr int PBUF = (NHC <= 32) ? 2 : 1;
  static constexpr int Q_REGION = NHC * 128;
  static constexpr int Q_BYTES = kNDB * Q_REGION;
  static constexpr int P_BYTES = NHC * 128;
  static constexpr int OFF_KV = 0;
  static constexpr int OFF_Q = OFF_KV + STAGES * kStageBytes;
  static constexpr int OFF_P = OFF_Q + QBUF * Q_BYTES;
  static constexpr int OFF_BAR = OFF_P + PBUF * P_BYTES;
  static constexpr int OFF_MASK = OFF_BAR + 256;
  static constexpr int OFF_MISC = OFF_MASK + 64;
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
  static_assert(OFF_Q % 1024 == 0 && OFF_P % 1024 == 0, "swizzle atoms need 1024-B alignment");
};

// Barrier slots (8 bytes each) inside the OFF_BAR block.
enum : int {
  B_KVF = 0, B_KVE = 4, B_QF = 8, B_QE = 10, B_SF = 12, B_SE = 14, B_PF = 16, B_PD = 18,
  B_DRAIN = 20  // used only when the MMA issuer stops early
};

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
  int32_t* counters;
  float* parts;
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

struct Waiter {
  volatile uint32_t* abort_flag;
  uint32_t* err;
  __device__ __forceinline__ bool operator()(uint32_t bar, uint32_t parity) const {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = ptx::globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
      if (ptx::mbar_try_wait(bar, parity)) return true;
      if ((it & 63u) == 0) {
        if (*abort_flag) return false;
        if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
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
  uint64_t* masks = reinterpret_cast<uint64_t*>(sgen + C::OFF_MASK);
  float* red = reinterpret_cast<float*>(sgen + C::OFF_RED);
  auto bar = [&](int k) -> uint32_t { return sbase + (uint32_t)C::OFF_BAR + 8u * (uint32_t)k; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      ptx::mbar_init(bar(B_KVF + s), 1);
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
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&tm_ckv);
    ptx::prefetch_tmap(&tm_kpe);
    ptx::prefetch_tmap(&tm_qn);
    ptx::prefetch_tmap(&tm_qp);
  }
  if (warp == 1) {
    ptx::tmem_alloc(sbase + (uint32_t)C::OFF_MISC, (uint32_t)C::TMEM_COLS);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = misc[0];

  const int64_t G = gridDim.x;
  const int64_t u_lo = u_begin(blockIdx.x, p.units, G);
  const int64_t u_hi = u_begin((int64_t)blockIdx.x + 1, p.units, G);
  const Waiter wait{misc + 2, p.err};

  if (warp == 0) {
    // ------------------------------------------------------------------ producer
    const uint64_t policy = ptx::policy_evict_first();
    int64_t i = 0;
    int seg = 0;
    bool ok = true;
    int64_t u = u_lo;
    Segment s;
    int64_t last_issue[C::STAGES];
    for (int k = 0; k < C::STAGES; ++k) last_issue[k] = -1;
    while (ok && next_segment(u, u_hi, p.tpr, s)) {
      const int64_t b = s.rh / p.hg_count;
      const int hg = (int)(s.rh % p.hg_count);
      const int qb = seg % C::QBUF;
      if (lane == 0) {
        ok = wait(bar(B_QE + qb), (uint32_t)(((seg / C::QBUF) & 1) ^ 1));
        if (ok) {
          ptx::mbar_arrive_expect_tx(bar(B_QF + qb), (uint32_t)C::Q_BYTES);
          const uint32_t qdst = sbase + (uint32_t)(C::OFF_Q + qb * C::Q_BYTES);
          for (int j = 0; j < 8; ++j)
            ptx::tma_load_3d(qdst + (uint32_t)(j * C::Q_REGION), &tm_qn, 64 * j, hg * NHC, (int)b,
                             bar(B_QF + qb));
          ptx::tma_load_3d(qdst + (uint32_t)(8 * C::Q_REGION), &tm_qp, 0, hg * NHC, (int)b,
                           bar(B_QF + qb));
        }
      }
      ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
      if (!ok) break;
      const int32_t* idx_row = p.idx + b * p.idx_sb;
      for (int t = s.t0; t < s.t1; ++t, ++i) {
        const int stage = (int)(i % C::STAGES);
        const int kbase = t * kBK + 4 * (lane >> 1);
        int r[4];
        bool bad = false;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int k = kbase + q;
          int v = -1;
          if (k < p.topk) {
            v = __ldg(idx_row + k);
            if (v < -1 || (int64_t)v >= p.num_slots) {
              bad = true;
              v = -1;
            }
          }
          r[q] = v;
        }
        if (bad) atomicOr(p.err, (uint32_t)DSA_DEVERR_BAD_INDEX);
        uint32_t bq[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) bq[q] = __ballot_sync(0xffffffffu, r[q] >= 0);
        if (lane == 0) {
          ok = wait(bar(B_KVE + stage), (uint32_t)(((i / C::STAGES) & 1) ^ 1));
          if (ok) {
            uint64_t mask = 0;
#pragma unroll
            for (int g = 0; g < 16; ++g)
#pragma unroll
              for (int q = 0; q < 4; ++q)
                mask |= (uint64_t)((bq[q] >> (2 * g)) & 1u) << (4 * g + q);
            masks[stage] = mask;
            ptx::mbar_arrive_expect_tx(bar(B_KVF + stage), (uint32_t)kStageBytes);
          }
        }
        ok = __shfl_sync(0xffffffffu, (int)ok, 0) != 0;
        if (!ok) break;
        last_issue[stage] = i;
        const int4 rows = make_int4(r[0], r[1], r[2], r[3]);
        const uint32_t dst0 =
            sbase + (uint32_t)(C::OFF_KV + stage * kStageBytes + (lane >> 1) * 512);
        const int jlo = (lane & 1) ? 5 : 0;
        const int jhi = (lane & 1) ? 9 : 5;
        for (int j = jlo; j < jhi; ++j) {
          if (j < 8)
            ptx::tma_gather4(dst0 + (uint32_t)(j * kRegion), &tm_ckv, 64 * j, rows,
                             bar(B_KVF + stage), policy);
          else
            ptx::tma_gather4(dst0 + (uint32_t)(j * kRegion), &tm_kpe, 0, rows, bar(B_KVF + stage),
                             policy);
        }
      }
      ++seg;
    }
    if (!ok && lane == 0) {
      // Stop early: let every copy this warp issued land before the CTA exits.
      const Waiter drain{misc + 3, p.err};
      for (int k = 0; k < C::STAGES; ++k)
        if (last_issue[k] >= 0) drain(bar(B_KVF + k), (uint32_t)((last_issue[k] / C::STAGES) & 1));
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdescS = idesc_bf16(64, NHC, false);
      constexpr uint32_t kIdescPV = idesc_bf16(128, NHC, true);
      int64_t i = 0;
      int seg = 0;
      bool ok = true;
      int64_t prev_i = -1;
      bool prev_first = false, prev_live = false;
      int64_t u = u_lo;
      Segment s;
      bool o_init = false;  // O holds this segment's sum (a live tile's PV was issued)
      auto issue_pv = [&](int64_t pi, bool first, bool live) -> bool {
        if (!wait(bar(B_PF + (int)(pi & 1)), (uint32_t)((pi >> 1) & 1))) return false;
        ptx::tc_fence_after();
        const int pst = (int)(pi % C::STAGES);
        if (first) o_init = false;
        if (live) {  // an all-padding tile has P == 0: its PV is skipped
          const uint32_t kv = sbase + (uint32_t)(C::OFF_KV + pst * kStageBytes);
          const uint32_t pb = sbase + (uint32_t)(C::OFF_P + (int)(pi % C::PBUF) * C::P_BYTES);
#pragma unroll
          for (int mt = 0; mt < 4; ++mt)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              ptx::umma_bf16(tmem + (uint32_t)(C::O_COL + mt * NHC),
                             sdesc(kv + (uint32_t)(2 * mt * kRegion + ks * 2048), kRegion, 1024),
                             sdesc(pb + (uint32_t)(ks * 32), 16, 1024), kIdescPV,
                             (o_init || ks > 0) ? 1u : 0u);
          o_init = true;
        }
        ptx::umma_commit(bar(B_KVE + pst));
        ptx::umma_commit(bar(B_PD + (int)(pi & 1)));
        return true;
      };
      while (ok && next_segment(u, u_hi, p.tpr, s)) {
        const int qb = seg % C::QBUF;
        const uint32_t qbase = sbase + (uint32_t)(C::OFF_Q + qb * C::Q_BYTES);
        for (int t = s.t0; t < s.t1; ++t, ++i) {
          const int stage = (int)(i % C::STAGES);
          const int sb = (int)(i & 1);
          if (t == s.t0) ok = wait(bar(B_QF + qb), (uint32_t)((seg / C::QBUF) & 1));
          ok = ok && wait(bar(B_KVF + stage), (uint32_t)((i / C::STAGES) & 1));
          ok = ok && wait(bar(B_SE + sb), (uint32_t)(((i >> 1) & 1) ^ 1));
          if (!ok) break;
          ptx::tc_fence_after();
          const bool live = masks[stage] != 0ull;
          if (live) {  // an all-padding tile's scores are all masked: skip its MMAs
            const uint32_t kv = sbase + (uint32_t)(C::OFF_KV + stage * kStageBytes);
            const uint32_t d_s = tmem + (uint32_t)(C::S_COL + sb * NHC);
#pragma unroll
            for (int j = 0; j < kNDB; ++j)
#pragma unroll
              for (int ks = 0; ks < 4; ++ks)
                ptx::umma_bf16(d_s, sdesc(kv + (uint32_t)(j * kRegion + ks * 32), 16, 1024),
                               sdesc(qbase + (uint32_t)(j * C::Q_REGION + ks * 32), 16, 1024),
                               kIdescS, (j | ks) ? 1u : 0u);
          }
          ptx::umma_commit(bar(B_SF + sb));
          if (t == s.t1 - 1) ptx::umma_commit(bar(B_QE + qb));
          if (prev_i >= 0) {
            ok = issue_pv(prev_i, prev_first, prev_live);
            if (!ok) break;
          }
          prev_i = i;
          prev_first = (t == s.t0);
          prev_live = live;
        }
        ++seg;
      }
      if (ok && prev_i >= 0) ok = issue_pv(prev_i, prev_first, prev_live);
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
    const int sp = warp & 3;                 // TMEM sub-partition of this warp
    const int tid = threadIdx.x - 64;        // 0..127
    const uint32_t lane_base = (uint32_t)(32 * sp) << 16;
    const int kv_row = 16 * sp + lane;       // score row (slot within the tile) of this lane
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
        const bool ok = !aborted && wait(bar(B_KVF + stage), (uint32_t)((i / C::STAGES) & 1)) &&
                        wait(bar(B_SF + sb), (uint32_t)((i >> 1) & 1));
        if (ptx::bar_red_or(kNamedBar, kSmThreads, aborted || !ok)) {
          aborted = true;
          break;
        }
        const uint64_t vmask = masks[stage];
        ptx::tc_fence_after();
        uint32_t sr[NHC];
#pragma unroll
        for (int c = 0; c < NHC / 16; ++c) {
          uint32_t chunk[16];
          ptx::tmem_ld16(tmem + lane_base + (uint32_t)(C::S_COL + sb * NHC + 16 * c), chunk);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) sr[16 * c + j] = chunk[j];
        }
        ptx::tc_fence_before();
        ptx::mbar_arrive(bar(B_SE + sb));
        const bool rv = (lane < 16) && ((vmask >> kv_row) & 1ull);
        float x[NHC];
        bool need = false;
#pragma unroll
        for (int h = 0; h < NHC; ++h) {
          x[h] = rv ? __uint_as_float(sr[h]) * p.scale_log2 : -INFINITY;
          need |= x[h] > m_run[h] + kTau;
        }
        if (ptx::bar_red_or(kNamedBar, kSmThreads, need)) {
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
                  uint32_t r[16];
                  ptx::tmem_ld16(ta, r);
                  ptx::tmem_wait_ld();
#pragma unroll
                  for (int j = 0; j < 16; ++j)
                    r[j] = __float_as_uint(__uint_as_float(r[j]) * alpha[16 * c + j]);
                  ptx::tmem_st16(ta, r);
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
          if (lane < 16)
            *reinterpret_cast<__nv_bfloat16*>(pbuf + sw128_off(h, kv_row)) = __float2bfloat16_rn(pv);
        }
        if (vmask != 0ull && lane < 16 && !rv) {
          // A padded slot of a live tile: its P is 0, but 0 * (non-finite stale bytes)
          // would poison the PV sum, so clear its value row (the 8 ckv d-blocks).
          uint8_t* row = sgen + C::OFF_KV + stage * kStageBytes + kv_row * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int q = 0; q < 8; ++q)
              *reinterpret_cast<uint4*>(row + j * kRegion + q * 16) = make_uint4(0u, 0u, 0u, 0u);
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
          uint32_t r[16];
          ptx::tmem_ld16(tmem + lane_base + (uint32_t)(C::O_COL + mt * NHC + 16 * c), r);
          ptx::tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int h = 16 * c + j;
            const float o = __uint_as_float(r[j]);
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
        const int h = tid;
        if (full) {
          p.lse[b * p.lse_sb + (int64_t)(head0 + h) * p.lse_sh] =
              L[h] > 0.f ? m_run[h] + ptx::lg2(L[h]) : -INFINITY;
        } else {
          part[NHC * kDCkv + h] = m_run[h];
          part[NHC * kDCkv + NHC + h] = L[h];
        }
      }
      ptx::tc_fence_before();
      if (!full) {
        // Split row: publish the partial; the last CTA to arrive merges all of them.
        __threadfence();
        ptx::bar_sync(kNamedBar, kSmThreads);
        if (tid == 0) {
          const int64_t c_lo = cta_of(s.rh * p.tpr, p.units, G);
          const int64_t c_hi = cta_of((s.rh + 1) * p.tpr - 1, p.units, G);
          const int old = atomicAdd(p.counters + s.rh, 1);
          misc[1] = (old == (int)(c_hi - c_lo)) ? 1u : 0u;
        }
        ptx::bar_sync(kNamedBar, kSmThreads);
        const bool merge = misc[1] != 0;
        if (merge) {
          __threadfence();
          const int64_t c_lo = cta_of(s.rh * p.tpr, p.units, G);
          const int64_t c_hi = cta_of((s.rh + 1) * p.tpr - 1, p.units, G);
          float M[NHC], Lt[NHC];
#pragma unroll
          for (int h = 0; h < NHC; ++h) {
            M[h] = -INFINITY;
            Lt[h] = 0.f;
          }
          for (int64_t c = c_lo; c <= c_hi; ++c) {
            const int64_t sl = 2 * c + ((u_begin(c, p.units, G) / p.tpr) == s.rh ? 0 : 1);
            const float* pp = p.parts + sl * C::SLOT_FLOATS + NHC * kDCkv;
#pragma unroll
            for (int h = 0; h < NHC; ++h)
              if (__ldcg(pp + NHC + h) > 0.f) M[h] = fmaxf(M[h], __ldcg(pp + h));
          }
          for (int64_t c = c_lo; c <= c_hi; ++c) {
            const int64_t sl = 2 * c + ((u_begin(c, p.units, G) / p.tpr) == s.rh ? 0 : 1);
            const float* pp = p.parts + sl * C::SLOT_FLOATS + NHC * kDCkv;
#pragma unroll
            for (int h = 0; h < NHC; ++h) {
              const float lp = __ldcg(pp + NHC + h);
              if (lp > 0.f) Lt[h] += ptx::ex2(__ldcg(pp + h) - M[h]) * lp;
            }
          }
#pragma unroll
          for (int mt = 0; mt < 4; ++mt) {
            const int d = 128 * mt + 32 * sp + lane;
            float acc[NHC];
#pragma unroll
            for (int h = 0; h < NHC; ++h) acc[h] = 0.f;
            for (int64_t c = c_lo; c <= c_hi; ++c) {
              const int64_t sl = 2 * c + ((u_begin(c, p.units, G) / p.tpr) == s.rh ? 0 : 1);
              const float* pp = p.parts + sl * C::SLOT_FLOATS;
#pragma unroll
              for (int h = 0; h < NHC; ++h) {
                const float lp = __ldcg(pp + NHC * kDCkv + NHC + h);
                if (lp > 0.f) {
                  const float w = ptx::ex2(__ldcg(pp + NHC * kDCkv + h) - M[h]);
                  acc[h] += w * __ldcg(pp + h * kDCkv + d);
                }
              }
            }
#pragma unroll
            for (int h = 0; h < NHC; ++h) {
              const float y = Lt[h] > 0.f ? acc[h] / Lt[h] : 0.f;
              p.out[b * p.out_sb + (int64_t)(head0 + h) * p.out_sh + d] = __float2bfloat16_rn(y);
            }
          }
          if (tid < NHC) {
            const int h = tid;
            p.lse[b * p.lse_sb + (int64_t)(head0 + h) * p.lse_sh] =
                Lt[h] > 0.f ? M[h] + ptx::lg2(Lt[h]) : -INFINITY;
          }
          if (tid == 0) p.counters[s.rh] = 0;
        }
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, (uint32_t)C::TMEM_COLS);
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
    const uint64_t t0 = ptx::globaltimer_ns();
    while (!ptx::mbar_try_wait(b, 0)) {
      if ((int64_t)(ptx::globaltimer_ns() - t0) > timeout_ns) {
        atomicOr(err, (uint32_t)DSA_DEVERR_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
}

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

int nhc_for(int heads) {
  switch (heads) {
    case 16: return 16;
    case 32: return 32;
    case 64: return 64;
    case 128: return 64;
    default: return 0;
  }
}

int slot_floats(int nhc) { return nhc * kDCkv + 2 * nhc; }

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct WsLayout {
  size_t counters_off, parts_off, total;
};

WsLayout ws_layout(int64_t num_rh, int64_t grid, int nhc) {
  WsLayout w;
  w.counters_off = 256;
  w.parts_off = align_up(w.counters_off + (size_t)num_rh * 4, 256);
  w.total = w.parts_off + (size_t)(2 * grid) * (size_t)slot_floats(nhc) * 4;
  return w;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int encode(CUtensorMap* m, const void* base, int rank, const cuuint64_t* dims,
           const cuuint64_t* strides_bytes, const cuuint32_t* box) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return DSA_ERR_DRIVER;
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, (cuuint32_t)rank, const_cast<void*>(base),
                  dims, strides_bytes, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSA_OK : DSA_ERR_DRIVER;
}

template <int NHC>
int launch(const CUtensorMap& ckv, const CUtensorMap& kpe, const CUtensorMap& qn,
           const CUtensorMap& qp, const Params& prm, int grid, int dev, cudaStream_t stream) {
  using C = Cfg<NHC>;
  const int ai = NHC == 16 ? 0 : NHC == 32 ? 1 : 2;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_dev[dev].attr_done[ai]) {
      if (cudaFuncSetAttribute(dsa_decode_kernel<NHC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               C::SMEM_BYTES) != cudaSuccess)
        return DSA_ERR_CUDA;
      g_dev[dev].attr_done[ai] = true;
    }
  }
  dsa_decode_kernel<NHC><<<grid, kThreads, C::SMEM_BYTES, stream>>>(ckv, kpe, qn, qp, prm);
  return cudaGetLastError() == cudaSuccess ? DSA_OK : DSA_ERR_CUDA;
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
    default: return "unknown status";
  }
}

size_t dsa_sparse_mla_decode_workspace_size(int64_t num_tokens, int32_t num_heads, int32_t topk,
                                            int32_t device) {
  const int nhc = nhc_for(num_heads);
  if (nhc == 0 || num_tokens < 0 || topk < 1) return 0;
  const int sms = device_sms(device);
  if (sms <= 0) return 0;
  const int64_t num_rh = num_tokens * (num_heads / nhc);
  const int64_t tpr = (topk + kBK - 1) / kBK;
  const int64_t units = num_rh * tpr;
  const int64_t grid = units < sms ? units : sms;
  return ws_layout(num_rh, grid > 0 ? grid : 1, nhc).total;
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
  if (num_tokens < 0 || topk < 1 || num_slots < 1 || num_slots > INT32_MAX ||
      num_tokens > INT32_MAX)
    return DSA_ERR_INVALID_ARGUMENT;
  const int nhc = nhc_for(num_heads);
  if (nhc == 0) return DSA_ERR_UNSUPPORTED;
  if (num_tokens == 0) return DSA_OK;
  if (!q_nope || !q_pe || !ckv_cache || !kpe_cache || !sparse_indices || !output || !lse)
    return DSA_ERR_INVALID_ARGUMENT;
  if (ckv_slot_stride < kDCkv || kpe_slot_stride < kDKpe || q_nope_stride_h < kDCkv ||
      q_pe_stride_h < kDKpe || q_nope_stride_b < 1 || q_pe_stride_b < 1 || indices_stride_b < topk)
    return DSA_ERR_INVALID_ARGUMENT;
  if (!aligned16(q_nope) || !aligned16(q_pe) || !aligned16(ckv_cache) || !aligned16(kpe_cache) ||
      (q_nope_stride_b * 2) % 16 || (q_nope_stride_h * 2) % 16 || (q_pe_stride_b * 2) % 16 ||
      (q_pe_stride_h * 2) % 16 || (ckv_slot_stride * 2) % 16 || (kpe_slot_stride * 2) % 16)
    return DSA_ERR_MISALIGNED;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DSA_ERR_CUDA;
  const int sms = device_sms(dev);
  if (sms <= 0) return DSA_ERR_CUDA;

  const int hg = num_heads / nhc;
  const int64_t num_rh = num_tokens * hg;
  const int tpr = (topk + kBK - 1) / kBK;
  const int64_t units = num_rh * tpr;
  const int64_t grid = units < sms ? units : sms;
  const WsLayout wl = ws_layout(num_rh, grid, nhc);
  if (!workspace || workspace_bytes < wl.total) return DSA_ERR_WORKSPACE;

  CUtensorMap m_ckv, m_kpe, m_qn, m_qp;
  int rc;
  {
    cuuint64_t dims[2] = {(cuuint64_t)kDCkv, (cuuint64_t)num_slots};
    cuuint64_t str[1] = {(cuuint64_t)ckv_slot_stride * 2};
    cuuint32_t box[2] = {64, 1};
    if ((rc = encode(&m_ckv, ckv_cache, 2, dims, str, box)) != DSA_OK) return rc;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)kDKpe, (cuuint64_t)num_slots};
    cuuint64_t str[1] = {(cuuint64_t)kpe_slot_stride * 2};
    cuuint32_t box[2] = {64, 1};
    if ((rc = encode(&m_kpe, kpe_cache, 2, dims, str, box)) != DSA_OK) return rc;
  }
  {
    cuuint64_t dims[3] = {(cuuint64_t)kDCkv, (cuuint64_t)num_heads, (cuuint64_t)num_tokens};
    cuuint64_t str[2] = {(cuuint64_t)q_nope_stride_h * 2, (cuuint64_t)q_nope_stride_b * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)nhc, 1};
    if ((rc = encode(&m_qn, q_nope, 3, dims, str, box)) != DSA_OK) return rc;
  }
  {
    cuuint64_t dims[3] = {(cuuint64_t)kDKpe, (cuuint64_t)num_heads, (cuuint64_t)num_tokens};
    cuuint64_t str[2] = {(cuuint64_t)q_pe_stride_h * 2, (cuuint64_t)q_pe_stride_b * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)nhc, 1};
    if ((rc = encode(&m_qp, q_pe, 3, dims, str, box)) != DSA_OK) return rc;
  }

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  Params prm;
  prm.idx = sparse_indices;
  prm.idx_sb = indices_stride_b;
  prm.out = static_cast<__nv_bfloat16*>(output);
  prm.out_sb = output_stride_b;
  prm.out_sh = output_stride_h;
  prm.lse = lse;
  prm.lse_sb = lse_stride_b;
  prm.lse_sh = lse_stride_h;
  prm.num_slots = num_slots;
  prm.units = units;
  prm.hg_count = hg;
  prm.topk = topk;
  prm.tpr = tpr;
  prm.scale_log2 = sm_scale * kLog2e;
  prm.err = reinterpret_cast<uint32_t*>(ws);
  prm.counters = reinterpret_cast<int32_t*>(ws + wl.counters_off);
  prm.parts = reinterpret_cast<float*>(ws + wl.parts_off);

  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (nhc) {
    case 16: return launch<16>(m_ckv, m_kpe, m_qn, m_qp, prm, (int)grid, dev, st);
    case 32: return launch<32>(m_ckv, m_kpe, m_qn, m_qp, prm, (int)grid, dev, st);
    default: return launch<64>(m_ckv, m_kpe, m_qn, m_qp, prm, (int)grid, dev, st);
  }
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
