// DSA decode on two-CTA clusters, one head group of one row per work unit: 16 heads for
// H = 16, 32 heads for H = 32, 64, 128 (a row with H heads is H/NH units that gather the
// same slots; the re-gathers of a row's other groups mostly hit L2).
//
// Why a pair: with NH heads the score MMA is S^T[slots x NH] = K . Q^T, whose cost is
// set by the number of MMA instructions (an M=128 MMA costs about as much as an M=64
// one), so a tile should be 128 rows of slots.  A whole 1152-byte slot per row,
// three stages deep (enough to hide the ~2-3 us gather latency under load), does not
// fit in one SM's shared memory.  So each CTA of the pair owns half of every slot:
//   rank r: ckv columns [256r, 256r + 256) (four 64-wide d-blocks, 128-byte swizzle)
//           and kpe columns [32r, 32r + 32) (one 32-wide block, 64-byte swizzle),
// i.e. 576 bytes per slot, three stages of 112 (16 heads) or 96 (32 heads) slots.  Each
// CTA computes a partial score
// over its 288 columns; the two partials are swapped through distributed shared
// memory and both CTAs add them (own + peer: IEEE addition commutes, so both hold
// bit-identical scores and take identical softmax decisions).  Each CTA then runs
// PV over its own 256 value columns: O^T[256 d x NH] += V^T . P^T.
//
// Per CTA (512 threads):
//   warp 0        Q loader: the unit's Q half (4 boxes of [NH x 64] + 1 of [NH x 32]).
//   warps 1-5     gather producers, one per d-block (warp 5: the kpe half); lane g
//                 issues one tile::gather4 (slots 4g..4g+3) per tile.
//   warp 6        score MMA issuer: 18 MMAs (M=128, N=NH) per tile.
//   warp 7        PV MMA issuer: 12 MMAs (M=128, N=NH) per tile.
//                 Two issuers, because an issuer's own shared-memory accesses (its
//                 barrier waits) queue behind the tensor core's operand reads; with one
//                 issuer those stalls, not the tensor core, set the tile period.
//   warps 8-15    softmax / epilogue: warp w reads TMEM lanes 32(w%4).. (slots) and
//                 handles heads (NH/2)((w-8)/4) .. + NH/2 - 1.
// The work split is stream-K over (row, tile) units per pair; a row cut between
// pairs is merged inside this kernel by the pair holding its first tiles (per rank, for
// its value half), after a bounded wait for the other pairs' partials.  Every wait is
// bounded.
#pragma once

namespace dsa {
namespace h16 {

constexpr int kBlk = pipe::kBlk;         // 64-wide ckv d-blocks per CTA
constexpr int kStages = 3;
constexpr int kMaskStride = 8;           // mask words per stage: [0, 4) slot bits, [7] any
constexpr int kMaskAny = pipe::kMaskAny;
constexpr int OFF_KV = 0;
constexpr int kThreads = 512;
constexpr int kQWarp = 0;
constexpr int kProd0 = 1;
constexpr int kProdWarps = pipe::kProdWarps;
constexpr int kMmaWarp = 6;     // score issuer; also allocates TMEM
constexpr int kPvWarp = 7;
constexpr int kSm0 = 8;
constexpr int kSmThreads = 256;
constexpr int kSmWarps = kSmThreads / 32;
constexpr uint32_t kNamedBar = 1;
// Register split after launch (512 threads x 128 = 65536): warpgroups 0-1 (loader,
// producers, MMA issuer) drop to kRegsLow, the two softmax warpgroups rise to kRegsHigh.
constexpr uint32_t kRegsLow = 72;
constexpr uint32_t kRegsHigh = 184;
static_assert(256 * (kRegsLow + kRegsHigh) <= 65536, "register split exceeds the pool");
using pipe::kSw128;
using pipe::kSw64;

// What depends on the head-group width NH (the N of both MMAs): 16 for H = 16, 32 for
// H = 32, 64, 128 (a 128-head row is then 4 units instead of 8, each tile doing twice the
// head work for about the same fixed cost), and the tile size: the score MMA covers 128
// slot rows whatever the tile holds, so 16-head units use 112-slot tiles (a 2048-slot row
// is 19 tiles of 32 MMAs instead of 22 of 30); 32-head units, whose Q half and exchange
// buffers are twice as large, keep 96.  Q is single-buffered (a segment's Q loads once its
// predecessor's last score is done); with 32 heads P has two buffers (softmax waits for
// the PV two tiles back).
template <int NH>
struct Cfg {
  static_assert(NH == 16 || NH == 32, "head group width");
  static constexpr int kTS = NH == 16 ? 112 : 96;  // slots per tile; score MMA rows >= kTS
                                                   // read past the region (never used)
  static constexpr int kRB = kTS * 128;            // one ckv d-block region of a stage
  static constexpr int kRK = kTS * 64;             // the 32-wide kpe region of a stage
  static constexpr int kStageB = kBlk * kRB + kRK;
  static constexpr int kGroups = kTS / 4;          // gather4 copies per d-block per tile
  static constexpr int kPVKs = kTS / 16;           // K steps of one PV MMA chain
  static constexpr int kMaskWords = (kTS + 31) / 32;
  static constexpr int kHT = NH / 2;               // heads per softmax thread
  static constexpr int kQBufs = 1;
  static constexpr int kPBufs = NH == 16 ? kStages : 2;
  static constexpr int kXBufs = 2;                 // partial-score exchange buffers
  static constexpr int kQBlk = NH * 128;           // one [NH x 64] SW128 Q block
  static constexpr int kQB = kBlk * kQBlk + NH * 64;  // + the [NH x 32] SW64 q_pe block
  static constexpr int kPBlk = NH * 128;           // P^T: [NH x 64 slots] bf16 SW128 block
  static constexpr int kPB = 2 * kPBlk;            // P^T [NH x 128 slots], K-major
  static constexpr int kXB = kTS * NH * 4;         // partial scores from the peer (xo_t layout)
  static constexpr int OFF_Q = kStages * kStageB;
  static constexpr int OFF_P = OFF_Q + kQBufs * kQB;
  static constexpr int OFF_X = OFF_P + kPBufs * kPB;
  static constexpr int OFF_BAR = OFF_X + kXBufs * kXB;
  static constexpr int OFF_MASK = OFF_BAR + 512;  // [stage][4] slot-validity words
  static constexpr int OFF_MISC = OFF_MASK + 128;  // [0] TMEM base, [2] abort flag, [3] drain
                                                  // flag, [6] the peer's abort flag (at exit),
                                                  // [8] a split-K merge gave up waiting
  static constexpr int OFF_RED = OFF_MISC + 64;   // [2 hh][4 quadrants][kHT heads] floats
  static_assert(kTS % 16 == 0 && kTS <= 128 && kGroups <= 32 && kMaskWords <= 4, "tile shape");
  static constexpr int SMEM_USED = OFF_RED + 2 * 4 * kHT * 4;
  static constexpr int SMEM_BYTES = SMEM_USED + 1024;
  static constexpr int TMEM_COLS = NH == 16 ? 64 : 128;
  static constexpr int S_COL = 0;        // two score buffers x NH columns
  static constexpr int O_COL = 2 * NH;   // two 128-d tiles x NH columns
  static constexpr int kSlotFloats = NH * kDCkv + 2 * NH;  // split-K partial: O, m, l

  static_assert(OFF_Q % 1024 == 0 && OFF_P % 1024 == 0 && kStageB % 1024 == 0 &&
                    kQB % 1024 == 0 && kPB % 1024 == 0,
                "128-byte swizzle atoms need 1024-byte alignment");
  static_assert((kBlk * kRB) % 512 == 0 && (kBlk * kQBlk) % 512 == 0,
                "64-byte swizzle atoms need 512-byte alignment");
  static_assert(SMEM_BYTES <= 232448, "shared memory budget");
  static_assert(kHT % 8 == 0, "softmax threads move heads in groups of 8 columns");
};

enum : int {
  B_KVF = 0,                     // [stage] landed: one arrive (with its bytes) per producer
                                 // warp; d-block 0's warp writes the slot masks first
  B_KVE = B_KVF + kStages,       // [stage][5] d-block region free again: the kpe region once
                                 // the score has read it, value d-blocks 0-1 / 2-3 once
                                 // their PV half has
  B_QF = B_KVE + kStages * 5, B_QE = B_QF + 2,
  B_SF = B_QE + 2, B_SE = B_SF + 2,  // score buffer full / read
  B_PF = B_SE + 2, B_PD = B_PF + 2,  // P written (+ O rescaled) / PV done
  B_XF = B_PD + 2,               // [kXBufs] the peer's partial scores are in X[b]
                                 // (complete_tx)
  B_OF = B_XF + 4,               // the epilogue has read O
  B_DRAIN = B_OF + 1,            // [2] used only when an issuer stops early
  B_COUNT = B_DRAIN + 2
};
__host__ __device__ constexpr int kve(int stage, int blk) { return B_KVE + stage * kProdWarps + blk; }
// Byte offset of the partial scores of slot `slot`, heads kHT*hh + c .. + 3 (c a multiple of
// 4) in an exchange buffer X: [head half hh][head quad c / 4][slot] float4, so that the 32
// slots of a warp write and read 512 contiguous bytes (four wavefronts per instruction).
template <int kTS, int kHT>
__device__ __forceinline__ uint32_t xo_t(int slot, int hh, int c) {
  return (uint32_t)(((hh * (kHT / 4) + (c >> 2)) * kTS + slot) * 16);
}
// The exchange buffers X need no "empty" barrier.  A thread sends its partial of tile j
// (into the peer's X[j % 2]) only after it finished tile j - 1, whose X wait needed every
// peer thread's partial of tile j - 1; a peer thread sends that only after it finished
// tile j - 2.  So X[j % 2] is rewritten only after both sides have read it for tile j - 2.

static_assert(B_COUNT * 8 <= 512, "barrier block");
static_assert(kStages * kMaskStride * 4 <= 128, "mask words");

using pipe::desc;

// Two bf16 (round to nearest), `lo` in the low half: two adjacent slots of one P^T row.
__device__ __forceinline__ uint32_t pack_p2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// kPaged: sparse_indices holds token positions, translated through the page table by the
// gather producers (ids are fetched two tiles ahead so the dependent page-table load is off
// the producer's path).
template <int NH, bool kPaged>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    dsa_decode_h16_kernel(const __grid_constant__ CUtensorMap tm_ckv,
                          const __grid_constant__ CUtensorMap tm_kpe,
                          const __grid_constant__ CUtensorMap tm_qn,
                          const __grid_constant__ CUtensorMap tm_qp,
                          const __grid_constant__ Params p) {
  using C = Cfg<NH>;
  constexpr int kHT = C::kHT, kQBufs = C::kQBufs, kPBufs = C::kPBufs, kXBufs = C::kXBufs;
  constexpr int kQB = C::kQB, kPB = C::kPB, kXB = C::kXB;
  constexpr int OFF_Q = C::OFF_Q, OFF_P = C::OFF_P, OFF_X = C::OFF_X, OFF_BAR = C::OFF_BAR;
  constexpr int OFF_MASK = C::OFF_MASK, OFF_MISC = C::OFF_MISC, OFF_RED = C::OFF_RED;
  constexpr int TMEM_COLS = C::TMEM_COLS, S_COL = C::S_COL, O_COL = C::O_COL;
  constexpr int kSlotFloats = C::kSlotFloats;
  constexpr int kTS = C::kTS, kRB = C::kRB, kStageB = C::kStageB;
  constexpr int kPVKs = C::kPVKs;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = ptx::smem_u32(smem_raw);
  const uint32_t sbase = (raw_addr + 1023u) & ~1023u;
  uint8_t* sgen = smem_raw + (sbase - raw_addr);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_ctarank();
  const uint32_t peer = rank ^ 1u;
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(sgen + OFF_MISC);
  volatile uint32_t* masks = reinterpret_cast<volatile uint32_t*>(sgen + OFF_MASK);
  float* red = reinterpret_cast<float*>(sgen + OFF_RED);
  const uint32_t bar0 = sbase + (uint32_t)OFF_BAR;
#define bar(k) (bar0 + 8u * (uint32_t)(k))

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(bar(B_KVF + s), kProdWarps);
      for (int j = 0; j < kProdWarps; ++j) ptx::mbar_init(bar(kve(s, j)), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar(B_QF + b), 1);
      ptx::mbar_init(bar(B_QE + b), 1);
      ptx::mbar_init(bar(B_SF + b), 1);
      ptx::mbar_init(bar(B_SE + b), kSmWarps);  // one arrive per softmax warp
      ptx::mbar_init(bar(B_PF + b), kSmWarps);
      ptx::mbar_init(bar(B_PD + b), 1);
    }
    // X[b] is full once this CTA armed it (one arrive with the expected bytes) and the
    // peer's st.async bytes landed; the peer's stores may come before the arming.
    for (int b = 0; b < kXBufs; ++b) ptx::mbar_init(bar(B_XF + b), 1);
    ptx::mbar_init(bar(B_OF), kSmWarps);
    ptx::mbar_init(bar(B_DRAIN), 1);
    ptx::mbar_init(bar(B_DRAIN + 1), 1);
    misc[2] = 0;
    misc[3] = 0;
    misc[6] = 0;
    misc[8] = 0;
    ptx::fence_mbar_init();
    for (int b = 0; b < kXBufs; ++b) ptx::mbar_arrive_expect_tx(bar(B_XF + b), (uint32_t)kXB);
  }
  if (warp == kQWarp && lane == 0) {
    ptx::prefetch_tmap(&tm_ckv);
    ptx::prefetch_tmap(&tm_kpe);
    ptx::prefetch_tmap(&tm_qn);
    ptx::prefetch_tmap(&tm_qp);
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(sbase + (uint32_t)OFF_MISC, (uint32_t)TMEM_COLS);
    ptx::tmem_relinquish();
  }
  // Both CTAs' barriers are initialised before either arrives on the other's.
  ptx::tc_fence_before();
  ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem = misc[0];
  // Launched with programmatic stream serialization: the set-up above overlapped the
  // previous grid's tail; nothing in global memory is touched before that grid is done.
  ptx::grid_dep_wait();
  ptx::launch_dependents();

  const int64_t pair = blockIdx.x >> 1;
  const int64_t G = gridDim.x >> 1;
  const int64_t u_lo = u_begin(pair, p.units, G);
  const int64_t u_hi = u_begin(pair + 1, p.units, G);
  const Waiter wait{misc + 2, p.err, p.wait_cycles};

  if (warp == kQWarp) {
    // ------------------------------------------------------------------ Q loader
    ptx::regs_dec<kRegsLow>();
    if (lane == 0)
      pipe::q_loader<NH>(p, &tm_qn, &tm_qp, rank, sbase + (uint32_t)OFF_Q, bar(B_QF), bar(B_QE),
                         u_lo, u_hi, wait, misc + 3);
    __syncwarp();
  } else if (warp >= kProd0 && warp < kProd0 + kProdWarps) {
    // ------------------------------------------------------------------ gather producers
    ptx::regs_dec<kRegsLow>();
    pipe::gather_producer<kTS, kStageB, kStages, kMaskStride, kPaged>(
        p, &tm_ckv, &tm_kpe, warp - kProd0, lane, rank, sbase + (uint32_t)OFF_KV, masks, bar(B_KVF),
        bar(B_KVE), u_lo, u_hi, wait, misc + 3);
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ score MMA issuer
    ptx::regs_dec<kRegsLow>();
    if (lane == 0) {
      const Waiter wait{misc + 2, p.err, p.wait_cycles, true};
      constexpr uint32_t kIdS = idesc_bf16(128, NH, false);
      // Descriptors of offset 0; an operand at byte offset o adds o >> 4.
      const uint64_t dk = desc(sbase + (uint32_t)OFF_KV, 16, 1024, kSw128);
      const uint64_t dkp = desc(sbase + (uint32_t)(OFF_KV + kBlk * kRB), 16, 512, kSw64);
      const uint64_t dq = desc(sbase + (uint32_t)OFF_Q, 16, 1024, kSw128);
      const uint64_t dqp = desc(sbase + (uint32_t)(OFF_Q + kBlk * C::kQBlk), 16, 512, kSw64);
      int64_t i = 0;
      int seg = 0;
      bool ok = true;
      int64_t u = u_lo;
      Segment s;
      while (ok && next_segment(u, u_hi, p.tpr, s)) {
        const int qb = seg % kQBufs;
        const uint64_t qo = (uint64_t)((qb * kQB) >> 4);
        for (int t = s.t0; t < s.t1; ++t, ++i) {
          const int st = (int)(i % kStages);
          const int sb = (int)(i & 1);
          if (t == s.t0) ok = wait(bar(B_QF + qb), (uint32_t)((seg / kQBufs) & 1));
          ok = ok && wait(bar(B_SE + sb), (uint32_t)(((i >> 1) & 1) ^ 1));
          ok = ok && wait(bar(B_KVF + st), (uint32_t)((i / kStages) & 1));
          if (!ok) break;
          // Partial S^T[128 x 16] over this CTA's 288 columns.  An all-padding tile
          // skips its MMAs (its scores are all masked).
          if (masks[st * kMaskStride + kMaskAny] != 0u) {
            ptx::tc_fence_after();
            const uint32_t d_s = tmem + (uint32_t)(S_COL + NH * sb);
            const uint64_t ko = (uint64_t)((st * kStageB) >> 4);
#pragma unroll
            for (int j = 0; j < kBlk; ++j)
#pragma unroll
              for (int ks = 0; ks < 4; ++ks)
                ptx::umma_bf16(d_s, dk + ko + (uint64_t)((j * kRB + ks * 32) >> 4),
                               dq + qo + (uint64_t)((j * C::kQBlk + ks * 32) >> 4), kIdS,
                               (j | ks) ? 1u : 0u);
#pragma unroll
            for (int ks = 0; ks < 2; ++ks)
              ptx::umma_bf16(d_s, dkp + ko + (uint64_t)((ks * 32) >> 4),
                             dqp + qo + (uint64_t)((ks * 32) >> 4), kIdS, 1u);
          }
          ptx::umma_commit(bar(B_SF + sb));
          ptx::umma_commit(bar(kve(st, kBlk)));  // the kpe region is read only by the score
          if (t == s.t1 - 1) ptx::umma_commit(bar(B_QE + qb));
        }
        ++seg;
      }
      if (!ok) {
        const Waiter drain{misc + 3, p.err, p.wait_cycles};
        ptx::umma_commit(bar(B_DRAIN));
        drain(bar(B_DRAIN), 0);
      }
    }
    __syncwarp();
  } else if (warp == kPvWarp) {
    // ------------------------------------------------------------------ PV MMA issuer
    // O^T[256 x 16] (+)= V^T . P^T over this CTA's value half, once softmax has written
    // P (and rescaled O); then the stage goes back to the producers.  The first PV of a
    // segment waits until the previous segment's epilogue has read O.
    ptx::regs_dec<kRegsLow>();
    if (lane == 0) {
      const Waiter wait{misc + 2, p.err, p.wait_cycles, true};
      constexpr uint32_t kIdPV = idesc_bf16(128, NH, true);
      const uint64_t dv = desc(sbase + (uint32_t)OFF_KV, kRB, 1024, kSw128);
      const uint64_t dp = desc(sbase + (uint32_t)OFF_P, 16, 1024, kSw128);
      int64_t j = 0;
      int seg = 0;
      bool ok = true;
      bool o_init = false;
      int64_t u = u_lo;
      Segment s;
      while (ok && next_segment(u, u_hi, p.tpr, s)) {
        for (int t = s.t0; t < s.t1; ++t, ++j) {
          const int st = (int)(j % kStages);
          ok = wait(bar(B_PF + (int)(j & 1)), (uint32_t)((j >> 1) & 1));
          if (ok && t == s.t0) {
            if (seg > 0) ok = wait(bar(B_OF), (uint32_t)((seg - 1) & 1));
            o_init = false;
          }
          if (!ok) break;
          if (masks[st * kMaskStride + kMaskAny] != 0u) {
            ptx::tc_fence_after();
            const uint64_t vo = (uint64_t)((st * kStageB) >> 4);
            const uint64_t po = (uint64_t)(((int)(j % kPBufs) * kPB) >> 4);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
#pragma unroll
              for (int ks = 0; ks < kPVKs; ++ks)
                ptx::umma_bf16(tmem + (uint32_t)(O_COL + NH * mt),
                               dv + vo + (uint64_t)((2 * mt * kRB + ks * 2048) >> 4),
                               dp + po + (uint64_t)(((ks >> 2) * C::kPBlk + (ks & 3) * 32) >> 4),
                               kIdPV, (o_init || ks > 0) ? 1u : 0u);
              // value d-blocks 2mt, 2mt+1 are free once this half's MMAs are done
              ptx::umma_commit(bar(kve(st, 2 * mt)));
              ptx::umma_commit(bar(kve(st, 2 * mt + 1)));
            }
            o_init = true;
          } else {
            for (int jb = 0; jb < kBlk; ++jb) ptx::umma_commit(bar(kve(st, jb)));
          }
          ptx::umma_commit(bar(B_PD + (int)(j & 1)));
        }
        ++seg;
      }
      if (!ok) {
        const Waiter drain{misc + 3, p.err, p.wait_cycles};
        ptx::umma_commit(bar(B_DRAIN + 1));
        drain(bar(B_DRAIN + 1), 0);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax / epilogue
    ptx::regs_inc<kRegsHigh>();
    const int qd = warp & 3;               // TMEM lane quadrant = slots 32qd .. 32qd+31
    const int hh = (warp - kSm0) >> 2;     // heads kHT*hh .. kHT*hh + kHT-1
    const int slot = 32 * qd + lane;
    const bool slot_ok = slot < kTS;
    const uint32_t lane_base = (uint32_t)(32 * qd) << 16;
    const uint32_t x_own = sbase + (uint32_t)OFF_X;
    const uint32_t x_peer = ptx::mapa(x_own, peer);
    const uint32_t xf_peer = ptx::mapa(bar(B_XF), peer);
    float* red_max = red;
    int64_t i = 0;
    bool aborted = false;
    int64_t u = u_lo;
    Segment s;
    float m_run[kHT], l_part[kHT];
    // ---------------------------------------------------------------- epilogue
    // A segment's output (or split-K partial / merge), from O in TMEM and the segment's
    // running max em and sums el.  Every thread votes in it, also one that gave up earlier;
    // returns false when the CTA gave up.
    auto finish = [&](const Segment& es, const float (&em)[kHT], const float (&el)[kHT],
                      int64_t eil) -> bool {
      // PV done for tile eil is a parity wait on B_PD[eil & 1], which is also the barrier
      // of tile eil - 2: if PV(eil - 2) were still running, that barrier would sit in the
      // phase of the opposite parity and the wait would pass at once.  PV completes in
      // order and PV(eil - 3) is done (tile eil's stage was refilled after it), so wait for
      // PV(eil - 1) first: then PV(eil - 2) is done and the wait for PV(eil) is exact.
      // (The next segment's PV cannot start before this epilogue has read O.)

        bool okw = !aborted;
        if (okw && eil >= 1)
          okw = wait(bar(B_PD + (int)((eil - 1) & 1)), (uint32_t)(((eil - 1) >> 1) & 1));
        okw = okw && wait(bar(B_PD + (int)(eil & 1)), (uint32_t)((eil >> 1) & 1));
        if (ptx::bar_red_or(kNamedBar, kSmThreads, aborted || !okw)) {
          aborted = true;
          return false;
        }
        ptx::tc_fence_after();
        float* red_sum = red;  // the max slots are free again: every thread passed the vote
#pragma unroll
        for (int h = 0; h < kHT; ++h) {
          float v = el[h];
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
          if (lane == 0) red_sum[(hh * 4 + qd) * kHT + h] = v;
        }
        ptx::bar_sync(kNamedBar, kSmThreads);
        float L[kHT];
#pragma unroll
        for (int h = 0; h < kHT; ++h) {
          const float* r4 = red_sum + hh * 4 * kHT + h;
          L[h] = (r4[0] + r4[kHT]) + (r4[2 * kHT] + r4[3 * kHT]);
        }
        const int64_t rh = es.rh;                        // (row, NH-head group)
        const int64_t b = rh >> p.hg_shift;
        const int h0 = NH * (int)(rh & ((1 << p.hg_shift) - 1));   // first head of the group
        const bool full = (es.t0 == 0 && es.t1 == p.tpr);
        // A row cut between pairs: the pair holding its first tiles (the head, p_lo) ends
        // its range with them; the others start theirs with the rest and so finish early.
        // They write their partial and count themselves; the head waits for the count and
        // merges from its own O in TMEM, so it writes no partial and no fence delays it.
        const int64_t p_lo = full ? pair : cta_of(rh * p.tpr, p.units, G);
        const int64_t p_hi = full ? pair : cta_of((rh + 1) * p.tpr - 1, p.units, G);
        const bool head = full || pair == p_lo;
        // a pair writes a partial only for the row its range starts inside: one slot each
        float* part = p.parts + pair * kSlotFloats;
        float o_mine[2][kHT];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt) {
          uint32_t rr[kHT];
#pragma unroll
          for (int c = 0; c < kHT; c += 8)
            ptx::tmem_ld8(tmem + lane_base + (uint32_t)(O_COL + NH * mt + kHT * hh + c), rr + c);
          ptx::tmem_wait_ld();
          const int d = (int)(256 * rank) + 128 * mt + 32 * qd + lane;
#pragma unroll
          for (int h = 0; h < kHT; ++h) {
            const float o = __uint_as_float(rr[h]);
            o_mine[mt][h] = o;
            const int head_idx = kHT * hh + h;
            if (full)
              p.out[b * p.out_sb + (int64_t)(h0 + head_idx) * p.out_sh + d] =
                  __float2bfloat16_rn(L[h] > 0.f ? o / L[h] : 0.f);
            else if (!head)
              part[head_idx * kDCkv + d] = o;
          }
        }
        if (qd == 0 && lane < kHT) {
          float mh = 0.f, lh = 0.f;  // unrolled select keeps m_run / L in registers
#pragma unroll
          for (int h = 0; h < kHT; ++h)
            if (h == lane) {
              mh = em[h];
              lh = L[h];
            }
          const int head_idx = kHT * hh + lane;
          if (full) {
            if (rank == 0)
              p.lse[b * p.lse_sb + (int64_t)(h0 + head_idx) * p.lse_sh] =
                  lh > 0.f ? mh + ptx::lg2(lh) : -INFINITY;
          } else if (!head) {
            // both ranks write the (identical) scalars, so each rank's merge finds them
            part[NH * kDCkv + head_idx] = mh;
            part[NH * kDCkv + NH + head_idx] = lh;
          }
        }
        uint32_t* cnt = p.counters + 2 * p_lo + rank;
        if (!full && !head) {
          // every thread's partial stores, then one release add (cumulative over the barrier)
          ptx::bar_sync(kNamedBar, kSmThreads);
          if (warp == kSm0 && lane == 0) ptx::red_release_gpu_add(cnt, 1u);
        } else if (!full) {
          if (warp == kSm0 && lane == 0) {
            // Bounded wait for the other parts of the row (all pairs are co-resident); the
            // acquire load orders the partial reads after it (through the barrier below).
            const uint32_t want = (uint32_t)(p_hi - p_lo);
            const uint64_t t0 = ptx::cycles();
            uint32_t got = ptx::ld_acquire_gpu(cnt);
            uint32_t lost = 0;
            while (got != want) {
              if (ptx::cycles() - t0 > p.wait_cycles || misc[2]) {
                misc[2] = 1;
                lost = 1;
                atomicOr(p.err, (uint32_t)DSA_DEVERR_TIMEOUT);
                break;
              }
              __nanosleep(32);
              got = ptx::ld_acquire_gpu(cnt);
            }
            misc[8] = lost;
          }
          ptx::bar_sync(kNamedBar, kSmThreads);
          // A merge that gave up would combine whatever partials are there: the row is
          // written as NaN instead, next to the timeout bit in the error word.
          const bool lost = misc[8] != 0u;
          float M[kHT], Lt[kHT], acc[2][kHT];
#pragma unroll
          for (int h = 0; h < kHT; ++h) {
            M[h] = em[h];
            Lt[h] = L[h];
            acc[0][h] = o_mine[0][h];
            acc[1][h] = o_mine[1][h];
          }
          for (int64_t cc = p_lo + 1; cc <= p_hi; ++cc) {
            // a later pair's range starts inside this row: its partial is in its slot
            const float* pp = p.parts + cc * kSlotFloats;
            float pm[kHT], pl[kHT], po[2][kHT];
            // every load of the part first, so that the part costs one L2 round trip
#pragma unroll
            for (int h = 0; h < kHT; ++h) {
              const int head_idx = kHT * hh + h;
              pm[h] = __ldcg(pp + NH * kDCkv + head_idx);
              pl[h] = __ldcg(pp + NH * kDCkv + NH + head_idx);
#pragma unroll
              for (int mt = 0; mt < 2; ++mt)
                po[mt][h] = __ldcg(pp + head_idx * kDCkv + (int)(256 * rank) + 128 * mt + 32 * qd + lane);
            }
#pragma unroll
            for (int h = 0; h < kHT; ++h) {
              // A part with l == 0 saw only padding; its O (maybe stale) is not used.
              const bool live = pl[h] > 0.f;
              const bool have = Lt[h] > 0.f;
              const float mn = !live ? M[h] : (!have ? pm[h] : fmaxf(M[h], pm[h]));
              const float keep = have ? ptx::ex2(M[h] - mn) : 0.f;
              const float w = live ? ptx::ex2(pm[h] - mn) : 0.f;
              Lt[h] = (have ? Lt[h] * keep : 0.f) + (live ? w * pl[h] : 0.f);
#pragma unroll
              for (int mt = 0; mt < 2; ++mt)
                acc[mt][h] = (have ? acc[mt][h] * keep : 0.f) + (live ? w * po[mt][h] : 0.f);
              M[h] = mn;
            }
          }
#pragma unroll
          for (int mt = 0; mt < 2; ++mt) {
            const int d = (int)(256 * rank) + 128 * mt + 32 * qd + lane;
#pragma unroll
            for (int h = 0; h < kHT; ++h)
              p.out[b * p.out_sb + (int64_t)(h0 + kHT * hh + h) * p.out_sh + d] =
                  lost ? __float2bfloat16_rn(NAN)
                       : __float2bfloat16_rn(Lt[h] > 0.f ? acc[mt][h] / Lt[h] : 0.f);
          }
          if (rank == 0 && qd == 0 && lane < kHT) {
            float mh = 0.f, lh = 0.f;
#pragma unroll
            for (int h = 0; h < kHT; ++h)
              if (h == lane) {
                mh = M[h];
                lh = Lt[h];
              }
            p.lse[b * p.lse_sb + (int64_t)(h0 + kHT * hh + lane) * p.lse_sh] =
                lost ? NAN : (lh > 0.f ? mh + ptx::lg2(lh) : -INFINITY);
          }
          // every part has been counted and read: the counter is ready for the next call
          if (warp == kSm0 && lane == 0) *reinterpret_cast<volatile uint32_t*>(cnt) = 0u;
        }
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(B_OF));
      return true;
    };
    // 16-head units run a segment's epilogue one tile into the next segment, so the
    // segment's last PVs have drained by then instead of being waited for (with 32 heads
    // the saved sums would not fit the softmax warps' registers)
    constexpr bool kDefer = NH == 16;
    bool pending = false;
    Segment ps;
    float pm_run[kHT], pl_part[kHT];
    int64_t pil = 0;
    while (!aborted && next_segment(u, u_hi, p.tpr, s)) {
#pragma unroll
      for (int h = 0; h < kHT; ++h) {
        m_run[h] = -INFINITY;
        l_part[h] = 0.f;
      }
      bool o_valid = false;
      // Two halves per tile: A(i) reads tile i's partial scores from TMEM and sends them to
      // the peer; B(i) waits for the peer's partial, runs the online softmax and writes P.
      uint32_t own_prev[kHT];  // the in-flight tile's own partial scores
      auto fetch_send = [&](int64_t ic, uint32_t* own) -> bool {
        const int st = (int)(ic % kStages);
        const int sb = (int)(ic & 1);
        const int xb = (int)(ic % kXBufs);
        const bool ok = !aborted && wait(bar(B_KVF + st), (uint32_t)((ic / kStages) & 1)) &&
                        wait(bar(B_SF + sb), (uint32_t)((ic >> 1) & 1));
        ptx::tc_fence_after();
#pragma unroll
        for (int c = 0; c < kHT; c += 8)
          ptx::tmem_ld8(tmem + lane_base + (uint32_t)(S_COL + NH * sb + kHT * hh + c), own + c);
        ptx::tmem_wait_ld();
        ptx::tc_fence_before();
        // One arrive per warp (a barrier arrive is an atomic on one shared word: 256 of them
        // would serialise); the warp's lanes agree first.
        if (__all_sync(0xffffffffu, ok) && lane == 0) ptx::mbar_arrive(bar(B_SE + sb));
        // st.async our partial into the peer's X[xb], completing its B_XF[xb] by bytes.
        if (ok && slot_ok) {
          const uint32_t a = x_peer + (uint32_t)(xb * kXB);
          const uint32_t xfb = xf_peer + 8u * (uint32_t)xb;
#pragma unroll
          for (int c = 0; c < kHT; c += 4)
            ptx::st_async_v4(a + xo_t<kTS, kHT>(slot, hh, c), own[c], own[c + 1], own[c + 2], own[c + 3],
                             xfb);
        }
        return ok;
      };
      // a segment is never empty: A of its first tile, then per tile B(ip) and A(ip + 1)
      bool ok_prev = fetch_send(i, own_prev);
      int64_t ip = i++;  // the tile in flight
      for (int t = s.t0 + 1;; ++t) {
        const bool more = t < s.t1;
        {
          // ------------------------------------------------ B(ip): finish the tile in flight
          const int st = (int)(ip % kStages);
          const int xb = (int)(ip % kXBufs);
          const uint32_t mw = qd < C::kMaskWords ? masks[st * kMaskStride + qd] : 0u;
          const bool live = masks[st * kMaskStride + kMaskAny] != 0u;
          const bool valid = slot_ok && ((mw >> lane) & 1u);
            bool ok = ok_prev && wait(bar(B_XF + xb), (uint32_t)((ip / kXBufs) & 1));
            float x[kHT];
            bool need = false;
            {
              float pr[kHT];
#pragma unroll
              for (int c = 0; c < kHT; c += 4) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                if (slot_ok)
                  v = *reinterpret_cast<const float4*>(
                      sgen + OFF_X + xb * kXB + xo_t<kTS, kHT>(slot, hh, c));
                pr[c] = v.x;
                pr[c + 1] = v.y;
                pr[c + 2] = v.z;
                pr[c + 3] = v.w;
              }
              // X[xb] is read: re-arm it for tile ip + kXBufs.
              if (warp == kSm0 && lane == 0) ptx::mbar_arrive_expect_tx(bar(B_XF + xb), (uint32_t)kXB);
#pragma unroll
              for (int h = 0; h < kHT; ++h) {
                x[h] = valid ? (__uint_as_float(own_prev[h]) + pr[h]) * p.scale_log2 : -INFINITY;
                need |= x[h] > m_run[h] + kTau;
              }
            }
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
              for (int h = 0; h < kHT; ++h) {
                float v = x[h];
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
                if (lane == 0) red_max[(hh * 4 + qd) * kHT + h] = v;
              }
              ptx::bar_sync(kNamedBar, kSmThreads);
              float alpha[kHT];
#pragma unroll
              for (int h = 0; h < kHT; ++h) {
                const float* r4 = red_max + hh * 4 * kHT + h;
                const float mt = fmaxf(fmaxf(r4[0], r4[kHT]), fmaxf(r4[2 * kHT], r4[3 * kHT]));
                const float mn = fmaxf(m_run[h], mt);
                alpha[h] = (m_run[h] == -INFINITY) ? 0.f : ptx::ex2(m_run[h] - mn);
                l_part[h] *= alpha[h];
                m_run[h] = mn;
              }
              if (o_valid) {
                // the outcome is made warp-uniform: the TMEM loads and stores below are
                // warp-collective, and a warp continues or stops as one
                const bool wok = wait(bar(B_PD + (int)((ip - 1) & 1)), (uint32_t)(((ip - 1) >> 1) & 1));
                if (!__all_sync(0xffffffffu, wok)) {
                  aborted = true;
                } else {
                  ptx::tc_fence_after();
#pragma unroll
                  for (int mt = 0; mt < 2; ++mt) {
                    const uint32_t ta = tmem + lane_base + (uint32_t)(O_COL + NH * mt + kHT * hh);
                    uint32_t rr[kHT];
#pragma unroll
                    for (int c = 0; c < kHT; c += 8) ptx::tmem_ld8(ta + (uint32_t)c, rr + c);
                    ptx::tmem_wait_ld();
#pragma unroll
                    for (int h = 0; h < kHT; ++h)
                      rr[h] = __float_as_uint(__uint_as_float(rr[h]) * alpha[h]);
#pragma unroll
                    for (int c = 0; c < kHT; c += 8) ptx::tmem_st8(ta + (uint32_t)c, rr + c);
                  }
                  ptx::tmem_wait_st();
                }
              }
            }
            if constexpr (kPBufs < kStages) {
              // Fewer P buffers than stages: P[i % kPBufs] was last read by the PV of tile
              // i - kPBufs, which must be done before it is overwritten (warp-uniform outcome).
              if (live && ip >= kPBufs && !aborted) {
                const int64_t iq = ip - kPBufs;
                const bool wok = wait(bar(B_PD + (int)(iq & 1)), (uint32_t)((iq >> 1) & 1));
                if (!__all_sync(0xffffffffu, wok)) aborted = true;
              }
            }
            if (!aborted) {  // else the next vote ends the loop for every thread
              uint8_t* pbuf = sgen + OFF_P + (int)(ip % kPBufs) * kPB + (slot >> 6) * C::kPBlk;
              float pv[kHT];
#pragma unroll
              for (int h = 0; h < kHT; ++h) {
                const float me = (m_run[h] == -INFINITY) ? 0.f : m_run[h];
                pv[h] = ptx::ex2(x[h] - me);
                l_part[h] += pv[h];
              }
              // P^T rows are heads: a 4-byte word holds one head's two adjacent slots.  Per
              // pair of heads (h, h + 1) a lane pair swaps one value, then the even lane writes
              // head h's word and the odd lane head h + 1's (four stores instead of eight
              // 2-byte stores that shared words)
              const bool odd = (lane & 1) != 0;
#pragma unroll
              for (int h = 0; h < kHT; h += 2) {
                const float r = __shfl_xor_sync(0xffffffffu, odd ? pv[h] : pv[h + 1], 1);
                if (live && slot_ok) {
                  const int hw = kHT * hh + h + (odd ? 1 : 0);
                  const uint32_t w = odd ? pack_p2(r, pv[h + 1]) : pack_p2(pv[h], r);
                  *reinterpret_cast<uint32_t*>(pbuf + sw128_off(hw, (slot & 63) & ~1)) = w;
                }
              }
              ptx::fence_proxy_async_smem();
              ptx::tc_fence_before();
              __syncwarp();
              if (lane == 0) ptx::mbar_arrive(bar(B_PF + (int)(ip & 1)));
              o_valid = o_valid || live;
            }
        }
        if (pending) {  // the previous segment's epilogue, now that its PVs have drained
          pending = false;
          if (!finish(ps, pm_run, pl_part, pil)) break;
        }
        if (!more) break;
        ok_prev = fetch_send(i, own_prev);  // own_prev is dead after B(ip)
        ip = i++;
      }
      if (aborted) break;
      if constexpr (kDefer) {
        ps = s;
#pragma unroll
        for (int h = 0; h < kHT; ++h) {
          pm_run[h] = m_run[h];
          pl_part[h] = l_part[h];
        }
        pil = i - 1;
        pending = true;
      } else {
        if (!finish(s, m_run, l_part, i - 1)) break;
      }
    }
    if (pending && !aborted) finish(ps, pm_run, pl_part, pil);
  }

  ptx::tc_fence_before();
  __syncthreads();
  // Neither CTA leaves while the other may still write its exchange buffer.  On the normal
  // path every partial sent was also received.  After a CTA gave up on a wait, the peer may
  // have sent partials it never waited for: once both CTAs are past their loops (no more
  // sends), let those in-flight stores land before either CTA exits.
  // Each CTA tells the other whether it gave up (both are alive until the first barrier),
  // so that both take the same exit path.
  if (threadIdx.x == 0)
    ptx::st_cluster_u32(ptx::mapa(sbase + (uint32_t)(OFF_MISC + 6 * 4), peer), misc[2]);
  ptx::cluster_sync();
  if (misc[2] | misc[6]) {
    if (threadIdx.x == 0) {
      const uint64_t t0 = ptx::cycles();
      while (ptx::cycles() - t0 < 200000ull) __nanosleep(256);  // ~0.1 ms >> store latency
    }
    __syncthreads();
    ptx::cluster_sync();
  }
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, (uint32_t)TMEM_COLS);
  }
#undef bar
}

}  // namespace h16
}  // namespace dsa
