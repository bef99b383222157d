// DSA decode of 128-head rows with the heads as the MMA's M dimension.  A work unit is one
// row (all 128 heads) and one tile of 64 slots, so each selected slot is gathered once for
// all heads (the 16/32-head kernel would gather a 128-head row four times) and both MMAs run
// at M = 128:
//   score  S[128 heads x 64 slots] = Q[128 x 288] . K[64 x 288]^T   (N = 64, 18 MMAs)
//   PV     O[128 heads x 256 d]   += P[128 x 64] . V[64 x 256]      (N = 256, 4 MMAs)
// on a two-CTA cluster that splits every slot's 576 columns as the other kernel does
// (rank r: ckv [256r, 256r + 256), kpe [32r, 32r + 32)): each CTA computes a partial score
// over its 288 columns, the partials of a tile (32 KB) are swapped through distributed
// shared memory and both CTAs add them (own + peer, the same bits on both sides), and each
// CTA accumulates O over its own 256 value columns.  P (bf16) never leaves the SM: the
// softmax threads write it to tensor memory, from where the PV MMA reads it as operand A.
//
// Per CTA (512 threads):
//   warp 0        Q loader: the row's Q half, [128 x 288] (72 KB)
//   warps 1-5     gather producers (pipe::gather_producer), 16 gather4 per warp per tile
//   warp 6        score MMA issuer (also allocates tensor memory)
//   warp 7        PV MMA issuer
//   warps 8-11    partial-score senders: warp w streams heads 32 (w % 4) .. + 31 (its TMEM
//                 lane quadrant) of every tile's partial S into the peer's exchange buffer
//   warps 12-15   softmax / epilogue: thread = one head (TMEM lane) over all 64 slots of a
//                 tile; the exchange of tile i + 1 runs while these warps finish tile i
// Tensor memory (512 columns): S [2][64] at 0, P [2][32] (bf16 pairs) at 128, O [256] at 256.
// The work split is stream-K over (row, tile) units on the persistent grid; a row cut
// between pairs is merged inside the kernel, as in the 16/32-head kernel.
#pragma once

namespace dsa {
namespace hm {

constexpr int NH = 128;                   // heads of a row = the MMAs' M
constexpr int kTS = 48;                   // slots per tile = the score MMA's N
constexpr int kStages = 3;
constexpr int kBlk = pipe::kBlk;
constexpr int kProdWarps = pipe::kProdWarps;
constexpr int kMaskAny = pipe::kMaskAny;
constexpr int kMaskStride = 8;
constexpr int kThreads = 512;
constexpr int kQWarp = 0, kProd0 = 1, kMmaWarp = 6, kPvWarp = 7, kSm0 = 8;
constexpr int kSmWarps = 8;       // 4 partial-score senders + 4 softmax warps
constexpr int kSoftmaxWarps = 4;
constexpr uint32_t kRegsLow = 72, kRegsHigh = 184;
static_assert(256 * (kRegsLow + kRegsHigh) <= 65536, "register split exceeds the pool");

constexpr int kRB = kTS * 128;                 // one ckv d-block region of a stage
constexpr int kRK = kTS * 64;                  // the 32-wide kpe region
constexpr int kStageB = kBlk * kRB + kRK;      // 36 KB
constexpr int kQBlk = NH * 128;                // one [128 x 64] SW128 Q block
constexpr int kQB = kBlk * kQBlk + NH * 64;    // + the [128 x 32] SW64 q_pe block: 72 KB
constexpr int kXB = NH * kTS * 4;              // the peer's partial scores of a tile: 32 KB
constexpr int OFF_KV = 0;
constexpr int OFF_Q = kStages * kStageB;
constexpr int OFF_X = OFF_Q + kQB;
constexpr int OFF_XS = OFF_X + kXB;            // this CTA's partials of a tile, staged for the
                                               // bulk copy into the peer's X (same layout)
constexpr int OFF_BAR = OFF_XS + kXB;
constexpr int OFF_MASK = OFF_BAR + 512;        // [stage][kMaskStride] slot-validity words
constexpr int OFF_MEMB = OFF_MASK + 128;       // grouped calls: [stage][kTS / 4] membership words
constexpr int OFF_MISC = OFF_MEMB + 256;       // [0] TMEM base, [2] abort, [3] drain, [6] the
                                               // peer's abort flag (at exit), [8] merge lost
constexpr int SMEM_USED = OFF_MISC + 64;
constexpr int SMEM_BYTES = SMEM_USED + 1024;
constexpr int TMEM_COLS = 512;
constexpr int S_COL = 0, P_COL = 128, O_COL = 256;
constexpr int kSlotFloats = NH * kDCkv + 2 * NH;  // split-K partial: O [128 x 512], m, l
// Float offset of O[h][d .. d + 3] (d a multiple of 4) in a split-K partial: column quads
// outermost, so the 32 heads of a warp store or load one float4 each of 512 contiguous bytes.
__device__ __forceinline__ int part_o(int h, int d) { return ((d >> 2) * NH + h) * 4; }

static_assert(OFF_Q % 1024 == 0 && OFF_X % 1024 == 0 && kStageB % 1024 == 0,
              "128-byte swizzle atoms need 1024-byte alignment");
static_assert(SMEM_BYTES <= 232448, "shared memory budget");

enum : int {
  B_KVF = 0,                              // [stage] landed (one arrive per producer warp)
  B_KVE = B_KVF + kStages,                // [stage][5] region free again
  B_QF = B_KVE + kStages * kProdWarps,    // Q full / empty
  B_QE = B_QF + 1,
  B_SF = B_QE + 1, B_SE = B_SF + 2,       // [2] score buffer full / read
  B_PF = B_SE + 2, B_PD = B_PF + 2,       // [2] P written / PV done
  B_XF = B_PD + 2,                        // the peer's partial scores are in X (complete_tx)
  B_XE,                                   // the peer has read its X: we may write it again
  B_XSF,                                  // the staging buffer holds a tile (4 sender warps)
  B_XSE,                                  // the staging buffer's bulk copy has read it
  B_OF,                                   // the epilogue has read O
  B_PW,                                   // a split-K partial is written (8 warps)
  B_CNT,                                  // the merge's arrival count has been read
  B_MRG,                                  // another part's partial is in shared memory
  B_MRE,                                  // ... and has been added into O (4 warps)
  B_DRAIN,                                // [2] used only when an issuer stops early
  B_COUNT = B_DRAIN + 2
};
static_assert(B_COUNT * 8 <= 512, "barrier block");
__host__ __device__ constexpr int kve(int stage, int blk) { return B_KVE + stage * kProdWarps + blk; }

// Byte offset of 16-byte chunk c (0..11) of head row h in an X buffer [128 heads][48 slots]
// fp32; chunks are rotated by h / 2 so that a warp (32 heads, one chunk each) reads or writes
// with the minimum of four wavefronts.
__device__ __forceinline__ uint32_t xoff(int h, int c) {
  return (uint32_t)(h * (kTS * 4) + ((c + (h >> 1)) % (kTS / 4)) * 16);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// kMember: a grouped call (each row is a group of 128 >> tok_shift tokens over the union of
// their selections; a membership byte per entry masks the other tokens' heads).
template <bool kPaged, bool kMember>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    dsa_decode_hm_kernel(const __grid_constant__ CUtensorMap tm_ckv,
                         const __grid_constant__ CUtensorMap tm_kpe,
                         const __grid_constant__ CUtensorMap tm_qn,
                         const __grid_constant__ CUtensorMap tm_qp,
                         const __grid_constant__ Params p) {
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
  volatile uint32_t* memb = reinterpret_cast<volatile uint32_t*>(sgen + OFF_MEMB);
  const uint32_t bar0 = sbase + (uint32_t)OFF_BAR;
#define bar(k) (bar0 + 8u * (uint32_t)(k))

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(bar(B_KVF + s), kProdWarps);
      for (int j = 0; j < kProdWarps; ++j) ptx::mbar_init(bar(kve(s, j)), 1);
    }
    ptx::mbar_init(bar(B_QF), 1);
    ptx::mbar_init(bar(B_QE), 1);
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar(B_SF + b), 1);
      ptx::mbar_init(bar(B_SE + b), kSmWarps);
      ptx::mbar_init(bar(B_PF + b), kSoftmaxWarps);
      ptx::mbar_init(bar(B_PD + b), 1);
      ptx::mbar_init(bar(B_DRAIN + b), 1);
    }
    // X is full once this CTA armed it (one arrive with the expected bytes) and the peer's
    // st.async bytes landed; XE counts the peer's softmax warps, remotely.
    ptx::mbar_init(bar(B_XF), 1);
    ptx::mbar_init(bar(B_XE), kSoftmaxWarps);
    ptx::mbar_init(bar(B_XSF), 4);
    ptx::mbar_init(bar(B_XSE), 1);
    ptx::mbar_init(bar(B_OF), kSoftmaxWarps);
    ptx::mbar_init(bar(B_PW), kSoftmaxWarps);
    ptx::mbar_init(bar(B_CNT), 1);
    ptx::mbar_init(bar(B_MRG), 1);
    ptx::mbar_init(bar(B_MRE), kSoftmaxWarps);
    misc[2] = 0;
    misc[3] = 0;
    misc[6] = 0;
    misc[8] = 0;
    ptx::fence_mbar_init();
    ptx::mbar_arrive_expect_tx(bar(B_XF), (uint32_t)kXB);
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
    pipe::gather_producer<kTS, kStageB, kStages, kMaskStride, kPaged, kMember>(
        p, &tm_ckv, &tm_kpe, warp - kProd0, lane, rank, sbase + (uint32_t)OFF_KV, masks, bar(B_KVF),
        bar(B_KVE), u_lo, u_hi, wait, misc + 3, memb);
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------------ score MMA issuer
    // Partial S[128 heads x 64 slots] over this CTA's 288 columns: A = Q (K-major), B = the
    // stage's K rows (K-major), 16 MMAs over the four d-blocks and 2 over the kpe block.
    ptx::regs_dec<kRegsLow>();
    if (lane == 0) {
      const Waiter swait{misc + 2, p.err, p.wait_cycles, true};
      constexpr uint32_t kIdS = idesc_bf16(NH, kTS, false);
      const uint64_t dq = pipe::desc(sbase + (uint32_t)OFF_Q, 16, 1024, pipe::kSw128);
      const uint64_t dqp = pipe::desc(sbase + (uint32_t)(OFF_Q + kBlk * kQBlk), 16, 512, pipe::kSw64);
      const uint64_t dk = pipe::desc(sbase + (uint32_t)OFF_KV, 16, 1024, pipe::kSw128);
      const uint64_t dkp = pipe::desc(sbase + (uint32_t)(OFF_KV + kBlk * kRB), 16, 512, pipe::kSw64);
      int64_t i = 0;
      int seg = 0;
      bool ok = true;
      int64_t u = u_lo;
      Segment s;
      while (ok && next_segment(u, u_hi, p.tpr, s)) {
        for (int t = s.t0; t < s.t1; ++t, ++i) {
          const int st = (int)(i % kStages);
          const int sb = (int)(i & 1);
          if (t == s.t0) ok = swait(bar(B_QF), (uint32_t)(seg & 1));
          ok = ok && swait(bar(B_SE + sb), (uint32_t)(((i >> 1) & 1) ^ 1));
          ok = ok && swait(bar(B_KVF + st), (uint32_t)((i / kStages) & 1));
          if (!ok) break;
          if (masks[st * kMaskStride + kMaskAny] != 0u) {  // an all-padding tile skips its MMAs
            ptx::tc_fence_after();
            const uint32_t d_s = tmem + (uint32_t)(S_COL + 64 * sb);
            const uint64_t ko = (uint64_t)((st * kStageB) >> 4);
#pragma unroll
            for (int j = 0; j < kBlk; ++j)
#pragma unroll
              for (int ks = 0; ks < 4; ++ks)
                ptx::umma_bf16(d_s, dq + (uint64_t)((j * kQBlk + ks * 32) >> 4),
                               dk + ko + (uint64_t)((j * kRB + ks * 32) >> 4), kIdS,
                               (j | ks) ? 1u : 0u);
#pragma unroll
            for (int ks = 0; ks < 2; ++ks)
              ptx::umma_bf16(d_s, dqp + (uint64_t)((ks * 32) >> 4),
                             dkp + ko + (uint64_t)((ks * 32) >> 4), kIdS, 1u);
          }
          ptx::umma_commit(bar(B_SF + sb));
          ptx::umma_commit(bar(kve(st, kBlk)));  // the kpe region is read only by the score
          if (t == s.t1 - 1) ptx::umma_commit(bar(B_QE));
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
    // O[128 heads x 256 d] (+)= P . V over this CTA's value half: A = P from tensor memory,
    // B = the stage's value rows read MN-major across the four d-blocks, 4 MMAs of 16 slots.
    ptx::regs_dec<kRegsLow>();
    if (lane == 0) {
      const Waiter swait{misc + 2, p.err, p.wait_cycles, true};
      constexpr uint32_t kIdPV = idesc_bf16(NH, 256, false, true);
      const uint64_t dv = pipe::desc(sbase + (uint32_t)OFF_KV, kRB, 1024, pipe::kSw128);
      int64_t j = 0;
      int seg = 0;
      bool ok = true;
      bool o_init = false;
      int64_t u = u_lo;
      Segment s;
      while (ok && next_segment(u, u_hi, p.tpr, s)) {
        for (int t = s.t0; t < s.t1; ++t, ++j) {
          const int st = (int)(j % kStages);
          const int pb = (int)(j & 1);
          ok = swait(bar(B_PF + pb), (uint32_t)((j >> 1) & 1));
          if (ok && t == s.t0) {
            if (seg > 0) ok = swait(bar(B_OF), (uint32_t)((seg - 1) & 1));
            o_init = false;
          }
          if (!ok) break;
          if (masks[st * kMaskStride + kMaskAny] != 0u) {
            ptx::tc_fence_after();
            const uint64_t vo = (uint64_t)((st * kStageB) >> 4);
#pragma unroll
            for (int ks = 0; ks < kTS / 16; ++ks)
              ptx::umma_bf16_tmem_a(tmem + (uint32_t)O_COL,
                                    tmem + (uint32_t)(P_COL + 32 * pb + 8 * ks),
                                    dv + vo + (uint64_t)((ks * 2048) >> 4), kIdPV,
                                    (o_init || ks > 0) ? 1u : 0u);
            o_init = true;
          }
          for (int jb = 0; jb < kBlk; ++jb) ptx::umma_commit(bar(kve(st, jb)));
          ptx::umma_commit(bar(B_PD + pb));
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
    // ------------------------------------------------------------------ partial-score senders
    // Warps 8-11 (lane quadrant q = heads 32q .. 32q + 31): the tile's partial scores of
    // this CTA, one head per thread (its 64 slots), staged in this CTA's shared memory in X's
    // layout and sent into the peer's X with one bulk copy once the peer has read X for the
    // previous tile.  The peer's softmax of that tile meanwhile goes on, so the exchange
    // overlaps the softmax.
    ptx::regs_inc<kRegsHigh>();
    const int q = warp & 3;
    const int h = 32 * q + lane;
    const uint32_t lane_base = (uint32_t)(32 * q) << 16;
    if (warp < kSm0 + 4) {
      const uint32_t x_peer = ptx::mapa(sbase + (uint32_t)OFF_X, peer);
      const uint32_t xf_peer = ptx::mapa(bar(B_XF), peer);
      bool ok = true;
      for (int64_t i = 0; ok && i < u_hi - u_lo; ++i) {
        const int sb = (int)(i & 1);
        ok = wait(bar(B_SF + sb), (uint32_t)((i >> 1) & 1));
        ptx::tc_fence_after();
        static_assert(kTS == 48, "the senders move 32 + 16 slots per head");
        uint32_t s0[32], s1[16];
        ptx::tmem_ld32(tmem + lane_base + (uint32_t)(S_COL + 64 * sb), s0);
        ptx::tmem_ld16(tmem + lane_base + (uint32_t)(S_COL + 64 * sb + 32), s1);
        ptx::tmem_wait_ld();
        ptx::tc_fence_before();
        ok = __all_sync(0xffffffffu, ok);
        if (ok && lane == 0) ptx::mbar_arrive(bar(B_SE + sb));
        // the staging buffer is free once the previous tile's bulk copy has read it
        if (ok && i > 0) ok = __all_sync(0xffffffffu, wait(bar(B_XSE), (uint32_t)((i - 1) & 1)));
        if (!ok) break;
        uint8_t* xs = sgen + OFF_XS;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(xs + xoff(h, c)) = make_uint4(s0[4 * c], s0[4 * c + 1], s0[4 * c + 2], s0[4 * c + 3]);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4*>(xs + xoff(h, 8 + c)) = make_uint4(s1[4 * c], s1[4 * c + 1], s1[4 * c + 2], s1[4 * c + 3]);
        ptx::fence_proxy_async_smem();  // the bulk copy (async proxy) reads these stores
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(B_XSF));
        if (warp == kSm0) {
          // One bulk copy of the tile's partials into the peer's X, once the four warps have
          // staged theirs and the peer has read X for the previous tile; the staging buffer
          // is released when the copy has read it.  (One copy instead of 4 x 32 x 16
          // st.async: their per-instruction cost, not the link's bytes, set the tile period.)
          bool go = true;
          if (lane == 0) {
            go = wait(bar(B_XSF), (uint32_t)(i & 1)) &&
                 (i == 0 || wait(bar(B_XE), (uint32_t)((i - 1) & 1)));
            if (go) {
              ptx::bulk_s2peer(x_peer, sbase + (uint32_t)OFF_XS, (uint32_t)kXB, xf_peer);
              ptx::bulk_commit_group();
              ptx::bulk_wait_read_all();
              ptx::mbar_arrive(bar(B_XSE));
            }
          }
          ok = __shfl_sync(0xffffffffu, (int)go, 0) != 0;
        }
      }
    } else {
    // ------------------------------------------------------------------ softmax / epilogue
    // Warps 12-15: head h = 32 (w % 4) + lane over all 64 slots of every tile: own partial
    // (TMEM) + the peer's (X), online softmax with a lazily rescaled running max, P as bf16
    // pairs into tensor memory for the PV MMA, and each segment's output.
    const uint32_t xe_peer = ptx::mapa(bar(B_XE), peer);
    int64_t i = 0;        // tiles done by this CTA
    int pw_phase = 0;     // B_PW phases used so far (partials written)
    int cnt_phase = 0;    // B_CNT phases used so far (merges)
    int mrg_phase = 0;    // B_MRG / B_MRE phases used so far (parts merged)
    bool aborted = false;
    int64_t u = u_lo;
    Segment s;

    // A segment's output (or split-K partial / merge) from O in TMEM (this head's 256 value
    // columns of this CTA) and the head's running max m and sum l; false if the CTA gave up.
    auto finish = [&](const Segment& es, float m, float l, int64_t eil) -> bool {
      // PV done for tile eil; PV(eil - 1) first, so that the parity wait is exact.
      bool okw = !aborted;
      if (okw && eil >= 1)
        okw = wait(bar(B_PD + (int)((eil - 1) & 1)), (uint32_t)(((eil - 1) >> 1) & 1));
      okw = okw && wait(bar(B_PD + (int)(eil & 1)), (uint32_t)((eil >> 1) & 1));
      if (!__all_sync(0xffffffffu, okw)) {
        aborted = true;
        return false;
      }
      ptx::tc_fence_after();
      const int64_t b = es.rh >> p.hg_shift;
      const bool full = (es.t0 == 0 && es.t1 == p.tpr);
      const int64_t p_lo = full ? pair : cta_of(es.rh * p.tpr, p.units, G);
      const int64_t p_hi = full ? pair : cta_of((es.rh + 1) * p.tpr - 1, p.units, G);
      const bool head = full || pair == p_lo;
      float* part = p.parts + pair * kSlotFloats;
      __nv_bfloat16* orow = p.out + b * p.out_sb + (int64_t)h * p.out_sh;
      const int d_half = 256 * (int)rank;  // this CTA's value columns
      if (full || !head) {
        // a row with no valid slot never wrote O (stale columns): it is written as zeros
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll 1
        for (int cc = 0; cc < 8; ++cc) {
          uint32_t r[32];
          ptx::tmem_ld32(tmem + lane_base + (uint32_t)(O_COL + 32 * cc), r);
          ptx::tmem_wait_ld();
          const int d0 = d_half + 32 * cc;
          if (full) {
            float o[32];
#pragma unroll
            for (int c = 0; c < 32; ++c) o[c] = l > 0.f ? __uint_as_float(r[c]) * inv : 0.f;
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint4 w;
              w.x = pack_bf16x2(o[8 * v + 0], o[8 * v + 1]);
              w.y = pack_bf16x2(o[8 * v + 2], o[8 * v + 3]);
              w.z = pack_bf16x2(o[8 * v + 4], o[8 * v + 5]);
              w.w = pack_bf16x2(o[8 * v + 6], o[8 * v + 7]);
              *reinterpret_cast<uint4*>(orow + d0 + 8 * v) = w;
            }
          } else {
#pragma unroll
            for (int v = 0; v < 8; ++v)
              *reinterpret_cast<float4*>(part + part_o(h, d0 + 4 * v)) =
                  make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                              __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]));
          }
        }
        if (full && rank == 0)
          p.lse[b * p.lse_sb + (int64_t)h * p.lse_sh] = l > 0.f ? m + ptx::lg2(l) : -INFINITY;
        if (!full) {
          // both ranks write the (identical) scalars, so each rank's merge finds them
          part[NH * kDCkv + h] = m;
          part[NH * kDCkv + NH + h] = l;
        }
      }
      uint32_t* cnt = p.counters + 2 * p_lo + rank;
      if (!full && !head) {
        // every warp's partial stores, then one release add for the CTA
        __syncwarp();
        if (lane == 0) {
          __threadfence();
          ptx::mbar_arrive(bar(B_PW));
        }
        if (warp == kSm0 + 4 && lane == 0 && wait(bar(B_PW), (uint32_t)(pw_phase & 1)))
          ptx::red_release_gpu_add(cnt, 1u);
        ++pw_phase;
      } else if (!full) {
        // Bounded wait for the other parts of the row by one thread; the others wait on
        // B_CNT for its verdict (the acquire load orders the partial reads after it).
        if (warp == kSm0 + 4 && lane == 0) {
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
          // every part has been counted: the counter is ready for the next call
          *reinterpret_cast<volatile uint32_t*>(cnt) = 0u;
          ptx::mbar_arrive(bar(B_CNT));
        }
        const bool cnt_ok = wait(bar(B_CNT), (uint32_t)(cnt_phase & 1));
        ++cnt_phase;
        // A merge that gave up would combine whatever partials are there: the row is written
        // as NaN instead, next to the timeout bit in the error word.
        const bool lost = !__all_sync(0xffffffffu, cnt_ok) || misc[8] != 0u;
        // final max over the live parts and their weights (one pass over the scalars)
        float M = l > 0.f ? m : -INFINITY;
        for (int64_t cc = p_lo + 1; cc <= p_hi; ++cc) {
          const float* pp = p.parts + cc * kSlotFloats;
          if (__ldcg(pp + NH * kDCkv + NH + h) > 0.f) M = fmaxf(M, __ldcg(pp + NH * kDCkv + h));
        }
        const bool any = M != -INFINITY;
        const float w_own = (any && l > 0.f) ? ptx::ex2(m - M) : 0.f;
        float Lt = w_own * l;
        // O = w_own O, then + w_j O_j for every other part j: the part's slab of this CTA's
        // 256 columns (128 KB, contiguous) is copied into the pipeline's shared memory, free
        // now that this segment's last PV is done, and added into O in tensor memory.
        const uint32_t slab = sbase + (uint32_t)OFF_KV;
        static_assert(NH * 256 * 4 <= OFF_X, "a part's slab fits in the stages and Q buffer");
        for (int64_t cc = p_lo + 1; cc <= p_hi; ++cc) {
          const float* pp = p.parts + cc * kSlotFloats;
          const float pl = __ldcg(pp + NH * kDCkv + NH + h);
          const float wj = pl > 0.f ? ptx::ex2(__ldcg(pp + NH * kDCkv + h) - M) : 0.f;
          Lt += wj * (pl > 0.f ? pl : 0.f);
          if (warp == kSm0 + 4 && lane == 0) {
            if (mrg_phase > 0) wait(bar(B_MRE), (uint32_t)((mrg_phase - 1) & 1));
            ptx::fence_proxy_async_global();
            ptx::mbar_arrive_expect_tx(bar(B_MRG), (uint32_t)(NH * 256 * 4));
            ptx::bulk_g2s(slab, pp + part_o(0, d_half), (uint32_t)(NH * 256 * 4), bar(B_MRG));
          }
          const bool got = __all_sync(0xffffffffu, wait(bar(B_MRG), (uint32_t)(mrg_phase & 1)));
          ptx::tc_fence_after();
#pragma unroll 1
          for (int c8 = 0; c8 < 8; ++c8) {
            const uint32_t ta = tmem + lane_base + (uint32_t)(O_COL + 32 * c8);
            uint32_t r[32];
            ptx::tmem_ld32(ta, r);
            ptx::tmem_wait_ld();
            const float wo = cc == p_lo + 1 ? w_own : 1.f;  // the own part's weight, once
#pragma unroll
            for (int v = 0; v < 8; ++v) {
              const float4 o4 = got ? *reinterpret_cast<const float4*>(
                                          sgen + OFF_KV + 4 * part_o(h, 32 * c8 + 4 * v))
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
              const float a[4] = {o4.x, o4.y, o4.z, o4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float own = __uint_as_float(r[4 * v + e]);
                const float base = wo > 0.f ? wo * own : 0.f;  // stale O when wo == 0
                r[4 * v + e] = __float_as_uint(wj > 0.f ? base + wj * a[e] : base);
              }
            }
            ptx::tmem_st32(ta, r);
          }
          ptx::tmem_wait_st();
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(bar(B_MRE));
          ++mrg_phase;
        }
        const float inv = Lt > 0.f ? 1.f / Lt : 0.f;
        ptx::tc_fence_after();
#pragma unroll 1
        for (int c8 = 0; c8 < 8; ++c8) {
          uint32_t r[32];
          ptx::tmem_ld32(tmem + lane_base + (uint32_t)(O_COL + 32 * c8), r);
          ptx::tmem_wait_ld();
          const int d0 = d_half + 32 * c8;
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint4 wv;
            wv.x = lost ? 0x7FC07FC0u : pack_bf16x2(__uint_as_float(r[8 * v]) * inv, __uint_as_float(r[8 * v + 1]) * inv);
            wv.y = lost ? 0x7FC07FC0u : pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv);
            wv.z = lost ? 0x7FC07FC0u : pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv);
            wv.w = lost ? 0x7FC07FC0u : pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + d0 + 8 * v) = wv;
          }
        }
        if (rank == 0)
          p.lse[b * p.lse_sb + (int64_t)h * p.lse_sh] =
              lost ? NAN : (Lt > 0.f ? M + ptx::lg2(Lt) : -INFINITY);
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(bar(B_OF));
      return true;
    };

    while (!aborted && next_segment(u, u_hi, p.tpr, s)) {
      float m_run = -INFINITY, l_run = 0.f;  // head h over the segment
      bool o_valid = false;
      for (int t = s.t0; t < s.t1; ++t, ++i) {
        const int st = (int)(i % kStages);
        const int sb = (int)(i & 1);
        // own partial scores (the stage's full barrier first: it orders the producers' mask
        // words before the reads below)
        bool ok = wait(bar(B_KVF + st), (uint32_t)((i / kStages) & 1)) &&
                  wait(bar(B_SF + sb), (uint32_t)((i >> 1) & 1));
        ptx::tc_fence_after();
        uint32_t own0[32], own1[16];
        ptx::tmem_ld32(tmem + lane_base + (uint32_t)(S_COL + 64 * sb), own0);
        ptx::tmem_ld16(tmem + lane_base + (uint32_t)(S_COL + 64 * sb + 32), own1);
        ptx::tmem_wait_ld();
        ptx::tc_fence_before();
        ok = __all_sync(0xffffffffu, ok);
        if (ok && lane == 0) ptx::mbar_arrive(bar(B_SE + sb));
        // the peer's partial of this tile
        ok = ok && __all_sync(0xffffffffu, wait(bar(B_XF), (uint32_t)(i & 1)));
        if (!ok) {
          aborted = true;
          break;
        }
        const uint32_t mw0 = masks[st * kMaskStride + 0], mw1 = masks[st * kMaskStride + 1];
        const bool live = masks[st * kMaskStride + kMaskAny] != 0u;
        float x[kTS];
        float mt = -INFINITY;
        const int tok = kMember ? (h >> p.tok_shift) : 0;  // this head's token in the group
#pragma unroll
        for (int c = 0; c < kTS / 4; ++c) {
          const float4 v = *reinterpret_cast<const float4*>(sgen + OFF_X + xoff(h, c));
          const float pv[4] = {v.x, v.y, v.z, v.w};
          const uint32_t mb = kMember ? memb[st * (kTS / 4) + c] >> tok : 0u;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int k = 4 * c + e;
            const uint32_t ob = k < 32 ? own0[k] : own1[k - 32];
            const bool valid = ((k < 32 ? mw0 >> k : mw1 >> (k - 32)) & 1u) != 0u &&
                               (!kMember || ((mb >> (8 * e)) & 1u) != 0u);
            x[k] = valid ? (__uint_as_float(ob) + pv[e]) * p.scale_log2 : -INFINITY;
            mt = fmaxf(mt, x[k]);
          }
        }
        // X is read (every lane's loads have returned: the vote consumes their maximum):
        // re-arm our barrier for the next tile (before this warp's release below, so that no
        // byte of the next tile can arrive before the arming), then release the buffer to the
        // peer's senders.
        const uint32_t read_all = __ballot_sync(0xffffffffu, mt == mt);
        if (lane == 0) {
          if (warp == kSm0 + 4) ptx::mbar_arrive_expect_tx(bar(B_XF), (uint32_t)kXB);
          ptx::mbar_arrive_remote_after(xe_peer, read_all == 0xFFFFFFFFu ? 0u : read_all);
        }
        // lazy rescale: only when the tile's max exceeds the running max by more than kTau
        float alpha = 1.f;
        const bool need = mt > m_run + kTau;
        if (need) {
          const float mn = fmaxf(m_run, mt);
          alpha = (m_run == -INFINITY) ? 0.f : ptx::ex2(m_run - mn);
          l_run *= alpha;
          m_run = mn;
        }
        if (__any_sync(0xffffffffu, need) && o_valid) {
          // rescale this head's O row once PV(i - 1) is done (warp-uniform outcome)
          const bool wok = wait(bar(B_PD + (int)((i - 1) & 1)), (uint32_t)(((i - 1) >> 1) & 1));
          if (!__all_sync(0xffffffffu, wok)) {
            aborted = true;
            break;
          }
          ptx::tc_fence_after();
#pragma unroll 1
          for (int cc = 0; cc < 8; ++cc) {
            const uint32_t ta = tmem + lane_base + (uint32_t)(O_COL + 32 * cc);
            uint32_t r[32];
            ptx::tmem_ld32(ta, r);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int c = 0; c < 32; ++c) r[c] = __float_as_uint(__uint_as_float(r[c]) * alpha);
            ptx::tmem_st32(ta, r);
          }
          ptx::tmem_wait_st();
        }
        // P[sb] was last read by PV(i - 2) (PV(i - 4) is done: tile i - 1's stage was
        // refilled after it, so this parity wait is exact)
        if (i >= 2) {
          const bool wok = wait(bar(B_PD + sb), (uint32_t)(((i - 2) >> 1) & 1));
          if (!__all_sync(0xffffffffu, wok)) {
            aborted = true;
            break;
          }
        }
        const float me = (m_run == -INFINITY) ? 0.f : m_run;
        uint32_t pk[16], pk2[8];
#pragma unroll
        for (int c = 0; c < kTS / 2; ++c) {
          const float a0 = ptx::ex2(x[2 * c] - me);
          const float a1 = ptx::ex2(x[2 * c + 1] - me);
          l_run += a0 + a1;
          if (c < 16) pk[c] = pack_bf16x2(a0, a1);
          else pk2[c - 16] = pack_bf16x2(a0, a1);
        }
        ptx::tmem_st16(tmem + lane_base + (uint32_t)(P_COL + 32 * sb), pk);
        ptx::tmem_st8(tmem + lane_base + (uint32_t)(P_COL + 32 * sb + 16), pk2);
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(B_PF + sb));
        o_valid = o_valid || live;
      }
      if (aborted) break;
      if (!finish(s, m_run, l_run, i - 1)) break;
    }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  // Neither CTA leaves while the other may still write its exchange buffer or arrive on
  // its barriers (see the 16/32-head kernel): each CTA tells the other whether it gave up,
  // and both then take the same exit path.
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

}  // namespace hm
}  // namespace dsa
