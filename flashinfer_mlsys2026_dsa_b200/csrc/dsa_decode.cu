// B200 (sm_100a) DeepSeek sparse-attention decode: one persistent kernel per call.
//
// Math (the reference PyTorch path, solution/triton/baseline.py:12-45):
//   for each decode row b and head h over the topk selected slots k:
//     z[h,k]  = sm_scale * (q_nope[b,h] . ckv[idx[b,k]] + q_pe[b,h] . kpe[idx[b,k]])
//     z[h,k]  = -inf where idx[b,k] == -1
//     lse[b,h] = log2(sum_k exp(z[h,k]))
//     out[b,h] = bf16(sum_k softmax(z)[h,k] * ckv[idx[b,k]])
//
// The kernel (dsa_decode_h16.cuh) runs on two-CTA clusters, one head group (16 or 32
// heads) of one row per work unit; this file holds what it shares with the host side (parameters, the
// bounded wait, the stream-K split) and the C ABI of include/dsa_b200.h.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <utility>

#include "dsa_b200.h"
#include "sm100_ptx.cuh"

namespace dsa {

constexpr int kDCkv = 512;            // latent (value) width
constexpr int kDKpe = 64;             // rope key width
constexpr float kTau = 8.0f;          // lazy-rescale threshold (log2 units)
constexpr float kLog2e = 1.4426950408889634f;
constexpr uint64_t kWaitCycles = 4000000000ull;  // default wait bound: ~2 s at ~2 GHz

struct Params {
  const int32_t* idx;
  int64_t idx_sb;
  __nv_bfloat16* out;
  int64_t out_sb, out_sh;
  float* lse;
  int64_t lse_sb, lse_sh;
  int64_t num_slots;
  int64_t units;  // (row, head group) pairs x tpr
  int32_t hg_shift;  // log2 of the head groups per row (0 to 2 for 32-head groups)
  int32_t topk;
  int32_t tpr;    // tiles per (row, head group)
  float scale_log2;
  uint32_t* err;
  float* parts;       // split-K partials, one slot per cluster pair
  uint32_t* counters;  // split-K arrival counters, zero between calls
  uint64_t wait_cycles;  // bound of every wait in the kernel (SM cycles)
  // paged calls only: idx holds token positions; page_table rows of pt_cols page ids
  const int32_t* pt;
  int64_t pt_sb;
  int32_t pt_cols;
  int32_t pg_shift;  // log2(page_size)
  // grouped calls only (128-head kernel): a membership byte per index entry, bit j = token
  // j of the row's token group selected the entry; head h belongs to token h >> tok_shift
  const uint8_t* member;
  int64_t member_sb;
  int32_t tok_shift;
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

// Instruction descriptor, kind::f16: bf16 A/B, fp32 D; A and B K-major unless flagged.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn_major,
                                                  bool b_mn_major = false) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
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
  uint64_t limit;  // cycles
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
        if (ptx::cycles() - t0 > limit) {
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
  int64_t rh;  // (row << hg_shift) + head group
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

#include "dsa_pipeline.cuh"
#include "dsa_decode_h16.cuh"
#include "dsa_decode_hm.cuh"

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

// Bound of every wait in the kernels, in SM cycles (dsa_set_wait_limit).
std::atomic<uint64_t> g_wait_cycles{kWaitCycles};

struct DeviceState {
  int sms = 0;
  int pairs = 0;  // co-resident two-CTA clusters of the decode kernel
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

using DecodeKernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, Params);
struct KernelVariant {
  int nh;       // heads per work unit
  bool paged;   // slot ids formed from page tables
  bool member;  // token groups: entries carry membership bytes
  DecodeKernelFn fn;
  int smem;
};
const KernelVariant kVariants[] = {
    {16, false, false, h16::dsa_decode_h16_kernel<16, false>, h16::Cfg<16>::SMEM_BYTES},
    {16, true, false, h16::dsa_decode_h16_kernel<16, true>, h16::Cfg<16>::SMEM_BYTES},
    {32, false, false, h16::dsa_decode_h16_kernel<32, false>, h16::Cfg<32>::SMEM_BYTES},
    {32, true, false, h16::dsa_decode_h16_kernel<32, true>, h16::Cfg<32>::SMEM_BYTES},
    {128, false, false, hm::dsa_decode_hm_kernel<false, false>, hm::SMEM_BYTES},
    {128, true, false, hm::dsa_decode_hm_kernel<true, false>, hm::SMEM_BYTES},
    {128, false, true, hm::dsa_decode_hm_kernel<false, true>, hm::SMEM_BYTES},
};
const KernelVariant& variant(int nh, bool paged, bool member) {
  for (const KernelVariant& kv : kVariants)
    if (kv.nh == nh && kv.paged == paged && kv.member == member) return kv;
  return kVariants[0];
}
// Heads per work unit: 16 for 16-head rows, 32 for 32- and 64-head rows (two units per
// 64-head row), 128 for 128-head rows (the heads-as-M kernel: one unit per row and tile).
int group_heads(int num_heads) { return num_heads == 16 ? 16 : (num_heads == 128 ? 128 : 32); }
constexpr size_t kMaxSlotFloats = (size_t)hm::kSlotFloats;

// Sets the decode kernels' shared-memory attribute and returns how many of their clusters
// fit on the device at once (the persistent grid's size), 0 on error.
int device_pairs(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (dev < 0 || dev >= kMaxDevices) return 0;
  DeviceState& d = g_dev[dev];
  if (d.pairs == 0) {
    // The kernel re-splits its register pool per warpgroup (setmaxnreg); refuse a build
    // whose pool is too small for that split, which would stall.
    // every instance (16- or 32-head groups, flat or paged ids) must fit the same grid
    int n = 0;
    for (const KernelVariant& kv : kVariants) {
      cudaFuncAttributes fa;
      if (cudaFuncGetAttributes(&fa, kv.fn) != cudaSuccess) return 0;
      if ((int64_t)fa.numRegs * h16::kThreads < 256 * (int64_t)(h16::kRegsLow + h16::kRegsHigh))
        return 0;
      if (cudaFuncSetAttribute(kv.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kv.smem) !=
          cudaSuccess)
        return 0;
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * (unsigned)(d.sms > 0 ? d.sms : 148), 1, 1);
      cfg.blockDim = dim3(h16::kThreads, 1, 1);
      cfg.dynamicSmemBytes = (size_t)kv.smem;
      int k = 0;
      if (cudaOccupancyMaxActiveClusters(&k, kv.fn, &cfg) != cudaSuccess || k <= 0) return 0;
      n = n == 0 ? k : (k < n ? k : n);
    }
    d.pairs = n;
  }
  return d.pairs;
}

bool heads_supported(int heads) {
  return heads == 16 || heads == 32 || heads == 64 || heads == 128;
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Workspace layout, fixed for a device so that calls of any shape can share it:
//   [0, 256)            header (word 0: sticky device error bits)
//   [256, 8448)         split-K arrival counters, 2 per CTA pair (one per rank; each
//                       returns to zero when its row is merged)
//   [8448, ...)         split-K partials: one slot per CTA pair (two SMs), each sized for
//                       a 128-head row (O, m and l: 263,168 bytes)
constexpr size_t kCountersOff = 256;
constexpr size_t kPartsOff = 8448;
constexpr int kMaxPairs = (int)((kPartsOff - kCountersOff) / 8);

struct WsLayout {
  size_t parts_off, total;
};

WsLayout ws_layout(int sms) {
  WsLayout w;
  w.parts_off = kPartsOff;
  // one partial slot per cluster pair (a pair occupies two SMs)
  w.total = align_up(w.parts_off + (size_t)((sms + 1) / 2) * kMaxSlotFloats * 4, 256);
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
  // paged calls: idx holds token positions, translated through page_table
  const int32_t* page_table = nullptr;
  int64_t pt_sb = 0;
  int32_t pt_cols = 0;
  int32_t page_size = 0;
  // grouped calls (128-head rows made of token groups): membership bytes beside idx
  const uint8_t* member = nullptr;
  int64_t member_sb = 0;
  int32_t tok_shift = 0;
};

int check_args(const DecodeArgs& a) {
  if (a.num_tokens < 0 || a.topk < 1 || a.num_slots < 1 || a.num_slots > INT32_MAX ||
      a.num_tokens > INT32_MAX)
    return DSA_ERR_INVALID_ARGUMENT;
  if (!heads_supported(a.num_heads)) return DSA_ERR_UNSUPPORTED;
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
  if (a.page_table != nullptr) {
    const int32_t ps = a.page_size;
    if (ps < 1 || ps > (1 << 20) || (ps & (ps - 1)) != 0 || a.pt_cols < 1 ||
        a.pt_sb < a.pt_cols || (int64_t)a.pt_cols * ps > INT32_MAX)
      return DSA_ERR_INVALID_ARGUMENT;
  }
  return DSA_OK;
}

// Which kernel a call runs, its persistent grid and the scratch it needs.
struct Plan {
  int nh = 16;        // heads per work unit (16 or 32)
  int tpr = 0;        // tiles per (row, head group)
  int64_t units = 0;  // (row, group) pairs x tpr
  int grid = 0;       // cluster pairs of the persistent grid
  size_t need = 0;    // bytes of error header, counters and partials
};

int make_plan(const DecodeArgs& a, int dev, Plan& pl) {
  const int cap = device_pairs(dev);
  if (cap <= 0) return DSA_ERR_CUDA;
  pl.nh = group_heads(a.num_heads);
  const int hg = a.num_heads / pl.nh;  // head groups per row
  const int ts = pl.nh == 16 ? h16::Cfg<16>::kTS
                             : (pl.nh == 32 ? h16::Cfg<32>::kTS : hm::kTS);  // slots per tile
  pl.tpr = (a.topk + ts - 1) / ts;
  const int64_t num_rh = a.num_tokens * hg;
  pl.units = num_rh * (int64_t)pl.tpr;
  if (pl.nh == 128) {
    // 128-head rows: stream-K over all pairs whatever the row count (a 128-head row is a
    // long unit, so its merge is cheap next to idle SMs); every pair may hold a partial.
    pl.grid = (int)(pl.units < cap ? pl.units : cap);
    if (pl.grid > kMaxPairs) pl.grid = kMaxPairs;
    pl.need = kPartsOff + (size_t)pl.grid * (size_t)hm::kSlotFloats * 4;
    return DSA_OK;
  }
  // With no more (row, group) pairs than the grid holds, each gets a whole cluster pair and
  // none is split: a split-K merge costs a few dependent global round trips on the tail,
  // each slow while the other SMs saturate HBM, which outweighs the idle SMs.  Otherwise
  // stream-K: every pair takes an equal share of the tiles and the rows cut between pairs
  // are merged in the kernel through one partial slot per pair.
  const bool whole = num_rh <= cap;
  pl.grid = (int)(whole ? num_rh : cap);
  if (pl.grid > kMaxPairs) pl.grid = kMaxPairs;
  const size_t slot_floats = pl.nh == 16 ? (size_t)h16::Cfg<16>::kSlotFloats
                                         : (size_t)h16::Cfg<32>::kSlotFloats;
  pl.need = kPartsOff + (whole ? 0 : (size_t)pl.grid * slot_floats * 4);
  return DSA_OK;
}

int run_plan(const DecodeArgs& a, const Plan& pl, uint8_t* ws, cudaStream_t st) {
  // The kernel loads 64-wide ckv and Q boxes and 32-wide kpe and q_pe halves (one per CTA
  // of a pair), all 16 heads of a group at once.
  CUtensorMap m_ckv, m_kpe, m_qn, m_qp;
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
    cuuint32_t box[2] = {32, 1};
    if ((rc = encode(&m_kpe, a.kpe, 2, dims, str, box, CU_TENSOR_MAP_SWIZZLE_64B)) != DSA_OK)
      return rc;
  }
  {
    cuuint64_t dims[3] = {(cuuint64_t)kDCkv, (cuuint64_t)a.num_heads, (cuuint64_t)a.num_tokens};
    cuuint64_t str[2] = {(cuuint64_t)a.qn_sh * 2, (cuuint64_t)a.qn_sb * 2};
    cuuint32_t box[3] = {64, (cuuint32_t)pl.nh, 1};
    if ((rc = encode(&m_qn, a.q_nope, 3, dims, str, box, CU_TENSOR_MAP_SWIZZLE_128B)) != DSA_OK)
      return rc;
  }
  {
    cuuint64_t dims[3] = {(cuuint64_t)kDKpe, (cuuint64_t)a.num_heads, (cuuint64_t)a.num_tokens};
    cuuint64_t str[2] = {(cuuint64_t)a.qp_sh * 2, (cuuint64_t)a.qp_sb * 2};
    cuuint32_t box[3] = {32, (cuuint32_t)pl.nh, 1};
    if ((rc = encode(&m_qp, a.q_pe, 3, dims, str, box, CU_TENSOR_MAP_SWIZZLE_64B)) != DSA_OK)
      return rc;
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
  prm.hg_shift = 0;  // log2 of the head groups per row
  while ((pl.nh << prm.hg_shift) < a.num_heads) ++prm.hg_shift;
  prm.topk = a.topk;
  prm.tpr = pl.tpr;
  prm.scale_log2 = a.sm_scale * kLog2e;
  prm.err = reinterpret_cast<uint32_t*>(ws);
  prm.parts = reinterpret_cast<float*>(ws + kPartsOff);
  prm.counters = reinterpret_cast<uint32_t*>(ws + kCountersOff);
  prm.wait_cycles = g_wait_cycles.load(std::memory_order_relaxed);
  prm.pt = a.page_table;
  prm.pt_sb = a.pt_sb;
  prm.pt_cols = a.pt_cols;
  prm.pg_shift = 0;
  while (a.page_table != nullptr && (1 << prm.pg_shift) < a.page_size) ++prm.pg_shift;
  prm.member = a.member;
  prm.member_sb = a.member_sb;
  prm.tok_shift = a.tok_shift;
  const KernelVariant& kv = variant(pl.nh, a.page_table != nullptr, a.member != nullptr);
  return launch_pdl(kv.fn, dim3((unsigned)(2 * pl.grid)), dim3(h16::kThreads),
                    (size_t)kv.smem, st, m_ckv, m_kpe, m_qn, m_qp, prm);
}

int current_device(int& dev) {
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return DSA_ERR_CUDA;
  return DSA_OK;
}

// The 128-head kernel writes each head's output with 16-byte stores.
int check_out_alignment(const DecodeArgs& a) {
  if (a.num_heads == 128 && (!aligned16(a.out) || (a.out_sb * 2) % 16 || (a.out_sh * 2) % 16))
    return DSA_ERR_MISALIGNED;
  return DSA_OK;
}

int decode_with_workspace(const DecodeArgs& a, void* workspace, size_t workspace_bytes,
                          void* stream) {
  int rc = check_args(a);
  if (rc == DSA_OK && a.num_tokens > 0) rc = check_out_alignment(a);
  if (rc != DSA_OK || a.num_tokens == 0) return rc;
  int dev = 0;
  if ((rc = current_device(dev)) != DSA_OK) return rc;
  const int sms = device_sms(dev);
  if (sms <= 0) return DSA_ERR_CUDA;
  if (!workspace || workspace_bytes < ws_layout(sms).total) return DSA_ERR_WORKSPACE;
  Plan pl;
  if ((rc = make_plan(a, dev, pl)) != DSA_OK) return rc;
  return run_plan(a, pl, static_cast<uint8_t*>(workspace), static_cast<cudaStream_t>(stream));
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
  if (!heads_supported(num_heads) || num_tokens < 0 || topk < 1) return 0;
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
  return decode_with_workspace(a, workspace, workspace_bytes, stream);
}

int dsa_sparse_mla_decode_paged(
    const void* q_nope, int64_t q_nope_stride_b, int64_t q_nope_stride_h, const void* q_pe,
    int64_t q_pe_stride_b, int64_t q_pe_stride_h, const void* ckv_cache, int64_t ckv_slot_stride,
    const void* kpe_cache, int64_t kpe_slot_stride, int64_t num_slots, const int32_t* page_table,
    int64_t page_table_stride_b, int32_t page_table_cols, int32_t page_size,
    const int32_t* positions, int64_t positions_stride_b, float sm_scale, void* output,
    int64_t output_stride_b, int64_t output_stride_h, float* lse, int64_t lse_stride_b,
    int64_t lse_stride_h, int64_t num_tokens, int32_t num_heads, int32_t topk, void* workspace,
    size_t workspace_bytes, void* stream) {
  if (page_table == nullptr && num_tokens > 0) return DSA_ERR_INVALID_ARGUMENT;
  DecodeArgs a{q_nope,          q_nope_stride_b, q_nope_stride_h, q_pe,
               q_pe_stride_b,   q_pe_stride_h,   ckv_cache,       ckv_slot_stride,
               kpe_cache,       kpe_slot_stride, num_slots,       positions,
               positions_stride_b, sm_scale,     output,          output_stride_b,
               output_stride_h, lse,             lse_stride_b,    lse_stride_h,
               num_tokens,      num_heads,       topk};
  a.page_table = page_table;
  a.pt_sb = page_table_stride_b;
  a.pt_cols = page_table_cols;
  a.page_size = page_size;
  return decode_with_workspace(a, workspace, workspace_bytes, stream);
}

int dsa_sparse_mla_decode_grouped(
    const void* q_nope, int64_t q_nope_stride_b, int64_t q_nope_stride_h, const void* q_pe,
    int64_t q_pe_stride_b, int64_t q_pe_stride_h, const void* ckv_cache, int64_t ckv_slot_stride,
    const void* kpe_cache, int64_t kpe_slot_stride, int64_t num_slots,
    const int32_t* union_indices, const uint8_t* member, int64_t union_stride_g,
    int32_t union_cols, float sm_scale, void* output, int64_t output_stride_b,
    int64_t output_stride_h, float* lse, int64_t lse_stride_b, int64_t lse_stride_h,
    int64_t num_tokens, int32_t num_heads, void* workspace, size_t workspace_bytes,
    void* stream) {
  // A group of G = 128 / num_heads consecutive tokens is one 128-head row: the token's
  // heads must follow each other in q_nope, q_pe, output and lse (stride_b = num_heads x
  // stride_h), so that the group's 128 heads are rows of one strided array.
  if (num_heads != 16 && num_heads != 32 && num_heads != 64) return DSA_ERR_UNSUPPORTED;
  const int64_t G = 128 / num_heads;
  if (num_tokens < 0 || num_tokens % G != 0 || union_cols < 1) return DSA_ERR_INVALID_ARGUMENT;
  if (num_tokens == 0) return DSA_OK;
  if (!union_indices || !member || union_stride_g < union_cols) return DSA_ERR_INVALID_ARGUMENT;
  if (q_nope_stride_b != num_heads * q_nope_stride_h || q_pe_stride_b != num_heads * q_pe_stride_h ||
      output_stride_b != num_heads * output_stride_h || lse_stride_b != num_heads * lse_stride_h)
    return DSA_ERR_INVALID_ARGUMENT;
  DecodeArgs a{q_nope,          G * q_nope_stride_b, q_nope_stride_h, q_pe,
               G * q_pe_stride_b, q_pe_stride_h,     ckv_cache,       ckv_slot_stride,
               kpe_cache,       kpe_slot_stride,     num_slots,       union_indices,
               union_stride_g,  sm_scale,            output,          G * output_stride_b,
               output_stride_h, lse,                 G * lse_stride_b, lse_stride_h,
               num_tokens / G,  128,                 union_cols};
  a.member = member;
  a.member_sb = union_stride_g;
  a.tok_shift = num_heads == 16 ? 4 : (num_heads == 32 ? 5 : 6);
  return decode_with_workspace(a, workspace, workspace_bytes, stream);
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

uint64_t dsa_set_wait_limit(uint64_t cycles) {
  return g_wait_cycles.exchange(cycles == 0 ? kWaitCycles : cycles);
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
constexpr size_t kNoAllocScratchBytes = size_t(2) << 20;  // header, counters, partials
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
  if (rc == DSA_OK && num_tokens > 0) rc = check_out_alignment(a);
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
  return run_plan(a, pl, static_cast<uint8_t*>(scratch), st);
}
