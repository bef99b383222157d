// TVM-FFI entry point `kernel` of the DSA sparse-MLA decode: the native solution slot of the
// reference contest packaging (solution/cuda/kernel.cu:13 and its TVM-FFI binding
// solution/cuda/binding.py:14, with `entry_point = "kernel.cu::kernel"` and
// `binding = "tvm-ffi"` as README.md:259-279 describes).
//
// The function has the reference operator's destination-passing signature
// (solution/triton/fused.py:150): seven tensors and the scale, `output` and `lse` written in
// place, nothing returned.  It reads the DLPack metadata, keeps one lazily allocated,
// zero-initialised workspace per (device, stream) for the split-K partials, and calls the C
// ABI (include/dsa_b200.h) on the stream the TVM-FFI environment names for the device (the
// caller's current CUDA stream).  Argument errors raise TypeError / ValueError, a non-zero
// native status raises RuntimeError.
//
// Built together with dsa_decode.cu for sm_100a only (-gencode arch=compute_100a,code=sm_100a,
// or TVM_FFI_CUDA_ARCH_LIST="10.0a" for tvm_ffi's builder).
#include <cuda_runtime.h>
#include <tvm/ffi/container/tensor.h>
#include <tvm/ffi/error.h>
#include <tvm/ffi/extra/c_env_api.h>
#include <tvm/ffi/function.h>

#include <map>
#include <mutex>
#include <utility>

#include "dsa_b200.h"

namespace {

using tvm::ffi::TensorView;

constexpr int64_t kDCkv = 512;
constexpr int64_t kDKpe = 64;

bool is_bf16(DLDataType t) { return t.code == kDLBfloat && t.bits == 16 && t.lanes == 1; }
bool is_f32(DLDataType t) { return t.code == kDLFloat && t.bits == 32 && t.lanes == 1; }
bool is_i32(DLDataType t) { return t.code == kDLInt && t.bits == 32 && t.lanes == 1; }

void* base_of(const TensorView& t) {
  return static_cast<char*>(t.data_ptr()) + t.byte_offset();
}

// Element stride between consecutive slots of a [..., page, width] pool viewed as a slot
// table (fused.py:155-156 flattens the pools with reshape(-1, D)); the pages must be
// uniformly spaced so that one stride addresses every slot.
int64_t slot_stride(const TensorView& t, int64_t width, const char* name) {
  if (t.ndim() < 2 || t.size(-1) != width)
    TVM_FFI_THROW(ValueError) << name << " must be [..., " << width << "], got ndim " << t.ndim();
  if (t.stride(-1) != 1) TVM_FFI_THROW(ValueError) << name << " must have a unit inner stride";
  if (t.ndim() == 2) return t.stride(0);
  if (t.ndim() == 3 && t.stride(0) == t.stride(1) * t.size(1)) return t.stride(1);
  TVM_FFI_THROW(ValueError) << name << " is not a uniform slot table ([pages, page_size, "
                            << width << "] with evenly spaced pages)";
  return -1;
}

struct Workspace {
  void* ptr = nullptr;
  size_t bytes = 0;
};

// One workspace per (device, stream): calls on one stream run in order, so they may share
// the split-K partial slots; calls on different streams may overlap and must not.
void* workspace_for(int device, void* stream, size_t need) {
  static std::mutex mu;
  static std::map<std::pair<int, void*>, Workspace> table;
  std::lock_guard<std::mutex> lock(mu);
  Workspace& w = table[{device, stream}];
  if (w.bytes >= need) return w.ptr;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(device);
  // The new buffer is allocated and cleared before the old one is released, so a failed
  // allocation leaves the table entry as it was and raises on every call that needs more.
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, need);
  if (e == cudaSuccess) e = cudaMemset(p, 0, need);
  if (e == cudaSuccess && w.ptr != nullptr) {
    cudaStreamSynchronize(static_cast<cudaStream_t>(stream));  // calls in flight use the old one
    cudaFree(w.ptr);
  }
  cudaSetDevice(prev);
  if (e != cudaSuccess) {
    if (p != nullptr) cudaFree(p);
    TVM_FFI_THROW(RuntimeError) << "workspace allocation of " << need
                                << " bytes failed: " << cudaGetErrorString(e);
  }
  w.ptr = p;
  w.bytes = need;
  return p;
}

void kernel(TensorView q_nope, TensorView q_pe, TensorView ckv_cache, TensorView kpe_cache,
            TensorView sparse_indices, double sm_scale, TensorView output, TensorView lse) {
  const DLDevice dev = q_nope.device();
  const std::pair<const char*, const TensorView*> all[] = {
      {"q_nope", &q_nope},       {"q_pe", &q_pe},     {"ckv_cache", &ckv_cache},
      {"kpe_cache", &kpe_cache}, {"sparse_indices", &sparse_indices},
      {"output", &output},       {"lse", &lse}};
  for (const auto& [name, t] : all) {
    if (t->device().device_type != kDLCUDA)
      TVM_FFI_THROW(ValueError) << name << " must be a CUDA tensor (this operator has no CPU path)";
    if (t->device().device_id != dev.device_id)
      TVM_FFI_THROW(ValueError) << name << " is on device " << t->device().device_id
                                << ", expected " << dev.device_id;
  }
  for (const auto& [name, t] : {all[0], all[1], all[2], all[3], all[5]})
    if (!is_bf16(t->dtype())) TVM_FFI_THROW(TypeError) << name << " must be bfloat16";
  if (!is_i32(sparse_indices.dtype())) TVM_FFI_THROW(TypeError) << "sparse_indices must be int32";
  if (!is_f32(lse.dtype())) TVM_FFI_THROW(TypeError) << "lse must be float32";

  if (q_nope.ndim() != 3 || q_nope.size(2) != kDCkv)
    TVM_FFI_THROW(ValueError) << "q_nope must be [num_tokens, num_heads, 512]";
  const int64_t B = q_nope.size(0), H = q_nope.size(1);
  if (q_pe.ndim() != 3 || q_pe.size(0) != B || q_pe.size(1) != H || q_pe.size(2) != kDKpe)
    TVM_FFI_THROW(ValueError) << "q_pe must be [" << B << ", " << H << ", 64]";
  if (sparse_indices.ndim() != 2 || sparse_indices.size(0) != B)
    TVM_FFI_THROW(ValueError) << "sparse_indices must be [" << B << ", topk]";
  if (output.ndim() != 3 || output.size(0) != B || output.size(1) != H || output.size(2) != kDCkv)
    TVM_FFI_THROW(ValueError) << "output must be [" << B << ", " << H << ", 512]";
  if (lse.ndim() != 2 || lse.size(0) != B || lse.size(1) != H)
    TVM_FFI_THROW(ValueError) << "lse must be [" << B << ", " << H << "]";
  if (H != 16 && H != 32 && H != 64 && H != 128)
    TVM_FFI_THROW(ValueError) << "num_heads=" << H << " is not supported (16, 32, 64 or 128)";
  for (const auto& [name, t] : {all[0], all[1], all[4], all[5]})
    if (t->stride(-1) != 1) TVM_FFI_THROW(ValueError) << name << " must have a unit inner stride";

  const int64_t ckv_ss = slot_stride(ckv_cache, kDCkv, "ckv_cache");
  const int64_t kpe_ss = slot_stride(kpe_cache, kDKpe, "kpe_cache");
  const int64_t slots = ckv_cache.numel() / kDCkv;
  if (slots != kpe_cache.numel() / kDKpe)
    TVM_FFI_THROW(ValueError) << "ckv_cache and kpe_cache hold different slot counts";
  if (B == 0) return;

  const int32_t topk = static_cast<int32_t>(sparse_indices.size(1));
  void* stream = TVMFFIEnvGetStream(kDLCUDA, dev.device_id);
  const size_t need = dsa_sparse_mla_decode_workspace_size(B, static_cast<int32_t>(H), topk,
                                                          dev.device_id);
  if (need == 0) TVM_FFI_THROW(ValueError) << "unsupported problem: topk=" << topk;
  void* ws = workspace_for(dev.device_id, stream, need);

  const int rc = dsa_sparse_mla_decode(
      base_of(q_nope), q_nope.stride(0), q_nope.stride(1), base_of(q_pe), q_pe.stride(0),
      q_pe.stride(1), base_of(ckv_cache), ckv_ss, base_of(kpe_cache), kpe_ss, slots,
      static_cast<const int32_t*>(base_of(sparse_indices)), sparse_indices.stride(0),
      static_cast<float>(sm_scale), base_of(output), output.stride(0), output.stride(1),
      static_cast<float*>(base_of(lse)), lse.stride(0), lse.stride(1), B,
      static_cast<int32_t>(H), topk, ws, need, stream);
  if (rc == DSA_ERR_INVALID_ARGUMENT || rc == DSA_ERR_UNSUPPORTED || rc == DSA_ERR_MISALIGNED)
    TVM_FFI_THROW(ValueError) << "dsa_sparse_mla_decode: " << dsa_status_string(rc);
  if (rc != DSA_OK)
    TVM_FFI_THROW(RuntimeError) << "dsa_sparse_mla_decode: " << dsa_status_string(rc)
                                << " (status " << rc << ")";
}

}  // namespace

TVM_FFI_DLL_EXPORT_TYPED_FUNC(kernel, kernel);
