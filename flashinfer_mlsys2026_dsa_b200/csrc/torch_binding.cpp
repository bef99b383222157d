// Python binding of the C ABI (include/dsa_b200.h) for torch tensors.  It reads the tensors'
// metadata in C++, so one decode call costs a few microseconds of host time instead of the
// tens that ctypes spends on 26 marshalled arguments and Python attribute reads.
//
// decode(...) returns the native status, or -1 when an argument is not in the plain form
// handled here (a CPU tensor, a dtype or shape mismatch, a non-unit inner stride, a pool
// that is not a uniform slot table); the Python caller then takes its general path, which
// validates, raises the precise error or copies to a supported layout.
#include <torch/extension.h>

#include "dsa_b200.h"

namespace {

constexpr int64_t kNotHandled = -1;

// Slot stride of a [..., page, width] pool whose pages are uniformly spaced, else -1.
int64_t slot_stride(const at::Tensor& t, int64_t width) {
  if (t.size(-1) != width || t.stride(-1) != 1) return -1;
  if (t.dim() == 2) return t.stride(0);
  if (t.dim() == 3 && t.stride(0) == t.stride(1) * t.size(1)) return t.stride(1);
  return -1;
}

int64_t decode(const at::Tensor& q_nope, const at::Tensor& q_pe, const at::Tensor& ckv,
               const at::Tensor& kpe, const at::Tensor& idx, double sm_scale,
               const at::Tensor& out, const at::Tensor& lse, const at::Tensor& ws,
               int64_t stream) {
  const auto bf16 = at::kBFloat16;
  if (!q_nope.is_cuda() || q_nope.dim() != 3 || q_nope.size(2) != 512) return kNotHandled;
  const int64_t B = q_nope.size(0), H = q_nope.size(1);
  const auto dev = q_nope.device();
  for (const at::Tensor* t : {&q_pe, &ckv, &kpe, &idx, &out, &lse, &ws})
    if (t->device() != dev) return kNotHandled;
  if (q_nope.scalar_type() != bf16 || q_pe.scalar_type() != bf16 || ckv.scalar_type() != bf16 ||
      kpe.scalar_type() != bf16 || out.scalar_type() != bf16 ||
      idx.scalar_type() != at::kInt || lse.scalar_type() != at::kFloat)
    return kNotHandled;
  if (q_pe.dim() != 3 || q_pe.size(0) != B || q_pe.size(1) != H || q_pe.size(2) != 64 ||
      idx.dim() != 2 || idx.size(0) != B || out.dim() != 3 || out.size(0) != B ||
      out.size(1) != H || out.size(2) != 512 || lse.dim() != 2 || lse.size(0) != B ||
      lse.size(1) != H)
    return kNotHandled;
  if (q_nope.stride(2) != 1 || q_pe.stride(2) != 1 || idx.stride(1) != 1 || out.stride(2) != 1)
    return kNotHandled;
  const int64_t ckv_ss = slot_stride(ckv, 512), kpe_ss = slot_stride(kpe, 64);
  if (ckv_ss < 0 || kpe_ss < 0) return kNotHandled;
  const int64_t ckv_slots = ckv.numel() / 512, kpe_slots = kpe.numel() / 64;
  if (ckv_slots != kpe_slots) return kNotHandled;
  return dsa_sparse_mla_decode(
      q_nope.data_ptr(), q_nope.stride(0), q_nope.stride(1), q_pe.data_ptr(), q_pe.stride(0),
      q_pe.stride(1), ckv.data_ptr(), ckv_ss, kpe.data_ptr(), kpe_ss, ckv_slots,
      static_cast<const int32_t*>(idx.data_ptr()), idx.stride(0), (float)sm_scale,
      out.data_ptr(), out.stride(0), out.stride(1), static_cast<float*>(lse.data_ptr()),
      lse.stride(0), lse.stride(1), B, (int32_t)H, (int32_t)idx.size(1), ws.data_ptr(),
      (size_t)ws.numel(), reinterpret_cast<void*>(stream));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("decode", &decode, "DSA sparse-MLA decode through the C ABI (status, -1: not handled)");
}
