"""B200-native DeepSeek sparse-attention (DSA) sparse-MLA decode.

Drop-in for the reference solution's entry point
``kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output, lse)``
(Dogacel/flashinfer-mlsys2026-dsa, solution/triton/fused.py:150), backed by one
hand-written sm_100a CUDA kernel reached through the C ABI in include/dsa_b200.h.
"""
from .ops import (DSAError, decode, kernel, kernel_paged, read_device_errors,  # noqa: F401
                  set_strict, topk_slots, workspace_for)

__all__ = ["kernel", "kernel_paged", "decode", "topk_slots", "read_device_errors",
           "set_strict", "workspace_for", "DSAError"]
__version__ = "0.1.0"
