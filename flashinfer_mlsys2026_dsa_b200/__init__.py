"""B200-native DeepSeek sparse-attention (DSA) sparse-MLA decode.

Drop-in for the reference solution's entry point
``kernel(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output, lse)``
(Dogacel/flashinfer-mlsys2026-dsa, solution/triton/fused.py:150), backed by one
hand-written sm_100a CUDA kernels reached through the C ABI in include/dsa_b200.h.
"""
from .ops import (DSAError, decode, kernel, kernel_grouped, kernel_paged,  # noqa: F401
                  read_device_errors, set_strict, topk_slots, union_groups, workspace_for)

__all__ = ["kernel", "kernel_paged", "kernel_grouped", "decode", "topk_slots", "union_groups",
           "read_device_errors", "set_strict", "workspace_for", "DSAError"]
__version__ = "0.1.0"
