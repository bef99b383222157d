"""ctypes binding of the C ABI in include/dsa_b200.h (libdsa_b200.so).

Loading fails loudly: there is no CPU or framework fallback for the decode.
"""
from __future__ import annotations

import ctypes
import os
import threading

from . import build as _build

_lock = threading.Lock()
_lib = None

DSA_OK = 0
DEVERR_BAD_INDEX = 1
DEVERR_TIMEOUT = 2
ERR_SCRATCH_LIMIT = 7

_c = ctypes
_DECODE_ARGTYPES = [
    _c.c_void_p, _c.c_int64, _c.c_int64,            # q_nope, stride_b, stride_h
    _c.c_void_p, _c.c_int64, _c.c_int64,            # q_pe, stride_b, stride_h
    _c.c_void_p, _c.c_int64,                        # ckv_cache, slot stride
    _c.c_void_p, _c.c_int64,                        # kpe_cache, slot stride
    _c.c_int64,                                     # num_slots
    _c.c_void_p, _c.c_int64,                        # sparse_indices, stride_b
    _c.c_float,                                     # sm_scale
    _c.c_void_p, _c.c_int64, _c.c_int64,            # output, stride_b, stride_h
    _c.c_void_p, _c.c_int64, _c.c_int64,            # lse, stride_b, stride_h
    _c.c_int64, _c.c_int32, _c.c_int32,             # num_tokens, num_heads, topk
    _c.c_void_p, _c.c_size_t,                       # workspace, bytes
    _c.c_void_p,                                    # stream
]

# dsa_sparse_mla_decode_paged: the slot ids replaced by page table + positions
_PAGED_ARGTYPES = (_DECODE_ARGTYPES[:11]
                   + [_c.c_void_p, _c.c_int64, _c.c_int32, _c.c_int32,  # page_table, stride_b,
                      #                                                    cols, page_size
                      _c.c_void_p, _c.c_int64]                          # positions, stride_b
                   + _DECODE_ARGTYPES[13:])

EXPORTED_SYMBOLS = (
    "dsa_sparse_mla_decode",
    "dsa_sparse_mla_decode_paged",
    "dsa_sparse_mla_decode_noalloc",
    "dsa_sparse_mla_decode_grouped",
    "dsa_topk_slots",
    "dsa_union_groups",
    "dsa_sparse_mla_decode_workspace_size",
    "dsa_read_error_word",
    "dsa_selftest_bounded_wait",
    "dsa_set_wait_limit",
    "dsa_status_string",
    "dsa_abi_version",
)


class NativeLibraryError(RuntimeError):
    pass


def library_path() -> str:
    return _build.LIB_PATH


def load(build_if_missing: bool = True):
    """Load libdsa_b200.so (building it with nvcc if it is missing)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB_PATH
        if not os.path.exists(path):
            if not build_if_missing:
                raise NativeLibraryError(f"{path} is missing; run flashinfer_mlsys2026_dsa_b200.build")
            _build.build()
        try:
            lib = ctypes.CDLL(path)
        except OSError as e:
            raise NativeLibraryError(f"cannot load {path}: {e}") from e
        lib.dsa_sparse_mla_decode.restype = _c.c_int
        lib.dsa_sparse_mla_decode.argtypes = _DECODE_ARGTYPES
        lib.dsa_sparse_mla_decode_paged.restype = _c.c_int
        lib.dsa_sparse_mla_decode_paged.argtypes = _PAGED_ARGTYPES
        lib.dsa_sparse_mla_decode_noalloc.restype = _c.c_int
        lib.dsa_sparse_mla_decode_noalloc.argtypes = _DECODE_ARGTYPES[:-3] + [_c.c_void_p]
        lib.dsa_topk_slots.restype = _c.c_int
        lib.dsa_topk_slots.argtypes = [_c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p,
                                       _c.c_int64, _c.c_int32, _c.c_int32, _c.c_int64,
                                       _c.c_int32, _c.c_int32, _c.c_void_p, _c.c_int64,
                                       _c.c_void_p]
        lib.dsa_union_groups.restype = _c.c_int
        lib.dsa_union_groups.argtypes = [_c.c_void_p, _c.c_int64, _c.c_int64, _c.c_int32,
                                         _c.c_int32, _c.c_void_p, _c.c_int64, _c.c_int32,
                                         _c.c_int32, _c.c_void_p, _c.c_void_p, _c.c_int64,
                                         _c.c_int32, _c.c_void_p, _c.c_void_p]
        lib.dsa_sparse_mla_decode_grouped.restype = _c.c_int
        lib.dsa_sparse_mla_decode_grouped.argtypes = [
            _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_int64,
            _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_int64,
            _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_int32, _c.c_float,
            _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_void_p, _c.c_int64, _c.c_int64,
            _c.c_int64, _c.c_int32, _c.c_void_p, _c.c_size_t, _c.c_void_p]
        lib.dsa_sparse_mla_decode_workspace_size.restype = _c.c_size_t
        lib.dsa_sparse_mla_decode_workspace_size.argtypes = [_c.c_int64, _c.c_int32, _c.c_int32,
                                                             _c.c_int32]
        lib.dsa_read_error_word.restype = _c.c_int
        lib.dsa_read_error_word.argtypes = [_c.c_void_p, _c.c_void_p, _c.c_int,
                                            _c.POINTER(_c.c_uint32)]
        lib.dsa_set_wait_limit.restype = _c.c_uint64
        lib.dsa_set_wait_limit.argtypes = [_c.c_uint64]
        lib.dsa_selftest_bounded_wait.restype = _c.c_int
        lib.dsa_selftest_bounded_wait.argtypes = [_c.c_int64, _c.c_void_p, _c.c_void_p]
        lib.dsa_status_string.restype = _c.c_char_p
        lib.dsa_status_string.argtypes = [_c.c_int]
        lib.dsa_abi_version.restype = _c.c_int
        lib.dsa_abi_version.argtypes = []
        _lib = lib
        return lib


_ext = None
_ext_tried = False


def ext():
    """The torch binding of the C ABI (built in-tree by ``build.build_ext``), or None.

    It is a faster route to the same native entry point, not a different implementation:
    when it is missing the ctypes route runs the same CUDA kernel.
    """
    global _ext, _ext_tried
    if _ext_tried:
        return _ext
    load()  # the binding links libdsa_b200.so; make sure that is the copy loaded (own lock)
    with _lock:
        if not _ext_tried:
            path = _build.EXT_PATH
            if os.path.exists(path) and not _build.ext_is_stale():
                import importlib.machinery
                import importlib.util

                loader = importlib.machinery.ExtensionFileLoader(_build.EXT_NAME, path)
                spec = importlib.util.spec_from_file_location(_build.EXT_NAME, path, loader=loader)
                mod = importlib.util.module_from_spec(spec)
                loader.exec_module(mod)
                _ext = mod
            _ext_tried = True
    return _ext


def status_text(code: int) -> str:
    return load().dsa_status_string(int(code)).decode()
