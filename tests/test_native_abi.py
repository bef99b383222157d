"""The C ABI library builds, loads and exports every symbol include/dsa_b200.h declares.

No compute call here: this file runs without a GPU.
"""
import ctypes
import os
import re
import subprocess

from flashinfer_mlsys2026_dsa_b200 import _native, build

HEADER = os.path.join(build.REPO_DIR, "include", "dsa_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(dsa_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_python_binding_symbols():
    assert declared_functions() == sorted(_native.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _native.library_path()],
                         capture_output=True, text=True, check=True).stdout
    for name in declared_functions():
        assert re.search(rf"\bT {name}\b", out), f"{name} is not an exported text symbol"


def test_library_targets_sm100a_only():
    """The library is compiled for sm_100a machine code and nothing else (no PTX to JIT).

    On a GPU, every decode test then doubles as the check that this code loads and runs.
    """
    assert build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_abi_version_and_status_text():
    lib = _native.load()
    assert lib.dsa_abi_version() == 1
    assert _native.status_text(0) == "ok"
    assert "num_heads" in _native.status_text(2)
    assert _native.status_text(99) == "unknown status"


def test_host_side_validation_needs_no_gpu():
    """Shape errors are rejected before any CUDA call."""
    lib = _native.load()
    args = [1, 512 * 8, 512, 1, 64 * 8, 64, 1, 512, 1, 64, 100, 1, 256, 0.1,
            1, 512 * 8, 512, 1, 8, 1, 2, 8, 256, 1, 1 << 20, None]
    assert lib.dsa_sparse_mla_decode(*args) == 2                  # 8 heads: unsupported
    args[21] = 16
    args[22] = 0
    assert lib.dsa_sparse_mla_decode(*args) == 1                  # topk = 0
    args[22] = 256
    args[10] = 0
    assert lib.dsa_sparse_mla_decode(*args) == 1                  # no slots
    assert lib.dsa_sparse_mla_decode_workspace_size(2, 8, 256, 0) == 0
    assert lib.dsa_read_error_word(None, None, 0, ctypes.pointer(ctypes.c_uint32())) == 1


def test_build_is_up_to_date():
    assert not build.is_stale(), "libdsa_b200.so is older than its sources"


def test_torch_binding_is_built_and_loads():
    """The fast host route (C++ binding of the C ABI) is present and up to date."""
    from flashinfer_mlsys2026_dsa_b200 import _native
    assert not build.ext_is_stale(), "the torch binding is older than its sources"
    ext = _native.ext()
    assert ext is not None and hasattr(ext, "decode")
