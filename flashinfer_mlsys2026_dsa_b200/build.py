"""Build the native library ``libdsa_b200.so`` in-tree with nvcc for sm_100a.

The library holds the CUDA kernels and the C ABI declared in
``include/dsa_b200.h``.  It links the CUDA runtime dynamically, so inside a
PyTorch process it shares the runtime (current device, streams) torch loaded.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
LIB_NAME = "libdsa_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
SOURCES = [os.path.join(CSRC, "dsa_decode.cu"), os.path.join(CSRC, "dsa_topk.cu")]
TVM_BINDING = os.path.join(CSRC, "kernel.cu")
# every source and header the library is built from (a change to any makes it stale)
DEPS = sorted(
    [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cuh", ".h"))]
    + [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the DSA decode library cannot be built")


def is_stale() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(d) > t for d in DEPS)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not is_stale():
        return LIB_PATH
    tmp = LIB_PATH + f".tmp{os.getpid()}"
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
           "-Xcompiler", "-fPIC", "-shared", "-cudart", "shared",
           "-Xlinker", "-rpath,/usr/local/cuda/lib64",
           "-I", INCLUDE, "-I", CSRC, "-o", tmp, *SOURCES]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


EXT_NAME = "_dsa_torch"
EXT_DIR = os.path.join(PKG_DIR, "_ext_build")
EXT_PATH = os.path.join(EXT_DIR, EXT_NAME + ".so")
EXT_SOURCES = [os.path.join(CSRC, "torch_binding.cpp")]


def ext_is_stale() -> bool:
    if not os.path.exists(EXT_PATH):
        return True
    t = os.path.getmtime(EXT_PATH)
    deps = EXT_SOURCES + [LIB_PATH, os.path.join(INCLUDE, "dsa_b200.h")]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build_ext(force: bool = False, verbose: bool = False) -> str:
    """Build the torch binding of the C ABI (a C++ extension linked to libdsa_b200.so)."""
    if not force and not ext_is_stale():
        return EXT_PATH
    from torch.utils import cpp_extension
    os.makedirs(EXT_DIR, exist_ok=True)
    cpp_extension.load(name=EXT_NAME, sources=EXT_SOURCES, extra_include_paths=[INCLUDE],
                       extra_cflags=["-O2"],
                       extra_ldflags=[f"-L{PKG_DIR}", "-ldsa_b200", f"-Wl,-rpath,{PKG_DIR}"],
                       build_directory=EXT_DIR, verbose=verbose)
    os.utime(EXT_PATH)  # mark it newer than its inputs even when ninja had nothing to do
    return EXT_PATH


TVM_NAME = "dsa_tvm_ffi"
TVM_PATH = os.path.join(EXT_DIR, TVM_NAME + ".so")


def tvm_ffi_present() -> bool:
    try:
        import tvm_ffi.libinfo  # noqa: F401
    except ImportError:
        return False
    return True


def tvm_is_stale() -> bool:
    if not os.path.exists(TVM_PATH):
        return True
    t = os.path.getmtime(TVM_PATH)
    return any(os.path.getmtime(d) > t for d in DEPS)


def build_tvm_ffi(force: bool = False, verbose: bool = False) -> str:
    """Build the TVM-FFI module (``kernel.cu`` + ``dsa_decode.cu``): the contest's CUDA slot."""
    if not force and not tvm_is_stale():
        return TVM_PATH
    from tvm_ffi import libinfo
    lib = libinfo.find_libtvm_ffi()
    os.makedirs(EXT_DIR, exist_ok=True)
    tmp = TVM_PATH + f".tmp{os.getpid()}"
    cmd = [nvcc_path(), *ARCH_FLAGS, "-O3", "-lineinfo", "-std=c++17",
           "-Xcompiler", "-fPIC", "-shared", "-cudart", "shared",
           "-Xlinker", "-rpath,/usr/local/cuda/lib64",
           "-Xlinker", f"-rpath,{os.path.dirname(lib)}",
           "-I", INCLUDE, "-I", CSRC, "-I", libinfo.find_include_path(),
           "-I", libinfo.find_dlpack_include_path(), "-o", tmp, TVM_BINDING, *SOURCES,
           f"-L{os.path.dirname(lib)}", "-ltvm_ffi"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, TVM_PATH)
    return TVM_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
    print(build_ext(force="--force" in sys.argv, verbose="-v" in sys.argv))
    if tvm_ffi_present():
        print(build_tvm_ffi(force="--force" in sys.argv, verbose="-v" in sys.argv))
