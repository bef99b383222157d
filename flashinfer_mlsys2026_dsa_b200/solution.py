"""Contest packaging of the CUDA solution: ``solution.json`` for flashinfer-bench.

The reference packs its solution with scripts/pack_solution.py (which reads config.toml and
calls flashinfer_bench's ``pack_solution_from_files``) into a Solution JSON: name,
definition, author, a build ``spec`` and the source files (README.md:233-279).  This
module writes the same document for the native solution: ``language = "cuda"``,
``entry_point = "kernel.cu::kernel"`` and ``binding = "tvm-ffi"``, with the sources
flattened into one directory (``kernel.cu`` is the TVM-FFI entry point,
``dsa_decode.cu`` the kernels and the C ABI, plus their headers).  flashinfer_bench is not
installed here, so the document follows the schema the README shows (the ``sources``
items carry ``path`` and ``content``); :func:`build_sources` compiles the flattened
directory with tvm_ffi's own builder, as the benchmark's tvm-ffi builder does.

    python -m flashinfer_mlsys2026_dsa_b200.solution --out solution.json
"""
from __future__ import annotations

import argparse
import json
import os

from . import build as _build

# the definition the reference solution is registered for (config.toml:3)
DEFINITION = "dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64"
ENTRY_POINT = "kernel.cu::kernel"
# (name in the solution, file in this repository)
SOURCE_FILES = (
    ("kernel.cu", os.path.join(_build.CSRC, "kernel.cu")),
    ("dsa_decode.cu", os.path.join(_build.CSRC, "dsa_decode.cu")),
    ("dsa_pipeline.cuh", os.path.join(_build.CSRC, "dsa_pipeline.cuh")),
    ("dsa_decode_h16.cuh", os.path.join(_build.CSRC, "dsa_decode_h16.cuh")),
    ("dsa_decode_hm.cuh", os.path.join(_build.CSRC, "dsa_decode_hm.cuh")),
    ("sm100_ptx.cuh", os.path.join(_build.CSRC, "sm100_ptx.cuh")),
    ("dsa_b200.h", os.path.join(_build.INCLUDE, "dsa_b200.h")),
)
CUDA_FILES = ("kernel.cu", "dsa_decode.cu")
# the kernels use tcgen05 and TMA gathers: sm_100a only
CUDA_ARCH_LIST = "10.0a"


def solution_dict(name: str = "dsa-b200-sparse-mla-decode",
                  author: str = "flashinfer_mlsys2026_dsa_b200") -> dict:
    sources = []
    for rel, path in SOURCE_FILES:
        with open(path, encoding="utf-8") as f:
            sources.append({"path": rel, "content": f.read()})
    return {
        "name": name,
        "definition": DEFINITION,
        "author": author,
        "spec": {
            "language": "cuda",
            "target_hardware": ["cuda"],
            "entry_point": ENTRY_POINT,
            "dependencies": [],
            "destination_passing_style": True,
            "binding": "tvm-ffi",
        },
        "sources": sources,
    }


def pack_solution(out_path: str, **kw) -> str:
    """Write the Solution JSON to ``out_path`` and return the path."""
    with open(out_path, "w", encoding="utf-8") as f:
        json.dump(solution_dict(**kw), f, indent=2)
        f.write("\n")
    return out_path


def write_sources(solution: dict, directory: str) -> list[str]:
    """Unpack a Solution document's sources into ``directory``; returns the CUDA files."""
    os.makedirs(directory, exist_ok=True)
    for src in solution["sources"]:
        rel = src["path"]
        if os.path.isabs(rel) or ".." in rel.split("/"):
            raise ValueError(f"source path escapes the solution directory: {rel}")
        with open(os.path.join(directory, rel), "w", encoding="utf-8") as f:
            f.write(src["content"])
    return [os.path.join(directory, rel) for rel in CUDA_FILES]


def build_sources(solution: dict, directory: str, name: str = "dsa_solution") -> str:
    """Compile an unpacked solution with tvm_ffi's builder for sm_100a; returns the .so path."""
    import tvm_ffi.cpp

    cuda_files = write_sources(solution, directory)
    prev = os.environ.get("TVM_FFI_CUDA_ARCH_LIST")
    os.environ["TVM_FFI_CUDA_ARCH_LIST"] = CUDA_ARCH_LIST
    try:
        return tvm_ffi.cpp.build(name, cuda_files=cuda_files,
                                 extra_cuda_cflags=["-O3", "-lineinfo"],
                                 extra_include_paths=[directory],
                                 build_directory=os.path.join(directory, "build"))
    finally:
        if prev is None:
            os.environ.pop("TVM_FFI_CUDA_ARCH_LIST", None)
        else:
            os.environ["TVM_FFI_CUDA_ARCH_LIST"] = prev


def load_module():
    """The in-tree TVM-FFI module (built by ``build.build_tvm_ffi``); ``.kernel`` is the op."""
    import tvm_ffi

    path = _build.build_tvm_ffi()
    return tvm_ffi.load_module(path)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--out", default="solution.json")
    ap.add_argument("--name", default="dsa-b200-sparse-mla-decode")
    ap.add_argument("--author", default="flashinfer_mlsys2026_dsa_b200")
    a = ap.parse_args(argv)
    print(pack_solution(a.out, name=a.name, author=a.author))


if __name__ == "__main__":
    main()
