"""Contest packaging: the Solution JSON, its sources built by tvm_ffi's builder, and the
TVM-FFI entry point ``kernel`` (solution/cuda/kernel.cu:13 / binding.py:14 slot of the
reference, README.md:259-279).

CPU tests check the document, that the flattened sources compile with tvm_ffi's own
builder for sm_100a, and the entry point's argument errors (raised before any CUDA call).
GPU tests call the TVM-FFI ``kernel`` with torch tensors and compare it with the Python
entry point (same kernels: bit-identical) and with the reference's golden outputs.
"""
import json
import os

import numpy as np
import pytest
import torch

tvm_ffi = pytest.importorskip("tvm_ffi")

from flashinfer_mlsys2026_dsa_b200 import build as nbuild  # noqa: E402
from flashinfer_mlsys2026_dsa_b200 import solution  # noqa: E402


def test_solution_document(tmp_path):
    path = solution.pack_solution(str(tmp_path / "solution.json"), name="n", author="a")
    doc = json.loads(open(path).read())
    assert doc["name"] == "n" and doc["author"] == "a"
    assert doc["definition"] == "dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64"
    spec = doc["spec"]
    assert spec["language"] == "cuda" and spec["binding"] == "tvm-ffi"
    assert spec["entry_point"] == "kernel.cu::kernel"
    assert spec["destination_passing_style"] is True
    names = [s["path"] for s in doc["sources"]]
    assert spec["entry_point"].split("::")[0] in names
    for rel, repo_path in solution.SOURCE_FILES:
        got = next(s["content"] for s in doc["sources"] if s["path"] == rel)
        assert got == open(repo_path).read()
    # every quoted include of a packed source resolves inside the flat directory
    for s in doc["sources"]:
        for line in s["content"].splitlines():
            if line.startswith('#include "'):
                assert line.split('"')[1] in names, (s["path"], line)


def test_unpack_rejects_escaping_paths(tmp_path):
    doc = {"sources": [{"path": "../x.cu", "content": ""}]}
    with pytest.raises(ValueError):
        solution.write_sources(doc, str(tmp_path))


def _cpu_args():
    B, H = 2, 16
    bf = torch.bfloat16
    return [torch.zeros(B, H, 512, dtype=bf), torch.zeros(B, H, 64, dtype=bf),
            torch.zeros(4, 64, 512, dtype=bf), torch.zeros(4, 64, 64, dtype=bf),
            torch.zeros(B, 8, dtype=torch.int32), 0.1,
            torch.empty(B, H, 512, dtype=bf), torch.empty(B, H)]


def test_packed_sources_build_with_tvm_ffi_builder(tmp_path):
    so = solution.build_sources(solution.solution_dict(), str(tmp_path / "sol"))
    mod = tvm_ffi.load_module(so)
    with pytest.raises(ValueError, match="CUDA tensor"):
        mod.kernel(*_cpu_args())


def test_in_tree_module_exports_kernel_and_rejects_cpu_tensors():
    mod = solution.load_module()
    assert os.path.exists(nbuild.TVM_PATH)
    with pytest.raises(ValueError, match="no CPU path"):
        mod.kernel(*_cpu_args())


# ---------------------------------------------------------------------------- GPU

def _golden_args(name):
    import cases
    from test_gpu_parity import to_dev
    return cases.make_case(name), to_dev(cases.make_case(name))


def _outputs(args):
    B, H, _ = args[0].shape
    out = torch.full((B, H, 512), float("nan"), dtype=torch.bfloat16, device="cuda")
    lse = torch.full((B, H), float("nan"), dtype=torch.float32, device="cuda")
    return out, lse


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["tiny_b2_h16_k256", "ragged_pad", "h128_k256", "many_rows", "neg_index"])
def test_tvm_ffi_kernel_matches_python_entry_and_reference(name):
    import cases
    from test_gpu_parity import GOLDEN, assert_close
    from oracle import oracle
    from flashinfer_mlsys2026_dsa_b200 import _native, kernel, read_device_errors

    read_device_errors(clear=True)

    _, args = _golden_args(name)
    mod = solution.load_module()
    out_t, lse_t = _outputs(args)
    mod.kernel(*args, out_t, lse_t)
    out_p, lse_p = _outputs(args)
    kernel(*args, out_p, lse_p)
    torch.cuda.synchronize()
    assert torch.equal(out_t.view(torch.int16), out_p.view(torch.int16))
    assert torch.equal(lse_t, lse_p)
    if name not in cases.REFERENCE_ONLY:
        assert_close(out_t.float().cpu().numpy(), lse_t.cpu().numpy(),
                     oracle.bf16_bits_to_f32(GOLDEN[f"{name}.out"]), GOLDEN[f"{name}.lse"])
    if name == "neg_index":  # the bad index is flagged in the Python entry's workspace
        assert read_device_errors() & _native.DEVERR_BAD_INDEX
    else:
        assert read_device_errors() == 0


@pytest.mark.gpu
def test_tvm_ffi_kernel_runs_on_the_torch_stream_it_is_given():
    from flashinfer_mlsys2026_dsa_b200 import workloads

    args = workloads.make("b64_h16", device="cuda", seed=3).args()
    mod = solution.load_module()
    ref_out, ref_lse = _outputs(args)
    mod.kernel(*args, ref_out, ref_lse)
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    out, lse = _outputs(args)
    s.wait_stream(torch.cuda.current_stream())
    with tvm_ffi.use_torch_stream(torch.cuda.stream(s)):
        for _ in range(3):
            mod.kernel(*args, out, lse)
    s.synchronize()
    assert torch.equal(out.view(torch.int16), ref_out.view(torch.int16))
    assert torch.equal(lse, ref_lse)


@pytest.mark.gpu
def test_tvm_ffi_kernel_argument_errors():
    _, args = _golden_args("tiny_b2_h16_k256")
    mod = solution.load_module()
    out, lse = _outputs(args)
    with pytest.raises(TypeError):
        mod.kernel(args[0].float(), *args[1:], out, lse)
    with pytest.raises(TypeError):
        mod.kernel(*args[:4], args[4].long(), args[5], out, lse)
    with pytest.raises(ValueError):
        mod.kernel(*args, out[:, :, :256], lse)
    q = args[0][:, :1].expand(-1, 24, -1)  # 24 heads: unsupported
    with pytest.raises(ValueError):
        mod.kernel(q, args[1][:, :1].expand(-1, 24, -1), *args[2:], out[:, :1].expand(-1, 24, -1),
                   lse[:, :1].expand(-1, 24))
