"""Stale shared memory never reaches the output.

A padded slot's shared-memory row is written by the gather itself: its id lies outside the
tensor map, so the copy fills the row with zeros (rows of all-padding tiles, which are
not copied, are never read: their score and PV are skipped). If that ever stopped holding,
the row would keep whatever the SM last stored there. These tests fill every SM's shared
memory with NaN bit patterns right before each
decode (a small kernel compiled at run time with NVRTC) and check that padding-heavy inputs
still give finite outputs within tolerance of the reference, bit-identical to an unpoisoned
run.
"""
import numpy as np
import pytest
import torch

import cases
from flashinfer_mlsys2026_dsa_b200 import kernel, read_device_errors, workloads
from oracle import oracle

pytestmark = pytest.mark.gpu

_SRC = r"""
extern "C" __global__ void fill_shared(unsigned int pattern, int words) {
  extern __shared__ unsigned int sm[];
  volatile unsigned int* v = sm;
  for (int i = threadIdx.x; i < words; i += blockDim.x) v[i] = pattern;
}
extern "C" __global__ void read_shared(unsigned int pattern, int words, unsigned int* hits) {
  extern __shared__ unsigned int sm[];
  volatile unsigned int* v = sm;
  unsigned int n = 0;
  for (int i = threadIdx.x; i < words; i += blockDim.x) n += v[i] == pattern;
  atomicAdd(hits, n);
}
"""
_SMEM = 232448  # the largest dynamic shared memory a B200 block may use
_NAN = 0xFFFFFFFF  # a NaN as bf16 pairs and as fp32


class _Poison:
    def __init__(self):
        from cuda.bindings import driver as drv
        from cuda.bindings import nvrtc
        torch.zeros(1, device="cuda")  # the primary context is current on this thread
        major, minor = torch.cuda.get_device_capability()
        err, prog = nvrtc.nvrtcCreateProgram(_SRC.encode(), b"poison.cu", 0, [], [])
        assert err == nvrtc.nvrtcResult.NVRTC_SUCCESS
        opts = [f"--gpu-architecture=sm_{major}{minor}".encode()]
        (err,) = nvrtc.nvrtcCompileProgram(prog, len(opts), opts)
        if err != nvrtc.nvrtcResult.NVRTC_SUCCESS:
            _, n = nvrtc.nvrtcGetProgramLogSize(prog)
            log = b" " * n
            nvrtc.nvrtcGetProgramLog(prog, log)
            raise RuntimeError(log.decode())
        _, n = nvrtc.nvrtcGetCUBINSize(prog)
        cubin = b" " * n
        nvrtc.nvrtcGetCUBIN(prog, cubin)
        err, self.mod = drv.cuModuleLoadData(cubin)
        assert err == drv.CUresult.CUDA_SUCCESS, err
        self.drv = drv
        self.fns = {}
        for name in ("fill_shared", "read_shared"):
            err, fn = drv.cuModuleGetFunction(self.mod, name.encode())
            assert err == drv.CUresult.CUDA_SUCCESS
            (err,) = drv.cuFuncSetAttribute(
                fn, drv.CUfunction_attribute.CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, _SMEM)
            assert err == drv.CUresult.CUDA_SUCCESS
            self.fns[name] = fn
        self.sms = torch.cuda.get_device_properties(0).multi_processor_count

    def _launch(self, name, args, types):
        import ctypes
        drv = self.drv
        stream = torch.cuda.current_stream().cuda_stream
        (err,) = drv.cuLaunchKernel(self.fns[name], 4 * self.sms, 1, 1, 1024, 1, 1, _SMEM,
                                    stream, (args, types), 0)
        assert err == drv.CUresult.CUDA_SUCCESS, err

    def fill(self):
        import ctypes
        self._launch("fill_shared", (_NAN, _SMEM // 4), (ctypes.c_uint32, ctypes.c_int))

    def hits(self):
        """Words of a fresh block's shared memory that still hold the pattern."""
        import ctypes
        h = torch.zeros(1, dtype=torch.int32, device="cuda")
        self._launch("read_shared", (_NAN, _SMEM // 4, h.data_ptr()),
                     (ctypes.c_uint32, ctypes.c_int, ctypes.c_void_p))
        torch.cuda.synchronize()
        return int(h.item())


@pytest.fixture(scope="module")
def poison():
    try:
        return _Poison()
    except ImportError:
        pytest.skip("cuda-python (NVRTC bindings) is not installed")


def _decode(args, poison=None):
    q = args[0]
    B, H, _ = q.shape
    out = torch.empty(B, H, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, H, dtype=torch.float32, device="cuda")
    if poison is not None:
        poison.fill()
    kernel(*args, out, lse)
    torch.cuda.synchronize()
    return out, lse


def test_filled_shared_memory_is_seen_by_the_next_kernel(poison):
    """The premise of the tests below: a block finds the previous kernel's bytes."""
    poison.fill()
    assert poison.hits() > 0


@pytest.mark.parametrize("name", ["ragged_pad", "mid_pad", "topk100", "all_pad_row", "h128_k256"])
def test_poisoned_shared_memory_golden_cases(poison, name):
    from test_gpu_parity import GOLDEN, assert_close, to_dev

    args = to_dev(cases.make_case(name))
    clean = _decode(args)
    out, lse = _decode(args, poison)
    assert torch.equal(out.view(torch.int16), clean[0].view(torch.int16))
    assert torch.equal(lse, clean[1])
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all()
    if name not in cases.REFERENCE_ONLY:
        assert_close(o, lse.cpu().numpy(), oracle.bf16_bits_to_f32(GOLDEN[f"{name}.out"]),
                     GOLDEN[f"{name}.lse"])
    assert read_device_errors() == 0


def test_poisoned_shared_memory_ragged_batch(poison):
    """256 ragged rows (many short ones padded with -1): split rows, padded tiles."""
    from test_gpu_parity import assert_close, oracle_on_workload

    w = workloads.make("ragged_b256", device="cuda", seed=2)
    clean = _decode(w.args())
    out, lse = _decode(w.args(), poison)
    assert torch.equal(out.view(torch.int16), clean[0].view(torch.int16))
    assert torch.equal(lse, clean[1])
    ref_out, ref_lse = oracle_on_workload(w)
    assert_close(out.float().cpu().numpy(), lse.cpu().numpy(), ref_out, ref_lse)
    assert read_device_errors() == 0
