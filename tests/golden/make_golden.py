"""Write tests/golden/golden.npz by running the reference implementation.

Run in a container that holds the reference checkout (it is read, never
copied):  python tests/golden/make_golden.py /path/to/reference

For every case of cases.py it imports solution/triton/baseline.py of the
reference, calls its ``kernel`` on CPU tensors and stores the outputs (bf16
bits and the base-2 LSE) with a SHA-256 of the inputs.  The tests never
need the reference at run time: they only read the .npz.
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import cases  # noqa: E402


def _load_reference(ref_root: str):
    path = os.path.join(ref_root, "solution", "triton", "baseline.py")
    spec = importlib.util.spec_from_file_location("dsa_reference_baseline", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _bf16_tensor(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)


def main(ref_root: str):
    ref = _load_reference(ref_root)
    arrays, meta = {}, {}
    for name in cases.CASES:
        c = cases.make_case(name)
        B, H, _ = c["q_nope"].shape
        out = torch.empty(B, H, 512, dtype=torch.bfloat16)
        lse = torch.empty(B, H, dtype=torch.float32)
        ref.kernel(_bf16_tensor(c["q_nope"]), _bf16_tensor(c["q_pe"]),
                   _bf16_tensor(c["ckv_cache"]), _bf16_tensor(c["kpe_cache"]),
                   torch.from_numpy(c["sparse_indices"]), c["sm_scale"], out, lse)
        arrays[f"{name}.out"] = out.view(torch.int16).numpy().view(np.uint16)
        arrays[f"{name}.lse"] = lse.numpy()
        meta[name] = dict(digest=cases.input_digest(c), spec=cases.CASES[name])
        print(f"{name}: out[0,0,:4]={out[0,0,:4].tolist()} lse[0,:2]={lse[0,:2].tolist()}")
    here = os.path.dirname(os.path.abspath(__file__))
    np.savez_compressed(os.path.join(here, "golden.npz"), **arrays)
    with open(os.path.join(here, "golden.json"), "w") as f:
        json.dump(dict(torch=torch.__version__, generator="numpy PCG64", cases=meta), f,
                  indent=1, sort_keys=True)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
