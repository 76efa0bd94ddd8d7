"""Generates tests/golden/ref_graph.npz by running the REFERENCE's own
pp_graph_qkv and pp_graph_swiglu (app/src/model/graph_ops.cu, compiled from the
reference sources into oracle/_ref/graph_ops_ref.cubin by `make -C oracle`)
on the decoder-step cases of cases.py, in f32 and in bf16.

Run on a machine with a GPU:  python tests/golden/make_graph_golden.py [extra_out.npz]
The output file is committed; the CPU tests check the oracle against it and the
GPU tests check the CUDA kernels against it bit for bit.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import cases as K  # noqa: E402
from ref_runner import RefGraphKernels  # noqa: E402

OUT = os.path.join(HERE, "ref_graph.npz")


def dev(x: np.ndarray, bf: bool) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    return t.to(torch.bfloat16) if bf else t


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    return t.cpu().numpy().view(np.uint32)


def main() -> int:
    ref = RefGraphKernels()
    out: dict[str, np.ndarray] = {}
    for name, seed, rows, heads, dim, max_ctx in K.QKV_CASES:
        c = K.qkv_case(seed, rows, heads, dim, max_ctx)
        out[f"{name}_input_sha"] = np.array(K.sha(c["qkv"], c["params"], c["positions"]))
        for bf in (False, True):
            pos = torch.from_numpy(c["positions"].astype(np.int32)).cuda()
            o = ref.qkv(dev(c["qkv"], bf), dev(c["params"], bf), pos, heads, dim, max_ctx)
            out[f"{name}_{'bf16' if bf else 'f32'}"] = bits(o)
    for name, seed, rows, hidden in K.SWIGLU_CASES:
        x = K.swiglu_case(seed, rows, hidden)
        out[f"{name}_input_sha"] = np.array(K.sha(x))
        for bf in (False, True):
            out[f"{name}_{'bf16' if bf else 'f32'}"] = bits(ref.swiglu(dev(x, bf)))
    torch.cuda.synchronize()
    np.savez_compressed(OUT, **out)
    if len(sys.argv) > 1:
        np.savez_compressed(sys.argv[1], **out)
    print(f"wrote {OUT}: {len(out)} arrays")
    return 0


if __name__ == "__main__":
    sys.exit(main())
