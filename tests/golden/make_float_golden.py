"""Generates tests/golden/ref_float_attn.npz by running the REFERENCE's own
float-KV decode attention (pp_attention_f32 / pp_attention_bf16 /
pp_attention_merge from app/src/model/decode_attention.cu, compiled from the
reference sources into oracle/_ref/decode_attention_ref.cubin by
`make -C oracle`) on the float attention cases of cases.py, with the launch
geometry of fused_attention.rs.

Run on a machine with a GPU:  python tests/golden/make_float_golden.py [extra_out.npz]
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
from ref_runner import RefFloatAttention  # noqa: E402

OUT = os.path.join(HERE, "ref_float_attn.npz")


def device_kv(a: np.ndarray) -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda().view(torch.bfloat16)
    return torch.from_numpy(a).cuda()


def main() -> int:
    ref = RefFloatAttention()
    out: dict[str, np.ndarray] = {}
    for name, seed, dtype, batch, heads, size, cap, lengths, split, qs in K.FLOAT_CASES:
        c = K.float_case(seed, dtype, batch, heads, size, cap, lengths, qs)
        lens = c["lengths"]
        out[f"{name}_input_sha"] = np.array(K.sha(c["q"], c["k"], c["v"], *([] if lens is None else [lens])))
        o = ref.attention(torch.from_numpy(c["q"]).cuda(), device_kv(c["k"]), device_kv(c["v"]),
                          None if lens is None else torch.from_numpy(lens.astype(np.int32)).cuda(), heads, split,
                          size=size)
        out[name] = o.cpu().numpy()
    torch.cuda.synchronize()
    np.savez_compressed(OUT, **out)
    if len(sys.argv) > 1:
        np.savez_compressed(sys.argv[1], **out)
    print(f"wrote {OUT}: {len(out)} arrays")
    return 0


if __name__ == "__main__":
    sys.exit(main())
