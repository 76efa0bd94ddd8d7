"""Generates tests/golden/ref_renyi.npz by running the REFERENCE's own
pp_renyi_sample (app/src/inference/renyi_sample.cu, compiled from the
reference sources into oracle/_ref/renyi_ref.cubin by `make -C oracle`) on
the sampling cases of cases.py.

Run on a machine with a GPU:  python tests/golden/make_renyi_golden.py [extra_out.npz]
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
from ref_runner import RefRenyiKernel  # noqa: E402

OUT = os.path.join(HERE, "ref_renyi.npz")


def main() -> int:
    ref = RefRenyiKernel()
    out: dict[str, np.ndarray] = {}
    for name, seed, batch, choices, guidance, alpha, cfg, offset in K.RENYI_CASES:
        c = K.renyi_case(seed, batch, choices, guidance)
        out[f"{name}_input_sha"] = np.array(K.sha(c["raw"], c["uniforms"], c["bounds"]))
        o = ref.sample(torch.from_numpy(c["raw"]).cuda(), torch.from_numpy(c["uniforms"]).cuda(),
                       torch.from_numpy(c["bounds"].astype(np.int32)).cuda(), guidance, alpha, cfg, offset)
        out[name] = o.cpu().numpy().view(np.uint32)
    torch.cuda.synchronize()
    np.savez_compressed(OUT, **out)
    if len(sys.argv) > 1:
        np.savez_compressed(sys.argv[1], **out)
    print(f"wrote {OUT}: {len(out)} arrays")
    return 0


if __name__ == "__main__":
    sys.exit(main())
