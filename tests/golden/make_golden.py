"""Generates tests/golden/ref_int8kv.npz by running the REFERENCE's own CUDA
kernels (app/src/model/int8_kv.cu, compiled from the reference sources into
oracle/_ref/int8_kv_ref.cubin by `make -C oracle`) on the cases of cases.py.

Run on a machine with a GPU:  python tests/golden/make_golden.py
The launch geometry is the reference's (oracle/ref_runner.py mirrors
int8_kv_ops.rs:120-161).  The output file is committed; the CPU test suite
checks the oracle against it and the GPU suite checks the CUDA path.
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
from ref_runner import RefInt8Kernels  # noqa: E402

OUT = os.path.join(HERE, "ref_int8kv.npz")


def dev(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def host(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def main() -> int:
    ref = RefInt8Kernels()
    out: dict[str, np.ndarray] = {}

    # --- prep1: quantize round trip + attention (int8_kv_ops.rs:59-73)
    c = K.prep1()
    codes, scales = ref.quantize(dev(c["x"]))
    out["prep1_codes"], out["prep1_scales"] = host(codes), host(scales)
    out["prep1_unpack"] = host(ref.dequantize(codes, scales))
    o = ref.attention(dev(c["q"]).reshape(2, 1, 64), codes, codes, scales, scales, dev(c["sk"]).reshape(2, 1, 64),
                      dev(c["sk"]).reshape(2, 1, 64), dev(c["past"].astype(np.int32)), c["heads"], c["split"])
    out["prep1_out"] = host(o)

    # --- prep2: view offsets, heads=2, past [0,66], splits {32,128} (:75-101)
    c = K.prep2()
    rows, cap, heads = c["rows"], c["cap"], c["heads"]
    hist = dev(c["hist"])[1:]
    vals = dev(c["vals"])[1:]
    k, ks = ref.quantize(hist.contiguous())
    v, vs = ref.quantize(vals.contiguous())
    out["prep2_k_codes"], out["prep2_k_scales"] = host(k), host(ks)
    out["prep2_v_codes"], out["prep2_v_scales"] = host(v), host(vs)
    kb = torch.cat([k[0:1], k])[1:]
    vb = torch.cat([v[0:1], v])[1:]
    ksb = torch.cat([ks[0:1], ks])[1:]
    vsb = torch.cat([vs[0:1], vs])[1:]
    q = dev(c["q"])[1:].reshape(rows, 1, 64)
    sk = dev(c["sk"])[1:].reshape(rows, 1, 64)
    sv = dev(c["sv"])[1:].reshape(rows, 1, 64)
    past = dev(c["past_all"].astype(np.int32))[1:]
    for split in (32, 128):
        out[f"prep2_out_s{split}"] = host(ref.attention(q, kb, vb, ksb, vsb, sk, sv, past, heads, split))

    # --- int8 layer-cache data generator (int8_cache.rs:19-23)
    for idx, (h, n, bias) in enumerate(K.CACHE_CASES):
        codes, scales = ref.quantize(dev(K.cache_data(h, n, bias)))
        out[f"cache{idx}_codes"], out[f"cache{idx}_scales"] = host(codes), host(scales)

    # --- bf16 inputs, widened exactly (kv_int8.cpp:168-176 shapes)
    c = K.hip_bf16()
    for name in ("k", "v"):
        x = K.bf16_to_f32(c[f"{name}_bits"])
        codes, scales = ref.quantize(dev(x))
        out[f"hip_{name}_codes_sha"] = np.array(K.sha(host(codes)))
        out[f"hip_{name}_scales"] = host(scales)

    # --- edge rows
    codes, scales = ref.quantize(dev(K.edge_rows()))
    out["edge_codes"], out["edge_scales"] = host(codes), host(scales)

    # --- random reference-mode cases
    for name, seed, b, h, cap, pasts, split in K.RANDOM_CASES:
        c = K.random_case(seed, b, h, cap)
        rows = b * h
        out[f"{name}_input_sha"] = np.array(K.sha(c["k"], c["v"], c["q"], c["sk"], c["sv"]))
        k, ks = ref.quantize(dev(c["k"]))
        v, vs = ref.quantize(dev(c["v"]))
        out[f"{name}_codes_sha"] = np.array(K.sha(host(k), host(ks), host(v), host(vs)))
        o = ref.attention(dev(c["q"]).reshape(rows, 1, 64), k, v, ks, vs, dev(c["sk"]).reshape(rows, 1, 64),
                          dev(c["sv"]).reshape(rows, 1, 64), dev(np.array(pasts, dtype=np.int32)), h, split)
        out[f"{name}_out"] = host(o)

    # --- BASELINE config 0 in all-int8 form: the reference kernel's scratch
    # token at index 1023 is fed the bf16 dequantized history token 1023.
    c = K.cfg0_case(0)
    out["cfg0_input_sha"] = np.array(K.sha(c["k"], c["v"], c["q"]))
    k, ks = ref.quantize(dev(c["k"]))
    v, vs = ref.quantize(dev(c["v"]))
    out["cfg0_codes_sha"] = np.array(K.sha(host(k), host(ks), host(v), host(vs)))
    kd = K.bf16_to_f32(K.to_bf16_bits(host(ref.dequantize(k, ks))))
    vd = K.bf16_to_f32(K.to_bf16_bits(host(ref.dequantize(v, vs))))
    sk = dev(kd[:, 1023, :]).reshape(16, 1, 64)
    sv = dev(vd[:, 1023, :]).reshape(16, 1, 64)
    past = dev(np.array([1023], dtype=np.int32))
    out["cfg0_out"] = host(ref.attention(dev(c["q"]).reshape(16, 1, 64), k, v, ks, vs, sk, sv, past, 16, 128))

    torch.cuda.synchronize()
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(out)} arrays, {os.path.getsize(OUT)} bytes")
    if len(sys.argv) > 1:  # optional extra copy (e.g. into a results folder)
        np.savez_compressed(sys.argv[1], **out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
