// Warp-level symmetric int8 quantization of one (token, head) row, shared by
// the append kernels so that every writer of the arena rounds identically.
//
// Semantics of the reference (app/src/model/int8_kv_ops.rs:13-21, int8_kv.cu:8-18):
//   s = max(max|x| / 127, 1e-12)            IEEE f32 division
//   q = clamp(round_half_even(x / s), -127, 127)
// Files including this are compiled with -fmad=false -prec-div=true.
#pragma once

#include <stdint.h>

namespace pp {

// Lane l holds elements [l*E, l*E+E) of the row in v[].  Writes the codes of
// its elements and (lane 0) the scale; returns false if any element of the
// row is not finite.
template <int E>
__device__ __forceinline__ bool quantize_vals_warp(const float (&v)[E], uint8_t* codes, float* scale_out, int lane) {
    bool finite = true;
    float m = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        finite = finite && isfinite(v[e]);
        m = fmaxf(m, fabsf(v[e]));
    }
#pragma unroll
    for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float s = fmaxf(__fdiv_rn(m, 127.f), 1e-12f);
    uint32_t packed = 0u;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        int q = __float2int_rn(__fdiv_rn(v[e], s));
        q = max(-127, min(127, q));
        packed |= (uint32_t)(q & 0xff) << (8 * e);
    }
    static_assert(E == 2 || E == 4, "rows of 64 or 128 elements");
    if constexpr (E == 4) {
        *reinterpret_cast<uint32_t*>(codes + (uint64_t)lane * 4) = packed;
    } else {
        *reinterpret_cast<uint16_t*>(codes + (uint64_t)lane * 2) = (uint16_t)packed;
    }
    if (lane == 0) *scale_out = s;
    return __all_sync(0xffffffffu, finite);
}

}  // namespace pp
