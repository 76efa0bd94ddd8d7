/*
 * graph_oracle.c -- CPU restatement of the decoder-step operations around the
 * int8 KV path.  TEST INFRASTRUCTURE ONLY: the product never links this file.
 *
 *   oracle_qkv_rope   graph_ops.cu:34-59 (pp_graph_qkv): per (row, head) q/k
 *                     RMSNorm with a 32-lane layout (lane t owns channels
 *                     t + 32e), lane sums in channel order, the shuffle-down
 *                     tree of the warp, x * inv * weight rounded, interleaved
 *                     RoPE with the rounding of every product and sum.
 *   oracle_swiglu     graph_ops.cu:60-74 (pp_graph_swiglu).
 *   oracle_rmsnorm    candle_nn::ops::rms_norm as PrimitiveModel uses it
 *                     (mod.rs:671): f32 sum of squares, x * rsqrt(mean + eps)
 *                     * weight, one rounding; optional residual add first.
 *
 * Parity: the device code uses the hardware reciprocal square root and the
 * CUDA exp; here they are 1/sqrtf and the C library's expf, so results agree
 * with the device within one bf16 unit, not bit for bit.  The bit-exact pin is
 * the reference's own pp_graph_qkv / pp_graph_swiglu run on a B200
 * (tests/golden/ref_graph.npz, made by tests/golden/make_graph_golden.py),
 * against which the GPU tests compare the CUDA kernels.
 * Compiled with -ffp-contract=off: no fused multiply-add anywhere.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

static uint32_t f2u(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    return u;
}
static float u2f(uint32_t u) {
    float x;
    memcpy(&x, &u, 4);
    return x;
}

/* graph_ops.cu:5-9: round to nearest even, NaN kept quiet */
static uint16_t bf_bits(float x) {
    uint32_t b = f2u(x);
    if ((b & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((b >> 16) | 0x40u);
    return (uint16_t)((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}
static float rnd(float x, int bf) { return bf ? u2f((uint32_t)bf_bits(x) << 16) : x; }
static float rd(const void* p, size_t i, int bf) {
    return bf ? u2f((uint32_t)((const uint16_t*)p)[i] << 16) : ((const float*)p)[i];
}
static void wr(void* p, size_t i, float x, int bf) {
    if (bf) ((uint16_t*)p)[i] = bf_bits(x);
    else ((float*)p)[i] = x;
}

/* Sum of one value per lane, in the order of the warp's shuffle-down tree
 * (deltas 16, 8, 4, 2, 1; a lane whose source is out of range adds itself). */
static float warp_tree_sum(float v[32]) {
    float cur[32], nxt[32];
    memcpy(cur, v, sizeof cur);
    for (int delta = 16; delta; delta >>= 1) {
        for (int t = 0; t < 32; ++t) nxt[t] = cur[t] + (t + delta < 32 ? cur[t + delta] : cur[t]);
        memcpy(cur, nxt, sizeof cur);
    }
    return cur[0];
}

int oracle_qkv_rope(const void* qkv, const void* params, const uint32_t* positions, void* out, uint32_t rows,
                    uint32_t heads, uint32_t dim, uint32_t max_context, int bf) {
    if (dim % 32 || dim > 128 || dim == 0) return 1;
    const uint32_t width = heads * dim, per = dim / 32;
    const size_t plane = (size_t)rows * width;
    float q[128], k[128];
    for (uint32_t hr = 0; hr < rows * heads; ++hr) {
        const uint32_t row = hr / heads, head = hr % heads;
        const size_t base = (size_t)row * 3 * width + (size_t)head * dim;
        float qs[32], ks[32];
        for (int t = 0; t < 32; ++t) {
            float a = rd(qkv, base + t, bf), b = rd(qkv, base + width + t, bf);
            qs[t] = a * a;
            ks[t] = b * b;
            for (uint32_t e = 1; e < per; ++e) {
                a = rd(qkv, base + t + 32 * e, bf);
                b = rd(qkv, base + width + t + 32 * e, bf);
                qs[t] = qs[t] + a * a;
                ks[t] = ks[t] + b * b;
            }
        }
        const float qi = 1.0f / sqrtf(warp_tree_sum(qs) / (float)dim + 1.e-6f);
        const float ki = 1.0f / sqrtf(warp_tree_sum(ks) / (float)dim + 1.e-6f);
        for (uint32_t c = 0; c < dim; ++c) {
            q[c] = rnd(rd(qkv, base + c, bf) * qi * rd(params, c, bf), bf);
            k[c] = rnd(rd(qkv, base + width + c, bf) * ki * rd(params, dim + c, bf), bf);
        }
        const uint32_t pos = positions[row];
        if (pos >= max_context) continue;
        const size_t at = (size_t)hr * dim;
        for (uint32_t c = 0; c < dim; ++c) {
            const uint32_t pair = c >> 1;
            const float co = rd(params, 2 * (size_t)dim + (size_t)pos * (dim / 2) + pair, bf);
            const float si = rd(params, 2 * (size_t)dim + (size_t)max_context * (dim / 2) + (size_t)pos * (dim / 2) + pair, bf);
            float qo, ko;
            if (c & 1) {
                qo = rnd(rnd(q[c - 1] * si, bf) + rnd(q[c] * co, bf), bf);
                ko = rnd(rnd(k[c - 1] * si, bf) + rnd(k[c] * co, bf), bf);
            } else {
                qo = rnd(rnd(q[c] * co, bf) - rnd(q[c + 1] * si, bf), bf);
                ko = rnd(rnd(k[c] * co, bf) - rnd(k[c + 1] * si, bf), bf);
            }
            wr(out, at + c, qo, bf);
            wr(out, plane + at + c, ko, bf);
            wr(out, 2 * plane + at + c, rd(qkv, base + 2 * (size_t)width + c, bf), bf);
        }
    }
    return 0;
}

int oracle_swiglu(const void* in, void* out, uint64_t rows, uint32_t hidden, int bf) {
    for (uint64_t i = 0; i < rows * hidden; ++i) {
        const uint64_t row = i / hidden, c = i % hidden;
        const float gate = rd(in, row * hidden * 2 + c, bf), up = rd(in, row * hidden * 2 + hidden + c, bf);
        const float exponential = rnd(expf(-gate), bf);
        const float denominator = rnd(1.f + exponential, bf);
        const float silu = rnd(gate / denominator, bf);
        wr(out, i, rnd(silu * up, bf), bf);
    }
    return 0;
}

int oracle_rmsnorm(const void* x, const void* residual, void* x_sum, const void* weight, void* out, uint64_t rows,
                   uint32_t width, float eps, int bf) {
    for (uint64_t r = 0; r < rows; ++r) {
        const size_t base = (size_t)r * width;
        float ss = 0.f;
        for (uint32_t c = 0; c < width; ++c) {
            float v = rd(x, base + c, bf);
            if (residual) {
                v = rnd(v + rd(residual, base + c, bf), bf);
                if (x_sum) wr(x_sum, base + c, v, bf);
            }
            ss = ss + v * v;
        }
        const float scale = 1.0f / sqrtf(ss / (float)width + eps);
        for (uint32_t c = 0; c < width; ++c) {
            float v = rd(x, base + c, bf);
            if (residual) v = rnd(v + rd(residual, base + c, bf), bf);
            wr(out, base + c, v * scale * rd(weight, c, bf), bf);
        }
    }
    return 0;
}
