/*
 * sample_oracle.c -- CPU restatement of the reference's fused Rényi sampler
 * (app/src/inference/renyi_sample.cu, launched by fused_sampling.rs:125-162
 * with 256 threads per row).  TEST INFRASTRUCTURE ONLY.
 *
 * The per-thread partial sums (columns t, t + 256, ...) and the pairwise tree
 * of the block are replayed in the same order.  The device uses fast
 * exponential / logarithm intrinsics; here they are expf / logf, so a support
 * that lands within a rounding step of .5 may differ by one.  The bit-exact
 * pin of the CUDA kernel is the reference kernel run on a B200
 * (tests/golden/ref_renyi.npz, made by tests/golden/make_renyi_golden.py).
 * Compiled with -ffp-contract=off.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define THREADS 256

static int finite_f(float v) {
    uint32_t u;
    memcpy(&u, &v, 4);
    return (u & 0x7fffffffu) < 0x7f800000u;
}
static int ahead(float a, uint32_t ai, float b, uint32_t bi) { return a > b || (a == b && ai < bi); }

static void put(uint32_t* out, uint32_t batch, uint32_t row, uint32_t tok, uint32_t ok, uint32_t sup) {
    out[row] = tok;
    out[batch + row] = ok;
    out[2 * batch + row] = sup;
}

int oracle_renyi_sample(const float* raw, const float* uniforms, const uint32_t* bounds, uint32_t* out,
                        uint32_t batch, uint32_t choices, uint32_t guidance, float alpha, float cfg,
                        uint32_t offset) {
    static float vals[2048];
    static uint32_t cols[2048];
    if (choices > 2048 || (guidance != 1 && guidance != 2)) return 1;
    for (uint32_t row = 0; row < batch; ++row) {
        const uint32_t start = bounds[2 * row], count = bounds[2 * row + 1];
        const float u = uniforms[row];
        const uint32_t clamped = start < choices ? start : 0u;
        if (!finite_f(u) || u < 0.f || u >= 1.f || start >= choices || count == 0 || count > choices - clamped) {
            put(out, batch, row, offset + clamped, 0, 1);
            continue;
        }
        const float* xr = raw + (size_t)row * guidance * choices;
        float tv[THREADS];
        uint32_t ti[THREADS], tb[THREADS];
        for (int t = 0; t < THREADS; ++t) {
            tv[t] = -INFINITY;
            ti[t] = 0xffffffffu;
            tb[t] = 0;
        }
        for (uint32_t c = 0; c < choices; ++c) {
            const int t = (int)(c % THREADS);
            const float x = xr[c];
            float v = x;
            int ok = finite_f(x);
            if (guidance == 2) {
                const float un = xr[choices + c];
                ok = ok && finite_f(un);
                v = un + cfg * (x - un);
            }
            ok = ok && finite_f(v);
            tb[t] |= !ok;
            if (!ok) v = 0.f;
            if (c >= start && c - start < count) {
                vals[c - start] = v;
                cols[c - start] = c;
                if (ahead(v, c, tv[t], ti[t])) {
                    tv[t] = v;
                    ti[t] = c;
                }
            }
        }
        for (int step = THREADS / 2; step; step >>= 1)
            for (int t = 0; t < step; ++t) {
                if (ahead(tv[t + step], ti[t + step], tv[t], ti[t])) {
                    tv[t] = tv[t + step];
                    ti[t] = ti[t + step];
                }
                tb[t] |= tb[t + step];
            }
        if (tb[0]) {
            put(out, batch, row, offset + start, 0, 1);
            continue;
        }
        const float m = tv[0];
        const uint32_t m_col = ti[0];
        float z[THREADS], za[THREADS];
        for (int t = 0; t < THREADS; ++t) z[t] = za[t] = 0.f;
        for (uint32_t c = 0; c < count; ++c) {
            const int t = (int)(c % THREADS);
            const float d = vals[c] - m;
            z[t] += expf(d);
            za[t] += expf(alpha * d);
        }
        for (int step = THREADS / 2; step; step >>= 1)
            for (int t = 0; t < step; ++t) {
                z[t] += z[t + step];
                za[t] += za[t + step];
            }
        const float lz = logf(z[0]), lza = logf(za[0]);
        float corr = lz - lza;
        if (corr < 0.f) corr = 0.f;
        float h = lz + corr / (alpha - 1.f);
        if (!finite_f(lz) || !finite_f(lza) || !finite_f(h)) {
            put(out, batch, row, offset + start, 0, 1);
            continue;
        }
        const float h_max = logf((float)count);
        if (h < 0.f) h = 0.f;
        if (h > h_max) h = h_max;
        uint32_t support = (uint32_t)(expf(h) + 0.5f);
        if (support < 1) support = 1;
        if (support > count) support = count;
        uint32_t rank = (uint32_t)(u * (float)support);
        if (rank >= support) rank = support - 1;
        if (rank == 0) {
            put(out, batch, row, offset + m_col, 1, support);
            continue;
        }
        /* rank-th by (value desc, column asc): count how many come ahead of each */
        for (uint32_t i = 0; i < count; ++i) {
            uint32_t before = 0;
            for (uint32_t j = 0; j < count; ++j)
                if (j != i && ahead(vals[j], cols[j], vals[i], cols[i])) ++before;
            if (before == rank) {
                put(out, batch, row, offset + cols[i], 1, support);
                break;
            }
        }
    }
    return 0;
}
