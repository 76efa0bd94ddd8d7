/*
 * int8kv_oracle.c -- CPU restatement of the reference int8 historical-KV path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: only tests/, the
 * smoke() entry point and bench.py's cpu_baseline / reference arm may load
 * it.  The product library (libpp_b200.so) never links or calls it.
 *
 * Parity pinning: the restatement is checked against the reference's own
 * CUDA kernels (app/src/model/int8_kv.cu, compiled from the reference
 * sources into oracle/_ref/ by oracle/Makefile and run on a B200 by
 * tests/golden/make_golden.py).  Their outputs are committed as
 * tests/golden/ref_int8kv_*.npz and tests/test_oracle_golden.py checks this
 * file against them (codes/scales bit-exact, attention within the
 * reference's own self-check tolerance of 2e-5).
 *
 * Every function cites the reference code it restates (paths relative to the
 * reference project root).  Compile with -ffp-contract=off so that products
 * and sums round separately, as Rust does.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include <pthread.h>

#define ORACLE_OK 0
#define ORACLE_NON_FINITE 1
#define ORACLE_BAD_GEOMETRY 2

static inline uint32_t f2u(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float u2f(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* bf16 round-to-nearest-even of an f32 value, returned widened to f32.
 * Restates half::bf16::from_f32 (half 2.7.1, the dependency pinned in
 * app/Cargo.lock) as used by Candle's F32->BF16 cast
 * (app/vendor/candle-core/src/cpu_backend/mod.rs:1885) and the identical
 * bit trick pp_round_bf16 in app/src/model/int8_kv.cu:3-7.  NaN stays NaN. */
float oracle_bf16_round(float x) {
    uint32_t u = f2u(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return u2f((u | 0x00400000u) & 0xffff0000u);
    uint32_t lsb = (u >> 16) & 1u;
    u += 0x7fffu + lsb;
    return u2f(u & 0xffff0000u);
}

/* bf16 bits -> f32 (exact widening), app/src/model/decode_attention.cu:2-4. */
float oracle_bf16_to_f32(uint16_t b) { return u2f(((uint32_t)b) << 16); }

uint16_t oracle_f32_to_bf16_bits(float x) { return (uint16_t)(f2u(oracle_bf16_round(x)) >> 16); }

/* Symmetric per-row int8 quantization, app/src/model/int8_kv_ops.rs:13-21:
 *   s = max(max|v| / 127, 1e-12)   (f32 division, then max)
 *   q = (v / s).round_ties_even().clamp(-127, 127) as i8
 * Rows of `d` elements.  Returns ORACLE_NON_FINITE on any non-finite input
 * (the reference's `ensure!` at :16); outputs are then unspecified. */
int oracle_quantize_f32(const float* x, uint64_t rows, uint32_t d, uint8_t* packed, float* scales) {
    if (d == 0) return ORACLE_BAD_GEOMETRY;
    for (uint64_t r = 0; r < rows; ++r) {
        const float* row = x + r * d;
        float m = 0.0f;
        for (uint32_t i = 0; i < d; ++i) {
            if (!isfinite(row[i])) return ORACLE_NON_FINITE;
            float a = fabsf(row[i]);
            m = a > m ? a : m;
        }
        float s = m / 127.0f;
        if (!(s >= 1e-12f)) s = 1e-12f;
        scales[r] = s;
        for (uint32_t i = 0; i < d; ++i) {
            float q = nearbyintf(row[i] / s); /* default FE_TONEAREST: ties to even */
            if (q < -127.0f) q = -127.0f;
            if (q > 127.0f) q = 127.0f;
            packed[r * d + i] = (uint8_t)(int8_t)q;
        }
    }
    return ORACLE_OK;
}

/* bf16 inputs are widened exactly to f32 first (int8_kv_ops.rs:12). */
int oracle_quantize_bf16(const uint16_t* x, uint64_t rows, uint32_t d, uint8_t* packed, float* scales) {
    float* tmp = (float*)malloc(sizeof(float) * (size_t)d);
    if (!tmp) return ORACLE_BAD_GEOMETRY;
    int rc = ORACLE_OK;
    for (uint64_t r = 0; r < rows && rc == ORACLE_OK; ++r) {
        for (uint32_t i = 0; i < d; ++i) tmp[i] = oracle_bf16_to_f32(x[r * d + i]);
        rc = oracle_quantize_f32(tmp, 1, d, packed + r * d, scales + r);
    }
    free(tmp);
    return rc;
}

/* Dequantization, app/src/model/int8_kv_ops.rs:33-36: (x as i8) as f32 * s[row].
 * round_bf16 != 0 adds the `.to_dtype(BF16)` rounding the attention path and
 * the prefill prefix apply (int8_kv_ops.rs:68,92-93; int8_cache.rs:368-369). */
void oracle_dequantize(const uint8_t* packed, const float* scales, uint64_t rows, uint32_t d,
                       float* out, int round_bf16) {
    for (uint64_t r = 0; r < rows; ++r)
        for (uint32_t i = 0; i < d; ++i) {
            float v = (float)(int8_t)packed[r * d + i] * scales[r];
            out[r * d + i] = round_bf16 ? oracle_bf16_round(v) : v;
        }
}

/* One physical head row of int8 decode attention, restating the reference's
 * scalar CPU checker loops (app/src/model/int8_kv_ops.rs:69-73 and :95-99,
 * app/src/model/int8_cache.rs:241-251), which define what pp_i8_attention
 * (int8_kv.cu:28-52) + pp_i8_merge (:53-59) must produce:
 *   history token t < len:  k_t = bf16(i8 * ks[t]), v_t = bf16(i8 * vs[t])
 *   scratch token (if sk):  k = sk, v = sv in f32, placed at index len
 *   score_t = (sum_d q_d * k_t,d) * scale        (sequential f32 sum)
 *   p_t = exp(score_t - max), z = sum p, out_d = (sum_t p_t * v_t,d) / z
 * `scale` is 0.125 in the reference (head_dim 64); the generalisation is
 * f32(1/sqrt(D)), the factor the reference's ordinary attention divides by
 * (app/src/model/batch.rs:216).  scores/p are caller scratch of len+1. */
static void attention_row(const float* q, const uint8_t* k, const uint8_t* v, const float* ks,
                          const float* vs, const float* sk, const float* sv, uint32_t len,
                          uint32_t d, float scale, float* out, float* scores) {
    uint32_t n = len + (sk ? 1u : 0u);
    float mx = -INFINITY;
    for (uint32_t t = 0; t < n; ++t) {
        float acc = 0.0f;
        if (t < len) {
            for (uint32_t i = 0; i < d; ++i) {
                float kt = oracle_bf16_round((float)(int8_t)k[(size_t)t * d + i] * ks[t]);
                acc += q[i] * kt;
            }
        } else {
            for (uint32_t i = 0; i < d; ++i) acc += q[i] * sk[i];
        }
        scores[t] = acc * scale;
        mx = scores[t] > mx ? scores[t] : mx;
    }
    float z = 0.0f;
    for (uint32_t t = 0; t < n; ++t) {
        scores[t] = expf(scores[t] - mx);
        z += scores[t];
    }
    for (uint32_t i = 0; i < d; ++i) {
        float acc = 0.0f;
        for (uint32_t t = 0; t < n; ++t) {
            float vt = t < len ? oracle_bf16_round((float)(int8_t)v[(size_t)t * d + i] * vs[t]) : sv[i];
            acc += scores[t] * vt;
        }
        out[i] = acc / z;
    }
}

/* Batched int8 decode attention over an arena laid out as the reference's
 * batch arena (app/src/model/int8_cache.rs:326-359, cache.rs:301-478):
 *   q      f32 [rows, d]                     (rows = branches * heads)
 *   k, v   u8  [rows, capacity, d]
 *   ks, vs f32 [rows, capacity]
 *   sk, sv f32 [rows, d] or NULL             (reference mode: fp32 scratch token)
 *   lengths u32 [rows / heads]               (per-branch history length)
 * With scratch (reference mode) a row attends to lengths[b] int8 tokens plus
 * the scratch token, and lengths[b] > capacity yields a NaN row, as the
 * `valid` test of int8_kv.cu:33,51 does.  Without scratch (all-int8 mode) a
 * row attends to lengths[b] tokens; 0 or > capacity yields NaN.
 * `threads` > 1 parallelises over rows with POSIX threads. */
struct attn_job {
    const float *q, *ks, *vs, *sk, *sv;
    const uint8_t *k, *v;
    const uint32_t* lengths;
    uint32_t rows, heads, d, capacity, stride, first;
    float scale;
    float* out;
};

static void* attention_worker(void* arg) {
    const struct attn_job* j = (const struct attn_job*)arg;
    int scratch = j->sk != NULL && j->sv != NULL;
    float* scores = (float*)malloc(sizeof(float) * ((size_t)j->capacity + 2));
    for (uint32_t r = j->first; r < j->rows; r += j->stride) {
        uint32_t len = j->lengths[r / j->heads];
        float* o = j->out + (size_t)r * j->d;
        int valid = scratch ? (len <= j->capacity) : (len > 0 && len <= j->capacity);
        if (!valid || !scores) {
            for (uint32_t i = 0; i < j->d; ++i) o[i] = NAN;
            continue;
        }
        size_t base = (size_t)r * j->capacity;
        attention_row(j->q + (size_t)r * j->d, j->k + base * j->d, j->v + base * j->d, j->ks + base,
                      j->vs + base, scratch ? j->sk + (size_t)r * j->d : NULL,
                      scratch ? j->sv + (size_t)r * j->d : NULL, len, j->d, j->scale, o, scores);
    }
    free(scores);
    return NULL;
}

int oracle_attention(const float* q, const uint8_t* k, const uint8_t* v, const float* ks,
                     const float* vs, const float* sk, const float* sv, const uint32_t* lengths,
                     uint32_t rows, uint32_t heads, uint32_t d, uint32_t capacity, float scale,
                     float* out, int threads) {
    if (heads == 0 || rows % heads != 0 || d == 0) return ORACLE_BAD_GEOMETRY;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if ((uint32_t)threads > rows) threads = rows ? (int)rows : 1;
    struct attn_job jobs[256];
    pthread_t tid[256];
    for (int i = 0; i < threads; ++i) {
        jobs[i] = (struct attn_job){q, ks, vs, sk, sv, k, v, lengths, rows, heads, d, capacity,
                                    (uint32_t)threads, (uint32_t)i, scale, out};
    }
    int started[256] = {0};
    for (int i = 1; i < threads; ++i)
        started[i] = pthread_create(&tid[i], NULL, attention_worker, &jobs[i]) == 0;
    attention_worker(&jobs[0]);
    for (int i = 1; i < threads; ++i) {
        if (started[i]) pthread_join(tid[i], NULL);
        else attention_worker(&jobs[i]); /* could not start a thread: run its rows here */
    }
    return ORACLE_OK;
}

/* Quantize-and-append of one new token per physical row into the arena, the
 * composition of Int8LayerCache::encoded (int8_cache.rs:293-312) and the
 * batched append LayerCache::query_batch_with_plan (cache.rs:415-459):
 *   commit:  row r's codes/scale written at token offsets[r / heads]
 *   partial: a zero code row and scale 1.0 written there instead
 * x_k, x_v f32 [rows, d].  Offsets must be < capacity. */
int oracle_quant_append(const float* x_k, const float* x_v, uint32_t rows, uint32_t heads, uint32_t d,
                        uint32_t capacity, const uint32_t* offsets, int commit, uint8_t* k_arena,
                        uint8_t* v_arena, float* ks_arena, float* vs_arena) {
    if (heads == 0 || rows % heads != 0 || d == 0) return ORACLE_BAD_GEOMETRY;
    for (uint32_t r = 0; r < rows; ++r)
        if (offsets[r / heads] >= capacity) return ORACLE_BAD_GEOMETRY;
    for (uint32_t r = 0; r < rows; ++r) {
        size_t slot = (size_t)r * capacity + offsets[r / heads];
        if (commit) {
            int rc = oracle_quantize_f32(x_k + (size_t)r * d, 1, d, k_arena + slot * d, ks_arena + slot);
            if (rc) return rc;
            rc = oracle_quantize_f32(x_v + (size_t)r * d, 1, d, v_arena + slot * d, vs_arena + slot);
            if (rc) return rc;
        } else {
            memset(k_arena + slot * d, 0, d);
            memset(v_arena + slot * d, 0, d);
            ks_arena[slot] = 1.0f;
            vs_arena[slot] = 1.0f;
        }
    }
    return ORACLE_OK;
}

int oracle_max_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}
