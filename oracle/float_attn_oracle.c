/*
 * float_attn_oracle.c -- CPU restatement of the reference's float-KV fused
 * decode attention (kernels pp_attention_f32 / pp_attention_bf16 /
 * pp_attention_merge, app/src/model/decode_attention.cu:7-59, launched by
 * app/src/model/fused_attention.rs:8-83).
 *
 * TEST INFRASTRUCTURE ONLY: the checker for pp_b200_decode_attention_float.
 * Only tests/, the smoke() entry point and bench.py's cpu_baseline /
 * reference arm may load it; the product library never links or calls it.
 *
 * Parity pinning: tests/golden/make_float_golden.py ran the reference's own
 * kernels (compiled from decode_attention.cu into oracle/_ref/ by
 * oracle/Makefile) on a B200 with the launch geometry of fused_attention.rs;
 * tests/golden/ref_float_attn.npz holds their outputs and
 * tests/test_float_attention.py checks this file against them.  The
 * restatement keeps the kernel's summation orders (lane products, the
 * shuffle tree, the 128-thread block trees, the sequential p.V sums); its
 * exp is the C library's rather than CUDA's, so agreement is to a few f32
 * ulps, not bit for bit.
 *
 * Compile with -ffp-contract=off: the reference is compiled with fmad=false,
 * so every product and sum rounds separately.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>

#define ORACLE_OK 0
#define ORACLE_BAD_GEOMETRY 2

#define BLOCK 128 /* threads of one reference CTA (fused_attention.rs:62) */

static inline float ld_kv(const void* p, int bf16, size_t i) {
    if (bf16) {
        uint32_t u = ((uint32_t)((const uint16_t*)p)[i]) << 16; /* bf16_load, decode_attention.cu:2-4 */
        float x;
        memcpy(&x, &u, 4);
        return x;
    }
    return ((const float*)p)[i];
}

/* One (row, part) CTA of attention_part (decode_attention.cu:7-46): writes
 * m, z and the unnormalised values (or the normalised output when splits == 1). */
static void attention_part(const float* q, const void* k, const void* v, int bf16, uint32_t length, int valid,
                           uint32_t d, uint32_t split, uint32_t part, uint32_t splits, float scale,
                           float* scores, float* m_out, float* z_out, float* value_out) {
    const uint32_t begin = part * split;
    const uint32_t end = valid ? (begin + split < length ? begin + split : length) : 0u;
    /* scores: lane l holds sum_e q[l + 32e] * k[l + 32e], then the shuffle-down tree (:19-26) */
    for (uint32_t t = 0; t < split; ++t) {
        const uint32_t token = begin + t;
        if (token >= end) {
            scores[t] = -FLT_MAX;
            continue;
        }
        float lane[32];
        for (uint32_t l = 0; l < 32; ++l) {
            float dot = q[l] * ld_kv(k, bf16, (size_t)token * d + l);
            for (uint32_t e = 1; e < d / 32; ++e) dot += q[l + 32 * e] * ld_kv(k, bf16, (size_t)token * d + l + 32 * e);
            lane[l] = dot;
        }
        for (uint32_t s = 16; s > 0; s >>= 1)
            for (uint32_t l = 0; l < s; ++l) lane[l] += lane[l + s];
        scores[t] = lane[0] * scale;
    }
    /* block max (:29-32): order-free */
    float m = -FLT_MAX;
    for (uint32_t t = 0; t < split; ++t) m = fmaxf(m, scores[t]);
    /* exp and the block sum: per-thread strided sums, then the tree (:33-36) */
    float part_z[BLOCK];
    for (uint32_t tid = 0; tid < BLOCK; ++tid) part_z[tid] = 0.f;
    for (uint32_t t = 0; t < split; ++t) {
        const float e = (begin + t < end) ? expf(scores[t] - m) : 0.f;
        scores[t] = e;
        part_z[t % BLOCK] += e;
    }
    for (uint32_t s = BLOCK / 2; s > 0; s >>= 1)
        for (uint32_t tid = 0; tid < s; ++tid) part_z[tid] += part_z[tid + s];
    const float z = part_z[0];
    /* p.V in token order per channel (:40-44) */
    for (uint32_t c = 0; c < d; ++c) {
        float value = 0.f;
        for (uint32_t t = begin; t < end; ++t) value += scores[t - begin] * ld_kv(v, bf16, (size_t)t * d + c);
        if (splits == 1) value_out[c] = (valid && z > 0.f) ? value / z : NAN;
        else value_out[c] = valid ? value : NAN;
    }
    *m_out = m;
    *z_out = z;
}

struct float_job {
    const float* q;
    const void* k;
    const void* v;
    const uint32_t* lengths;
    uint64_t qs, ks, vs;
    uint32_t rows, heads, d, size, split, splits, bf16, stride, first;
    float scale;
    float* out;
};

static void* float_worker(void* arg) {
    const struct float_job* j = (const struct float_job*)arg;
    float* scores = (float*)malloc(sizeof(float) * j->split);
    float* parts = (float*)malloc(sizeof(float) * (size_t)j->splits * (j->d + 2));
    if (!scores || !parts) {
        free(scores);
        free(parts);
        return (void*)1;
    }
    for (uint32_t h = j->first; h < j->rows; h += j->stride) {
        const uint32_t length = j->lengths ? j->lengths[h / j->heads] : j->size;
        const int valid = length > 0 && length <= j->size;
        float* o = j->out + (size_t)h * j->d;
        const float* qh = j->q + (size_t)h * j->qs;
        const char* kh = (const char*)j->k + (size_t)h * j->ks * (j->bf16 ? 2 : 4);
        const char* vh = (const char*)j->v + (size_t)h * j->vs * (j->bf16 ? 2 : 4);
        if (j->splits == 1) {
            float m, z;
            attention_part(qh, kh, vh, (int)j->bf16, length, valid, j->d, j->split, 0, 1, j->scale, scores, &m, &z, o);
            continue;
        }
        for (uint32_t p = 0; p < j->splits; ++p) {
            float* b = parts + (size_t)p * (j->d + 2);
            attention_part(qh, kh, vh, (int)j->bf16, length, valid, j->d, j->split, p, j->splits, j->scale, scores,
                           &b[0], &b[1], b + 2);
        }
        /* pp_attention_merge (:49-59) */
        float m = -FLT_MAX;
        for (uint32_t p = 0; p < j->splits; ++p) m = fmaxf(m, parts[(size_t)p * (j->d + 2)]);
        for (uint32_t c = 0; c < j->d; ++c) {
            float z = 0.f, value = 0.f;
            for (uint32_t p = 0; p < j->splits; ++p) {
                const float* b = parts + (size_t)p * (j->d + 2);
                const float w = expf(b[0] - m);
                z += w * b[1];
                value += w * b[2 + c];
            }
            o[c] = z > 0.f ? value / z : NAN;
        }
    }
    free(scores);
    free(parts);
    return NULL;
}

/* The whole CustomOp (fused_attention.rs:8-33 + :46-83): q f32 rows of stride
 * qs; k, v (f32, or bf16 bits when bf16 != 0) [rows, size, d] with row
 * strides ks, vs elements and token stride d; lengths u32 [rows/heads] or
 * NULL (every row attends to all `size` tokens).  split_tokens 0 keeps one
 * part per row, otherwise parts of clamp(split_tokens, 32, 1024) tokens. */
int oracle_float_attention(const float* q, uint64_t qs, const void* k, uint64_t ks, const void* v, uint64_t vs,
                           int bf16, const uint32_t* lengths, uint32_t rows, uint32_t heads, uint32_t d,
                           uint32_t size, uint32_t split_tokens, float scale, float* out, int threads) {
    if (heads == 0 || rows == 0 || rows % heads != 0 || size == 0 || d == 0 || d % 32 != 0) return ORACLE_BAD_GEOMETRY;
    uint32_t split = split_tokens == 0 ? size : (split_tokens < 32 ? 32 : split_tokens > 1024 ? 1024 : split_tokens);
    const uint32_t splits = (size + split - 1) / split;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if ((uint32_t)threads > rows) threads = (int)rows;
    struct float_job jobs[256];
    pthread_t tid[256];
    int started[256] = {0};
    for (int i = 0; i < threads; ++i)
        jobs[i] = (struct float_job){q, k, v, lengths, qs, ks, vs, rows, heads, d, size, split, splits,
                                     (uint32_t)(bf16 != 0), (uint32_t)threads, (uint32_t)i, scale, out};
    for (int i = 1; i < threads; ++i) started[i] = pthread_create(&tid[i], NULL, float_worker, &jobs[i]) == 0;
    int bad = float_worker(&jobs[0]) != NULL;
    for (int i = 1; i < threads; ++i) {
        void* r = NULL;
        if (started[i]) pthread_join(tid[i], &r);
        else r = float_worker(&jobs[i]);
        bad |= r != NULL;
    }
    return bad ? ORACLE_BAD_GEOMETRY : ORACLE_OK;
}
