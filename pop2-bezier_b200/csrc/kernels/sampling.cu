// Rényi-entropy truncated sampling with classifier-free guidance, on the
// device after the output heads: replaces the reference's fused sampler
// (app/src/inference/fused_sampling.rs, kernel pp_renyi_sample in
// renyi_sample.cu).  Per logical row r:
//   value[c] = guidance 2 ? u[c] + cfg * (x[c] - u[c]) : x[c]   (x: conditional row, u: unconditional)
//   every value of the head must be finite; the legal window is [start, start + count)
//   m = max over the window (ties: lower column), z = sum exp(v - m), za = sum exp(alpha (v - m))
//   H = log z + max(log z - log za, 0) / (alpha - 1)      (Rényi entropy of order alpha)
//   support = clamp(round(exp(clamp(H, 0, log count))), 1, count), rank = floor(U * support)
//   token = the rank-th column of the window by (value desc, column asc)
// Outputs [3][batch]: token_offset + column, ok (1) / fallback (0), support;
// an invalid row yields (token_offset + start, 0, 1).
//
// Equal results need equal arithmetic: one 256-thread block per row as in the
// reference launch (fused_sampling.rs:151-158), per-thread sums over columns
// tid, tid + 256, ..., the same pairwise tree (here shared memory down to one
// warp, then shuffles with the same pairing), the same fast exp/log
// intrinsics, and the file is built with -fmad=false -prec-div=true like the
// reference's NVRTC compile.  The rank-th element is found with the same
// total order, so any exact selection gives the reference's token; a bitonic
// sort of the window in shared memory is used.
#include "common.cuh"
#include "../host/internal.h"

namespace pp {
namespace {

constexpr int kSampleThreads = 256;

__device__ __forceinline__ bool finite_f(float v) { return (__float_as_uint(v) & 0x7fffffffu) < 0x7f800000u; }

// (a, ai) comes before (b, bi): larger value first, then lower column
__device__ __forceinline__ bool ahead(float a, uint32_t ai, float b, uint32_t bi) {
    return a > b || (a == b && ai < bi);
}

struct SampleArgs {
    const float* raw;
    const float* uniforms;
    const uint32_t* bounds;
    uint32_t* out;
    uint32_t batch, choices, guidance, token_offset, padded;
    float alpha, cfg;
};

__device__ __forceinline__ void write_row(const SampleArgs& a, uint32_t row, uint32_t token, uint32_t ok,
                                          uint32_t support) {
    a.out[row] = token;
    a.out[(uint64_t)a.batch + row] = ok;
    a.out[2ull * a.batch + row] = support;
}

__global__ void __launch_bounds__(kSampleThreads) renyi_kernel(const SampleArgs a) {
    extern __shared__ unsigned char dyn[];
    float* vals = reinterpret_cast<float*>(dyn);
    uint32_t* cols = reinterpret_cast<uint32_t*>(vals + a.padded);
    __shared__ float red_v[kSampleThreads];
    __shared__ uint32_t red_i[kSampleThreads];
    __shared__ float red_w[kSampleThreads];
    __shared__ uint32_t s_bad, s_start, s_count, s_stop, s_support, s_rank;
    const uint32_t row = blockIdx.x, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    if (tid == 0) {
        const uint32_t start = a.bounds[2 * row], count = a.bounds[2 * row + 1];
        const float u = a.uniforms[row];
        const uint32_t clamped = start < a.choices ? start : 0u;
        const bool bad = !finite_f(u) || u < 0.f || u >= 1.f || start >= a.choices || count == 0 ||
                         count > a.choices - clamped;
        if (bad) write_row(a, row, a.token_offset + clamped, 0u, 1u);
        s_start = start;
        s_count = count;
        s_stop = bad;
    }
    __syncthreads();
    if (s_stop) return;
    const uint32_t start = s_start, count = s_count;
    uint32_t width = 1;
    while (width < count) width <<= 1;

    // pass over the whole head: finiteness, the legal window, its arg-max
    float best = -INFINITY;
    uint32_t best_col = 0xffffffffu, bad = 0;
    const float* xr = a.raw + (uint64_t)row * a.guidance * a.choices;
    for (uint32_t c = tid; c < a.choices; c += kSampleThreads) {
        const float x = xr[c];
        float v = x;
        bool ok = finite_f(x);
        if (a.guidance == 2) {
            const float un = xr[a.choices + c];
            ok = ok && finite_f(un);
            v = un + a.cfg * (x - un);
        }
        ok = ok && finite_f(v);
        bad |= !ok;
        if (!ok) v = 0.f;
        if (c >= start && c - start < count) {
            vals[c - start] = v;
            cols[c - start] = c;
            if (ahead(v, c, best, best_col)) {
                best = v;
                best_col = c;
            }
        }
    }
    for (uint32_t c = count + tid; c < width; c += kSampleThreads) {
        vals[c] = -INFINITY;
        cols[c] = 0xffffffffu;
    }
    // block arg-max and OR, pairing (t, t + step) for step = 128 .. 1
    red_v[tid] = best;
    red_i[tid] = best_col;
    red_w[tid] = __uint_as_float(bad);
    __syncthreads();
    for (uint32_t step = kSampleThreads / 2; step >= 32; step >>= 1) {
        if (tid < step) {
            if (ahead(red_v[tid + step], red_i[tid + step], red_v[tid], red_i[tid])) {
                red_v[tid] = red_v[tid + step];
                red_i[tid] = red_i[tid + step];
            }
            red_w[tid] = __uint_as_float(__float_as_uint(red_w[tid]) | __float_as_uint(red_w[tid + step]));
        }
        __syncthreads();
    }
    if (warp == 0) {
        float v = red_v[tid];
        uint32_t i = red_i[tid], b = __float_as_uint(red_w[tid]);
        for (int step = 16; step; step >>= 1) {
            const float ov = __shfl_down_sync(0xffffffffu, v, step);
            const uint32_t oi = __shfl_down_sync(0xffffffffu, i, step);
            b |= __shfl_down_sync(0xffffffffu, b, step);
            if (ahead(ov, oi, v, i)) {
                v = ov;
                i = oi;
            }
        }
        if (lane == 0) {
            red_v[0] = v;
            red_i[0] = i;
            s_bad = b;
            if (b) write_row(a, row, a.token_offset + start, 0u, 1u);
        }
    }
    __syncthreads();
    if (s_bad) return;
    const float m = red_v[0];
    const uint32_t m_col = red_i[0];

    // z and z_alpha: per-thread sums over columns tid, tid + 256, ..., then the tree
    float z = 0.f, za = 0.f;
    for (uint32_t c = tid; c < count; c += kSampleThreads) {
        const float d = vals[c] - m;
        z += __expf(d);
        za += __expf(a.alpha * d);
    }
    __syncthreads();  // red_v/red_i are reused below
    red_v[tid] = z;
    red_w[tid] = za;
    __syncthreads();
    for (uint32_t step = kSampleThreads / 2; step >= 32; step >>= 1) {
        if (tid < step) {
            red_v[tid] += red_v[tid + step];
            red_w[tid] += red_w[tid + step];
        }
        __syncthreads();
    }
    if (warp == 0) {
        z = red_v[tid];
        za = red_w[tid];
        for (int step = 16; step; step >>= 1) {
            z += __shfl_down_sync(0xffffffffu, z, step);
            za += __shfl_down_sync(0xffffffffu, za, step);
        }
        if (lane == 0) {
            const float lz = __logf(z), lza = __logf(za);
            float corr = lz - lza;
            if (corr < 0.f) corr = 0.f;
            float h = lz + corr / (a.alpha - 1.f);
            const bool fail = !finite_f(lz) || !finite_f(lza) || !finite_f(h);
            s_stop = fail;
            if (fail) {
                write_row(a, row, a.token_offset + start, 0u, 1u);
            } else {
                const float h_max = __logf((float)count);
                if (h < 0.f) h = 0.f;
                if (h > h_max) h = h_max;
                uint32_t support = (uint32_t)(__expf(h) + 0.5f);
                if (support < 1) support = 1;
                if (support > count) support = count;
                uint32_t rank = (uint32_t)(a.uniforms[row] * (float)support);
                if (rank >= support) rank = support - 1;
                s_support = support;
                s_rank = rank;
                if (rank == 0) write_row(a, row, a.token_offset + m_col, 1u, support);
            }
        }
    }
    __syncthreads();
    if (s_stop || s_rank == 0) return;

    // the rank-th element by (value desc, column asc): bitonic sort of the window
    for (uint32_t stage = 2; stage <= width; stage <<= 1) {
        for (uint32_t dist = stage >> 1; dist; dist >>= 1) {
            for (uint32_t c = tid; c < width; c += kSampleThreads) {
                const uint32_t o = c ^ dist;
                if (o > c) {
                    const bool down = (c & stage) == 0;
                    const bool swap = down ? ahead(vals[o], cols[o], vals[c], cols[c])
                                           : ahead(vals[c], cols[c], vals[o], cols[o]);
                    if (swap) {
                        const float tv = vals[c];
                        vals[c] = vals[o];
                        vals[o] = tv;
                        const uint32_t ti = cols[c];
                        cols[c] = cols[o];
                        cols[o] = ti;
                    }
                }
            }
            __syncthreads();
        }
    }
    if (tid == 0) write_row(a, row, a.token_offset + cols[s_rank], 1u, s_support);
}

}  // namespace

cudaError_t launch_renyi_sample(const float* raw, const float* uniforms, const uint32_t* bounds, uint32_t* out,
                                uint32_t batch, uint32_t choices, uint32_t guidance, float alpha, float cfg,
                                uint32_t token_offset, cudaStream_t stream) {
    SampleArgs a{};
    a.raw = raw;
    a.uniforms = uniforms;
    a.bounds = bounds;
    a.out = out;
    a.batch = batch;
    a.choices = choices;
    a.guidance = guidance;
    a.token_offset = token_offset;
    a.alpha = alpha;
    a.cfg = cfg;
    uint32_t p = 1;
    while (p < choices) p <<= 1;
    a.padded = p;
    renyi_kernel<<<batch, kSampleThreads, (size_t)p * 8, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace pp
