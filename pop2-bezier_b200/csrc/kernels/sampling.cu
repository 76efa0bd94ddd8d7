// Rényi-entropy truncated sampling with classifier-free guidance on the
// device, after the output heads: the drop-in for the reference's fused
// sampler (app/src/inference/fused_sampling.rs:69-158, kernel
// pp_renyi_sample in app/src/inference/renyi_sample.cu).
//
// Per logical row, with x the conditional and u the unconditional head:
//   v[c] = guidance 2 ? u[c] + cfg * (x[c] - u[c]) : x[c]
//   every value of the head must be finite; the legal window is [start, start + count)
//   m = max of the window, z = sum exp(v - m), za = sum exp(alpha (v - m))
//   H = log z + max(log z - log za, 0) / (alpha - 1)       (Rényi entropy of order alpha)
//   support = clamp(round(exp(clamp(H, 0, log count))), 1, count), rank = floor(U * support)
//   token = the rank-th column of the window in the order (value desc, column asc)
// Outputs [3][batch]: token_offset + column, 1 (sampled) or 0 (fallback), support;
// a row with bad arguments, a non-finite value or a non-finite entropy yields
// (token_offset + start, 0, 1) (start clamped to 0 when it lies outside the head).
//
// What must equal the reference bit for bit is the floating-point arithmetic
// of z, za, H and the support: 256 partial sums, partial t summing window
// positions t, t + 256, ... in that order; then a pairwise tree in which
// partial t absorbs partial t + s for s = 128, 64, ..., 1; the fast exp / log
// intrinsics; and no contraction (the file is built with -fmad=false
// -prec-div=true like the reference's NVRTC compile).  Everything else is
// exact and is organised for this GPU:
//   * thread t keeps window positions t + 256 k (k < 8) in registers: no
//     shared-memory copy of the window;
//   * the maximum and its first column come from one reduction of a 64-bit
//     key (order-preserving value bits above the inverted position);
//   * the tree's first three levels are evaluated by warp 0 from one shared
//     array after a single barrier (the same additions in the same order);
//   * the rank-th element is found by radix selection on the 32-bit
//     order-preserving value key (four 8-bit digits, most significant first;
//     per digit a histogram built with warp-aggregated atomics and a block
//     scan from the largest digit), then, among the values equal to the
//     selected key, the remaining rank is resolved by column order with one
//     round of ballots.  The key treats -0 and +0 as one value, as the
//     reference's comparison does.
#include "common.cuh"
#include "../host/internal.h"

namespace pp {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kPerThread = 8;  // window positions per thread: up to 2048 choices

__device__ __forceinline__ bool finite_f(float v) { return (__float_as_uint(v) & 0x7fffffffu) < 0x7f800000u; }

// Unsigned key with the order of the float values (larger value, larger key);
// -0 is mapped to +0 first.
__device__ __forceinline__ uint32_t order_key(float v) {
    uint32_t b = __float_as_uint(v);
    if ((b & 0x7fffffffu) == 0) b = 0;
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float key_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

__device__ __forceinline__ unsigned long long max_u64(unsigned long long a, unsigned long long b) {
    return a > b ? a : b;
}

struct SampleArgs {
    const float* raw;
    const float* uniforms;
    const uint32_t* bounds;
    uint32_t* out;
    uint32_t batch, choices, guidance, token_offset;
    float alpha, cfg;
};

struct Shared {
    unsigned long long best[kWarps];
    float z[kThreads], za[kThreads];
    uint32_t hist[256];
    uint32_t warp_sum[kWarps];
    uint32_t chunk_count[kPerThread][kWarps];
    uint32_t bad, stop, support, rank, digit, rank_left;
};

__device__ __forceinline__ void emit(const SampleArgs& a, uint32_t row, uint32_t token, uint32_t ok,
                                     uint32_t support) {
    a.out[row] = token;
    a.out[(uint64_t)a.batch + row] = ok;
    a.out[2ull * a.batch + row] = support;
}

// The guided value of head column c, and whether it and its inputs are finite.
__device__ __forceinline__ float head_value(const SampleArgs& a, const float* xr, uint32_t c, bool& ok) {
    const float x = xr[c];
    float v = x;
    ok = finite_f(x);
    if (a.guidance == 2) {
        const float un = xr[a.choices + c];
        ok = ok && finite_f(un);
        v = un + a.cfg * (x - un);
    }
    ok = ok && finite_f(v);
    return v;
}

// Inclusive block scan of one value per thread; returns the inclusive prefix.
__device__ __forceinline__ uint32_t block_scan(uint32_t v, Shared& sh, int lane, int warp) {
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, v, d);
        if (lane >= d) v += o;
    }
    if (lane == 31) sh.warp_sum[warp] = v;
    __syncthreads();
    uint32_t before = 0;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) before += (w < warp) ? sh.warp_sum[w] : 0u;
    return v + before;
}

__global__ void __launch_bounds__(kThreads) renyi_sample_kernel(const SampleArgs a) {
    __shared__ Shared sh;
    const uint32_t row = blockIdx.x, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const uint32_t start = a.bounds[2 * row], count = a.bounds[2 * row + 1];
    const float u = a.uniforms[row];
    {
        const uint32_t clamped = start < a.choices ? start : 0u;
        const bool bad_args = !finite_f(u) || u < 0.f || u >= 1.f || start >= a.choices || count == 0 ||
                              count > a.choices - clamped;
        if (bad_args) {  // uniform across the block: nothing else is touched
            if (tid == 0) emit(a, row, a.token_offset + clamped, 0u, 1u);
            return;
        }
    }
    const float* xr = a.raw + (uint64_t)row * a.guidance * a.choices;

    // every value of the head must be finite
    bool all_ok = true;
#pragma unroll
    for (int k = 0; k < kPerThread; ++k) {
        const uint32_t c = tid + k * kThreads;
        if (c < a.choices) {
            bool ok;
            head_value(a, xr, c, ok);
            all_ok = all_ok && ok;
        }
    }
    // the window, in registers, and its maximum with the first position holding it
    float v[kPerThread];
    uint32_t key[kPerThread];
    unsigned long long best = 0;
#pragma unroll
    for (int k = 0; k < kPerThread; ++k) {
        const uint32_t p = tid + k * kThreads;
        v[k] = 0.f;
        key[k] = 0;
        if (p < count) {
            bool ok;
            v[k] = head_value(a, xr, start + p, ok);
            key[k] = order_key(v[k]);
            best = max_u64(best, ((unsigned long long)key[k] << 32) | (0xffffffffu - p));
        }
    }
#pragma unroll
    for (int d = 16; d; d >>= 1) best = max_u64(best, __shfl_xor_sync(0xffffffffu, best, d));
    const bool any_bad = __syncthreads_or(!all_ok);
    if (any_bad) {
        if (tid == 0) emit(a, row, a.token_offset + start, 0u, 1u);
        return;
    }
    if (lane == 0) sh.best[warp] = best;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kWarps; ++w) best = max_u64(best, sh.best[w]);
    const uint32_t max_key = (uint32_t)(best >> 32);
    const uint32_t max_pos = 0xffffffffu - (uint32_t)best;
    const float m = key_value(max_key);

    // partial sums over positions tid, tid + 256, ... in that order
    float z = 0.f, za = 0.f;
#pragma unroll
    for (int k = 0; k < kPerThread; ++k) {
        if (tid + k * kThreads < count) {
            const float d = v[k] - m;
            z += __expf(d);
            za += __expf(a.alpha * d);
        }
    }
    sh.z[tid] = z;
    sh.za[tid] = za;
    __syncthreads();
    if (warp == 0) {
        // levels 128, 64, 32 of the tree for partial `lane`, then 16 .. 1 across the warp
        float q[8], qa[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            q[j] = sh.z[lane + 32 * j];
            qa[j] = sh.za[lane + 32 * j];
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {  // + 128
            q[j] = q[j] + q[j + 4];
            qa[j] = qa[j] + qa[j + 4];
        }
#pragma unroll
        for (int j = 0; j < 2; ++j) {  // + 64
            q[j] = q[j] + q[j + 2];
            qa[j] = qa[j] + qa[j + 2];
        }
        z = q[0] + q[1];  // + 32
        za = qa[0] + qa[1];
#pragma unroll
        for (int d = 16; d; d >>= 1) {
            z += __shfl_down_sync(0xffffffffu, z, d);
            za += __shfl_down_sync(0xffffffffu, za, d);
        }
        if (lane == 0) {
            const float lz = __logf(z), lza = __logf(za);
            float corr = lz - lza;
            if (corr < 0.f) corr = 0.f;
            float h = lz + corr / (a.alpha - 1.f);
            const bool fail = !finite_f(lz) || !finite_f(lza) || !finite_f(h);
            uint32_t support = 1, rank = 0;
            if (!fail) {
                const float h_max = __logf((float)count);
                if (h < 0.f) h = 0.f;
                if (h > h_max) h = h_max;
                support = (uint32_t)(__expf(h) + 0.5f);
                if (support < 1) support = 1;
                if (support > count) support = count;
                rank = (uint32_t)(u * (float)support);
                if (rank >= support) rank = support - 1;
            }
            if (fail) emit(a, row, a.token_offset + start, 0u, 1u);
            else if (rank == 0) emit(a, row, a.token_offset + start + max_pos, 1u, support);
            sh.stop = fail || rank == 0;
            sh.support = support;
            sh.rank = rank;
        }
    }
    __syncthreads();
    if (sh.stop) return;
    const uint32_t support = sh.support;

    // radix selection of the key of the rank-th largest value
    uint32_t prefix = 0, mask = 0, left = sh.rank;
#pragma unroll 1
    for (int shift = 24; shift >= 0; shift -= 8) {
        sh.hist[tid] = 0;
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kPerThread; ++k) {
            const bool mine = tid + k * kThreads < count && (key[k] & mask) == prefix;
            const uint32_t dig = mine ? (key[k] >> shift) & 0xffu : 0x100u;
            const uint32_t peers = __match_any_sync(0xffffffffu, dig);
            if (mine && lane == __ffs(peers) - 1) atomicAdd(&sh.hist[dig], (uint32_t)__popc(peers));
        }
        __syncthreads();
        // thread t looks at digit 255 - t: counts from the largest digit down
        const uint32_t h = sh.hist[255 - tid];
        const uint32_t incl = block_scan(h, sh, lane, warp);
        if (incl - h <= left && left < incl) {
            sh.digit = 255 - tid;
            sh.rank_left = left - (incl - h);
        }
        __syncthreads();
        prefix |= sh.digit << shift;
        mask |= 0xffu << shift;
        left = sh.rank_left;
        __syncthreads();  // hist and digit are rewritten by the next pass
    }

    // among the values with that key, the `left`-th by column
    uint32_t ball[kPerThread];
#pragma unroll
    for (int k = 0; k < kPerThread; ++k) {
        ball[k] = __ballot_sync(0xffffffffu, tid + k * kThreads < count && key[k] == prefix);
        if (lane == 0) sh.chunk_count[k][warp] = __popc(ball[k]);
    }
    __syncthreads();
    uint32_t before = 0;
    const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
    for (int k = 0; k < kPerThread; ++k) {
        uint32_t here = before;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) here += (w < warp) ? sh.chunk_count[k][w] : 0u;
        if ((ball[k] >> lane) & 1u) {
            if (here + __popc(ball[k] & lt) == left)
                emit(a, row, a.token_offset + start + tid + k * kThreads, 1u, support);
        }
#pragma unroll
        for (int w = 0; w < kWarps; ++w) before += sh.chunk_count[k][w];
    }
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
    renyi_sample_kernel<<<batch, kThreads, 0, stream>>>(a);
    return cudaGetLastError();
}

}  // namespace pp
