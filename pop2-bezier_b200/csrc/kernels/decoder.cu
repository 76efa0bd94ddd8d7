// Decoder-step kernels around the int8 KV path: q/k RMSNorm + interleaved
// RoPE over the QKV projection (alone, or fused with the int8 quantize-and-
// append of K and V and the f32 scratch the attention reads), SwiGLU, and
// RMSNorm with an optional residual add.
//
// Rounding follows the reference's own device versions of these operations
// (app/src/model/graph_ops.cu): every intermediate that the reference rounds
// to the model dtype is rounded here at the same point, and the file is
// compiled with -fmad=false -prec-div=true -prec-sqrt=true, the options of
// the reference's NVRTC build, so products and sums are not contracted.
#include "common.cuh"
#include "quant_row.cuh"
#include "../host/internal.h"

namespace pp {
namespace {



// Element access in the model dtype: bf16 (BF = true) or f32.
template <bool BF>
__device__ __forceinline__ float rd(const void* p, uint64_t i) {
    if constexpr (BF) return __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(p)[i] << 16);
    else return reinterpret_cast<const float*>(p)[i];
}

// Round to nearest even on the upper 16 bits; a NaN stays a quiet NaN with
// its sign and top payload bits (the rounding of graph_ops.cu:5-9).
__device__ __forceinline__ uint16_t bf16_bits(float x) {
    const uint32_t b = __float_as_uint(x);
    if ((b & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((b >> 16) | 0x40u);
    return (uint16_t)((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}

template <bool BF>
__device__ __forceinline__ float rnd(float x) {
    if constexpr (BF) return __uint_as_float((uint32_t)bf16_bits(x) << 16);
    else return x;
}

template <bool BF>
__device__ __forceinline__ void wr(void* p, uint64_t i, float x) {
    if constexpr (BF) reinterpret_cast<uint16_t*>(p)[i] = bf16_bits(x);
    else reinterpret_cast<float*>(p)[i] = x;
}

constexpr int kQkvWarps = 4;  // (row, head) items per CTA of the QKV kernels

struct QkvArgs {
    const void* qkv;        // [rows, 3 * heads * D] model dtype: q | k | v
    const void* params;     // [q_norm D | k_norm D | cos max_ctx*D/2 | sin max_ctx*D/2]
    const uint32_t* positions;  // RoPE position per row
    uint32_t rows, heads, max_context;
    // plain output: planes [3][rows*heads][D] (q, k, v), model dtype
    void* out;
    // fused output: q [rows*heads][D] model dtype, scratch k/v f32, int8 append
    void* q_out;
    float* sk;
    float* sv;
    uint8_t* k_arena;
    uint8_t* v_arena;
    float* ks_arena;
    float* vs_arena;
    const uint32_t* offsets;  // arena slot per row
    uint32_t capacity, commit;
    uint32_t* status;
};

// One warp per (row, head); lane t holds channels t + 32 e, e < D/32.  q and
// k are RMS-normalised (sum of squares in channel order per lane, then a
// shuffle-down tree, as graph_ops.cu:41-45), scaled by their norm weights and
// rounded; RoPE pairs channels (2i, 2i+1) with cos/sin row `position`
// (graph_ops.cu:49-58).  APPEND quantizes the rotated k and the v row into
// the arena at offsets[row] and writes q and the f32 scratch instead of the
// three planes.
template <int D, bool BF, bool APPEND>
__global__ void __launch_bounds__(32 * kQkvWarps) qkv_rope_kernel(const QkvArgs a) {
    constexpr int E = D / 32;
    __shared__ float sq[kQkvWarps][D], skk[kQkvWarps][D], svv[kQkvWarps][D];
    // launched as a programmatic dependent: wait for the kernel before (the QKV
    // projection), then let a dependent attention launch start and stream
    // history (which this kernel does not write); it waits for this kernel
    // before reading q/k/v
    pdl_wait_primary();
    pdl_launch_dependents();
    const int t = threadIdx.x & 31, w = threadIdx.x >> 5;
    const uint32_t headrow = blockIdx.x * kQkvWarps + w;
    if (headrow >= a.rows * a.heads) return;
    const uint32_t row = headrow / a.heads, head = headrow % a.heads, width = a.heads * D;
    const uint64_t base = (uint64_t)row * 3 * width + (uint64_t)head * D;
    float qv[E], kv[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        qv[e] = rd<BF>(a.qkv, base + t + 32 * e);
        kv[e] = rd<BF>(a.qkv, base + width + t + 32 * e);
    }
    float qs = qv[0] * qv[0], ks = kv[0] * kv[0];
#pragma unroll
    for (int e = 1; e < E; ++e) {
        qs = qs + qv[e] * qv[e];
        ks = ks + kv[e] * kv[e];
    }
#pragma unroll
    for (int delta = 16; delta; delta >>= 1) {
        qs += __shfl_down_sync(0xffffffffu, qs, delta);
        ks += __shfl_down_sync(0xffffffffu, ks, delta);
    }
    const float qi = rsqrtf(__shfl_sync(0xffffffffu, qs, 0) / (float)D + 1.e-6f);
    const float ki = rsqrtf(__shfl_sync(0xffffffffu, ks, 0) / (float)D + 1.e-6f);
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int c = t + 32 * e;
        sq[w][c] = rnd<BF>(qv[e] * qi * rd<BF>(a.params, c));
        skk[w][c] = rnd<BF>(kv[e] * ki * rd<BF>(a.params, D + c));
    }
    __syncwarp();
    const uint32_t pos = a.positions[row];
    if (pos >= a.max_context) {
        if (t == 0 && a.status) atomicOr(a.status, PP_DEV_POSITION_RANGE);
        return;
    }
    const uint64_t cos0 = 2ull * D + (uint64_t)pos * (D / 2);
    const uint64_t sin0 = 2ull * D + (uint64_t)a.max_context * (D / 2) + (uint64_t)pos * (D / 2);
    float qo[E], ko[E], vo[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
        const int c = t + 32 * e, pair = c >> 1;
        const float co = rd<BF>(a.params, cos0 + pair), si = rd<BF>(a.params, sin0 + pair);
        if (c & 1) {
            qo[e] = rnd<BF>(rnd<BF>(sq[w][c - 1] * si) + rnd<BF>(sq[w][c] * co));
            ko[e] = rnd<BF>(rnd<BF>(skk[w][c - 1] * si) + rnd<BF>(skk[w][c] * co));
        } else {
            qo[e] = rnd<BF>(rnd<BF>(sq[w][c] * co) - rnd<BF>(sq[w][c + 1] * si));
            ko[e] = rnd<BF>(rnd<BF>(skk[w][c] * co) - rnd<BF>(skk[w][c + 1] * si));
        }
        vo[e] = rd<BF>(a.qkv, base + 2ull * width + c);
    }
    const uint64_t at = (uint64_t)headrow * D;
    if constexpr (!APPEND) {
        const uint64_t plane = (uint64_t)a.rows * width;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const int c = t + 32 * e;
            wr<BF>(a.out, at + c, qo[e]);
            wr<BF>(a.out, plane + at + c, ko[e]);
            wr<BF>(a.out, 2 * plane + at + c, vo[e]);
        }
    } else {
        __syncwarp();
#pragma unroll
        for (int e = 0; e < E; ++e) {
            const int c = t + 32 * e;
            wr<BF>(a.q_out, at + c, qo[e]);
            a.sk[at + c] = ko[e];
            a.sv[at + c] = vo[e];
            skk[w][c] = ko[e];
            svv[w][c] = vo[e];
        }
        __syncwarp();
        const uint32_t off = a.offsets[row];
        if (off >= a.capacity) {
            if (t == 0 && a.status) atomicOr(a.status, PP_DEV_OFFSET_RANGE);
            return;
        }
        const uint64_t slot = (uint64_t)headrow * a.capacity + off;
        if (a.commit) {
            // lane t quantizes elements [t*E, t*E + E) of each row
            float kr[E], vr[E];
#pragma unroll
            for (int e = 0; e < E; ++e) {
                kr[e] = skk[w][t * E + e];
                vr[e] = svv[w][t * E + e];
            }
            const bool okk = quantize_vals_warp<E>(kr, a.k_arena + slot * D, a.ks_arena + slot, t);
            const bool okv = quantize_vals_warp<E>(vr, a.v_arena + slot * D, a.vs_arena + slot, t);
            if (!(okk && okv) && t == 0 && a.status) atomicOr(a.status, PP_DEV_NONFINITE_INPUT);
        } else {
            // partial query: zero placeholder codes and unit scale (int8_cache.rs:305-310)
            if constexpr (E == 4) {
                *reinterpret_cast<uint32_t*>(a.k_arena + slot * D + t * 4) = 0u;
                *reinterpret_cast<uint32_t*>(a.v_arena + slot * D + t * 4) = 0u;
            } else {
                *reinterpret_cast<uint16_t*>(a.k_arena + slot * D + t * 2) = 0u;
                *reinterpret_cast<uint16_t*>(a.v_arena + slot * D + t * 2) = 0u;
            }
            if (t == 0) {
                a.ks_arena[slot] = 1.0f;
                a.vs_arena[slot] = 1.0f;
            }
        }
    }
}

// SwiGLU over [rows, 2*hidden] (gate | up) -> [rows, hidden], with the
// reference's rounding of exp, the sum and the quotient (graph_ops.cu:60-74).
template <bool BF>
__global__ void __launch_bounds__(256) swiglu_kernel(const void* in, void* out, uint64_t rows, uint32_t hidden) {
    // launched as a programmatic dependent: wait for the kernel before, then a
    // dependent decode-row GEMM may start streaming its weights; it waits for
    // this kernel before reading the activations
    pdl_wait_primary();
    pdl_launch_dependents();
    const uint64_t n = rows * hidden, stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t row = i / hidden, c = i % hidden;
        const float gate = rd<BF>(in, row * hidden * 2 + c);
        const float up = rd<BF>(in, row * hidden * 2 + hidden + c);
        const float exponential = rnd<BF>(expf(-gate));
        const float denominator = rnd<BF>(1.f + exponential);
        const float silu = rnd<BF>(gate / denominator);
        wr<BF>(out, i, rnd<BF>(silu * up));
    }
}

// RMSNorm of one row per CTA: optionally x <- round(x + residual) (stored to
// x_sum, which may be x itself), then out = round(x * rsqrt(mean(x^2) + eps)
// * weight).  The sum of squares is in f32: per thread over its strided
// elements, then a shuffle tree and a sum over the warps.
template <bool BF>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const void* x, const void* residual, void* x_sum,
                                                      const void* weight, void* out, uint32_t width, float eps) {
    pdl_wait_primary();  // as swiglu_kernel
    pdl_launch_dependents();
    __shared__ float part[8];
    const uint64_t base = (uint64_t)blockIdx.x * width;
    float ss = 0.f;
    for (uint32_t c = threadIdx.x; c < width; c += blockDim.x) {
        float v = rd<BF>(x, base + c);
        if (residual) {
            v = rnd<BF>(v + rd<BF>(residual, base + c));
            if (x_sum) wr<BF>(x_sum, base + c, v);
        }
        ss = ss + v * v;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    const int nw = blockDim.x >> 5;
    for (int i = 0; i < nw; ++i) tot = tot + part[i];
    const float scale = rsqrtf(tot / (float)width + eps);
    for (uint32_t c = threadIdx.x; c < width; c += blockDim.x) {
        // x_sum may alias x: this thread wrote element c of it above
        float v;
        if (!residual) v = rd<BF>(x, base + c);
        else if (x_sum) v = rd<BF>(x_sum, base + c);
        else v = rnd<BF>(rd<BF>(x, base + c) + rd<BF>(residual, base + c));
        wr<BF>(out, base + c, v * scale * rd<BF>(weight, c));
    }
}

// The same with 8 consecutive elements per thread held in registers (one
// pass over memory, 16-byte accesses): width = 8 * blockDim.x, 16-byte aligned
// rows.  Sum of squares per thread in element order, shuffle tree, then warps.
template <bool BF>
__device__ __forceinline__ void load8(const void* p, uint64_t i, float (&v)[8]) {
    if constexpr (BF) {
        const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p) + i);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            v[2 * k] = __uint_as_float(w[k] << 16);
            v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
        }
    } else {
        const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
        const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    }
}

template <bool BF>
__device__ __forceinline__ void store8(void* p, uint64_t i, const float (&v)[8]) {
    if constexpr (BF) {
        uint4 u;
        u.x = (uint32_t)bf16_bits(v[0]) | ((uint32_t)bf16_bits(v[1]) << 16);
        u.y = (uint32_t)bf16_bits(v[2]) | ((uint32_t)bf16_bits(v[3]) << 16);
        u.z = (uint32_t)bf16_bits(v[4]) | ((uint32_t)bf16_bits(v[5]) << 16);
        u.w = (uint32_t)bf16_bits(v[6]) | ((uint32_t)bf16_bits(v[7]) << 16);
        *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(p) + i) = u;
    } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i) = make_float4(v[0], v[1], v[2], v[3]);
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
}

template <bool BF>
__global__ void __launch_bounds__(1024) rmsnorm_vec_kernel(const void* x, const void* residual, void* x_sum,
                                                           const void* weight, void* out, uint32_t width, float eps) {
    pdl_wait_primary();  // as swiglu_kernel
    pdl_launch_dependents();
    __shared__ float part[32];
    const uint64_t i = (uint64_t)blockIdx.x * width + threadIdx.x * 8u;
    float v[8];
    load8<BF>(x, i, v);
    if (residual) {
        float r[8];
        load8<BF>(residual, i, r);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = rnd<BF>(v[k] + r[k]);
        if (x_sum) store8<BF>(x_sum, i, v);
    }
    float ss = v[0] * v[0];
#pragma unroll
    for (int k = 1; k < 8; ++k) ss = ss + v[k] * v[k];
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    const int nw = blockDim.x >> 5;
    for (int k = 0; k < nw; ++k) tot = tot + part[k];
    const float scale = rsqrtf(tot / (float)width + eps);
    float wv[8];
    load8<BF>(weight, threadIdx.x * 8u, wv);
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = v[k] * scale * wv[k];
    store8<BF>(out, i, v);
}

template <int D, bool BF, bool APPEND>
cudaError_t launch_qkv_t(const QkvArgs& a, cudaStream_t stream) {
    const uint64_t items = (uint64_t)a.rows * a.heads;
    const uint32_t blocks = (uint32_t)((items + kQkvWarps - 1) / kQkvWarps);
    return launch_pdl(qkv_rope_kernel<D, BF, APPEND>, dim3(blocks), dim3(32 * kQkvWarps), stream, a);
}

template <bool APPEND>
cudaError_t launch_qkv(const QkvArgs& a, uint32_t head_dim, bool bf, cudaStream_t stream) {
    if (head_dim == 128)
        return bf ? launch_qkv_t<128, true, APPEND>(a, stream) : launch_qkv_t<128, false, APPEND>(a, stream);
    return bf ? launch_qkv_t<64, true, APPEND>(a, stream) : launch_qkv_t<64, false, APPEND>(a, stream);
}

}  // namespace

cudaError_t launch_qkv_rope(const QkvRopeLaunch& L, cudaStream_t stream) {
    QkvArgs a{};
    a.qkv = L.qkv;
    a.params = L.params;
    a.positions = L.positions;
    a.rows = L.rows;
    a.heads = L.heads;
    a.max_context = L.max_context;
    a.status = L.status;
    if (!L.arena) {
        a.out = L.out;
        return launch_qkv<false>(a, L.head_dim, L.bf16, stream);
    }
    a.q_out = L.out;
    a.sk = L.scratch_k;
    a.sv = L.scratch_v;
    a.k_arena = L.arena->k;
    a.v_arena = L.arena->v;
    a.ks_arena = L.arena->k_scale;
    a.vs_arena = L.arena->v_scale;
    a.offsets = L.offsets;
    a.capacity = L.arena->capacity;
    a.commit = L.commit;
    return launch_qkv<true>(a, L.head_dim, L.bf16, stream);
}

cudaError_t launch_swiglu(const void* in, void* out, uint64_t rows, uint32_t hidden, bool bf, cudaStream_t stream) {
    const uint64_t n = rows * hidden;
    const uint32_t blocks = (uint32_t)((n + 255) / 256 < 148 * 16 ? (n + 255) / 256 : 148 * 16);
    if (bf) return launch_pdl(swiglu_kernel<true>, dim3(blocks), dim3(256), stream, in, out, rows, hidden);
    return launch_pdl(swiglu_kernel<false>, dim3(blocks), dim3(256), stream, in, out, rows, hidden);
}

cudaError_t launch_rmsnorm(const void* x, const void* residual, void* x_sum, const void* weight, void* out,
                           uint64_t rows, uint32_t width, float eps, bool bf, cudaStream_t stream) {
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (width % 256 == 0 && width <= 8192 && a16(x) && a16(weight) && a16(out) && (!residual || a16(residual)) &&
        (!x_sum || a16(x_sum))) {
        const uint32_t threads = width / 8;
        if (bf)
            return launch_pdl(rmsnorm_vec_kernel<true>, dim3((uint32_t)rows), dim3(threads), stream, x, residual, x_sum,
                              weight, out, width, eps);
        return launch_pdl(rmsnorm_vec_kernel<false>, dim3((uint32_t)rows), dim3(threads), stream, x, residual, x_sum,
                          weight, out, width, eps);
    }
    const uint32_t threads = width >= 256 ? 256 : 32 * ((width + 31) / 32);
    if (bf)
        return launch_pdl(rmsnorm_kernel<true>, dim3((uint32_t)rows), dim3(threads), stream, x, residual, x_sum, weight,
                          out, width, eps);
    return launch_pdl(rmsnorm_kernel<false>, dim3((uint32_t)rows), dim3(threads), stream, x, residual, x_sum, weight,
                      out, width, eps);
}

}  // namespace pp
