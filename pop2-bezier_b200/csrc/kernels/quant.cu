// Per-(token, head) symmetric int8 quantization, dequantization, the fused
// quantize-and-append into the caller's arena, and the committed-prefix copy.
//
// Quantization semantics follow the reference exactly (app/src/model/
// int8_kv_ops.rs:13-21 on CPU, int8_kv.cu:8-18 on CUDA):
//   s = max(max|x| / 127, 1e-12)            IEEE f32 division
//   q = clamp(round_half_even(x / s), -127, 127)
// This file is compiled without fast-math and with -fmad=false so that every
// division and product rounds exactly as in the reference.
#include <type_traits>

#include "common.cuh"
#include "quant_row.cuh"
#include "../host/internal.h"

namespace pp {
namespace {

template <typename T>
__device__ __forceinline__ float load_elem(const T* p, uint64_t i);
template <>
__device__ __forceinline__ float load_elem<float>(const float* p, uint64_t i) {
    return __ldg(p + i);
}
template <>
__device__ __forceinline__ float load_elem<__nv_bfloat16>(const __nv_bfloat16* p, uint64_t i) {
    return __bfloat162float(__ldg(p + i));
}

// One warp quantizes one row of D elements: lane l owns elements
// [l*E, l*E+E), E = D/32.  Returns false if an element is not finite.
template <int D, typename T>
__device__ __forceinline__ bool quantize_row_warp(const T* x, uint8_t* codes, float* scale_out, int lane) {
    constexpr int E = D / 32;
    float v[E];
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = load_elem<T>(x, (uint64_t)lane * E + e);
    return quantize_vals_warp<E>(v, codes, scale_out, lane);
}

template <int D, typename T>
__global__ void __launch_bounds__(256) quantize_kernel(const T* __restrict__ x, uint64_t rows,
                                                       uint8_t* __restrict__ packed, float* __restrict__ scales,
                                                       uint32_t* status) {
    const int lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
    for (uint64_t r = (uint64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += warps) {
        bool ok = quantize_row_warp<D, T>(x + r * D, packed + r * D, scales + r, lane);
        if (!ok && lane == 0 && status) atomicOr(status, PP_DEV_NONFINITE_INPUT);
    }
}

// Quantize-and-append: warp w of the grid handles (row, K or V).  The target
// slot is offsets[row / heads]; out-of-range offsets are reported, not written.
template <int D, typename T>
__global__ void __launch_bounds__(256) quant_append_kernel(const T* __restrict__ k_new, const T* __restrict__ v_new,
                                                           uint32_t rows, uint32_t heads, uint32_t capacity,
                                                           const uint32_t* __restrict__ offsets, uint32_t commit,
                                                           uint8_t* k_arena, uint8_t* v_arena, float* ks_arena,
                                                           float* vs_arena, uint32_t* status) {
    // launched as a programmatic dependent: wait for the kernel before.  No early
    // trigger: the history this kernel appends to is released only when it is
    // complete, whatever the next launch streams before its own wait.
    pdl_wait_primary();
    const int lane = threadIdx.x & 31;
    const uint64_t item = (uint64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    if (item >= 2ull * rows) return;
    const uint32_t row = (uint32_t)(item >> 1);
    const bool is_v = item & 1;
    const uint32_t off = __ldg(offsets + row / heads);
    if (off >= capacity) {
        if (lane == 0 && status) atomicOr(status, PP_DEV_OFFSET_RANGE);
        return;
    }
    const uint64_t slot = (uint64_t)row * capacity + off;
    uint8_t* codes = (is_v ? v_arena : k_arena) + slot * D;
    float* scale = (is_v ? vs_arena : ks_arena) + slot;
    if (commit) {
        const T* src = (is_v ? v_new : k_new) + (uint64_t)row * D;
        bool ok = quantize_row_warp<D, T>(src, codes, scale, lane);
        if (!ok && lane == 0 && status) atomicOr(status, PP_DEV_NONFINITE_INPUT);
    } else {
        // Partial query: zero placeholder codes and unit scale (int8_cache.rs:305-310).
        constexpr int E = D / 32;
        if constexpr (E == 4) {
            *reinterpret_cast<uint32_t*>(codes + lane * 4) = 0u;
        } else {
            *reinterpret_cast<uint16_t*>(codes + lane * 2) = 0u;
        }
        if (lane == 0) *scale = 1.0f;
    }
}

template <typename O>
__device__ __forceinline__ void store_elem(O* p, uint64_t i, float v);
template <>
__device__ __forceinline__ void store_elem<float>(float* p, uint64_t i, float v) {
    p[i] = v;
}
template <>
__device__ __forceinline__ void store_elem<__nv_bfloat16>(__nv_bfloat16* p, uint64_t i, float v) {
    p[i] = __float2bfloat16_rn(v);
}

template <typename O>
__global__ void __launch_bounds__(256) dequantize_kernel(const uint8_t* __restrict__ packed,
                                                         const float* __restrict__ scales, uint64_t n,
                                                         uint32_t head_dim, int round_bf16, O* __restrict__ out) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float v = (float)(int8_t)packed[i] * __ldg(scales + i / head_dim);
        if (round_bf16) v = bf16_round(v);
        store_elem<O>(out, i, v);
    }
}

// The same over 16-byte groups of codes (16 elements of one row, d % 16 == 0):
// one 16-byte load of codes, one scale, 16 products, 32 or 64 bytes stored.
// Each thread keeps kDqUnroll groups in flight (loads issued before any use)
// and the grid is one resident wave, so the loads of a whole SM cover the
// memory latency.  The codes become floats exactly (byte permute into
// 2^23 + 128 + c, packed subtract of the bias), the product is the reference's
// f32 multiply and the bf16 pack rounds to nearest even.
constexpr int kDqUnroll = 4;

__device__ __forceinline__ uint4 ld_stream(const uint4* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_stream(uint4* p, uint4 v) {
    asm volatile("st.global.cs.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

template <typename O>
__device__ __forceinline__ void dequant_group(uint4 w, float s, int round_bf16, O* out) {
    const uint64_t s2 = f2_pack(s, s);
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    uint64_t p[8];  // element pairs (2k, 2k+1)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        i8x4_to_f32x2(words[k], p[2 * k], p[2 * k + 1]);
        p[2 * k] = f2_mul(p[2 * k], s2);
        p[2 * k + 1] = f2_mul(p[2 * k + 1], s2);
    }
    if constexpr (std::is_same<O, float>::value) {
        uint4* o = reinterpret_cast<uint4*>(out);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            float a, b, c, d;
            f2_unpack(p[2 * k], a, b);
            f2_unpack(p[2 * k + 1], c, d);
            if (round_bf16) {
                a = bf16_round(a);
                b = bf16_round(b);
                c = bf16_round(c);
                d = bf16_round(d);
            }
            st_stream(o + k, make_uint4(__float_as_uint(a), __float_as_uint(b), __float_as_uint(c), __float_as_uint(d)));
        }
    } else {
        uint4* o = reinterpret_cast<uint4*>(out);
#pragma unroll
        for (int k = 0; k < 2; ++k)
            st_stream(o + k, make_uint4(pack_bf16x2_f2(p[4 * k]), pack_bf16x2_f2(p[4 * k + 1]),
                                        pack_bf16x2_f2(p[4 * k + 2]), pack_bf16x2_f2(p[4 * k + 3])));
    }
}

template <typename O>
__global__ void __launch_bounds__(256, 4) dequantize16_kernel(const uint4* __restrict__ packed,
                                                           const float* __restrict__ scales, uint64_t groups,
                                                           uint32_t groups_per_row, int round_bf16, O* __restrict__ out) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + (kDqUnroll - 1) * stride < groups; i += kDqUnroll * stride) {
        uint4 w[kDqUnroll];
        float s[kDqUnroll];
#pragma unroll
        for (int u = 0; u < kDqUnroll; ++u) {
            w[u] = ld_stream(packed + i + u * stride);
            s[u] = __ldg(scales + (i + u * stride) / groups_per_row);
        }
#pragma unroll
        for (int u = 0; u < kDqUnroll; ++u) dequant_group<O>(w[u], s[u], round_bf16, out + (i + u * stride) * 16);
    }
    for (; i < groups; i += stride)
        dequant_group<O>(ld_stream(packed + i), __ldg(scales + i / groups_per_row), round_bf16, out + i * 16);
}

// Row-prefix copy between arenas: block (row, chunk) copies 16-byte vectors of
// codes and 4-byte scales of the committed prefix.
__global__ void __launch_bounds__(256) copy_prefix_kernel(const uint8_t* __restrict__ sk, const uint8_t* __restrict__ sv,
                                                          const float* __restrict__ sks, const float* __restrict__ svs,
                                                          uint32_t src_cap, uint8_t* dk, uint8_t* dv, float* dks,
                                                          float* dvs, uint32_t dst_cap, uint32_t head_dim,
                                                          uint32_t heads, const uint32_t* __restrict__ lengths,
                                                          uint32_t* status) {
    const uint32_t row = blockIdx.y;
    uint32_t len = __ldg(lengths + row / heads);
    if (len > src_cap || len > dst_cap) {
        if (threadIdx.x == 0 && blockIdx.x == 0 && status) atomicOr(status, PP_DEV_LENGTH_RANGE);
        return;
    }
    const uint64_t vec_per_row = (uint64_t)len * head_dim / 16;
    const uint4* s_k = reinterpret_cast<const uint4*>(sk + (uint64_t)row * src_cap * head_dim);
    const uint4* s_v = reinterpret_cast<const uint4*>(sv + (uint64_t)row * src_cap * head_dim);
    uint4* d_k = reinterpret_cast<uint4*>(dk + (uint64_t)row * dst_cap * head_dim);
    uint4* d_v = reinterpret_cast<uint4*>(dv + (uint64_t)row * dst_cap * head_dim);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < vec_per_row; i += stride) {
        d_k[i] = s_k[i];
        d_v[i] = s_v[i];
    }
    for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < len; t += stride) {
        dks[(uint64_t)row * dst_cap + t] = sks[(uint64_t)row * src_cap + t];
        dvs[(uint64_t)row * dst_cap + t] = svs[(uint64_t)row * src_cap + t];
    }
}

uint32_t grid_for_warps(uint64_t warps, uint32_t warps_per_block, uint32_t cap) {
    uint64_t blocks = (warps + warps_per_block - 1) / warps_per_block;
    if (blocks == 0) blocks = 1;
    return (uint32_t)(blocks < cap ? blocks : cap);
}

}  // namespace

cudaError_t launch_quantize(const void* x, int dtype, uint64_t rows, uint32_t d, uint8_t* packed, float* scales,
                            uint32_t* status, cudaStream_t stream) {
    const uint32_t grid = grid_for_warps(rows, 8, 148u * 64u);
    if (d == 128) {
        if (dtype == PP_DTYPE_F32)
            quantize_kernel<128, float><<<grid, 256, 0, stream>>>((const float*)x, rows, packed, scales, status);
        else
            quantize_kernel<128, __nv_bfloat16>
                <<<grid, 256, 0, stream>>>((const __nv_bfloat16*)x, rows, packed, scales, status);
    } else {
        if (dtype == PP_DTYPE_F32)
            quantize_kernel<64, float><<<grid, 256, 0, stream>>>((const float*)x, rows, packed, scales, status);
        else
            quantize_kernel<64, __nv_bfloat16>
                <<<grid, 256, 0, stream>>>((const __nv_bfloat16*)x, rows, packed, scales, status);
    }
    return cudaGetLastError();
}

cudaError_t launch_quant_append(const PpKvArena& a, const void* k_new, const void* v_new, int dtype,
                                const uint32_t* offsets, uint32_t commit, uint32_t* status, cudaStream_t stream) {
    const uint64_t warps = 2ull * a.rows;
    const uint32_t grid = (uint32_t)((warps + 7) / 8);
    cudaError_t e;
#define PP_APPEND(D, T)                                                                                       \
    e = launch_pdl(quant_append_kernel<D, T>, dim3(grid), dim3(256), stream, (const T*)k_new, (const T*)v_new,    \
                   a.rows, a.heads, a.capacity, offsets, commit, a.k, a.v, a.k_scale, a.v_scale, status)
    if (a.head_dim == 128) {
        if (dtype == PP_DTYPE_F32) PP_APPEND(128, float);
        else PP_APPEND(128, __nv_bfloat16);
    } else {
        if (dtype == PP_DTYPE_F32) PP_APPEND(64, float);
        else PP_APPEND(64, __nv_bfloat16);
    }
#undef PP_APPEND
    return e;
}

cudaError_t launch_dequantize(const uint8_t* packed, const float* scales, uint64_t rows, uint32_t d, int round_bf16,
                              int out_dtype, void* out, cudaStream_t stream) {
    const uint64_t n = rows * d;
    const bool vec = d % 16 == 0 && (reinterpret_cast<uintptr_t>(packed) & 15u) == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
    if (vec) {
        const uint64_t groups = n / 16;
        const uint64_t blocks = (groups + 255) / 256;
        // one resident wave: 4 blocks of 256 threads per SM (<= 64 registers a
        // thread), 4 x 16 bytes in flight per thread = 64 KB per SM
        const uint32_t grid = (uint32_t)(blocks < 148u * 4u ? blocks : 148u * 4u);
        if (out_dtype == PP_DTYPE_F32)
            dequantize16_kernel<float><<<grid, 256, 0, stream>>>(reinterpret_cast<const uint4*>(packed), scales, groups,
                                                                 d / 16, round_bf16, (float*)out);
        else
            dequantize16_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(reinterpret_cast<const uint4*>(packed), scales,
                                                                         groups, d / 16, round_bf16,
                                                                         (__nv_bfloat16*)out);
        return cudaGetLastError();
    }
    uint64_t blocks = (n + 255) / 256;
    const uint32_t grid = (uint32_t)(blocks == 0 ? 1 : (blocks < 148u * 32u ? blocks : 148u * 32u));
    if (out_dtype == PP_DTYPE_F32)
        dequantize_kernel<float><<<grid, 256, 0, stream>>>(packed, scales, n, d, round_bf16, (float*)out);
    else
        dequantize_kernel<__nv_bfloat16>
            <<<grid, 256, 0, stream>>>(packed, scales, n, d, round_bf16, (__nv_bfloat16*)out);
    return cudaGetLastError();
}

cudaError_t launch_copy_prefix(const PpKvArena& s, const PpKvArena& d, const uint32_t* lengths, uint32_t* status,
                               cudaStream_t stream) {
    uint64_t vec = (uint64_t)s.capacity * s.head_dim / 16;
    uint32_t gx = (uint32_t)((vec + 255) / 256);
    if (gx > 64) gx = 64;
    if (gx == 0) gx = 1;
    dim3 grid(gx, s.rows);
    copy_prefix_kernel<<<grid, 256, 0, stream>>>(s.k, s.v, s.k_scale, s.v_scale, s.capacity, d.k, d.v, d.k_scale,
                                                 d.v_scale, d.capacity, s.head_dim, s.heads, lengths, status);
    return cudaGetLastError();
}

}  // namespace pp
