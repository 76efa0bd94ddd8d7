// C ABI implementation: host-side validation, TMA descriptor encoding and
// kernel launches for the int8 historical-KV engine.
//
// Validation mirrors the reference's checks before any device work
// (app/src/model/int8_kv_ops.rs:5-10 `geometry`, :44-48 attention `ensure!`s,
// app/src/model/write_plan.rs:27-45 `checked_shape`).  Nothing is launched
// when a check fails (status PP_STATUS_PRECONDITION).
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "internal.h"

namespace {

thread_local std::string g_last_error;

int32_t fail(int32_t status, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return status;
}

// CUDA errors: allocation/unsupported failures leave the device usable (the
// reference classifies them as safe, inference.rs:57-82); anything else makes
// the execution uncertain and the caller must discard its KV state.
int32_t cuda_fail(cudaError_t e, const char* what) {
    const bool safe = e == cudaErrorMemoryAllocation || e == cudaErrorNotSupported ||
                      e == cudaErrorNoKernelImageForDevice || e == cudaErrorInvalidDeviceFunction;
    if (safe) return fail(PP_STATUS_PRECONDITION, "%s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    return fail(PP_STATUS_UNCERTAIN, "EXECUTION_UNCERTAIN: %s failed: %s (%s)", what, cudaGetErrorName(e),
                cudaGetErrorString(e));
}

struct DeviceInfo {
    bool ready = false;
    unsigned long long ctx_id = 0;  // context the kernel attributes were set in
    int num_sms = 0;
    int major = 0;
};

std::mutex g_dev_mu;
DeviceInfo g_dev[64];
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int32_t device_info(DeviceInfo& out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    if (dev < 0 || dev >= 64) return fail(PP_STATUS_PRECONDITION, "device ordinal %d out of range", dev);
    unsigned long long ctx = 0;
    if (pp::current_context_id(&ctx) != PP_STATUS_OK) return PP_STATUS_PRECONDITION;
    std::lock_guard<std::mutex> lock(g_dev_mu);
    DeviceInfo& d = g_dev[dev];
    // kernel attributes belong to the context: a context made anew (after
    // cudaDeviceReset, or a released and re-created primary context) needs them again
    if (!d.ready || d.ctx_id != ctx) {
        d.ready = false;
        int minor = 0;
        if ((e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
            return cuda_fail(e, "cudaDeviceGetAttribute");
        if ((e = cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
            return cuda_fail(e, "cudaDeviceGetAttribute");
        if ((e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess)
            return cuda_fail(e, "cudaDeviceGetAttribute");
        if (d.major != 10 || minor != 0)
            return fail(PP_STATUS_PRECONDITION,
                        "CUDA_ERROR_NO_BINARY_FOR_GPU: this library is built for sm_100a (B200); device is sm_%d%d",
                        d.major, minor);
        if ((e = pp::configure_attention_kernels(dev)) != cudaSuccess) return cuda_fail(e, "kernel configuration");
        if (!g_encode) {
            void* fn = nullptr;
            cudaDriverEntryPointQueryResult q{};
            e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
            if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
                return fail(PP_STATUS_PRECONDITION, "CUDA_ERROR_NOT_SUPPORTED: cuTensorMapEncodeTiled unavailable");
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
        }
        d.ctx_id = ctx;
        d.ready = true;
    }
    out = d;
    return PP_STATUS_OK;
}

PFN_cuCtxGetCurrent_v4000 g_ctx_current = nullptr;
PFN_cuCtxGetId_v12000 g_ctx_id = nullptr;
std::once_flag g_ctx_once;

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int32_t check_arena(const PpKvArena* a, const char* what) {
    if (!a) return fail(PP_STATUS_PRECONDITION, "%s: arena is NULL", what);
    if (a->struct_size < sizeof(PpKvArena)) return fail(PP_STATUS_PRECONDITION, "%s: PpKvArena struct_size too small", what);
    if (a->rows == 0 || a->heads == 0 || a->rows % a->heads != 0 || a->capacity == 0)
        return fail(PP_STATUS_PRECONDITION, "INT8 attention geometry differs: rows=%u heads=%u capacity=%u", a->rows,
                    a->heads, a->capacity);
    if (a->head_dim != 64 && a->head_dim != 128)
        return fail(PP_STATUS_PRECONDITION, "INT8 KV requires dense [heads,tokens,64|128], head_dim=%u", a->head_dim);
    if ((uint64_t)a->rows * a->capacity > 0x7fffff00ull)
        return fail(PP_STATUS_PRECONDITION, "INT8 KV dimensions overflow: rows*capacity=%llu exceeds 2^31-256",
                    (unsigned long long)a->rows * a->capacity);
    if (!a->k || !a->v || !a->k_scale || !a->v_scale) return fail(PP_STATUS_PRECONDITION, "%s: NULL arena pointer", what);
    if (!aligned(a->k, 16) || !aligned(a->v, 16))
        return fail(PP_STATUS_PRECONDITION, "%s: packed K/V arenas must be 16-byte aligned", what);
    if (!aligned(a->k_scale, 4) || !aligned(a->v_scale, 4))
        return fail(PP_STATUS_PRECONDITION, "%s: scale arenas must be 4-byte aligned", what);
    return PP_STATUS_OK;
}

int32_t check_dtype(int32_t t, const char* what) {
    if (t != PP_DTYPE_F32 && t != PP_DTYPE_BF16) return fail(PP_STATUS_PRECONDITION, "%s: unsupported dtype %d", what, t);
    return PP_STATUS_OK;
}

PpAttnParams effective_params(const PpAttnParams* p) {
    PpAttnParams e{};
    e.struct_size = sizeof(PpAttnParams);
    e.q_dtype = PP_DTYPE_F32;
    e.out_dtype = PP_DTYPE_F32;
    if (p) {
        const size_t n = p->struct_size < sizeof(PpAttnParams) ? p->struct_size : sizeof(PpAttnParams);
        std::memcpy(&e, p, n);
    }
    return e;
}

uint32_t ctas_for(const PpAttnParams& p, const DeviceInfo& d) {
    uint32_t g = p.max_ctas ? p.max_ctas : (uint32_t)d.num_sms;
    return g ? g : 1u;
}

// 2-D map over the packed codes: dims {head_dim, rows*capacity} bytes, boxes of
// `box_tokens` tokens, swizzled so the consumer warps read shared memory
// without bank conflicts.
int32_t encode_codes_map(CUtensorMap* map, const uint8_t* base, const PpKvArena& a, uint32_t box_tokens) {
    cuuint64_t dims[2] = {a.head_dim, (cuuint64_t)a.rows * a.capacity};
    cuuint64_t strides[1] = {a.head_dim};
    cuuint32_t box[2] = {a.head_dim, box_tokens};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE,
                          a.head_dim == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(PP_STATUS_PRECONDITION, "cuTensorMapEncodeTiled (codes) failed: %d", (int)r);
    return PP_STATUS_OK;
}

// 1-D map over a scale array whose base may be only 4-byte aligned: the map
// starts at the 16-byte boundary below it and `mis` counts the elements skipped.
int32_t encode_scale_map(CUtensorMap* map, uint32_t* mis, const float* base, const PpKvArena& a) {
    const uintptr_t addr = reinterpret_cast<uintptr_t>(base);
    const uintptr_t aligned_addr = addr & ~uintptr_t(15);
    *mis = (uint32_t)((addr - aligned_addr) / 4);
    cuuint64_t dims[1] = {(cuuint64_t)*mis + (cuuint64_t)a.rows * a.capacity};
    cuuint64_t strides[1] = {0};
    cuuint32_t box[1] = {pp::attention_scale_box_elems()};
    cuuint32_t estr[1] = {1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 1, reinterpret_cast<void*>(aligned_addr), dims, strides,
                          box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(PP_STATUS_PRECONDITION, "cuTensorMapEncodeTiled (scales) failed: %d", (int)r);
    return PP_STATUS_OK;
}

// Launch fields shared by the int8 and float entry points: options, device,
// plan layout and workspace.  `split` is the fixed split (0: stream-K).
int32_t prepare_common(const PpAttnParams& p, uint32_t split, const uint32_t* lengths, void* workspace,
                       size_t ws_bytes, pp::AttnLaunch& L, const char* what) {
    int32_t s;
    if ((s = check_dtype(p.q_dtype, "q"))) return s;
    if ((s = check_dtype(p.out_dtype, "out"))) return s;
    if (!(p.softmax_scale >= 0.f) || !std::isfinite(p.softmax_scale))
        return fail(PP_STATUS_PRECONDITION, "softmax_scale must be finite and >= 0");
    DeviceInfo d;
    if ((s = device_info(d))) return s;
    const uint32_t hd = L.arena.head_dim;
    L.split = split;
    L.q_dtype = p.q_dtype;
    L.out_dtype = p.out_dtype;
    const float scale = p.softmax_scale > 0.f ? p.softmax_scale
                                              : (hd == 64 ? 0.125f : (float)(1.0 / std::sqrt((double)hd)));
    L.scale_log2 = scale * 1.4426950408889634f;
    L.max_ctas = ctas_for(p, d);
    L.num_sms = (uint32_t)d.num_sms;
    L.lengths = lengths;
    L.layout = pp::ws_layout(L.arena.rows, L.arena.capacity, hd, L.split, L.max_ctas);
    L.plan_ready = (p.flags & PP_ATTN_PLAN_READY) != 0;
    L.prefetch = (p.flags & PP_ATTN_PREFETCH_HISTORY) != 0;
    if (L.prefetch && !L.plan_ready)
        return fail(PP_STATUS_PRECONDITION, "%s: PP_ATTN_PREFETCH_HISTORY needs PP_ATTN_PLAN_READY (the plan kernel "
                    "writes what the prefetch reads)", what);
    L.use_pdl = true;
    if (!workspace) return fail(PP_STATUS_PRECONDITION, "%s: workspace is NULL", what);
    if (!aligned(workspace, 256)) return fail(PP_STATUS_PRECONDITION, "%s: workspace must be 256-byte aligned", what);
    if (ws_bytes < L.layout.total)
        return fail(PP_STATUS_PRECONDITION, "%s: workspace too small (%zu < %zu bytes)", what, ws_bytes, L.layout.total);
    L.ws = static_cast<unsigned char*>(workspace);
    return PP_STATUS_OK;
}

int32_t prepare_launch(const PpKvArena* arena, const PpAttnParams* params, const uint32_t* lengths,
                       const float* scratch_k, const float* scratch_v, void* workspace, size_t ws_bytes,
                       pp::AttnLaunch& L, const char* what) {
    int32_t s;
    if ((s = check_arena(arena, what))) return s;
    const PpAttnParams p = effective_params(params);
    if (!lengths) return fail(PP_STATUS_PRECONDITION, "INT8 attention lengths differ: lengths pointer is NULL");
    if ((scratch_k == nullptr) != (scratch_v == nullptr))
        return fail(PP_STATUS_PRECONDITION, "INT8 scratch must be F32[head_rows,1,%u]: pass both or neither", arena->head_dim);
    if ((scratch_k && !aligned(scratch_k, 4)) || (scratch_v && !aligned(scratch_v, 4)))
        return fail(PP_STATUS_PRECONDITION, "INT8 scratch must be 4-byte aligned");
    L = pp::AttnLaunch{};
    L.arena = *arena;
    L.kv_kind = pp::kKvInt8;
    L.q_stride = arena->head_dim;
    L.scratch_k = scratch_k;
    L.scratch_v = scratch_v;
    return prepare_common(p, p.split_tokens, lengths, workspace, ws_bytes, L, what);
}

// Geometry checks of fused_attention.rs:12-25, plus what the tensor copies need.
int32_t check_float_kv(const PpFloatKv* kv, const char* what) {
    if (!kv || kv->struct_size < sizeof(PpFloatKv)) return fail(PP_STATUS_PRECONDITION, "%s: PpFloatKv missing", what);
    const PpFloatKv& g = *kv;
    if (g.rows == 0 || g.heads == 0 || g.rows % g.heads != 0 || g.tokens == 0 ||
        (g.head_dim != 64 && g.head_dim != 128) || (g.dtype != PP_DTYPE_F32 && g.dtype != PP_DTYPE_BF16))
        return fail(PP_STATUS_PRECONDITION,
                    "fused decode attention requires F32[batch*heads,1,64|128] and same-device BF16/F32 K/V: "
                    "rows=%u heads=%u head_dim=%u tokens=%u dtype=%d",
                    g.rows, g.heads, g.head_dim, g.tokens, g.dtype);
    if (g.rows > 0x7fffffffu || g.tokens > 0x7fffff00u)
        return fail(PP_STATUS_PRECONDITION, "fused attention dimensions overflow: rows=%u tokens=%u", g.rows, g.tokens);
    if (!g.k || !g.v) return fail(PP_STATUS_PRECONDITION, "%s: NULL K/V pointer", what);
    const uint64_t elem = g.dtype == PP_DTYPE_F32 ? 4 : 2, dense = (uint64_t)g.tokens * g.head_dim;
    if (g.k_row_stride < dense || g.v_row_stride < dense)
        return fail(PP_STATUS_PRECONDITION, "fused attention requires dense width and token strides: row strides %llu/%llu "
                    "< tokens*head_dim=%llu", (unsigned long long)g.k_row_stride, (unsigned long long)g.v_row_stride,
                    (unsigned long long)dense);
    if (!aligned(g.k, 16) || !aligned(g.v, 16) || (g.k_row_stride * elem) % 16 || (g.v_row_stride * elem) % 16 ||
        g.k_row_stride * elem >= (1ull << 40) || g.v_row_stride * elem >= (1ull << 40))
        return fail(PP_STATUS_PRECONDITION, "fused attention requires dense width and token strides: K/V rows must "
                    "start on 16-byte boundaries (base and row stride)");
    return PP_STATUS_OK;
}

int32_t prepare_float_launch(const PpFloatKv* kv, const PpAttnParams* params, const uint32_t* lengths,
                             void* workspace, size_t ws_bytes, pp::AttnLaunch& L, const char* what) {
    int32_t s;
    if ((s = check_float_kv(kv, what))) return s;
    const PpAttnParams p = effective_params(params);
    L = pp::AttnLaunch{};
    L.arena.struct_size = sizeof(PpKvArena);
    L.arena.rows = kv->rows;
    L.arena.heads = kv->heads;
    L.arena.head_dim = kv->head_dim;
    L.arena.capacity = kv->tokens;
    L.kv_kind = kv->dtype == PP_DTYPE_BF16 ? pp::kKvBf16 : pp::kKvF32;
    L.q_stride = kv->head_dim;
    // fused_attention.rs:29: split_tokens.clamp(32, 1024), 0 = whole rows
    const uint32_t split = p.split_tokens == 0 ? 0u : p.split_tokens < 32 ? 32u : p.split_tokens > 1024 ? 1024u
                                                                                                      : p.split_tokens;
    return prepare_common(p, split, lengths, workspace, ws_bytes, L, what);
}

// 3-D map over float K or V rows: dims {head_dim, tokens, rows}, boxes of one
// 128-byte panel x `box_tokens` tokens, 128-byte swizzle.
int32_t encode_float_map(CUtensorMap* map, const void* base, uint64_t row_stride, const PpFloatKv& kv,
                         uint32_t box_tokens) {
    const uint32_t elem = kv.dtype == PP_DTYPE_F32 ? 4u : 2u;
    cuuint64_t dims[3] = {kv.head_dim, kv.tokens, kv.rows};
    cuuint64_t strides[2] = {(cuuint64_t)kv.head_dim * elem, (cuuint64_t)row_stride * elem};
    cuuint32_t box[3] = {128u / elem, box_tokens, 1u};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = g_encode(map, elem == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                          const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(PP_STATUS_PRECONDITION, "cuTensorMapEncodeTiled (float K/V) failed: %d", (int)r);
    return PP_STATUS_OK;
}

}  // namespace

namespace pp {
int32_t fail_msg(int32_t status, const char* msg) {
    g_last_error = msg;
    return status;
}

int32_t current_context_id(unsigned long long* id) {
    // the driver's context calls, reached through the runtime (the library
    // links only the runtime); cudaFree(nullptr) makes the primary context current
    std::call_once(g_ctx_once, [] {
        void* a = nullptr;
        void* b = nullptr;
        cudaDriverEntryPointQueryResult qa{}, qb{};
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &a, 4000, cudaEnableDefault, &qa) == cudaSuccess &&
            qa == cudaDriverEntryPointSuccess)
            g_ctx_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(a);
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &b, 12000, cudaEnableDefault, &qb) == cudaSuccess &&
            qb == cudaDriverEntryPointSuccess)
            g_ctx_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(b);
    });
    if (!g_ctx_current || !g_ctx_id)
        return fail(PP_STATUS_PRECONDITION, "CUDA_ERROR_NOT_SUPPORTED: cuCtxGetCurrent / cuCtxGetId unavailable");
    CUcontext ctx = nullptr;
    if (g_ctx_current(&ctx) != CUDA_SUCCESS || !ctx) {
        cudaError_t e = cudaFree(nullptr);
        if (e != cudaSuccess) return cuda_fail(e, "cudaFree(nullptr) (context set-up)");
        if (g_ctx_current(&ctx) != CUDA_SUCCESS || !ctx)
            return fail(PP_STATUS_UNCERTAIN, "EXECUTION_UNCERTAIN: no current CUDA context");
    }
    if (g_ctx_id(ctx, id) != CUDA_SUCCESS) return fail(PP_STATUS_UNCERTAIN, "EXECUTION_UNCERTAIN: cuCtxGetId failed");
    return PP_STATUS_OK;
}
}  // namespace pp

extern "C" {

uint32_t pp_b200_abi_version(void) { return PP_B200_ABI_VERSION; }

const char* pp_b200_last_error(void) { return g_last_error.c_str(); }

int32_t pp_b200_quantize(const void* x, int32_t x_dtype, uint64_t rows, uint32_t head_dim, uint8_t* packed,
                         float* scales, uint32_t* status, void* stream) {
    int32_t s;
    if (rows == 0 || (head_dim != 64 && head_dim != 128))
        return fail(PP_STATUS_PRECONDITION, "INT8 KV requires dense [heads,tokens,64|128] (rows=%llu, head_dim=%u)",
                    (unsigned long long)rows, head_dim);
    if (rows > (UINT64_MAX / head_dim)) return fail(PP_STATUS_PRECONDITION, "INT8 KV dimensions overflow");
    if ((s = check_dtype(x_dtype, "quantize input"))) return s;
    if (!x || !packed || !scales) return fail(PP_STATUS_PRECONDITION, "quantize: NULL pointer");
    if (!aligned(x, x_dtype == PP_DTYPE_F32 ? 16 : 8) || !aligned(packed, 4) || !aligned(scales, 4))
        return fail(PP_STATUS_PRECONDITION, "quantize: misaligned pointer");
    DeviceInfo d;
    if ((s = device_info(d))) return s;
    cudaError_t e = pp::launch_quantize(x, x_dtype, rows, head_dim, packed, scales, status, (cudaStream_t)stream);
    return e == cudaSuccess ? PP_STATUS_OK : cuda_fail(e, "INT8 quantize launch");
}

int32_t pp_b200_dequantize(const uint8_t* packed, const float* scales, uint64_t rows, uint32_t head_dim,
                           int32_t round_bf16, int32_t out_dtype, void* out, void* stream) {
    int32_t s;
    if (rows == 0 || (head_dim != 64 && head_dim != 128))
        return fail(PP_STATUS_PRECONDITION, "INT8 KV scales differ: rows=%llu head_dim=%u", (unsigned long long)rows, head_dim);
    if ((s = check_dtype(out_dtype, "dequantize output"))) return s;
    if (!packed || !scales || !out) return fail(PP_STATUS_PRECONDITION, "dequantize: NULL pointer");
    DeviceInfo d;
    if ((s = device_info(d))) return s;
    cudaError_t e = pp::launch_dequantize(packed, scales, rows, head_dim, round_bf16, out_dtype, out, (cudaStream_t)stream);
    return e == cudaSuccess ? PP_STATUS_OK : cuda_fail(e, "INT8 dequantize launch");
}

int32_t pp_b200_quant_append(const PpKvArena* arena, const void* k_new, const void* v_new, int32_t dtype,
                             const uint32_t* offsets, uint32_t commit, uint32_t* status, void* stream) {
    int32_t s;
    if ((s = check_arena(arena, "quant_append"))) return s;
    if ((s = check_dtype(dtype, "append input"))) return s;
    if (!k_new || !v_new || !offsets) return fail(PP_STATUS_PRECONDITION, "INT8 batch requires [B,H,1,D] scratch: NULL input");
    const uintptr_t need = dtype == PP_DTYPE_F32 ? 16 : 8;
    if (!aligned(k_new, need) || !aligned(v_new, need)) return fail(PP_STATUS_PRECONDITION, "quant_append: misaligned K/V input");
    DeviceInfo d;
    if ((s = device_info(d))) return s;
    cudaError_t e = pp::launch_quant_append(*arena, k_new, v_new, dtype, offsets, commit, status, (cudaStream_t)stream);
    return e == cudaSuccess ? PP_STATUS_OK : cuda_fail(e, "INT8 quant_append launch");
}

int32_t pp_b200_copy_prefix(const PpKvArena* src, const PpKvArena* dst, const uint32_t* lengths, void* stream) {
    int32_t s;
    if ((s = check_arena(src, "copy_prefix src"))) return s;
    if ((s = check_arena(dst, "copy_prefix dst"))) return s;
    if (src->rows != dst->rows || src->heads != dst->heads || src->head_dim != dst->head_dim)
        return fail(PP_STATUS_PRECONDITION, "batch KV existing row is incompatible: arenas differ in rows/heads/head_dim");
    if (!lengths) return fail(PP_STATUS_PRECONDITION, "copy_prefix: lengths is NULL");
    DeviceInfo d;
    if ((s = device_info(d))) return s;
    cudaError_t e = pp::launch_copy_prefix(*src, *dst, lengths, nullptr, (cudaStream_t)stream);
    return e == cudaSuccess ? PP_STATUS_OK : cuda_fail(e, "INT8 copy_prefix launch");
}

size_t pp_b200_attention_workspace_size(const PpKvArena* arena, const PpAttnParams* params) {
    if (!arena || arena->rows == 0 || (arena->head_dim != 64 && arena->head_dim != 128)) return 0;
    const PpAttnParams p = effective_params(params);
    uint32_t g = p.max_ctas;
    if (!g) {
        DeviceInfo d;
        if (device_info(d) != PP_STATUS_OK) g = 1024;  // conservative without a device
        else g = (uint32_t)d.num_sms;
    }
    return pp::ws_layout(arena->rows, arena->capacity, arena->head_dim, p.split_tokens, g).total;
}

int32_t pp_b200_plan_ragged(const PpKvArena* arena, const PpAttnParams* params, const uint32_t* lengths,
                            uint32_t scratch_token, void* workspace, size_t workspace_bytes, void* stream) {
    pp::AttnLaunch L;
    static const float kDummy = 0.f;
    const float* sk = scratch_token ? &kDummy : nullptr;  // only its presence matters to the plan
    int32_t s = prepare_launch(arena, params, lengths, sk, sk, workspace, workspace_bytes, L, "plan_ragged");
    if (s) return s;
    cudaError_t e = pp::launch_plan(L, (cudaStream_t)stream);
    return e == cudaSuccess ? PP_STATUS_OK : cuda_fail(e, "INT8 plan launch");
}

int32_t pp_b200_decode_attention(const PpKvArena* arena, const PpAttnParams* params, const void* q,
                                 const float* scratch_k, const float* scratch_v, const uint32_t* lengths, void* out,
                                 void* workspace, size_t workspace_bytes, uint32_t* status, void* stream) {
    pp::AttnLaunch L;
    int32_t s = prepare_launch(arena, params, lengths, scratch_k, scratch_v, workspace, workspace_bytes, L,
                               "decode_attention");
    if (s) return s;
    if (!q || !out) return fail(PP_STATUS_PRECONDITION, "INT8 scratch must be F32[head_rows,1,%u]: NULL q/out", arena->head_dim);
    if (!aligned(q, 16)) return fail(PP_STATUS_PRECONDITION, "decode_attention: q must be 16-byte aligned");
    if (!aligned(out, L.out_dtype == PP_DTYPE_F32 ? 4 : 2))
        return fail(PP_STATUS_PRECONDITION, "decode_attention: out is misaligned");
    L.q = q;
    L.out = out;
    L.status = status;
    L.short_stages = pp::attention_short_stages(arena->head_dim, arena->rows, arena->capacity, L.max_ctas);
    const uint32_t stage = pp::attention_stage_tokens(arena->head_dim, L.short_stages);  // rows of one whole-stage box
    for (int i = 0; i < pp::kTailBoxes; ++i) {
        if ((s = encode_codes_map(&L.tails.k[i], arena->k, *arena, 16u << i))) return s;
        if ((s = encode_codes_map(&L.tails.v[i], arena->v, *arena, 16u << i))) return s;
    }
    if ((s = encode_codes_map(&L.map_k_stage, arena->k, *arena, stage))) return s;
    if ((s = encode_codes_map(&L.map_v_stage, arena->v, *arena, stage))) return s;
    if ((s = encode_scale_map(&L.map_ks, &L.ks_mis, arena->k_scale, *arena))) return s;
    if ((s = encode_scale_map(&L.map_vs, &L.vs_mis, arena->v_scale, *arena))) return s;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    if (!L.plan_ready && (e = pp::launch_plan(L, st)) != cudaSuccess) return cuda_fail(e, "INT8 plan launch");
    if ((e = pp::launch_attention(L, st)) != cudaSuccess) return cuda_fail(e, "INT8 attention launch");
    // stream-K plans are finished inside the attention kernel; fixed splits need the combine
    if (L.split && (e = pp::launch_combine(L, st)) != cudaSuccess) return cuda_fail(e, "INT8 combine launch");
    return PP_STATUS_OK;
}

size_t pp_b200_float_attention_workspace_size(const PpFloatKv* kv, const PpAttnParams* params) {
    if (!kv || kv->struct_size < sizeof(PpFloatKv) || kv->rows == 0 || (kv->head_dim != 64 && kv->head_dim != 128))
        return 0;
    const PpAttnParams p = effective_params(params);
    uint32_t g = p.max_ctas;
    if (!g) {
        DeviceInfo d;
        if (device_info(d) != PP_STATUS_OK) g = 1024;  // conservative without a device
        else g = (uint32_t)d.num_sms;
    }
    const uint32_t split = p.split_tokens == 0 ? 0u : p.split_tokens < 32 ? 32u : p.split_tokens > 1024 ? 1024u
                                                                                                      : p.split_tokens;
    return pp::ws_layout(kv->rows, kv->tokens, kv->head_dim, split, g).total;
}

int32_t pp_b200_plan_ragged_float(const PpFloatKv* kv, const PpAttnParams* params, const uint32_t* lengths,
                                  void* workspace, size_t workspace_bytes, void* stream) {
    pp::AttnLaunch L;
    int32_t s = prepare_float_launch(kv, params, lengths, workspace, workspace_bytes, L, "plan_ragged_float");
    if (s) return s;
    cudaError_t e = pp::launch_plan(L, (cudaStream_t)stream);
    return e == cudaSuccess ? PP_STATUS_OK : cuda_fail(e, "fused attention plan launch");
}

int32_t pp_b200_decode_attention_float(const PpFloatKv* kv, const PpAttnParams* params, const void* q,
                                       uint64_t q_row_stride, const uint32_t* lengths, void* out, void* workspace,
                                       size_t workspace_bytes, uint32_t* status, void* stream) {
    pp::AttnLaunch L;
    int32_t s = prepare_float_launch(kv, params, lengths, workspace, workspace_bytes, L, "decode_attention_float");
    if (s) return s;
    if (!q || !out)
        return fail(PP_STATUS_PRECONDITION, "fused decode attention requires F32[batch*heads,1,%u]: NULL q/out",
                    kv->head_dim);
    const uint64_t qe = L.q_dtype == PP_DTYPE_F32 ? 4 : 2;
    if (q_row_stride < kv->head_dim || !aligned(q, 16) || (q_row_stride * qe) % 16)
        return fail(PP_STATUS_PRECONDITION, "fused attention requires dense width and token strides: q rows must "
                    "start on 16-byte boundaries (q_row_stride=%llu)", (unsigned long long)q_row_stride);
    if (!aligned(out, L.out_dtype == PP_DTYPE_F32 ? 4 : 2))
        return fail(PP_STATUS_PRECONDITION, "decode_attention_float: out is misaligned");
    L.q = q;
    L.q_stride = q_row_stride;
    L.out = out;
    L.status = status;
    const uint32_t stage = pp::attention_float_stage_tokens(kv->head_dim, L.kv_kind);
    for (int i = 0; i < pp::kTailBoxes; ++i) {
        if ((s = encode_float_map(&L.tails.k[i], kv->k, kv->k_row_stride, *kv, 16u << i))) return s;
        if ((s = encode_float_map(&L.tails.v[i], kv->v, kv->v_row_stride, *kv, 16u << i))) return s;
    }
    if ((s = encode_float_map(&L.map_k_stage, kv->k, kv->k_row_stride, *kv, stage))) return s;
    if ((s = encode_float_map(&L.map_v_stage, kv->v, kv->v_row_stride, *kv, stage))) return s;
    cudaStream_t st = (cudaStream_t)stream;
    cudaError_t e;
    if (!L.plan_ready && (e = pp::launch_plan(L, st)) != cudaSuccess) return cuda_fail(e, "fused attention plan launch");
    if ((e = pp::launch_attention(L, st)) != cudaSuccess) return cuda_fail(e, "fused attention launch");
    if (L.split && (e = pp::launch_combine(L, st)) != cudaSuccess) return cuda_fail(e, "fused attention merge launch");
    return PP_STATUS_OK;
}

}  // extern "C"

namespace {

int32_t check_qkv(const PpQkvRope* g, const void* qkv, const void* params, const uint32_t* positions, const void* out,
                  const char* what, PpQkvRope& e) {
    if (!g || g->struct_size < sizeof(PpQkvRope)) return fail(PP_STATUS_PRECONDITION, "%s: PpQkvRope missing", what);
    e = *g;
    if (e.rows == 0 || e.heads == 0 || (e.head_dim != 64 && e.head_dim != 128) || e.max_context == 0)
        return fail(PP_STATUS_PRECONDITION, "graph QKV/RoPE geometry differs: rows=%u heads=%u head_dim=%u max_context=%u",
                    e.rows, e.heads, e.head_dim, e.max_context);
    if ((uint64_t)e.rows * e.heads > 0xffffffffull || 3ull * e.heads * e.head_dim > 0xffffffffull)
        return fail(PP_STATUS_PRECONDITION, "graph metadata exceeds U32 indexing");
    int32_t s;
    if ((s = check_dtype(e.dtype, what))) return s;
    if (!qkv || !params || !positions || !out) return fail(PP_STATUS_PRECONDITION, "%s: NULL pointer", what);
    return PP_STATUS_OK;
}

}  // namespace

extern "C" {

int32_t pp_b200_qkv_rope(const PpQkvRope* geometry, const void* qkv, const void* params, const uint32_t* positions,
                         void* out, uint32_t* status, void* stream) {
    PpQkvRope g;
    int32_t s;
    if ((s = check_qkv(geometry, qkv, params, positions, out, "qkv_rope", g))) return s;
    DeviceInfo d;
    if ((s = device_info(d))) return s;
    pp::QkvRopeLaunch L{};
    L.qkv = qkv;
    L.params = params;
    L.positions = positions;
    L.rows = g.rows;
    L.heads = g.heads;
    L.head_dim = g.head_dim;
    L.max_context = g.max_context;
    L.bf16 = g.dtype == PP_DTYPE_BF16;
    L.out = out;
    L.status = status;
    cudaError_t e = pp::launch_qkv_rope(L, (cudaStream_t)stream);
    return e == cudaSuccess ? PP_STATUS_OK : cuda_fail(e, "graph QKV launch");
}

int32_t pp_b200_qkv_rope_append(const PpQkvRope* geometry, const void* qkv, const void* params,
                                const uint32_t* positions, const PpKvArena* arena, const uint32_t* offsets,
                                uint32_t commit, void* q_out, float* scratch_k, float* scratch_v, uint32_t* status,
                                void* stream) {
    PpQkvRope g;
    int32_t s;
    if ((s = check_qkv(geometry, qkv, params, positions, q_out, "qkv_rope_append", g))) return s;
    if ((s = check_arena(arena, "qkv_rope_append"))) return s;
    if (arena->heads != g.heads || arena->head_dim != g.head_dim || (uint64_t)arena->rows != (uint64_t)g.rows * g.heads)
        return fail(PP_STATUS_PRECONDITION,
                    "INT8 batch requires [B,H,1,D] scratch and matching row histories: arena %ux%u/%u vs qkv %ux%u/%u",
                    arena->rows, arena->heads, arena->head_dim, g.rows, g.heads, g.head_dim);
    if (!offsets || !scratch_k || !scratch_v) return fail(PP_STATUS_PRECONDITION, "qkv_rope_append: NULL pointer");
    DeviceInfo d;
    if ((s = device_info(d))) return s;
    pp::QkvRopeLaunch L{};
    L.qkv = qkv;
    L.params = params;
    L.positions = positions;
    L.rows = g.rows;
    L.heads = g.heads;
    L.head_dim = g.head_dim;
    L.max_context = g.max_context;
    L.bf16 = g.dtype == PP_DTYPE_BF16;
    L.out = q_out;
    L.scratch_k = scratch_k;
    L.scratch_v = scratch_v;
    L.arena = arena;
    L.offsets = offsets;
    L.commit = commit;
    L.status = status;
    cudaError_t e = pp::launch_qkv_rope(L, (cudaStream_t)stream);
    return e == cudaSuccess ? PP_STATUS_OK : cuda_fail(e, "graph QKV append launch");
}

int32_t pp_b200_swiglu(const void* in, void* out, uint64_t rows, uint32_t hidden, int32_t dtype, void* stream) {
    int32_t s;
    if (rows == 0 || hidden == 0) return fail(PP_STATUS_PRECONDITION, "graph operation has an empty dimension");
    if (rows > UINT64_MAX / (2ull * hidden)) return fail(PP_STATUS_PRECONDITION, "graph operation element count overflow");
    if ((s = check_dtype(dtype, "swiglu"))) return s;
    if (!in || !out) return fail(PP_STATUS_PRECONDITION, "swiglu: NULL pointer");
    DeviceInfo d;
    if ((s = device_info(d))) return s;
    cudaError_t e = pp::launch_swiglu(in, out, rows, hidden, dtype == PP_DTYPE_BF16, (cudaStream_t)stream);
    return e == cudaSuccess ? PP_STATUS_OK : cuda_fail(e, "graph SwiGLU launch");
}

int32_t pp_b200_rmsnorm(const void* x, const void* residual, void* x_sum, const void* weight, void* out, uint64_t rows,
                        uint32_t width, float eps, int32_t dtype, void* stream) {
    int32_t s;
    if (rows == 0 || width == 0 || rows > 0x7fffffffull)
        return fail(PP_STATUS_PRECONDITION, "rms_norm geometry differs: rows=%llu width=%u", (unsigned long long)rows, width);
    if (!(eps >= 0.f) || !std::isfinite(eps)) return fail(PP_STATUS_PRECONDITION, "rms_norm eps must be finite and >= 0");
    if ((s = check_dtype(dtype, "rms_norm"))) return s;
    if (!x || !weight || !out) return fail(PP_STATUS_PRECONDITION, "rms_norm: NULL pointer");
    DeviceInfo d;
    if ((s = device_info(d))) return s;
    cudaError_t e = pp::launch_rmsnorm(x, residual, x_sum, weight, out, rows, width, eps, dtype == PP_DTYPE_BF16,
                                       (cudaStream_t)stream);
    return e == cudaSuccess ? PP_STATUS_OK : cuda_fail(e, "rms_norm launch");
}

int32_t pp_b200_renyi_sample(const float* raw, const float* uniforms, const uint32_t* bounds, uint32_t* out,
                             uint32_t batch, uint32_t choices, uint32_t guidance, float alpha, float cfg,
                             uint32_t token_offset, void* stream) {
    int32_t s;
    // the checks of fused_sampling.rs:17-67 `validate`
    if ((guidance != 1 && guidance != 2) || batch == 0 || choices == 0 || choices > 2048)
        return fail(PP_STATUS_PRECONDITION,
                    "fused sampler needs 1/2 guidance rows and a nonempty head of at most 2048 choices");
    if (batch > 0x7fffffffu) return fail(PP_STATUS_PRECONDITION, "fused sampler logical row, uniform or bounds shape mismatch");
    if (!std::isfinite(alpha) || alpha <= 1.f || !std::isfinite(cfg) || cfg < 0.f || (guidance == 1 && cfg != 1.f))
        return fail(PP_STATUS_PRECONDITION, "invalid fused sampler alpha/CFG/guidance combination");
    if ((uint64_t)token_offset + (choices - 1) > 0xffffffffull) return fail(PP_STATUS_PRECONDITION, "fused token range overflow");
    if (!raw || !uniforms || !bounds || !out) return fail(PP_STATUS_PRECONDITION, "fused sampler: NULL pointer");
    if (!aligned(raw, 4) || !aligned(uniforms, 4) || !aligned(bounds, 4) || !aligned(out, 4))
        return fail(PP_STATUS_PRECONDITION, "fused sampler inputs must be 4-byte aligned");
    DeviceInfo d;
    if ((s = device_info(d))) return s;
    cudaError_t e = pp::launch_renyi_sample(raw, uniforms, bounds, out, batch, choices, guidance, alpha, cfg,
                                            token_offset, (cudaStream_t)stream);
    return e == cudaSuccess ? PP_STATUS_OK : cuda_fail(e, "fused sampler launch");
}

const char* pp_b200_status_message(uint32_t bits) {
    if (bits == 0) return "ok";
    if (bits & PP_DEV_WAIT_TIMEOUT) return "EXECUTION_UNCERTAIN: a bounded device pipeline wait timed out";
    if (bits & PP_DEV_NONFINITE_INPUT) return "non-finite INT8 KV input";
    if (bits & PP_DEV_OFFSET_RANGE) return "batch KV needs context rebuild: append offset outside capacity";
    if (bits & PP_DEV_LENGTH_RANGE) return "INT8 attention lengths differ: length exceeds capacity (row output is NaN)";
    if (bits & PP_DEV_POSITION_RANGE) return "graph QKV/RoPE position exceeds the RoPE table (row not written)";
    return "unknown device status";
}


int32_t pp_b200_diag_bounded_wait(uint32_t* status, uint32_t limit_us, void* stream) {
    if (!status || limit_us == 0 || limit_us > 1000000)
        return fail(PP_STATUS_PRECONDITION, "diag_bounded_wait: status pointer and a limit of 1..1000000 us required");
    DeviceInfo d;
    int32_t s;
    if ((s = device_info(d))) return s;
    cudaError_t e = pp::launch_wait_probe(status, (uint64_t)limit_us * 1000ull, (cudaStream_t)stream);
    return e == cudaSuccess ? PP_STATUS_OK : cuda_fail(e, "diag_bounded_wait launch");
}

}  // extern "C"
