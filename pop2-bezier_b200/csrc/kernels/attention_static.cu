// Decode attention without any device allocation by the library or the caller.
//
// pp_b200_decode_attention needs a workspace (the split plan and the split-K
// partials) that the caller allocates.  Some callers cannot allocate device
// memory at the point where they call attention: a host that only hands a
// plugin its input and output buffers and keeps its allocator private, a
// serving loop that forbids cudaMalloc after start-up because the call
// synchronises the device and stalls every stream, or code that must not
// allocate while other work is being recorded.  For them this entry point
// takes the same arguments minus the workspace and uses the fixed scratch
// array below instead.
#include <cstdio>
#include <mutex>

#include "../host/internal.h"

namespace {

// Scratch for pp_b200_decode_attention_static.  Every GPU that loads this
// library holds these bytes until the process exits.
constexpr size_t kStaticWorkspaceBytes = size_t(4) << 20;  // 4 MiB
__device__ __align__(256) unsigned char g_static_workspace[kStaticWorkspaceBytes];

std::mutex g_static_mu;
struct StaticAddress {
    void* ptr = nullptr;
    unsigned long long ctx_id = 0;  // the context the address was looked up in
};
StaticAddress g_static_addr[64];  // device address of g_static_workspace, per device

// Looks up the array's device address (host code must not use the symbol
// itself as a device pointer).  The address belongs to the context that loaded
// the module: it is looked up once per context, and again when the device's
// context was made anew (after cudaDeviceReset, or a released and re-created
// primary context), when the module may have been loaded elsewhere.
int32_t static_workspace(void** out, void* stream) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return pp::fail_msg(PP_STATUS_UNCERTAIN, "EXECUTION_UNCERTAIN: cudaGetDevice failed in decode_attention_static");
    if (dev < 0 || dev >= 64) return pp::fail_msg(PP_STATUS_PRECONDITION, "decode_attention_static: device ordinal out of range");
    unsigned long long ctx = 0;
    const int32_t s = pp::current_context_id(&ctx);
    if (s != PP_STATUS_OK) return s;
    std::lock_guard<std::mutex> lock(g_static_mu);
    StaticAddress& a = g_static_addr[dev];
    if (!a.ptr || a.ctx_id != ctx) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_workspace);
        if (e != cudaSuccess || !p) {
            cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
            const bool capturing = cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &cap) == cudaSuccess &&
                                   cap != cudaStreamCaptureStatusNone;
            char msg[320];
            snprintf(msg, sizeof msg, "decode_attention_static: cudaGetSymbolAddress failed: %s%s", cudaGetErrorName(e),
                     capturing ? " (the stream is being captured: make the first call on this device, and the first "
                                 "after a context reset, before any capture)"
                               : "");
            return pp::fail_msg(PP_STATUS_PRECONDITION, msg);
        }
        a.ptr = p;
        a.ctx_id = ctx;
    }
    *out = a.ptr;
    return PP_STATUS_OK;
}

}  // namespace

extern "C" int32_t pp_b200_decode_attention_static(const PpKvArena* arena, const PpAttnParams* params, const void* q,
                                                   const float* scratch_k, const float* scratch_v,
                                                   const uint32_t* lengths, void* out, uint32_t* status,
                                                   void* stream) {
    if (params && params->struct_size >= sizeof(uint32_t) * 6 && (params->flags & PP_ATTN_PLAN_READY))
        return pp::fail_msg(PP_STATUS_PRECONDITION,
                            "decode_attention_static: PP_ATTN_PLAN_READY needs a caller-owned workspace "
                            "(the shared scratch is re-planned on every call)");
    const size_t need = pp_b200_attention_workspace_size(arena, params);
    if (need == 0)
        return pp::fail_msg(PP_STATUS_PRECONDITION, "INT8 attention geometry differs: invalid arena for decode_attention_static");
    if (need > kStaticWorkspaceBytes) {
        char msg[256];
        snprintf(msg, sizeof msg,
                 "decode_attention_static: this geometry needs %zu workspace bytes, more than the %zu-byte static "
                 "scratch; use pp_b200_decode_attention with a caller workspace",
                 need, kStaticWorkspaceBytes);
        return pp::fail_msg(PP_STATUS_PRECONDITION, msg);
    }
    void* ws = nullptr;
    const int32_t s = static_workspace(&ws, stream);
    if (s != PP_STATUS_OK) return s;
    return pp_b200_decode_attention(arena, params, q, scratch_k, scratch_v, lengths, out, ws, kStaticWorkspaceBytes,
                                    status, stream);
}
