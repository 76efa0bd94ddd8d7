// Internal declarations shared by the kernels and the C ABI implementation.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../../include/pp_b200.h"

namespace pp {

// ----------------------------------------------------------- attention plan
//
// Workspace layout (all offsets from the workspace base, 256-byte aligned):
//   PlanHeader                                    @ 0
//   row_len   u32 [rows]      history tokens per row, kInvalidRow if invalid
//   row_seg   u32 [rows + 1]  first segment of each row (segments are row-sorted)
//   cta_seg   u32 [max_ctas + 1]  first segment of each CTA
//   segs      SegDesc [max_segs]
//   partials  f32 [max_segs][head_dim + 4]   acc[0..D), m (log2 units), z
//   row_cnt   u32 [rows]      finished segments per row (zero between calls)
//   orphans   u32 [rows]      rows without segments (invalid, or reference
//                             mode with no history: only the scratch token)
// A segment is a contiguous token range of one row processed by one CTA and
// producing one partial (m, z, acc) for the log-sum-exp combine.  With
// stream-K segments the attention kernel also finishes the rows: a row held
// by one segment is normalised in place, and of a row split over several
// CTAs the CTA that completes it last (row_cnt) merges the partials.  Fixed
// splits leave the merge to the combine kernel.

constexpr uint32_t kInvalidRow = 0xffffffffu;

struct PlanHeader {
    unsigned long long total_tokens;
    unsigned long long tokens_per_cta;
    uint32_t n_segs;
    uint32_t n_ctas;
    uint32_t rows;
    uint32_t heads;
    uint32_t capacity;
    uint32_t split;
    uint32_t scratch;
    uint32_t max_segs;
    uint32_t max_ctas;
    uint32_t n_orphans;
    uint32_t pad[2];
};

struct SegDesc {
    uint32_t row, t0, t1, row_segs;  // row_segs: segments of this row
};

struct WsLayout {
    size_t row_len, row_seg, cta_seg, segs, partials, row_cnt, orphans, total;
    uint32_t max_segs, max_ctas;
};

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Stream-K segments: at most one per row plus one per CTA boundary.
// Fixed split: at most ceil(capacity / split) per row.
inline WsLayout ws_layout(uint32_t rows, uint32_t capacity, uint32_t head_dim, uint32_t split, uint32_t max_ctas) {
    WsLayout l{};
    l.max_ctas = max_ctas;
    uint64_t segs = split ? (uint64_t)rows * ((capacity + split - 1) / split) : (uint64_t)rows + max_ctas;
    if (segs == 0) segs = 1;
    l.max_segs = (uint32_t)(segs > 0xffffffffull ? 0xffffffffull : segs);
    size_t off = align_up(sizeof(PlanHeader), 256);
    l.row_len = off;
    off = align_up(off + 4ull * rows, 256);
    l.row_seg = off;
    off = align_up(off + 4ull * (rows + 1), 256);
    l.cta_seg = off;
    off = align_up(off + 4ull * (max_ctas + 1), 256);
    l.segs = off;
    off = align_up(off + sizeof(SegDesc) * (size_t)l.max_segs, 256);
    l.partials = off;
    off = align_up(off + 4ull * (head_dim + 4) * (size_t)l.max_segs, 256);
    l.row_cnt = off;
    off = align_up(off + 4ull * rows, 256);
    l.orphans = off;
    off = align_up(off + 4ull * rows, 256);
    l.total = off;
    return l;
}

// Element type of the attended K/V (internal codes, not PP_DTYPE_*).
constexpr int kKvInt8 = 0, kKvBf16 = 1, kKvF32 = 2;

// Tensor maps for segment tails: the same K / V boxes of 16, 32, 64, 128 and
// 256 tokens, so that a tail of n tokens takes at most 5 copies per tensor.
constexpr int kTailBoxes = 5;
struct TailMaps {
    CUtensorMap k[kTailBoxes], v[kTailBoxes];
};

struct AttnLaunch {
    // int8 arena geometry; for float K/V, capacity is the key length (size)
    // and k/v/k_scale/v_scale are unused
    PpKvArena arena;
    int kv_kind;        // kKvInt8, kKvBf16 or kKvF32
    uint64_t q_stride;  // elements between q rows (head_dim for the int8 entry points)
    uint32_t split;
    int q_dtype, out_dtype;
    float scale_log2;     // softmax scale * log2(e)
    uint32_t max_ctas;    // grid of the attention kernel
    uint32_t num_sms;
    const void* q;
    const float* scratch_k;
    const float* scratch_v;
    const uint32_t* lengths;
    void* out;
    unsigned char* ws;
    WsLayout layout;
    uint32_t* status;
    bool plan_ready;
    bool prefetch;  // PP_ATTN_PREFETCH_HISTORY
    bool use_pdl;
    bool short_stages;  // int8 head_dim 64 with few tokens per CTA: the 12-warp, 384-token-stage kernel
    // Tensor maps (host-encoded): K, V codes in whole-stage boxes and in the
    // tail boxes, and K, V scales (int8 only).  Float K/V maps are 3-D
    // {channel, token, row} with one 128-byte panel per box.
    TailMaps tails;
    CUtensorMap map_k_stage, map_v_stage, map_ks, map_vs;
    uint32_t ks_mis, vs_mis;  // element offset of the scale arrays inside their maps
};

// QKV RoPE (+ int8 append): see decoder.cu.
struct QkvRopeLaunch {
    const void* qkv;
    const void* params;
    const uint32_t* positions;
    uint32_t rows, heads, head_dim, max_context;
    bool bf16;
    void* out;  // plain: the three planes; fused: q
    float* scratch_k;
    float* scratch_v;
    const PpKvArena* arena;  // NULL: plain
    const uint32_t* offsets;
    uint32_t commit;
    uint32_t* status;
};

cudaError_t launch_qkv_rope(const QkvRopeLaunch& L, cudaStream_t stream);
cudaError_t launch_swiglu(const void* in, void* out, uint64_t rows, uint32_t hidden, bool bf, cudaStream_t stream);
cudaError_t launch_rmsnorm(const void* x, const void* residual, void* x_sum, const void* weight, void* out,
                           uint64_t rows, uint32_t width, float eps, bool bf, cudaStream_t stream);
cudaError_t launch_renyi_sample(const float* raw, const float* uniforms, const uint32_t* bounds, uint32_t* out,
                                uint32_t batch, uint32_t choices, uint32_t guidance, float alpha, float cfg,
                                uint32_t token_offset, cudaStream_t stream);
cudaError_t launch_quantize(const void* x, int dtype, uint64_t rows, uint32_t d, uint8_t* packed, float* scales,
                            uint32_t* status, cudaStream_t stream);
cudaError_t launch_quant_append(const PpKvArena& a, const void* k_new, const void* v_new, int dtype,
                                const uint32_t* offsets, uint32_t commit, uint32_t* status, cudaStream_t stream);
cudaError_t launch_dequantize(const uint8_t* packed, const float* scales, uint64_t rows, uint32_t d, int round_bf16,
                              int out_dtype, void* out, cudaStream_t stream);
cudaError_t launch_copy_prefix(const PpKvArena& s, const PpKvArena& d, const uint32_t* lengths, uint32_t* status,
                               cudaStream_t stream);
cudaError_t launch_plan(const AttnLaunch& L, cudaStream_t stream);
cudaError_t launch_attention(const AttnLaunch& L, cudaStream_t stream);
cudaError_t launch_combine(const AttnLaunch& L, cudaStream_t stream);
cudaError_t configure_attention_kernels(int device);
uint32_t attention_scale_box_elems();
bool attention_short_stages(uint32_t head_dim, uint32_t rows, uint32_t capacity, uint32_t ctas);
uint32_t attention_stage_tokens(uint32_t head_dim, bool short_stages);
uint32_t attention_float_stage_tokens(uint32_t head_dim, int kv_kind);
cudaError_t launch_wait_probe(uint32_t* status, uint64_t limit_ns, cudaStream_t stream);
cudaError_t launch_lane_uniforms(const uint64_t* seeds, uint64_t* draws, const uint32_t* active, uint32_t rows,
                                 float* out, cudaStream_t stream);

// Records `msg` as the calling thread's last error and returns `status`.
int32_t fail_msg(int32_t status, const char* msg);

// The unique ID of the calling thread's current CUDA context (the primary
// context is made current if none is).  Per-context state (kernel attributes,
// module symbol addresses) is cached against it: an ID that changed means the
// context was made anew and that state must be set up again.
int32_t current_context_id(unsigned long long* id);

}  // namespace pp
