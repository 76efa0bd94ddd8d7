/*
 * pp_b200.h -- C ABI of the B200 int8 historical-KV decode engine.
 *
 * This is the drop-in boundary for the reference's `int8_kv_ops` module
 * (app/src/model/int8_kv_ops.rs), whose CUDA branches are Candle CustomOps
 * launched through cudarc.  A Rust `extern "C"` crate binds these entry points
 * in place of those CustomOps.
 *
 * Conventions (style of app/native/aten_hip/cpp/painter_ffi.h:20-25):
 *   - every entry point returns an int32 status:
 *       PP_STATUS_OK (0)             success
 *       PP_STATUS_PRECONDITION (1)   invalid geometry/argument: nothing was launched
 *       PP_STATUS_INVALID_OUTPUT (2) the class a caller reports when the device status word
 *                                    (PP_DEV_* bits below, text from pp_b200_status_message)
 *                                    is non-zero after the stream completes; kernels cannot
 *                                    return it, so no entry point does
 *       PP_STATUS_UNCERTAIN (3)      a CUDA launch/runtime error: device state uncertain,
 *                                    the caller must discard the KV state (reload)
 *   - pp_b200_last_error() returns a thread-local UTF-8 message for the last
 *     non-OK status on the calling thread.  Messages carry the reference's
 *     classifiable tokens (e.g. "CUDA_ERROR_OUT_OF_MEMORY", "EXECUTION_UNCERTAIN")
 *     so app/src/inference.rs:34-92 keeps classifying them.
 *   - all data pointers are caller-owned device memory; the library never
 *     allocates device memory on the decode path (the workspace is supplied).
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *   - all geometry is validated on the host before anything is launched.
 *   - entry points are reentrant per stream; the only global state is a
 *     per-device cache of device properties and kernel attributes.
 */
#ifndef PP_B200_H
#define PP_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PP_B200_ABI_VERSION 1u

#define PP_STATUS_OK 0
#define PP_STATUS_PRECONDITION 1
#define PP_STATUS_INVALID_OUTPUT 2
#define PP_STATUS_UNCERTAIN 3

/* Element types of floating inputs/outputs. */
#define PP_DTYPE_F32 0
#define PP_DTYPE_BF16 1

/* Bits a kernel may set in a caller-supplied device status word (uint32). */
#define PP_DEV_NONFINITE_INPUT 0x1u  /* quantize saw a NaN/Inf (int8_kv_ops.rs:16) */
#define PP_DEV_OFFSET_RANGE 0x2u     /* append offset >= capacity: row not written */
#define PP_DEV_LENGTH_RANGE 0x4u     /* attention length > capacity: row output is NaN */
#define PP_DEV_WAIT_TIMEOUT 0x8u     /* a bounded pipeline wait gave up: output undefined */
#define PP_DEV_POSITION_RANGE 0x10u  /* RoPE position >= max_context: row not written */

/* Geometry of a caller-owned int8 KV arena for one layer, in the reference's
 * batch-arena layout (app/src/model/cache.rs:301-478, int8_cache.rs:326-359):
 *   k, v       u8  [rows, capacity, head_dim]   (signed int8 codes)
 *   k_scale,
 *   v_scale    f32 [rows, capacity]             (one scale per token and head)
 * Row r = branch * heads + head.  k and v must be 16-byte aligned; scales
 * need only 4-byte alignment (views at any row offset are accepted). */
typedef struct PpKvArena {
    uint32_t struct_size; /* sizeof(PpKvArena) */
    uint32_t rows;        /* physical head rows = branches * heads */
    uint32_t heads;       /* heads per branch (rows % heads == 0) */
    uint32_t head_dim;    /* 64 or 128 */
    uint32_t capacity;    /* token slots per row */
    uint32_t reserved;
    uint8_t* k;
    uint8_t* v;
    float* k_scale;
    float* v_scale;
} PpKvArena;

/* Attention options. */
typedef struct PpAttnParams {
    uint32_t struct_size;   /* sizeof(PpAttnParams) */
    uint32_t split_tokens;  /* 0: automatic: equal tokens per SM (stream-K), or
                               whole rows per CTA when the rows are of one
                               length and that costs little more; split rows
                               are merged inside the attention kernel;
                               else: fixed split size in tokens (the reference's
                               split_tokens, int8_kv_ops.rs:52) */
    int32_t q_dtype;        /* PP_DTYPE_F32 or PP_DTYPE_BF16, q is [rows, head_dim] */
    int32_t out_dtype;      /* PP_DTYPE_F32 or PP_DTYPE_BF16, out is [rows, head_dim] */
    float softmax_scale;    /* 0: 0.125 at head_dim 64 (int8_kv.cu:40), f32(1/sqrt(d)) otherwise */
    uint32_t flags;         /* PP_ATTN_* */
    uint32_t max_ctas;      /* 0: one CTA per SM */
    uint32_t reserved;
} PpAttnParams;

/* The workspace already holds the plan made by pp_b200_plan_ragged for the
 * same arena geometry, params and lengths (reuse across layers and queries,
 * as DecodeMetadataCache does, app/src/model/decode_metadata.rs:39-142). */
#define PP_ATTN_PLAN_READY 0x1u

/* With PP_ATTN_PLAN_READY: the kernel enqueued just before this call on the
 * stream writes neither this arena's history (the tokens attended from it)
 * nor the workspace plan; for instance another layer's attention, or
 * pp_b200_qkv_rope_append in reference mode (it writes slot `past`, after the
 * history).  The attention then starts streaming history while that kernel
 * finishes (programmatic dependent launch) and waits for it only before
 * reading q, the scratch token or anything else it may have written. */
#define PP_ATTN_PREFETCH_HISTORY 0x2u

uint32_t pp_b200_abi_version(void);
const char* pp_b200_last_error(void);

/* Symmetric per-(token, head) int8 quantization of `rows` vectors of
 * head_dim elements: replaces int8_kv_ops::quantize (int8_kv_ops.rs:11-29,
 * kernels pp_i8_scale + pp_i8_pack, int8_kv.cu:8-18).
 * x: f32/bf16 [rows, head_dim]; packed: u8 [rows, head_dim]; scales: f32 [rows].
 * status (nullable, device uint32): PP_DEV_NONFINITE_INPUT is OR-ed in when
 * an input element is not finite. */
int32_t pp_b200_quantize(const void* x, int32_t x_dtype, uint64_t rows, uint32_t head_dim,
                         uint8_t* packed, float* scales, uint32_t* status, void* stream);

/* Dequantization: replaces int8_kv_ops::dequantize (int8_kv_ops.rs:30-40,
 * kernel pp_i8_unpack int8_kv.cu:19-22).  out = (i8) packed * scale[row],
 * rounded to bf16 first when round_bf16 != 0 (the `to_dtype(BF16)` of
 * int8_cache.rs:368), written as out_dtype. */
int32_t pp_b200_dequantize(const uint8_t* packed, const float* scales, uint64_t rows,
                           uint32_t head_dim, int32_t round_bf16, int32_t out_dtype, void* out,
                           void* stream);

/* Quantize-and-append one new K/V token per row: replaces the commit branch of
 * Int8LayerCache::encoded (int8_cache.rs:293-312) plus the arena writes of
 * LayerCache::query_batch_with_plan (cache.rs:415-459, slice_set / scatter_set).
 * k_new, v_new: f32/bf16 [rows, head_dim].  offsets: device u32 [rows/heads],
 * the per-branch write slot (the past length).  commit=0 writes the partial
 * query placeholder (zero codes, scale 1.0, int8_cache.rs:305-310) instead.
 * status (nullable): PP_DEV_NONFINITE_INPUT, PP_DEV_OFFSET_RANGE. */
int32_t pp_b200_quant_append(const PpKvArena* arena, const void* k_new, const void* v_new,
                             int32_t dtype, const uint32_t* offsets, uint32_t commit,
                             uint32_t* status, void* stream);

/* Copies each row's committed prefix from one arena to another of larger
 * capacity: the growth/COW copy of LayerCache::query (cache.rs:246-266) and the
 * batch-row adoption copy (cache.rs:393-414).  lengths: device u32 [rows/heads]. */
int32_t pp_b200_copy_prefix(const PpKvArena* src, const PpKvArena* dst, const uint32_t* lengths,
                            void* stream);

/* Workspace bytes pp_b200_decode_attention / pp_b200_plan_ragged need for this
 * geometry (an upper bound independent of the device-resident lengths). */
size_t pp_b200_attention_workspace_size(const PpKvArena* arena, const PpAttnParams* params);

/* Ragged bookkeeping: turns device-resident per-branch lengths into the split
 * work list the attention kernel consumes, inside `workspace`.  Restates the
 * per-row geometry of BatchWritePlan / DecodeMetadataCache
 * (write_plan.rs:48-93, decode_metadata.rs:107-125) as device tables.
 * scratch_token != 0 selects the reference mode of pp_b200_decode_attention. */
int32_t pp_b200_plan_ragged(const PpKvArena* arena, const PpAttnParams* params,
                            const uint32_t* lengths, uint32_t scratch_token, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Fused int8 decode attention (dequant -> QK^T -> softmax -> PV, split-K with
 * a log-sum-exp combine): replaces int8_kv_ops::attention (int8_kv_ops.rs:42-55,
 * kernels pp_i8_attention + pp_i8_merge, int8_kv.cu:28-59).
 *   q        [rows, head_dim] (params->q_dtype)
 *   lengths  device u32 [rows/heads]
 *   scratch_k, scratch_v: f32 [rows, head_dim] or both NULL.
 *     non-NULL (reference mode): a row attends to lengths[b] int8 history
 *       tokens plus the f32 scratch token; lengths[b] > capacity gives NaN.
 *     NULL (history mode): a row attends to lengths[b] int8 tokens;
 *       0 or > capacity gives NaN.
 *   out      [rows, head_dim] (params->out_dtype)
 * History values are dequantized exactly as pp_i8_load does: bf16(i8 * scale).
 * status (nullable): PP_DEV_LENGTH_RANGE, PP_DEV_WAIT_TIMEOUT. */
int32_t pp_b200_decode_attention(const PpKvArena* arena, const PpAttnParams* params,
                                 const void* q, const float* scratch_k, const float* scratch_v,
                                 const uint32_t* lengths, void* out, void* workspace,
                                 size_t workspace_bytes, uint32_t* status, void* stream);

/* pp_b200_decode_attention for callers that cannot allocate device memory
 * when they call attention (a host that passes a plugin only its input and
 * output buffers, a serving loop that forbids cudaMalloc after start-up).
 * No counterpart in the reference: its CustomOp allocates per call.
 * Same arguments and results as pp_b200_decode_attention, without the
 * workspace: the plan and split-K partials live in a 4 MiB scratch array
 * compiled into the library, which every GPU that loads the library keeps
 * until the process exits.  Geometries whose workspace
 * (pp_b200_attention_workspace_size) exceeds 4 MiB are rejected with
 * PP_STATUS_PRECONDITION; PP_ATTN_PLAN_READY is rejected (the scratch is
 * re-planned on every call).  Nothing in the scratch needs to start at zero.
 * All calls share the one array: calls that may run at the same time on the
 * GPU (different streams, or several host threads) race and must be
 * serialised by the caller.  The first call on each device looks up the
 * array's device address; make that first call before any stream capture.
 * The address is looked up again, by the next call, when the device's
 * context has been made anew (after cudaDeviceReset): that call too must come
 * before any capture.
 * Nothing is allocated: no cudaMalloc, cudaFree or allocating library call. */
int32_t pp_b200_decode_attention_static(const PpKvArena* arena, const PpAttnParams* params, const void* q,
                                        const float* scratch_k, const float* scratch_v,
                                        const uint32_t* lengths, void* out, uint32_t* status, void* stream);

/* Float K/V rows for the float-KV fused decode attention, in the layout the
 * reference's decode_attention requires (fused_attention.rs:12-23: dense
 * width and token strides):
 *   k, v  [rows, tokens, head_dim] of dtype (f32 or bf16); token stride
 *         head_dim elements, row strides k_row_stride / v_row_stride elements
 * Row r = branch * heads + head.  k and v must be 16-byte aligned and the
 * row strides multiples of 16 bytes (the tensor copies' rule); a view of a
 * larger cache (row stride = capacity * head_dim) is accepted as is. */
typedef struct PpFloatKv {
    uint32_t struct_size; /* sizeof(PpFloatKv) */
    uint32_t rows;        /* physical head rows = branches * heads */
    uint32_t heads;       /* heads per branch (rows % heads == 0) */
    uint32_t head_dim;    /* 64 or 128 */
    uint32_t tokens;      /* key length of every row (the reference's `length` dim) */
    int32_t dtype;        /* PP_DTYPE_F32 or PP_DTYPE_BF16, both K and V */
    uint64_t k_row_stride;
    uint64_t v_row_stride;
    const void* k;
    const void* v;
} PpFloatKv;

/* Workspace bytes pp_b200_decode_attention_float / pp_b200_plan_ragged_float
 * need for this geometry. */
size_t pp_b200_float_attention_workspace_size(const PpFloatKv* kv, const PpAttnParams* params);

/* The ragged plan of pp_b200_plan_ragged for float K/V: lengths (device u32
 * [rows/heads], or NULL for every row attending to all `tokens`) become the
 * split work list in `workspace`, reusable across layers with
 * PP_ATTN_PLAN_READY. */
int32_t pp_b200_plan_ragged_float(const PpFloatKv* kv, const PpAttnParams* params, const uint32_t* lengths,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* Fused float-KV decode attention (QK^T -> softmax -> PV, split-K with a
 * log-sum-exp combine): replaces fused_attention::decode_attention
 * (fused_attention.rs:8-83, kernels pp_attention_f32 / pp_attention_bf16 /
 * pp_attention_merge, decode_attention.cu:7-59).
 *   q        [rows, head_dim] (params->q_dtype) with row stride q_row_stride
 *            elements (16-byte aligned rows)
 *   lengths  device u32 [rows/heads], or NULL: row r attends to its first
 *            lengths[r / heads] tokens; 0 or > tokens gives NaN (the
 *            reference's `valid`, decode_attention.cu:14)
 *   out      [rows, head_dim] (params->out_dtype), dense
 * Scale 0.125 at head_dim 64 as the reference, f32(1/sqrt(d)) otherwise,
 * unless params->softmax_scale is set.  params->split_tokens 0 selects the
 * stream-K plan (balanced over all SMs whatever the raggedness; the reference
 * keeps each row whole in one CTA); otherwise rows are cut into fixed splits
 * of clamp(split_tokens, 32, 1024) tokens as fused_attention.rs:29 does.
 * status (nullable): PP_DEV_LENGTH_RANGE, PP_DEV_WAIT_TIMEOUT. */
int32_t pp_b200_decode_attention_float(const PpFloatKv* kv, const PpAttnParams* params, const void* q,
                                       uint64_t q_row_stride, const uint32_t* lengths, void* out, void* workspace,
                                       size_t workspace_bytes, uint32_t* status, void* stream);

/* Diagnostic: runs one bounded wait on a barrier that nothing completes, with
 * the library's wait loop and a limit of limit_us microseconds (1..10^6), so a
 * host can confirm on its device that a stalled pipeline ends with
 * PP_DEV_WAIT_TIMEOUT OR-ed into *status (device memory) and a usable context
 * instead of a hang.  No counterpart in the reference. */
int32_t pp_b200_diag_bounded_wait(uint32_t* status, uint32_t limit_us, void* stream);

/* Decodes device status bits into a message (static storage). */
const char* pp_b200_status_message(uint32_t status_bits);

/* Physical batch rows with the reference's overflow rules:
 * checked_batch_rows (app/src/model/batch_geometry.rs:4-16). */
int32_t pp_b200_checked_batch_rows(uint64_t logical_rows, uint32_t guidance,
                                   uint64_t* physical_rows);

/* Host-side write-plan validation: checked_shape (write_plan.rs:27-45) with
 * the arena capacity in place of MAX_CONTEXT (offsets must leave a slot). */
int32_t pp_b200_check_write_offsets(const uint64_t* past_lens, uint64_t count, uint32_t heads,
                                    uint32_t head_dim, uint32_t capacity);

/* Branch scheduler: deterministic longest-processing-time partition of
 * independent branches across shards (GPUs).  cost[i] is branch i's KV work
 * (its context length); shard_of_branch[i] receives its shard and
 * shard_cost[s] the total per shard.  Branches are the independent lanes of
 * NativeEngine::generate_parallel (app/src/inference/batch.rs:241-558), which
 * the reference runs on one device. */
int32_t pp_b200_sched_partition(const uint64_t* cost, uint32_t n_branches, uint32_t n_shards,
                                uint32_t* shard_of_branch, uint64_t* shard_cost);

/* parallel_seed (app/src/inference/batch.rs:9-11): the seed of lane `lane`
 * of a parallel generation seeded `base` is base + lane (wrapping). */
uint64_t pp_b200_sched_lane_seed(uint64_t base, uint64_t lane);

/* Draw `draw` (from 0) of the lane stream seeded `lane_seed`: the draw-th
 * output of a SplitMix64 generator seeded lane_seed, top 24 bits / 2^24, a
 * float in [0, 1).  The host form of pp_b200_sched_uniforms, bit for bit.
 * Replaces the per-lane StdRng draws of device::draw_uniforms
 * (app/src/inference/batch.rs:747-754) with a counter-based stream, so a
 * lane draws the same values whichever shard or batch row it occupies. */
float pp_b200_sched_uniform(uint64_t lane_seed, uint64_t draw);

/* One sampling uniform per batch row on the device: for rows with
 * active[r] != 0, out[r] = pp_b200_sched_uniform(lane_seeds[r], draws[r]) and
 * draws[r] += 1; inactive rows get 0 and keep their counter (a retired lane
 * draws nothing, as the reference draws only for ready lanes).
 * lane_seeds, draws: device u64 [rows]; active: device u32 [rows]; out:
 * device f32 [rows]. */
int32_t pp_b200_sched_uniforms(const uint64_t* lane_seeds, uint64_t* draws, const uint32_t* active, uint32_t rows,
                               float* out, void* stream);

/* ---- decoder step around the int8 KV path (graph_ops.cu / batch.rs) ---- */

/* Geometry of a QKV projection output: rows (batch rows) x [q | k | v], each
 * heads * head_dim wide, head_dim 64 or 128; dtype PP_DTYPE_BF16 or F32. */
typedef struct PpQkvRope {
    uint32_t struct_size;  /* sizeof(PpQkvRope) */
    uint32_t rows;
    uint32_t heads;
    uint32_t head_dim;
    uint32_t max_context;  /* rows of the cos / sin tables */
    int32_t dtype;
    uint32_t reserved[2];
} PpQkvRope;

/* q/k RMSNorm (eps 1e-6, per-head weights) and interleaved RoPE: replaces
 * graph_ops::qkv, kernel pp_graph_qkv (app/src/model/graph_ops.rs:144-174,
 * graph_ops.cu:34-59), with its rounding points, generalised to head_dim 128
 * and any max_context.  qkv: [rows, 3*heads*head_dim]; params:
 * [q_norm head_dim | k_norm head_dim | cos max_context*head_dim/2 |
 * sin max_context*head_dim/2] (the reference's qk_rope_parameters);
 * positions: device u32 [rows]; out: [3][rows*heads][head_dim] (q, k, v).
 * status (nullable): PP_DEV_POSITION_RANGE (row not written). */
int32_t pp_b200_qkv_rope(const PpQkvRope* geometry, const void* qkv, const void* params,
                         const uint32_t* positions, void* out, uint32_t* status, void* stream);

/* The same, fused with what the int8 decode path does next (batch.rs:143-155,
 * int8_cache.rs:326-359): the rotated k and the v of each (row, head) are
 * quantized and appended to `arena` at slot offsets[row] (commit = 0 writes
 * the partial-query placeholder), q is written as [rows*heads, head_dim] in
 * the model dtype, and k / v as the f32 scratch [rows*heads, head_dim] that
 * pp_b200_decode_attention reads in reference mode.  arena: heads and
 * head_dim as the geometry, arena rows = rows * heads.  status (nullable):
 * PP_DEV_POSITION_RANGE, PP_DEV_OFFSET_RANGE, PP_DEV_NONFINITE_INPUT. */
int32_t pp_b200_qkv_rope_append(const PpQkvRope* geometry, const void* qkv, const void* params,
                                const uint32_t* positions, const PpKvArena* arena,
                                const uint32_t* offsets, uint32_t commit, void* q_out,
                                float* scratch_k, float* scratch_v, uint32_t* status, void* stream);

/* SwiGLU: out[r, c] = silu(gate[r, c]) * up[r, c] over in = [rows, 2*hidden]
 * (gate | up), with the reference's rounding of exp, sum and quotient:
 * graph_ops::swiglu, kernel pp_graph_swiglu (graph_ops.rs:175-193,
 * graph_ops.cu:60-74).  dtype PP_DTYPE_BF16 or F32. */
int32_t pp_b200_swiglu(const void* in, void* out, uint64_t rows, uint32_t hidden, int32_t dtype,
                       void* stream);

/* RMSNorm of [rows, width]: out = x * rsqrt(mean(x^2) + eps) * weight, the
 * candle_nn::ops::rms_norm of PrimitiveModel (mod.rs:671,729,746, batch.rs:132).
 * With residual != NULL, x is first replaced by round(x + residual) (the
 * residual adds of mod.rs:722,744), which is also written to x_sum when
 * x_sum != NULL.  dtype PP_DTYPE_BF16 or F32. */
int32_t pp_b200_rmsnorm(const void* x, const void* residual, void* x_sum, const void* weight,
                        void* out, uint64_t rows, uint32_t width, float eps, int32_t dtype,
                        void* stream);

/* Rényi-entropy truncated sampling with classifier-free guidance, one logical
 * row per block: replaces fused_sampling::sample, kernel pp_renyi_sample
 * (app/src/inference/fused_sampling.rs:69-90, renyi_sample.cu), with its
 * checks and its results.  raw: f32 [batch * guidance, choices] (guidance 2:
 * conditional then unconditional row); uniforms: f32 [batch] in [0, 1);
 * bounds: u32 [batch, 2] = (start, count) of the legal window; out: u32
 * [3, batch] = (token_offset + column, 1 or 0 for the fallback, support). */
int32_t pp_b200_renyi_sample(const float* raw, const float* uniforms, const uint32_t* bounds, uint32_t* out,
                             uint32_t batch, uint32_t choices, uint32_t guidance, float alpha, float cfg,
                             uint32_t token_offset, void* stream);

/* On-device self-check run before int8 caches are created: replaces
 * int8_kv_ops::prepare (int8_kv_ops.rs:57-103) and is called where
 * PrimitiveModel::prepare_int8_kv calls it (int8_policy.rs:29-56).  Runs the
 * reference's own fixtures (quantize round trip within 0.009, attention within
 * 2e-5 of scalar host loops, offsets/splits {32,128}) on `device`. */
int32_t pp_b200_prepare(int32_t device);

/* On-device check that gates the optional fused decode kernels: replaces
 * PrimitiveModel::prepare_optional_kernels (app/src/model/mod.rs:440-460).
 * With split_k or fusion set, runs pp_b200_decode_attention_float on zero
 * q [1,1,head_width] f32 and zero K/V [1,257,head_width] of model_dtype
 * (split_tokens 128 with split_k, else 0) and, with fusion, pp_b200_swiglu on a
 * zero [1, 2*ffn_hidden] gate; every output must be finite and within 1e-6 of
 * zero.  Fails with the reference's messages (PP_STATUS_PRECONDITION). */
int32_t pp_b200_prepare_optional(int32_t device, uint32_t fusion, uint32_t split_k, int32_t model_dtype,
                                 uint32_t head_width, uint32_t ffn_hidden);

#ifdef __cplusplus
}
#endif

#endif /* PP_B200_H */
