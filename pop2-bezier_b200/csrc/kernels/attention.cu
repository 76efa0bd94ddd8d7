// Int8 historical-KV decode attention for sm_100a.
//
// Replaces the reference's pp_i8_attention + pp_i8_merge (app/src/model/
// int8_kv.cu:28-59).  Same arithmetic contract:
//   k_t = bf16(i8 * ks[t]), v_t = bf16(i8 * vs[t])          (pp_i8_load, :23-27)
//   score_t = (q . k_t) * scale,  p_t = exp(score_t - max),  out = sum p v / sum p
//   reference mode: the token at index `past` is the f32 scratch (sk, sv), :36-37,49
// Different machinery:
//   * plan_kernel turns device lengths into a stream-K segment list (every CTA
//     gets the same number of tokens whatever the raggedness), or into
//     fixed-size splits when the caller asks for the reference's split_tokens.
//   * attn_kernel is persistent, one CTA per SM: a producer warp streams
//     whole stages of int8 K/V (TMA, 128B/64B swizzle) and their scales into
//     a multi-stage shared-memory ring guarded by mbarriers; consumer warps
//     dequantize to bf16 in registers and run the two dot products (q.k and
//     p.V) on the tensor cores (mma.sync m16n8k16, f32 accumulate), with q
//     and p split into three bf16 terms so the products are exact in f32.
//   * dequant per element: a byte permute builds the float 2^23 + 128 + i,
//     a packed f32 add removes the bias exactly, a packed f32 multiply
//     applies the scale (the reference's f32 product) and a bf16x2 pack
//     rounds to nearest even, so bf16(i8 * scale) is reproduced bit for bit.
//   * rows end with a log-sum-exp merge of their per-segment partials (and,
//     in reference mode, the scratch token).  With stream-K plans the
//     attention kernel does it: a row held by one segment is normalised in
//     place, a row split over CTAs by the CTA that completes it last.  With
//     fixed splits, combine_kernel does it after the attention kernel.
// All softmax arithmetic runs in base 2 (scores pre-scaled by log2 e).
#include <type_traits>

#include "common.cuh"
#include "../host/internal.h"

namespace pp {
namespace {

// Fewest history tokens per CTA in a stream-K plan: a smaller call uses fewer
// CTAs (a CTA's fixed cost outweighs a few hundred tokens of work).
#ifndef PP_PLAN_MIN_TOKENS
#define PP_PLAN_MIN_TOKENS 512
#endif

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s: generous, never hit in normal runs
constexpr float kSlack = 8.0f;  // log2-domain headroom before the softmax reference point moves

// ------------------------------------------------------------------ plan

__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t* warp_tot, uint32_t& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        uint32_t y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = (lane < (int)(blockDim.x >> 5)) ? warp_tot[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            uint32_t y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        warp_tot[lane] = w;  // inclusive
    }
    __syncthreads();
    const uint32_t before = (warp ? warp_tot[warp - 1] : 0u) + x - v;
    total = warp_tot[(blockDim.x >> 5) - 1];
    __syncthreads();
    return before;
}

struct PlanArgs {
    const uint32_t* lengths;
    unsigned char* ws;
    WsLayout l;
    uint32_t rows, heads, capacity, split, scratch, max_ctas, min_tokens;
    // whole rows per CTA instead of stream-K cuts when the rows are of one length and
    // that adds fewer tokens per CTA than this (the cost of a row split across CTAs)
    uint32_t whole_row_slack;
    uint32_t* status;
};

__global__ void __launch_bounds__(1024) plan_kernel(PlanArgs a) {
    // launched as a programmatic dependent: the lengths may come from the kernel
    // before.  Dependents are released only when the plan is complete (no early
    // trigger), so nothing can read a half-written plan.
    pdl_wait_primary();
    __shared__ uint32_t warp_tot[32];
    __shared__ uint32_t s_n_ctas, s_per_cta, s_total, s_bad, s_hmin, s_hmax, s_rows;
    PlanHeader* hdr = reinterpret_cast<PlanHeader*>(a.ws);
    uint32_t* row_len = reinterpret_cast<uint32_t*>(a.ws + a.l.row_len);
    uint32_t* row_seg = reinterpret_cast<uint32_t*>(a.ws + a.l.row_seg);
    uint32_t* cta_seg = reinterpret_cast<uint32_t*>(a.ws + a.l.cta_seg);
    SegDesc* segs = reinterpret_cast<SegDesc*>(a.ws + a.l.segs);
    uint32_t* row_cnt = reinterpret_cast<uint32_t*>(a.ws + a.l.row_cnt);
    uint32_t* orphans = reinterpret_cast<uint32_t*>(a.ws + a.l.orphans);
    if (threadIdx.x == 0) {
        s_bad = 0;
        s_hmin = 0xffffffffu;
        s_hmax = 0;
        s_rows = 0;
    }
    __syncthreads();

    auto history = [&](uint32_t r, bool& valid) -> uint32_t {
        uint32_t len = a.lengths ? __ldg(a.lengths + r / a.heads) : a.capacity;  // no lengths: every row is full
        valid = a.scratch ? (len <= a.capacity) : (len > 0 && len <= a.capacity);
        return valid ? len : 0u;
    };

    // Pass 1: per-row history lengths and the total token count.
    uint32_t carry = 0;
    for (uint32_t base = 0; base < a.rows; base += blockDim.x) {
        const uint32_t r = base + threadIdx.x;
        bool valid = true;
        uint32_t h = r < a.rows ? history(r, valid) : 0u;
        if (r < a.rows) {
            row_len[r] = valid ? h : kInvalidRow;
            if (!valid) s_bad = 1;
            if (h) {  // rows with history: their count and length range
                atomicMin(&s_hmin, h);
                atomicMax(&s_hmax, h);
                atomicAdd(&s_rows, 1u);
            }
        }
        uint32_t tot;
        block_exclusive_scan(h, warp_tot, tot);
        carry += tot;
    }
    if (threadIdx.x == 0) {
        const uint32_t total = carry;
        uint32_t n_ctas = 0, per = 0;
        if (total) {
            if (a.split) {
                n_ctas = a.max_ctas;  // refined after the segment count is known
            } else {
                uint32_t want = (total + a.min_tokens - 1) / a.min_tokens;
                n_ctas = want < a.max_ctas ? want : a.max_ctas;
                per = (total + n_ctas - 1) / n_ctas;
                if (s_hmin == s_hmax) {
                    // rows of one length h: k whole rows per CTA put every cut on a row
                    // boundary, so no row is split across CTAs; taken when the larger
                    // share costs less than the splits it avoids
                    const uint32_t k = (s_rows + a.max_ctas - 1) / a.max_ctas;
                    const unsigned long long whole = (unsigned long long)k * s_hmax;
                    if (whole >= per && whole - per < a.whole_row_slack && whole <= 0xffffffffull)
                        per = (uint32_t)whole;
                }
                n_ctas = (total + per - 1) / per;  // every CTA range non-empty
            }
        }
        s_n_ctas = n_ctas;
        s_per_cta = per;
        s_total = total;
        if (s_bad && a.status) atomicOr(a.status, PP_DEV_LENGTH_RANGE);
    }
    __syncthreads();
    const uint32_t per = s_per_cta;

    // Pass 2: token prefix -> segment counts -> segment prefix -> descriptors;
    // rows without segments go to the orphan list.
    uint32_t tok_carry = 0, seg_carry = 0, orphan_carry = 0;
    for (uint32_t base = 0; base < a.rows; base += blockDim.x) {
        const uint32_t r = base + threadIdx.x;
        bool valid = true;
        const uint32_t h = r < a.rows ? history(r, valid) : 0u;
        uint32_t tot;
        const uint32_t p0 = tok_carry + block_exclusive_scan(h, warp_tot, tot);
        tok_carry += tot;
        uint32_t n = 0;
        if (h) {
            if (a.split) n = (h + a.split - 1) / a.split;
            else n = (p0 + h - 1) / per - p0 / per + 1;
        }
        const uint32_t s0 = seg_carry + block_exclusive_scan(n, warp_tot, tot);
        seg_carry += tot;
        const uint32_t orphan = (r < a.rows && n == 0) ? 1u : 0u;
        const uint32_t o0 = orphan_carry + block_exclusive_scan(orphan, warp_tot, tot);
        orphan_carry += tot;
        if (r < a.rows) {
            row_seg[r] = s0;
            row_cnt[r] = 0u;
            if (orphan) orphans[o0] = r;
            if (a.split) {
                for (uint32_t k = 0; k < n; ++k) {
                    uint32_t t0 = k * a.split, t1 = min(h, t0 + a.split);
                    segs[s0 + k] = SegDesc{r, t0, t1, n};
                }
            } else if (n) {
                const uint32_t j0 = p0 / per;
                for (uint32_t k = 0; k < n; ++k) {
                    const uint32_t j = j0 + k;
                    const uint32_t lo = max(p0, j * per), hi = min(p0 + h, (j + 1) * per);
                    segs[s0 + k] = SegDesc{r, lo - p0, hi - p0, n};
                    if (j * per >= p0) cta_seg[j] = s0 + k;  // CTA j starts inside this row
                }
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) row_seg[a.rows] = seg_carry;
    uint32_t n_ctas = s_n_ctas;
    if (a.split) {
        n_ctas = seg_carry < a.max_ctas ? seg_carry : a.max_ctas;
        for (uint32_t j = threadIdx.x; j <= n_ctas; j += blockDim.x)
            cta_seg[j] = n_ctas ? (uint32_t)(((unsigned long long)j * seg_carry) / n_ctas) : 0u;
    } else if (threadIdx.x == 0) {
        cta_seg[n_ctas] = seg_carry;
        if (n_ctas == 0) cta_seg[0] = 0;
    }
    if (threadIdx.x == 0) {
        hdr->total_tokens = s_total;
        hdr->tokens_per_cta = per;
        hdr->n_segs = seg_carry;
        hdr->n_ctas = n_ctas;
        hdr->rows = a.rows;
        hdr->heads = a.heads;
        hdr->capacity = a.capacity;
        hdr->split = a.split;
        hdr->scratch = a.scratch;
        hdr->max_segs = a.l.max_segs;
        hdr->max_ctas = a.max_ctas;
        hdr->n_orphans = orphan_carry;
    }
}

template <typename T>
__device__ __forceinline__ float ldq(const T* p, uint64_t i);
template <>
__device__ __forceinline__ float ldq<float>(const float* p, uint64_t i) {
    return p[i];
}
template <>
__device__ __forceinline__ float ldq<__nv_bfloat16>(const __nv_bfloat16* p, uint64_t i) {
    return __bfloat162float(p[i]);
}

template <typename O>
__device__ __forceinline__ void st_out(O* p, uint64_t i, float v);
template <>
__device__ __forceinline__ void st_out<float>(float* p, uint64_t i, float v) {
    p[i] = v;
}
template <>
__device__ __forceinline__ void st_out<__nv_bfloat16>(__nv_bfloat16* p, uint64_t i, float v) {
    p[i] = __float2bfloat16_rn(v);
}


// The scratch token of reference-mode row r: its score q.sk (softmax scale,
// log2 units; every lane holds it) and sv for lane l's channels [l*E, l*E+E),
// E = D/32.  Loaded ahead of the merge that needs them, so that their latency
// overlaps other work.
template <int D>
struct ScratchVals {
    bool on;
    float ms;
    float sv[D / 32];
};

template <int D, typename QT>
__device__ __forceinline__ ScratchVals<D> load_scratch(int lane, uint32_t r, const void* q, const float* sk,
                                                       const float* sv, float scale_log2) {
    constexpr int E = D / 32;
    ScratchVals<D> v;
    v.on = sk != nullptr;
    v.ms = -INFINITY;
    if (v.on) {
        const QT* qr = reinterpret_cast<const QT*>(q) + (uint64_t)r * D;
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            v.sv[e] = sv[(uint64_t)r * D + lane * E + e];
            dot += (ldq<QT>(qr, lane * E + e) * scale_log2) * sk[(uint64_t)r * D + lane * E + e];
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        v.ms = dot;
    }
    return v;
}

// Writes row r: acc / z, or NaN for an invalid row or one whose weights sum to zero.
template <int D, typename OT>
__device__ __forceinline__ void store_row(int lane, uint32_t r, bool invalid, const float* acc, float z, void* out_base) {
    constexpr int E = D / 32;
    OT* out = reinterpret_cast<OT*>(out_base) + (uint64_t)r * D;
#pragma unroll
    for (int e = 0; e < E; ++e)
        st_out<OT>(out, lane * E + e, !invalid && z > 0.f ? acc[e] / z : __uint_as_float(0x7fc00000u));
}

// Log-sum-exp finish of row r by one warp (lane l owns channels [l*E, l*E+E),
// E = D/32): merges the row's n partials (m in log2 units, z, acc), taken in
// segment order from `part`, and in reference mode the f32 scratch token
// (q.sk, sv), then writes acc / z.  The merge of pp_i8_merge
// (int8_kv.cu:53-59) with the scratch token of pp_i8_attention (:36-37, 49)
// folded in; an invalid row, or one whose weights sum to zero, is NaN.
template <int D, typename OT, typename Part>
__device__ __forceinline__ void finish_row(int lane, uint32_t r, uint32_t n, bool invalid, const Part& part,
                                           const ScratchVals<D>& sc, void* out_base) {
    constexpr int E = D / 32;
    float acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0.f;
    if (invalid) {
        store_row<D, OT>(lane, r, true, acc, 0.f, out_base);
        return;
    }
    float mx = -INFINITY;
    for (uint32_t s = 0; s < n; ++s) mx = fmaxf(mx, part.m(s));
    const float ms = sc.ms;
    if (sc.on) mx = fmaxf(mx, ms);
    float z = 0.f;
    for (uint32_t s = 0; s < n; ++s) {
        const float m = part.m(s);
        const float f = m == -INFINITY ? 0.f : fast_exp2(m - mx);
        z += part.z(s) * f;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] += part.acc(s, lane, e) * f;
    }
    if (sc.on) {
        const float f = fast_exp2(ms - mx);
        z += f;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] += sc.sv[e] * f;
    }
    store_row<D, OT>(lane, r, false, acc, z, out_base);
}

// The final merge of a row split over n <= batch_segs<D>() segments, by the CTA
// that completed the row last: its own partial (segment `own` of the row)
// comes from registers and the others are all loaded at once, then the same
// arithmetic as finish_row, in the same segment order.
template <int D>
__host__ __device__ constexpr uint32_t batch_segs() { return D == 128 ? 2u : 3u; }  // register budget of the batch

template <int D, typename OT, typename Own>
__device__ __forceinline__ void finish_split(int lane, uint32_t r, uint32_t n, uint32_t own, const Own& mine,
                                             const float* base, const ScratchVals<D>& sc, void* out_base) {
    constexpr int E = D / 32;
    constexpr uint32_t kBatchSegs = batch_segs<D>();
    float mv[kBatchSegs], zv[kBatchSegs], av[kBatchSegs][E];
#pragma unroll
    for (uint32_t s = 0; s < kBatchSegs; ++s) {
        mv[s] = -INFINITY;
        zv[s] = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) av[s][e] = 0.f;
        if (s < n) {
            if (s == own) {
                mv[s] = mine.mv;
                zv[s] = mine.zv;
#pragma unroll
                for (int e = 0; e < E; ++e) av[s][e] = mine.a[e];
            } else {
                const float* p = base + (uint64_t)s * (D + 4);  // written by other CTAs: read through L2
                mv[s] = __ldcg(p + D);
                zv[s] = __ldcg(p + D + 1);
#pragma unroll
                for (int e = 0; e < E; ++e) av[s][e] = __ldcg(p + lane * E + e);
            }
        }
    }
    float acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0.f;
    float mx = -INFINITY;
#pragma unroll
    for (uint32_t s = 0; s < kBatchSegs; ++s)
        if (s < n) mx = fmaxf(mx, mv[s]);
    const float ms = sc.ms;
    if (sc.on) mx = fmaxf(mx, ms);
    float z = 0.f;
#pragma unroll
    for (uint32_t s = 0; s < kBatchSegs; ++s) {
        if (s < n) {
            const float f = mv[s] == -INFINITY ? 0.f : fast_exp2(mv[s] - mx);
            z += zv[s] * f;
#pragma unroll
            for (int e = 0; e < E; ++e) acc[e] += av[s][e] * f;
        }
    }
    if (sc.on) {
        const float f = fast_exp2(ms - mx);
        z += f;
#pragma unroll
        for (int e = 0; e < E; ++e) acc[e] += sc.sv[e] * f;
    }
    store_row<D, OT>(lane, r, false, acc, z, out_base);
}

// Partials of one row in the workspace, [segment][D + 4] from `base`.
// Coherent: read through L2 only (partials written by other CTAs of the
// same launch); otherwise plain loads.
template <int D, bool Coherent>
struct GlobalPartials {
    const float* base;
    __device__ __forceinline__ float ld(const float* p) const {
        if constexpr (Coherent) return __ldcg(p);
        else return *p;
    }
    __device__ __forceinline__ float m(uint32_t s) const { return ld(base + (uint64_t)s * (D + 4) + D); }
    __device__ __forceinline__ float z(uint32_t s) const { return ld(base + (uint64_t)s * (D + 4) + D + 1); }
    __device__ __forceinline__ float acc(uint32_t s, int lane, int e) const {
        return ld(base + (uint64_t)s * (D + 4) + lane * (D / 32) + e);
    }
};

// The single partial of a row, held in registers (the lane's E channels).
template <int D>
struct RegPartial {
    float mv, zv;
    float a[D / 32];
    __device__ __forceinline__ float m(uint32_t) const { return mv; }
    __device__ __forceinline__ float z(uint32_t) const { return zv; }
    __device__ __forceinline__ float acc(uint32_t, int, int e) const { return a[e]; }
};

// ------------------------------------------------------------- attention

// Consumer warps per CTA, 16-token MMA blocks per warp per stage, and ring
// depth (tuning knobs; the defaults were chosen by measurement on B200).
#ifndef PP_ATTN_NC
#define PP_ATTN_NC 15
#endif
#ifndef PP_ATTN_NB_D128
#define PP_ATTN_NB_D128 1
#endif
#ifndef PP_ATTN_NB_D64
#define PP_ATTN_NB_D64 2  // two 16-token blocks per warp keep more independent work in flight
#endif
#ifndef PP_ATTN_STAGES_D128
#define PP_ATTN_STAGES_D128 3
#endif
#ifndef PP_ATTN_STAGES_D64
#define PP_ATTN_STAGES_D64 3  // 480-token stages of 64 KB: three fit
#endif
// int8 head_dim 64 calls with few tokens per CTA (the reference model's own
// steps: rows of at most 1024 tokens) run 12 consumer warps, 384-token stages:
// the ring fills and drains sooner, and a 1023-token row is three stages
#ifndef PP_ATTN_NC_SHORT_D64
#define PP_ATTN_NC_SHORT_D64 12
#endif
#ifndef PP_ATTN_SHORT_TOKENS_PER_CTA
#define PP_ATTN_SHORT_TOKENS_PER_CTA 6144  // rows x capacity per CTA at most this: short stages
#endif

// Element type of the K/V history: int8 codes with per-token scales (the
// int8 arena), or plain bf16 / f32 rows (the float-KV cache).
enum class Kv : int { I8 = kKvInt8, BF16 = kKvBf16, F32 = kKvF32 };

template <int D, Kv KV = Kv::I8, int NCW = 0>  // NCW: consumer warps (0: by row width)
struct Cfg {
    static constexpr bool SCALED = KV == Kv::I8;    // int8 codes + scale arrays
    static constexpr int ELEM = KV == Kv::I8 ? 1 : KV == Kv::BF16 ? 2 : 4;
    static constexpr int ROW = D * ELEM;            // bytes of one token of K (or V)
    // Shared-memory tiles are swizzled panels of at most 128-byte rows: a row
    // wider than 128 bytes is split into ROW / 128 panels, each a separate
    // [tokens][128 B] tile, so reads stay bank-conflict free.
    static constexpr int PANEL = ROW < 128 ? ROW : 128;
    static constexpr int PANELS = ROW / PANEL;
    // consumer warps: all 15 while a stage of 240 tokens fits ~62 KB, fewer
    // (fewer tokens per stage) for the wider float rows
    static constexpr int NC = NCW ? NCW : ROW <= 128 ? PP_ATTN_NC : ROW == 256 ? 8 : 4;
    static constexpr int THREADS = (NC + 1) * 32;   // + one producer warp
    static constexpr int BOX = 16;                  // tokens per MMA block and per tail TMA box
    // MMA blocks per consumer warp per stage (independent blocks interleaved for ILP)
    static constexpr int NB = !SCALED ? 1 : D == 128 ? PP_ATTN_NB_D128 : PP_ATTN_NB_D64;
    static constexpr int TPW = BOX * NB;            // tokens per consumer warp per stage
    static constexpr int T = TPW * NC;              // tokens per stage
    static constexpr int KV_BYTES = T * ROW;
    // scale elements per TMA box: one box covers a stage's T tokens plus the
    // alignment slack (a copy costs the SM's copy engine a fixed ~130 ns on
    // top of its bytes, so a stage is as few copies as possible)
    static constexpr int SC_BOX = 256;
    static constexpr int SC_BOXES = SCALED ? (T + 4 + SC_BOX - 1) / SC_BOX : 0;  // T tokens + alignment slack
    static constexpr int SC_BYTES = SC_BOXES * SC_BOX * 4;
    static constexpr int Q_BYTES = D * 4;
    static constexpr int OFF_K = 0;
    static constexpr int OFF_V = KV_BYTES;
    static constexpr int OFF_KS = 2 * KV_BYTES;
    static constexpr int SC_SLOT = ((SC_BYTES + 127) / 128) * 128;  // tensor copies land 128B-aligned
    static constexpr int OFF_VS = OFF_KS + SC_SLOT;
    static constexpr int OFF_Q = OFF_VS + SC_SLOT;
    static constexpr int OFF_META = OFF_Q + Q_BYTES;
    static constexpr int STAGE_BYTES = ((OFF_META + 64 + 1023) / 1024) * 1024;
    static constexpr int STAGES = !SCALED ? 3 : D == 128 ? PP_ATTN_STAGES_D128 : PP_ATTN_STAGES_D64;
    static constexpr int STAGE_BOXES = (T + 255) / 256;  // TMA boxes hold at most 256 rows
    static constexpr int STAGE_BOX = T / STAGE_BOXES;    // tokens per whole-stage box
    static_assert(STAGE_BOX * STAGE_BOXES == T && STAGE_BOX % BOX == 0, "stage splits into equal boxes");
    static_assert(SCALED || STAGE_BOXES == 1, "float stages are one box per panel");
    static constexpr int RED_FLOATS = NC * (D + 4);
    static constexpr int OFF_RED = STAGES * STAGE_BYTES;
    static constexpr int OFF_BAR = OFF_RED + 2 * RED_FLOATS * 4;
    // full, empty, reduction ready x2, reduction free x2, q split ready x QSLOTS
    static constexpr int QSLOTS = 16;
    static constexpr int BAR_COUNT = 2 * STAGES + 4 + QSLOTS;
    // q of the CTA's segments 1 .. QSLOTS-1, scaled and split into three bf16
    // terms ([term][channel]), prepared at kernel start (slot 0 unused: the
    // first segment's warps split q themselves rather than wait)
    static constexpr int QT_BYTES = 3 * D * 2;
    static constexpr int OFF_QT = ((OFF_BAR + BAR_COUNT * 8 + 16 + 127) / 128) * 128;
    static constexpr int SMEM_BYTES = OFF_QT + QSLOTS * QT_BYTES + 1024;  // + base alignment
    static_assert(SMEM_BYTES <= 232448, "shared memory budget of one CTA");
    // Tensor-copy destinations in shared memory must be 128-byte aligned, and
    // the swizzled tiles 1024-byte aligned (stage bases are 1024-aligned).
    static_assert((SC_BOX * 4) % 128 == 0 && OFF_KS % 128 == 0 && OFF_VS % 128 == 0, "scale boxes 128B-aligned");
    static_assert(!SCALED || SC_BOXES <= 2, "at most two scale boxes per tensor per stage");
    static_assert(OFF_K % 1024 == 0 && OFF_V % 1024 == 0 && (BOX * PANEL) % 1024 == 0 &&
                      (STAGE_BOX * PANEL) % 1024 == 0 && (T * PANEL) % 1024 == 0,
                  "tiles 1024B-aligned");
    static_assert(STAGE_BYTES % 1024 == 0 && OFF_Q % 16 == 0 && OFF_META % 16 == 0, "stage layout alignment");
    static_assert(T / BOX < 32, "a tail of fewer than T tokens is at most 31 units: one box each of 256/128/64/32/16");
    static constexpr int NI = D / 16;  // q.k MMAs per 16-token block (k = 16 channels each)
    static constexpr int NJ = D / 16;  // p.V MMAs per 16-token block (m = 16 channels each)

    // Channel maps.  In q.k MMA i, thread (g, c) supplies the k positions
    // 2c, 2c+1, 2c+8, 2c+9, which stand for the four channels from qk_ch(c, i)
    // on (K as the A operand, q as B: both from the same thread, so any
    // per-thread assignment is consistent).  In p.V, row m = g of the A tile
    // (V^T) in MMA j is channel pv_ch(g, j) and row m = g + 8 is
    // pv_ch(g, D/16 + j).  Int8 rows (<= 128 B) use contiguous runs; float
    // rows take 16-byte chunks 2c, 2c+1 (q.k) and chunk g (p.V) of every
    // panel, which keeps the loads of a quarter warp on distinct banks.
    static constexpr int CH_ELEMS = 16 / ELEM;  // channels per 16-byte chunk
    // 16-byte chunk k (0 .. ROW/64 - 1) of thread c's q.k slice, counted over the panels
    __device__ static __forceinline__ int qk_chunk(int c, int k) {
        if constexpr (SCALED) return c * (ROW / 64) + k;
        else return (k >> 1) * 8 + 2 * c + (k & 1);
    }
    __device__ static __forceinline__ int qk_ch(int c, int i) {
        if constexpr (SCALED) return (D / 4) * c + 4 * i;
        else if constexpr (KV == Kv::BF16) return qk_chunk(c, i >> 1) * CH_ELEMS + 4 * (i & 1);
        else return qk_chunk(c, i) * CH_ELEMS;
    }
    __device__ static __forceinline__ int pv_ch(int g, int l) {  // l: 0 .. D/8 - 1
        if constexpr (SCALED) return (D / 8) * g + l;
        else return (l / CH_ELEMS) * (128 / ELEM) + g * CH_ELEMS + l % CH_ELEMS;
    }
};

struct StageMeta {
    uint32_t row, t, nvalid, slot, flags, ks_off, vs_off, row_segs;
    // the CTA's work, for the consumers' first stage: segment range, rows without segments
    uint32_t seg_begin, seg_count, n_orphans, pad[5];
};
constexpr uint32_t kFirst = 1u, kLast = 2u, kTerm = 4u;

struct AttnArgs {
    const void* q;
    uint64_t q_stride;  // elements between q rows
    unsigned char* ws;
    float* partials;
    WsLayout l;
    uint32_t capacity;
    uint32_t ks_mis, vs_mis;
    float scale_log2;
    uint32_t* status;
    // row finish (stream-K plans): outputs, reference-mode scratch token
    uint32_t finish;    // 1: this kernel writes the outputs; 0: the combine kernel does
    uint32_t prefetch;  // PP_ATTN_PREFETCH_HISTORY: stream history before the previous kernel completes
    uint32_t out_bf16;  // output element type: bf16 (1) or f32 (0)
    void* out;
    const float* sk;
    const float* sv;
};

// Channels [ch, ch + 4) of the staged q row.
template <typename QT>
__device__ __forceinline__ void load_q4(uint32_t q_smem, int ch, float* out);
template <>
__device__ __forceinline__ void load_q4<float>(uint32_t q_smem, int ch, float* out) {
    const uint4 v = lds128(q_smem + (uint32_t)ch * 4u);
    out[0] = __uint_as_float(v.x);
    out[1] = __uint_as_float(v.y);
    out[2] = __uint_as_float(v.z);
    out[3] = __uint_as_float(v.w);
}
template <>
__device__ __forceinline__ void load_q4<__nv_bfloat16>(uint32_t q_smem, int ch, float* out) {
    const uint2 v = lds64(q_smem + (uint32_t)ch * 2u);
    out[0] = bf16_lo_to_f32(v.x);
    out[1] = bf16_hi_to_f32(v.x);
    out[2] = bf16_lo_to_f32(v.y);
    out[3] = bf16_hi_to_f32(v.y);
}

// bf16 term `part` (0: hi, 1: lo, 2: lo2, else 0) of the exact three-term
// split of two f32 values, packed.  hi + lo + lo2 == x exactly for normal x.
__device__ __forceinline__ uint32_t split_term_pack(float a, float b, int part) {
    const uint32_t h = pack_bf16x2(a, b);
    const float ra = a - bf16_lo_to_f32(h), rb = b - bf16_hi_to_f32(h);
    const uint32_t l = pack_bf16x2(ra, rb);
    const uint32_t l2 = pack_bf16x2(ra - bf16_lo_to_f32(l), rb - bf16_hi_to_f32(l));
    return part == 0 ? h : part == 1 ? l : part == 2 ? l2 : 0u;
}

// The three bf16x2 terms of an f32 pair: h + l + l2 == (a, b) for normal values.
__device__ __forceinline__ void split3_pair(float a, float b, uint32_t& h, uint32_t& l, uint32_t& l2) {
    h = pack_bf16x2(a, b);
    const uint64_t r = f2_sub(f2_pack(a, b), f2_pack(bf16_lo_to_f32(h), bf16_hi_to_f32(h)));
    l = pack_bf16x2_f2(r);
    l2 = pack_bf16x2_f2(f2_sub(r, f2_pack(bf16_lo_to_f32(l), bf16_hi_to_f32(l))));
}

__device__ __forceinline__ uint32_t u4_word(const uint4& v, int w) {
    return w == 0 ? v.x : w == 1 ? v.y : w == 2 ? v.z : v.w;
}

template <int D, typename QT, Kv KV, int NCW>
__global__ void __launch_bounds__(Cfg<D, KV, NCW>::THREADS, 1)
    attn_kernel(const __grid_constant__ TailMaps tails,
                const __grid_constant__ CUtensorMap map_k_stage, const __grid_constant__ CUtensorMap map_v_stage,
                const __grid_constant__ CUtensorMap map_ks, const __grid_constant__ CUtensorMap map_vs,
                const AttnArgs args) {
    using C = Cfg<D, KV, NCW>;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* empty = full + C::STAGES;
    uint64_t* red_bar = empty + C::STAGES;  // [2]: all consumer warps' states are in reduction buffer p
    uint64_t* red_free = red_bar + 2;       // [2]: the finishing warp has read reduction buffer p
    uint64_t* q_ready = red_free + 2;       // [QSLOTS]: q split of segment k is in its slot
    volatile int* abort_flag = reinterpret_cast<volatile int*>(q_ready + C::QSLOTS);
    float* red = reinterpret_cast<float*>(smem + C::OFF_RED);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], C::NC);
        }
        mbar_init(&red_bar[0], C::NC);
        mbar_init(&red_bar[1], C::NC);
        mbar_init(&red_free[0], 1);
        mbar_init(&red_free[1], 1);
        for (int k = 0; k < C::QSLOTS; ++k) mbar_init(&q_ready[k], 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == C::NC && lane == 0) {
        for (int i = 0; i < kTailBoxes; ++i) {
            tma_prefetch_desc(&tails.k[i]);
            tma_prefetch_desc(&tails.v[i]);
        }
        tma_prefetch_desc(&map_k_stage);
        tma_prefetch_desc(&map_v_stage);
        if constexpr (C::SCALED) {
            tma_prefetch_desc(&map_ks);
            tma_prefetch_desc(&map_vs);
        }
    }
    __syncthreads();
    // The kernel before this one on the stream may still be running (programmatic
    // dependent launch).  Without PP_ATTN_PREFETCH_HISTORY every thread waits for
    // it here.  With it, the producer reads the plan and streams K/V history first
    // (the caller vouches that kernel writes neither) and waits before loading q;
    // the consumers wait before reading anything.  Dependents of this kernel are
    // released only after the wait, so a chain of such launches never lets a
    // kernel start before the ones two places earlier have completed.
    if (!args.prefetch) {
        pdl_wait_primary();
        pdl_launch_dependents();
    }

    const PlanHeader* hdr = reinterpret_cast<const PlanHeader*>(args.ws);
    const uint32_t* cta_seg = reinterpret_cast<const uint32_t*>(args.ws + args.l.cta_seg);
    const SegDesc* segs = reinterpret_cast<const SegDesc*>(args.ws + args.l.segs);

    if (warp == C::NC) {
        // ------------------------------------------------------ producer
        if (lane != 0) return;
        const uint32_t n_ctas = hdr->n_ctas;
        const uint32_t n_orphans = args.finish ? hdr->n_orphans : 0u;
        uint32_t s_begin = 0, s_end = 0;
        if (blockIdx.x < n_ctas) {
            s_begin = cta_seg[blockIdx.x];
            s_end = cta_seg[blockIdx.x + 1];
        }
        constexpr uint32_t q_bytes = D * sizeof(QT);
        uint32_t it = 0;
        bool ok = true;
        // q loads of stages issued before the wait (at most one ring's worth)
        bool waited = !args.prefetch;
        uint32_t pend_n = 0, pend_slot[C::STAGES];
        const unsigned char* pend_src[C::STAGES];
        auto release_q = [&]() {
            if (waited) return;
            pdl_wait_primary();
            pdl_launch_dependents();
            waited = true;
            for (uint32_t i = 0; i < pend_n; ++i)
                bulk_load(smem + pend_slot[i] * C::STAGE_BYTES + C::OFF_Q, pend_src[i], q_bytes, &full[pend_slot[i]]);
            pend_n = 0;
        };
        SegDesc next = s_begin < s_end ? segs[s_begin] : SegDesc{0, 0, 0, 0};
        for (uint32_t s = s_begin; s < s_end && ok; ++s) {
            const SegDesc sd = next;
            if (s + 1 < s_end) next = segs[s + 1];
            for (uint32_t t = sd.t0, n = 0; t < sd.t1; t += n, ++it) {
                // T tokens per stage, except that a remainder which would leave the
                // segment's last stage less than half full is split with the stage
                // before it into two stages of about equal size (whole 16-token
                // units first): a nearly empty stage holds a ring slot while the
                // consumers get through it at once and then wait for the next
                const uint32_t rem = sd.t1 - t;
                n = rem <= (uint32_t)C::T ? rem
                    : rem < (uint32_t)(C::T + C::T / 2) ? ((rem + 1) / 2 + C::BOX - 1) / C::BOX * C::BOX
                                                        : (uint32_t)C::T;
                const uint32_t slot = it % C::STAGES, ph = (it / C::STAGES) & 1u;
                if (it == (uint32_t)C::STAGES) release_q();  // the ring is full: q before anything else
                if (!mbar_wait_bounded(&empty[slot], ph ^ 1u, abort_flag, kWaitLimitNs)) {
                    ok = false;
                    break;
                }
                unsigned char* st = smem + slot * C::STAGE_BYTES;
                const uint32_t nbox = (n + C::BOX - 1) / C::BOX;
                const uint32_t tok = sd.row * args.capacity + t;
                const uint32_t ksx = (args.ks_mis + tok) & ~3u, vsx = (args.vs_mis + tok) & ~3u;
                StageMeta* meta = reinterpret_cast<StageMeta*>(st + C::OFF_META);
                const bool first = t == sd.t0, last = t + n >= sd.t1;
                meta->row = sd.row;
                meta->t = t;
                meta->nvalid = n;
                meta->slot = s;
                meta->flags = (first ? kFirst : 0u) | (last ? kLast : 0u);
                meta->ks_off = args.ks_mis + tok - ksx;
                meta->vs_off = args.vs_mis + tok - vsx;
                meta->row_segs = sd.row_segs;
                meta->seg_begin = s_begin;
                meta->seg_count = s_end - s_begin;
                meta->n_orphans = n_orphans;
                // q goes with a segment's first stage only when the consumers read it
                // there: the CTA's first segment, and segments past the q splits
                // prepared at kernel start (the others would only make the stage
                // wait for one more copy).  It is issued before the K/V copies.
                const uint32_t rel = s - s_begin;
                const bool load_q = first && (rel == 0 || rel >= (uint32_t)C::QSLOTS);
                const uint32_t bytes = nbox * C::BOX * C::ROW * 2u + 2u * C::SC_BYTES + (load_q ? q_bytes : 0u);
                mbar_arrive_expect_tx(&full[slot], bytes);
                if (load_q) {
                    const unsigned char* qrow =
                        reinterpret_cast<const unsigned char*>(args.q) + (uint64_t)sd.row * args.q_stride * sizeof(QT);
                    if (waited) {
                        bulk_load(st + C::OFF_Q, qrow, q_bytes, &full[slot]);
                    } else {
                        pend_slot[pend_n] = slot;
                        pend_src[pend_n++] = qrow;
                    }
                }
                if constexpr (!C::SCALED) {
                    // float rows: 3-D maps {channel, token, row}, one copy per 128-byte panel
                    constexpr int PX = 128 / C::ELEM;  // channels per panel
                    if (n == (uint32_t)C::T) {
#pragma unroll
                        for (int p = 0; p < C::PANELS; ++p) {
                            tma_load_3d(st + C::OFF_K + p * C::T * 128, &map_k_stage, &full[slot], p * PX, (int32_t)t,
                                        (int32_t)sd.row);
                            tma_load_3d(st + C::OFF_V + p * C::T * 128, &map_v_stage, &full[slot], p * PX, (int32_t)t,
                                        (int32_t)sd.row);
                        }
                    } else {  // segment tail: nbox 16-token units as boxes of 256 / 128 / 64 / 32 / 16 tokens
                        uint32_t off = 0;
#pragma unroll
                        for (int i = 4; i >= 0; --i) {
                            if (!(nbox & (1u << i))) continue;
#pragma unroll
                            for (int p = 0; p < C::PANELS; ++p) {
                                tma_load_3d(st + C::OFF_K + p * C::T * 128 + off * 128, &tails.k[i], &full[slot], p * PX,
                                            (int32_t)(t + off), (int32_t)sd.row);
                                tma_load_3d(st + C::OFF_V + p * C::T * 128 + off * 128, &tails.v[i], &full[slot], p * PX,
                                            (int32_t)(t + off), (int32_t)sd.row);
                            }
                            off += 16u << i;
                        }
                    }
                } else if (n == (uint32_t)C::T) {  // full stage: whole-stage boxes for K and V
#pragma unroll
                    for (int b = 0; b < C::STAGE_BOXES; ++b) {
                        tma_load_2d(st + C::OFF_K + b * C::STAGE_BOX * D, &map_k_stage, &full[slot], 0,
                                    (int32_t)(tok + b * C::STAGE_BOX));
                        tma_load_2d(st + C::OFF_V + b * C::STAGE_BOX * D, &map_v_stage, &full[slot], 0,
                                    (int32_t)(tok + b * C::STAGE_BOX));
                    }
                } else {  // segment tail: nbox 16-token units as boxes of 256 / 128 / 64 / 32 / 16 tokens
                    uint32_t off = 0;
#pragma unroll
                    for (int i = 4; i >= 0; --i) {
                        if (!(nbox & (1u << i))) continue;
                        tma_load_2d(st + C::OFF_K + off * D, &tails.k[i], &full[slot], 0, (int32_t)(tok + off));
                        tma_load_2d(st + C::OFF_V + off * D, &tails.v[i], &full[slot], 0, (int32_t)(tok + off));
                        off += 16u << i;
                    }
                }
#pragma unroll
                for (int b = 0; b < C::SC_BOXES; ++b) {  // int8 only (no boxes for float rows)
                    tma_load_1d(st + C::OFF_KS + b * C::SC_BOX * 4, &map_ks, &full[slot], (int32_t)(ksx + b * C::SC_BOX));
                    tma_load_1d(st + C::OFF_VS + b * C::SC_BOX * 4, &map_vs, &full[slot], (int32_t)(vsx + b * C::SC_BOX));
                }
            }
        }
        release_q();  // fewer stages than the ring holds, or an abort: the q loads still go out
        if (ok) {
            const uint32_t slot = it % C::STAGES, ph = (it / C::STAGES) & 1u;
            if (mbar_wait_bounded(&empty[slot], ph ^ 1u, abort_flag, kWaitLimitNs)) {
                StageMeta* meta = reinterpret_cast<StageMeta*>(smem + slot * C::STAGE_BYTES + C::OFF_META);
                meta->flags = kTerm;
                meta->seg_begin = s_begin;
                meta->seg_count = s_end - s_begin;
                meta->n_orphans = n_orphans;
                mbar_arrive(&full[slot]);
                return;
            }
        }
        // Abort: report, then wait (bounded) for the copies this warp issued.
        *abort_flag = 1;
        if (args.status) atomicOr(args.status, PP_DEV_WAIT_TIMEOUT);
        const uint32_t lo = it > (uint32_t)C::STAGES ? it - C::STAGES : 0u;
        for (uint32_t i = lo; i < it; ++i) {
            volatile int never = 0;
            mbar_wait_bounded(&full[i % C::STAGES], (i / C::STAGES) & 1u, &never, kWaitLimitNs);
        }
        return;
    }

    // ---------------------------------------------------------- consumers
    if (args.prefetch) {
        pdl_wait_primary();
        pdl_launch_dependents();
    }
    const int g = lane >> 2, c = lane & 3;
    uint32_t qb[C::NI][2];
    float acc[C::NJ][4];
    float m2 = -INFINITY, zsum = 0.f;
#pragma unroll
    for (int j = 0; j < C::NJ; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
    for (int i = 0; i < C::NI; ++i) qb[i][0] = qb[i][1] = 0u;
    uint32_t seg_count = 0;
    float* partials = args.partials;
    uint32_t* row_cnt = reinterpret_cast<uint32_t*>(args.ws + args.l.row_cnt);
    const uint32_t* row_seg = reinterpret_cast<const uint32_t*>(args.ws + args.l.row_seg);
    // writes output row r from its n partials (stream-K plans only)
    auto finish_out = [&](uint32_t r, uint32_t n, const auto& part, const ScratchVals<D>& sc) {
        const bool invalid = n == 0 && __ldg(reinterpret_cast<const uint32_t*>(args.ws + args.l.row_len) + r) == kInvalidRow;
        if (args.out_bf16)
            finish_row<D, __nv_bfloat16>(lane, r, n, invalid, part, sc, args.out);
        else
            finish_row<D, float>(lane, r, n, invalid, part, sc, args.out);
    };
    auto scratch_of = [&](uint32_t r) {
        return load_scratch<D, QT>(lane, r, args.q, args.sk, args.sv, args.scale_log2);
    };

    {
        // The CTA's work, told by the producer with the first stage: prepare what
        // later segments need (q splits) and write the rows that have no segments.
        if (!mbar_wait_bounded(&full[0], 0u, abort_flag, kWaitLimitNs)) {
            *abort_flag = 1;
            if (lane == 0 && args.status) atomicOr(args.status, PP_DEV_WAIT_TIMEOUT);
            return;
        }
        const uint4 m2w = lds128(smem_addr(smem + C::OFF_META) + 32u);
        const uint32_t seg_begin = m2w.x, n_pre = min(m2w.y, (uint32_t)C::QSLOTS), n_orphans = m2w.z;
        for (uint32_t k = 1 + warp; k < n_pre; k += C::NC) {
            const uint32_t r = segs[seg_begin + k].row;
            const QT* qr = reinterpret_cast<const QT*>(args.q) + (uint64_t)r * args.q_stride;
            __nv_bfloat16* qslot = reinterpret_cast<__nv_bfloat16*>(smem + C::OFF_QT + k * C::QT_BYTES);
#pragma unroll
            for (int e = 0; e < D / 32; ++e) {
                const int ch = lane * (D / 32) + e;
                const float x = ldq<QT>(qr, ch) * args.scale_log2;
                const __nv_bfloat16 t0 = __float2bfloat16_rn(x);
                const float r1 = x - __bfloat162float(t0);
                const __nv_bfloat16 t1 = __float2bfloat16_rn(r1);
                const __nv_bfloat16 t2 = __float2bfloat16_rn(r1 - __bfloat162float(t1));
                qslot[ch] = t0;
                qslot[D + ch] = t1;
                qslot[2 * D + ch] = t2;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&q_ready[k]);
        }
        if (n_orphans) {
            // invalid rows (NaN) or, in reference mode, the scratch token alone
            const uint32_t* orphans = reinterpret_cast<const uint32_t*>(args.ws + args.l.orphans);
            for (uint32_t k = blockIdx.x * C::NC + warp; k < n_orphans; k += gridDim.x * C::NC)
                finish_out(orphans[k], 0u, GlobalPartials<D, false>{partials}, scratch_of(orphans[k]));
        }
    }

    for (uint32_t it = 0;; ++it) {
        const uint32_t slot = it % C::STAGES, ph = (it / C::STAGES) & 1u;
        if (!mbar_wait_bounded(&full[slot], ph, abort_flag, kWaitLimitNs)) {
            *abort_flag = 1;
            if (lane == 0 && args.status) atomicOr(args.status, PP_DEV_WAIT_TIMEOUT);
            return;
        }
        unsigned char* st = smem + slot * C::STAGE_BYTES;
        // StageMeta {row, t, nvalid, slot | flags, ks_off, vs_off, row_segs}
        const uint4 m0 = lds128(smem_addr(st + C::OFF_META));
        const uint4 m1 = lds128(smem_addr(st + C::OFF_META) + 16u);
        const uint32_t flags = m1.x;
        if (flags & kTerm) break;
        const uint32_t nvalid = m0.z, seg_slot = m0.w, ks_off = m1.y, vs_off = m1.z;

        if (flags & kFirst) {
            // q row -> three-term bf16 B fragments for channel slice of thread c
            // (channels [D/4 * c, D/4 * c + D/4), term g; zero for g >= 3)
            if (seg_count > 0 && seg_count < (uint32_t)C::QSLOTS) {
                if (!mbar_wait_bounded(&q_ready[seg_count], 0u, abort_flag, kWaitLimitNs)) {
                    *abort_flag = 1;
                    if (lane == 0 && args.status) atomicOr(args.status, PP_DEV_WAIT_TIMEOUT);
                    return;
                }
                const uint32_t qt = smem_addr(smem + C::OFF_QT + seg_count * C::QT_BYTES) + (uint32_t)g * (D * 2);
#pragma unroll
                for (int i = 0; i < C::NI; i += 2) {  // channels qk_ch(c, i) .. + 8 are contiguous
                    const uint4 w = g < 3 ? lds128(qt + 2u * (uint32_t)C::qk_ch(c, i)) : make_uint4(0u, 0u, 0u, 0u);
                    qb[i][0] = w.x;
                    qb[i][1] = w.y;
                    qb[i + 1][0] = w.z;
                    qb[i + 1][1] = w.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < C::NI; ++i) {
                    float qv[4];
                    load_q4<QT>(smem_addr(st + C::OFF_Q), C::qk_ch(c, i), qv);
                    const float a0 = qv[0] * args.scale_log2, a1 = qv[1] * args.scale_log2;
                    const float a2 = qv[2] * args.scale_log2, a3 = qv[3] * args.scale_log2;
                    qb[i][0] = split_term_pack(a0, a1, g);
                    qb[i][1] = split_term_pack(a2, a3, g);
                }
            }
            m2 = -INFINITY;
            zsum = 0.f;
#pragma unroll
            for (int j = 0; j < C::NJ; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
        }

        const int tok0 = warp * C::TPW;
        const int nv = (int)nvalid - tok0;  // valid tokens from this warp's first token on
        // NBLK consecutive 16-token blocks of this warp, interleaved for ILP.
        // MASKED handles a segment's ragged end (tokens >= nv contribute nothing).
        auto blocks = [&](auto nblk_tag, auto masked_tag) {
            constexpr int NBLK = decltype(nblk_tag)::value;
            constexpr bool MASKED = decltype(masked_tag)::value;
            const uint32_t kt = smem_addr(st + C::OFF_K + tok0 * C::PANEL);
            const uint32_t vt = smem_addr(st + C::OFF_V + tok0 * C::PANEL);
            const uint32_t ks = smem_addr(st + C::OFF_KS) + (ks_off + tok0) * 4u;
            const uint32_t vs = smem_addr(st + C::OFF_VS) + (vs_off + tok0) * 4u;
            auto scale = [&](uint32_t addr, int e) -> float {  // e: token index from tok0
                if constexpr (MASKED) return e < nv ? lds_f32(addr + e * 4) : 0.f;
                else return lds_f32(addr + e * 4);
            };

            // ---- scores: q . k for tokens g and g+8 of each block
            float s_g[NBLK], s_g8[NBLK];
            {
                float sacc[NBLK][2][4];
#pragma unroll
                for (int b = 0; b < NBLK; ++b)
#pragma unroll
                    for (int h = 0; h < 2; ++h) sacc[b][h][0] = sacc[b][h][1] = sacc[b][h][2] = sacc[b][h][3] = 0.f;
                if constexpr (C::SCALED) {
                uint64_t sg2[NBLK], sg82[NBLK];
                uint32_t wa[NBLK][C::NI], wb[NBLK][C::NI];
#pragma unroll
                for (int b = 0; b < NBLK; ++b) {
                    const float sg = scale(ks, 16 * b + g), sg8 = scale(ks, 16 * b + g + 8);
                    sg2[b] = f2_pack(sg, sg);
                    sg82[b] = f2_pack(sg8, sg8);
                    const uint32_t kb = kt + b * 16 * D;
                    if constexpr (D == 128) {
                        // 128B swizzle: row e, 16B chunk x stored at chunk x ^ (e & 7).
                        const uint4 ka0 = lds128(kb + g * 128 + (((2 * c) ^ g) << 4));
                        const uint4 ka1 = lds128(kb + g * 128 + (((2 * c + 1) ^ g) << 4));
                        const uint4 kb0 = lds128(kb + (g + 8) * 128 + (((2 * c) ^ g) << 4));
                        const uint4 kb1 = lds128(kb + (g + 8) * 128 + (((2 * c + 1) ^ g) << 4));
                        wa[b][0] = ka0.x; wa[b][1] = ka0.y; wa[b][2] = ka0.z; wa[b][3] = ka0.w;
                        wa[b][4] = ka1.x; wa[b][5] = ka1.y; wa[b][6] = ka1.z; wa[b][7] = ka1.w;
                        wb[b][0] = kb0.x; wb[b][1] = kb0.y; wb[b][2] = kb0.z; wb[b][3] = kb0.w;
                        wb[b][4] = kb1.x; wb[b][5] = kb1.y; wb[b][6] = kb1.z; wb[b][7] = kb1.w;
                    } else {
                        // 64B swizzle: row e, 16B chunk x stored at chunk x ^ ((e >> 1) & 3).
                        const int sw = (g >> 1) & 3;
                        const uint4 ka = lds128(kb + g * 64 + ((c ^ sw) << 4));
                        const uint4 kc = lds128(kb + (g + 8) * 64 + ((c ^ sw) << 4));
                        wa[b][0] = ka.x; wa[b][1] = ka.y; wa[b][2] = ka.z; wa[b][3] = ka.w;
                        wb[b][0] = kc.x; wb[b][1] = kc.y; wb[b][2] = kc.z; wb[b][3] = kc.w;
                    }
                }
                // k_t = bf16(i8 * ks[t]) for 4 channels of token g (wa) and g+8 (wb),
                // against the q fragments of MMA i; two accumulator chains per block
#pragma unroll
                for (int i = 0; i < C::NI; ++i) {
#pragma unroll
                    for (int b = 0; b < NBLK; ++b) {
                        uint64_t a01, a23, b01, b23;
                        i8x4_to_f32x2(wa[b][i], a01, a23);
                        i8x4_to_f32x2(wb[b][i], b01, b23);
                        a01 = f2_mul(a01, sg2[b]);
                        a23 = f2_mul(a23, sg2[b]);
                        b01 = f2_mul(b01, sg82[b]);
                        b23 = f2_mul(b23, sg82[b]);
                        mma_bf16_16816(sacc[b][i & 1], pack_bf16x2_f2(a01), pack_bf16x2_f2(b01),
                                       pack_bf16x2_f2(a23), pack_bf16x2_f2(b23), qb[i][0], qb[i][1]);
                    }
                }
                } else {
                    // float rows: thread c's 16-byte chunks qk_chunk(c, k) of tokens g and g + 8
                    constexpr int NCH = C::ROW / 64;
                    uint4 ka[NBLK][NCH], kc[NBLK][NCH];
#pragma unroll
                    for (int b = 0; b < NBLK; ++b) {
#pragma unroll
                        for (int k = 0; k < NCH; ++k) {
                            const int gc = C::qk_chunk(c, k);
                            const uint32_t pb = kt + (uint32_t)(gc >> 3) * (C::T * 128) + b * 16 * 128;
                            const uint32_t sw = (uint32_t)(((gc & 7) ^ g) << 4);  // rows g, g + 8: swizzle phase g
                            ka[b][k] = lds128(pb + g * 128 + sw);
                            kc[b][k] = lds128(pb + (g + 8) * 128 + sw);
                        }
                    }
#pragma unroll
                    for (int i = 0; i < C::NI; ++i) {
#pragma unroll
                        for (int b = 0; b < NBLK; ++b) {
                            if constexpr (KV == Kv::BF16) {
                                // channels qk_ch(c, i) .. + 3: words 2(i&1), 2(i&1)+1 of chunk i/2
                                const uint4& A = ka[b][i >> 1];
                                const uint4& B = kc[b][i >> 1];
                                const int w = 2 * (i & 1);
                                mma_bf16_16816(sacc[b][i & 1], u4_word(A, w), u4_word(B, w), u4_word(A, w + 1),
                                               u4_word(B, w + 1), qb[i][0], qb[i][1]);
                            } else {
                                // f32: chunk i holds channels qk_ch(c, i) .. + 3; three bf16 terms each
                                const uint4& A = ka[b][i];
                                const uint4& B = kc[b][i];
                                uint32_t a0[3], a1[3], a2[3], a3[3];
                                split3_pair(__uint_as_float(A.x), __uint_as_float(A.y), a0[0], a0[1], a0[2]);
                                split3_pair(__uint_as_float(B.x), __uint_as_float(B.y), a1[0], a1[1], a1[2]);
                                split3_pair(__uint_as_float(A.z), __uint_as_float(A.w), a2[0], a2[1], a2[2]);
                                split3_pair(__uint_as_float(B.z), __uint_as_float(B.w), a3[0], a3[1], a3[2]);
#pragma unroll
                                for (int tm = 0; tm < 3; ++tm)
                                    mma_bf16_16816(sacc[b][i & 1], a0[tm], a1[tm], a2[tm], a3[tm], qb[i][0], qb[i][1]);
                            }
                        }
                    }
                }
#pragma unroll
                for (int b = 0; b < NBLK; ++b) {
                    float x = (sacc[b][0][0] + sacc[b][1][0]) + (sacc[b][0][1] + sacc[b][1][1]);
                    float y = (sacc[b][0][2] + sacc[b][1][2]) + (sacc[b][0][3] + sacc[b][1][3]);
                    x += __shfl_xor_sync(0xffffffffu, x, 1);
                    y += __shfl_xor_sync(0xffffffffu, y, 1);
                    x += __shfl_xor_sync(0xffffffffu, x, 2);
                    y += __shfl_xor_sync(0xffffffffu, y, 2);
                    if constexpr (MASKED) {
                        if (16 * b + g >= nv) x = -INFINITY;
                        if (16 * b + g + 8 >= nv) y = -INFINITY;
                    }
                    s_g[b] = x;
                    s_g8[b] = y;
                }
            }

            // ---- online softmax (base 2) with a lazy reference point: m2 moves
            // only when a score exceeds it by more than kSlack, so p <= 2^kSlack.
            float sm = fmaxf(s_g[0], s_g8[0]);
#pragma unroll
            for (int b = 1; b < NBLK; ++b) sm = fmaxf(sm, fmaxf(s_g[b], s_g8[b]));
            if (__any_sync(0xffffffffu, sm > m2 + kSlack)) {
                float bm = fmaxf(sm, __shfl_xor_sync(0xffffffffu, sm, 4));
                bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 8));
                bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 16));
                const float alpha = fast_exp2(m2 - bm);
                zsum *= alpha;
#pragma unroll
                for (int j = 0; j < C::NJ; ++j) {
                    acc[j][0] *= alpha;
                    acc[j][1] *= alpha;
                    acc[j][2] *= alpha;
                    acc[j][3] *= alpha;
                }
                m2 = bm;
            }

#pragma unroll
            for (int b = 0; b < NBLK; ++b) {
                const float p_g = fast_exp2(s_g[b] - m2), p_g8 = fast_exp2(s_g8[b] - m2);
                zsum += p_g + p_g8;
                // p as the B operand (k = tokens 2c, 2c+1, 2c+8, 2c+9; n = term g).
                // Lane (G, c) holds term c of its tokens G and G+8; thread (g, c)
                // pulls term g of tokens 2c, 2c+1 from the lanes of groups 2c, 2c+1.
                uint32_t terms;
                {
                    const uint32_t h = pack_bf16x2(p_g, p_g8);
                    const float r0 = p_g - bf16_lo_to_f32(h), r1 = p_g8 - bf16_hi_to_f32(h);
                    const uint32_t l = pack_bf16x2(r0, r1);
                    const uint32_t l2 = pack_bf16x2(r0 - bf16_lo_to_f32(l), r1 - bf16_hi_to_f32(l));
                    terms = c == 0 ? h : c == 1 ? l : c == 2 ? l2 : 0u;
                }
                const uint32_t tx = __shfl_sync(0xffffffffu, terms, 8 * c + (g & 3));
                const uint32_t ty = __shfl_sync(0xffffffffu, terms, 8 * c + 4 + (g & 3));
                const uint32_t pb0 = g < 3 ? __byte_perm(tx, ty, 0x5410) : 0u;
                const uint32_t pb1 = g < 3 ? __byte_perm(tx, ty, 0x7632) : 0u;

                // ---- p . V: A = V^T (rows = channels, k = tokens 2c, 2c+1, 2c+8, 2c+9)
                const int e0 = 16 * b + 2 * c, e1 = e0 + 1, e2 = e0 + 8, e3 = e0 + 9;
                if constexpr (C::SCALED) {
                const float v0s = scale(vs, e0), v1s = scale(vs, e1), v2s = scale(vs, e2), v3s = scale(vs, e3);
                const uint64_t s0 = f2_pack(v0s, v0s), s1 = f2_pack(v1s, v1s);
                const uint64_t s2 = f2_pack(v2s, v2s), s3 = f2_pack(v3s, v3s);
                // channels x..x+3 of the four tokens (words w0..w3) -> 4 MMAs, starting at
                // accumulator j0 (channel rows of the A tile: m = g -> word wa, m = g+8 -> word wb)
                auto pv_mma4 = [&](int j0, uint32_t wa0, uint32_t wa1, uint32_t wa2, uint32_t wa3, uint32_t wb0,
                                   uint32_t wb1, uint32_t wb2, uint32_t wb3) {
                    uint64_t a[4][2], bb[4][2];  // [token][pair]: channels (x, x+1), (x+2, x+3)
                    i8x4_to_f32x2(wa0, a[0][0], a[0][1]);
                    i8x4_to_f32x2(wa1, a[1][0], a[1][1]);
                    i8x4_to_f32x2(wa2, a[2][0], a[2][1]);
                    i8x4_to_f32x2(wa3, a[3][0], a[3][1]);
                    i8x4_to_f32x2(wb0, bb[0][0], bb[0][1]);
                    i8x4_to_f32x2(wb1, bb[1][0], bb[1][1]);
                    i8x4_to_f32x2(wb2, bb[2][0], bb[2][1]);
                    i8x4_to_f32x2(wb3, bb[3][0], bb[3][1]);
                    const uint64_t sc[4] = {s0, s1, s2, s3};
                    float fa[4][4], fb[4][4];
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        f2_unpack(f2_mul(a[t][0], sc[t]), fa[t][0], fa[t][1]);
                        f2_unpack(f2_mul(a[t][1], sc[t]), fa[t][2], fa[t][3]);
                        f2_unpack(f2_mul(bb[t][0], sc[t]), fb[t][0], fb[t][1]);
                        f2_unpack(f2_mul(bb[t][1], sc[t]), fb[t][2], fb[t][3]);
                    }
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        mma_bf16_16816(acc[j0 + e], pack_bf16x2(fa[0][e], fa[1][e]), pack_bf16x2(fb[0][e], fb[1][e]),
                                       pack_bf16x2(fa[2][e], fa[3][e]), pack_bf16x2(fb[2][e], fb[3][e]), pb0, pb1);
                    }
                };
                if constexpr (D == 128) {
                    // thread holds channels [16g, 16g+16) of its four tokens; rows e0..e3
                    // of this block sit at 128B swizzle phase (e & 7) == (2c, 2c+1, 2c, 2c+1)
                    const uint32_t vb = vt + b * 16 * 128;
                    const uint4 v0 = lds128(vb + (2 * c) * 128 + ((g ^ (2 * c)) << 4));
                    const uint4 v1 = lds128(vb + (2 * c + 1) * 128 + ((g ^ (2 * c + 1)) << 4));
                    const uint4 v2 = lds128(vb + (2 * c + 8) * 128 + ((g ^ (2 * c)) << 4));
                    const uint4 v3 = lds128(vb + (2 * c + 9) * 128 + ((g ^ (2 * c + 1)) << 4));
                    // accumulator j: channel 16g + j (m = g) and 16g + 8 + j (m = g + 8)
                    pv_mma4(0, v0.x, v1.x, v2.x, v3.x, v0.z, v1.z, v2.z, v3.z);
                    pv_mma4(4, v0.y, v1.y, v2.y, v3.y, v0.w, v1.w, v2.w, v3.w);
                } else {
                    // thread holds channels [8g, 8g+8) of its four tokens
                    const uint32_t vb = vt + b * 16 * 64;
                    const uint32_t off = ((((uint32_t)g >> 1) ^ (uint32_t)c) << 4) + (((uint32_t)g & 1u) << 3);
                    const uint2 v0 = lds64(vb + (2 * c) * 64 + off);
                    const uint2 v1 = lds64(vb + (2 * c + 1) * 64 + off);
                    const uint2 v2 = lds64(vb + (2 * c + 8) * 64 + off);
                    const uint2 v3 = lds64(vb + (2 * c + 9) * 64 + off);
                    // accumulator j: channel 8g + j (m = g) and 8g + 4 + j (m = g + 8)
                    pv_mma4(0, v0.x, v1.x, v2.x, v3.x, v0.y, v1.y, v2.y, v3.y);
                }
                } else {
                    // float rows: chunk g of every panel of tokens e0..e3; MMA j takes
                    // channels pv_ch(g, j) (m = g) and pv_ch(g, D/16 + j) (m = g + 8)
                    constexpr int NVC = C::PANELS, CE = C::CH_ELEMS;
                    uint4 vv[4][NVC];
                    const int er[4] = {e0, e1, e2, e3};
#pragma unroll
                    for (int t = 0; t < 4; ++t) {
                        const uint32_t sw = (uint32_t)((g ^ (er[t] & 7)) << 4);
#pragma unroll
                        for (int k = 0; k < NVC; ++k) {
                            vv[t][k] = lds128(vt + (uint32_t)k * (C::T * 128) + (uint32_t)er[t] * 128u + sw);
                            // past the segment end p is 0, but the row there may hold anything (NaN)
                            if constexpr (MASKED)
                                if (er[t] >= nv) vv[t][k] = make_uint4(0u, 0u, 0u, 0u);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < C::NJ; ++j) {
                        constexpr int H = D / 16;
                        if constexpr (KV == Kv::BF16) {
                            // bf16 pairs of two tokens for one channel: halves (j & 1) of word w
                            const uint32_t sel = (j & 1) ? 0x7632u : 0x5410u;
                            const int p0 = j / CE, w0 = (j % CE) >> 1, p1 = (H + j) / CE, w1 = ((H + j) % CE) >> 1;
                            mma_bf16_16816(acc[j], __byte_perm(u4_word(vv[0][p0], w0), u4_word(vv[1][p0], w0), sel),
                                           __byte_perm(u4_word(vv[0][p1], w1), u4_word(vv[1][p1], w1), sel),
                                           __byte_perm(u4_word(vv[2][p0], w0), u4_word(vv[3][p0], w0), sel),
                                           __byte_perm(u4_word(vv[2][p1], w1), u4_word(vv[3][p1], w1), sel), pb0, pb1);
                        } else {
                            const int p0 = j / CE, f0 = j % CE, p1 = (H + j) / CE, f1 = (H + j) % CE;
                            uint32_t a0[3], a1[3], a2[3], a3[3];
                            split3_pair(__uint_as_float(u4_word(vv[0][p0], f0)), __uint_as_float(u4_word(vv[1][p0], f0)),
                                        a0[0], a0[1], a0[2]);
                            split3_pair(__uint_as_float(u4_word(vv[0][p1], f1)), __uint_as_float(u4_word(vv[1][p1], f1)),
                                        a1[0], a1[1], a1[2]);
                            split3_pair(__uint_as_float(u4_word(vv[2][p0], f0)), __uint_as_float(u4_word(vv[3][p0], f0)),
                                        a2[0], a2[1], a2[2]);
                            split3_pair(__uint_as_float(u4_word(vv[2][p1], f1)), __uint_as_float(u4_word(vv[3][p1], f1)),
                                        a3[0], a3[1], a3[2]);
#pragma unroll
                            for (int tm = 0; tm < 3; ++tm)
                                mma_bf16_16816(acc[j], a0[tm], a1[tm], a2[tm], a3[tm], pb0, pb1);
                        }
                    }
                }
            }
        };
        using I1 = std::integral_constant<int, 1>;
        using INB = std::integral_constant<int, C::NB>;
        if (nv >= C::TPW) blocks(INB{}, std::false_type{});
        else if (nv > C::BOX && C::NB > 1) blocks(INB{}, std::true_type{});
        else if (nv > 0) blocks(I1{}, std::true_type{});
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);

        if (flags & kLast) {
            // ---- segment end: every warp leaves its state (m, z, acc) in reduction
            // buffer `par`; one warp per segment (in turn) merges the states into the
            // segment's partial and, with stream-K plans, finishes the row, while the
            // other warps go on with the next stage.
            const uint32_t par = seg_count & 1u, use = seg_count >> 1;
            float* buf = red + par * C::RED_FLOATS;
            float* mine = buf + warp * (D + 4);
            // the previous use of this buffer has been read by its finishing warp
            if (!mbar_wait_bounded(&red_free[par], (use & 1u) ^ 1u, abort_flag, kWaitLimitNs)) {
                *abort_flag = 1;
                if (lane == 0 && args.status) atomicOr(args.status, PP_DEV_WAIT_TIMEOUT);
                return;
            }
#pragma unroll
            for (int j = 0; j < C::NJ; ++j) {
                float a = acc[j][0] + acc[j][1];
                float b = acc[j][2] + acc[j][3];
                a += __shfl_xor_sync(0xffffffffu, a, 1);
                b += __shfl_xor_sync(0xffffffffu, b, 1);
                a += __shfl_xor_sync(0xffffffffu, a, 2);
                b += __shfl_xor_sync(0xffffffffu, b, 2);
                if (c == (j & 3)) {
                    // accumulator j holds channels pv_ch(g, j) and pv_ch(g, D/16 + j)
                    mine[C::pv_ch(g, j)] = a;
                    mine[C::pv_ch(g, D / 16 + j)] = b;
                }
            }
            float zt = zsum;
            zt += __shfl_xor_sync(0xffffffffu, zt, 4);
            zt += __shfl_xor_sync(0xffffffffu, zt, 8);
            zt += __shfl_xor_sync(0xffffffffu, zt, 16);
            if (lane == 0) {
                mine[D] = m2;
                mine[D + 1] = zt;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&red_bar[par]);
            if (warp == (int)(seg_count % C::NC)) {
                // what the row's finish reads from global memory goes out now, before the
                // wait for the other warps' states and the merge: the scratch token and
                // the row's first partial
                const uint32_t row = m0.x, row_segs = m1.w;
                ScratchVals<D> sc;
                sc.on = false;
                uint32_t first_seg = 0;
                if (args.finish) {
                    sc = scratch_of(row);
                    if (row_segs > 1) first_seg = __ldg(row_seg + row);
                }
                if (!mbar_wait_bounded(&red_bar[par], use & 1u, abort_flag, kWaitLimitNs)) {
                    *abort_flag = 1;
                    if (lane == 0 && args.status) atomicOr(args.status, PP_DEV_WAIT_TIMEOUT);
                    return;
                }
                // merge the NC warp states; lane owns channels [lane*E, lane*E + E)
                constexpr int E = D / 32;
                RegPartial<D> seg;
                float mx = -INFINITY;
#pragma unroll
                for (int w = 0; w < C::NC; ++w) mx = fmaxf(mx, buf[w * (D + 4) + D]);
                float sz = 0.f;
#pragma unroll
                for (int e = 0; e < E; ++e) seg.a[e] = 0.f;
#pragma unroll
                for (int w = 0; w < C::NC; ++w) {
                    const float mw = buf[w * (D + 4) + D];
                    const float f = mw == -INFINITY ? 0.f : fast_exp2(mw - mx);
#pragma unroll
                    for (int e = 0; e < E; ++e) seg.a[e] += buf[w * (D + 4) + lane * E + e] * f;
                    sz += buf[w * (D + 4) + D + 1] * f;
                }
                seg.mv = mx;
                seg.zv = sz;
                __syncwarp();
                if (lane == 0) mbar_arrive(&red_free[par]);
                if (args.finish && row_segs == 1) {
                    finish_out(row, 1u, seg, sc);
                } else {
                    float* dst = partials + (uint64_t)seg_slot * (D + 4);
#pragma unroll
                    for (int e = 0; e < E; ++e) dst[lane * E + e] = seg.a[e];
                    if (lane == 0) {
                        dst[D] = mx;
                        dst[D + 1] = sz;
                    }
                    if (args.finish) {
                        // publish the partial and count it; the CTA that counts the
                        // row's last segment merges all of them
                        __threadfence();
                        __syncwarp();
                        uint32_t done = 0;
                        if (lane == 0) done = atomicAdd(row_cnt + row, 1u) + 1u;
                        done = __shfl_sync(0xffffffffu, done, 0);
                        if (done == row_segs) {
                            __threadfence();
                            const float* rp = partials + (uint64_t)first_seg * (D + 4);
                            if (row_segs <= batch_segs<D>()) {
                                if (args.out_bf16)
                                    finish_split<D, __nv_bfloat16>(lane, row, row_segs, seg_slot - first_seg, seg, rp, sc,
                                                                   args.out);
                                else
                                    finish_split<D, float>(lane, row, row_segs, seg_slot - first_seg, seg, rp, sc, args.out);
                            } else {
                                finish_out(row, row_segs, GlobalPartials<D, true>{rp}, sc);
                            }
                            if (lane == 0) row_cnt[row] = 0u;  // zero again for the next call
                        }
                    }
                }
            }
            ++seg_count;
        }
    }
}

// ---------------------------------------------------------------- combine

struct CombineArgs {
    const unsigned char* ws;
    WsLayout l;
    const void* q;
    const float* sk;
    const float* sv;
    float scale_log2;
    void* out;
    uint32_t rows;
};

// One warp per row (fixed-split plans): the log-sum-exp merge of the row's
// partials and, in reference mode, the scratch token.
template <int D, typename QT, typename OT>
__global__ void __launch_bounds__(256) combine_kernel(const CombineArgs a) {
    pdl_wait_primary();
    const int lane = threadIdx.x & 31;
    const uint32_t r = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (r >= a.rows) return;
    const uint32_t* row_len = reinterpret_cast<const uint32_t*>(a.ws + a.l.row_len);
    const uint32_t* row_seg = reinterpret_cast<const uint32_t*>(a.ws + a.l.row_seg);
    const float* partials = reinterpret_cast<const float*>(a.ws + a.l.partials);
    const uint32_t s0 = row_seg[r], s1 = row_seg[r + 1];
    finish_row<D, OT>(lane, r, s1 - s0, row_len[r] == kInvalidRow,
                      GlobalPartials<D, false>{partials + (uint64_t)s0 * (D + 4)},
                      load_scratch<D, QT>(lane, r, a.q, a.sk, a.sv, a.scale_log2), a.out);
}

template <int D, typename QT, Kv KV, int NCW = 0>
cudaError_t launch_attn_t(const AttnLaunch& L, cudaStream_t stream) {
    using C = Cfg<D, KV, NCW>;
    AttnArgs args{};
    args.q = L.q;
    args.q_stride = L.q_stride;
    args.ws = L.ws;
    args.partials = reinterpret_cast<float*>(L.ws + L.layout.partials);
    args.l = L.layout;
    args.capacity = L.arena.capacity;
    args.ks_mis = L.ks_mis;
    args.vs_mis = L.vs_mis;
    args.scale_log2 = L.scale_log2;
    args.status = L.status;
    args.finish = L.split == 0 ? 1u : 0u;
    args.prefetch = L.prefetch ? 1u : 0u;
    args.out_bf16 = L.out_dtype == PP_DTYPE_BF16 ? 1u : 0u;
    args.out = L.out;
    args.sk = L.scratch_k;
    args.sv = L.scratch_v;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(L.max_ctas);
    cfg.blockDim = dim3(C::THREADS);
    cfg.dynamicSmemBytes = C::SMEM_BYTES;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = L.use_pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, attn_kernel<D, QT, KV, NCW>, L.tails, L.map_k_stage, L.map_v_stage, L.map_ks,
                              L.map_vs, args);
}

template <int D, typename QT, typename OT>
cudaError_t launch_combine_t(const AttnLaunch& L, cudaStream_t stream) {
    CombineArgs a{};
    a.ws = L.ws;
    a.l = L.layout;
    a.q = L.q;
    a.sk = L.scratch_k;
    a.sv = L.scratch_v;
    a.scale_log2 = L.scale_log2;
    a.out = L.out;
    a.rows = L.arena.rows;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((L.arena.rows + 7) / 8);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = L.use_pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, combine_kernel<D, QT, OT>, a);
}

// One bounded wait on an mbarrier that nothing completes: the wait gives up
// after limit_ns and the kernel reports PP_DEV_WAIT_TIMEOUT, as every wait in
// this library does, instead of hanging.
__global__ void wait_probe_kernel(uint32_t* status, uint64_t limit_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    volatile int never = 0;
    if (!mbar_wait_bounded(&bar, 0u, &never, limit_ns)) atomicOr(status, PP_DEV_WAIT_TIMEOUT);
}

}  // namespace

cudaError_t launch_wait_probe(uint32_t* status, uint64_t limit_ns, cudaStream_t stream) {
    wait_probe_kernel<<<1, 32, 0, stream>>>(status, limit_ns);
    return cudaGetLastError();
}

namespace {
template <int D, typename QT, Kv KV, int NCW = 0>
cudaError_t configure_one() {
    return cudaFuncSetAttribute(attn_kernel<D, QT, KV, NCW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                Cfg<D, KV, NCW>::SMEM_BYTES);
}
template <Kv KV>
cudaError_t configure_kind() {
    cudaError_t e;
    if ((e = configure_one<128, float, KV>()) != cudaSuccess) return e;
    if ((e = configure_one<128, __nv_bfloat16, KV>()) != cudaSuccess) return e;
    if ((e = configure_one<64, float, KV>()) != cudaSuccess) return e;
    if ((e = configure_one<64, __nv_bfloat16, KV>()) != cudaSuccess) return e;
    if constexpr (KV == Kv::I8) {
        if ((e = configure_one<64, float, KV, PP_ATTN_NC_SHORT_D64>()) != cudaSuccess) return e;
        if ((e = configure_one<64, __nv_bfloat16, KV, PP_ATTN_NC_SHORT_D64>()) != cudaSuccess) return e;
    }
    return cudaSuccess;
}
template <Kv KV>
cudaError_t launch_kind(const AttnLaunch& L, cudaStream_t stream) {
    const bool bq = L.q_dtype == PP_DTYPE_BF16;
    if (L.arena.head_dim == 128)
        return bq ? launch_attn_t<128, __nv_bfloat16, KV>(L, stream) : launch_attn_t<128, float, KV>(L, stream);
    if constexpr (KV == Kv::I8) {
        if (L.short_stages)
            return bq ? launch_attn_t<64, __nv_bfloat16, KV, PP_ATTN_NC_SHORT_D64>(L, stream)
                      : launch_attn_t<64, float, KV, PP_ATTN_NC_SHORT_D64>(L, stream);
    }
    return bq ? launch_attn_t<64, __nv_bfloat16, KV>(L, stream) : launch_attn_t<64, float, KV>(L, stream);
}
}  // namespace

cudaError_t configure_attention_kernels(int /*device*/) {
    cudaError_t e;
    if ((e = configure_kind<Kv::I8>()) != cudaSuccess) return e;
    if ((e = configure_kind<Kv::BF16>()) != cudaSuccess) return e;
    return configure_kind<Kv::F32>();
}

uint32_t attention_scale_box_elems() { return Cfg<128>::SC_BOX; }
bool attention_short_stages(uint32_t head_dim, uint32_t rows, uint32_t capacity, uint32_t ctas) {
    return head_dim == 64 && ctas &&
           (uint64_t)rows * capacity <= (uint64_t)PP_ATTN_SHORT_TOKENS_PER_CTA * ctas;
}
uint32_t attention_stage_tokens(uint32_t head_dim, bool short_stages) {
    if (head_dim == 128) return Cfg<128>::STAGE_BOX;
    return short_stages ? Cfg<64, Kv::I8, PP_ATTN_NC_SHORT_D64>::STAGE_BOX : Cfg<64>::STAGE_BOX;
}
uint32_t attention_float_stage_tokens(uint32_t head_dim, int kv_kind) {
    if (kv_kind == kKvBf16) return head_dim == 128 ? Cfg<128, Kv::BF16>::T : Cfg<64, Kv::BF16>::T;
    return head_dim == 128 ? Cfg<128, Kv::F32>::T : Cfg<64, Kv::F32>::T;
}

cudaError_t launch_plan(const AttnLaunch& L, cudaStream_t stream) {
    PlanArgs a{};
    a.lengths = L.lengths;
    a.ws = L.ws;
    a.l = L.layout;
    a.rows = L.arena.rows;
    a.heads = L.arena.heads;
    a.capacity = L.arena.capacity;
    a.split = L.split;
    a.scratch = L.scratch_k ? 1u : 0u;
    a.max_ctas = L.max_ctas;
    a.min_tokens = PP_PLAN_MIN_TOKENS;
    // a split row costs its CTAs a partial merge and the row a final merge: measured worth about
    // 1024 int8 tokens of head_dim 64 and fewer than 553 of the wider rows
    a.whole_row_slack = (L.kv_kind == kKvInt8 && L.arena.head_dim == 64) ? 1024u : 512u;
    a.status = L.status;
    return launch_pdl(plan_kernel, dim3(1), dim3(1024), stream, a);
}

cudaError_t launch_attention(const AttnLaunch& L, cudaStream_t stream) {
    if (L.kv_kind == kKvBf16) return launch_kind<Kv::BF16>(L, stream);
    if (L.kv_kind == kKvF32) return launch_kind<Kv::F32>(L, stream);
    return launch_kind<Kv::I8>(L, stream);
}

cudaError_t launch_combine(const AttnLaunch& L, cudaStream_t stream) {
    const bool bq = L.q_dtype == PP_DTYPE_BF16, bo = L.out_dtype == PP_DTYPE_BF16;
    if (L.arena.head_dim == 128) {
        if (bq) return bo ? launch_combine_t<128, __nv_bfloat16, __nv_bfloat16>(L, stream)
                          : launch_combine_t<128, __nv_bfloat16, float>(L, stream);
        return bo ? launch_combine_t<128, float, __nv_bfloat16>(L, stream) : launch_combine_t<128, float, float>(L, stream);
    }
    if (bq) return bo ? launch_combine_t<64, __nv_bfloat16, __nv_bfloat16>(L, stream)
                      : launch_combine_t<64, __nv_bfloat16, float>(L, stream);
    return bo ? launch_combine_t<64, float, __nv_bfloat16>(L, stream) : launch_combine_t<64, float, float>(L, stream);
}

}  // namespace pp
