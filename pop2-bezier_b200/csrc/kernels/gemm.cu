// Decode-row GEMM for the projections of the decoder step:
//   out[m, n] = sum_k x[m, k] * w[n, k]      (m <= 16 rows, bf16 in/out, f32 accumulate)
// replacing the reference's `matmul(&w.t())` on the rows of a decode step
// (app/src/model/batch.rs:134,155-170).  With at most 16 rows the product is a
// weight stream: every byte of w is read once and used 16 times, so the
// kernel is built to move w at HBM speed:
//   * persistent CTAs, one per SM; CTA i owns a contiguous range of 8-row
//     blocks of w, so its weights are one contiguous stretch of memory;
//   * w is packed once (pack_kernel, at weight-load time) into 8-row blocks
//     of [k / 64][8 rows][128 bytes] with the 16-byte chunks of row r XOR-ed
//     by r, the layout the ldmatrix reads want without bank conflicts; a stage
//     of 8 rows x kc k (kc 1024, or 512 when x leaves little room) is then one
//     contiguous bulk copy of 16 (8) KB: a copy costs a fixed ~170 ns of the
//     SM's copy engine whatever its size, so copies of 1-2 KB stream at 6-12
//     GB/s per SM and copies of 16 KB at the HBM share (~42 GB/s per SM);
//   * x (16 rows x k) is copied into shared memory (16 KB tensor copies,
//     128-byte swizzle, no multicast) and stays; when it would leave the ring
//     fewer than 8 stages, k is taken in passes of kp and the x slice of the
//     next pass replaces the last once every warp is done with it (the w ring
//     keeps streaming meanwhile);
//   * each of the 8 consumer warps owns whole 8-row blocks (the CTA's blocks
//     in waves of 8) and the stage order interleaves the stages of a wave's
//     blocks, so eight stages are in the tensor cores at once; the producer
//     warp only fills the ring once, after that the warp that has consumed a
//     stage re-issues the stage one ring further into the same slot (no
//     central producer loop to wait on, no empty barriers): per pair of
//     16-k steps one ldmatrix of w (the B operand: the block's 8 output
//     columns), one ldmatrix of x per step (the A operand: the 16 decode
//     rows) and one mma.sync m16n8k16 with f32 accumulators; the warp writes
//     its block's bf16 outputs when the last stage is done (one warp sums a
//     block in k order: deterministic);
//   * w does not depend on the previous kernel, so the producer warp issues
//     the first ring of w copies before griddepcontrol.wait (programmatic
//     dependent launch); the x copies follow the wait.
// Every wait is bounded; a timeout sets PP_DEV_WAIT_TIMEOUT and returns.
#include "common.cuh"
#include "../host/internal.h"

namespace pp {
namespace {

constexpr int kWarps = 8;                     // consumer warps
constexpr int kThreads = (kWarps + 1) * 32;   // + producer warp
constexpr int kKBox = 64;                     // k per tensor copy (128 bytes of bf16)
constexpr int kKC = 512;                      // k per x chunk
constexpr int kXBoxBytes = 16 * 128;          // one 64-k chunk of 16 rows
constexpr int kXChunkBytes = (kKC / kKBox) * kXBoxBytes;  // one copy of x: [k chunk][row][128 B]
constexpr int kMaxStages = 24;
constexpr int kMaxXChunks = 16;               // x arrives in chunks of kKC (k <= 16 * 512)
constexpr int kBarBytes = (kMaxStages + kMaxXChunks + kWarps) * 8 + 16;
constexpr int kSmemCap = 232448;              // dynamic shared memory of one CTA
constexpr uint64_t kGemmWaitNs = 2000000000ull;
static_assert(kXBoxBytes % 1024 == 0 && kXChunkBytes % 1024 == 0, "swizzled x tiles 1024B-aligned");

struct GemmArgs {
    const unsigned char* w;  // packed weights
    __nv_bfloat16* out;
    uint64_t ldo;
    uint32_t m, n, k, stages, blocks;  // blocks: 8-row blocks of w
    uint32_t kc_len;                   // k per w stage
    uint32_t kp, passes;               // k per x pass (a multiple of kc_len and 512), passes
    uint32_t off_w, off_bar;
    uint32_t* status;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// Byte address of 16-byte chunk `chunk` of row `row` in a 128B-swizzled tile.
__device__ __forceinline__ uint32_t swz(uint32_t tile, uint32_t row, uint32_t chunk) {
    return tile + row * 128u + ((chunk ^ (row & 7u)) << 4);
}

__global__ void __launch_bounds__(kThreads, 1)
    rows_gemm_kernel(const __grid_constant__ CUtensorMap map_x, const GemmArgs a) {
    extern __shared__ unsigned char smem_raw[];
    unsigned char* smem =
        reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
    uint64_t* x_full = full + kMaxStages;    // [kMaxXChunks]: chunk loaded (once per x round)
    uint64_t* x_free = x_full + kMaxXChunks;  // [kWarps]: warp w is done with an x round
    volatile int* abort_flag = reinterpret_cast<volatile int*>(x_free + kWarps);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t S = a.stages;
    const uint32_t b_lo = (uint32_t)(((uint64_t)blockIdx.x * a.blocks) / gridDim.x);
    const uint32_t b_hi = (uint32_t)(((uint64_t)(blockIdx.x + 1) * a.blocks) / gridDim.x);
    const uint32_t spb = (a.k + a.kc_len - 1) / a.kc_len;  // w stages per block
    const uint32_t xch = a.kp / kKC;                       // x chunks per round
    const uint32_t stage_bytes = a.kc_len * 16;  // 8 rows x kc_len bf16
    const uint32_t nb = b_hi - b_lo, total = nb * spb;
    // x rounds: one per (wave, pass) when k takes several passes, else one for all
    const uint32_t waves = (nb + kWarps - 1) / kWarps;
    const uint32_t rounds = a.passes > 1 ? waves * a.passes : 1u;
    // stage order: wave v (blocks b_lo + 8v .. + nw - 1), then k chunk, then block:
    // stage v*8*spb + kc*nw + j is chunk kc of block b_lo + 8v + j, consumed by warp j
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < S; ++s) mbar_init(&full[s], 1);
        for (uint32_t ch = 0; ch < xch; ++ch) mbar_init(&x_full[ch], 1);
        for (int w = 0; w < kWarps; ++w) mbar_init(&x_free[w], 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    auto seg_bytes = [&](uint32_t kc) { return min(a.kc_len, a.k - kc * a.kc_len) * 2u; };
    // stage `it` (lane 0): one contiguous copy of the packed block's k range
    auto issue = [&](uint32_t it) {
        const uint32_t v = it / (kWarps * spb), rem = it % (kWarps * spb);
        const uint32_t nw = min((uint32_t)kWarps, nb - kWarps * v);
        const uint32_t kc = rem / nw, blk = b_lo + kWarps * v + rem % nw, slot = it % S;
        const uint32_t bytes = seg_bytes(kc) * 8;  // 8 rows
        mbar_arrive_expect_tx(&full[slot], bytes);
        bulk_load(smem + a.off_w + slot * stage_bytes, a.w + (uint64_t)blk * a.k * 16 + (uint64_t)kc * a.kc_len * 16,
                  bytes, &full[slot]);
    };

    if (warp == kWarps) {
        // ------------------------------------------------------------ producer
        if (lane == 0) tma_prefetch_desc(&map_x);
        // w for the first ring before the previous kernel has finished; x after it
        if (lane != 0) return;
        const uint32_t first = total < S ? total : S;
        for (uint32_t it = 0; it < first; ++it) issue(it);
        pdl_wait_primary();
        pdl_launch_dependents();
        // x round rd = pass rd % passes (of wave rd / passes); every chunk of the
        // region is loaded each round (past k: zero fill) so barrier phases match rounds
        for (uint32_t rd = 0; rd < rounds; ++rd) {
            if (rd > 0) {
                // the warps that read round rd - 1: those with a block in its wave
                const uint32_t vp = (rd - 1) / a.passes, nwp = min((uint32_t)kWarps, nb - kWarps * vp);
                volatile int never = 0;
                for (uint32_t w = 0; w < nwp; ++w)
                    if (!mbar_wait_bounded(&x_free[w], (rd - 1) & 1u, &never, kGemmWaitNs)) {
                        *abort_flag = 1;
                        if (a.status) atomicOr(a.status, PP_DEV_WAIT_TIMEOUT);
                        return;
                    }
            }
            const uint32_t k_first = (rd % a.passes) * a.kp;
            for (uint32_t ch = 0; ch < xch; ++ch) {
                mbar_arrive_expect_tx(&x_full[ch], kXChunkBytes);
                tma_load_3d(smem + ch * kXChunkBytes, &map_x, &x_full[ch], 0, 0,
                            (int32_t)((k_first + ch * kKC) / kKBox));
            }
        }
        return;
    }

    // ---------------------------------------------------------------- consumers
    const int g = lane >> 2, c = lane & 3;
    const uint32_t q = (uint32_t)lane >> 3, r = (uint32_t)lane & 7u;  // ldmatrix: matrix q, row r
    const uint32_t xs = smem_addr(smem), wsm = smem_addr(smem + a.off_w);
    // a wait gave up (2 s): report, then keep the CTA alive 1 ms more so that
    // copies this warp issued land before its shared memory goes away
    auto fail = [&]() {
        *abort_flag = 1;
        if (lane == 0) {
            if (a.status) atomicOr(a.status, PP_DEV_WAIT_TIMEOUT);
            const uint64_t t0 = global_timer_ns();
            while (global_timer_ns() - t0 < 1000000ull) {
            }
        }
    };
    // x_free[w] completes one phase per round warp w has read, in order; the
    // producer waits for round r - 1 only on the warps with a block in its wave
    // and loads round r after, so no warp runs two phases ahead of that wait
    uint32_t rd_have = ~0u;  // x round this warp is reading
    auto release = [&]() {
        __syncwarp();
        if (lane == 0) mbar_arrive(&x_free[warp]);
    };
    for (uint32_t v = 0; kWarps * v < nb; ++v) {
        const uint32_t nw = min((uint32_t)kWarps, nb - kWarps * v);
        if ((uint32_t)warp >= nw) {  // later waves are never larger: this warp is done
            if (rounds > 1 && rd_have != ~0u) release();  // its last round (of the previous wave)
            break;
        }
        const uint32_t blk = b_lo + kWarps * v + warp;
        float acc[2][4];  // two accumulator chains (even / odd k steps)
#pragma unroll
        for (int h = 0; h < 2; ++h) acc[h][0] = acc[h][1] = acc[h][2] = acc[h][3] = 0.f;
        for (uint32_t kc = 0; kc < spb; ++kc) {
            const uint32_t it = v * kWarps * spb + kc * nw + warp, slot = it % S;
            const uint32_t k0 = kc * a.kc_len;  // first k of the stage
            const uint32_t ps = k0 / a.kp, kx = k0 - ps * a.kp;  // pass, k within the x region
            const uint32_t rd = rounds > 1 ? v * a.passes + ps : 0u;
            if (rd != rd_have) {
                if (rounds > 1 && rd_have != ~0u) release();  // done with the previous round
                rd_have = rd;
            }
            // the x chunks this stage reads (a completed phase is seen again until this warp releases it)
            for (uint32_t ch = kx / kKC; ch < (kx + a.kc_len + kKC - 1) / kKC && ch < xch; ++ch)
                if (!mbar_wait_bounded(&x_full[ch], rd & 1u, abort_flag, kGemmWaitNs)) return fail();
            if (!mbar_wait_bounded(&full[slot], (it / S) & 1u, abort_flag, kGemmWaitNs)) return fail();
            const uint32_t wt = wsm + slot * stage_bytes;
            const uint32_t pairs = seg_bytes(kc) / 64;  // pairs of 16-k steps (32 k = 64 bytes of a row)
#pragma unroll 4
            for (uint32_t p2 = 0; p2 < pairs; ++p2) {
                // steps 2p, 2p + 1: 64-k chunk p / 2, 16-byte chunks 4 (p % 2) + q of rows r
                // (the block's 8 output columns)
                uint32_t b0, b1, b2, b3;
                ldsm_x4(swz(wt + (p2 >> 1) * 1024u, r, 4u * (p2 & 1u) + q), b0, b1, b2, b3);
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    // x: 16-k step kk of the whole row = x tile kk / 4, 16-byte chunk 2 (kk % 4) + (q >> 1),
                    // rows r + 8 (q & 1) (matrices: rows 0-7 / 8-15 x k 0-7 / 8-15)
                    const uint32_t kk = kx / 16 + 2 * p2 + h;
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4(swz(xs + (kk >> 2) * kXBoxBytes, r + 8u * (q & 1u), 2u * (kk & 3u) + (q >> 1)), a0, a1,
                            a2, a3);
                    mma_bf16_16816(acc[h], a0, a1, a2, a3, h ? b2 : b0, h ? b3 : b1);
                }
            }
            __syncwarp();
            // the slot is free: refill it with the stage one ring further on
            if (lane == 0 && it + S < total) issue(it + S);
        }
        // accumulator layout: (row g, columns 2c, 2c+1) and (row g + 8, the same columns)
        const uint32_t col = blk * 8u + 2u * c;
        if (col < a.n) {
            if (g < (int)a.m)
                *reinterpret_cast<uint32_t*>(a.out + (uint64_t)g * a.ldo + col) =
                    pack_bf16x2(acc[0][0] + acc[1][0], acc[0][1] + acc[1][1]);
            if (g + 8 < (int)a.m)
                *reinterpret_cast<uint32_t*>(a.out + (uint64_t)(g + 8) * a.ldo + col) =
                    pack_bf16x2(acc[0][2] + acc[1][2], acc[0][3] + acc[1][3]);
        }
    }
}

struct GemmPlan {
    uint32_t stages, kc_len, kp, passes, off_w, off_bar, smem;
};

// Shared-memory plan for k: the x region (one 16 KB chunk per 512 k), then
// the w ring (stages of 8 rows x 1024 k, as many as fit, at most 24), then the
// barriers.  x stays whole when that leaves at least 8 stages; otherwise k is
// taken in passes whose x slice leaves exactly 8.
bool plan_for(uint32_t k, GemmPlan& p) {
    constexpr uint32_t kStage = 1024 * 16, kMinStages = 8;
    const uint32_t fixed = kBarBytes + 1024;
    const uint32_t whole = (k + kKC - 1) / kKC;  // x chunks for all of k
    uint32_t xc = whole;
    if (xc > (uint32_t)kMaxXChunks || fixed + xc * kXChunkBytes + kMinStages * kStage > (uint32_t)kSmemCap) {
        xc = (kSmemCap - fixed - kMinStages * kStage) / kXChunkBytes;
        xc &= ~1u;  // passes of whole w stages (1024 k = 2 x chunks)
    }
    if (xc == 0) return false;
    p.kc_len = 1024;
    p.kp = xc * kKC;
    p.passes = (k + p.kp - 1) / p.kp;
    if (p.passes == 1) p.kp = whole * kKC;  // one round: all of x
    const uint32_t x_bytes = xc * kXChunkBytes;
    const uint32_t s = (kSmemCap - fixed - x_bytes) / kStage;
    p.stages = s < (uint32_t)kMaxStages ? s : (uint32_t)kMaxStages;
    p.off_w = x_bytes;
    p.off_bar = p.off_w + p.stages * kStage;
    p.smem = p.off_bar + kBarBytes + 1024;
    return true;
}

}  // namespace

bool rows_gemm_supported(uint32_t k) {
    GemmPlan p;
    return plan_for(k, p);
}

cudaError_t configure_rows_gemm() {
    return cudaFuncSetAttribute(rows_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap);
}

cudaError_t launch_rows_gemm(const CUtensorMap& map_x, const void* packed_w, void* out, uint64_t ldo, uint32_t m,
                             uint32_t n, uint32_t k, uint32_t num_sms, uint32_t* status, cudaStream_t stream) {
    GemmPlan p;
    if (!plan_for(k, p)) return cudaErrorInvalidValue;
    GemmArgs a{};
    a.w = reinterpret_cast<const unsigned char*>(packed_w);
    a.out = reinterpret_cast<__nv_bfloat16*>(out);
    a.ldo = ldo;
    a.m = m;
    a.n = n;
    a.k = k;
    a.stages = p.stages;
    a.kc_len = p.kc_len;
    a.kp = p.kp;
    a.passes = p.passes;
    a.blocks = n / 8;
    a.off_w = p.off_w;
    a.off_bar = p.off_bar;
    a.status = status;
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(a.blocks < num_sms ? a.blocks : num_sms);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, rows_gemm_kernel, map_x, a);
}

namespace {
// w [n, k] (row stride ldw) -> packed: block b = rows 8b..8b+7 at b * k * 16
// bytes, as [k / 64][row r][128 bytes] with 16-byte chunk c of row r stored at
// chunk c ^ r.  One thread per 16 bytes.
__global__ void __launch_bounds__(256) pack_kernel(const uint4* __restrict__ w, uint64_t ldw16, uint32_t n, uint32_t k,
                                                   uint4* __restrict__ packed) {
    const uint32_t per_row = k / 8;  // 16-byte pieces per row
    const uint64_t total = (uint64_t)n * per_row;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const uint32_t row = (uint32_t)(i / per_row), piece = (uint32_t)(i % per_row);
        const uint32_t blk = row / 8, r = row % 8, chunk64 = piece / 8, c = piece % 8;
        const uint64_t dst = (uint64_t)blk * (k / 8) * 8 + (uint64_t)chunk64 * 64 + r * 8 + (c ^ r);
        packed[dst] = w[(uint64_t)row * ldw16 + piece];
    }
}
}  // namespace

cudaError_t launch_rows_gemm_pack(const void* w, uint64_t ldw, uint32_t n, uint32_t k, void* packed,
                                  cudaStream_t stream) {
    const uint64_t total = (uint64_t)n * (k / 8);
    const uint64_t blocks = (total + 255) / 256;
    pack_kernel<<<(uint32_t)(blocks < 148u * 16u ? blocks : 148u * 16u), 256, 0, stream>>>(
        reinterpret_cast<const uint4*>(w), ldw / 8, n, k, reinterpret_cast<uint4*>(packed));
    return cudaGetLastError();
}

}  // namespace pp
