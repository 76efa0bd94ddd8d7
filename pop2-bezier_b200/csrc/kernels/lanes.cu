// Per-lane random streams of the branch scheduler.
//
// The reference seeds lane i of a parallel generation with `base + i`
// (parallel_seed, app/src/inference/batch.rs:9-11) and draws each sampling
// uniform from that lane's own generator, only while the lane is ready
// (device::draw_uniforms over the ready lanes, batch.rs:747-754).  Here a
// lane's stream is counter based: draw n of the lane seeded s is
//   u(s, n) = top 24 bits of mix(s + (n + 1) * 0x9E3779B97F4A7C15) / 2^24
// where mix is the SplitMix64 output function (Steele, Lea and Flood,
// "Fast splittable pseudorandom number generators", OOPSLA 2014), i.e. the
// n-th output of a SplitMix64 generator seeded with s.  The value depends only
// on (seed, lane, draw count), never on which shard or batch row the lane
// occupies, so a run sharded over GPUs draws exactly what one GPU would.
// The draw counters live on the device and advance only for active lanes, so
// a decode loop needs no host round trip per sampled field.
#include "common.cuh"
#include "lanes.cuh"
#include "../host/internal.h"

namespace pp {
namespace {

__global__ void __launch_bounds__(256) lane_uniforms_kernel(const uint64_t* __restrict__ seeds,
                                                            uint64_t* __restrict__ draws,
                                                            const uint32_t* __restrict__ active, uint32_t rows,
                                                            float* __restrict__ out) {
    const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    if (active[r]) {
        const uint64_t n = draws[r];
        out[r] = lane_uniform(seeds[r], n);
        draws[r] = n + 1;
    } else {
        out[r] = 0.f;
    }
}

}  // namespace

cudaError_t launch_lane_uniforms(const uint64_t* seeds, uint64_t* draws, const uint32_t* active, uint32_t rows,
                                 float* out, cudaStream_t stream) {
    lane_uniforms_kernel<<<(rows + 255) / 256, 256, 0, stream>>>(seeds, draws, active, rows, out);
    return cudaGetLastError();
}

}  // namespace pp
