// Host-side batch geometry, write-offset validation and the branch scheduler.
#include <algorithm>
#include <cstdio>
#include <numeric>
#include <vector>

#include "../kernels/lanes.cuh"
#include "internal.h"

extern "C" {

// app/src/model/batch_geometry.rs:4-16: logical rows * guidance (CFG 1|2) must
// be non-zero, fit u32, and 9 attribute indices per logical row must fit u32.
int32_t pp_b200_checked_batch_rows(uint64_t logical_rows, uint32_t guidance, uint64_t* physical_rows) {
    if (logical_rows == 0 || (guidance != 1 && guidance != 2))
        return pp::fail_msg(PP_STATUS_PRECONDITION, "parallel row count must be non-zero and CFG branches 1 or 2");
    if (logical_rows > UINT64_MAX / guidance)
        return pp::fail_msg(PP_STATUS_PRECONDITION, "parallel rows times CFG branches overflow");
    const uint64_t physical = logical_rows * guidance;
    if (physical > 0xffffffffull)
        return pp::fail_msg(PP_STATUS_PRECONDITION, "physical rows exceed the device U32 index range");
    if (logical_rows > UINT64_MAX / 9 || logical_rows * 9 > 0xffffffffull)
        return pp::fail_msg(PP_STATUS_PRECONDITION, "parallel attribute count exceeds the device U32 index range");
    if (physical_rows) *physical_rows = physical;
    return PP_STATUS_OK;
}

// app/src/model/write_plan.rs:27-45 with the arena capacity in place of
// MAX_CONTEXT: non-empty rows/heads/width, every offset leaves a slot, and
// rows*heads*width*4 bytes of u32 indices are representable.
int32_t pp_b200_check_write_offsets(const uint64_t* past_lens, uint64_t count, uint32_t heads, uint32_t head_dim,
                                    uint32_t capacity) {
    if (!past_lens || count == 0 || heads == 0 || head_dim == 0)
        return pp::fail_msg(PP_STATUS_PRECONDITION, "write plan requires nonempty rows, heads and width");
    for (uint64_t i = 0; i < count; ++i)
        if (past_lens[i] >= capacity)
            return pp::fail_msg(PP_STATUS_PRECONDITION, "write plan offsets must leave a slot inside the maximum context");
    if (count > UINT64_MAX / heads) return pp::fail_msg(PP_STATUS_PRECONDITION, "write plan row count overflow");
    const uint64_t rows = count * heads;
    if (rows > UINT64_MAX / head_dim) return pp::fail_msg(PP_STATUS_PRECONDITION, "write plan index count overflow");
    const uint64_t elems = rows * head_dim;
    if (elems > UINT64_MAX / 4) return pp::fail_msg(PP_STATUS_PRECONDITION, "write plan index byte count overflow");
    return PP_STATUS_OK;
}

// Longest-processing-time partition: branches sorted by cost (descending,
// ties by index) are placed one by one on the currently lightest shard (ties
// by lowest shard index).  Deterministic, and within 4/3 of the optimal
// makespan.  Weak scaling of equal branches reduces to contiguous
// round-robin blocks of equal size.
int32_t pp_b200_sched_partition(const uint64_t* cost, uint32_t n_branches, uint32_t n_shards, uint32_t* shard_of_branch,
                                uint64_t* shard_cost) {
    if (!cost || !shard_of_branch || n_branches == 0 || n_shards == 0)
        return pp::fail_msg(PP_STATUS_PRECONDITION, "branch partition needs branches, shards and output storage");
    std::vector<uint32_t> order(n_branches);
    std::iota(order.begin(), order.end(), 0u);
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return cost[a] > cost[b]; });
    std::vector<uint64_t> load(n_shards, 0);
    std::vector<uint32_t> count(n_shards, 0);
    for (uint32_t b : order) {
        uint32_t best = 0;
        for (uint32_t s = 1; s < n_shards; ++s)
            if (load[s] < load[best] || (load[s] == load[best] && count[s] < count[best])) best = s;
        shard_of_branch[b] = best;
        load[best] += cost[b];
        count[best] += 1;
    }
    if (shard_cost)
        for (uint32_t s = 0; s < n_shards; ++s) shard_cost[s] = load[s];
    return PP_STATUS_OK;
}

// parallel_seed (app/src/inference/batch.rs:9-11): lane i of a parallel
// generation seeded `base` draws from the stream seeded base + i (wrapping).
uint64_t pp_b200_sched_lane_seed(uint64_t base, uint64_t lane) { return base + lane; }

// Host restatement of the device lane streams (lanes.cuh), bit for bit.
float pp_b200_sched_uniform(uint64_t lane_seed, uint64_t draw) { return pp::lane_uniform(lane_seed, draw); }

int32_t pp_b200_sched_uniforms(const uint64_t* lane_seeds, uint64_t* draws, const uint32_t* active, uint32_t rows,
                               float* out, void* stream) {
    if (!lane_seeds || !draws || !active || !out || rows == 0)
        return pp::fail_msg(PP_STATUS_PRECONDITION, "lane uniforms need seeds, draw counters, the active mask, "
                                                    "an output and at least one row");
    if (reinterpret_cast<uintptr_t>(lane_seeds) % 8 || reinterpret_cast<uintptr_t>(draws) % 8 ||
        reinterpret_cast<uintptr_t>(active) % 4 || reinterpret_cast<uintptr_t>(out) % 4)
        return pp::fail_msg(PP_STATUS_PRECONDITION, "lane uniforms: seeds and draws must be 8-byte aligned, "
                                                    "active and out 4-byte aligned");
    const cudaError_t e = pp::launch_lane_uniforms(lane_seeds, draws, active, rows, out, (cudaStream_t)stream);
    if (e != cudaSuccess) {
        char msg[256];
        snprintf(msg, sizeof msg, "EXECUTION_UNCERTAIN: lane uniforms launch failed: %s", cudaGetErrorName(e));
        return pp::fail_msg(PP_STATUS_UNCERTAIN, msg);
    }
    return PP_STATUS_OK;
}

}  // extern "C"
