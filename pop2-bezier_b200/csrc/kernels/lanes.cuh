// SplitMix64 lane streams shared by the device kernel (lanes.cu) and the
// host entry point that restates it (sched.cpp).
#pragma once
#include <cstdint>

#ifdef __CUDACC__
#define PP_HD __host__ __device__ __forceinline__
#else
#define PP_HD inline
#endif

namespace pp {

// SplitMix64's output function (Steele, Lea and Flood, OOPSLA 2014).
PP_HD uint64_t splitmix64_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Draw n (from 0) of the lane stream seeded `seed`: a float in [0, 1) with
// 24 random bits, exactly representable, so host and device agree bit for bit.
PP_HD float lane_uniform(uint64_t seed, uint64_t n) {
    const uint64_t z = splitmix64_mix(seed + (n + 1) * 0x9E3779B97F4A7C15ull);
    return (float)(uint32_t)(z >> 40) * (1.0f / 16777216.0f);
}

}  // namespace pp
