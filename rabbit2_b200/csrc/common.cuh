// common.cuh -- shared device helpers for the RABBIT2 MoE kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rbt {

constexpr unsigned FULL_MASK = 0xffffffffu;

// bf16 bits -> f32: a 16-bit left shift, the widening of rabbit2.c:304-309.
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

// Weight element traits: WT is uint16_t (bf16 bit patterns) or float.
template <typename WT>
struct WeightTraits;

template <>
struct WeightTraits<uint16_t> {
    static constexpr int kVec = 8;  // elements per 16-byte vector
    __device__ __forceinline__ static float load1(const uint16_t* p) { return bf16_bits_to_f32(*p); }
    __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
        f[0] = __uint_as_float(v.x << 16);
        f[1] = __uint_as_float(v.x & 0xffff0000u);
        f[2] = __uint_as_float(v.y << 16);
        f[3] = __uint_as_float(v.y & 0xffff0000u);
        f[4] = __uint_as_float(v.z << 16);
        f[5] = __uint_as_float(v.z & 0xffff0000u);
        f[6] = __uint_as_float(v.w << 16);
        f[7] = __uint_as_float(v.w & 0xffff0000u);
    }
};

template <>
struct WeightTraits<float> {
    static constexpr int kVec = 4;
    __device__ __forceinline__ static float load1(const float* p) { return *p; }
    __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
        f[0] = __uint_as_float(v.x);
        f[1] = __uint_as_float(v.y);
        f[2] = __uint_as_float(v.z);
        f[3] = __uint_as_float(v.w);
    }
};

// Streaming 16-byte load of weights that are read once per call: read-only
// path, no L1 allocation (the 126 MB L2 still sees it).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL_MASK, v, o);
    return v;
}

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

}  // namespace rbt
