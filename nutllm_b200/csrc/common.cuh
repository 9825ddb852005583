#pragma once
/* Shared device helpers for the sm_100a token loop. */
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace nut {

constexpr int kBlock = 32;  /* quantisation block (include/quant.hpp:17) */
constexpr float kEps = 1e-5f; /* rmsnorm epsilon (src/quant_model.cpp:182) */

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

/* Sum over the whole CTA; `scratch` holds one float per warp.  Every thread
 * returns the total. */
__device__ __forceinline__ float block_sum(float v, float *scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int warps = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0)
        scratch[warp] = v;
    __syncthreads();
    float t = 0.0f;
    for (int w = 0; w < warps; w++)
        t += scratch[w];
    return t;
}

__device__ __forceinline__ float block_max(float v, float *scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int warps = (blockDim.x + 31) >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0)
        scratch[warp] = v;
    __syncthreads();
    float t = -INFINITY;
    for (int w = 0; w < warps; w++)
        t = fmaxf(t, scratch[w]);
    return t;
}

/* fp16 scale bits to fp32 (exact widening, including fp16 subnormals). */
__device__ __forceinline__ float half_bits_to_float(uint16_t bits) {
    return __half2float(__ushort_as_half(bits));
}

/* Order-preserving map of a finite float to uint32 (-0 folded onto +0), and
 * the argmax key: larger value wins, then the smaller index, which is the
 * first-index tie rule of std::max_element (src/generate.cpp:28-30). */
__device__ __forceinline__ uint32_t ordered_bits(float v) {
    if (v == 0.0f)
        v = 0.0f;
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t index) {
    return (static_cast<unsigned long long>(ordered_bits(v)) << 32) |
           static_cast<unsigned long long>(~index);
}

__device__ __forceinline__ uint32_t argmax_index(unsigned long long key) {
    return ~static_cast<uint32_t>(key & 0xffffffffull);
}

} // namespace nut
