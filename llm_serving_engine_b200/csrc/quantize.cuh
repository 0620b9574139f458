// Load-time symmetric per-output-channel int8 quantization.
//
//   amax[n] = max_k |w[n,k]|;  s[n] = amax / 127 (1.0 for an all-zero row)
//   q[n,k]  = clamp(rint(w[n,k] / s[n]), -127, 127)
//
// fp32 arithmetic with IEEE division and round-half-to-even, so the result is bit-identical
// to a float32 restatement on the host.  One CTA per row: a block max-reduction, then one
// pass writing q.  Runs once per weight at model load, so it is written for clarity.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace lse {

template <typename T>
__device__ __forceinline__ float load_as_f32(const T *p);
template <>
__device__ __forceinline__ float load_as_f32<__nv_bfloat16>(const __nv_bfloat16 *p) {
    return __bfloat162float(*p);
}
template <>
__device__ __forceinline__ float load_as_f32<__half>(const __half *p) {
    return __half2float(*p);
}
template <>
__device__ __forceinline__ float load_as_f32<float>(const float *p) {
    return *p;
}

constexpr int kQuantThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kQuantThreads)
quantize_rows_kernel(const T *__restrict__ w, int64_t ldw, int64_t K, int8_t *__restrict__ q,
                     float *__restrict__ s) {
    const int64_t n = blockIdx.x;
    const T *row = w + n * ldw;
    float amax = 0.f;
    for (int64_t k = threadIdx.x; k < K; k += kQuantThreads) amax = fmaxf(amax, fabsf(load_as_f32(row + k)));
    __shared__ float red[kQuantThreads / 32];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < kQuantThreads / 32; ++i) m = fmaxf(m, red[i]);
    const float sc = __fdiv_rn(m, 127.0f);
    const float scale = sc > 0.f ? sc : 1.0f;
    if (threadIdx.x == 0) s[n] = scale;
    for (int64_t k = threadIdx.x; k < K; k += kQuantThreads) {
        float v = rintf(__fdiv_rn(load_as_f32(row + k), scale));
        v = fminf(fmaxf(v, -127.f), 127.f);
        q[n * K + k] = (int8_t)v;
    }
}

}  // namespace lse
