// RMSNorm of bf16 or fp16 rows (transformers' LlamaRMSNorm, reached at model_runner.py:213-224 through
// every decoder layer's input_layernorm / post_attention_layernorm and the final norm):
//
//   y[m, :] = bf16( w[:] * bf16( x[m, :] * rsqrt(mean(x[m, :]^2) + eps) ) )   (fp32 arithmetic)
//
// One CTA per row: 16-byte loads, the sum of squares reduced through warp shuffles and a
// small shared buffer; like transformers, the normalised row is rounded to bf16 before the
// weight multiply, whose product is rounded again.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>

namespace lse {
namespace norm {

constexpr int THREADS = 256;

// The two 16-bit elements (bf16 or fp16, T) of a 32-bit word as fp32 (exact), and back (one
// rounding each).
template <typename T>
__device__ __forceinline__ float word_lo(uint32_t u) {
    if constexpr (std::is_same_v<T, __half>) return __half2float(__ushort_as_half(static_cast<uint16_t>(u & 0xffffu)));
    else return __uint_as_float(u << 16);
}
template <typename T>
__device__ __forceinline__ float word_hi(uint32_t u) {
    if constexpr (std::is_same_v<T, __half>) return __half2float(__ushort_as_half(static_cast<uint16_t>(u >> 16)));
    else return __uint_as_float(u & 0xffff0000u);
}
template <typename T>
__device__ __forceinline__ uint32_t word_of(float a, float b) {
    if constexpr (std::is_same_v<T, __half>) {
        const __half2 p = __floats2half2_rn(a, b);
        return *reinterpret_cast<const uint32_t *>(&p);
    } else {
        const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<const uint32_t *>(&p);
    }
}

// Two elements (a 32-bit word) of a row with 1 / rms `r` and their two weights:
// round(w * round(x * r)) each in the row's type, transformers' LlamaRMSNorm rounding.
template <typename T = __nv_bfloat16>
__device__ __forceinline__ uint32_t rms_scale_pair(uint32_t u, uint32_t g, float r) {
    const uint32_t t = word_of<T>(word_lo<T>(u) * r, word_hi<T>(u) * r);
    return word_of<T>(word_lo<T>(t) * word_lo<T>(g), word_hi<T>(t) * word_hi<T>(g));
}

template <typename T>
__global__ void __launch_bounds__(THREADS) rms_norm_kernel(const T *__restrict__ x, int64_t ldx,
                                                           const T *__restrict__ w, int N, float eps,
                                                           T *__restrict__ y, int64_t ldy) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x is the previous kernel's output
    const int m = blockIdx.x;
    const T *xr = x + m * ldx;
    T *yr = y + m * ldy;
    const int n8 = N / 8;  // N % 8 == 0 (host-checked): 16-byte vectors
    float ss = 0.f;
    for (int i = threadIdx.x; i < n8; i += THREADS) {
        const uint4 v = reinterpret_cast<const uint4 *>(xr)[i];
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float a = word_lo<T>(u[j]), b = word_hi<T>(u[j]);
            ss = fmaf(a, a, fmaf(b, b, ss));
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    __shared__ float part[THREADS / 32];
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < THREADS / 32; ++i) tot += part[i];
    const float r = rsqrtf(tot / static_cast<float>(N) + eps);
    for (int i = threadIdx.x; i < n8; i += THREADS) {
        const uint4 v = reinterpret_cast<const uint4 *>(xr)[i];
        const uint4 g = reinterpret_cast<const uint4 *>(w)[i];
        const uint32_t u[4] = {v.x, v.y, v.z, v.w}, gw[4] = {g.x, g.y, g.z, g.w};
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            o[j] = rms_scale_pair<T>(u[j], gw[j], r);
        }
        reinterpret_cast<uint4 *>(yr)[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

}  // namespace norm
}  // namespace lse
