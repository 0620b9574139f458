// RMSNorm of bf16 rows (transformers' LlamaRMSNorm, reached at model_runner.py:213-224 through
// every decoder layer's input_layernorm / post_attention_layernorm and the final norm):
//
//   y[m, :] = bf16( x[m, :] * rsqrt(mean(x[m, :]^2) + eps) * w[:] )     (fp32 arithmetic)
//
// One CTA per row: 16-byte loads, the sum of squares reduced through warp shuffles and a
// small shared buffer, one bf16 rounding (transformers rounds the normalised row to the
// input dtype before the weight multiply; the difference is within one bf16 ulp).
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace lse {
namespace norm {

constexpr int THREADS = 256;

__global__ void __launch_bounds__(THREADS) rms_norm_kernel(const __nv_bfloat16 *__restrict__ x, int64_t ldx,
                                                           const __nv_bfloat16 *__restrict__ w, int N, float eps,
                                                           __nv_bfloat16 *__restrict__ y, int64_t ldy) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x is the previous kernel's output
    const int m = blockIdx.x;
    const __nv_bfloat16 *xr = x + m * ldx;
    __nv_bfloat16 *yr = y + m * ldy;
    const int n8 = N / 8;  // N % 8 == 0 (host-checked): 16-byte vectors
    float ss = 0.f;
    for (int i = threadIdx.x; i < n8; i += THREADS) {
        const uint4 v = reinterpret_cast<const uint4 *>(xr)[i];
        const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float a = __uint_as_float(u[j] << 16), b = __uint_as_float(u[j] & 0xffff0000u);
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
            const float a = __uint_as_float(u[j] << 16) * r * __uint_as_float(gw[j] << 16);
            const float b = __uint_as_float(u[j] & 0xffff0000u) * r * __uint_as_float(gw[j] & 0xffff0000u);
            const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
            o[j] = *reinterpret_cast<const uint32_t *>(&p);
        }
        reinterpret_cast<uint4 *>(yr)[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

}  // namespace norm
}  // namespace lse
