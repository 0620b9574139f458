// CUDA-core int8 weight-only GEMV for tiny M (decode with 1-4 tokens) on row-major W.
//
// y[m, n] = s[n] * sum_k x[m, k] * w[n, k]
//
// One CTA of 256 threads owns ROWS consecutive output channels and a group of up to MT
// tokens.  Each thread streams 16-byte chunks of the ROWS weight rows with 128-bit
// L1-bypassing loads (chunk c = tid, tid+256, ...), widens the int8 values to exact fp32 with
// a byte-permute + packed add, and accumulates against the matching bf16 activations (read
// through L1, where every CTA of the SM shares them) with packed fp32 FMAs.  The ROWS x MT
// partial sums are reduced with warp shuffles, then across the 8 warps through shared memory;
// the per-channel scale is applied once to the reduced sum.
//
// The grid has ceil(N / ROWS) x ceil(M / MT) CTAs, so thousands of short CTAs keep every SM
// streaming: the kernel is bound by HBM bandwidth, not by the FMA pipes, for M <= 2
// (about 2.3 instructions per weight byte at M = 1).
#pragma once

#include "common.cuh"

namespace lse {

constexpr int kGemvThreads = 256;

template <int MT, int ROWS>
__global__ void __launch_bounds__(kGemvThreads)
gemv_i8_kernel(const __nv_bfloat16 *__restrict__ x, int64_t ldx, int M, int K,
               const int8_t *__restrict__ w, const float *__restrict__ scale, int N,
               __nv_bfloat16 *__restrict__ y, int64_t ldy) {
    const int n0 = blockIdx.x * ROWS;
    const int m0 = blockIdx.y * MT;
    const int chunks = K >> 4;  // K % 16 == 0 is checked on the host

    float2 acc[ROWS][MT];
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[r][t] = make_float2(0.f, 0.f);

    // Weights never depend on the previous kernel: issue the first chunk's weight loads,
    // then wait for the previous kernel's output (programmatic dependent launch) before
    // reading activations or writing y.
    int4 wv[ROWS];
    auto load_w = [&](int c) {
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
            const int n = n0 + r;
            wv[r] = (n < N && c < chunks) ? ld_stream_v4(w + static_cast<int64_t>(n) * K + static_cast<int64_t>(c) * 16)
                                          : make_int4(0, 0, 0, 0);
        }
    };
    load_w(threadIdx.x);
    asm volatile("griddepcontrol.wait;" ::: "memory");

    for (int c = threadIdx.x; c < chunks; c += kGemvThreads) {
        int4 cur[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) cur[r] = wv[r];
        load_w(c + kGemvThreads);  // next chunk in flight while this one is consumed
        // Activations for this chunk: 16 bf16 per token = two 128-bit loads.
        float2 xf[MT][8];
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            const int m = m0 + t;
            uint4 a = make_uint4(0, 0, 0, 0), b = make_uint4(0, 0, 0, 0);
            if (m < M) {
                const uint4 *xp = reinterpret_cast<const uint4 *>(x + (int64_t)m * ldx + (int64_t)c * 16);
                a = __ldg(xp);
                b = __ldg(xp + 1);
            }
            xf[t][0] = bf16x2_to_f32x2(a.x);
            xf[t][1] = bf16x2_to_f32x2(a.y);
            xf[t][2] = bf16x2_to_f32x2(a.z);
            xf[t][3] = bf16x2_to_f32x2(a.w);
            xf[t][4] = bf16x2_to_f32x2(b.x);
            xf[t][5] = bf16x2_to_f32x2(b.y);
            xf[t][6] = bf16x2_to_f32x2(b.z);
            xf[t][7] = bf16x2_to_f32x2(b.w);
        }
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
            const uint32_t words[4] = {(uint32_t)cur[r].x, (uint32_t)cur[r].y, (uint32_t)cur[r].z,
                                       (uint32_t)cur[r].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float2 lo, hi;
                i8x4_to_f32x4(words[j], lo, hi);
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    acc[r][t] = __ffma2_rn(lo, xf[t][2 * j], acc[r][t]);
                    acc[r][t] = __ffma2_rn(hi, xf[t][2 * j + 1], acc[r][t]);
                }
            }
        }
    }

    // Multi-wave grid: admit the next kernel's CTAs only as this one winds down.
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // Reduce: pair -> warp (shuffle) -> CTA (shared memory, 8 warps).
    __shared__ float red[kGemvThreads / 32][ROWS * MT];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int r = 0; r < ROWS; ++r)
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            float v = acc[r][t].x + acc[r][t].y;
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) red[warp][r * MT + t] = v;
        }
    __syncthreads();
    if (threadIdx.x < ROWS * MT) {
        const int r = threadIdx.x / MT, t = threadIdx.x % MT;
        const int n = n0 + r, m = m0 + t;
        if (n < N && m < M) {
            float v = 0.f;
#pragma unroll
            for (int q = 0; q < kGemvThreads / 32; ++q) v += red[q][threadIdx.x];
            y[(int64_t)m * ldy + n] = __float2bfloat16_rn(v * __ldg(scale + n));
        }
    }
}

}  // namespace lse
