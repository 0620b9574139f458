// Activation digit planes for the int8 tensor-core kernel (sm_100a).
//
// The tensor-core kernel multiplies int8 weights by int8 activations (tcgen05.mma
// kind::i8, exact int32 accumulation).  The activations (bf16 or fp16, XT) are written, per
// token row m, as a fixed-point integer in S signed 8-bit digits under a power-of-two row scale:
//
//   r[m] = 2^e[m],  v[m, k] = rint(x[m, k] / r[m]) = sum_p d_p[m, k] * 256^(S-1-p),
//   d_p in [-128, 127]   (p = 0 the most significant digit plane)
//
// so that  y[m, n] = s[n] * r[m] * sum_p 256^(S-1-p) * sum_k w[n, k] d_p[m, k].
//
// e[m] is the smallest exponent with max_k |x[m, k]| / 2^e <= V_S = 127 * (256^S - 1) / 255
// (32639 for S = 2, 8355711 for S = 3), i.e. max |x| / 2^e in [2^(8S-2), 2^(8S-1)).
// Hence every bf16 element with |x| >= max|x| * 2^(10-8S) (2^-6 of the row maximum for S = 2,
// 2^-14 for S = 3) is represented exactly (its 8 significant bits sit at or above the quantum;
// for fp16's 11 bits the bound is max|x| * 2^(13-8S)), and any element's error is at most half
// a quantum, below max|x| * 2^-(8S-2).  A row
// of zeros gets r = 1 and zero digits; a row holding a NaN or an infinity gets r = NaN (the
// whole output row is NaN, as a matmul over it would be at least partly).
//
// Layout: plane p of row m is the int8 run planes[p * plane_stride + m * Kp + k], k < Kp
// (zeros for K <= k < Kp), K-contiguous: the kernel's tensor map reads a box of
// [S planes][token tile][128 K bytes] as one K-major B operand of S * NT rows.
//
// One CTA per row, every load of the row in flight at once (up to 16,384 elements); CTA 0 also
// clears the stream-K arrival counters of the projection launch that follows.  Programmatic
// dependent launch: the CTA releases its dependents on entry (the projection kernel's weight
// copies start under it) and waits for the kernel that wrote x before touching any memory.
#pragma once

#include <type_traits>

#include "common.cuh"
#include "rms_norm.cuh"

namespace lse {
namespace split {

constexpr int THREADS = 256;

template <int S>
struct Digits {
    static_assert(S == 2 || S == 3, "2 or 3 digit planes");
    static constexpr int kMaxV = S == 2 ? 32639 : 8355711;  // 127 * (256^S - 1) / 255
    static constexpr int kTopExp = 8 * S - 2;                // max|x| / 2^e in [2^kTopExp, 2^(kTopExp+1))
};

// The two activations (bf16 or fp16, XT) packed in a 32-bit word, as fp32 (exact).
template <typename XT>
__device__ __forceinline__ float act_lo(uint32_t w) {
    if constexpr (std::is_same_v<XT, __half>) return __half2float(__ushort_as_half(static_cast<uint16_t>(w & 0xFFFFu)));
    else return __uint_as_float(w << 16);
}
template <typename XT>
__device__ __forceinline__ float act_hi(uint32_t w) {
    if constexpr (std::is_same_v<XT, __half>) return __half2float(__ushort_as_half(static_cast<uint16_t>(w >> 16)));
    else return __uint_as_float(w & 0xFFFF0000u);
}

// Balanced base-256 digits of v (|v| <= kMaxV), most significant first, packed per plane into
// byte `slot & 3` of d[p].
template <int S>
__device__ __forceinline__ void digits_of(int v, uint32_t (&d)[S], int slot) {
#pragma unroll
    for (int p = S - 1; p >= 0; --p) {
        int dig = v;
        if (p > 0) {
            dig = ((v + 128) & 255) - 128;
            v = (v - dig) >> 8;  // exact: v - dig is a multiple of 256
        }
        d[p] |= static_cast<uint32_t>(dig & 255) << (8 * (slot & 3));
    }
}

// Chunks of 8 elements each thread keeps in registers: a row of up to THREADS * CPT * 8 =
// 16,384 elements is read once, with every load in flight together; a longer row is read in
// batches of that size (twice: once for the maximum, once for the digits).
constexpr int CPT = 8;

// 2^k as a float for an exponent of the normal range [-126, 127] (exact, from the bits).
__device__ __forceinline__ float exp2_exact(int k) { return __int_as_float((k + 127) << 23); }

// x / 2^e rounded to the nearest integer (ties to even) as inv_hi * inv_lo = 2^-e, each factor a
// normal power of two, so both multiplications are exact: the quotient is below 2^(8S-1).
template <int S, typename XT>
__device__ __forceinline__ void store_digits(int8_t *__restrict__ planes, int64_t plane_stride, int64_t row_off, int c,
                                             const uint4 &v, float inv_hi, float inv_lo, bool valid) {
    uint32_t d0[S] = {}, d1[S] = {};
    if (valid) {
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float f = h ? act_hi<XT>(w[i]) : act_lo<XT>(w[i]);
                int q = __float2int_rn((f * inv_hi) * inv_lo);
                q = max(-Digits<S>::kMaxV, min(Digits<S>::kMaxV, q));
                const int slot = 2 * i + h;
                if (slot < 4) digits_of<S>(q, d0, slot);
                else digits_of<S>(q, d1, slot);
            }
        }
    }
#pragma unroll
    for (int p = 0; p < S; ++p)
        *reinterpret_cast<uint2 *>(planes + p * plane_stride + row_off + 8 * c) = make_uint2(d0[p], d1[p]);
}

template <int S, typename XT = __nv_bfloat16>
__global__ void __launch_bounds__(THREADS)
act_split_kernel(const XT *__restrict__ x, int64_t ldx, int K, int Kp, int8_t *__restrict__ planes,
                 int64_t plane_stride, float *__restrict__ row_scale, int *__restrict__ counters, int n_counters) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x is the previous kernel's output
    const int m = blockIdx.x;
    // The projection kernel that follows counts stream-K arrivals in `counters`: they start at
    // zero for every launch without any invariant on the workspace's earlier contents.
    if (m == 0)
        for (int i = threadIdx.x; i < n_counters; i += THREADS) counters[i] = 0;
    const XT *xr = x + static_cast<int64_t>(m) * ldx;
    const int nk = K >> 3;  // 8-element chunks (K % 16 == 0, rows 16-byte aligned)
    constexpr int BATCH = THREADS * CPT;
    uint4 v[CPT];
    float amax = 0.f;
    bool bad = false;
    for (int base = 0; base < nk; base += BATCH) {
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const int c = base + threadIdx.x + i * THREADS;
            v[i] = c < nk ? __ldg(reinterpret_cast<const uint4 *>(xr + 8 * c)) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const uint32_t w[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float a = fabsf(act_lo<XT>(w[k])), b = fabsf(act_hi<XT>(w[k]));
                bad |= !(a <= 3.4e38f) || !(b <= 3.4e38f);  // NaN or infinity
                amax = fmaxf(amax, fmaxf(a, b));
            }
        }
    }
    __shared__ float s_max[THREADS / 32];
    __shared__ int s_bad[THREADS / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        bad |= __shfl_xor_sync(0xffffffffu, static_cast<int>(bad), o) != 0;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) {
        s_max[warp] = amax;
        s_bad[warp] = bad;
    }
    __syncthreads();
    amax = 0.f;
    bad = false;
#pragma unroll
    for (int i = 0; i < THREADS / 32; ++i) {
        amax = fmaxf(amax, s_max[i]);
        bad |= s_bad[i] != 0;
    }
    int e = 0;
    if (!bad && amax > 0.f) {
        e = ilogbf(amax) - Digits<S>::kTopExp;
        if (ldexpf(amax, -e) > static_cast<float>(Digits<S>::kMaxV)) ++e;  // an all-ones mantissa
    }
    // 2^-e split into two normal powers of two (e ranges over about [-155, 106])
    const int ne = -e;
    const int ne_hi = max(-126, min(127, ne));
    const float inv_hi = exp2_exact(ne_hi), inv_lo = exp2_exact(ne - ne_hi);
    // digits: 8 elements per chunk -> S planes x 8 bytes; a row that fits one batch is still
    // in registers
    const int64_t row_off = static_cast<int64_t>(m) * Kp;
    const int nkp = Kp >> 3;
    for (int base = 0; base < nkp; base += BATCH) {
        if (nk > BATCH) {
#pragma unroll
            for (int i = 0; i < CPT; ++i) {
                const int c = base + threadIdx.x + i * THREADS;
                v[i] = c < nk ? __ldg(reinterpret_cast<const uint4 *>(xr + 8 * c)) : make_uint4(0, 0, 0, 0);
            }
        }
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const int c = base + threadIdx.x + i * THREADS;
            if (c < nkp) store_digits<S, XT>(planes, plane_stride, row_off, c, v[i], inv_hi, inv_lo, c < nk && !bad);
        }
    }
    if (threadIdx.x == 0) row_scale[m] = bad ? __int_as_float(0x7FC00000) : ldexpf(1.f, e);
}

// RMSNorm fused in front of the split (bf16): the digit planes and row scale of
//   x_n[m, :] = bf16( w[:] * bf16( x[m, :] * rsqrt(mean(x[m, :]^2) + eps) ) )
// without writing x_n.  The sum of squares is accumulated in rms_norm_kernel's order (thread t
// takes the 8-element chunks t, t + THREADS, ...; shuffle tree; the warps' sums in order) and
// x_n is the same expression with the same roundings, so the planes equal act_split_kernel's planes
// of rms_norm_kernel's output bit for bit.  A row of up to THREADS * CPT * 8 elements stays in
// registers; a longer one is read again per pass.
template <int S>
__global__ void __launch_bounds__(THREADS)
rms_norm_split_kernel(const __nv_bfloat16 *__restrict__ x, int64_t ldx, const __nv_bfloat16 *__restrict__ w,
                      float eps, int K, int Kp, int8_t *__restrict__ planes, int64_t plane_stride,
                      float *__restrict__ row_scale, int *__restrict__ counters, int n_counters) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // x is the previous kernel's output
    const int m = blockIdx.x;
    if (m == 0)
        for (int i = threadIdx.x; i < n_counters; i += THREADS) counters[i] = 0;
    const __nv_bfloat16 *xr = x + static_cast<int64_t>(m) * ldx;
    const int nk = K >> 3;
    constexpr int BATCH = THREADS * CPT;
    const bool one_batch = nk <= BATCH;
    uint4 v[CPT];
    auto load_x = [&](int base) {
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const int c = base + threadIdx.x + i * THREADS;
            v[i] = c < nk ? __ldg(reinterpret_cast<const uint4 *>(xr + 8 * c)) : make_uint4(0, 0, 0, 0);
        }
    };
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __shared__ float s_red[THREADS / 32];
    __shared__ int s_bad[THREADS / 32];
    // pass 1: sum of squares
    float ss = 0.f;
    for (int base = 0; base < nk; base += BATCH) {
        load_x(base);
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float a = __uint_as_float(u[j] << 16), b = __uint_as_float(u[j] & 0xffff0000u);
                ss = fmaf(a, a, fmaf(b, b, ss));
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (lane == 0) s_red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < THREADS / 32; ++i) tot += s_red[i];
    const float r = rsqrtf(tot / static_cast<float>(K) + eps);
    __syncthreads();  // s_red is reused below
    // pass 2: the normalised bf16 row and its maximum magnitude
    auto normalise = [&](int base) {
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const int c = base + threadIdx.x + i * THREADS;
            if (c < nk) {
                const uint4 g = __ldg(reinterpret_cast<const uint4 *>(w) + c);
                v[i] = make_uint4(norm::rms_scale_pair(v[i].x, g.x, r), norm::rms_scale_pair(v[i].y, g.y, r),
                                  norm::rms_scale_pair(v[i].z, g.z, r), norm::rms_scale_pair(v[i].w, g.w, r));
            }
        }
    };
    float amax = 0.f;
    bool bad = false;
    for (int base = 0; base < nk; base += BATCH) {
        if (!one_batch) load_x(base);
        normalise(base);
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const uint32_t u[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float a = fabsf(act_lo<__nv_bfloat16>(u[k])), b = fabsf(act_hi<__nv_bfloat16>(u[k]));
                bad |= !(a <= 3.4e38f) || !(b <= 3.4e38f);  // NaN or infinity
                amax = fmaxf(amax, fmaxf(a, b));
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        bad |= __shfl_xor_sync(0xffffffffu, static_cast<int>(bad), o) != 0;
    }
    if (lane == 0) {
        s_red[warp] = amax;
        s_bad[warp] = bad;
    }
    __syncthreads();
    amax = 0.f;
    bad = false;
#pragma unroll
    for (int i = 0; i < THREADS / 32; ++i) {
        amax = fmaxf(amax, s_red[i]);
        bad |= s_bad[i] != 0;
    }
    int e = 0;
    if (!bad && amax > 0.f) {
        e = ilogbf(amax) - Digits<S>::kTopExp;
        if (ldexpf(amax, -e) > static_cast<float>(Digits<S>::kMaxV)) ++e;  // an all-ones mantissa
    }
    const int ne = -e;
    const int ne_hi = max(-126, min(127, ne));
    const float inv_hi = exp2_exact(ne_hi), inv_lo = exp2_exact(ne - ne_hi);
    // pass 3: digits
    const int64_t row_off = static_cast<int64_t>(m) * Kp;
    const int nkp = Kp >> 3;
    for (int base = 0; base < nkp; base += BATCH) {
        if (!one_batch) {
            load_x(base);
            normalise(base);
        }
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const int c = base + threadIdx.x + i * THREADS;
            if (c < nkp)
                store_digits<S, __nv_bfloat16>(planes, plane_stride, row_off, c, v[i], inv_hi, inv_lo, c < nk && !bad);
        }
    }
    if (threadIdx.x == 0) row_scale[m] = bad ? __int_as_float(0x7FC00000) : ldexpf(1.f, e);
}

}  // namespace split
}  // namespace lse
