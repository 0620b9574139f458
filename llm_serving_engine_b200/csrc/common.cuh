// Shared device helpers for the sm_100a int8 linear kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/lse_int8.h"

namespace lse {

// Device-side status word (zero-initialised = LSE_OK): a kernel whose bounded wait gives up
// stores LSE_ERR_DEVICE_TIMEOUT here (never traps); lse_device_status() reads and clears it.
// The library is one translation unit, so the definition lives here.
__device__ int g_device_status;

// First nonzero status wins (a kernel that finds a bad argument on the device, e.g. a block
// id outside the pool, records it and skips the access).
__device__ __forceinline__ void report_status(int status) { atomicCAS(&g_device_status, LSE_OK, status); }

__device__ __forceinline__ void report_timeout() {
    atomicCAS(&g_device_status, LSE_OK, LSE_ERR_DEVICE_TIMEOUT);
}

// ~2 s at the B200's 1.9 GHz boost clock, ~3 s under the power cap: far above any
// legitimate wait in these kernels, short enough that a lost arrival ends the launch.
constexpr long long kWaitLimitCycles = 4000000000LL;
// The limit of data waits (lse_set_wait_limit); drains of a CTA's own copies and MMAs keep
// kWaitLimitCycles.
__device__ long long g_wait_limit = kWaitLimitCycles;

// Streaming 128-bit load of read-once weight bytes: skip L1, keep L2 normal.
__device__ __forceinline__ int4 ld_stream_v4(const void *p) {
    int4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// 4 int8 (two's complement, little-endian in a 32-bit word) -> 4 exact fp32 values.
// Each byte b is biased to u = b ^ 0x80 in [0, 255], placed in the mantissa of 2^23
// (bit pattern 0x4B0000uu == 8388608 + u), then 2^23 + 128 is subtracted: exact, since every
// intermediate is an integer below 2^24.
__device__ __forceinline__ void i8x4_to_f32x4(uint32_t v, float2 &lo, float2 &hi) {
    const uint32_t u = v ^ 0x80808080u;
    const float2 bias = make_float2(-8388736.0f, -8388736.0f);
    float2 a, b;
    a.x = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540));
    a.y = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541));
    b.x = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542));
    b.y = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543));
    lo = __fadd2_rn(a, bias);
    hi = __fadd2_rn(b, bias);
}

// 2 bf16 packed in a 32-bit word -> 2 fp32 (exact).
__device__ __forceinline__ float2 bf16x2_to_f32x2(uint32_t v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
}

// 2 int8 values (bytes 0 and 1 of the 16-bit lanes of `spread`: b0 in bits 0-7,
// b1 in bits 16-23) -> bf16x2, exact.  With t = 0x4300 | (b & 0x7F) (= 128 + (b & 127)) and
// c = 0x4300 | (b & 0x80) (= 128, or 256 when the sign bit is set), t - c == b as a signed
// byte; the difference is an integer of magnitude <= 128, so bf16 subtraction is exact.
__device__ __forceinline__ uint32_t i8pair_to_bf16x2(uint32_t spread) {
    uint32_t t, c, r;
    asm("lop3.b32 %0, %1, 0x007F007F, 0x43004300, 0xEA;" : "=r"(t) : "r"(spread));  // (a&b)|c
    asm("lop3.b32 %0, %1, 0x00800080, 0x43004300, 0xEA;" : "=r"(c) : "r"(spread));
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(t), "r"(c));
    return r;
}

// 4 int8 in a word -> 2 bf16x2 words: (k0,k1) and (k2,k3), low half = lower k.
__device__ __forceinline__ void i8x4_to_bf16x4(uint32_t v, uint32_t &p01, uint32_t &p23) {
    p01 = i8pair_to_bf16x2(__byte_perm(v, 0u, 0x4140));
    p23 = i8pair_to_bf16x2(__byte_perm(v, 0u, 0x4342));
}

// Biased weights (u = v ^ 0x80, the packed layout's storage) -> bf16x2.  Same construction as
// above; only the sign term flips: c = 0x4300 | (~u & 0x80).
__device__ __forceinline__ uint32_t u8pair_to_bf16x2(uint32_t spread) {
    uint32_t t, c, r;
    asm("lop3.b32 %0, %1, 0x007F007F, 0x43004300, 0xEA;" : "=r"(t) : "r"(spread));  // (a&b)|c
    asm("lop3.b32 %0, %1, 0x00800080, 0x43004300, 0xAE;" : "=r"(c) : "r"(spread));  // (~a&b)|c
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(t), "r"(c));
    return r;
}
__device__ __forceinline__ void u8x4_to_bf16x4(uint32_t v, uint32_t &p01, uint32_t &p23) {
    p01 = u8pair_to_bf16x2(__byte_perm(v, 0u, 0x4140));
    p23 = u8pair_to_bf16x2(__byte_perm(v, 0u, 0x4342));
}

// Biased weights -> f16x2 in two instructions per pair: the byte permute builds
// 0x64uu = 1024 + u (exact: fp16 has 10 mantissa bits) and 1024 + u - 1152 = v is exact.
__device__ __forceinline__ void u8x4_to_f16x4(uint32_t v, uint32_t &p01, uint32_t &p23) {
    const uint32_t k1152 = 0x64806480u;  // (1152, 1152) in f16
    const uint32_t a = __byte_perm(v, 0x64646464u, 0x5140);
    const uint32_t b = __byte_perm(v, 0x64646464u, 0x5342);
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(p01) : "r"(a), "r"(k1152));
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(p23) : "r"(b), "r"(k1152));
}

// bf16x2 -> f16x2, round to nearest, saturating to +-65504 (exact for |x| in [2^-14, 65504]).
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t v) {
    const float lo = __uint_as_float(v << 16), hi = __uint_as_float(v & 0xFFFF0000u);
    uint32_t r;
    asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// Activation element types: bf16 or fp16 <-> fp32 (round to nearest on the way out).
__device__ __forceinline__ float to_float(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_float(__half v) { return __half2float(v); }
template <typename T>
__device__ __forceinline__ T from_float(float v);
template <>
__device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <>
__device__ __forceinline__ __half from_float<__half>(float v) { return __float2half_rn(v); }

__device__ __forceinline__ long long clock64_now() {
    long long c;
    asm volatile("mov.u64 %0, %%clock64;" : "=l"(c));
    return c;
}

}  // namespace lse
