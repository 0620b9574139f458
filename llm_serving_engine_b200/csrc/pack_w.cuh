// Load-time repack of int8 weights into the fragment-major layout both kernels stream.
//
// W [N, K] (row-major int8) is zero padded to Np = 128*ceil(N/128) rows and
// Kp = 128*ceil(K/128) columns and cut into row blocks of 16 rows.  Row block rb is ONE
// contiguous run of 16 * Kp bytes, made of 512-byte chunks, one per 32 columns:
//
//   chunk (rb, kc) at byte (rb * (Kp / 32) + kc) * 512
//   inside it, lane t = 4 * r0 + q (r0 < 8, q < 4) owns 16 bytes at t * 16:
//       [h = 0: row r0 K 4q..4q+3 | row r0+8 K 4q..4q+3 | h = 1: the same at K + 16]
//   i.e. W[rb*16 + rr*8 + r0][kc*32 + h*16 + 4q + e] sits at t*16 + h*8 + rr*4 + e.
//
// Every byte is stored biased, u = v ^ 0x80 (= v + 128, in [1, 255] for v in [-127, 127]):
// fp16 holds 1024 + u exactly, so one byte permute that inserts the fp16 exponent plus one
// fp16 subtraction widens a pair of weights (the decode kernel), and the bf16 widening of
// the prefill kernel is as cheap as for plain two's complement.
//
// Why this order:
//   * a warp loads a chunk with one 128-bit load per lane, 512 contiguous bytes, and each
//     lane's 8 bytes of one half are exactly the A fragment of a 16x8x16 warp MMA (rows
//     r0, r0+8; the K quad 4q..4q+3 stands in for the fragment's K pairs 2q,2q+1 and
//     2q+8,2q+9 - a fixed permutation of K inside each 16-block, applied to the
//     activations too, so the dot product is unchanged);
//   * the same 8 bytes are what one thread hands to a 16-lane x 256-bit TMEM store, which
//     writes rows r0, r0+8 and the four K columns 4q..4q+3 in TRUE order, so the
//     tensor-core kernel's A operand needs no permutation;
//   * a 128 x 128 tile of the tensor-core kernel is 8 row-block runs of 2 KB each: one 2-D
//     bulk-tensor copy (8-byte elements, box 256 x 8) moves it.
// Runs once per weight, at model load.
#pragma once

#include "common.cuh"

namespace lse {

constexpr int kPackTile = 128;

__host__ __device__ inline int64_t packed_rows(int64_t N) { return (N + kPackTile - 1) / kPackTile * kPackTile; }
__host__ __device__ inline int64_t packed_cols(int64_t K) { return (K + kPackTile - 1) / kPackTile * kPackTile; }
__host__ __device__ inline int64_t packed_weight_bytes(int64_t N, int64_t K) { return packed_rows(N) * packed_cols(K); }

// Byte offset of W[n][k] in the packed buffer (Kp = packed_cols(K)).
__host__ __device__ inline int64_t packed_offset(int64_t n, int64_t k, int64_t Kp) {
    const int64_t rb = n >> 4, kc = k >> 5;
    const int r = static_cast<int>(n & 15), kk = static_cast<int>(k & 31);
    const int h = kk >> 4, q = (kk & 15) >> 2, e = kk & 3, r0 = r & 7, rr = r >> 3;
    return (rb * (Kp >> 5) + kc) * 512 + (4 * r0 + q) * 16 + h * 8 + rr * 4 + e;
}

// One thread per packed output byte group of 4 (e = 0..3 contiguous in both layouts).
__global__ void pack_weight_kernel(const int8_t *__restrict__ w, int64_t N, int64_t K, int64_t ldw,
                                   int8_t *__restrict__ out, int64_t Kp, int64_t total_quads) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= total_quads) return;
    // decode (rb, kc, t, h, rr) from the output position
    const int64_t chunk = i >> 7;                 // 128 quads per 512-byte chunk
    const int within = static_cast<int>(i & 127); // quad index inside the chunk
    const int t = within >> 2, h = (within >> 1) & 1, rr = within & 1;
    const int64_t rb = chunk / (Kp >> 5), kc = chunk % (Kp >> 5);
    const int r0 = t >> 2, q = t & 3;
    const int64_t n = rb * 16 + rr * 8 + r0;
    const int64_t k0 = kc * 32 + h * 16 + 4 * q;
    uint32_t v = 0;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int8_t b = (n < N && k0 + e < K) ? w[n * ldw + k0 + e] : int8_t(0);  // padding: v = 0
        v |= static_cast<uint32_t>(static_cast<uint8_t>(b)) << (8 * e);
    }
    reinterpret_cast<uint32_t *>(out)[i] = v ^ 0x80808080u;  // biased: u = v ^ 0x80
}

// Packed -> row-major (inspection / dequantization of a packed weight).
__global__ void unpack_weight_kernel(const int8_t *__restrict__ packed, int64_t N, int64_t K,
                                     int8_t *__restrict__ w, int64_t Kp) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= N * K) return;
    const int64_t n = i / K, k = i % K;
    w[i] = static_cast<int8_t>(packed[packed_offset(n, k, Kp)] ^ 0x80);
}

}  // namespace lse
