// Load-time repack of int8 weights into the layout both kernels stream.
//
// W [N, K] (row-major int8) is zero padded to Np = 128*ceil(N/128) rows and
// Kp = 128*ceil(K/128) columns and cut into row blocks of 16 rows.  Row block b (rows
// 16b..16b+15) is ONE contiguous run of 16 * Kp bytes made of 2 KB blocks, one per 128
// columns; a 2 KB block holds the block's two 8-row groups (h = 0: rows 16b..16b+7, h = 1:
// the next 8) one after the other, each as two 512-byte atoms of 64 columns; an atom holds its
// 8 rows' 64 columns, 64 bytes per row, with the 16-byte chunks of row r swapped by the tensor
// core's 64-byte swizzle (chunk c of row r stored at chunk position c ^ ((r >> 1) & 3)):
//
//   W[16b + 8h + r][128t + 64a + 16c + e]  at
//       b * 16 * Kp + t * 2048 + h * 1024 + a * 512 + r * 64 + ((c ^ ((r >> 1) & 3)) * 16) + e
//
//   (h, a < 2, r < 8, c < 4, e < 16).  Bytes are the plain two's-complement int8 values.
//
// Why this order:
//   * a 128 x 128 tile (8 row blocks x 2 KB) is the tensor core's canonical K-major operand
//     with the 64-byte swizzle (8-row groups 1 KB apart, the second 64 columns of a group 512
//     bytes on): the tensor-core kernel hands it to tcgen05.mma kind::i8 as its A operand
//     straight from shared memory, after one 2-D bulk-tensor copy (8-byte elements, box
//     256 x 8: eight runs of 2 KB);
//   * for the decode kernel, lane 4 * r0 + q of a warp loads row r0's 16 columns 16q..16q+15 of
//     an atom with one 128-bit load; the swizzle keeps the four lanes of a row on its 64
//     contiguous bytes and the eight lanes of two rows on one 128-byte line, so a warp load is
//     512 contiguous bytes in 4 line requests.  The matching load 1 KB on (the row block's
//     second group) gets row r0 + 8's, so a warp streams one contiguous run per row block.
//     Word j of those 16 bytes (columns 16q + 4j .. +3, rows r0 and r0 + 8) is the A
//     fragment of the j-th 16x8x16 warp MMA of the atom, taking the columns 16q + 4j + e for
//     the fragment's K pairs (2q, 2q+1) and (2q+8, 2q+9) - a fixed permutation of K inside each
//     64-column block, applied to the activations too, so the dot product is unchanged.
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
    const int r = static_cast<int>(n & 7), c = static_cast<int>((k >> 4) & 3);
    return (n >> 4) * 16 * Kp + (k >> 7) * 2048 + ((n >> 3) & 1) * 1024 + ((k >> 6) & 1) * 512 + r * 64 +
           ((c ^ ((r >> 1) & 3)) << 4) + (k & 15);
}

// Byte offset of 64-column unit u (u = k / 64) inside a row block's run: 2 KB per two units,
// the odd unit 512 bytes into the pair's block; the block's second group is 1 KB further on.
__host__ __device__ inline int64_t packed_unit_offset(int64_t u) { return (u >> 1) * 2048 + (u & 1) * 512; }

// One thread per 16-byte row run (16 consecutive columns of one row); consecutive threads take
// consecutive runs of the same row, so the reads are coalesced.
__global__ void pack_weight_kernel(const int8_t *__restrict__ w, int64_t N, int64_t K, int64_t ldw,
                                   int8_t *__restrict__ out, int64_t Kp, int64_t total_runs) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= total_runs) return;
    const int64_t n = i / (Kp >> 4), c = i % (Kp >> 4);  // row, 16-column run
    const int64_t k0 = c * 16;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (n < N) {
        const int8_t *src = w + n * ldw + k0;
        if (k0 + 16 <= K && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
            v = *reinterpret_cast<const uint4 *>(src);
        } else {
            uint32_t b[4] = {0, 0, 0, 0};
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const int8_t x = k0 + e < K ? src[e] : int8_t(0);  // padding: 0
                b[e >> 2] |= static_cast<uint32_t>(static_cast<uint8_t>(x)) << (8 * (e & 3));
            }
            v = make_uint4(b[0], b[1], b[2], b[3]);
        }
    }
    *reinterpret_cast<uint4 *>(out + packed_offset(n, k0, Kp)) = v;
}

// Packed -> row-major (inspection / dequantization of a packed weight).
__global__ void unpack_weight_kernel(const int8_t *__restrict__ packed, int64_t N, int64_t K,
                                     int8_t *__restrict__ w, int64_t Kp) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= N * K) return;
    const int64_t n = i / K, k = i % K;
    w[i] = packed[packed_offset(n, k, Kp)];
}

}  // namespace lse
