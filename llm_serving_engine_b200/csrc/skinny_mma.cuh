// Skinny int8 weight-only GEMM for decode (M <= 32 tokens), on the fragment-major packed
// weights of pack_w.cuh.
//
//   y[m, n] = s[n] * sum_k x[m, k] * w[n, k]
//
// Decode is bound by the weight stream (2 flop per weight byte per token), so the kernel is
// shaped to keep HBM busy rather than to maximise tensor throughput:
//   * one CTA of KW warps owns a block of 16 output channels over all of K; each warp
//     streams its share of the block's contiguous 16*Kp-byte run through a private ring of
//     4 KB slots in shared memory, each slot filled by ONE 1-D bulk copy issued by lane 0
//     and completed on an mbarrier: the bytes in flight cost no registers and the lanes do
//     no copy bookkeeping (the integer pipe, not HBM, bounded a per-lane-copy variant);
//   * every lane's 16 bytes of a 512-byte chunk ARE two 16x16 A fragments (pack_w.cuh),
//     widened to fp16 in registers with one byte permute + one fp16 subtraction per pair
//     (exact: the packed bytes are biased, u = v + 128, and fp16 holds 1024 + u) and fed to
//     16x8x16 warp MMAs with fp32 accumulation - every warp issues its own MMAs, so no
//     single thread serialises the stream.  The integer pipe runs at half rate and was the
//     bound with a bf16 widening (3 integer ops per pair, bf16 has 7 mantissa bits); the
//     activations are rounded bf16 -> fp16 per fragment (exact for |x| in [2^-14, 65504],
//     saturating beyond), which costs less than it saves;
//   * the activation fragments of a slot are read from global memory (L1/L2-resident:
//     every CTA on the SM reads the same rows) before the slot's weights are waited for, in
//     the K order the packed layout implies;
//   * the K split is reduced across the warps through shared memory, in a fixed order, and
//     the per-channel scale is applied once to each reduced sum.
// No workspace, no cross-CTA traffic.  The ring is filled before waiting on the previous
// kernel (programmatic dependent launch): weights never depend on it.  Every mbarrier wait
// is bounded; a wait that gives up records LSE_ERR_DEVICE_TIMEOUT and ends the CTA.
#pragma once

#include <type_traits>

#include "tc_ptx.cuh"

namespace lse {

// D (16x8 fp32) += A (16x16 f16, row) * B (16x8 f16, col).
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Per warp: a ring of RS slots, each SC chunks (SC * 512 contiguous bytes of the warp's share
// of the row block).  Small grids (few row blocks) split K over 16 warps, large grids over 4;
// either way ~100-200 KB of weights per SM are in flight.
template <int KW>
struct SkinnyCfg {
    static constexpr int SC = 8;                 // chunks per slot (4 KB)
    static constexpr int RS = KW >= 16 ? 2 : 4;  // slots per warp
    static constexpr int SLOT_BYTES = SC * 512;
    static constexpr int RING_BYTES = RS * SLOT_BYTES;
    static constexpr int SMEM = KW * RING_BYTES + KW * RS * 8 + 16;
};

template <int MT, int KW>  // token tiles of 8 per CTA, warps splitting K
__global__ void __launch_bounds__(KW * 32)
skinny_i8_kernel(const __nv_bfloat16 *__restrict__ x, int64_t ldx, int M, int K,
                 const int8_t *__restrict__ wp, const float *__restrict__ scale, int N,
                 __nv_bfloat16 *__restrict__ y, int64_t ldy, int Kp) {
    using C = SkinnyCfg<KW>;
    constexpr int SC = C::SC, RS = C::RS;
    const int rb = blockIdx.x;
    const int m0 = blockIdx.y * MT * 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = lane >> 2, q = lane & 3;
    const int kc_all = Kp >> 5;         // 32-column chunks per row block (padded)
    const int kc_real = (K + 31) >> 5;  // chunks holding real columns
    const int per = (kc_real + KW - 1) / KW;
    const int c0 = min(kc_real, warp * per), c1 = min(kc_real, c0 + per);
    const int nslots = (c1 - c0 + SC - 1) / SC;
    const int8_t *wsrc = wp + (static_cast<int64_t>(rb) * kc_all + c0) * 512;

    extern __shared__ __align__(128) uint8_t skinny_smem[];
    uint8_t *ring = skinny_smem + warp * C::RING_BYTES;
    uint64_t *bars = reinterpret_cast<uint64_t *>(skinny_smem + KW * C::RING_BYTES) + warp * RS;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(skinny_smem + KW * C::RING_BYTES + KW * RS * 8);

    auto issue = [&](int g) {  // lane 0 only: weights of slot g -> ring slot g % RS
        const uint32_t bar = ptx::smem_u32(&bars[g % RS]);
        const uint32_t nb = static_cast<uint32_t>(min(SC, c1 - c0 - g * SC) * 512);
        ptx::mbar_arrive_expect_tx(bar, nb);
        ptx::bulk_load(ptx::smem_u32(ring + (g % RS) * C::SLOT_BYTES), wsrc + static_cast<int64_t>(g) * C::SLOT_BYTES,
                       nb, bar, ptx::policy_evict_first());
    };
    if (threadIdx.x == 0) *abort_flag = 0;
    if (lane == 0) {
        for (int i = 0; i < RS; ++i) ptx::mbar_init(ptx::smem_u32(&bars[i]), 1);
        ptx::fence_mbar_init();
        // Weights never depend on the previous kernel: fill the ring before waiting for it.
        for (int g = 0; g < RS && g < nslots; ++g) issue(g);
    }
    __syncthreads();
    asm volatile("griddepcontrol.wait;" ::: "memory");

    // Activation rows this lane feeds as the B fragment of token tile t: token m0 + 8t + r0,
    // K quad 4q..4q+3 of each 16-column step (rows past M are never read and count as zero).
    const __nv_bfloat16 *xrow[MT];
    bool xok[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        const int m = m0 + 8 * t + r0;
        xok[t] = m < M;
        xrow[t] = x + static_cast<int64_t>(xok[t] ? m : 0) * ldx + 4 * q + static_cast<int64_t>(c0) * 32;
    }

    float acc[2][MT][4];  // two accumulator sets alternate by chunk parity
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[u][t][0] = acc[u][t][1] = acc[u][t][2] = acc[u][t][3] = 0.f;

    const int kcols = K - c0 * 32;  // real columns from this warp's first chunk on
    bool ok = true;
    // One slot: activation fragments first (requested before waiting for the weights), then
    // widen + MMA per chunk.  FULL slots (all SC chunks real, every column < K) skip the
    // per-chunk bounds predicates.
    auto run_slot = [&](int g, auto full_tag) -> bool {
        constexpr bool FULL = decltype(full_tag)::value;
        const int nch = FULL ? SC : min(SC, c1 - c0 - g * SC);
        uint32_t xs[SC][MT][2][2];  // f16x2 B fragments
#pragma unroll
        for (int j = 0; j < SC; ++j)
#pragma unroll
            for (int t = 0; t < MT; ++t)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int col = (g * SC + j) * 32 + h * 16;  // relative to chunk c0
                    uint2 v = make_uint2(0, 0);
                    if (xok[t] && (FULL || (j < nch && col < kcols)))
                        v = __ldg(reinterpret_cast<const uint2 *>(xrow[t] + col));
                    xs[j][t][h][0] = bf16x2_to_f16x2(v.x);
                    xs[j][t][h][1] = bf16x2_to_f16x2(v.y);
                }
        const bool landed = ptx::mbar_wait(ptx::smem_u32(&bars[g % RS]), (g / RS) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, landed)) return false;
        const uint8_t *sl = ring + (g % RS) * C::SLOT_BYTES + lane * 16;
#pragma unroll
        for (int j = 0; j < SC; ++j) {
            if (FULL || j < nch) {
                const uint4 wv = *reinterpret_cast<const uint4 *>(sl + j * 512);
                const uint32_t words[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    // words[2h] = row r0, words[2h+1] = row r0+8; K quad 4q..4q+3 each.  A
                    // 16-column step past K holds zero weights and zero activations.
                    uint32_t r_lo01, r_lo23, r_hi01, r_hi23;
                    u8x4_to_f16x4(words[2 * h], r_lo01, r_lo23);
                    u8x4_to_f16x4(words[2 * h + 1], r_hi01, r_hi23);
                    const uint32_t a[4] = {r_lo01, r_hi01, r_lo23, r_hi23};
#pragma unroll
                    for (int t = 0; t < MT; ++t) mma_16816(acc[j & 1][t], a, xs[j][t][h][0], xs[j][t][h][1]);
                }
            }
        }
        __syncwarp();  // every lane has read the slot: lane 0 may refill it
        if (lane == 0 && g + RS < nslots) issue(g + RS);
        return true;
    };
    for (int g = 0; g < nslots && ok; ++g) {
        const bool full = (g + 1) * SC <= c1 - c0 && (g + 1) * SC * 32 <= kcols;
        ok = full ? run_slot(g, std::true_type{}) : run_slot(g, std::false_type{});
    }
    if (!ok && lane == 0) {
        // a wait gave up: let this warp's outstanding copies land before shared memory is freed
        for (int g = 0; g < nslots; ++g) ptx::mbar_drain(ptx::smem_u32(&bars[g % RS]), (g / RS) & 1);
    }

    // The grid runs in several waves: let the next kernel's CTAs in only as this CTA winds
    // down, so they never take the slots of this kernel's later waves.
    if (threadIdx.x == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // K-split reduction across the accumulator sets and warps (fixed order), scale, store.
    __shared__ float red[KW][MT][4][32];
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int j = 0; j < 4; ++j) red[warp][t][j][lane] = acc[0][t][j] + acc[1][t][j];
    __syncthreads();
    // warps 0-3: warp j finishes accumulator register j of every token tile: row r0 + 8*(j>>1),
    // token 2q + (j & 1) of the tile (16x8 accumulator layout).
    if (warp < 4) {
        const int j = warp;
        const int n = rb * 16 + r0 + 8 * (j >> 1);
        if (n < N) {
            const float sc = __ldg(scale + n);
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                const int m = m0 + 8 * t + 2 * q + (j & 1);
                if (m < M) {
                    float v = 0.f;
#pragma unroll
                    for (int w = 0; w < KW; ++w) v += red[w][t][j][lane];
                    y[static_cast<int64_t>(m) * ldy + n] = __float2bfloat16_rn(v * sc);
                }
            }
        }
    }
}

}  // namespace lse
