// Skinny int8 weight-only GEMM for decode (M <= 32 tokens; the auto policy uses it up to 16),
// on the fragment-major packed weights of pack_w.cuh.
//
//   y[m, n] = s[n] * sum_k x[m, k] * w[n, k]
//
// Decode is bound by the weight stream (2 flop per weight byte per token).  The kernel is
// shaped so that nothing but HBM bounds it, and so that consecutive projections overlap:
//   * one CTA of KW warps owns R blocks of 16 output channels over all of K; warp w takes a
//     contiguous slice of each block's 32-column chunks;
//   * every lane loads its 16 bytes of a 512-byte chunk straight into registers with one
//     128-bit streaming load (L1 no-allocate, L2 evict-first): those bytes ARE two 16x16 A
//     fragments of a 16x8x16 warp MMA (pack_w.cuh), so there is no shared-memory staging,
//     no copy bookkeeping and no wait on a barrier.  U chunks per block are kept in flight
//     per lane (issued before the previous kernel is waited for: weights never depend on
//     it);
//   * weights are widened in registers - to fp16 with one byte permute + one fp16
//     subtraction per pair (exact: the bytes are biased, u = v + 128, and fp16 holds
//     1024 + u), with the activations rounded bf16 -> fp16 per fragment (exact for |x| in
//     [2^-14, 65504], saturating beyond); or, with BF16 set, to bf16 (two logic ops + one
//     bf16 subtraction per pair, exact) against the bf16 activations as they are - and fed
//     to warp MMAs with fp32 accumulation;
//   * the K split is reduced across the warps through shared memory in a fixed order and
//     the per-channel scale is applied once to each reduced sum (deterministic);
//   * the CTA signals programmatic launch completion on entry: it holds only a small
//     reduction buffer in shared memory, so the next kernel's CTAs become resident as soon
//     as registers free up and start their own weight streams under this kernel's tail.
//   * optional epilogues: the residual add (y = res + s * acc) and, for the MLP, SiLU(gate) *
//     up on gate/up rows interleaved in 8-row blocks.
// No workspace, no cross-CTA traffic, no spin-waits.
#pragma once

#include <type_traits>

#include "tc_ptx.cuh"

namespace lse {

// D (16x8 fp32) += A (16x16, row) * B (16x8, col), fp16 or bf16 operands.
template <bool BF16>
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    if constexpr (BF16) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
}

// 16 weight bytes of one lane: streaming load, no L1 allocation, L2 evict-first (each
// weight byte is read exactly once per call).  Volatile, so the compiler keeps every load
// where it is issued - ahead of the wait on the previous kernel and U chunks ahead of its
// use - instead of sinking it to the first use.
__device__ __forceinline__ uint4 ld_weight16(const int8_t *p, uint64_t policy) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p), "l"(policy));
    return r;
}

// 16 weight bytes of one lane into its own shared-memory slot (cp.async, L2 only, evict-first
// hint).  Only the issuing lane reads the slot back, after its own wait_group, so no barrier
// is involved.
__device__ __forceinline__ void cp_async16(uint32_t dst, const int8_t *src, uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "l"(policy)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ uint4 lds16(uint32_t addr) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(addr)
                 : "memory");
    return r;
}

// Dynamic shared memory of the cp.async weight ring: KW warps x P groups x U chunks x R row
// blocks x 512 bytes (16 per lane).
template <int KW, int R, int U, int P>
constexpr int skinny_ring_bytes() { return KW * P * U * R * 512; }

// y = bf16(s * acc), or bf16(res + s * acc) when `res` is given (it may be y itself: each
// element is read, then written, by one thread).
//
// MT token tiles of 8 per CTA (M <= 8 * MT), KW warps splitting K, R row blocks per CTA
// (sharing every activation load), U chunks per row block in flight per lane, BF16 selects
// the bf16 MMA.
//
// Bytes in flight per SM (resident warps x U x 512), then instructions per chunk, bound this
// kernel, so the main path is written for both: warp w streams a contiguous slice of the
// row block's chunks in whole groups of U, with every load at a constant offset from a
// pointer that moves once per group and no per-chunk predicate; the groups are visited in
// an order rotated per CTA, so the CTAs resident together read different offsets of their
// row blocks.  A slice that is not a whole number of groups (ragged K) takes a
// bounds-checked path.  `pf_groups` groups per row block beyond the U chunks in registers
// are prefetched into L2 by lane 0 (bulk prefetches), which deepens the stream at no
// register cost.
//
// P > 0 stages the weight stream through shared memory instead of registers: each lane
// keeps P groups of U chunks (per row block) in flight with cp.async into its own 16-byte
// slots, and reads a group back with shared loads once its cp.async group has completed.
// The depth in flight is then set by shared memory (P * U * R * 16 bytes per lane), not by
// registers, which matters for M > 8 where the accumulators and activation fragments take
// the registers a deeper register ring would need.
//
// SILU_MUL: the weight rows interleave 8-row blocks of the MLP's gate and up projections
// (row block b = gate rows 8b..8b+7, then the matching up rows 8b..8b+7), so the 16x8
// accumulator of one lane holds gate row r0 (registers 0, 1) and up row r0 (registers 2, 3)
// of the same tokens, and the epilogue writes y[m, 8b + r0] = silu(s_g * gate) * (s_u * up)
// (fp32, one bf16 rounding) for the N = I intermediate columns; `scale` is interleaved the
// same way.
template <int MT, int KW, int R, int U, bool BF16, int MINB, bool SILU_MUL = false, int P = 0>
__global__ void __launch_bounds__(KW * 32, MINB)
skinny_i8_kernel(const __nv_bfloat16 *__restrict__ x, int64_t ldx, int M, int K,
                 const int8_t *__restrict__ wp, const float *__restrict__ scale, int N,
                 __nv_bfloat16 *y, int64_t ldy, const __nv_bfloat16 *res, int64_t ldr, int Kp, int pf_groups) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int rg = blockIdx.x;
    const int m0 = blockIdx.y * MT * 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = lane >> 2, q = lane & 3;
    const int kc_all = Kp >> 5;         // 32-column chunks per row block (padded)
    const int kc_real = (K + 31) >> 5;  // chunks holding real columns
    const int per = (kc_real + KW - 1) / KW;
    const int c0 = min(kc_real, warp * per), c1 = min(kc_real, c0 + per);
    const int nch = c1 - c0;
    // Whole groups, and every column < K (only the last chunk of the row can be partial).
    const bool fast = nch > 0 && nch % U == 0 && c1 * 32 <= K;
    const int ng = nch / U;
    const int rot = fast ? rg % ng : 0;

    const uint64_t pol = ptx::policy_evict_first();
    // Row block rg*R + r (padded row blocks past N hold zeros) at wbase + r * rb_bytes.
    const int64_t rb_bytes = static_cast<int64_t>(kc_all) * 512;
    const int8_t *const wbase = wp + (static_cast<int64_t>(rg) * R * kc_all + c0) * 512 + lane * 16;
    const int8_t *gp = wbase + rot * (U * 512);
    // cp.async ring (P > 0, whole-group slices): this lane's slot for (ring group p, chunk j,
    // row block r) is at ring_lane + ((p * U + j) * R + r) * 512.
    extern __shared__ __align__(16) uint4 ring_smem[];
    const uint32_t ring_lane = ptx::smem_u32(ring_smem) + ((warp * P * U * R) * 32 + lane) * 16;
    auto issue_group = [&](int p, int gv) {  // slice group gv -> ring group p, one commit group
#pragma unroll
        for (int j = 0; j < U; ++j)
#pragma unroll
            for (int r = 0; r < R; ++r)
                cp_async16(ring_lane + ((p * U + j) * R + r) * 512, wbase + gv * (U * 512) + r * rb_bytes + j * 512, pol);
    };
    constexpr bool RING = P > 0;
    uint4 wb[U][R];
    if (RING && fast) {
        // groups rot, rot + 1, ... (mod ng) into ring groups 0..P-1; one commit per ring group
        // (empty when the slice has fewer groups) so wait_group counts stay uniform
#pragma unroll
        for (int p = 0; p < (RING ? P : 1); ++p) {
            if (p < ng) issue_group(p, rot + p < ng ? rot + p : rot + p - ng);
            cp_async_commit();
        }
    } else {
#pragma unroll
        for (int j = 0; j < U; ++j)
#pragma unroll
            for (int r = 0; r < R; ++r)
                wb[j][r] = (fast || j < nch) ? ld_weight16(gp + r * rb_bytes + j * 512, pol) : make_uint4(0, 0, 0, 0);
    }
    // L2 prefetch of the group `v` visits ahead (lane 0, one bulk prefetch per row block): the
    // register loads then hit L2, so the registers hold only U chunks while DRAM has
    // pf_groups more groups per row block in flight.
    auto prefetch_group = [&](int v) {
        if (lane == 0 && v < ng) {
            int gv = rot + v;
            if (gv >= ng) gv -= ng;
#pragma unroll
            for (int r = 0; r < R; ++r) ptx::bulk_prefetch_l2(wbase + r * rb_bytes + gv * (U * 512), U * 512);
        }
    };
    if (fast && !RING)
        for (int v = 1; v <= pf_groups; ++v) prefetch_group(v);

    asm volatile("griddepcontrol.wait;" ::: "memory");  // x is the previous kernel's output

    // Activation rows this lane feeds as the B fragment of token tile t: token m0 + 8t + r0,
    // K quad 4q..4q+3 of each 16-column step.  A token past M reads the last real row
    // instead: its MMA column is independent of the others and is never stored.
    const __nv_bfloat16 *xbase[MT];
    const __nv_bfloat16 *xp[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        const int m = min(m0 + 8 * t + r0, M - 1);
        xbase[t] = x + static_cast<int64_t>(m) * ldx + 4 * q + c0 * 32;
        xp[t] = xbase[t] + rot * (U * 32);
    }

    // With a single MMA chain (R * MT == 1) alternate two accumulator sets by chunk parity.
    constexpr int NACC = R * MT == 1 ? 2 : 1;
    float acc[NACC][R][MT][4];
#pragma unroll
    for (int u = 0; u < NACC; ++u)
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[u][r][t][0] = acc[u][r][t][1] = acc[u][r][t][2] = acc[u][r][t][3] = 0.f;

    // One chunk: B fragments from the two activation quads, A fragments widened from the
    // lane's 16 weight bytes of each row block, two 16x8x16 MMAs per token tile and block.
    auto compute = [&](int j, const uint4 (&wr)[R], const uint2 (&xv)[MT][2]) {
        uint32_t bx[MT][2][2];
#pragma unroll
        for (int t = 0; t < MT; ++t)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if constexpr (BF16) {
                    bx[t][h][0] = xv[t][h].x;
                    bx[t][h][1] = xv[t][h].y;
                } else {
                    bx[t][h][0] = bf16x2_to_f16x2(xv[t][h].x);
                    bx[t][h][1] = bf16x2_to_f16x2(xv[t][h].y);
                }
            }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const uint32_t words[4] = {wr[r].x, wr[r].y, wr[r].z, wr[r].w};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                // words[2h] = row r0, words[2h+1] = row r0+8; K quad 4q..4q+3 each.
                uint32_t lo01, lo23, hi01, hi23;
                if constexpr (BF16) {
                    u8x4_to_bf16x4(words[2 * h], lo01, lo23);
                    u8x4_to_bf16x4(words[2 * h + 1], hi01, hi23);
                } else {
                    u8x4_to_f16x4(words[2 * h], lo01, lo23);
                    u8x4_to_f16x4(words[2 * h + 1], hi01, hi23);
                }
                const uint32_t a[4] = {lo01, hi01, lo23, hi23};
#pragma unroll
                for (int t = 0; t < MT; ++t)
                    mma_16816<BF16>(acc[NACC == 2 ? (j & 1) : 0][r][t], a, bx[t][h][0], bx[t][h][1]);
            }
        }
    };
    // One whole group at gp / xp; with REFILL, slot j is reloaded from the next group (np)
    // as soon as it has been read.
    auto group = [&](const int8_t *np, auto refill_tag) {
        constexpr bool REFILL = decltype(refill_tag)::value;
#pragma unroll
        for (int j = 0; j < U; ++j) {
            uint4 w[R];
#pragma unroll
            for (int r = 0; r < R; ++r) {
                w[r] = wb[j][r];
                if constexpr (REFILL) wb[j][r] = ld_weight16(np + r * rb_bytes + j * 512, pol);
            }
            uint2 xv[MT][2];
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                xv[t][0] = __ldg(reinterpret_cast<const uint2 *>(xp[t] + j * 32));
                xv[t][1] = __ldg(reinterpret_cast<const uint2 *>(xp[t] + j * 32 + 16));
            }
            compute(j, w, xv);
        }
    };

    if (RING && fast) {
        int gi = rot;                              // slice group being processed
        int gn = rot + P < ng ? rot + P : rot + P - ng;  // slice group P ahead (valid while g + P < ng)
        for (int g = 0; g < ng; ++g) {
            cp_async_wait<(RING ? P : 1) - 1>();  // this lane's copies of group g have landed
            const int p = g % (RING ? P : 1);
            uint4 w[U][R];
#pragma unroll
            for (int j = 0; j < U; ++j)
#pragma unroll
                for (int r = 0; r < R; ++r) w[j][r] = lds16(ring_lane + ((p * U + j) * R + r) * 512);
            if (g + P < ng) {  // refill the ring group just read (same lane, program order)
                issue_group(p, gn);
                gn = gn + 1 == ng ? 0 : gn + 1;
            }
            cp_async_commit();
#pragma unroll
            for (int j = 0; j < U; ++j) {
                uint2 xv[MT][2];
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    xv[t][0] = __ldg(reinterpret_cast<const uint2 *>(xp[t] + j * 32));
                    xv[t][1] = __ldg(reinterpret_cast<const uint2 *>(xp[t] + j * 32 + 16));
                }
                compute(j, w[j], xv);
            }
            const bool wrap = gi + 1 == ng;
#pragma unroll
            for (int t = 0; t < MT; ++t) xp[t] = wrap ? xbase[t] : xp[t] + U * 32;
            gi = wrap ? 0 : gi + 1;
        }
    } else if (fast) {
        int gi = rot;  // slice group being processed
        for (int g = 0; g < ng; ++g) {
            if (pf_groups > 0) prefetch_group(g + pf_groups + 1);
            const bool wrap = gi + 1 == ng;  // the next group in the rotated order is group 0
            const int8_t *np = wrap ? wbase : gp + U * 512;
            if (g + 1 < ng) group(np, std::true_type{});
            else group(np, std::false_type{});
            gp = np;
#pragma unroll
            for (int t = 0; t < MT; ++t) xp[t] = wrap ? xbase[t] : xp[t] + U * 32;
            gi = wrap ? 0 : gi + 1;
        }
    } else {
        // Ragged slice: chunk by chunk with bounds checks; a 16-column half past K holds zero
        // weights and its activations are not read.
        const int kcols = K - c0 * 32;
        for (int c = 0; c < nch; c += U) {
#pragma unroll
            for (int j = 0; j < U; ++j) {
                if (c + j < nch) {
                    uint4 w[R];
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        w[r] = wb[j][r];
                        if (c + j + U < nch) wb[j][r] = ld_weight16(gp + r * rb_bytes + (U + j) * 512, pol);
                    }
                    uint2 xv[MT][2];
#pragma unroll
                    for (int t = 0; t < MT; ++t)
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int col = (c + j) * 32 + h * 16;
                            xv[t][h] = col < kcols ? __ldg(reinterpret_cast<const uint2 *>(xp[t] + j * 32 + h * 16))
                                                   : make_uint2(0, 0);
                        }
                    compute(j, w, xv);
                }
            }
            gp += U * 512;
#pragma unroll
            for (int t = 0; t < MT; ++t) xp[t] += U * 32;
        }
    }

    // K-split reduction across the accumulator sets and warps (fixed order), scale, store.
    __shared__ float red[KW][R][MT][4][32];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < MT; ++t)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float v = acc[0][r][t][j];
                if constexpr (NACC == 2) v += acc[1][r][t][j];
                red[warp][r][t][j][lane] = v;
            }
    __syncthreads();
    if constexpr (SILU_MUL) {
        // item (r, jj) = (wi >> 1, wi & 1) finishes row block r: gate row r0 (register jj)
        // and up row r0 (register 2 + jj), token 2q + jj of each tile.
        for (int wi = warp; wi < 2 * R; wi += KW) {  // KW may be smaller than 2R
            const int r = wi >> 1, jj = wi & 1;
            const int b = rg * R + r;
            const int n = b * 8 + r0;  // intermediate column
            if (n < N) {
                const float sg = __ldg(scale + b * 16 + r0), su = __ldg(scale + b * 16 + 8 + r0);
#pragma unroll
                for (int t = 0; t < MT; ++t) {
                    const int m = m0 + 8 * t + 2 * q + jj;
                    if (m < M) {
                        float vg = 0.f, vu = 0.f;
#pragma unroll
                        for (int w = 0; w < KW; ++w) {
                            vg += red[w][r][t][jj][lane];
                            vu += red[w][r][t][2 + jj][lane];
                        }
                        const float g = vg * sg, u = vu * su;
                        y[static_cast<int64_t>(m) * ldy + n] = __float2bfloat16_rn(g / (1.f + expf(-g)) * u);
                    }
                }
            }
        }
    } else {
    // item (r, j) = (wi >> 2, wi & 3) finishes accumulator register j of row block r:
    // row r0 + 8*(j>>1), token 2q + (j & 1) of each tile (16x8 accumulator layout).
    for (int wi = warp; wi < 4 * R; wi += KW) {  // KW may be smaller than 4R
        const int r = wi >> 2, j = wi & 3;
        const int n = (rg * R + r) * 16 + r0 + 8 * (j >> 1);
        if (n < N) {
            const float sc = __ldg(scale + n);
#pragma unroll
            for (int t = 0; t < MT; ++t) {
                const int m = m0 + 8 * t + 2 * q + (j & 1);
                if (m < M) {
                    float v = 0.f;
#pragma unroll
                    for (int w = 0; w < KW; ++w) v += red[w][r][t][j][lane];
                    v *= sc;
                    if (res) v += __bfloat162float(res[static_cast<int64_t>(m) * ldr + n]);
                    y[static_cast<int64_t>(m) * ldy + n] = __float2bfloat16_rn(v);
                }
            }
        }
    }
    }
}

}  // namespace lse

