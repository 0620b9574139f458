// Skinny int8 weight-only GEMM for decode (M <= 32 tokens; the auto policy uses it up to 16),
// on the packed weights of pack_w.cuh.
//
//   y[m, n] = s[n] * sum_k x[m, k] * w[n, k]
//
// Decode is bound by the weight stream (2 flop per weight byte per token).  The kernel is
// shaped so that nothing but HBM bounds it, and so that consecutive projections overlap:
//   * one CTA of KW warps owns R blocks of 16 output channels over all of K; warp w takes a
//     contiguous slice of each block's 64-column units;
//   * a unit is two 128-bit streaming loads per lane (L1 no-allocate, L2 evict-first) that
//     read 512 contiguous bytes each per warp, four 128-byte lines, 1 KB apart: row r0's 16
//     columns 16q..16q+15 of the unit and row r0 + 8's (lane 4 * r0 + q); a warp's slice of
//     a row block is one contiguous run (pack_w.cuh).  Word j of the two loads is
//     the A fragment of the unit's j-th 16x8x16 warp MMA (pack_w.cuh), so there is no
//     shared-memory staging, no copy bookkeeping and no wait on a barrier.  U loads per row
//     block (U / 2 units) are kept in flight per lane, issued before the previous kernel is
//     waited for (weights never depend on it);
//   * the activations of a unit are 32 contiguous bytes per lane (columns 16q..16q+15 of its
//     token), two 128-bit loads (one per 32-column half, consumed as it is loaded), whose
//     4-column quads pair with the weight words;
//   * weights are widened in registers - to fp16 with one byte permute + one fp16
//     subtraction per pair after flipping the sign bits (exact: fp16 holds 1024 + (v + 128)),
//     with the activations rounded bf16 -> fp16 per fragment (exact for |x| in
//     [2^-14, 65504], saturating beyond); or, with BF16 set, to bf16 (two logic ops + one bf16
//     subtraction per pair, exact) against the bf16 activations as they are - and fed to warp
//     MMAs with fp32 accumulation;
//   * the K split is reduced across the warps through shared memory in a fixed order and the
//     per-channel scale is applied once to each reduced sum (deterministic);
//   * the CTA signals programmatic launch completion on entry: it holds only a small
//     reduction buffer in shared memory, so the next kernel's CTAs become resident as soon as
//     registers free up and start their own weight streams under this kernel's tail.
//   * optional epilogues: the residual add (y = res + s * acc) and, for the MLP, SiLU(gate) *
//     up on gate/up rows interleaved in 8-row blocks.
// No workspace, no cross-CTA traffic, no spin-waits.
#pragma once

#include <type_traits>

#include "pack_w.cuh"
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
// where it is issued - ahead of the wait on the previous kernel and U loads ahead of its
// use - instead of sinking it to the first use.
__device__ __forceinline__ uint4 ld_weight16(const int8_t *p, uint64_t policy) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p), "l"(policy));
    return r;
}

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int j) {
    return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

// y = bf16(s * acc), or bf16(res + s * acc) when `res` is given (it may be y itself: each
// element is read, then written, by one thread).
//
// MT token tiles of 8 per CTA (M <= 8 * MT), KW warps splitting K, R row blocks per CTA
// (sharing every activation load), U 512-byte loads (U / 2 units) per row block in flight
// per lane, BF16 selects the bf16 MMA.
//
// Bytes in flight per SM (resident warps x U x 512), then instructions per unit, bound this
// kernel, so the main path is written for both: warp w streams a contiguous slice of the
// row block's units in whole groups of U / 2, with every load at a constant offset from a
// pointer that moves once per group and no per-unit predicate; the groups are visited in an
// order rotated per CTA, so the CTAs resident together read different offsets of their row
// blocks.  A slice that is not a whole number of groups (ragged K) takes a bounds-checked
// path.  `pf_groups` groups per row block beyond the units in registers are prefetched into
// L2 by lane 0 (bulk prefetches), which deepens the stream at no register cost.
//
// SILU_MUL: the weight rows interleave 8-row blocks of the MLP's gate and up projections
// (row block b = gate rows 8b..8b+7, then the matching up rows 8b..8b+7), so the 16x8
// accumulator of one lane holds gate row r0 (registers 0, 1) and up row r0 (registers 2, 3)
// of the same tokens, and the epilogue writes y[m, 8b + r0] = silu(s_g * gate) * (s_u * up)
// (fp32, one bf16 rounding) for the N = I intermediate columns; `scale` is interleaved the
// same way.
//
// XT is the activation type of x, y and res: bf16, or fp16 (then the MMA is fp16 and the
// activations enter it as they are).
template <int MT, int KW, int R, int U, bool BF16, int MINB, bool SILU_MUL = false, typename XT = __nv_bfloat16>
__global__ void __launch_bounds__(KW * 32, MINB)
skinny_i8_kernel(const XT *__restrict__ x, int64_t ldx, int M, int K,
                 const int8_t *__restrict__ wp, const float *__restrict__ scale, int N,
                 XT *y, int64_t ldy, const XT *res, int64_t ldr, int Kp, int pf_groups) {
    constexpr bool XF16 = std::is_same_v<XT, __half>;
    static_assert(!(XF16 && BF16), "fp16 activations take the fp16 MMA");
    constexpr int UB = U >= 2 ? U / 2 : 1;  // 64-column units per row block in registers
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int rg = blockIdx.x;
    const int m0 = blockIdx.y * MT * 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = lane >> 2, q = lane & 3;
    const int ku_real = (K + 63) >> 6;  // 64-column units holding real columns
    // an even number of units per warp: a slice then starts on a 2 KB block, and a unit j of a
    // group of UB (even) sits at the compile-time offset packed_unit_offset(j) from its group
    const int per = ((ku_real + KW - 1) / KW + 1) & ~1;
    const int c0 = min(ku_real, warp * per), c1 = min(ku_real, c0 + per);
    const int nch = c1 - c0;
    // Whole groups, and every column < K (only the last unit of the row can be partial).
    const bool fast = nch > 0 && nch % UB == 0 && c1 * 64 <= K;
    const int ng = nch / UB;
    const int rot = fast ? rg % ng : 0;

    const uint64_t pol = ptx::policy_evict_first();
    // Row block rg*R + r (padded rows past N hold zeros) is one run of 16 * Kp bytes at
    // row_base + r * rb_bytes; unit u of it at packed_unit_offset(u), its second 8-row group
    // 1 KB further on.  Lane (r0, q) reads row r0's 16-byte chunk q of each 512-byte atom,
    // stored at chunk position q ^ ((r0 >> 1) & 3), so eight consecutive lanes read one
    // 128-byte line.
    const int64_t rb_bytes = static_cast<int64_t>(Kp) * 16;
    constexpr int64_t grp_bytes = 1024;
    const int8_t *const row_base = wp + static_cast<int64_t>(rg) * R * rb_bytes;
    const int8_t *const lane_base = row_base + r0 * 64 + ((q ^ ((r0 >> 1) & 3)) << 4);
    // first unit of slice group gv (groups start on even units when UB is even)
    auto group_ptr = [&](int gv) { return lane_base + packed_unit_offset(c0 + gv * UB); };
    const int8_t *gp = group_ptr(rot);
    uint4 wb[UB][R][2];
#pragma unroll
    for (int j = 0; j < UB; ++j)
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int h = 0; h < 2; ++h)
                wb[j][r][h] = (fast || j < nch)
                                  ? ld_weight16((fast ? gp + packed_unit_offset(j) : lane_base + packed_unit_offset(c0 + j)) +
                                                    r * rb_bytes + h * grp_bytes, pol)
                                  : make_uint4(0, 0, 0, 0);
    // L2 prefetch of the group `v` visits ahead (lane 0, one bulk prefetch per row block of the
    // 2 KB blocks holding the group's units): the register loads then hit L2, so the registers
    // hold only UB units while DRAM has pf_groups more groups per row block in flight.
    auto prefetch_group = [&](int v) {
        if (lane == 0 && v < ng) {
            int gv = rot + v;
            if (gv >= ng) gv -= ng;
            const int u0 = c0 + gv * UB;
            const int blocks = ((u0 + UB - 1) >> 1) - (u0 >> 1) + 1;
            const int8_t *base = row_base + static_cast<int64_t>(u0 >> 1) * 2048;
#pragma unroll
            for (int r = 0; r < R; ++r) ptx::bulk_prefetch_l2(base + r * rb_bytes, blocks * 2048);
        }
    };
    if (fast)
        for (int v = 1; v <= pf_groups; ++v) prefetch_group(v);

    asm volatile("griddepcontrol.wait;" ::: "memory");  // x is the previous kernel's output

    // Activation rows this lane feeds as the B fragment of token tile t: token m0 + 8t + r0,
    // columns 16q..16q+15 of each unit.  A token past M reads the last real row instead: its
    // MMA column is independent of the others and is never stored.
    const XT *xbase[MT];
    const XT *xp[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        const int m = min(m0 + 8 * t + r0, M - 1);
        xbase[t] = x + static_cast<int64_t>(m) * ldx + 16 * q + c0 * 64;
        xp[t] = xbase[t] + rot * (UB * 64);
    }

    // With a single MMA chain (R * MT == 1) alternate two accumulator sets by MMA parity.
    constexpr int NACC = R * MT == 1 ? 2 : 1;
    float acc[NACC][R][MT][4];
#pragma unroll
    for (int u = 0; u < NACC; ++u)
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
            for (int t = 0; t < MT; ++t) acc[u][r][t][0] = acc[u][r][t][1] = acc[u][r][t][2] = acc[u][r][t][3] = 0.f;

    // Half a unit (32 columns, h = 0 or 1): B fragments from 8 of the lane's activation columns
    // per token tile (one 128-bit load), A fragments widened from words 2h and 2h + 1 of the two
    // weight loads of each row block, two 16x8x16 MMAs per token tile and block (MMA j takes
    // the 4-column quad j of the lane's 16 columns).
    auto compute_half = [&](const uint4 (&wr)[R][2], int h, const uint4 (&xv)[MT]) {
        uint32_t bx[MT][2][2];
#pragma unroll
        for (int t = 0; t < MT; ++t)
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                const uint32_t lo = jj ? xv[t].z : xv[t].x, hi = jj ? xv[t].w : xv[t].y;
                if constexpr (BF16 || XF16) {
                    bx[t][jj][0] = lo;
                    bx[t][jj][1] = hi;
                } else {
                    bx[t][jj][0] = bf16x2_to_f16x2(lo);
                    bx[t][jj][1] = bf16x2_to_f16x2(hi);
                }
            }
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                const int j = 2 * h + jj;
                const uint32_t wa = word_of(wr[r][0], j), wb8 = word_of(wr[r][1], j);  // rows r0, r0 + 8
                uint32_t lo01, lo23, hi01, hi23;
                if constexpr (BF16) {
                    i8x4_to_bf16x4(wa, lo01, lo23);
                    i8x4_to_bf16x4(wb8, hi01, hi23);
                } else {
                    u8x4_to_f16x4(wa ^ 0x80808080u, lo01, lo23);
                    u8x4_to_f16x4(wb8 ^ 0x80808080u, hi01, hi23);
                }
                const uint32_t a[4] = {lo01, hi01, lo23, hi23};
#pragma unroll
                for (int t = 0; t < MT; ++t) mma_16816<BF16>(acc[NACC == 2 ? jj : 0][r][t], a, bx[t][jj][0], bx[t][jj][1]);
            }
        }
    };
    // One unit at xp offset j: both halves.
    auto compute = [&](const uint4 (&wr)[R][2], int j, bool col_ok) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            uint4 xv[MT];
#pragma unroll
            for (int t = 0; t < MT; ++t)
                xv[t] = col_ok ? __ldg(reinterpret_cast<const uint4 *>(xp[t] + j * 64 + 8 * h)) : make_uint4(0, 0, 0, 0);
            compute_half(wr, h, xv);
        }
    };
    // One whole group at gp / xp; with REFILL, slot j is reloaded from the next group (np)
    // as soon as it has been read.
    auto group = [&](const int8_t *np, auto refill_tag) {
        constexpr bool REFILL = decltype(refill_tag)::value;
#pragma unroll
        for (int j = 0; j < UB; ++j) {
            uint4 w[R][2];
#pragma unroll
            for (int r = 0; r < R; ++r)
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    w[r][h] = wb[j][r][h];
                    if constexpr (REFILL)
                        wb[j][r][h] = ld_weight16(np + packed_unit_offset(j) + r * rb_bytes + h * grp_bytes, pol);
                }
            compute(w, j, true);
        }
    };

    if (fast) {
        int gi = rot;  // slice group being processed
        for (int g = 0; g < ng; ++g) {
            if (pf_groups > 0) prefetch_group(g + pf_groups + 1);
            const bool wrap = gi + 1 == ng;  // the next group in the rotated order is group 0
            const int8_t *np = group_ptr(wrap ? 0 : gi + 1);
            if (g + 1 < ng) group(np, std::true_type{});
            else group(np, std::false_type{});
            gp = np;
#pragma unroll
            for (int t = 0; t < MT; ++t) xp[t] = wrap ? xbase[t] : xp[t] + UB * 64;
            gi = wrap ? 0 : gi + 1;
        }
    } else {
        // Ragged slice: unit by unit with bounds checks; a lane's 16 columns past K hold zero
        // weights and their activations are not read.
        const int kcols = K - c0 * 64;
        for (int c = 0; c < nch; c += UB) {
#pragma unroll
            for (int j = 0; j < UB; ++j) {
                if (c + j < nch) {
                    uint4 w[R][2];
#pragma unroll
                    for (int r = 0; r < R; ++r)
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            w[r][h] = wb[j][r][h];
                            if (c + j + UB < nch)
                                wb[j][r][h] = ld_weight16(lane_base + packed_unit_offset(c0 + c + UB + j) + r * rb_bytes +
                                                              h * grp_bytes,
                                                          pol);
                        }
                    const bool col_ok = (c + j) * 64 + 16 * q < kcols;  // K % 16 == 0: all 16 or none
                    compute(w, j, col_ok);
                }
            }
#pragma unroll
            for (int t = 0; t < MT; ++t) xp[t] += UB * 64;
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
                        y[static_cast<int64_t>(m) * ldy + n] = from_float<XT>(g / (1.f + expf(-g)) * u);
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
                    if (res) v += to_float(res[static_cast<int64_t>(m) * ldr + n]);
                    y[static_cast<int64_t>(m) * ldy + n] = from_float<XT>(v);
                }
            }
        }
    }
    }
}

}  // namespace lse
