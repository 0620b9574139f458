// tcgen05 int8 x int8 tensor-core kernel for the int8 weight-only linear (sm_100a).
//
//   y[m, n] = s[n] * r[m] * sum_p 256^(S-1-p) * sum_k w[n, k] * d_p[m, k]
//
// where d_p are the S digit planes of the activations under the row scale r (act_split.cuh:
// x[m, k] ~= r[m] * sum_p 256^(S-1-p) d_p[m, k], exact for every element at least 2^(10-8S)
// times the row maximum, see there).  Every product and sum of the contraction is exact
// (tcgen05.mma kind::i8, int32 accumulators); the only roundings are the activations'
// fixed-point representation, the fp32 combination of the S planes and the scales, and the
// final bf16 rounding.
//
// Operand roles ("swap-AB"): the 128 weight rows of a tile are the MMA's A operand (M = 128)
// and the token columns of the S planes its N dimension (N = S * NT), so one
// tcgen05.mma.kind::i8 computes D[128 rows, S * NT] over 32 K.  Both operands come from
// shared memory, written there by TMA and read by the tensor core through matrix
// descriptors; nothing widens the weights and nothing but the MMA touches them between the
// copy and the accumulator.
//   * W: row-major int8 [N, K] with a 128-byte swizzle (box 128 K x 128 rows), or the
//     packed layout (pack_w.cuh: 512-byte atoms of 8 rows x 64 columns stored with the 64-byte
//     swizzle, 2 KB per 16-row block and 128 columns; box 8 row blocks x 2 KB, copied as it is).
//   * digit planes: int8 [S][M][Kp], one 3-D box [S][NT][128 K] with a 128-byte swizzle.
//   * D: int32 in tensor memory, double-buffered; four epilogue warps read it (tcgen05.ld),
//     combine the planes, apply s[n] * r[m] (and the optional residual or SiLU * mul) and
//     store bf16 y.
//   * SILU = true: the MLP's gate_up with SiLU * mul, rows interleaved in 8-row blocks of
//     gate and up (as in the decode kernel): a 16-row block's gate row and up row are TMEM
//     lanes 8 apart in one warp; y is [M, N / 2].
//
// Warp roles (256 threads): warp 0 TMA producer, warp 1 TMEM allocator + single-thread MMA
// issuer, warp 2 L2 prefetcher of the weight stream, warps 4-7 epilogue (TMEM lane quarter =
// warp % 4).
//
// Work distribution (the host plan's schedule): tiles are (128 weight rows) x (NT tokens),
// tile = n_tile * m_tiles + m_tile.  Full waves are dealt round-robin to a persistent grid
// (data-parallel part); the remaining tiles are cut into 128-K units spread over the grid
// (stream-K part).  A tile whose K range is split is finished by whichever CTA arrives last on
// the tile's counter: every segment writes its fp32 partial (the planes already combined) to
// the workspace and bumps the counter; the last one re-zeroes the counter and, once its role
// loops are done, sums all partials in segment order (deterministic) with all 256 threads,
// applies the scales and stores y.  No CTA ever waits for another CTA.
//
// CLUSTER = true (few tiles, decode): every tile's K range is split evenly over the p.cluster
// CTAs of one thread-block cluster, each CTA holding one segment.  Each CTA leaves its fp32
// partial in its own shared memory (the drained stage buffers); after a cluster barrier CTA r
// sums token rows [NT r / c, NT (r + 1) / c) of all c partials through distributed shared
// memory in rank order (deterministic), applies the scales and stores y; a second cluster
// barrier keeps every partial alive until all have been read.  No global partials, counters or
// last-arriver tail.  The cluster's CTAs are co-scheduled, and every CTA reaches both barriers
// on every path (a CTA whose bounded wait gave up skips its data work, not the barriers).
//
// Every mbarrier wait is bounded (tc_ptx.cuh: mbar_wait); on a timeout the CTA raises an
// abort flag, records LSE_ERR_DEVICE_TIMEOUT, drains its own copies and MMAs, frees TMEM
// and returns.
#pragma once

#include "tc_ptx.cuh"

namespace lse {
namespace tci8 {

constexpr int BN = 128;                 // weight rows per tile (MMA M)
constexpr int BK = 128;                 // K per pipeline stage (bytes of int8)
constexpr int UK = 32;                  // K per tcgen05.mma kind::i8
constexpr int KSTEPS = BK / UK;         // MMAs per stage
constexpr int W_STAGE_BYTES = BN * BK;  // int8 weight tile per stage
constexpr int NUM_THREADS = 256;
constexpr int WARP_TMA = 0, WARP_MMA = 1, WARP_PREFETCH = 2, WARP_EPI0 = 4;
constexpr int NUM_EPI_WARPS = 4;
constexpr int EPI_BAR = 1;              // named barrier of the epilogue warps
constexpr int TMEM_COLS = 512;
// A throttle wait of the L2 prefetcher that exceeds this gives up prefetching (~20 us).
constexpr long long kPrefetchWaitCycles = 40000;
constexpr int kSmemBudget = 220 * 1024;  // stages + control block (227 KB per CTA at most)
constexpr int kMaxCluster = 8;          // CTAs per cluster in the CLUSTER schedule (portable size)

template <int NT, int S>
struct Cfg {
    static_assert(NT == 32 || NT == 64 || NT == 128, "token tile");
    static_assert(S == 2 || S == 3, "digit planes");
    static constexpr int NMMA = S * NT;  // MMA N: token columns of every plane
    static_assert(NMMA % 16 == 0 && NMMA <= 256, "tcgen05 N for M = 128");
    static constexpr int X_STAGE_BYTES = S * NT * BK;
    static constexpr int STAGE_BYTES = W_STAGE_BYTES + X_STAGE_BYTES;
    static constexpr int ACC_BUFS = 2;
    // Independent accumulators per buffer where tensor memory allows: consecutive K32 MMAs of
    // a stage alternate between them, so small-N MMAs do not queue on one accumulator.
    static constexpr int NACC = ACC_BUFS * 2 * NMMA <= TMEM_COLS ? 2 : 1;
    static constexpr int ACC_COLS = NACC * NMMA;
    static_assert(ACC_BUFS * ACC_COLS <= TMEM_COLS, "TMEM budget");
    static constexpr int STAGES_FIT = (kSmemBudget - 1024 - 256) / STAGE_BYTES;
    static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
    static_assert(STAGES >= 3, "pipeline depth");
    // barrier block after the stages: full, empty (STAGES each), d_full, d_empty (ACC_BUFS),
    // drain, teardown; then tmem address, abort flag and the pending stream-K reductions (count + 2 x
    // {tile, first CTA, last CTA}).
    static constexpr int NUM_BARS = 2 * STAGES + 2 * ACC_BUFS + 2;
    static constexpr int CTRL_BYTES = NUM_BARS * 8 + 48;
    static constexpr int SMEM_BYTES = 1024 /*alignment slack*/ + STAGES * STAGE_BYTES + CTRL_BYTES;
    // kind::i8: D s32 (bits 4-5 = 2), A s8 (bits 7-9 = 1), B s8 (bits 10-12 = 1), both
    // K-major, N >> 3 at [17, 23), M >> 4 at [24, 29).
    static constexpr uint32_t IDESC =
        (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(NMMA >> 3) << 17) | (static_cast<uint32_t>(BN >> 4) << 24);
};

struct Params {
    int M, N, K;
    uint16_t *y;               // bf16, or fp16 when y_f16 (the activation type)
    int64_t ldy;
    const uint16_t *res;       // null, or the residual added before rounding (may alias y), same type
    int64_t ldr;
    int y_f16;
    const float *scale;        // s[n]
    const float *row_scale;    // r[m] (act_split)
    float *partials;           // [2 * grid][NT][BN] fp32 partial tiles
    int *counters;             // [stream-K tiles] arrival counters (zeroed by the split kernel)
    int m_tiles, tiles, kb, dp_tiles, grid;
    long long sk_units;
    int cluster;               // CTAs per tile in a thread-block cluster (CLUSTER kernels)
    const int8_t *w;           // weights (L2 prefetch addresses; the copies use the tensor map)
    int64_t kp;                // packed layout: padded K
    int pf_stages;             // L2 prefetch distance in stages beyond the shared-memory ring
};

// Shared-memory descriptor of the packed weight tile: K-major with the 64-byte swizzle (rows
// of 64 bytes, 8-row atoms of 512 bytes, the next 64 columns of a group in the next atom),
// 8-row groups 1 KB apart (stride byte offset), leading byte offset unused (1); version 1
// [46,48), layout SWIZZLE_64B (4) [61,64).  Atoms sit at 512-byte-aligned shared addresses, so
// the swizzle the hardware applies (address bits [4,5] ^= [7,8]) is the one the pack kernel
// stored; stepping K by 32 inside a 64-byte row adds 32 to the start address.
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t addr) {
    uint64_t d = 0;
    d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(4u) << 61;
    return d;
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::i8 (s8 x s8 -> s32), 1 CTA.
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 3-D tiled load global -> shared (box [c2][c1][c0]), completion counted in bytes on `bar`.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void *tmap, uint32_t bar, int c0, int c1, int c2,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
        : "memory");
}

// silu(a) = a / (1 + e^-a) with the fast exponential and division intrinsics (relative error a
// few fp32 ulp, far below the one bf16 rounding of the result); for a below about -88 the
// exponential overflows and the quotient is -0, the limit of silu.
__device__ __forceinline__ float silu_fast(float a) { return __fdividef(a, 1.f + __expf(-a)); }

// The activation type of y and the residual is bf16 or fp16 (p.y_f16, uniform in a launch).
__device__ __forceinline__ uint16_t out_bits(const Params &p, float v) {
    return p.y_f16 ? __half_as_ushort(__float2half_rn(v)) : __bfloat16_as_ushort(__float2bfloat16_rn(v));
}
__device__ __forceinline__ float res_value(const Params &p, int64_t i) {
    const uint16_t b = p.res[i];
    return p.y_f16 ? __half2float(__ushort_as_half(b)) : __bfloat162float(__ushort_as_bfloat16(b));
}

// ---- schedule (identical in every role and on the host) -----------------------------------
__device__ __forceinline__ long long sk_begin(const Params &p, int c) { return p.sk_units * c / p.grid; }
// Owner CTA of stream-K unit u: the largest c with sk_begin(c) <= u.
__device__ __forceinline__ int sk_owner(const Params &p, long long u) {
    return static_cast<int>(((u + 1) * p.grid + p.sk_units - 1) / p.sk_units) - 1;
}

struct Seg {
    int tile, k0, k1;
};

struct SegIter {
    int t_dp;
    long long u, u_end;
    __device__ __forceinline__ void init(const Params &p, int c) {
        t_dp = c;
        u = sk_begin(p, c);
        u_end = sk_begin(p, c + 1);
    }
    __device__ __forceinline__ bool next(const Params &p, Seg &s) {
        if (t_dp < p.dp_tiles) {
            s.tile = t_dp;
            s.k0 = 0;
            s.k1 = p.kb;
            t_dp += p.grid;
            return true;
        }
        if (u < u_end) {
            const long long ts = u / p.kb;
            s.tile = p.dp_tiles + static_cast<int>(ts);
            s.k0 = static_cast<int>(u - ts * p.kb);
            const long long rem = u_end - u;
            s.k1 = static_cast<int>(rem < (p.kb - s.k0) ? s.k0 + rem : p.kb);
            u += s.k1 - s.k0;
            return true;
        }
        return false;
    }
};

// Partial slot CTA c uses for stream-K tile `tile`: 2c for the first tile it touches, 2c+1 for
// the last (a CTA's middle tiles are complete and need no slot).
__device__ __forceinline__ int partial_slot(const Params &p, int c, int tile) {
    const int first_tile = p.dp_tiles + static_cast<int>(sk_begin(p, c) / p.kb);
    return 2 * c + (tile == first_tile ? 0 : 1);
}

// This CTA's (tile, k-block) stages in pipeline order (the L2 prefetcher's cursor).
struct StageCursor {
    SegIter it;
    Seg s;
    int kb = 0, k1 = 0;
    __device__ __forceinline__ void init(const Params &p, int c) { it.init(p, c); }
    __device__ __forceinline__ bool next(const Params &p, int &n0, int &kbo) {
        while (kb >= k1) {
            if (!it.next(p, s)) return false;
            kb = s.k0;
            k1 = s.k1;
        }
        n0 = (s.tile / p.m_tiles) * BN;
        kbo = kb++;
        return true;
    }
};

// Weights are read once when there is a single token tile (decode): stream them evict-first so
// the digit planes and the partial tiles keep L2.  With several token tiles each weight tile
// is re-read once per token tile: normal priority.
__device__ __forceinline__ uint64_t policy_w_for(const Params &p) {
    return p.m_tiles == 1 ? ptx::policy_evict_first() : ptx::policy_evict_normal();
}

// Weight tile (n0 / BN, kb) -> shared memory.  Packed: the tensor map views the buffer as
// [Np / 16 row blocks][2 * Kp eight-byte elements] and the box is 256 x 8 (8 row blocks x
// 2 KB), landing as 16 groups 1 KB apart.  Row-major: [N][K] bytes, box 128 x 128, 128-byte
// swizzle.
template <bool WPACK>
__device__ __forceinline__ void load_w_tile(const CUtensorMap *tmap_w, uint32_t dst, int n0, int kb, uint32_t bar,
                                            uint64_t pol) {
    if constexpr (WPACK) ptx::tma_load_2d(dst, tmap_w, bar, kb * 256, n0 / 16, pol);
    else ptx::tma_load_2d(dst, tmap_w, bar, kb * BK, n0, pol);
}

// One warp pulls weight tile (n0 / BN, kb) into L2 ahead of its TMA copy: 128 lines of 128
// bytes, 4 per lane.
template <bool WPACK>
__device__ __forceinline__ void prefetch_w_tile_l2(const Params &p, int n0, int kb, int lane) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int line = i * 32 + lane;
        if constexpr (WPACK) {
            const int b = line >> 4;  // row block within the tile, 16 lines of 128 bytes each
            ptx::prefetch_line_l2(p.w + static_cast<int64_t>(n0 / 16 + b) * 16 * p.kp + kb * 2048 + (line & 15) * 128);
        } else {
            const int r = n0 + line;
            if (r < p.N) ptx::prefetch_line_l2(p.w + static_cast<int64_t>(r) * p.K + kb * BK);
        }
    }
}

// y of row quad rq..rq+3 and token j of a tile from its fully reduced fp32 sums `acc` (planes
// combined): y = bf16(acc * s[n] * r[m] (+ residual)), or for SILU the gate quad takes the up
// quad's sums from lane + 2 (quad rq + 8) and writes silu(g) * u.  Called by whole warps whose
// lanes hold the 32 quads of one token in order.
template <bool SILU>
__device__ __forceinline__ void finish_quad(const Params &p, float4 acc, int j, int rq, int n_tile, int m0, int mval) {
    const int n = n_tile * BN + rq;
    const float rs = j < mval ? __ldg(p.row_scale + m0 + j) : 0.f;
    if constexpr (SILU) {
        const float u4[4] = {__shfl_xor_sync(0xffffffffu, acc.x, 2), __shfl_xor_sync(0xffffffffu, acc.y, 2),
                             __shfl_xor_sync(0xffffffffu, acc.z, 2), __shfl_xor_sync(0xffffffffu, acc.w, 2)};
        if (j >= mval || (rq & 8)) return;
        const float g4[4] = {acc.x, acc.y, acc.z, acc.w};
        uint16_t *yr = p.y + static_cast<int64_t>(m0 + j) * p.ldy + (n >> 4) * 8 + (n & 7);
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (n + e < p.N) {
                const float g = g4[e] * (__ldg(p.scale + n + e) * rs);
                const float u = u4[e] * (__ldg(p.scale + n + 8 + e) * rs);
                yr[e] = out_bits(p, silu_fast(g) * u);
            }
    } else {
        if (j >= mval) return;
        uint16_t *yr = p.y + static_cast<int64_t>(m0 + j) * p.ldy + n;
        const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (n + e < p.N) {
                float o = a4[e] * (__ldg(p.scale + n + e) * rs);
                if (p.res) o += res_value(p, static_cast<int64_t>(m0 + j) * p.ldr + n + e);
                yr[e] = out_bits(p, o);
            }
    }
}

// finish_quad with the row quad's scales already loaded: s4 = s[n..n+3], s4u = s[n+8..n+11]
// (SILU's up quad) and rs = r[m].
template <bool SILU>
__device__ __forceinline__ void finish_quad_scaled(const Params &p, float4 acc, float4 s4, float4 s4u, float rs, int j,
                                                   int rq, int n_tile, int m0, int mval) {
    const int n = n_tile * BN + rq;
    if constexpr (SILU) {
        const float u4[4] = {__shfl_xor_sync(0xffffffffu, acc.x, 2), __shfl_xor_sync(0xffffffffu, acc.y, 2),
                             __shfl_xor_sync(0xffffffffu, acc.z, 2), __shfl_xor_sync(0xffffffffu, acc.w, 2)};
        if (j >= mval || (rq & 8)) return;
        const float g4[4] = {acc.x, acc.y, acc.z, acc.w};
        const float sg[4] = {s4.x, s4.y, s4.z, s4.w};
        const float su[4] = {s4u.x, s4u.y, s4u.z, s4u.w};
        uint16_t *yr = p.y + static_cast<int64_t>(m0 + j) * p.ldy + (n >> 4) * 8 + (n & 7);
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (n + e < p.N) yr[e] = out_bits(p, silu_fast(g4[e] * (sg[e] * rs)) * (u4[e] * (su[e] * rs)));
    } else {
        if (j >= mval) return;
        uint16_t *yr = p.y + static_cast<int64_t>(m0 + j) * p.ldy + n;
        const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
        const float sc[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (n + e < p.N) {
                float o = a4[e] * (sc[e] * rs);
                if (p.res) o += res_value(p, static_cast<int64_t>(m0 + j) * p.ldr + n + e);
                yr[e] = out_bits(p, o);
            }
    }
}

// Combine the S planes of one accumulator column: sum_p 256^(S-1-p) d_p.
template <int S>
__device__ __forceinline__ float combine_planes(const int32_t (&d)[S]) {
    if constexpr (S == 2) return fmaf(static_cast<float>(d[0]), 256.f, static_cast<float>(d[1]));
    else return fmaf(static_cast<float>(d[0]), 65536.f, fmaf(static_cast<float>(d[1]), 256.f, static_cast<float>(d[2])));
}

// ---- the kernel -------------------------------------------------------------------------
template <int NT, int S, bool SILU, bool WPACK, bool CLUSTER = false>
__global__ void __launch_bounds__(NUM_THREADS, 1)
tc_i8_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
             const Params p) {
    using C = Cfg<NT, S>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~static_cast<uintptr_t>(1023));
    uint8_t *w_smem = smem;                               // STAGES x 16 KB
    uint8_t *x_smem = smem + C::STAGES * W_STAGE_BYTES;   // STAGES x X_STAGE_BYTES
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE_BYTES);
    uint64_t *full = bars;
    uint64_t *empty = full + C::STAGES;
    uint64_t *d_full = empty + C::STAGES;
    uint64_t *d_empty = d_full + C::ACC_BUFS;
    uint64_t *drain = d_empty + C::ACC_BUFS;
    uint64_t *td_bar = drain + 1;  // teardown: one arrival per warp
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(td_bar + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(td_bar + 1) + 1;
    volatile int *pending = reinterpret_cast<volatile int *>(td_bar + 1) + 2;  // [0] count, then triples

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < C::STAGES; ++i) {
            ptx::mbar_init(ptx::smem_u32(&full[i]), 1);
            ptx::mbar_init(ptx::smem_u32(&empty[i]), 1);
        }
        for (int i = 0; i < C::ACC_BUFS; ++i) {
            ptx::mbar_init(ptx::smem_u32(&d_full[i]), 1);
            ptx::mbar_init(ptx::smem_u32(&d_empty[i]), NUM_EPI_WARPS);
        }
        ptx::mbar_init(ptx::smem_u32(drain), 1);
        ptx::mbar_init(ptx::smem_u32(td_bar), NUM_THREADS / 32);
        *abort_flag = 0;
        pending[0] = 0;
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tmap_w);
        ptx::prefetch_tmap(&tmap_x);
    }
    if (warp == WARP_MMA) {
        ptx::tmem_alloc(ptx::smem_u32(const_cast<uint32_t *>(tmem_slot)), TMEM_COLS);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    ptx::cta_sync_all();
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    SegIter it;
    it.init(p, blockIdx.x);
    Seg s;

    if (threadIdx.x == 0) ptx::grid_dep_launch();

    if (warp == WARP_TMA) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            const uint64_t pol_w = policy_w_for(p);
            const uint64_t pol_x = ptx::policy_evict_last();
            // Weights never depend on the previous kernels: the first stages' weight copies
            // start before the wait (programmatic dependent launch); the digit planes follow
            // once the split kernel's output is visible.
            long long pre = 0;
            {
                SegIter ip = it;
                Seg sp;
                while (pre < C::STAGES && ip.next(p, sp)) {
                    const int n0 = (sp.tile / p.m_tiles) * BN;
                    for (int kb = sp.k0; kb < sp.k1 && pre < C::STAGES; ++kb, ++pre) {
                        const uint32_t fb = ptx::smem_u32(&full[pre]);
                        ptx::mbar_arrive_expect_tx(fb, C::STAGE_BYTES);
                        load_w_tile<WPACK>(&tmap_w, ptx::smem_u32(w_smem + pre * W_STAGE_BYTES), n0, kb, fb, pol_w);
                    }
                }
            }

            ptx::grid_dep_wait();
            long long pos = 0;  // stages issued so far
            bool ok = true;
            while (ok && it.next(p, s)) {
                const int n0 = (s.tile / p.m_tiles) * BN;
                const int m0 = (s.tile % p.m_tiles) * NT;
                for (int kb = s.k0; kb < s.k1; ++kb, ++pos) {
                    const int st = static_cast<int>(pos % C::STAGES);
                    const uint32_t ph = static_cast<uint32_t>((pos / C::STAGES) & 1);
                    const uint32_t fb = ptx::smem_u32(&full[st]);
                    if (pos >= pre) {
                        if (!ptx::mbar_wait(ptx::smem_u32(&empty[st]), ph ^ 1, abort_flag)) {
                            ok = false;
                            break;
                        }
                        ptx::mbar_arrive_expect_tx(fb, C::STAGE_BYTES);
                        load_w_tile<WPACK>(&tmap_w, ptx::smem_u32(w_smem + st * W_STAGE_BYTES), n0, kb, fb, pol_w);
                    }
                    tma_load_3d(ptx::smem_u32(x_smem + st * C::X_STAGE_BYTES), &tmap_x, fb, kb * BK, m0, 0, pol_x);
                }
            }
            // Drain: every copy this CTA issued must land before shared memory is released.
            if (pos < pre) {
                // aborted before the loop reached every prefetched stage: issue their plane
                // copies so each prefetched barrier can complete, then drain
                for (long long q = pos; q < pre; ++q)
                    tma_load_3d(ptx::smem_u32(x_smem + q * C::X_STAGE_BYTES), &tmap_x, ptx::smem_u32(&full[q]), 0, 0, 0,
                                pol_x);
                pos = pre;
            }
            const long long first = pos > C::STAGES ? pos - C::STAGES : 0;
            for (long long q = first; q < pos; ++q)
                ptx::mbar_drain(ptx::smem_u32(&full[q % C::STAGES]), static_cast<uint32_t>((q / C::STAGES) & 1));
        }
    } else if (warp == WARP_MMA) {
        // ---------------- MMA issuer (one thread) ----------------
        if (lane == 0) {
            long long pos = 0, dpos = 0;
            bool ok = true;
            while (ok && it.next(p, s)) {
                const int buf = static_cast<int>(dpos % C::ACC_BUFS);
                const uint32_t dph = static_cast<uint32_t>((dpos / C::ACC_BUFS) & 1);
                if (!ptx::mbar_wait(ptx::smem_u32(&d_empty[buf]), dph ^ 1, abort_flag)) break;
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem_base + buf * C::ACC_COLS;
                for (int kb = s.k0; kb < s.k1; ++kb, ++pos) {
                    const int st = static_cast<int>(pos % C::STAGES);
                    const uint32_t ph = static_cast<uint32_t>((pos / C::STAGES) & 1);
                    if (!ptx::mbar_wait(ptx::smem_u32(&full[st]), ph, abort_flag)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const uint32_t wa = ptx::smem_u32(w_smem + st * W_STAGE_BYTES);
                    const uint32_t xa = ptx::smem_u32(x_smem + st * C::X_STAGE_BYTES);
#pragma unroll
                    for (int j = 0; j < KSTEPS; ++j) {
                        // A: packed = 32 bytes inside a 64-byte row, the next atom every 64 K;
                        // row-major = 32 bytes inside the 128-byte row.  B: 32 bytes inside its row.
                        const uint64_t a_desc = WPACK ? smem_desc_sw64(wa + (j >> 1) * 512 + (j & 1) * UK)
                                                      : ptx::smem_desc_sw128(wa + j * UK);
                        const uint64_t b_desc = ptx::smem_desc_sw128(xa + j * UK);
                        const int acc = j % C::NACC;
                        mma_i8_ss(d_tmem + acc * C::NMMA, a_desc, b_desc, C::IDESC, (kb > s.k0 || j >= C::NACC) ? 1u : 0u);
                    }
                    // One commit per stage frees the shared-memory stage for the producer.
                    ptx::mma_commit(ptx::smem_u32(&empty[st]));
                }
                if (!ok) break;
                ptx::mma_commit(ptx::smem_u32(&d_full[buf]));
                ++dpos;
            }
            // Drain: all MMAs this thread issued must finish before TMEM is freed.
            ptx::mma_commit(ptx::smem_u32(drain));
            ptx::mbar_drain(ptx::smem_u32(drain), 0);
        }
    } else if (warp == WARP_PREFETCH) {
        // ---------------- L2 prefetcher ----------------
        // Keeps p.pf_stages weight tiles of this CTA in flight to L2 ahead of the bulk-copy
        // engine, throttled by the `full` barriers; only a hint: a long throttle wait stops it.
        if (p.pf_stages > 0) {
            StageCursor cur;
            cur.init(p, blockIdx.x);
            int n0, kbo;
            for (long long i = 0; cur.next(p, n0, kbo); ++i) {
                const long long j = i - p.pf_stages;
                if (j >= 0) {
                    const uint32_t bar = ptx::smem_u32(&full[j % C::STAGES]);
                    const uint32_t par = static_cast<uint32_t>((j / C::STAGES) & 1);
                    bool landed = false;
                    const long long t0 = clock64_now();
                    while (!(landed = ptx::mbar_try_wait(bar, par)) && !*abort_flag &&
                           clock64_now() - t0 < kPrefetchWaitCycles) {
                    }
                    landed = __all_sync(0xffffffffu, landed);
                    if (!landed) break;
                }
                prefetch_w_tile_l2<WPACK>(p, n0, kbo, lane);
            }
        }
    } else if (warp >= WARP_EPI0 && warp < WARP_EPI0 + NUM_EPI_WARPS) {
        // ---------------- epilogue: TMEM -> planes combined -> scales -> bf16 y or partial ----
        ptx::grid_dep_wait();  // y, partials, counters and r[m] belong to earlier kernels until now
        const int q = warp & 3;
        const int row = q * 32 + lane;
        long long dpos = 0;
        while (it.next(p, s)) {
            const int buf = static_cast<int>(dpos % C::ACC_BUFS);
            const uint32_t dph = static_cast<uint32_t>((dpos / C::ACC_BUFS) & 1);
            const bool w_ok = ptx::mbar_wait(ptx::smem_u32(&d_full[buf]), dph, abort_flag);
            if (!ptx::bar_and(EPI_BAR, NUM_EPI_WARPS * 32, w_ok)) break;
            ptx::tc_fence_after();
            const int n_tile = s.tile / p.m_tiles;
            const int m0 = (s.tile % p.m_tiles) * NT;
            const int n = n_tile * BN + row;
            const bool n_ok = n < p.N;
            const float sc = n_ok ? __ldg(p.scale + n) : 0.f;
            const bool whole = (s.k0 == 0 && s.k1 == p.kb);
            const int mval = min(NT, p.M - m0);  // valid token columns of this tile
            const uint32_t d_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * C::ACC_COLS;
            float *part = nullptr;
            if (CLUSTER) part = reinterpret_cast<float *>(smem);  // this CTA's partial, in the drained stages
            else if (!whole) part = p.partials + static_cast<size_t>(partial_slot(p, blockIdx.x, s.tile)) * (NT * BN);
#pragma unroll 1
            for (int c0 = 0; c0 < NT; c0 += 32) {
                if (c0 >= mval) break;
                int32_t dv[S][32];
#pragma unroll
                for (int pl = 0; pl < S; ++pl) {
                    uint32_t v[32];
                    ptx::tmem_ld_32x32b_x32(d_lane + pl * NT + c0, v);
                    ptx::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) dv[pl][j] = static_cast<int32_t>(v[j]);
#pragma unroll
                    for (int a = 1; a < C::NACC; ++a) {  // exact integer sum of the accumulators
                        ptx::tmem_ld_32x32b_x32(d_lane + a * C::NMMA + pl * NT + c0, v);
                        ptx::tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 32; ++j) dv[pl][j] += static_cast<int32_t>(v[j]);
                    }
                }
                // r[m] of the chunk's tokens, one per lane, shuffled to every lane below
                const float rs_lane = (c0 + lane < mval) ? __ldg(p.row_scale + m0 + c0 + lane) : 0.f;
                if (CLUSTER) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        int32_t d[S];
#pragma unroll
                        for (int pl = 0; pl < S; ++pl) d[pl] = dv[pl][j];
                        part[(c0 + j) * BN + row] = combine_planes<S>(d);
                    }
                } else if (whole && SILU) {
                    // gate lanes ((lane & 8) == 0) take the up value of their row from lane + 8
                    const int col = (n >> 4) * 8 + (n & 7);
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        int32_t d[S];
#pragma unroll
                        for (int pl = 0; pl < S; ++pl) d[pl] = dv[pl][j];
                        const float rs = __shfl_sync(0xffffffffu, rs_lane, j);
                        const float a = combine_planes<S>(d) * (sc * rs);
                        const float u = __shfl_xor_sync(0xffffffffu, a, 8);
                        if (!(lane & 8) && n_ok && c0 + j < mval)
                            p.y[static_cast<int64_t>(m0 + c0 + j) * p.ldy + col] = out_bits(p, silu_fast(a) * u);
                    }
                } else if (whole) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        int32_t d[S];
#pragma unroll
                        for (int pl = 0; pl < S; ++pl) d[pl] = dv[pl][j];
                        const float rs = __shfl_sync(0xffffffffu, rs_lane, j);
                        if (n_ok && c0 + j < mval) {
                            float o = combine_planes<S>(d) * (sc * rs);
                            if (p.res) o += res_value(p, static_cast<int64_t>(m0 + c0 + j) * p.ldr + n);
                            p.y[static_cast<int64_t>(m0 + c0 + j) * p.ldy + n] = out_bits(p, o);
                        }
                    }
                } else {
                    // partial tile layout [token j][row]: one 128-byte line per warp per j
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        int32_t d[S];
#pragma unroll
                        for (int pl = 0; pl < S; ++pl) d[pl] = dv[pl][j];
                        if (c0 + j < mval) part[(c0 + j) * BN + row] = combine_planes<S>(d);
                    }
                }
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&d_empty[buf]));
            ++dpos;
            if (!CLUSTER && !whole) {
                // Publish this segment's partial, then count arrivals on the tile.
                const long long ts = s.tile - p.dp_tiles;
                const int c_first = sk_owner(p, ts * p.kb);
                const int c_last = sk_owner(p, (ts + 1) * p.kb - 1);
                __threadfence();
                ptx::bar_sync(EPI_BAR, NUM_EPI_WARPS * 32);
                if (threadIdx.x == WARP_EPI0 * 32) {
                    const int old = atomicAdd(p.counters + ts, 1);
                    if (old == c_last - c_first) {
                        // every segment has arrived: re-arm the counter and leave the tile to the
                        // CTA-wide reduction after the role loops
                        p.counters[ts] = 0;
                        const int k = pending[0];
                        pending[1 + 3 * k] = s.tile;
                        pending[2 + 3 * k] = c_first;
                        pending[3 + 3 * k] = c_last;
                        pending[0] = k + 1;
                    }
                }
            }
        }
    }

    // ---------------- teardown ----------------
    // In warps 0-2 only lane 0 ran a role loop (or none); every role is done (the epilogue has
    // read TMEM and recorded its pending reductions) once all 8 warps have arrived.
    ptx::tc_fence_before();
    ptx::cta_sync_roles(ptx::smem_u32(td_bar));

    // ---------------- cluster reduction (all 256 threads of every CTA) ----------------
    if constexpr (CLUSTER) {
        const int c = p.cluster;
        const uint32_t rank = ptx::cluster_ctarank();
        const int tile = blockIdx.x / c;
        const int n_tile = tile / p.m_tiles;
        const int m0 = (tile % p.m_tiles) * NT;
        const int mval = min(NT, p.M - m0);
        const int j0 = NT * static_cast<int>(rank) / c, j1 = NT * (static_cast<int>(rank) + 1) / c;
        // s[n] of this lane's row quad (and, for SILU, of the up quad 8 rows on), loaded before
        // the barrier
        const int nq = n_tile * BN + lane * 4;
        float4 s4, s4u = make_float4(0.f, 0.f, 0.f, 0.f);
        s4.x = nq < p.N ? __ldg(p.scale + nq) : 0.f;
        s4.y = nq + 1 < p.N ? __ldg(p.scale + nq + 1) : 0.f;
        s4.z = nq + 2 < p.N ? __ldg(p.scale + nq + 2) : 0.f;
        s4.w = nq + 3 < p.N ? __ldg(p.scale + nq + 3) : 0.f;
        if constexpr (SILU) {
            s4u.x = nq + 8 < p.N ? __ldg(p.scale + nq + 8) : 0.f;
            s4u.y = nq + 9 < p.N ? __ldg(p.scale + nq + 9) : 0.f;
            s4u.z = nq + 10 < p.N ? __ldg(p.scale + nq + 10) : 0.f;
            s4u.w = nq + 11 < p.N ? __ldg(p.scale + nq + 11) : 0.f;
        }
        ptx::cluster_sync();  // every CTA's partial is in its shared memory
        if (!*abort_flag) {
            const uint32_t mine = ptx::smem_u32(smem) + (lane * 4) * 4;  // quad `lane` of token 0
            // One token per warp and lane = row quad; two tokens per round, every partial of a
            // round loaded (distributed shared memory) before any is added, in rank order
            // (deterministic).
            constexpr int WARPS = NUM_THREADS / 32;
#pragma unroll 1
            for (int j = j0 + warp; j < j1; j += 2 * WARPS) {
                float4 v[2][tci8::kMaxCluster];
                float rs[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int jj = j + h * WARPS;
                    const bool ok = jj < j1 && jj < mval;
                    rs[h] = ok ? __ldg(p.row_scale + m0 + jj) : 0.f;
#pragma unroll
                    for (int q = 0; q < tci8::kMaxCluster; ++q)
                        v[h][q] = (ok && q < c) ? ptx::ld_shared_cluster_v4(ptx::map_shared_rank(mine + jj * BN * 4, q))
                                                : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int jj = j + h * WARPS;
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int q = 0; q < tci8::kMaxCluster; ++q) {
                        acc.x += v[h][q].x;
                        acc.y += v[h][q].y;
                        acc.z += v[h][q].z;
                        acc.w += v[h][q].w;
                    }
                    if (jj < j1) finish_quad_scaled<SILU>(p, acc, s4, s4u, rs[h], jj, lane * 4, n_tile, m0, mval);
                }
            }
        }
        ptx::cluster_sync();  // no CTA leaves while its partial may still be read
    }

    // ---------------- stream-K reductions (all 256 threads) ----------------
    // A tile whose last segment arrived here: sum every segment's partial in segment order
    // (deterministic), apply s[n] * r[m], store y.  Item (token j, rows rq..rq+3):
    // consecutive threads take consecutive row quads, so a warp reads 512 contiguous bytes of
    // each partial; each thread keeps IPT items x SB segments of loads in flight per round.
    if (!*abort_flag && pending[0] > 0) {
        __threadfence();
        constexpr int QUADS = BN / 4;
        constexpr int IPT = (NT * QUADS + NUM_THREADS - 1) / NUM_THREADS;  // items per thread
        constexpr int SB = IPT >= 16 ? 1 : 16 / IPT;                        // segments per round
        const int npend = pending[0];
        for (int pi = 0; pi < npend; ++pi) {
            const int tile = pending[1 + 3 * pi], c_first = pending[2 + 3 * pi], c_last = pending[3 + 3 * pi];
            const int n_tile = tile / p.m_tiles;
            const int m0 = (tile % p.m_tiles) * NT;
            const int mval = min(NT, p.M - m0);
            // every CTA after the first starts inside this tile (its slot 2c); only the first
            // may have started earlier (slot 2c + 1)
            const int first_off = partial_slot(p, c_first, tile) - 2 * c_first;
            float4 acc[IPT];
#pragma unroll
            for (int i = 0; i < IPT; ++i) acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int cb = c_first; cb <= c_last; cb += SB) {
                float4 v[IPT][SB];
#pragma unroll
                for (int i = 0; i < IPT; ++i) {
                    const int item = threadIdx.x + i * NUM_THREADS;
                    const int j = item / QUADS, rq = (item % QUADS) * 4;
#pragma unroll
                    for (int u = 0; u < SB; ++u) {
                        v[i][u] = make_float4(0.f, 0.f, 0.f, 0.f);
                        if (j < mval && cb + u <= c_last)
                            v[i][u] = __ldcg(reinterpret_cast<const float4 *>(
                                p.partials + static_cast<size_t>(2 * (cb + u) + (cb + u == c_first ? first_off : 0)) * (NT * BN) +
                                j * BN + rq));
                    }
                }
#pragma unroll
                for (int i = 0; i < IPT; ++i)
#pragma unroll
                    for (int u = 0; u < SB; ++u) {
                        acc[i].x += v[i][u].x;
                        acc[i].y += v[i][u].y;
                        acc[i].z += v[i][u].z;
                        acc[i].w += v[i][u].w;
                    }
            }
            static_assert(QUADS == 32 && NUM_THREADS % 32 == 0, "a warp holds the 32 quads of one token");
#pragma unroll
            for (int i = 0; i < IPT; ++i) {
                const int item = threadIdx.x + i * NUM_THREADS;
                finish_quad<SILU>(p, acc[i], item / QUADS, (item % QUADS) * 4, n_tile, m0, mval);
            }
        }
    }

    if (warp == WARP_MMA) {
        __syncwarp();
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

}  // namespace tci8
}  // namespace lse
