// tcgen05 / TMEM tensor-core kernel for the int8 weight-only linear (sm_100a).
//
//   y[m, n] = s[n] * sum_k x[m, k] * w[n, k]      (x bf16, w int8, fp32 accumulate, y bf16)
//
// Operand roles ("swap-AB"): the 128 weight rows of a tile are the MMA's A operand (M = 128)
// and the tokens are its N dimension, so one tcgen05.mma computes D[128 rows, NT tokens].
//
//   * W (int8) arrives by TMA into shared memory (128-byte swizzle, 128 rows x 128 K per
//     stage).  Eight converter warps widen it to bf16 in registers (exact: int8 values are
//     bf16-representable) and write it straight into tensor memory with tcgen05.st, where
//     tcgen05.mma reads A.  The bf16 copy never touches shared memory, which keeps the
//     shared-memory traffic per weight byte at TMA-write + one read instead of the four
//     passes an smem->smem dequant would need.
//   * x (bf16) arrives by TMA (128-byte swizzle, K-major) and is the B operand, read by the
//     MMA through a shared-memory descriptor.
//   * The fp32 accumulator lives in TMEM (double-buffered when it fits) and four epilogue
//     warps read it with tcgen05.ld, apply s[n] and store bf16 y.
//
// Warp roles (512 threads): warp 0 TMA producer, warp 1 TMEM allocator + single-thread MMA
// issuer, warps 4-7 epilogue (TMEM lane quarter = warp % 4), warps 8-15 converters (two
// warps per lane quarter, each widening half of a stage's K).
//
// Work distribution: tiles are (128 weight rows) x (NT tokens), tile = n_tile * m_tiles +
// m_tile.  Full waves of tiles are dealt round-robin to a persistent grid of G CTAs
// (data-parallel part); the remaining tiles are cut into 128-K units spread evenly over the
// G CTAs (stream-K part).  A tile whose K range is split across CTAs is finished by
// whichever CTA arrives last on the tile's counter: every segment writes its fp32 partial
// to the workspace, bumps the counter, and the last one sums all partials in segment order
// (deterministic), applies the scale, stores y and re-zeroes the counter.  No CTA ever
// waits for another CTA.
//
// Every mbarrier wait is bounded (tc_ptx.cuh: mbar_wait); on a timeout the CTA raises an
// abort flag, records LSE_ERR_DEVICE_TIMEOUT, drains its own copies and MMAs, frees TMEM
// and returns.
#pragma once

#include "tc_ptx.cuh"

namespace lse {
namespace tc {

constexpr int BN = 128;                   // weight rows per tile (MMA M)
constexpr int BK = 128;                   // K per pipeline stage
constexpr int UK = 16;                    // K per tcgen05.mma kind::f16
constexpr int KSTEPS = BK / UK;           // MMAs per stage
constexpr int W_STAGE_BYTES = BN * BK;    // int8 weight tile per stage
constexpr int A_SLOT_COLS = BK / 2;       // TMEM columns per A slot (2 bf16 per column)
constexpr int ASLOTS = 4;                 // A slots in TMEM
constexpr int NUM_THREADS = 512;
constexpr int WARP_TMA = 0, WARP_MMA = 1, WARP_EPI0 = 4, WARP_CONV0 = 8;
constexpr int NUM_EPI_WARPS = 4, NUM_CONV_WARPS = 8;
constexpr int EPI_BAR = 1;                // named barrier id used by the epilogue warps
constexpr int TMEM_COLS = 512;

template <int NT>
struct Cfg {
    static_assert(NT == 16 || NT == 32 || NT == 64 || NT == 128, "token tile");
    static constexpr int X_BOX_BYTES = NT * 128;   // one [NT rows x 64 bf16] TMA box
    static constexpr int X_STAGE_BYTES = 2 * X_BOX_BYTES;
    static constexpr int STAGE_BYTES = W_STAGE_BYTES + X_STAGE_BYTES;
    static constexpr int ACC_BUFS = 2;
    static constexpr int STAGES = NT <= 32 ? 8 : (NT <= 64 ? 6 : 4);
    static constexpr int D_COL0 = 0;
    static constexpr int A_COL0 = ACC_BUFS * NT;
    static_assert(A_COL0 + ASLOTS * A_SLOT_COLS <= TMEM_COLS, "TMEM budget");
    // barrier block after the stages: full, empty (STAGES each), a_full, a_empty (ASLOTS),
    // d_full, d_empty (ACC_BUFS), drain; then tmem address, abort flag, reduce flag.
    static constexpr int NUM_BARS = 2 * STAGES + 2 * ASLOTS + 2 * ACC_BUFS + 1;
    static constexpr int CTRL_BYTES = NUM_BARS * 8 + 16;
    static constexpr int SMEM_BYTES = 1024 /*alignment slack*/ + STAGES * STAGE_BYTES + CTRL_BYTES;
    static constexpr uint32_t IDESC = ptx::idesc_bf16_f32(BN, NT);
};

struct Params {
    int M, N, K;
    __nv_bfloat16 *y;
    int64_t ldy;
    const float *scale;
    float *partials;   // [2 * grid][NT][BN] fp32 partial tiles
    int *counters;     // [stream-K tiles] arrival counters, zero between launches
    int m_tiles, tiles, kb, dp_tiles, grid;
    long long sk_units;
};

// ---- schedule (identical in every role) -------------------------------------------------
__device__ __forceinline__ long long sk_begin(const Params &p, int c) {
    return p.sk_units * c / p.grid;
}
// Owner CTA of stream-K unit u: the largest c with sk_begin(c) <= u (grid <= sk_units, so
// every CTA owns at least one unit and owners of consecutive units are consecutive).
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

// Partial slot CTA c uses for stream-K tile `tile`: 2c for the first tile it touches, 2c+1
// for the last (a CTA's middle tiles are complete and need no slot).
__device__ __forceinline__ int partial_slot(const Params &p, int c, int tile) {
    const int first_tile = p.dp_tiles + static_cast<int>(sk_begin(p, c) / p.kb);
    return 2 * c + (tile == first_tile ? 0 : 1);
}

// Weights are read exactly once when there is a single token tile (decode): stream them
// with evict-first so x and the partial tiles keep L2.  With several token tiles each weight
// tile is re-read once per token tile, so leave it at normal priority.
__device__ __forceinline__ uint64_t policy_w_for(const Params &p) {
    return p.m_tiles == 1 ? ptx::policy_evict_first() : ptx::policy_evict_normal();
}

// ---- the kernel -------------------------------------------------------------------------
template <int NT>
__global__ void __launch_bounds__(NUM_THREADS, 1)
tc_gemm_i8_kernel(const __grid_constant__ CUtensorMap tmap_w,
                  const __grid_constant__ CUtensorMap tmap_x, const Params p) {
    using C = Cfg<NT>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~static_cast<uintptr_t>(1023));
    uint8_t *w_smem = smem;                                  // STAGES x 16 KB
    uint8_t *x_smem = smem + C::STAGES * W_STAGE_BYTES;      // STAGES x X_STAGE_BYTES
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C::STAGES * C::STAGE_BYTES);
    uint64_t *full = bars;
    uint64_t *empty = full + C::STAGES;
    uint64_t *a_full = empty + C::STAGES;
    uint64_t *a_empty = a_full + ASLOTS;
    uint64_t *d_full = a_empty + ASLOTS;
    uint64_t *d_empty = d_full + C::ACC_BUFS;
    uint64_t *drain = d_empty + C::ACC_BUFS;
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(drain + 1) + 1;
    volatile int *reduce_flag = reinterpret_cast<volatile int *>(drain + 1) + 2;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < C::STAGES; ++i) {
            ptx::mbar_init(ptx::smem_u32(&full[i]), 1);
            ptx::mbar_init(ptx::smem_u32(&empty[i]), 1 + NUM_CONV_WARPS);
        }
        for (int i = 0; i < ASLOTS; ++i) {
            ptx::mbar_init(ptx::smem_u32(&a_full[i]), NUM_CONV_WARPS);
            ptx::mbar_init(ptx::smem_u32(&a_empty[i]), 1);
        }
        for (int i = 0; i < C::ACC_BUFS; ++i) {
            ptx::mbar_init(ptx::smem_u32(&d_full[i]), 1);
            ptx::mbar_init(ptx::smem_u32(&d_empty[i]), NUM_EPI_WARPS);
        }
        ptx::mbar_init(ptx::smem_u32(drain), 1);
        *abort_flag = 0;
        *reduce_flag = 0;
        ptx::fence_mbar_init();
        ptx::prefetch_tmap(&tmap_w);
        ptx::prefetch_tmap(&tmap_x);
    }
    if (warp == WARP_MMA) {
        ptx::tmem_alloc(ptx::smem_u32(const_cast<uint32_t *>(tmem_slot)), TMEM_COLS);
        ptx::tmem_relinquish();
    }
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    SegIter it;
    it.init(p, blockIdx.x);
    Seg s;

    if (warp == WARP_TMA) {
        // ---------------- TMA producer ----------------
        if (lane == 0) {
            const uint64_t pol_w = policy_w_for(p);
            const uint64_t pol_x = ptx::policy_evict_last();
            long long pos = 0;  // stages issued so far
            bool ok = true;
            while (ok && it.next(p, s)) {
                const int n0 = (s.tile / p.m_tiles) * BN;
                const int m0 = (s.tile % p.m_tiles) * NT;
                for (int kb = s.k0; kb < s.k1; ++kb, ++pos) {
                    const int st = static_cast<int>(pos % C::STAGES);
                    const uint32_t ph = static_cast<uint32_t>((pos / C::STAGES) & 1);
                    if (!ptx::mbar_wait(ptx::smem_u32(&empty[st]), ph ^ 1, abort_flag)) {
                        ok = false;
                        break;
                    }
                    const uint32_t fb = ptx::smem_u32(&full[st]);
                    ptx::mbar_arrive_expect_tx(fb, C::STAGE_BYTES);
                    ptx::tma_load_2d(ptx::smem_u32(w_smem + st * W_STAGE_BYTES), &tmap_w, fb, kb * BK, n0,
                                     pol_w);
                    uint8_t *xs = x_smem + st * C::X_STAGE_BYTES;
                    ptx::tma_load_2d(ptx::smem_u32(xs), &tmap_x, fb, kb * BK, m0, pol_x);
                    ptx::tma_load_2d(ptx::smem_u32(xs + C::X_BOX_BYTES), &tmap_x, fb, kb * BK + 64, m0, pol_x);
                }
            }
            // Drain: every copy this CTA issued must land before shared memory is released.
            const long long first = pos > C::STAGES ? pos - C::STAGES : 0;
            for (long long q = first; q < pos; ++q)
                ptx::mbar_drain(ptx::smem_u32(&full[q % C::STAGES]), static_cast<uint32_t>((q / C::STAGES) & 1));
        }
    } else if (warp == WARP_MMA) {
        // ---------------- MMA issuer (one thread) ----------------
        if (lane == 0) {
            long long pos = 0, apos = 0, dpos = 0;
            bool ok = true;
            while (ok && it.next(p, s)) {
                const int buf = static_cast<int>(dpos % C::ACC_BUFS);
                const uint32_t dph = static_cast<uint32_t>((dpos / C::ACC_BUFS) & 1);
                if (!ptx::mbar_wait(ptx::smem_u32(&d_empty[buf]), dph ^ 1, abort_flag)) break;
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem_base + C::D_COL0 + buf * NT;
                for (int kb = s.k0; kb < s.k1; ++kb, ++pos, ++apos) {
                    const int st = static_cast<int>(pos % C::STAGES);
                    const uint32_t ph = static_cast<uint32_t>((pos / C::STAGES) & 1);
                    const int as = static_cast<int>(apos % ASLOTS);
                    const uint32_t aph = static_cast<uint32_t>((apos / ASLOTS) & 1);
                    if (!ptx::mbar_wait(ptx::smem_u32(&full[st]), ph, abort_flag) ||
                        !ptx::mbar_wait(ptx::smem_u32(&a_full[as]), aph, abort_flag)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const uint32_t xs = ptx::smem_u32(x_smem + st * C::X_STAGE_BYTES);
#pragma unroll
                    for (int j = 0; j < KSTEPS; ++j) {
                        const uint32_t a_tmem = tmem_base + C::A_COL0 + as * A_SLOT_COLS + j * (UK / 2);
                        const uint64_t b_desc =
                            ptx::smem_desc_sw128(xs + (j >> 2) * C::X_BOX_BYTES + (j & 3) * (UK * 2));
                        ptx::mma_bf16_ts(d_tmem, a_tmem, b_desc, C::IDESC, (kb > s.k0 || j > 0) ? 1u : 0u);
                    }
                    ptx::mma_commit(ptx::smem_u32(&empty[st]));
                    ptx::mma_commit(ptx::smem_u32(&a_empty[as]));
                }
                if (!ok) break;
                ptx::mma_commit(ptx::smem_u32(&d_full[buf]));
                ++dpos;
            }
            // Drain: all MMAs this thread issued must finish before TMEM is freed.
            ptx::mma_commit(ptx::smem_u32(drain));
            ptx::mbar_drain(ptx::smem_u32(drain), 0);
        }
    } else if (warp >= WARP_CONV0) {
        // ---------------- converters: int8 smem -> bf16 TMEM (A operand) ----------------
        const int q = warp & 3;                 // TMEM lane quarter this warp may access
        const int half = (warp - WARP_CONV0) >> 2;  // which 64-K half of the stage
        const int row = q * 32 + lane;          // weight row within the tile
        long long pos = 0, apos = 0;
        bool ok = true;
        while (ok && it.next(p, s)) {
            for (int kb = s.k0; kb < s.k1; ++kb, ++pos, ++apos) {
                const int st = static_cast<int>(pos % C::STAGES);
                const uint32_t ph = static_cast<uint32_t>((pos / C::STAGES) & 1);
                const int as = static_cast<int>(apos % ASLOTS);
                const uint32_t aph = static_cast<uint32_t>((apos / ASLOTS) & 1);
                bool w_ok = ptx::mbar_wait(ptx::smem_u32(&full[st]), ph, abort_flag) &&
                            ptx::mbar_wait(ptx::smem_u32(&a_empty[as]), aph ^ 1, abort_flag);
                if (!__all_sync(0xffffffffu, w_ok)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint8_t *wrow = w_smem + st * W_STAGE_BYTES + row * BK;
                uint32_t out[32];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int c = half * 4 + j;  // 16-byte chunk (K16 step) within the row
                    const uint4 v = *reinterpret_cast<const uint4 *>(wrow + ((c ^ (row & 7)) << 4));
                    i8x4_to_bf16x4(v.x, out[8 * j + 0], out[8 * j + 1]);
                    i8x4_to_bf16x4(v.y, out[8 * j + 2], out[8 * j + 3]);
                    i8x4_to_bf16x4(v.z, out[8 * j + 4], out[8 * j + 5]);
                    i8x4_to_bf16x4(v.w, out[8 * j + 6], out[8 * j + 7]);
                }
                const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + C::A_COL0 +
                                       as * A_SLOT_COLS + half * (A_SLOT_COLS / 2);
                ptx::tmem_st_32x32b_x32(taddr, out);
                ptx::tmem_wait_st();
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    ptx::mbar_arrive(ptx::smem_u32(&a_full[as]));
                    ptx::mbar_arrive(ptx::smem_u32(&empty[st]));
                }
            }
        }
    } else if (warp >= WARP_EPI0 && warp < WARP_EPI0 + NUM_EPI_WARPS) {
        // ---------------- epilogue: TMEM -> scale -> bf16 y (or fp32 partial) ----------------
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
            const uint32_t d_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + C::D_COL0 + buf * NT;
            float *part = nullptr;
            if (!whole) part = p.partials + static_cast<size_t>(partial_slot(p, blockIdx.x, s.tile)) * (NT * BN);
            constexpr int CH = NT < 32 ? NT : 32;
#pragma unroll 1
            for (int c0 = 0; c0 < NT; c0 += CH) {
                uint32_t v[32];
                if constexpr (CH == 32) ptx::tmem_ld_32x32b_x32(d_lane + c0, v);
                else ptx::tmem_ld_32x32b_x16(d_lane + c0, v);
                ptx::tmem_wait_ld();
                if (whole) {
#pragma unroll
                    for (int j = 0; j < CH; ++j) {
                        const int m = m0 + c0 + j;
                        if (n_ok && m < p.M)
                            p.y[static_cast<int64_t>(m) * p.ldy + n] = __float2bfloat16_rn(__uint_as_float(v[j]) * sc);
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < CH; ++j) part[(c0 + j) * BN + row] = __uint_as_float(v[j]);
                }
            }
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(ptx::smem_u32(&d_empty[buf]));
            ++dpos;
            if (!whole) {
                // Publish this segment's partial, then count arrivals on the tile.
                const long long ts = s.tile - p.dp_tiles;
                const int c_first = sk_owner(p, ts * p.kb);
                const int c_last = sk_owner(p, (ts + 1) * p.kb - 1);
                __threadfence();
                ptx::bar_sync(EPI_BAR, NUM_EPI_WARPS * 32);
                if (threadIdx.x == WARP_EPI0 * 32) {
                    const int old = atomicAdd(p.counters + ts, 1);
                    const int last = (old == c_last - c_first);
                    if (last) p.counters[ts] = 0;  // every segment has arrived: re-arm for next launch
                    *reduce_flag = last;
                }
                ptx::bar_sync(EPI_BAR, NUM_EPI_WARPS * 32);
                const bool last = *reduce_flag != 0;
                ptx::bar_sync(EPI_BAR, NUM_EPI_WARPS * 32);  // flag read by all before reuse
                if (last) {
                    __threadfence();
#pragma unroll 1
                    for (int j = 0; j < NT; ++j) {
                        const int m = m0 + j;
                        if (m >= p.M) break;
                        float acc = 0.f;
                        for (int c = c_first; c <= c_last; ++c) {
                            const float *pc = p.partials + static_cast<size_t>(partial_slot(p, c, s.tile)) * (NT * BN);
                            acc += __ldcg(pc + j * BN + row);
                        }
                        if (n_ok) p.y[static_cast<int64_t>(m) * p.ldy + n] = __float2bfloat16_rn(acc * sc);
                    }
                }
            }
        }
    }

    // ---------------- teardown ----------------
    ptx::tc_fence_before();
    __syncthreads();
    if (warp == WARP_MMA) {
        __syncwarp();
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

}  // namespace tc
}  // namespace lse
