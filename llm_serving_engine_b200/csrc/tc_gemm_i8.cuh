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
//     warps read it with tcgen05.ld, apply s[n] (and add the optional residual) and store
//     bf16 y.
//   * SILU = true is the MLP's gate_up projection with SiLU * mul fused: the weight rows
//     interleave 8-row blocks of gate and up (row block b = gate rows 8b..8b+7, then the
//     matching up rows, `scale` interleaved the same way), so a 16-row block's gate row sits
//     8 TMEM lanes (8 lanes of the same warp) from its up row; y is [M, N / 2] with
//     y[m, 8b + r] = silu(s_g * gate) * (s_u * up) (fp32, one bf16 rounding).
//
// Warp roles (512 threads): warp 0 TMA producer, warp 1 TMEM allocator + single-thread MMA
// issuer, warp 2 L2 prefetcher for the weight stream, warps 4-7 epilogue (TMEM lane quarter = warp % 4), warps 8-15 converters (two
// groups of four, one warp per lane quarter; the groups take alternate stages).
//
// Work distribution: tiles are (128 weight rows) x (NT tokens), tile = n_tile * m_tiles +
// m_tile.  Full waves of tiles are dealt round-robin to a persistent grid of G CTAs
// (data-parallel part); the remaining tiles are cut into 128-K units spread evenly over the
// G CTAs (stream-K part).  A tile whose K range is split across CTAs is finished by
// whichever CTA arrives last on the tile's counter: every segment writes its fp32 partial
// to the workspace and bumps the counter; the last one re-zeroes the counter and, once its
// role loops are done, sums all partials in segment order (deterministic) with all 512
// threads and every segment's loads in flight together, applies the scale and stores y.
// No CTA ever waits for another CTA.
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
constexpr int WARP_TMA = 0, WARP_MMA = 1, WARP_PREFETCH = 2, WARP_EPI0 = 4, WARP_CONV0 = 8;
// A throttle wait of the L2 prefetcher that exceeds this gives up prefetching (~20 us).
constexpr long long kPrefetchWaitCycles = 40000;
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
    // Independent accumulators per buffer: consecutive K16 MMAs of a stage go to different
    // accumulators, so small-N MMAs do not wait on each other's read-modify-write of one
    // TMEM tile; the epilogue sums them.
    static constexpr int NACC = NT <= 32 ? 4 : (NT <= 64 ? 2 : 1);
    static constexpr int ACC_COLS = NACC * NT;   // TMEM columns of one accumulator buffer
    static constexpr int STAGES = NT <= 32 ? 8 : (NT <= 64 ? 6 : 4);
    static constexpr int D_COL0 = 0;
    static constexpr int A_COL0 = ACC_BUFS * ACC_COLS;
    static_assert(A_COL0 + ASLOTS * A_SLOT_COLS <= TMEM_COLS, "TMEM budget");
    // barrier block after the stages: full, empty (STAGES each), a_full (ASLOTS),
    // d_full, d_empty (ACC_BUFS), drain; then tmem address, abort flag and the pending
    // stream-K reductions (count + 2 x {tile, first CTA, last CTA}).
    static constexpr int NUM_BARS = 2 * STAGES + ASLOTS + 2 * ACC_BUFS + 1;
    static constexpr int CTRL_BYTES = NUM_BARS * 8 + 48;
    static constexpr int SMEM_BYTES = 1024 /*alignment slack*/ + STAGES * STAGE_BYTES + CTRL_BYTES;
    static constexpr uint32_t IDESC = ptx::idesc_bf16_f32(BN, NT);
};

struct Params {
    int M, N, K;
    __nv_bfloat16 *y;
    int64_t ldy;
    const __nv_bfloat16 *res;  // null, or the residual added before rounding (may alias y)
    int64_t ldr;
    const float *scale;
    float *partials;   // [2 * grid][NT][BN] fp32 partial tiles
    int *counters;     // [stream-K tiles] arrival counters, zero between launches
    int m_tiles, tiles, kb, dp_tiles, grid;
    long long sk_units;
    int w_packed;      // 1: weights in the tile-contiguous packed layout (see pack_w.cuh)
    const int8_t *w;   // packed weights (read with 1-D bulk copies, no tensor map)
    int pf_stages;     // L2 prefetch distance in stages beyond the shared-memory ring
};

// Weight tile (n0 / BN, kb) -> shared memory, one TMA copy either way.
//   Packed W (pack_w.cuh): the tile is 8 row-block runs of 2 KB, stride 16*Kp bytes; the
//   tensor map views the buffer as [Np/16 rows][2*Kp 8-byte elements] and the box is
//   256 x 8, landing as [row block j][2 KB] in shared memory.
//   Row-major W [N, K]: a box of 128 rows x 128 bytes at (kb * BK, n0), 128-byte swizzled.
__device__ __forceinline__ void load_w_tile(const Params &p, const CUtensorMap *tmap_w, uint32_t dst, int n0,
                                            int kb, uint32_t bar, uint64_t pol) {
    if (p.w_packed) ptx::tma_load_2d(dst, tmap_w, bar, kb * (BK * 16 / 8), n0 / 16, pol);
    else ptx::tma_load_2d(dst, tmap_w, bar, kb * BK, n0, pol);
}
// One warp pulls weight tile (n0 / BN, kb) into L2 ahead of its TMA copy: 128 lines of
// 128 bytes, 4 per lane.
__device__ __forceinline__ void prefetch_w_tile_l2(const Params &p, int n0, int kb, int lane) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int line = i * 32 + lane;
        if (p.w_packed) {
            const int j = line >> 4;  // row block within the tile
            const int64_t run = (static_cast<int64_t>(n0 / 16 + j) * (p.kb * 4) + kb * 4) * 512;
            ptx::prefetch_line_l2(p.w + run + (line & 15) * 128);
        } else {
            const int r = n0 + line;
            if (r < p.N) ptx::prefetch_line_l2(p.w + static_cast<int64_t>(r) * p.K + kb * BK);
        }
    }
}

// silu(a) = a / (1 + e^-a) with the fast exponential and division intrinsics: a few
// instructions instead of the full-precision sequences, which the SiLU epilogue and the
// stream-K reduction would otherwise spend most of their issue slots on.  Their relative
// error (a few ulp of fp32) is far below the one bf16 rounding of the result; for a below
// about -88 the exponential overflows and the quotient is -0, the limit of silu.
__device__ __forceinline__ float silu_fast(float a) { return __fdividef(a, 1.f + __expf(-a)); }

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

// Walks this CTA's (tile, k-block) stages in the order the pipeline consumes them; used
// by the producer to issue L2 prefetches a fixed distance ahead of the TMA loads.
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
    __device__ __forceinline__ void skip(const Params &p) {
        int a, b;
        next(p, a, b);
    }

};

// Weights are read exactly once when there is a single token tile (decode): stream them
// with evict-first so x and the partial tiles keep L2.  With several token tiles each weight
// tile is re-read once per token tile, so leave it at normal priority.
__device__ __forceinline__ uint64_t policy_w_for(const Params &p) {
    return p.m_tiles == 1 ? ptx::policy_evict_first() : ptx::policy_evict_normal();
}

// ---- the kernel -------------------------------------------------------------------------
template <int NT, bool SILU = false>
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
    uint64_t *d_full = a_full + ASLOTS;
    uint64_t *d_empty = d_full + C::ACC_BUFS;
    uint64_t *drain = d_empty + C::ACC_BUFS;
    volatile uint32_t *tmem_slot = reinterpret_cast<volatile uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(drain + 1) + 1;
    volatile int *pending = reinterpret_cast<volatile int *>(drain + 1) + 2;  // [0] count, then triples

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < C::STAGES; ++i) {
            ptx::mbar_init(ptx::smem_u32(&full[i]), 1);
            ptx::mbar_init(ptx::smem_u32(&empty[i]), 1 + NUM_CONV_WARPS / 2);
        }
        for (int i = 0; i < ASLOTS; ++i) {
            ptx::mbar_init(ptx::smem_u32(&a_full[i]), NUM_CONV_WARPS / 2);
        }
        for (int i = 0; i < C::ACC_BUFS; ++i) {
            ptx::mbar_init(ptx::smem_u32(&d_full[i]), 1);
            ptx::mbar_init(ptx::smem_u32(&d_empty[i]), NUM_EPI_WARPS);
        }
        ptx::mbar_init(ptx::smem_u32(drain), 1);
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
            // Weights never depend on the previous kernel: start the first stages' weight
            // copies before waiting for it (programmatic dependent launch), then add the
            // activations once the previous kernel's output is visible.
            long long pre = 0;
            {
                SegIter ip = it;
                Seg sp;
                while (pre < C::STAGES && ip.next(p, sp)) {
                    const int n0 = (sp.tile / p.m_tiles) * BN;
                    for (int kb = sp.k0; kb < sp.k1 && pre < C::STAGES; ++kb, ++pre) {
                        const uint32_t fb = ptx::smem_u32(&full[pre]);
                        ptx::mbar_arrive_expect_tx(fb, C::STAGE_BYTES);
                        load_w_tile(p, &tmap_w, ptx::smem_u32(w_smem + pre * W_STAGE_BYTES), n0, kb, fb, pol_w);
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
                        load_w_tile(p, &tmap_w, ptx::smem_u32(w_smem + st * W_STAGE_BYTES), n0, kb, fb, pol_w);
                    }
                    uint8_t *xs = x_smem + st * C::X_STAGE_BYTES;
                    ptx::tma_load_2d(ptx::smem_u32(xs), &tmap_x, fb, kb * BK, m0, pol_x);
                    ptx::tma_load_2d(ptx::smem_u32(xs + C::X_BOX_BYTES), &tmap_x, fb, kb * BK + 64, m0, pol_x);
                }
            }
            // Drain: every copy this CTA issued must land before shared memory is released
            // (stages prefetched but never reached still complete their weight bytes only if
            // their activations were issued too, so drain exactly the issued set).
            if (pos < pre) {
                // aborted before the loop reached every prefetched stage: issue their
                // activation copies so each prefetched barrier can complete, then drain
                for (long long q = pos; q < pre; ++q) {
                    uint8_t *xs = x_smem + q * C::X_STAGE_BYTES;
                    const uint32_t fb = ptx::smem_u32(&full[q]);
                    ptx::tma_load_2d(ptx::smem_u32(xs), &tmap_x, fb, 0, 0, pol_x);
                    ptx::tma_load_2d(ptx::smem_u32(xs + C::X_BOX_BYTES), &tmap_x, fb, 64, 0, pol_x);
                }
                pos = pre;
            }
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
                const uint32_t d_tmem = tmem_base + C::D_COL0 + buf * C::ACC_COLS;
                for (int kb = s.k0; kb < s.k1; ++kb, ++pos, ++apos) {
                    const int st = static_cast<int>(pos % C::STAGES);
                    const uint32_t ph = static_cast<uint32_t>((pos / C::STAGES) & 1);
                    const int as = static_cast<int>(apos % ASLOTS);
                    const uint32_t aph = static_cast<uint32_t>((apos / ASLOTS) & 1);
                    // The converters arrive on a_full only after they observed the stage's
                    // `full` barrier, so a_full also orders the x tile's arrival before the MMA.
                    (void)ph;
                    if (!ptx::mbar_wait(ptx::smem_u32(&a_full[as]), aph, abort_flag)) {
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    // Descriptors advance by constants inside a stage: B (x) by 32 bytes per
                    // K16 step within a 64-wide box, A (TMEM) by 8 columns.
                    const uint64_t b0 = ptx::smem_desc_sw128(ptx::smem_u32(x_smem + st * C::X_STAGE_BYTES));
                    const uint32_t a0 = tmem_base + C::A_COL0 + as * A_SLOT_COLS;
#pragma unroll
                    for (int j = 0; j < KSTEPS; ++j) {
                        const uint64_t b_desc = b0 + static_cast<uint64_t>(((j >> 2) * C::X_BOX_BYTES + (j & 3) * (UK * 2)) >> 4);
                        const int acc = j % C::NACC;
                        ptx::mma_bf16_ts(d_tmem + acc * NT, a0 + j * (UK / 2), b_desc, C::IDESC,
                                         (kb > s.k0 || j >= C::NACC) ? 1u : 0u);
                    }
                    // One commit per stage: it frees the shared-memory stage (producer) and, seen
                    // ASLOTS stages later, the stage's TMEM A slot (converters).
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
    } else if (warp >= WARP_CONV0) {
        // ---------------- converters: int8 smem -> bf16 TMEM (A operand) ----------------
        // Two groups of four warps (one warp per TMEM lane quarter each) take alternate
        // stages, so each group has two stage-times per stage; inside a stage the two 64-K
        // halves are converted back to back, the first half's tcgen05.st draining while the
        // second half is converted.
        const int q = warp & 3;                       // TMEM lane quarter this warp may access
        const int grp = (warp - WARP_CONV0) >> 2;     // stages with (pos & 1) == grp
        const int row = q * 32 + lane;                // weight row within the tile
        const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + C::A_COL0;
        long long pos = 0;
        bool ok = true;
        while (ok && it.next(p, s)) {
            for (int kb = s.k0; kb < s.k1; ++kb, ++pos) {
                if ((pos & 1) != grp) continue;
                const int st = static_cast<int>(pos % C::STAGES);
                const uint32_t ph = static_cast<uint32_t>((pos / C::STAGES) & 1);
                const int as = static_cast<int>(pos % ASLOTS);
                const uint32_t aph = static_cast<uint32_t>((pos / ASLOTS) & 1);
                // A slot `as` was last read by the MMAs of stage pos - ASLOTS; their completion is
                // the last arrival on that stage's `empty` barrier (its converters arrived when
                // they finished it).  That barrier's next phase needs this stage converted
                // first, so its parity cannot alias.
                (void)aph;
                bool w_ok = ptx::mbar_wait(ptx::smem_u32(&full[st]), ph, abort_flag);
                if (w_ok && pos >= ASLOTS) {
                    const long long pp = pos - ASLOTS;
                    w_ok = ptx::mbar_wait(ptx::smem_u32(&empty[pp % C::STAGES]),
                                          static_cast<uint32_t>((pp / C::STAGES) & 1), abort_flag);
                }
                if (!__all_sync(0xffffffffu, w_ok)) {
                    ok = false;
                    break;
                }
                ptx::tc_fence_after();
                const uint8_t *wst = w_smem + st * W_STAGE_BYTES;
                if (p.w_packed) {
                    // rows 32q..32q+31 = row blocks 2q, 2q+1; lane owns rows lane/4 (+8) of each
                    // and the K quad 4(lane%4) of every 16-column step (pack_w.cuh)
#pragma unroll
                    for (int jb = 0; jb < 2; ++jb) {
                        const uint8_t *src = wst + (2 * q + jb) * 2048 + lane * 16;
                        uint4 v[4];
#pragma unroll
                        for (int i = 0; i < 4; ++i) v[i] = *reinterpret_cast<const uint4 *>(src + i * 512);
                        uint32_t out[32];
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            u8x4_to_bf16x4(v[i].x, out[8 * i + 0], out[8 * i + 1]);  // step 2i, row r0
                            u8x4_to_bf16x4(v[i].y, out[8 * i + 2], out[8 * i + 3]);  // step 2i, row r0+8
                            u8x4_to_bf16x4(v[i].z, out[8 * i + 4], out[8 * i + 5]);  // step 2i+1, row r0
                            u8x4_to_bf16x4(v[i].w, out[8 * i + 6], out[8 * i + 7]);  // step 2i+1, row r0+8
                        }
                        ptx::tmem_st_16x256b_x8(lane_base + (static_cast<uint32_t>(16 * jb) << 16) + as * A_SLOT_COLS,
                                                out);
                    }
                } else {
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        uint4 v[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int c = h * 4 + j;  // 16-byte chunk (K16 step) within the row
                            v[j] = *reinterpret_cast<const uint4 *>(wst + row * BK + ((c ^ (row & 7)) << 4));
                        }
                        uint32_t out[32];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            i8x4_to_bf16x4(v[j].x, out[8 * j + 0], out[8 * j + 1]);
                            i8x4_to_bf16x4(v[j].y, out[8 * j + 2], out[8 * j + 3]);
                            i8x4_to_bf16x4(v[j].z, out[8 * j + 4], out[8 * j + 5]);
                            i8x4_to_bf16x4(v[j].w, out[8 * j + 6], out[8 * j + 7]);
                        }
                        ptx::tmem_st_32x32b_x32(lane_base + as * A_SLOT_COLS + h * (A_SLOT_COLS / 2), out);
                    }
                }
                ptx::tmem_wait_st();
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    ptx::mbar_arrive(ptx::smem_u32(&a_full[as]));
                    ptx::mbar_arrive(ptx::smem_u32(&empty[st]));
                }
            }
        }
    } else if (warp == WARP_PREFETCH) {
        // ---------------- L2 prefetcher ----------------
        // Keeps p.pf_stages weight tiles of this CTA in flight to L2 ahead of the bulk-copy
        // engine, through the load/store path: the engine's own request slots then only
        // cover L2 latency, not DRAM latency.  Throttled by the `full` barriers (it never
        // runs more than pf_stages stages past the data that has landed), and only a hint:
        // if a throttle wait runs long it stops prefetching, it never aborts the CTA.
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
                prefetch_w_tile_l2(p, n0, kbo, lane);
            }
        }
    } else if (warp >= WARP_EPI0 && warp < WARP_EPI0 + NUM_EPI_WARPS) {
        // ---------------- epilogue: TMEM -> scale -> bf16 y (or fp32 partial) ----------------
        ptx::grid_dep_wait();  // y, partials and counters may still be in use by the previous kernel
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
            const uint32_t d_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + C::D_COL0 + buf * C::ACC_COLS;
            float *part = nullptr;
            if (!whole) part = p.partials + static_cast<size_t>(partial_slot(p, blockIdx.x, s.tile)) * (NT * BN);
            constexpr int CH = NT < 32 ? NT : 32;
#pragma unroll 1
            for (int c0 = 0; c0 < NT; c0 += CH) {
                if (c0 >= mval) break;
                uint32_t v[32];
                if constexpr (CH == 32) ptx::tmem_ld_32x32b_x32(d_lane + c0, v);
                else ptx::tmem_ld_32x32b_x16(d_lane + c0, v);
                ptx::tmem_wait_ld();
#pragma unroll
                for (int a = 1; a < C::NACC; ++a) {  // fold the other accumulators in, fixed order
                    uint32_t u[32];
                    if constexpr (CH == 32) ptx::tmem_ld_32x32b_x32(d_lane + a * NT + c0, u);
                    else ptx::tmem_ld_32x32b_x16(d_lane + a * NT + c0, u);
                    ptx::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < CH; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(u[j]));
                }
                if (whole && SILU) {
                    // gate lanes ((lane & 8) == 0) take the up value of their row from lane + 8
                    const int col = (n >> 4) * 8 + (n & 7);
#pragma unroll
                    for (int j = 0; j < CH; ++j) {
                        const float a = __uint_as_float(v[j]) * sc;
                        const float u = __shfl_xor_sync(0xffffffffu, a, 8);
                        if (!(lane & 8) && n_ok && c0 + j < mval)
                            p.y[static_cast<int64_t>(m0 + c0 + j) * p.ldy + col] = __float2bfloat16_rn(silu_fast(a) * u);
                    }
                } else if (whole) {
#pragma unroll
                    for (int j = 0; j < CH; ++j) {
                        if (n_ok && c0 + j < mval) {
                            float o = __uint_as_float(v[j]) * sc;
                            if (p.res) o += __bfloat162float(p.res[static_cast<int64_t>(m0 + c0 + j) * p.ldr + n]);
                            p.y[static_cast<int64_t>(m0 + c0 + j) * p.ldy + n] = __float2bfloat16_rn(o);
                        }
                    }
                } else {
                    // partial tile layout [token j][row]: one 128-byte line per warp per j
#pragma unroll
                    for (int j = 0; j < CH; ++j)
                        if (c0 + j < mval) part[(c0 + j) * BN + row] = __uint_as_float(v[j]);
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
                    if (old == c_last - c_first) {
                        // every segment has arrived: re-arm the counter for the next launch and
                        // leave the tile to the CTA-wide reduction after the role loops
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
    // In warps 0 and 1 only lane 0 ran the role loop; the compiler may place each branch's
    // barrier separately, so the teardown barrier is the non-aligned form that counts every
    // thread, and it waits for the epilogue before TMEM is freed.
    __syncwarp();
    ptx::tc_fence_before();
    ptx::cta_sync_all();

    // ---------------- stream-K reductions (all 512 threads) ----------------
    // A tile whose last segment arrived here: sum every segment's partial in segment order
    // (deterministic), scale, store y.  Item (token j, rows rq..rq+3): consecutive threads
    // take consecutive row quads, so a warp reads 512 contiguous bytes of each partial; each
    // thread keeps IPT items x SB segments of loads in flight per round.
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
            // Partial slots of the segments: every CTA after the first starts inside this
            // tile, so it is that CTA's first tile (slot 2c); only the first CTA may have
            // started earlier (slot 2c + 1).  One division per tile instead of one per load.
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
#pragma unroll
            for (int i = 0; i < IPT; ++i) {
                const int item = threadIdx.x + i * NUM_THREADS;
                const int j = item / QUADS, rq = (item % QUADS) * 4;
                const int n = n_tile * BN + rq;
                if constexpr (SILU) {
                    // quad rq + 8 (the up rows of gate quad rq) is item + 2: lane + 2 of this warp
                    static_assert(QUADS == 32 && NUM_THREADS % 32 == 0, "quad exchange stays in the warp");
                    const float u4[4] = {__shfl_xor_sync(0xffffffffu, acc[i].x, 2), __shfl_xor_sync(0xffffffffu, acc[i].y, 2),
                                         __shfl_xor_sync(0xffffffffu, acc[i].z, 2), __shfl_xor_sync(0xffffffffu, acc[i].w, 2)};
                    if (j >= mval || (rq & 8)) continue;
                    const float g4[4] = {acc[i].x, acc[i].y, acc[i].z, acc[i].w};
                    __nv_bfloat16 *yr = p.y + static_cast<int64_t>(m0 + j) * p.ldy + (n >> 4) * 8 + (n & 7);
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        if (n + e < p.N) {
                            const float g = g4[e] * __ldg(p.scale + n + e), u = u4[e] * __ldg(p.scale + n + 8 + e);
                            yr[e] = __float2bfloat16_rn(silu_fast(g) * u);
                        }
                } else {
                    if (j >= mval) continue;
                    __nv_bfloat16 *yr = p.y + static_cast<int64_t>(m0 + j) * p.ldy + n;
                    const float a4[4] = {acc[i].x, acc[i].y, acc[i].z, acc[i].w};
#pragma unroll
                    for (int e = 0; e < 4; ++e)
                        if (n + e < p.N) {
                            float o = a4[e] * __ldg(p.scale + n + e);
                            if (p.res) o += __bfloat162float(p.res[static_cast<int64_t>(m0 + j) * p.ldr + n + e]);
                            yr[e] = __float2bfloat16_rn(o);
                        }
                }
            }
        }
    }

    if (warp == WARP_MMA) {
        __syncwarp();
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

}  // namespace tc
}  // namespace lse
