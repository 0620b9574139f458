// Paged decode attention (one query token per sequence) for sm_100a.
//
//   o[e, h, :] = softmax(q[e, h, :] . K[e, 0:ctx, kvh(h), :]^T * scale) V[e, 0:ctx, kvh(h), :]
//
// with K/V in the reference engine's shared per-layer pool [num_blocks, block_size, H_KV, D]
// (bf16 or fp16, contiguous) and key position p of sequence e in pool block block_table[e, p /
// block_size], slot p % block_size.  Grouped-query attention: the G = H / H_KV query heads
// of one KV head share every K/V row read.
//
// Decode attention is a stream over the K/V of every sequence (512 bytes per position and
// KV head at D = 128), so the kernel is shaped for HBM:
//   * grid (splits, H_KV, sequences): each CTA streams a contiguous range of positions of
//     one (sequence, KV head) and serves its G query heads; each of four warps takes
//     interleaved iterations of 16 positions;
//   * a warp keeps STAGES iterations of K/V rows in flight with cp.async into its own
//     shared-memory ring (no CTA barrier in the loop), and works on the tensor cores: the
//     scores S = Q K^T are warp MMAs with the query heads as rows, the online softmax runs
//     on the S accumulators, which are then the row operand of O += P V (V transposed by
//     ldmatrix.trans);
//   * the four warps' (max, sum, acc) merge in shared memory; positions are split over
//     several CTAs only for small batches (the host plan), in which case each CTA writes its
//     partial to the workspace and the CTA that arrives last on the (sequence, KV head)
//     counter merges them in split order and writes o (deterministic; it re-arms the
//     counter).  No CTA waits for another.
// A block id outside [0, num_blocks) makes that position masked (never read) and records
// LSE_ERR_INVALID_ARG in the device status word.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>
#include <type_traits>

#include "common.cuh"

namespace lse {
namespace attn {

constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;
constexpr int MAX_TABLE = 1024;  // block-table entries one CTA stages (chunk / block_size + 1)
constexpr int STAGES = 3;        // cp.async iterations in flight per warp
constexpr int MAX_SPLITS = 64;   // position splits per (sequence, KV head) the merge stages

// Dynamic shared memory of one CTA: per warp STAGES x (16 K rows + 16 V rows) of D 16-bit elements.
template <int D>
constexpr int attn_smem_bytes() { return WARPS * STAGES * 2 * 16 * D * 2; }

// q, the pools and o hold bf16 or fp16 elements (the kernel's T).
struct Params {
    const void *q;            // [E, H, D], d contiguous
    int64_t q_stride_e, q_stride_h;
    const void *k_pool, *v_pool;  // [num_blocks, block_size, H_KV, D] contiguous
    const int *block_table;   // [E, >= ceil(ctx / block_size)]
    int64_t bt_stride;
    const int *context_len;   // [E]
    void *o;                  // [E, H, D], d contiguous
    int64_t o_stride_e, o_stride_h;
    int E, H_kv, block_size, num_blocks, chunk, splits, max_ctx;
    float scale_log2;         // softmax scale * log2(e)
    float *part;              // splits > 1: fp32 partials, [E, H_kv, splits, G, D] accumulators
                              // then [E, H_kv, splits, G, 2] (max, sum)
    int *counters;            // [E * H_kv] arrival counters, zero between launches
};

__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void *src, bool valid) {
    // 16 bytes global -> shared; a masked row is zero-filled (source size 0), never read
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
// D (16x8 fp32) += A (16x16, row) * B (16x8, col), bf16 or fp16 operands (T)
template <typename T>
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    if constexpr (std::is_same_v<T, __half>)
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    else
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    if constexpr (std::is_same_v<T, __half>) {
        const __half2 v = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<const uint32_t *>(&v);
    } else {
        const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<const uint32_t *>(&v);
    }
}

// Per warp and iteration, 16 positions: K and V rows staged in shared memory by cp.async
// (STAGES iterations in flight), rows swizzled in 16-byte chunks (chunk c of row r at
// c ^ (r & 7)) so that ldmatrix reads them without bank conflicts.
//   S[head, key] = Q K^T: warp MMA m16n8k16 with the G query heads as rows (padded to 16,
//     zero), K from ldmatrix as the column operand, two 8-key tiles x D/16 K-steps;
//   online softmax on the S accumulators (base 2), whose two tiles are exactly the row
//     operand of P V;
//   O[head, dims] += P V: V from ldmatrix.trans as the column operand, D/8 dim tiles.
template <int D, int G, typename T = __nv_bfloat16>
__global__ void __launch_bounds__(THREADS) paged_decode_kernel(const Params p) {
    const T *q_ptr = static_cast<const T *>(p.q);
    const T *k_ptr = static_cast<const T *>(p.k_pool);
    const T *v_ptr = static_cast<const T *>(p.v_pool);
    T *o_ptr = static_cast<T *>(p.o);
    static_assert(D == 64 || D == 128, "head_dim");
    static_assert(G == 1 || G == 2 || G == 4 || G == 8, "query heads per KV head");
    constexpr int CH = D / 8;           // 16-byte chunks per row
    constexpr int ROWB = D * 2;         // bytes per staged row
    constexpr int KEYS = 16;            // positions per warp iteration
    constexpr int TILE_B = KEYS * ROWB; // one K (or V) tile
    constexpr int STAGE_B = 2 * TILE_B;
    constexpr int NT = D / 8;           // output dim tiles
    const int split = blockIdx.x, kvh = blockIdx.y, e = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = lane >> 2, q4 = lane & 3;
    const float NEG_INF = -__int_as_float(0x7f800000);
    extern __shared__ __align__(128) uint8_t dsmem[];  // [WARPS][STAGES][K tile, V tile]

    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // q and the pool come from earlier kernels

    // The context length, this CTA's slice of the block table (every entry of positions below
    // max_context, at most MAX_TABLE of them: independent of the context length, so both loads
    // are in flight together) and q (below) are read at once; block ids are range-checked where
    // they are used.  A split launch sizes its chunks so that a chunk's entries always fit; an
    // unsplit launch (no workspace) sized for a long max_context stages the first MAX_TABLE
    // entries and covers contexts up to MAX_TABLE blocks, reporting a longer one.
    __shared__ int s_blk[MAX_TABLE];
    const int begin = split * p.chunk;
    const int first_bi = begin / p.block_size;
    const int span = min(p.max_ctx, begin + p.chunk);  // positions this CTA may cover
    const int n_bi = span > begin ? min((span - 1) / p.block_size - first_bi + 1, MAX_TABLE) : 0;
    for (int i = threadIdx.x; i < n_bi; i += THREADS) s_blk[i] = p.block_table[e * p.bt_stride + first_bi + i];
    int ctx = p.context_len[e];
    if (ctx > p.max_ctx) {  // beyond the max_context the launch was sized for
        if (split == 0 && threadIdx.x == 0) report_status(LSE_ERR_INVALID_ARG);
        ctx = p.max_ctx;
    }
    int end = min(ctx, begin + p.chunk);
    if (end > (first_bi + n_bi) * p.block_size) {  // positions whose block ids were not staged
        if (threadIdx.x == 0) report_status(LSE_ERR_UNSUPPORTED);
        end = (first_bi + n_bi) * p.block_size;
    }

    // Q as the row operand, rows = query heads (rows >= G and 8..15 are zero): per K16 step
    // j, a0 = Q[r0][16j + 2q4 .. +1], a2 = Q[r0][16j + 8 + 2q4 .. +1].
    uint32_t qa[D / 16][2];
#pragma unroll
    for (int j = 0; j < D / 16; ++j) {
        qa[j][0] = qa[j][1] = 0u;
        if (r0 < G) {
            const T *qp = q_ptr + e * p.q_stride_e + (kvh * G + r0) * p.q_stride_h + 16 * j + 2 * q4;
            qa[j][0] = *reinterpret_cast<const uint32_t *>(qp);
            qa[j][1] = *reinterpret_cast<const uint32_t *>(qp + 8);
        }
    }
    __syncthreads();  // s_blk

    const int64_t row_elems = static_cast<int64_t>(p.H_kv) * D;  // one pool slot, all KV heads
    const uint32_t wbase = static_cast<uint32_t>(__cvta_generic_to_shared(dsmem)) + warp * STAGES * STAGE_B;
    // Issue the K/V rows of the iteration at position g0 into stage st (one commit group).
    auto issue = [&](int g0, int st) {
        int my_slot = -1;  // pool slot of position g0 + lane (lanes < 16)
        if (lane < KEYS && g0 + lane < end) {
            const int pos = g0 + lane;
            const int bi = pos / p.block_size;
            const int blk = s_blk[bi - first_bi];
            if (blk >= 0 && blk < p.num_blocks) my_slot = blk * p.block_size + (pos - bi * p.block_size);
            else report_status(LSE_ERR_INVALID_ARG);  // masked: the position is not read
        }
        const uint32_t kdst = wbase + st * STAGE_B, vdst = kdst + TILE_B;
        constexpr int RPI = 32 / CH;  // rows per instruction
#pragma unroll
        for (int i = 0; i < KEYS / RPI; ++i) {
            const int r = lane / CH + RPI * i, c = lane % CH;
            const int slot = __shfl_sync(0xffffffffu, my_slot, r);
            const bool ok = g0 < end && slot >= 0;
            const int64_t off = (ok ? slot : 0) * row_elems + kvh * D + c * 8;
            const uint32_t sw = r * ROWB + ((c ^ (r & 7)) << 4);
            cp_async16_zfill(kdst + sw, k_ptr + off, ok);
            cp_async16_zfill(vdst + sw, v_ptr + off, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        return __ballot_sync(0xffffffffu, lane < KEYS && my_slot >= 0);  // bit k: position g0 + k valid
    };

    float m_run = NEG_INF, l_run = 0.f;  // row r0 (head r0 when r0 < G)
    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;

    // vmask[i]: valid positions of iteration it + i (shifted down every iteration, so that
    // every index is a compile-time constant)
    unsigned vmask[STAGES];
#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) vmask[s] = issue(begin + (warp + s * WARPS) * KEYS, s);
    int st = 0;  // stage of iteration it
    for (int it = 0;; ++it) {
        const int g0 = begin + (warp + it * WARPS) * KEYS;
        if (g0 >= end) break;
        {
            const int nx = it + STAGES - 1;
            const int nst = st == 0 ? STAGES - 1 : st - 1;  // (it + STAGES - 1) % STAGES
            vmask[STAGES - 1] = issue(begin + (warp + nx * WARPS) * KEYS, nst);
        }
        asm volatile("cp.async.wait_group %0;" ::"n"(STAGES - 1) : "memory");
        __syncwarp();  // every lane's copies of this stage have landed
        const unsigned valid = vmask[0];
#pragma unroll
        for (int i = 0; i + 1 < STAGES; ++i) vmask[i] = vmask[i + 1];
        const uint32_t kt = wbase + st * STAGE_B, vt = kt + TILE_B;

        // S = Q K^T for keys 0-7 (s[0]) and 8-15 (s[1]); even and odd K16 steps accumulate
        // separately (two independent MMA chains per tile), summed after the loop
        float s[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        float s2[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        {
            const int r = (lane & 7) + ((lane >> 4) << 3), cl = (lane >> 3) & 1;
            const uint32_t rowp = kt + r * ROWB;
#pragma unroll
            for (int j = 0; j < D / 16; ++j) {
                // matrices: keys 0-7 / dims 16j.., keys 0-7 / 16j+8.., keys 8-15 / 16j.., keys 8-15 / 16j+8..
                const int c = 2 * j + cl;
                uint32_t b[4];
                ldsm_x4(rowp + ((c ^ (r & 7)) << 4), b);
                float (&d0)[4] = (j & 1) ? s2[0] : s[0];
                float (&d1)[4] = (j & 1) ? s2[1] : s[1];
                mma_16816<T>(d0, qa[j][0], 0u, qa[j][1], 0u, b[0], b[1]);
                mma_16816<T>(d1, qa[j][0], 0u, qa[j][1], 0u, b[2], b[3]);
            }
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int k = 0; k < 4; ++k) s[i][k] += s2[i][k];
        }
        // online softmax on row r0: this lane holds keys 2q4, 2q4+1 (tile 0) and 8 + 2q4, 9 + 2q4
        float sv[4] = {s[0][0] * p.scale_log2, s[0][1] * p.scale_log2, s[1][0] * p.scale_log2,
                       s[1][1] * p.scale_log2};
        const int kk[4] = {2 * q4, 2 * q4 + 1, 8 + 2 * q4, 9 + 2 * q4};
        float mx = NEG_INF;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if (!((valid >> kk[i]) & 1u)) sv[i] = NEG_INF;
            mx = fmaxf(mx, sv[i]);
        }
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run, mx);
        const float alpha = m_new == NEG_INF ? 1.f : exp2f(m_run - m_new);
        float pv[4], ps = 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            pv[i] = sv[i] == NEG_INF ? 0.f : exp2f(sv[i] - m_new);
            ps += pv[i];
        }
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        l_run = l_run * alpha + ps;
        m_run = m_new;
        // P as the row operand: a0 = row r0 keys 2q4..+1, a2 = row r0 keys 8+2q4..+1
        const uint32_t pa0 = pack2<T>(pv[0], pv[1]), pa2 = pack2<T>(pv[2], pv[3]);
#pragma unroll
        for (int t = 0; t < NT; t += 2) {
            // matrices: keys 0-7 / dims 8t.., keys 8-15 / 8t.., keys 0-7 / 8t+8.., keys 8-15 / 8t+8..
            const int r = (lane & 7) + (((lane >> 3) & 1) << 3), c = t + (lane >> 4);
            uint32_t b[4];
            ldsm_x4_trans(vt + r * ROWB + ((c ^ (r & 7)) << 4), b);
            acc[t][0] *= alpha;
            acc[t][1] *= alpha;
            acc[t + 1][0] *= alpha;
            acc[t + 1][1] *= alpha;
            mma_16816<T>(acc[t], pa0, 0u, pa2, 0u, b[0], b[1]);
            mma_16816<T>(acc[t + 1], pa0, 0u, pa2, 0u, b[2], b[3]);
        }
        __syncwarp();  // the stage is free for the copies issued next iteration
        st = st + 1 == STAGES ? 0 : st + 1;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");  // nothing in flight at exit

    // ---- merge the four warps (fixed order); the stage ring is reused for the sums ----
    __shared__ float sm_ml[WARPS][G][2];
    auto sm_acc = reinterpret_cast<float (*)[G][D]>(dsmem);  // [WARPS][G][D]
    static_assert(WARPS * G * D * 4 <= WARPS * STAGES * 2 * 16 * D * 2, "merge buffer fits the ring");
    __syncthreads();  // every warp is done with its stages
    if (r0 < G) {
        if (q4 == 0) {
            sm_ml[warp][r0][0] = m_run;
            sm_ml[warp][r0][1] = l_run;
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {  // row r0, dims 8t + 2q4, +1
            sm_acc[warp][r0][8 * t + 2 * q4] = acc[t][0];
            sm_acc[warp][r0][8 * t + 2 * q4 + 1] = acc[t][1];
        }
    }
    __syncthreads();

    const int pair = e * p.H_kv + kvh;
    // item (h, d) per thread, G * D / THREADS items each
    constexpr int ITEMS = (G * D + THREADS - 1) / THREADS;
    float res_m[ITEMS], res_l[ITEMS], res_a[ITEMS];
#pragma unroll
    for (int it = 0; it < ITEMS; ++it) {
        const int idx = threadIdx.x + it * THREADS;
        res_m[it] = NEG_INF;
        res_l[it] = 0.f;
        res_a[it] = 0.f;
        if (idx >= G * D) continue;
        const int h = idx / D, d = idx % D;
        float M = NEG_INF;
#pragma unroll
        for (int w = 0; w < WARPS; ++w) M = fmaxf(M, sm_ml[w][h][0]);
        float L = 0.f, A = 0.f;
        if (M != NEG_INF)
#pragma unroll
            for (int w = 0; w < WARPS; ++w) {
                const float f = sm_ml[w][h][0] == NEG_INF ? 0.f : exp2f(sm_ml[w][h][0] - M);
                L += sm_ml[w][h][1] * f;
                A += sm_acc[w][h][d] * f;
            }
        res_m[it] = M;
        res_l[it] = L;
        res_a[it] = A;
    }

    if (p.splits == 1) {
#pragma unroll
        for (int it = 0; it < ITEMS; ++it) {
            const int idx = threadIdx.x + it * THREADS;
            if (idx >= G * D) continue;
            const int h = idx / D, d = idx % D;
            const float out = res_l[it] > 0.f ? res_a[it] / res_l[it] : 0.f;
            o_ptr[e * p.o_stride_e + (kvh * G + h) * p.o_stride_h + d] = from_float<T>(out);
        }
        return;
    }

    // ---- several splits: publish this partial; the last CTA of the pair merges ----
    const int64_t acc_region = static_cast<int64_t>(p.E) * p.H_kv * p.splits * (G * D);
    const int64_t slot = static_cast<int64_t>(pair) * p.splits + split;
    float *acc_mine = p.part + slot * (G * D);            // [G][D], item idx = h * D + d
    float *ml_mine = p.part + acc_region + slot * (G * 2);  // [G][2]
#pragma unroll
    for (int it = 0; it < ITEMS; ++it) {
        const int idx = threadIdx.x + it * THREADS;
        if (idx >= G * D) continue;
        acc_mine[idx] = res_a[it];
        if (idx % D == 0) {
            ml_mine[(idx / D) * 2] = res_m[it];
            ml_mine[(idx / D) * 2 + 1] = res_l[it];
        }
    }
    __threadfence();
    __syncthreads();
    __shared__ int last;
    if (threadIdx.x == 0) {
        const int old = atomicAdd(p.counters + pair, 1);
        last = old == p.splits - 1;
        if (last) p.counters[pair] = 0;  // re-armed for the next launch
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    const float *acc_all = p.part + static_cast<int64_t>(pair) * p.splits * (G * D);
    const float *ml_all = p.part + acc_region + static_cast<int64_t>(pair) * p.splits * (G * 2);
    // Every split's (max, sum) per head in one cooperative pass, then each head's weights
    // exp2(m_s - M).
    __shared__ float s_w[MAX_SPLITS][G];
    __shared__ float s_ml[MAX_SPLITS][G][2];
    __shared__ float s_L[G];
    for (int i = threadIdx.x; i < p.splits * G; i += THREADS) {
        s_ml[i / G][i % G][0] = __ldcg(ml_all + 2 * i);
        s_ml[i / G][i % G][1] = __ldcg(ml_all + 2 * i + 1);
    }
    __syncthreads();
    if (threadIdx.x < G) {
        const int h = threadIdx.x;
        float M = NEG_INF;
        for (int sp = 0; sp < p.splits; ++sp) M = fmaxf(M, s_ml[sp][h][0]);
        float L = 0.f;
        for (int sp = 0; sp < p.splits; ++sp) {
            const float ms = s_ml[sp][h][0];
            const float f = (M == NEG_INF || ms == NEG_INF) ? 0.f : exp2f(ms - M);
            s_w[sp][h] = f;
            L += s_ml[sp][h][1] * f;
        }
        s_L[h] = L;
    }
    __syncthreads();
    // Accumulators: thread t owns dims 4f..4f+3 (f = t, t + THREADS, ...) of the G x D
    // output and loads them from SB splits at once (one 16-byte load each, all in flight
    // together), then folds them in split order (deterministic).
    constexpr int F4 = G * D / 4;
    constexpr int I4 = (F4 + THREADS - 1) / THREADS;
    constexpr int SB = I4 >= 2 ? 8 : 16;
    float4 A[I4];
#pragma unroll
    for (int i = 0; i < I4; ++i) A[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int sp0 = 0; sp0 < p.splits; sp0 += SB) {
        float4 v[I4][SB];
#pragma unroll
        for (int i = 0; i < I4; ++i) {
            const int f = threadIdx.x + i * THREADS;
#pragma unroll
            for (int u = 0; u < SB; ++u) {
                v[i][u] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (f < F4 && sp0 + u < p.splits)
                    v[i][u] = __ldcg(reinterpret_cast<const float4 *>(acc_all + static_cast<int64_t>(sp0 + u) * (G * D)) + f);
            }
        }
#pragma unroll
        for (int i = 0; i < I4; ++i) {
            const int f = threadIdx.x + i * THREADS;
            const int h = f < F4 ? (4 * f) / D : 0;
#pragma unroll
            for (int u = 0; u < SB; ++u) {
                if (sp0 + u < p.splits) {
                    const float w = s_w[sp0 + u][h];
                    A[i].x = fmaf(v[i][u].x, w, A[i].x);
                    A[i].y = fmaf(v[i][u].y, w, A[i].y);
                    A[i].z = fmaf(v[i][u].z, w, A[i].z);
                    A[i].w = fmaf(v[i][u].w, w, A[i].w);
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < I4; ++i) {
        const int f = threadIdx.x + i * THREADS;
        if (f >= F4) continue;
        const int h = (4 * f) / D, d = (4 * f) % D;
        const float L = s_L[h];
        T *op = o_ptr + e * p.o_stride_e + (kvh * G + h) * p.o_stride_h + d;
        op[0] = from_float<T>(L > 0.f ? A[i].x / L : 0.f);
        op[1] = from_float<T>(L > 0.f ? A[i].y / L : 0.f);
        op[2] = from_float<T>(L > 0.f ? A[i].z / L : 0.f);
        op[3] = from_float<T>(L > 0.f ? A[i].w / L : 0.f);
    }
}

}  // namespace attn
}  // namespace lse
