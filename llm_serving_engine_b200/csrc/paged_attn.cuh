// Paged attention for any number of query tokens per batch entry (prefill chunks, mixed
// prefill + decode batches) on sm_100a: the general case of the reference's
// `paged_attention_2` (src/llm_serving_engine/kernels/flash_attention.py:202-284).
//
//   o[h, q_start[e] + i, :] = softmax_p( q[h, q_start[e] + i, :] . K[e, p, kvh(h), :] * scale ) V[e, p, kvh(h), :]
//     over positions p < context_len[e] with p <= query_offset[e] + i   (i < q_len[e])
//
// K/V in the engine's per-layer pool [num_blocks, block_size, H_KV, D] (position p of entry e
// in block block_table[e, p / block_size], slot p % block_size), q and o [H, tokens, D] with
// any head and token strides (d contiguous), element type bf16 or fp16.
//
// Shape: grid (token tiles, entries, KV heads).  A CTA takes 128 rows = the G query heads of
// 128 / G consecutive tokens of one entry, all reading the same KV head, so every K/V tile it
// stages serves the whole group (the G-fold reuse a per-head program would read again).  Eight
// warps, 16 rows each:
//   * K/V tiles of 64 positions are staged in shared memory by cp.async from all 256 threads,
//     three tiles in flight; rows are 16-byte-chunk swizzled (chunk c of row r at c ^ (r & 7)) so
//     ldmatrix reads them without bank conflicts;
//   * S = Q K^T on warp MMAs (m16n8k16, fp32 accumulate) with Q held in registers as the row
//     operand; causal and context masks on the accumulators; online softmax in base 2 per row;
//   * P (rounded to the element type, as the reference's `p.to(v.dtype)`) is the row operand of
//     O += P V straight from the S accumulators, V read by ldmatrix.trans.
// The key loop of a CTA stops at the furthest position any of its rows may see (as the
// reference's `end_n`).  A block id outside [0, num_blocks) masks that position (never read)
// and records LSE_ERR_INVALID_ARG on the device status word; a row with no position to attend
// to gets zeros.
#pragma once

#include <cuda_fp16.h>

#include "decode_attn.cuh"

namespace lse {
namespace pattn {

constexpr int WARPS = 8;
constexpr int THREADS = WARPS * 32;
constexpr int ROWS = WARPS * 16;  // (token, head) rows per CTA
constexpr int KEYS = 64;          // positions per K/V tile
constexpr int STAGES = 3;

template <int D>
constexpr int smem_bytes() { return STAGES * 2 * KEYS * D * 2; }

struct Params {
    const void *q;             // [H, tokens, D], element (h, t, d) at q[h * q_sh + t * q_sm + d]
    int64_t q_sh, q_sm;
    const void *k_pool, *v_pool;  // [num_blocks, block_size, H_KV, D] contiguous
    const int *block_table;    // [E, >= ceil(context_len / block_size)]
    int64_t bt_stride;
    const int *context_len, *query_offset, *q_start, *q_len;  // [E]
    void *o;                   // [H, tokens, D], element (h, t, d) at o[h * o_sh + t * o_sm + d]
    int64_t o_sh, o_sm;
    int H_kv, block_size, num_blocks;
    float scale_log2;          // softmax scale * log2(e)
};

// 2^x (the SFU's approximation: relative error ~2^-22, subnormal results flushed to 0;
// 2^-inf = 0)
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// D (16x8 fp32) += A (16x16, row) * B (16x8, col), A and B of element type T
template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
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

// Two fp32 -> one 32-bit word of two T (round to nearest), low half = first
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

template <int D, int G, typename T>
__global__ void __launch_bounds__(THREADS, 1) paged_attn_kernel(const Params p) {
    static_assert(D == 64 || D == 128, "head_dim");
    static_assert(G == 1 || G == 2 || G == 4 || G == 8, "query heads per KV head");
    constexpr int TOKS = ROWS / G;     // tokens per CTA
    constexpr int CH = D / 8;          // 16-byte chunks per K/V row
    constexpr int ROWB = D * 2;        // bytes per staged row
    constexpr int TILE_B = KEYS * ROWB;
    constexpr int STAGE_B = 2 * TILE_B;
    constexpr int NT = D / 8;          // output dim tiles
    constexpr int SN = KEYS / 8;       // score tiles of 8 positions
    const int tile = blockIdx.x, e = blockIdx.y, kvh = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = lane >> 2, q4 = lane & 3;
    const float NEG_INF = -__int_as_float(0x7f800000);
    extern __shared__ __align__(128) uint8_t dsmem[];  // [STAGES][K tile, V tile]

    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // q and the pool come from earlier kernels

    const int qlen = p.q_len[e];
    const int t0 = tile * TOKS;
    if (t0 >= qlen) return;  // the grid is sized for the longest entry
    const int qs = p.q_start[e], ctx = p.context_len[e], qoff = p.query_offset[e];
    const int t_hi = min(qlen, t0 + TOKS);
    const int kend = max(0, min(ctx, qoff + t_hi));  // one past the furthest position any row sees

    // This thread's two rows (MMA rows r0 and r0 + 8 of its warp): token and query head.
    const int ra = 16 * warp + r0, rb = ra + 8;
    const int ta = t0 + ra / G, ha = ra % G, tb = t0 + rb / G, hb = rb % G;
    const bool va = ta < t_hi, vb = tb < t_hi;
    const int lim_a = min(ctx, qoff + ta + 1), lim_b = min(ctx, qoff + tb + 1);  // positions < lim are seen

    // Q as the row operand: per K16 step j, a0/a2 = row a dims 16j + 2q4 (+8), a1/a3 = row b.
    const T *q = static_cast<const T *>(p.q);
    const T *qra = q + static_cast<int64_t>(kvh * G + ha) * p.q_sh + static_cast<int64_t>(qs + ta) * p.q_sm;
    const T *qrb = q + static_cast<int64_t>(kvh * G + hb) * p.q_sh + static_cast<int64_t>(qs + tb) * p.q_sm;
    uint32_t qa[D / 16][4];
#pragma unroll
    for (int j = 0; j < D / 16; ++j) {
        qa[j][0] = va ? *reinterpret_cast<const uint32_t *>(qra + 16 * j + 2 * q4) : 0u;
        qa[j][1] = vb ? *reinterpret_cast<const uint32_t *>(qrb + 16 * j + 2 * q4) : 0u;
        qa[j][2] = va ? *reinterpret_cast<const uint32_t *>(qra + 16 * j + 8 + 2 * q4) : 0u;
        qa[j][3] = vb ? *reinterpret_cast<const uint32_t *>(qrb + 16 * j + 8 + 2 * q4) : 0u;
    }

    const T *kpool = static_cast<const T *>(p.k_pool);
    const T *vpool = static_cast<const T *>(p.v_pool);
    const int64_t row_elems = static_cast<int64_t>(p.H_kv) * D;  // one pool slot, all KV heads
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(dsmem));
    // Positions kb0 .. kb0 + 63 of K and V into stage st (one commit group); a position at or
    // beyond kend, or with a bad block id, is zero-filled and never read as data.
    auto issue = [&](int kb0, int st) {
        const uint32_t kdst = sbase + st * STAGE_B, vdst = kdst + TILE_B;
        constexpr int PER = KEYS * CH / THREADS;
#pragma unroll
        for (int c = 0; c < PER; ++c) {
            const int ci = threadIdx.x + c * THREADS;
            const int r = ci / CH, ch = ci % CH;
            const int pos = kb0 + r;
            bool ok = pos < kend;
            int64_t off = 0;
            if (ok) {
                const int bi = pos / p.block_size;
                const int blk = p.block_table[e * p.bt_stride + bi];
                if (blk >= 0 && blk < p.num_blocks) {
                    off = (static_cast<int64_t>(blk) * p.block_size + (pos - bi * p.block_size)) * row_elems + kvh * D + ch * 8;
                } else {
                    ok = false;
                    report_status(LSE_ERR_INVALID_ARG);
                }
            }
            const uint32_t sw = r * ROWB + ((ch ^ (r & 7)) << 4);
            attn::cp_async16_zfill(kdst + sw, kpool + off, ok);
            attn::cp_async16_zfill(vdst + sw, vpool + off, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    float m_a = NEG_INF, l_a = 0.f, m_b = NEG_INF, l_b = 0.f;
    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.f;

    const int ntiles = (kend + KEYS - 1) / KEYS;
    if (ntiles > 0) issue(0, 0);
    if (ntiles > 1) issue(KEYS, 1);
    for (int it = 0; it < ntiles; ++it) {
        const int st = it % STAGES;
        if (it + 2 < ntiles) {
            issue((it + 2) * KEYS, (it + 2) % STAGES);  // the stage tile it - 1 used: free since its barrier
            asm volatile("cp.async.wait_group 2;" ::: "memory");
        } else if (it + 1 < ntiles) {
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();  // every thread's copies of tile `it` have landed
        const uint32_t kt = sbase + st * STAGE_B, vt = kt + TILE_B;
        const int kb0 = it * KEYS;

        // S = Q K^T, score tile n = positions kb0 + 8n .. +7
        float s[SN][4];
#pragma unroll
        for (int n = 0; n < SN; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
        {
            const int r = (lane & 7) + ((lane >> 4) << 3), cl = (lane >> 3) & 1;
#pragma unroll
            for (int m = 0; m < SN / 2; ++m) {
                const uint32_t rowp = kt + (16 * m + r) * ROWB;
#pragma unroll
                for (int j = 0; j < D / 16; ++j) {
                    // matrices: positions 16m..+7 / dims 16j.., 16m..+7 / 16j+8.., 16m+8.. / 16j.., 16m+8.. / 16j+8..
                    const int c = 2 * j + cl;
                    uint32_t b[4];
                    attn::ldsm_x4(rowp + ((c ^ (r & 7)) << 4), b);
                    mma16816<T>(s[2 * m], qa[j][0], qa[j][1], qa[j][2], qa[j][3], b[0], b[1]);
                    mma16816<T>(s[2 * m + 1], qa[j][0], qa[j][1], qa[j][2], qa[j][3], b[2], b[3]);
                }
            }
        }
        // masks and online softmax (base 2, scale folded into one FMA per score): this lane
        // holds, per score tile n, positions kb0 + 8n + 2q4 (+1) of row a (s[n][0..1]) and row b
        // (s[n][2..3]).  A tile every row of the CTA sees in full needs no mask.
        const float c = p.scale_log2;
        if (kb0 + KEYS > min(ctx, qoff + t0 + 1)) {
#pragma unroll
            for (int n = 0; n < SN; ++n)
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const int pos = kb0 + 8 * n + 2 * q4 + u;
                    if (pos >= lim_a) s[n][u] = NEG_INF;
                    if (pos >= lim_b) s[n][2 + u] = NEG_INF;
                }
        }
        float mxa = NEG_INF, mxb = NEG_INF;
#pragma unroll
        for (int n = 0; n < SN; ++n) {
            mxa = fmaxf(mxa, fmaxf(s[n][0], s[n][1]));
            mxb = fmaxf(mxb, fmaxf(s[n][2], s[n][3]));
        }
        mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 1));
        mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, 2));
        mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 1));
        mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, 2));
        const float mna = fmaxf(m_a, mxa), mnb = fmaxf(m_b, mxb);  // raw (unscaled) running maxima
        const float alpha_a = mna == NEG_INF ? 1.f : ex2((m_a - mna) * c);
        const float alpha_b = mnb == NEG_INF ? 1.f : ex2((m_b - mnb) * c);
        const float mca = mna == NEG_INF ? 0.f : mna * c, mcb = mnb == NEG_INF ? 0.f : mnb * c;
        float psa = 0.f, psb = 0.f;
#pragma unroll
        for (int n = 0; n < SN; ++n)
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                s[n][u] = ex2(fmaf(s[n][u], c, -mca));  // a masked score gives 2^-inf = 0
                s[n][2 + u] = ex2(fmaf(s[n][2 + u], c, -mcb));
                psa += s[n][u];
                psb += s[n][2 + u];
            }
        psa += __shfl_xor_sync(0xffffffffu, psa, 1);
        psa += __shfl_xor_sync(0xffffffffu, psa, 2);
        psb += __shfl_xor_sync(0xffffffffu, psb, 1);
        psb += __shfl_xor_sync(0xffffffffu, psb, 2);
        l_a = l_a * alpha_a + psa;
        l_b = l_b * alpha_b + psb;
        m_a = mna;
        m_b = mnb;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
            acc[t][0] *= alpha_a;
            acc[t][1] *= alpha_a;
            acc[t][2] *= alpha_b;
            acc[t][3] *= alpha_b;
        }
        // O += P V: the score tiles 2k, 2k + 1 are the row operand of K16 step k
#pragma unroll
        for (int k = 0; k < SN / 2; ++k) {
            const uint32_t a0 = pack2<T>(s[2 * k][0], s[2 * k][1]), a1 = pack2<T>(s[2 * k][2], s[2 * k][3]);
            const uint32_t a2 = pack2<T>(s[2 * k + 1][0], s[2 * k + 1][1]), a3 = pack2<T>(s[2 * k + 1][2], s[2 * k + 1][3]);
            const int r = 16 * k + (lane & 7) + (((lane >> 3) & 1) << 3);
#pragma unroll
            for (int t = 0; t < NT; t += 2) {
                // matrices: positions 16k..+7 / dims 8t.., 16k+8.. / 8t.., 16k.. / 8t+8.., 16k+8.. / 8t+8..
                const int c = t + (lane >> 4);
                uint32_t b[4];
                attn::ldsm_x4_trans(vt + r * ROWB + ((c ^ (r & 7)) << 4), b);
                mma16816<T>(acc[t], a0, a1, a2, a3, b[0], b[1]);
                mma16816<T>(acc[t + 1], a0, a1, a2, a3, b[2], b[3]);
            }
        }
        __syncthreads();  // every warp is done with this stage before it is refilled
    }

    // o = acc / l (zeros for a row that saw no position)
    T *o = static_cast<T *>(p.o);
    const float ia = l_a > 0.f ? 1.f / l_a : 0.f, ib = l_b > 0.f ? 1.f / l_b : 0.f;
    if (va) {
        T *orow = o + static_cast<int64_t>(kvh * G + ha) * p.o_sh + static_cast<int64_t>(qs + ta) * p.o_sm + 2 * q4;
#pragma unroll
        for (int t = 0; t < NT; ++t)
            *reinterpret_cast<uint32_t *>(orow + 8 * t) = pack2<T>(acc[t][0] * ia, acc[t][1] * ia);
    }
    if (vb) {
        T *orow = o + static_cast<int64_t>(kvh * G + hb) * p.o_sh + static_cast<int64_t>(qs + tb) * p.o_sm + 2 * q4;
#pragma unroll
        for (int t = 0; t < NT; ++t)
            *reinterpret_cast<uint32_t *>(orow + 8 * t) = pack2<T>(acc[t][2] * ib, acc[t][3] * ib);
    }
}

}  // namespace pattn
}  // namespace lse
