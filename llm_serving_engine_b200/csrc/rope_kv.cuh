// RoPE + K/V write on the fused QKV projection output (the reference's
// write_kv_and_project_q, src/llm_serving_engine/model/model_runner.py:342-355, with
// _project_qkv's view/transpose and transformers' apply_rotary_pos_emb): one launch instead
// of the rotation's elementwise kernels, the two pool scatters and q's transpose.
//
//   qkv [M, (H + 2 H_kv) * D] bf16 or fp16, T (row stride ld_qkv): q heads, then k, then v
//   cos, sin [M, D] (row stride ld_cs, fp32, bf16 or fp16 per `cs_type`): per-token rotation
//   rotate-half convention: out[d] = x[d] cos[d] - x[d + D/2] sin[d],
//                           out[d + D/2] = x[d + D/2] cos[d + D/2] + x[d] sin[d + D/2]
//   q_out[h, m, d]    rotated q, (n_heads, tokens, head_dim) as the reference returns it
//   k_dst[kv_off[m] + kvh * kv_head_stride + d]  rotated k (and v, unrotated, into v_dst):
//     the pool slot (block id * block_size + within) * H_kv * D for the reference's
//     [num_blocks, block_size, H_kv, D] pool, or any other per-token offset
// fp32 arithmetic, one rounding to T per output.  Memory-bound and tiny (a few hundred KB
// per decode step); one thread per (token, head, dim pair).
#pragma once

#include "common.cuh"

namespace lse {
namespace rope {

template <typename T>
struct Params {
    const T *qkv;
    int64_t ld_qkv;
    const void *cos, *sin;
    int64_t ld_cs;
    int cs_type;  // 0 fp32, 1 bf16, 2 fp16
    T *q_out;          // [H, M, D]
    T *k_dst, *v_dst;
    const int64_t *kv_off;         // [M] element offset of token m's slot (KV head 0)
    int64_t kv_head_stride;
    int M, H, H_kv, D;
};

__device__ __forceinline__ float load_cs(const void *p, int cs_type, int64_t i) {
    if (cs_type == 1) return __bfloat162float(static_cast<const __nv_bfloat16 *>(p)[i]);
    if (cs_type == 2) return __half2float(static_cast<const __half *>(p)[i]);
    return static_cast<const float *>(p)[i];
}

template <typename T>
__global__ void __launch_bounds__(256) rope_kv_kernel(const Params<T> p) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");  // qkv is the previous kernel's output
    const int half = p.D / 2;
    const int heads = p.H + 2 * p.H_kv;
    const int64_t total = static_cast<int64_t>(p.M) * heads * half;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int d = static_cast<int>(i % half);
        const int64_t mh = i / half;
        const int h = static_cast<int>(mh % heads);
        const int m = static_cast<int>(mh / heads);
        const T *src = p.qkv + m * p.ld_qkv + static_cast<int64_t>(h) * p.D;
        float x0 = to_float(src[d]), x1 = to_float(src[d + half]);
        if (h < p.H + p.H_kv) {  // q and k heads rotate
            const int64_t c = m * p.ld_cs;
            const float c0 = load_cs(p.cos, p.cs_type, c + d), c1 = load_cs(p.cos, p.cs_type, c + d + half);
            const float s0 = load_cs(p.sin, p.cs_type, c + d), s1 = load_cs(p.sin, p.cs_type, c + d + half);
            const float r0 = x0 * c0 - x1 * s0, r1 = x1 * c1 + x0 * s1;
            x0 = r0;
            x1 = r1;
        }
        T *dst;
        if (h < p.H) {
            dst = p.q_out + (static_cast<int64_t>(h) * p.M + m) * p.D;
        } else {
            const bool is_k = h < p.H + p.H_kv;
            const int kvh = is_k ? h - p.H : h - p.H - p.H_kv;
            dst = (is_k ? p.k_dst : p.v_dst) + p.kv_off[m] + kvh * p.kv_head_stride;
        }
        dst[d] = from_float<T>(x0);
        dst[d + half] = from_float<T>(x1);
    }
}

}  // namespace rope
}  // namespace lse
