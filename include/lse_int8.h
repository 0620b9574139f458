/*
 * lse_int8.h -- C ABI of the B200 (sm_100a) int8 weight-only linear for
 * vladimirfilip/llm-serving-engine.
 *
 * The reference engine calls each projection as a torch.nn.Linear module
 * (src/llm_serving_engine/model/model_runner.py:322-324 q/k/v, :369 and :418 o_proj,
 * :223 the MLP; src/llm_serving_engine/model/piecewise_graph.py:163-166) with
 * y = x W^T, W [out_features, in_features], no bias, and raises NotImplementedError for
 * ModelConfig.quantize == "int8" (model_runner.py:45-46; config.py:32,46).  This library
 * is what that `quantize="int8"` switch binds to: each entry point below replaces one
 * piece of the nn.Linear call the engine makes.
 *
 * Conventions (all entry points):
 *   - Plain pointers to device memory, sizes in elements, row strides in elements.
 *   - `stream` is a cudaStream_t passed as void*; every launch goes to that stream, no
 *     entry point synchronizes, allocates device memory, or changes device settings, so
 *     each one can be captured in a CUDA graph (after lse_init on that device).
 *     lse_int8_linear_packed_noalloc is outside this paragraph: its notes are its own.
 *   - Return value is an lse_status; nonzero means nothing was launched (argument errors)
 *     or the launch failed (LSE_ERR_CUDA).  The library never aborts or traps.
 *   - The caller owns every buffer.
 */
#ifndef LSE_INT8_H
#define LSE_INT8_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum lse_status {
    LSE_OK = 0,
    LSE_ERR_INVALID_ARG = 1,   /* null pointer, negative size, ld < K, ... */
    LSE_ERR_ALIGNMENT = 2,     /* K % 16, ldx % 8, ldy % 8 or a pointer not 16-byte aligned */
    LSE_ERR_UNSUPPORTED = 3,   /* shape/algo combination this build does not run */
    LSE_ERR_WORKSPACE = 4,     /* workspace missing or smaller than lse_int8_linear_workspace() */
    LSE_ERR_CUDA = 5,          /* a CUDA runtime/driver call failed (see lse_last_cuda_error) */
    LSE_ERR_DEVICE_TIMEOUT = 6 /* a device-side wait ran out (reported by lse_device_status) */
} lse_status;

/* Kernel selection for lse_int8_linear_ex. */
typedef enum lse_algo {
    LSE_ALGO_AUTO = 0,     /* pick by M, weight layout and weight size (see lse_int8_linear_packed) */
    LSE_ALGO_GEMV = 1,     /* row-major W only: CUDA-core GEMV, 128-bit int8 streams, warp-shuffle reduction */
    LSE_ALGO_TCGEN05 = 2,  /* tcgen05/TMEM tensor-core GEMM fed by TMA (whole tiles, stream-K
                              or a cluster split of K, by shape) */
    LSE_ALGO_SKINNY = 3    /* packed W only, M <= 32: warp-MMA skinny GEMM for decode, weights
                              streamed straight into registers (fp16 MMA for M <= 8 with bf16->fp16
                              activations, bf16 MMA above), K split reduced across warps with the
                              scale folded in */
} lse_algo;

/* Weight dtypes accepted by lse_int8_quantize. */
typedef enum lse_dtype { LSE_BF16 = 0, LSE_F16 = 1, LSE_F32 = 2 } lse_dtype;

/*
 * One-time per-device set-up (SM count, kernel attributes, driver entry points).  Optional:
 * the first call of any entry point on a device does it; call it explicitly before a CUDA
 * graph capture so that capture records only kernel launches.
 */
int lse_init(int device);

/*
 * y[m, n] = bf16( s[n] * sum_k x[m, k] * w[n, k] )       m < M, n < N
 *
 * Replaces nn.Linear.forward at the call sites above (model_runner.py:322-324,369,418,223).
 *   x      bf16 [M, K], row stride ldx (>= K, multiple of 8), 16-byte aligned
 *   w      int8 [N, K] row-major (nn.Linear [out, in] layout), K % 16 == 0, 16-byte aligned
 *   scale  fp32 [N] per-output-channel scale
 *   y      bf16 [M, N], row stride ldy (>= N), 2-byte aligned
 *   workspace  device scratch of at least lse_int8_linear_workspace(M, K, N) bytes (0 and NULL
 *              are allowed when lse_int8_linear_workspace_for reports 0 for the call), 16-byte
 *              aligned, contents irrelevant: the call initialises what it uses, so a fresh
 *              allocation from any allocator (a caching allocator's block, memory captured
 *              into a CUDA graph's pool) serves.
 * M == 0 or N == 0 is a no-op returning LSE_OK.  K == 0 writes zeros.
 * Calls that share one workspace must be ordered on the GPU (same stream, or events).
 *
 * The tensor-core path (LSE_ALGO_TCGEN05) multiplies int8 weights by int8 activation digits:
 * a first kernel writes each token row as S signed 8-bit digit planes under a power-of-two
 * row scale (S = 3 up to 64 tokens, 2 above: every element at least 2^(10-8S) times the
 * row's largest is represented exactly, any element to within 2^-(8S-2) of the largest),
 * the projection accumulates in exact int32 (tcgen05.mma kind::i8) and applies the scales
 * in fp32.  A row holding a NaN or an infinity produces a NaN output row.
 */
int lse_int8_linear(const void *x, int64_t M, int64_t K, int64_t ldx,
                    const int8_t *w, const float *scale, int64_t N,
                    void *y, int64_t ldy,
                    void *workspace, size_t workspace_bytes,
                    void *stream);

/* Same as lse_int8_linear with an explicit kernel choice (lse_algo). */
int lse_int8_linear_ex(const void *x, int64_t M, int64_t K, int64_t ldx,
                       const int8_t *w, const float *scale, int64_t N,
                       void *y, int64_t ldy,
                       void *workspace, size_t workspace_bytes,
                       int algo, void *stream);

/*
 * Packed weights.  Both kernels stream weights from one packed layout: W is zero padded to
 * Np = 128*ceil(N/128) rows and Kp = 128*ceil(K/128) columns and cut into row blocks of 16
 * rows; row block b is one contiguous run of 16*Kp bytes made of 2 KB blocks, one per 128
 * columns, each holding the block's two 8-row groups (h) one after the other as two 512-byte
 * atoms of 64 columns (a); an atom holds its 8 rows' 64 columns (64 bytes per row) with the
 * 16-byte chunk c of row r stored at chunk position c ^ ((r >> 1) & 3) (the tensor core's
 * 64-byte swizzle):
 *   W[16b + 8h + r][128t + 64a + 16c + e]  at
 *     b*16*Kp + t*2048 + h*1024 + a*512 + r*64 + (c ^ ((r >> 1) & 3))*16 + e
 * (h, a < 2, r < 8, c < 4, e < 16), plain two's-complement bytes.  A 128 x 128 tile is then
 * the tensor core's K-major operand as it stands (eight runs of 2 KB, one bulk-tensor copy),
 * and one 128-bit load per lane gives the decode kernel a warp-MMA operand fragment, without
 * any shuffling.
 * The repack happens once, at load (the build's counterpart of the reference loading
 * nn.Linear weights at model_runner.py:50-53); lse_int8_linear_packed then has the same
 * contract as lse_int8_linear_ex with `w_packed` in place of the row-major W.  Its auto
 * choice is LSE_ALGO_SKINNY for M <= 16 (decode), and for M <= 32 when N * K <= 32 MiB (where
 * the tensor-core kernel's fixed cost per launch outweighs its faster weight stream), and
 * LSE_ALGO_TCGEN05 otherwise.
 */
size_t lse_int8_packed_weight_bytes(int64_t N, int64_t K);
int lse_int8_pack_weight(const int8_t *w, int64_t N, int64_t K, int64_t ldw, int8_t *w_packed, void *stream);
int lse_int8_unpack_weight(const int8_t *w_packed, int64_t N, int64_t K, int8_t *w, void *stream);
int lse_int8_linear_packed(const void *x, int64_t M, int64_t K, int64_t ldx,
                           const int8_t *w_packed, const float *scale, int64_t N,
                           void *y, int64_t ldy,
                           void *workspace, size_t workspace_bytes,
                           int algo, void *stream);

/*
 * y[m, n] = bf16( residual[m, n] + s[n] * sum_k x[m,k] * W[n,k] )
 *
 * lse_int8_linear_packed with the decoder layer's residual add fused into the epilogue (the
 * `hidden = residual + o_proj(...)` and `hidden = residual + mlp(...)` steps of transformers'
 * LlamaDecoderLayer.forward, reached at model_runner.py:213-224): the sum is formed in fp32
 * and rounded to bf16 once.  residual: bf16 [M, N], row stride ldr (>= N), 2-byte aligned;
 * it may be y itself (residual == y and ldr == ldy: in-place update), other overlaps are
 * not allowed.  residual == NULL is LSE_ERR_INVALID_ARG.  All algorithms (LSE_ALGO_*).
 */
int lse_int8_linear_packed_residual(const void *x, int64_t M, int64_t K, int64_t ldx,
                                    const int8_t *w_packed, const float *scale, int64_t N,
                                    const void *residual, int64_t ldr,
                                    void *y, int64_t ldy,
                                    void *workspace, size_t workspace_bytes,
                                    int algo, void *stream);

/*
 * y[m, i] = bf16( silu(s_g[i] * sum_k x[m,k] * w_g[i,k]) * (s_u[i] * sum_k x[m,k] * w_u[i,k]) )
 *
 * The Llama MLP's gate and up projections and SiLU * mul (transformers' LlamaMLP.forward,
 * reached at model_runner.py:223 and piecewise_graph.py:166) in one decode-kernel launch,
 * for M <= 16 (LSE_ERR_UNSUPPORTED above: run lse_int8_linear_packed on the same weights
 * and pair the columns).  No workspace.
 *   w_packed  the packed layout (lse_int8_pack_weight) of a [2I, K] int8 matrix whose rows
 *             interleave 8-row blocks: rows 16j..16j+7 are gate rows 8j..8j+7 and rows
 *             16j+8..16j+15 the matching up rows
 *   scale     fp32 [2I], interleaved the same way
 *   y         bf16 [M, I], row stride ldy (>= I);  I % 8 == 0 (LSE_ERR_UNSUPPORTED otherwise)
 * SiLU and the product are evaluated in fp32 and rounded to bf16 once.
 */
int lse_int8_gate_up_silu_packed(const void *x, int64_t M, int64_t K, int64_t ldx,
                                 const int8_t *w_packed, const float *scale, int64_t I,
                                 void *y, int64_t ldy, void *stream);

/*
 * The same for any M, with a workspace of at least lse_int8_linear_workspace(M, K, 2 * I)
 * bytes (any contents, as for lse_int8_linear_packed; unused for M <= 16): M <= 16
 * runs the decode kernel above, larger M the tcgen05 kernel with SiLU * mul in its epilogue,
 * so that the [M, 2I] gate/up output never reaches memory.  Same weights, scales, y and
 * error codes as lse_int8_gate_up_silu_packed, plus LSE_ERR_WORKSPACE.
 */
int lse_int8_gate_up_silu_packed_ws(const void *x, int64_t M, int64_t K, int64_t ldx,
                                    const int8_t *w_packed, const float *scale, int64_t I,
                                    void *y, int64_t ldy, void *workspace, size_t workspace_bytes,
                                    void *stream);

/*
 * The packed-weight entry points with the activation type as an argument: `dtype` LSE_BF16 or
 * LSE_F16 (the reference's ModelConfig.dtype default, src/llm_serving_engine/config.py:31) for
 * x, y and the residual alike; arguments and workspace otherwise as lse_int8_linear_packed
 * (with the optional `residual`: null, or as lse_int8_linear_packed_residual) and
 * lse_int8_gate_up_silu_packed_ws.  fp16 activations enter the decode kernel's fp16 MMA as they
 * are and the tensor-core kernel's digit planes the same way as bf16 (exact for every element
 * at least 2^(13-8S) times its row maximum); one rounding of y to fp16.
 */
int lse_int8_linear_packed_dt(const void *x, int dtype, int64_t M, int64_t K, int64_t ldx, const int8_t *w_packed,
                              const float *scale, int64_t N, const void *residual, int64_t ldr, void *y, int64_t ldy,
                              void *workspace, size_t workspace_bytes, int algo, void *stream);
int lse_int8_gate_up_silu_packed_dt(const void *x, int dtype, int64_t M, int64_t K, int64_t ldx,
                                    const int8_t *w_packed, const float *scale, int64_t I, void *y, int64_t ldy,
                                    void *workspace, size_t workspace_bytes, void *stream);

/*
 * Paged decode attention, one query token per sequence (the decode-step call of the
 * reference's paged_attention_forward, src/llm_serving_engine/kernels/flash_attention.py:
 * 287-332, with q_len = 1 and query_offset = context_len - 1):
 *
 *   o[e, h, :] = softmax_p( q[e, h, :] . K[e, p, h / G, :] * scale ) V[e, p, h / G, :],
 *                p = 0 .. context_len[e] - 1,  G = H / H_kv
 *
 *   q        bf16, element (e, h, d) at q[e * q_stride_e + h * q_stride_h + d]
 *   k_pool, v_pool  bf16 [num_blocks, block_size, H_kv, D], contiguous; position p of
 *            sequence e is block block_table[e * bt_stride + p / block_size], slot
 *            p % block_size
 *   context_len  int32 [E], each <= max_context (the launch is sized for max_context; a
 *            larger entry is cut there and reported as LSE_ERR_INVALID_ARG by
 *            lse_device_status, as is a block id outside [0, num_blocks))
 *   o        bf16, element (e, h, d) at o[e * o_stride_e + h * o_stride_h + d]
 *   workspace  >= lse_paged_decode_attention_workspace(E, H, H_kv, D, max_context, block_size)
 *            bytes (0 allowed when that is 0), 16-byte aligned, zeroed once before its first
 *            use; the split-K arrival counters at its start have the same place for every
 *            launch shape and every call leaves them at zero, so one buffer per stream
 *            (grown when a shape needs more) serves all shapes.  workspace = NULL with
 *            workspace_bytes = 0 asks for the unsplit launch (one CTA per sequence and KV head,
 *            no workspace) for any max_context; it covers a sequence's first 1024 blocks of
 *            positions, and a longer context_len is cut there and reported as
 *            LSE_ERR_UNSUPPORTED by lse_device_status
 * D = 64 or 128 and G in {1, 2, 4, 8} (LSE_ERR_UNSUPPORTED otherwise).  fp32 softmax and
 * accumulation, one bf16 rounding of o.  A sequence with context_len 0 gets zeros.
 */
size_t lse_paged_decode_attention_workspace(int64_t E, int64_t H, int64_t H_kv, int64_t D, int64_t max_context,
                                            int64_t block_size);
int lse_paged_decode_attention(const void *q, int64_t E, int64_t H, int64_t D, int64_t q_stride_e,
                               int64_t q_stride_h, const void *k_pool, const void *v_pool, int64_t num_blocks,
                               int64_t block_size, int64_t H_kv, const int32_t *block_table, int64_t bt_stride,
                               const int32_t *context_len, int64_t max_context, float scale, void *o,
                               int64_t o_stride_e, int64_t o_stride_h, void *workspace, size_t workspace_bytes,
                               void *stream);
/* The same with q, the pools and o of `dtype` (LSE_BF16 or LSE_F16; fp16 MMA for fp16). */
int lse_paged_decode_attention_dt(const void *q, int dtype, int64_t E, int64_t H, int64_t D, int64_t q_stride_e,
                                  int64_t q_stride_h, const void *k_pool, const void *v_pool, int64_t num_blocks,
                                  int64_t block_size, int64_t H_kv, const int32_t *block_table, int64_t bt_stride,
                                  const int32_t *context_len, int64_t max_context, float scale, void *o,
                                  int64_t o_stride_e, int64_t o_stride_h, void *workspace, size_t workspace_bytes,
                                  void *stream);

/*
 * RoPE and K/V write on the fused QKV output (the reference's write_kv_and_project_q,
 * src/llm_serving_engine/model/model_runner.py:342-355, with transformers'
 * apply_rotary_pos_emb): for token m (of M) and head h of qkv [M, (H + 2 H_kv) * D] (row stride
 * ld_qkv; q heads, then k heads, then v heads),
 *   q and k are rotated (rotate-half): out[d] = x[d] cos[m,d] - x[d+D/2] sin[m,d],
 *                                      out[d+D/2] = x[d+D/2] cos[m,d+D/2] + x[d] sin[m,d+D/2]
 *   q_out[h, m, :]                                   rotated q, bf16 [H, M, D]
 *   k_dst[kv_offset[m] + kvh * kv_head_stride + :]   rotated k, bf16
 *   v_dst[kv_offset[m] + kvh * kv_head_stride + :]   v as it is, bf16
 * cos, sin: [M, D] with row stride ld_cs, fp32 (LSE_F32) or bf16 (LSE_BF16).  For the
 * reference's pool [num_blocks, block_size, H_kv, D], kv_offset[m] =
 * (dest_block_id[m] * block_size + dest_within[m]) * H_kv * D and kv_head_stride = D.
 * fp32 arithmetic, one bf16 rounding per output.
 */
int lse_rope_kv_write(const void *qkv, int64_t M, int64_t ld_qkv, int64_t H, int64_t H_kv, int64_t D,
                      const void *cos, const void *sin, int64_t ld_cs, int cs_dtype, void *q_out,
                      void *k_dst, void *v_dst, const int64_t *kv_offset, int64_t kv_head_stride, void *stream);
/* The same with the rows' type given: dtype LSE_BF16 or LSE_F16 for qkv, q_out and the
 * caches; cs_dtype LSE_F32, LSE_BF16 or LSE_F16 for the cos / sin tables. */
int lse_rope_kv_write_dt(const void *qkv, int dtype, int64_t M, int64_t ld_qkv, int64_t H, int64_t H_kv, int64_t D,
                         const void *cos, const void *sin, int64_t ld_cs, int cs_dtype, void *q_out, void *k_dst,
                         void *v_dst, const int64_t *kv_offset, int64_t kv_head_stride, void *stream);

/*
 * RMSNorm of bf16 rows (transformers' LlamaRMSNorm, every decoder layer's input and
 * post-attention norm and the final norm):
 *   y[m, :] = bf16( x[m, :] * rsqrt(mean_n x[m, n]^2 + eps) * weight[:] )   (fp32 arithmetic)
 * x [M, N] row stride ldx, weight bf16 [N], y [M, N] row stride ldy (may be x itself);
 * N, ldx, ldy multiples of 8, x / weight / y 16-byte aligned.
 */
int lse_rms_norm(const void *x, int64_t M, int64_t N, int64_t ldx, const void *weight, float eps, void *y,
                 int64_t ldy, void *stream);
/* The same with the rows' type given: dtype LSE_BF16 or LSE_F16 (x, weight and y alike). */
int lse_rms_norm_dt(const void *x, int dtype, int64_t M, int64_t N, int64_t ldx, const void *weight, float eps,
                    void *y, int64_t ldy, void *stream);

/*
 * RMSNorm fused with the packed projection that consumes it, bf16 activations: the decoder
 * layer's qkv(input_layernorm(h)) (model_runner.py:213-224 with the fused QKV of :310-326) and
 * mlp(post_attention_layernorm(h)) up to the SiLU * mul (modeling_llama.py:171-184):
 *   lse_int8_rms_norm_linear_packed:       y = lse_int8_linear_packed(rms_norm(x, norm_weight, eps))
 *   lse_int8_rms_norm_gate_up_silu_packed: y = lse_int8_gate_up_silu_packed_ws(rms_norm(x, ...))
 * with rms_norm as lse_rms_norm (K = the normalised width), and the same results bit for bit
 * as those two calls in sequence.  Where the projection alone takes the tensor-core kernel
 * (the entries' automatic choice) the normalisation writes its activation digit planes
 * directly (no normalised copy of x, one launch fewer); where it takes the decode kernel the
 * normalised rows pass through the workspace to it.
 *   norm_weight  bf16 [K], 16-byte aligned; eps >= 0
 *   workspace    >= lse_int8_rms_norm_proj_workspace(M, K) bytes (N-independent: M * K * 2
 *                bytes up to 16 tokens, at least lse_int8_linear_workspace's bound above),
 *                16-byte aligned, contents irrelevant
 * Other arguments and status codes as the unfused entries.
 */
size_t lse_int8_rms_norm_proj_workspace(int64_t M, int64_t K);
int lse_int8_rms_norm_linear_packed(const void *x, int64_t M, int64_t K, int64_t ldx, const void *norm_weight,
                                    float eps, const int8_t *w_packed, const float *scale, int64_t N, void *y,
                                    int64_t ldy, void *workspace, size_t workspace_bytes, void *stream);
int lse_int8_rms_norm_gate_up_silu_packed(const void *x, int64_t M, int64_t K, int64_t ldx, const void *norm_weight,
                                          float eps, const int8_t *w_packed, const float *scale, int64_t I, void *y,
                                          int64_t ldy, void *workspace, size_t workspace_bytes, void *stream);

/* Bytes of the counter region at the start of every linear workspace (the tensor-core path
 * clears the counters it uses before each launch). */
#define LSE_WS_COUNTER_BYTES 65536

/* Workspace bytes the tensor-core path needs for this shape (any weight layout): stream-K
 * counters, partial tiles, the activation digit planes and row scales; always >= the counter
 * region.  Enough for every algorithm. */
size_t lse_int8_linear_workspace(int64_t M, int64_t K, int64_t N);

/* Workspace bytes one call with this algorithm choice (lse_algo, after LSE_ALGO_AUTO's choice
 * by M and layout) and weight layout (packed nonzero: lse_int8_linear_packed and the gate_up
 * entries; 0: lse_int8_linear / _ex) needs: 0 when the chosen kernel uses none (the decode
 * kernel, the GEMV), lse_int8_linear_workspace(M, K, N) otherwise. */
size_t lse_int8_linear_workspace_for(int64_t M, int64_t K, int64_t N, int algo, int packed);

/*
 * Symmetric per-output-channel quantization at load time (the build's replacement for the
 * reference's raise at model_runner.py:45-46):
 *   s[n] = max_k |w[n,k]| / 127   (1.0 for an all-zero row)
 *   q[n,k] = clamp(rint(w[n,k] / s[n]), -127, 127)      (fp32 arithmetic, half-to-even)
 *   w      [N, K] in `dtype` (lse_dtype), row stride ldw elements, any alignment
 *   q_out  int8 [N, K] row-major;  s_out fp32 [N]
 */
int lse_int8_quantize(const void *w, int dtype, int64_t N, int64_t K, int64_t ldw,
                      int8_t *q_out, float *s_out, void *stream);

/* Human-readable name of a status code (static string). */
const char *lse_status_string(int status);

/* Text of the last CUDA error this thread saw inside the library ("" if none). */
const char *lse_last_cuda_error(void);

/*
 * Device-side status of `device`: LSE_OK, or LSE_ERR_DEVICE_TIMEOUT when a bounded
 * wait inside a kernel gave up since the last reset.  Synchronizes the device.  When
 * `reset` is nonzero the flag is cleared.  After a timeout the decode-attention workspace
 * (lse_paged_decode_attention) must be zeroed again before its next use; the linear
 * workspaces need nothing.
 */
int lse_device_status(int device, int reset);

/*
 * lse_paged_attention -- replaces the reference's paged_attention_forward /
 * paged_attention_2 (src/llm_serving_engine/kernels/flash_attention.py:202-332) for any number
 * of query tokens per batch entry: prefill chunks and mixed prefill + decode batches, as
 * ModelRunner.attend_paged (src/llm_serving_engine/model/model_runner.py:357-363) calls it.
 *
 *   q        [H, tokens, D] of `dtype` (LSE_BF16 or LSE_F16), element (h, t, d) at
 *            q[h * q_stride_h + t * q_stride_m + d]; even strides, 16-byte aligned
 *   k_pool, v_pool  [num_blocks, block_size, H_kv, D] of `dtype`, contiguous, holding this
 *            call's new tokens already
 *   block_table int32 [E, >= ceil(context_len / block_size)], row stride bt_stride
 *   context_len, query_offset, q_start, q_len  int32 [E]: entry e's queries are rows
 *            q_start[e] .. q_start[e] + q_len[e] - 1 of q, row i at position
 *            query_offset[e] + i, attending to positions p < context_len[e] with
 *            p <= query_offset[e] + i
 *   max_q_len  >= every q_len[e] (sizes the launch)
 *   o        [H, tokens, D] of `dtype`, element (h, t, d) at o[h * o_stride_h + t * o_stride_m + d];
 *            rows of no entry are not written
 * D = 64 or 128, H / H_kv in {1, 2, 4, 8} (LSE_ERR_UNSUPPORTED otherwise).  fp32 scores and
 * accumulation, P rounded to `dtype` before P V (as the reference), one rounding of o.  A block
 * id outside [0, num_blocks) is not read and is reported as LSE_ERR_INVALID_ARG by
 * lse_device_status.  No workspace.
 */
int lse_paged_attention(const void *q, int dtype, int64_t H, int64_t D, int64_t q_stride_h, int64_t q_stride_m,
                        const void *k_pool, const void *v_pool, int64_t num_blocks, int64_t block_size, int64_t H_kv,
                        const int32_t *block_table, int64_t bt_stride, const int32_t *context_len,
                        const int32_t *query_offset, const int32_t *q_start, const int32_t *q_len, int64_t E,
                        int64_t max_q_len, float scale, void *o, int64_t o_stride_h, int64_t o_stride_m, void *stream);

/*
 * Wait limit of the tensor-core kernels on `device`, in SM clock cycles: a bounded mbarrier wait
 * for data (a copy, an MMA, a stage) that has not completed after this many cycles raises the
 * CTA's abort flag and records LSE_ERR_DEVICE_TIMEOUT (lse_device_status); the CTA then drains
 * its own copies and MMAs under the default limit, frees its tensor memory and returns, and the
 * next call starts clean.  cycles <= 0 restores the default (4e9 cycles, ~2 s).  Takes effect
 * for launches after the call; meant for tests of the timeout path (a limit of 1 cycle makes
 * every data wait of a tensor-core launch give up).
 */
int lse_set_wait_limit(int device, long long cycles);

/*
 * lse_int8_linear_packed_noalloc -- no counterpart in the reference: an addition of this
 * library for callers that cannot allocate a workspace.
 *
 * Same result as lse_int8_linear_packed(..., LSE_ALGO_TCGEN05, ...), without the workspace
 * arguments: the tensor-core path's scratch (stream-K arrival counters, partial tiles, the
 * activation digit planes and row scales) is a fixed array of LSE_NOALLOC_SCRATCH_BYTES
 * (16 MiB) per device, a static device
 * variable of this library, so the call allocates nothing, neither device nor host memory.
 * Who needs it: a binding that mirrors the engine's nn.Linear call (x, W, s -> y) has no
 * workspace to pass and often no device allocator of its own (a plain C, ctypes or cgo
 * host holding raw pointers another framework owns); and the engine hands about 95% of the
 * HBM that is free after loading to its KV-cache pool (src/llm_serving_engine/config.py:
 * 52-87), so a workspace allocated at the first projection call can find no memory.
 *
 *   x, w_packed, scale, y, strides: as lse_int8_linear_packed.
 *   M: 1 .. LSE_NOALLOC_MAX_M (64) tokens -- the largest token tile whose partial tiles fit
 *      the fixed array.  A larger M returns LSE_ERR_WORKSPACE before touching the GPU, with
 *      the limit in lse_last_cuda_error(); use lse_int8_linear_packed with a workspace.
 *      K: the digit planes take 3 * M * K bytes, so at M = 64 K up to about 36,000 fits on
 *      a 148-SM GPU (every Llama-3 8B and 70B projection); a larger need also returns
 *      LSE_ERR_WORKSPACE.  M == 0 or N == 0 is a no-op; K == 0 writes zeros.
 *
 * Every call on a device shares the one array, and the array keeps the last call's
 * contents.  Calls that overlap on the GPU (different streams with no ordering between
 * them) race on it and give wrong results: order them on one stream or with events.  Each
 * call's first kernel (the activation split) clears the arrival counters the call uses, so a
 * call never depends on an earlier one having finished cleanly.  The first
 * call on a device does the set-up (lse_init's work plus looking up the array's device
 * address) and should come before any stream capture.
 *
 * "Allocates nothing" is per call: the 16 MiB array itself is device memory, reserved when
 * this library's module loads on the device.  With CUDA's lazy module loading (the default)
 * that happens at lse_init or at the first entry-point call on that device.  A host that
 * sizes a memory pool from the free memory it sees (the engine's KV pool) must therefore call
 * lse_init(device) before sizing it; otherwise the module load can find no memory and the
 * call returns LSE_ERR_CUDA.
 */
#define LSE_NOALLOC_SCRATCH_BYTES 16777216
#define LSE_NOALLOC_MAX_M 64
int lse_int8_linear_packed_noalloc(const void *x, int64_t M, int64_t K, int64_t ldx,
                                   const int8_t *w_packed, const float *scale, int64_t N,
                                   void *y, int64_t ldy, void *stream);

/* Library ABI version (LSE_ABI_VERSION). */
#define LSE_ABI_VERSION 1
int lse_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* LSE_INT8_H */
