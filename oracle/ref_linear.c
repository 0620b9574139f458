/*
 * Plain-C restatement of the int8 weight-only linear (test infrastructure only: the
 * checker, never the shipped path).  Torch- and BLAS-free so the Python oracle's
 * arithmetic is pinned independently of any library.
 *
 * The reference engine has no int8 linear (src/llm_serving_engine/model/model_runner.py:45-46
 * raises NotImplementedError); its projections are nn.Linear (model_runner.py:322-324, 369,
 * 223) with y = x W^T, weight [out, in], no bias.  The int8 layer stores W ~= q * s[n], so
 *
 *     y[m, n] = sum_k x[m, k] * (q[n, k] * s[n])        (double accumulation)
 *
 * Quantization restates the symmetric per-output-channel rule in float32, step for step as
 * the CUDA kernel computes it: s = amax / 127 (1.0 for an all-zero row),
 * q = clamp(rint(w / s), -127, 127) with round-half-to-even.
 *
 * Built by oracle/Makefile into oracle/_build/liboracle.so.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* x: float32 [M, ldx] row-major (bf16 values widened by the caller), q: int8 [N, K],
 * s: float32 [N]; y: float64 [M, N]. */
void oracle_int8_linear_f64(const float *x, int64_t M, int64_t K, int64_t ldx,
                            const int8_t *q, const float *s, int64_t N, double *y) {
    for (int64_t m = 0; m < M; ++m) {
        const float *xr = x + m * ldx;
        for (int64_t n = 0; n < N; ++n) {
            const int8_t *wr = q + n * K;
            double acc = 0.0;
            for (int64_t k = 0; k < K; ++k) acc += (double)xr[k] * ((double)wr[k] * (double)s[n]);
            y[m * N + n] = acc;
        }
    }
}

/* w: float32 [N, K] -> q int8 [N, K], s float32 [N]. */
void oracle_quantize_f32(const float *w, int64_t N, int64_t K, int8_t *q, float *s) {
    for (int64_t n = 0; n < N; ++n) {
        const float *wr = w + n * K;
        float amax = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            float a = fabsf(wr[k]);
            if (a > amax) amax = a;
        }
        volatile float sc = amax / 127.0f; /* volatile: keep the fp32 rounding step */
        float scale = sc > 0.0f ? sc : 1.0f;
        s[n] = scale;
        for (int64_t k = 0; k < K; ++k) {
            volatile float r = wr[k] / scale;
            float v = rintf(r);
            if (v > 127.0f) v = 127.0f;
            if (v < -127.0f) v = -127.0f;
            q[n * K + k] = (int8_t)v;
        }
    }
}

/* bf16 bits -> float32, exact. */
void oracle_bf16_to_f32(const uint16_t *in, int64_t n, float *out) {
    for (int64_t i = 0; i < n; ++i) {
        uint32_t u = (uint32_t)in[i] << 16;
        memcpy(&out[i], &u, sizeof(u));
    }
}
