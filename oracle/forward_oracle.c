/*
 * CPU oracle for the compiled forward pass -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the arithmetic that ForgeTune's generated
 * C++ forward pass performs for each fused node, in the same operation order,
 * so that its results are bit-identical to the reference runtime built with
 * `g++ -O2 -fno-signed-zeros` on x86-64 (no FMA contraction).  It is compiled
 * with -ffp-contract=off for the same reason.  Only the test-suite, the smoke
 * check and the CPU-baseline leg of the benchmark may load it; the product
 * path never does.
 *
 * Weight layout follows the reference IR: Linear weights pre-transposed to
 * W[K,N] row-major (python/forgetune/export_frontend.py:246-257), conv weights
 * OIHW, activations row-major / NCHW.
 *
 * There are exactly two accumulation orders in the reference codegen:
 *   bias-first  acc = bias; acc += x*w for k = 0..K-1
 *               (FUSED_MATMUL_ADD_RELU with variant fused_ikj or loop_ikj,
 *                src/codegen.cpp:381-396; every conv, src/codegen.cpp:532-560)
 *   bias-last   acc = 0;    acc += x*w for k = 0..K-1; acc += bias
 *               (naive/tiled fused nodes, src/codegen.cpp:353-380, 397-408;
 *                plain MATMUL followed by the ADD loop, src/codegen.cpp:277-339
 *                and 870-914 -- MATMUL has no fused_ikj emitter and falls back
 *                to the naive loop, src/codegen.cpp:637-648).
 * The C++ interpreter (src/interpreter.cpp:8-33, 463-475) uses bias-last.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORA_EXPORT __attribute__((visibility("default")))

/* ReLU that keeps NaN, as the reference emits it:
 * (std::isnan(v) || v > 0.0f) ? v : 0.0f   (src/codegen.cpp:394, 406, 840). */
static inline float ora_relu1(float v) { return (isnan(v) || v > 0.0f) ? v : 0.0f; }

/* y[M,N] = (relu?)(bias + sum_k x[m,k] w[k,n]) with the bias-first order.
 * bias may be NULL (treated as 0), [N] (bias_rows == 0) or [M,N]
 * (bias_rows != 0, src/codegen.cpp:351). */
ORA_EXPORT void ora_gemm_bias_first(int64_t M, int64_t K, int64_t N,
                                    const float* x, const float* w,
                                    const float* bias, int bias_rows, int relu,
                                    float* y) {
    for (int64_t i = 0; i < M; ++i) {
        float* yr = y + i * N;
        for (int64_t j = 0; j < N; ++j)
            yr[j] = bias ? (bias_rows ? bias[i * N + j] : bias[j]) : 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            const float a = x[i * K + k];
            const float* wr = w + k * N;
            for (int64_t j = 0; j < N; ++j) yr[j] += a * wr[j];
        }
        if (relu)
            for (int64_t j = 0; j < N; ++j) yr[j] = ora_relu1(yr[j]);
    }
}

/* y[M,N] = (relu?)((sum_k x[m,k] w[k,n]) + bias) with the bias-last order.
 * Each output is 0 + x0*w0 + x1*w1 + ... in k order, then + bias: the same
 * rounding sequence as the reference's naive i-j-k loop, evaluated here in
 * i-k-j order so the weight rows stream through the cache. */
ORA_EXPORT void ora_gemm_bias_last(int64_t M, int64_t K, int64_t N,
                                   const float* x, const float* w,
                                   const float* bias, int bias_rows, int relu,
                                   float* y) {
    for (int64_t i = 0; i < M; ++i) {
        float* yr = y + i * N;
        for (int64_t j = 0; j < N; ++j) yr[j] = 0.0f;
        for (int64_t k = 0; k < K; ++k) {
            const float a = x[i * K + k];
            const float* wr = w + k * N;
            for (int64_t j = 0; j < N; ++j) yr[j] += a * wr[j];
        }
        for (int64_t j = 0; j < N; ++j) {
            float sum = yr[j];
            if (bias) sum += bias_rows ? bias[i * N + j] : bias[j];
            yr[j] = relu ? ora_relu1(sum) : sum;
        }
    }
}

/* Same-shape elementwise add, y = a + b (src/codegen.cpp:876-880). */
ORA_EXPORT void ora_add(int64_t n, const float* a, const float* b, float* y) {
    for (int64_t i = 0; i < n; ++i) y[i] = a[i] + b[i];
}

/* Row broadcast add, y[i,j] = a[i,j] + b[j] (src/codegen.cpp:881-898). */
ORA_EXPORT void ora_add_row(int64_t M, int64_t N, const float* a, const float* b, float* y) {
    for (int64_t i = 0; i < M; ++i)
        for (int64_t j = 0; j < N; ++j) y[i * N + j] = a[i * N + j] + b[j];
}

/* Channel broadcast add on NCHW, y[b,c,h,w] = a[b,c,h,w] + bias[c]
 * (src/codegen.cpp:899-913). */
ORA_EXPORT void ora_add_channel(int64_t B, int64_t C, int64_t HW, const float* a,
                                const float* bias, float* y) {
    for (int64_t b = 0; b < B; ++b)
        for (int64_t c = 0; c < C; ++c)
            for (int64_t i = 0; i < HW; ++i) {
                int64_t idx = (b * C + c) * HW + i;
                y[idx] = a[idx] + bias[c];
            }
}

/* Elementwise multiply in the reference's three broadcast forms
 * (src/codegen.cpp:916-958): same shape, row ([N] or [1,N]) and NCHW channel. */
ORA_EXPORT void ora_mul(int64_t n, const float* a, const float* b, float* y) {
    for (int64_t i = 0; i < n; ++i) y[i] = a[i] * b[i];
}

ORA_EXPORT void ora_mul_row(int64_t M, int64_t N, const float* a, const float* b, float* y) {
    for (int64_t i = 0; i < M; ++i)
        for (int64_t j = 0; j < N; ++j) y[i * N + j] = a[i * N + j] * b[j];
}

ORA_EXPORT void ora_mul_channel(int64_t B, int64_t C, int64_t HW, const float* a,
                                const float* scale, float* y) {
    for (int64_t b = 0; b < B; ++b)
        for (int64_t c = 0; c < C; ++c)
            for (int64_t i = 0; i < HW; ++i) {
                int64_t idx = (b * C + c) * HW + i;
                y[idx] = a[idx] * scale[c];
            }
}

/* SIGMOID 1 / (1 + exp(-x)) and TANH with the C library's float functions,
 * the ones std::exp / std::tanh on a float resolve to (src/codegen.cpp:844-859). */
ORA_EXPORT void ora_sigmoid(int64_t n, const float* a, float* y) {
    for (int64_t i = 0; i < n; ++i) y[i] = 1.0f / (1.0f + expf(-a[i]));
}

ORA_EXPORT void ora_tanh(int64_t n, const float* a, float* y) {
    for (int64_t i = 0; i < n; ++i) y[i] = tanhf(a[i]);
}

/* Standalone NaN-keeping ReLU (src/codegen.cpp:835-843). */
ORA_EXPORT void ora_relu(int64_t n, const float* a, float* y) {
    for (int64_t i = 0; i < n; ++i) y[i] = ora_relu1(a[i]);
}

/* Direct NCHW convolution, OIHW weights, groups = 1, bias-first, with the
 * input copied into a zero-padded plane first so padded taps contribute
 * 0*w exactly as the reference does (src/codegen.cpp:412-624).  The
 * accumulation order per output is ci, kh, kw.  Returns 0, or -4 when the
 * padding scratch cannot be allocated (src/codegen.cpp:466-476). */
ORA_EXPORT int ora_conv2d(int64_t B, int64_t Cin, int64_t H, int64_t W,
                          int64_t Cout, int64_t Kh, int64_t Kw,
                          int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                          int64_t dh, int64_t dw,
                          const float* x, const float* wt, const float* bias,
                          int relu, float* y) {
    const int64_t Ho = (H + 2 * ph - (dh * (Kh - 1) + 1)) / sh + 1;
    const int64_t Wo = (W + 2 * pw - (dw * (Kw - 1) + 1)) / sw + 1;
    const int64_t Hp = H + 2 * ph, Wp = W + 2 * pw;
    float* pad = (float*)calloc((size_t)(Cin * Hp * Wp), sizeof(float));
    if (!pad) return -4;
    for (int64_t b = 0; b < B; ++b) {
        const float* xb = x + b * Cin * H * W;
        float* yb = y + b * Cout * Ho * Wo;
        for (int64_t ci = 0; ci < Cin; ++ci)
            for (int64_t h = 0; h < H; ++h)
                memcpy(pad + (ci * Hp + h + ph) * Wp + pw, xb + (ci * H + h) * W,
                       (size_t)W * sizeof(float));
        for (int64_t co = 0; co < Cout; ++co) {
            const float bv = bias ? bias[co] : 0.0f;
            const float* wc = wt + co * Cin * Kh * Kw;
            for (int64_t ho = 0; ho < Ho; ++ho)
                for (int64_t wo = 0; wo < Wo; ++wo) {
                    float acc = bv;
                    for (int64_t ci = 0; ci < Cin; ++ci)
                        for (int64_t kh = 0; kh < Kh; ++kh) {
                            const float* row = pad + (ci * Hp + ho * sh + kh * dh) * Wp;
                            const float* wr = wc + (ci * Kh + kh) * Kw;
                            for (int64_t kw = 0; kw < Kw; ++kw)
                                acc += row[wo * sw + kw * dw] * wr[kw];
                        }
                    yb[(co * Ho + ho) * Wo + wo] = relu ? ora_relu1(acc) : acc;
                }
        }
    }
    free(pad);
    return 0;
}

/* ---------------------------------------------------------------------------
 * Counter-based normal generator used for the wide-MLP input, restated on the
 * host so the oracle can regenerate any sampled row.
 *
 * Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
 * easy as 1, 2, 3", SC'11): 10 rounds of the 4x32 Philox S-box with the
 * published multipliers and Weyl key increments.  Element e of the tensor
 * uses counter (e / 4, 0, 0, 0) ... see philox_normal below: each counter
 * block yields 4 uniforms u0..u3, turned into 4 normals by two Box-Muller
 * transforms (u0,u1) and (u2,u3).
 * ------------------------------------------------------------------------- */
static void philox4x32_10(uint32_t ctr[4], uint32_t k0, uint32_t k1) {
    const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
    const uint32_t W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
    for (int r = 0; r < 10; ++r) {
        uint64_t p0 = (uint64_t)M0 * ctr[0];
        uint64_t p1 = (uint64_t)M1 * ctr[2];
        uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
        uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
        uint32_t n0 = hi1 ^ ctr[1] ^ k0;
        uint32_t n1 = lo1;
        uint32_t n2 = hi0 ^ ctr[3] ^ k1;
        uint32_t n3 = lo0;
        ctr[0] = n0; ctr[1] = n1; ctr[2] = n2; ctr[3] = n3;
        k0 += W0; k1 += W1;
    }
}

/* Raw Philox blocks for blocks [first, first+count): out[4*i + j]. */
ORA_EXPORT void ora_philox_blocks(uint64_t seed, uint64_t first, uint64_t count, uint32_t* out) {
    for (uint64_t i = 0; i < count; ++i) {
        uint64_t c = first + i;
        uint32_t ctr[4] = {(uint32_t)c, (uint32_t)(c >> 32), 0u, 0u};
        philox4x32_10(ctr, (uint32_t)seed, (uint32_t)(seed >> 32));
        memcpy(out + 4 * i, ctr, sizeof(ctr));
    }
}

/* uniform in (0, 1]: (u + 1) * 2^-32 computed in float. */
static inline float ora_u01(uint32_t u) { return ((float)u + 1.0f) * 2.3283064365386963e-10f; }

/* Normal elements [first, first+count) of the stream keyed by seed. */
ORA_EXPORT void ora_philox_normal(uint64_t seed, uint64_t first, uint64_t count, float* out) {
    const float two_pi = 6.2831853071795864769f;
    for (uint64_t e = first; e < first + count; ++e) {
        uint64_t blk = e >> 2;
        uint32_t ctr[4] = {(uint32_t)blk, (uint32_t)(blk >> 32), 0u, 0u};
        philox4x32_10(ctr, (uint32_t)seed, (uint32_t)(seed >> 32));
        int lane = (int)(e & 3);
        int pair = lane >> 1;
        float u1 = ora_u01(ctr[2 * pair]);
        float u2 = ora_u01(ctr[2 * pair + 1]);
        float r = sqrtf(-2.0f * logf(u1));
        float t = two_pi * u2;
        out[e - first] = (lane & 1) ? r * sinf(t) : r * cosf(t);
    }
}
