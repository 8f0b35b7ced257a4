/*
 * TEST INFRASTRUCTURE ONLY -- the CPU checker for the 4-bit qGEMM, never the product path.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference arm
 * may load the library built from this file.
 *
 * A plain-C restatement of the arithmetic the reference's Metal qmv kernels perform
 * (IronMule ironmule/qmv_k3840.py:62-244, ironmule/qmv_shared.py:66-138,
 * ironmule/qmv_fast_shared.py:30-131, all transcribed there from MLX 0.32.0 quantized.h),
 * generalised to M activation rows. MLX computes every activation row separately
 * (the row index is the grid's x coordinate, qmv_k3840.py:175-176), so a row's result does not
 * depend on M.
 *
 * Weight format (MLX affine, bits=4, group 64): w uint32 [N, K/8], eight nibbles per word, low
 * nibble first; scales and biases bf16 [N, K/64]; dequantised w = scale * q + bias.
 *
 * Per output (m, n), per SIMD lane l (32 lanes), per block b of VPT*32 values:
 *   xs       = x[m, b*BLOCK + l*VPT ...]                          (VPT = 8 or 16 values)
 *   sum      = sum over 4-chunks of (x0 + x1 + x2 + x3)            (load_vector, :66-76)
 *   xt[i]    = x[i] / {1, 16, 256, 4096}[i % 4]                    (pre-scaled for masked nibbles)
 *   accum    = sum_i over uint16 words of (xt0*(u&0xf) + xt1*(u&0xf0) + xt2*(u&0xf00) + xt3*(u&0xf000))
 *   result  += scale[g] * accum + sum * bias[g]                   (qdot, :93-109)
 * with g = the group of the lane's values, then a 32-lane reduction (simd_sum) and one bf16 cast.
 *
 * Two points the Metal source does not settle on this machine are fixed here and named:
 *  - the 4-term partial sums in load_vector add bf16 operands; MLX's bfloat type may round each
 *    partial to bf16. FOUR_TERM_ROUNDS_BF16=0 (default) keeps them in f32, =1 rounds each add to
 *    bf16. Both are exported; they differ only in the sum*bias term, well inside bf16 tolerance.
 *  - simd_sum's hardware order is unspecified; this file reduces with an xor butterfly
 *    (16, 8, 4, 2, 1), the usual SIMD-group tree.
 * All float operations are separate IEEE single operations in source order (no FMA
 * contraction: build with -ffp-contract=off).
 */
#include <stdint.h>
#include <string.h>
#include <math.h>

static inline float bf16_to_f32(uint16_t h) {
    uint32_t u = ((uint32_t)h) << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
    u += 0x7fffu + ((u >> 16) & 1u);                                       /* round to nearest even */
    return (uint16_t)(u >> 16);
}

static inline float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

/* One lane's contribution for one block, VPT in {8, 16}. `xs` points at the lane's first value,
 * `wb` at the lane's first weight byte, s/b are the group's scale and bias. */
static inline float lane_block(const uint16_t* xs, const uint8_t* wb, float s, float b, int vpt,
                               int nvalid, int bf16_partials) {
    float xt[16];
    float sum = 0.0f;
    for (int i = 0; i < nvalid; i += 4) {
        float x0 = bf16_to_f32(xs[i]), x1 = bf16_to_f32(xs[i + 1]);
        float x2 = bf16_to_f32(xs[i + 2]), x3 = bf16_to_f32(xs[i + 3]);
        float part;
        if (bf16_partials) {
            part = round_bf16(round_bf16(round_bf16(x0 + x1) + x2) + x3);
        } else {
            part = ((x0 + x1) + x2) + x3;
        }
        sum = sum + part;
        xt[i] = x0;
        xt[i + 1] = x1 / 16.0f;
        xt[i + 2] = x2 / 256.0f;
        xt[i + 3] = x3 / 4096.0f;
    }
    for (int i = nvalid; i < vpt; i++) xt[i] = 0.0f;
    float accum = 0.0f;
    for (int i = 0; i < nvalid / 4; i++) {
        uint32_t u = (uint32_t)wb[2 * i] | ((uint32_t)wb[2 * i + 1] << 8);
        float t0 = xt[4 * i] * (float)(u & 0x000fu);
        float t1 = xt[4 * i + 1] * (float)(u & 0x00f0u);
        float t2 = xt[4 * i + 2] * (float)(u & 0x0f00u);
        float t3 = xt[4 * i + 3] * (float)(u & 0xf000u);
        accum = accum + (((t0 + t1) + t2) + t3);
    }
    float a = s * accum;
    float c = sum * b;
    return a + c;
}

/* y[m, n] for one (m, n): the 32 lanes' block loops, then the butterfly reduction. */
static uint16_t qmv_one(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                        const uint16_t* xrow, int64_t n, int64_t K, int vpt, int bf16_partials) {
    const int block = vpt * 32;
    const int64_t kg = K / 64;
    const uint8_t* wrow = (const uint8_t*)(w + n * (K / 8));
    const uint16_t* srow = scales + n * kg;
    const uint16_t* brow = biases + n * kg;
    float res[32];
    for (int l = 0; l < 32; l++) {
        float r = 0.0f;
        for (int64_t k0 = 0; k0 < K; k0 += block) {
            int64_t first = k0 + (int64_t)l * vpt;
            int64_t rem = K - first;
            if (rem <= 0) continue;
            int nvalid = rem >= vpt ? vpt : (int)rem;
            int64_t g = first / 64;
            float s = bf16_to_f32(srow[g]);
            float b = bf16_to_f32(brow[g]);
            r = r + lane_block(xrow + first, wrow + first / 2, s, b, vpt, nvalid, bf16_partials);
        }
        res[l] = r;
    }
    for (int off = 16; off > 0; off >>= 1) {
        float nxt[32];
        for (int l = 0; l < 32; l++) nxt[l] = res[l] + res[l ^ off];
        memcpy(res, nxt, sizeof(res));
    }
    return f32_to_bf16(res[0]);
}

/*
 * y[M, N] = x[M, K] . deq(w)[N, K]^T in the reference's arithmetic.
 * vpt = 8: qmv_impl (qmv_k3840 / qmv_shared / qmv_variant); any K that is a multiple of 64.
 * vpt = 16: qmv_fast_impl (qmv_fast_shared); K a multiple of 512.
 * Returns 0, or -1 for a shape the chosen arithmetic does not cover.
 */
int oracle_qmv_w4g64(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                     const uint16_t* x, uint16_t* y, int64_t M, int64_t N, int64_t K, int vpt,
                     int bf16_partials) {
    if (M < 0 || N < 0 || K <= 0 || K % 64) return -1;
    if (vpt != 8 && vpt != 16) return -1;
    if (vpt == 16 && K % 512) return -1;
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t m = 0; m < M; m++) {
        for (int64_t n = 0; n < N; n++) {
            y[m * N + n] = qmv_one(w, scales, biases, x + m * K, n, K, vpt, bf16_partials);
        }
    }
    return 0;
}

/* Dequantised float32 reference: out[M, N] = sum_k x * (scale*q + bias), accumulated in double.
 * The tolerance reference used beside the order-exact restatement above. */
int oracle_qmm_f64(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                   const uint16_t* x, float* out, int64_t M, int64_t N, int64_t K) {
    if (K % 64) return -1;
#pragma omp parallel for schedule(static) collapse(2)
    for (int64_t m = 0; m < M; m++) {
        for (int64_t n = 0; n < N; n++) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; k++) {
                uint32_t word = w[n * (K / 8) + k / 8];
                uint32_t q = (word >> (4 * (k % 8))) & 0xfu;
                double s = bf16_to_f32(scales[n * (K / 64) + k / 64]);
                double b = bf16_to_f32(biases[n * (K / 64) + k / 64]);
                acc += (s * (double)q + b) * (double)bf16_to_f32(x[m * K + k]);
            }
            out[m * N + n] = (float)acc;
        }
    }
    return 0;
}

/* The CPU baseline's qGEMM (test infrastructure and timed baseline only): per output row, dequantise one
 * group of 64 weights to float32 (scale*q + bias) and dot it with every activation row, accumulating in
 * float32 (SIMD partial sums); one bf16 cast per output. The usual CPU formulation of the reference's
 * quantized matmul (mx.quantized_matmul on the CPU, ironmule/qmv_k3840.py:336-339). */
#include <stdlib.h>
int oracle_qmm_fast(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const uint16_t* x,
                    uint16_t* y, int64_t M, int64_t N, int64_t K) {
    if (K % 64 || M < 1 || M > 64) return -1;
    const int64_t G = K / 64;
    float* xf = (float*)malloc(sizeof(float) * (size_t)(M * K));
    if (!xf) return -1;
    for (int64_t i = 0; i < M * K; i++) xf[i] = bf16_to_f32(x[i]);
#pragma omp parallel for schedule(static)
    for (int64_t n = 0; n < N; n++) {
        float acc[64];
        float wf[64];
        for (int64_t m = 0; m < M; m++) acc[m] = 0.0f;
        for (int64_t g = 0; g < G; g++) {
            const float s = bf16_to_f32(scales[n * G + g]);
            const float b = bf16_to_f32(biases[n * G + g]);
            const uint32_t* wp = w + n * (K / 8) + g * 8;
            for (int i = 0; i < 64; i++) wf[i] = s * (float)((wp[i >> 3] >> (4 * (i & 7))) & 0xfu) + b;
            for (int64_t m = 0; m < M; m++) {
                const float* xp = xf + m * K + g * 64;
                float part = 0.0f;
#pragma omp simd reduction(+ : part)
                for (int i = 0; i < 64; i++) part += wf[i] * xp[i];
                acc[m] += part;
            }
        }
        for (int64_t m = 0; m < M; m++) y[m * N + n] = f32_to_bf16(acc[m]);
    }
    free(xf);
    return 0;
}
