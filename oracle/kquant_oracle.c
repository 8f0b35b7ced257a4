/*
 * TEST INFRASTRUCTURE ONLY: the CPU checker for the GGUF k-quant matmul (ironmule_b200/csrc/kquant.cu). Nothing in the
 * product links or calls it.
 *
 * Restates, in plain C:
 *   - ggml's Q4_K and Q6_K block formats and their float32 dequantization (the formats the reference's generated
 *     kernels read, ironmule/kernel_gen.py:68-97 and :429-460; the reference's own float64 checkers ref64 / ref64_q6,
 *     kernel_gen.py:565-652, decode them element by element the same way);
 *   - the activation rounding to 8 bits per 32 values (kernel_gen.py:86-97: d = amax / 127, q = round(x / d));
 *   - the device kernel's arithmetic in its exact operation order: exact integer sub-block dot products, then per
 *     sub-block fp32 fmas into per-lane accumulators, summed as a fixed pairwise tree -- so the device results must
 *     equal these bit for bit;
 *   - a float64 reference (weights dequantized in double, activations unrounded) for error bounds.
 * Built with -ffp-contract=off so that only the fmaf calls written here fuse.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define Q4K 12
#define Q6K 14

/* IEEE half -> single, exact (normal, subnormal, zero, inf, nan). */
static float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t exp = (h >> 10) & 0x1F, man = h & 0x3FF;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: value = man * 2^-24 */
      float v = (float)man * 5.9604644775390625e-08f;
      memcpy(&bits, &v, 4);
      bits |= sign;
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Q4_K sub-block j's 6-bit scale and min from the 12 packed bytes s[] (ggml's get_scale_min_k4). */
static void q4k_scale_min(const uint8_t* s, int j, int* sc, int* m) {
  if (j < 4) {
    *sc = s[j] & 63;
    *m = s[j + 4] & 63;
  } else {
    *sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
    *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

/* Q4_K quant (0..15) of weight i (0..255) of a block: sub-block i / 32, byte 32 (i / 64) + i % 32. */
static int q4k_q(const uint8_t* blk, int i) {
  const uint8_t b = blk[16 + 32 * (i / 64) + (i % 32)];
  return ((i / 32) & 1) ? (b >> 4) : (b & 0xF);
}

/* Q6_K quant (-32..31) of weight i of a block; its scale is scales[i / 16]. */
static int q6k_q(const uint8_t* blk, int i) {
  const int h = i / 128, r = i % 128, quarter = r / 32, l = r % 32;
  const uint8_t* ql = blk + 64 * h;
  const uint8_t qh = blk[128 + 32 * h + l];
  int lo;
  switch (quarter) {
    case 0: lo = ql[l] & 0xF; break;
    case 1: lo = ql[l + 32] & 0xF; break;
    case 2: lo = ql[l] >> 4; break;
    default: lo = ql[l + 32] >> 4; break;
  }
  return (lo | (((qh >> (2 * quarter)) & 3) << 4)) - 32;
}

static int block_bytes(int type) { return type == Q4K ? 144 : 210; }

/* ggml's float32 dequantization of `nblocks` consecutive blocks. */
void kq_dequant(int type, const uint8_t* blocks, int64_t nblocks, float* out) {
  for (int64_t b = 0; b < nblocks; b++) {
    const uint8_t* blk = blocks + b * block_bytes(type);
    if (type == Q4K) {
      const float d = f16_to_f32(rd16(blk)), dmin = f16_to_f32(rd16(blk + 2));
      for (int i = 0; i < 256; i++) {
        int sc, m;
        q4k_scale_min(blk + 4, i / 32, &sc, &m);
        const float d1 = d * (float)sc, m1 = dmin * (float)m;
        out[b * 256 + i] = d1 * (float)q4k_q(blk, i) - m1;
      }
    } else {
      const float d = f16_to_f32(rd16(blk + 208));
      for (int i = 0; i < 256; i++) {
        const int8_t sc = (int8_t)blk[192 + i / 16];
        out[b * 256 + i] = d * (float)sc * (float)q6k_q(blk, i);
      }
    }
  }
}

/* Activations to 8 bits per 32 values: dx = amax / 127, xq = round-half-even(x / dx), xs = sum of xq. */
void kq_quantize_x(const float* x, int64_t n, int8_t* xq, float* dx, int32_t* xs) {
  for (int64_t b = 0; b < n / 32; b++) {
    float a = 0.0f;
    for (int i = 0; i < 32; i++) a = fmaxf(a, fabsf(x[b * 32 + i]));
    const float d = a / 127.0f;
    int32_t s = 0;
    for (int i = 0; i < 32; i++) {
      const int q = d == 0.0f ? 0 : (int)nearbyintf(x[b * 32 + i] / d);
      xq[b * 32 + i] = (int8_t)q;
      s += q;
    }
    dx[b] = d;
    xs[b] = s;
  }
}

/* The fixed pairwise tree the kernel's shuffles form: level by level over the index bits, a[i] + a[i + bit]. */
static float tree(float* a, int n) {
  for (int bit = 1; bit < n; bit <<= 1)
    for (int i = 0; i < n; i += 2 * bit) a[i] = a[i] + a[i + bit];
  return a[0];
}

/* The device kernel's result for rows [0, N) and tokens [0, B): xq/dx/xs from kq_quantize_x of x [B][K]. A warp
 * takes blocks ib = 4 it + j; Q4_K keeps accumulator 4 j + c (chunk c: sub-blocks 2c then 2c + 1), Q6_K accumulator
 * 8 j + 4 h + 2 p + hf (sub-block s = 8h + 2p + hf, then s + 4); each runs over its blocks in order. */
void kq_gemv(int type, const uint8_t* w, int64_t N, int64_t K, const int8_t* xq, const float* dx, const int32_t* xs,
             int64_t B, float* y) {
  const int64_t nb = K / 256, S = K / 32;
  for (int64_t t = 0; t < B; t++) {
    const int8_t* xt = xq + t * K;
    for (int64_t n = 0; n < N; n++) {
      float acc[32];
      for (int i = 0; i < 32; i++) acc[i] = 0.0f;
      for (int64_t ib = 0; ib < nb; ib++) {
        const int j = (int)(ib & 3);
        const uint8_t* blk = w + (n * nb + ib) * block_bytes(type);
        const int8_t* xb = xt + ib * 256;
        if (type == Q4K) {
          const float d = f16_to_f32(rd16(blk)), dmin = f16_to_f32(rd16(blk + 2));
          for (int c = 0; c < 4; c++) {
            for (int sb = 2 * c; sb <= 2 * c + 1; sb++) {
              int32_t isum = 0;
              for (int i = 0; i < 32; i++) isum += q4k_q(blk, 32 * sb + i) * xb[32 * sb + i];
              int sc, m;
              q4k_scale_min(blk + 4, sb, &sc, &m);
              const float dsc = d * (float)sc, dm = dmin * (float)m;
              const int64_t xo = t * S + ib * 8 + sb;
              const float v = fmaf(dsc, (float)isum, -(dm * (float)xs[xo]));
              acc[4 * j + c] = fmaf(v, dx[xo], acc[4 * j + c]);
            }
          }
        } else {
          const float d = f16_to_f32(rd16(blk + 208));
          for (int g = 0; g < 8; g++) {
            const int h = g >> 2, p = (g >> 1) & 1, hf = g & 1;
            const int s_lo = 8 * h + 2 * p + hf;
            for (int half = 0; half < 2; half++) {
              const int s = s_lo + 4 * half;
              int32_t isum = 0;
              for (int i = 0; i < 16; i++) isum += q6k_q(blk, 16 * s + i) * xb[16 * s + i];
              const float dsc = d * (float)(int8_t)blk[192 + s];
              const int64_t xo = t * S + ib * 8 + 4 * h + p + 2 * half;
              acc[8 * j + g] = fmaf(dsc * (float)isum, dx[xo], acc[8 * j + g]);
            }
          }
        }
      }
      y[t * N + n] = tree(acc, type == Q4K ? 16 : 32);
    }
  }
}

/* float64: weights dequantized in double (exact), activations as given, dot products in double. */
void kq_ref64(int type, const uint8_t* w, int64_t N, int64_t K, const double* x, int64_t B, double* y) {
  const int64_t nb = K / 256;
  for (int64_t n = 0; n < N; n++) {
    for (int64_t t = 0; t < B; t++) y[t * N + n] = 0.0;
    for (int64_t ib = 0; ib < nb; ib++) {
      const uint8_t* blk = w + (n * nb + ib) * block_bytes(type);
      for (int i = 0; i < 256; i++) {
        double wv;
        if (type == Q4K) {
          int sc, m;
          q4k_scale_min(blk + 4, i / 32, &sc, &m);
          wv = (double)f16_to_f32(rd16(blk)) * sc * q4k_q(blk, i) - (double)f16_to_f32(rd16(blk + 2)) * m;
        } else {
          wv = (double)f16_to_f32(rd16(blk + 208)) * (int8_t)blk[192 + i / 16] * q6k_q(blk, i);
        }
        for (int64_t t = 0; t < B; t++) y[t * N + n] += wv * x[t * K + ib * 256 + i];
      }
    }
  }
}
