// GGUF k-quant matmul for 1-32 tokens: y[B][N] = x[B][K] . W^T with W in llama.cpp's Q4_K (type 12) or Q6_K (type 14)
// blocks, the job of the reference's generated kernels behind its llama.cpp hook `ironmule_kg_mul_mat`
// (ironmule/kernel_gen.py:58-862).
//
// Block formats (ggml's, 256 weights per block):
//   Q4_K, 144 B: f16 d, f16 dmin, 12 bytes of packed 6-bit (scale, min) for 8 sub-blocks of 32, 128 bytes of 4-bit
//     quants: chunk c (64 weights) = bytes 32c..32c+31, low nibbles sub-block 2c, high nibbles sub-block 2c+1;
//     w = d * sc * q - dmin * m.
//   Q6_K, 210 B: ql[128] (low 4 bits), qh[64] (high 2 bits), int8 scales[16] (16 sub-blocks of 16), f16 d;
//     half h (128 weights) uses ql[64h..], qh[32h..], scales[8h..]; w = d * sc * (q - 32).
//
// Arithmetic, as llama.cpp's own quantized matmuls do it: the activations are rounded to 8 bits per 32 values
// (dx = amax / 127, xq = round(x / dx), xs = sum of xq) by kq_quant_kernel; each sub-block's integer dot product
// sum(q * xq) is exact (dp4a, then integer shuffles); then per sub-block, in fp32 with the operation order below:
//   Q4_K: v = fma(d*sc, isum, -(dmin*m * xs)); acc = fma(v, dx, acc)
//   Q6_K: v = (d*sc) * isum;                   acc = fma(v, dx, acc)
// A row's accumulators are per lane (Q4_K: lane 8j + 2c for chunk c of the blocks ib = j mod 4, sub-blocks 2c then
// 2c + 1; Q6_K: every lane, sub-block s then s + 4), each over its blocks in order, then summed as a fixed pairwise tree
// over the lane index. So results are bit-exact against the CPU restatement in the oracle and independent of B and
// of the other tokens.
//
// Layout of a launch: one warp per output row over all of K (8 rows per 256-thread CTA); a warp takes 4 consecutive
// blocks per iteration, each lane 16 bytes of quants, with KQ_DEPTH iterations in flight in registers and the rest of
// the row asked into L2 up front.
#include <cuda_fp16.h>

#include <mutex>

#include "common.cuh"

namespace im {

constexpr int KQ_Q4K = 12, KQ_Q6K = 14;
constexpr int KQ_WARPS = 8;
constexpr int KQ_MAX_TOKENS = 32;

__host__ __device__ constexpr size_t kq_round(size_t v) { return (v + 255) & ~(size_t)255; }

// workspace: xq [B][K] int8, dx [B][K/32] float, xs [B][K/32] int32
static size_t kq_ws_bytes(int64_t K, int64_t B) {
  return kq_round((size_t)B * K) + 2 * kq_round((size_t)B * (K / 32) * 4);
}

__device__ __forceinline__ float kq_half(uint32_t bits16) { return __half2float(__ushort_as_half((unsigned short)bits16)); }

// x [B][K] float -> 8-bit values per 32, one warp per 32 values
__global__ void __launch_bounds__(256) kq_quant_kernel(const float* __restrict__ x, int8_t* __restrict__ xq,
                                                       float* __restrict__ dx, int* __restrict__ xs, int blocks) {
  pdl_wait();
  pdl_trigger();
  const int blk = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (blk >= blocks) return;
  const float v = x[(size_t)blk * 32 + lane];
  float a = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  const float d = __fdiv_rn(a, 127.0f);
  const int q = d == 0.0f ? 0 : __float2int_rn(__fdiv_rn(v, d));
  int s = q;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  xq[(size_t)blk * 32 + lane] = (int8_t)q;
  if (lane == 0) {
    dx[blk] = d;
    xs[blk] = s;
  }
}

// 6-bit scale and min of Q4_K sub-block j from the 12 packed bytes (b0..b11 = s[0..11])
__device__ __forceinline__ uint32_t kq_byte(uint32_t s0, uint32_t s1, uint32_t s2, int k) {
  const uint32_t word = k < 4 ? s0 : (k < 8 ? s1 : s2);
  return (word >> (8 * (k & 3))) & 0xFFu;
}
__device__ __forceinline__ void kq_scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j, int& sc, int& m) {
  if (j < 4) {
    sc = (int)(kq_byte(s0, s1, s2, j) & 63u);
    m = (int)(kq_byte(s0, s1, s2, j + 4) & 63u);
  } else {
    sc = (int)((kq_byte(s0, s1, s2, j + 4) & 0xFu) | ((kq_byte(s0, s1, s2, j - 4) >> 6) << 4));
    m = (int)((kq_byte(s0, s1, s2, j + 4) >> 4) | ((kq_byte(s0, s1, s2, j) >> 6) << 4));
  }
}

constexpr int KQ_DEPTH = 2;  // warp iterations (4 blocks each) in flight per warp (register ring)

// Asks the TMA unit to bring the 16-byte-aligned interior of [p, p + bytes) into L2 (nothing waits on it); the
// interior never reaches outside the range.
__device__ __forceinline__ void kq_prefetch_row(const unsigned char* p, size_t bytes) {
  const uintptr_t a = (reinterpret_cast<uintptr_t>(p) + 15) & ~(uintptr_t)15;
  const uintptr_t e = (reinterpret_cast<uintptr_t>(p) + bytes) & ~(uintptr_t)15;
  for (uintptr_t q = a; q < e; q += 16384) {
    const uint32_t n = (uint32_t)((e - q) < 16384 ? (e - q) : 16384);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(q), "r"(n) : "memory");
  }
}

__device__ __forceinline__ int kq_dot16(uint4 w, uint4 x) {
  int s = __dp4a((int)w.x, (int)x.x, 0);
  s = __dp4a((int)w.y, (int)x.y, s);
  s = __dp4a((int)w.z, (int)x.z, s);
  return __dp4a((int)w.w, (int)x.w, s);
}

// The 32 lanes' accumulators summed as a fixed pairwise tree over lane-index bits `from`..4 (lane 0 gets the sum).
__device__ __forceinline__ float kq_tree(float v, int from) {
  for (int o = 1 << from; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Q4_K: a warp takes 4 blocks of its row per iteration (ib = 4 it + j); lane 8j + 2c + hf reads quant bytes
// 32c + 16hf .. + 15 of block ib: low nibbles = weights 64c + 16hf + i (sub-block 2c), high = weights 64c + 32 + 16hf
// + i (sub-block 2c + 1). The two lanes of a chunk add their integer sums; lane 8j + 2c keeps accumulator (j, c).
template <int BT>
__global__ void __launch_bounds__(KQ_WARPS * 32) kq_q4k_kernel(const unsigned char* __restrict__ w,
                                                               const int8_t* __restrict__ xq,
                                                               const float* __restrict__ dx,
                                                               const int* __restrict__ xs, float* __restrict__ y,
                                                               int N, int K, int B) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * KQ_WARPS + warp;
  const int j = lane >> 3, c = (lane >> 1) & 3, hf = lane & 1;
  const int nb = K >> 8, S = K >> 5, nit = (nb + 3) >> 2;
  const bool live = row < N;
  const unsigned char* rp = w + (size_t)(live ? row : 0) * nb * 144;
  uint4 qv[KQ_DEPTH], hv[KQ_DEPTH];
  // the first iterations' bytes before the dependency wait (weights are never written by an earlier kernel)
  if (live) {
    if (lane == 0 && nb > 4 * KQ_DEPTH) kq_prefetch_row(rp + 4 * KQ_DEPTH * 144, (size_t)(nb - 4 * KQ_DEPTH) * 144);
#pragma unroll
    for (int d = 0; d < KQ_DEPTH; d++) {
      const int ib = 4 * d + j;
      if (ib < nb) {
        qv[d] = __ldg(reinterpret_cast<const uint4*>(rp + (size_t)ib * 144 + 16 + 32 * c + 16 * hf));
        hv[d] = __ldg(reinterpret_cast<const uint4*>(rp + (size_t)ib * 144));
      }
    }
  }
  pdl_wait();
  pdl_trigger();
  if (!live) return;
  float acc[BT];
#pragma unroll
  for (int t = 0; t < BT; t++) acc[t] = 0.0f;
#pragma unroll 1
  for (int it0 = 0; it0 < nit; it0 += KQ_DEPTH) {
#pragma unroll
    for (int dd = 0; dd < KQ_DEPTH; dd++) {
      const int it = it0 + dd;
      if (it >= nit) break;
      const int ib = 4 * it + j;
      const bool valid = ib < nb;
      const uint4 cq = qv[dd], ch = hv[dd];
      if (4 * (it + KQ_DEPTH) + j < nb) {
        const unsigned char* np = rp + (size_t)(4 * (it + KQ_DEPTH) + j) * 144;
        qv[dd] = __ldg(reinterpret_cast<const uint4*>(np + 16 + 32 * c + 16 * hf));
        hv[dd] = __ldg(reinterpret_cast<const uint4*>(np));
      }
      const uint4 wl = make_uint4(cq.x & 0x0F0F0F0Fu, cq.y & 0x0F0F0F0Fu, cq.z & 0x0F0F0F0Fu, cq.w & 0x0F0F0F0Fu);
      const uint4 wh = make_uint4((cq.x >> 4) & 0x0F0F0F0Fu, (cq.y >> 4) & 0x0F0F0F0Fu, (cq.z >> 4) & 0x0F0F0F0Fu,
                                  (cq.w >> 4) & 0x0F0F0F0Fu);
      int sc0 = 0, m0 = 0, sc1 = 0, m1 = 0;
      kq_scale_min(ch.y, ch.z, ch.w, 2 * c, sc0, m0);
      kq_scale_min(ch.y, ch.z, ch.w, 2 * c + 1, sc1, m1);
      const float d = kq_half(ch.x & 0xFFFFu), dmin = kq_half(ch.x >> 16);
      const float dsc0 = __fmul_rn(d, (float)sc0), dm0 = __fmul_rn(dmin, (float)m0);
      const float dsc1 = __fmul_rn(d, (float)sc1), dm1 = __fmul_rn(dmin, (float)m1);
      const int vb = valid ? ib : 0;  // an idle slot of the last iteration reads block 0's activations (in bounds)
#pragma unroll
      for (int t = 0; t < BT; t++) {
        if (t < B) {
          const int8_t* xr = xq + (size_t)t * K + vb * 256 + 64 * c + 16 * hf;
          int lo = valid ? kq_dot16(wl, __ldg(reinterpret_cast<const uint4*>(xr))) : 0;
          int hi = valid ? kq_dot16(wh, __ldg(reinterpret_cast<const uint4*>(xr + 32))) : 0;
          lo += __shfl_xor_sync(0xffffffffu, lo, 1);
          hi += __shfl_xor_sync(0xffffffffu, hi, 1);
          if (hf == 0 && valid) {
            const size_t xo = (size_t)t * S + ib * 8 + 2 * c;
            float v = __fmaf_rn(dsc0, (float)lo, -__fmul_rn(dm0, (float)__ldg(xs + xo)));
            acc[t] = __fmaf_rn(v, __ldg(dx + xo), acc[t]);
            v = __fmaf_rn(dsc1, (float)hi, -__fmul_rn(dm1, (float)__ldg(xs + xo + 1)));
            acc[t] = __fmaf_rn(v, __ldg(dx + xo + 1), acc[t]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < BT; t++) {
    if (t < B) {
      const float v = kq_tree(acc[t], 1);
      if (lane == 0) y[(size_t)t * N + row] = v;
    }
  }
}

// 16 bytes at a 2-byte-aligned address as 4 words: five aligned words from a & ~3, realigned by a funnel shift when
// a % 4 == 2 (reads at most 2 bytes before a and 3 after a + 16; callers keep both inside the block's row).
__device__ __forceinline__ uint4 kq_ld16_2(const unsigned char* a) {
  const uint32_t* b = reinterpret_cast<const uint32_t*>(reinterpret_cast<uintptr_t>(a) & ~(uintptr_t)3);
  const uint32_t w0 = __ldg(b), w1 = __ldg(b + 1), w2 = __ldg(b + 2), w3 = __ldg(b + 3), w4 = __ldg(b + 4);
  if (reinterpret_cast<uintptr_t>(a) & 2)
    return make_uint4(__funnelshift_r(w0, w1, 16), __funnelshift_r(w1, w2, 16), __funnelshift_r(w2, w3, 16),
                      __funnelshift_r(w3, w4, 16));
  return make_uint4(w0, w1, w2, w3);
}

// Q6_K: 4 blocks per warp iteration (ib = 4 it + j); lane 8j + 4h + 2p + hf reads ql bytes 64h + 32p + 16hf .. + 15
// and qh bytes 32h + 16hf .. + 15: its low quants are the 16 weights of sub-block s = 8h + 2p + hf, its high quants
// those of sub-block s + 4, so each lane's integer sums are whole sub-blocks; every lane keeps an accumulator.
struct KqQ6 {
  uint4 ql, qh;
  uint32_t meta;  // scale of sub-block s, of s + 4, f16 d
};
__device__ __forceinline__ KqQ6 kq_q6_load(const unsigned char* bp, int h, int p, int hf, int s) {
  KqQ6 r;
  r.ql = kq_ld16_2(bp + 64 * h + 32 * p + 16 * hf);
  r.qh = kq_ld16_2(bp + 128 + 32 * h + 16 * hf);
  r.meta = (uint32_t)(uint8_t)__ldg(bp + 192 + s) | ((uint32_t)(uint8_t)__ldg(bp + 196 + s) << 8) |
           ((uint32_t)__ldg(reinterpret_cast<const uint16_t*>(bp + 208)) << 16);
  return r;
}

__device__ __forceinline__ uint32_t kq_q6_word(uint32_t ql, uint32_t qh, int lo_shift, int hi_shift) {
  return __vsub4(((ql >> lo_shift) & 0x0F0F0F0Fu) | (((qh >> hi_shift) & 0x03030303u) << 4), 0x20202020u);
}

template <int BT>
__global__ void __launch_bounds__(KQ_WARPS * 32) kq_q6k_kernel(const unsigned char* __restrict__ w,
                                                               const int8_t* __restrict__ xq,
                                                               const float* __restrict__ dx,
                                                               const int* __restrict__ xs, float* __restrict__ y,
                                                               int N, int K, int B) {
  (void)xs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * KQ_WARPS + warp;
  const int j = lane >> 3, h = (lane >> 2) & 1, p = (lane >> 1) & 1, hf = lane & 1;
  const int s = 8 * h + 2 * p + hf;
  const int nb = K >> 8, S = K >> 5, nit = (nb + 3) >> 2;
  const bool live = row < N;
  const unsigned char* rp = w + (size_t)(live ? row : 0) * nb * 210;
  KqQ6 ring[KQ_DEPTH];
  if (live) {
    if (lane == 0 && nb > 4 * KQ_DEPTH) kq_prefetch_row(rp + 4 * KQ_DEPTH * 210, (size_t)(nb - 4 * KQ_DEPTH) * 210);
#pragma unroll
    for (int d = 0; d < KQ_DEPTH; d++)
      if (4 * d + j < nb) ring[d] = kq_q6_load(rp + (size_t)(4 * d + j) * 210, h, p, hf, s);
  }
  pdl_wait();
  pdl_trigger();
  if (!live) return;
  float acc[BT];
#pragma unroll
  for (int t = 0; t < BT; t++) acc[t] = 0.0f;
#pragma unroll 1
  for (int it0 = 0; it0 < nit; it0 += KQ_DEPTH) {
#pragma unroll
    for (int dd = 0; dd < KQ_DEPTH; dd++) {
      const int it = it0 + dd;
      if (it >= nit) break;
      const int ib = 4 * it + j;
      const bool valid = ib < nb;
      const KqQ6 cur = ring[dd];
      if (4 * (it + KQ_DEPTH) + j < nb) ring[dd] = kq_q6_load(rp + (size_t)(4 * (it + KQ_DEPTH) + j) * 210, h, p, hf, s);
      const uint4 wl = make_uint4(kq_q6_word(cur.ql.x, cur.qh.x, 0, 2 * p), kq_q6_word(cur.ql.y, cur.qh.y, 0, 2 * p),
                                  kq_q6_word(cur.ql.z, cur.qh.z, 0, 2 * p), kq_q6_word(cur.ql.w, cur.qh.w, 0, 2 * p));
      const uint4 wh = make_uint4(
          kq_q6_word(cur.ql.x, cur.qh.x, 4, 4 + 2 * p), kq_q6_word(cur.ql.y, cur.qh.y, 4, 4 + 2 * p),
          kq_q6_word(cur.ql.z, cur.qh.z, 4, 4 + 2 * p), kq_q6_word(cur.ql.w, cur.qh.w, 4, 4 + 2 * p));
      const float d = kq_half(cur.meta >> 16);
      const float dsc_lo = __fmul_rn(d, (float)(int8_t)(cur.meta & 0xFFu));
      const float dsc_hi = __fmul_rn(d, (float)(int8_t)((cur.meta >> 8) & 0xFFu));
      if (valid) {
#pragma unroll
        for (int t = 0; t < BT; t++) {
          if (t < B) {
            const int8_t* xr = xq + (size_t)t * K + ib * 256 + 128 * h + 32 * p + 16 * hf;
            const int lo = kq_dot16(wl, __ldg(reinterpret_cast<const uint4*>(xr)));
            const int hi = kq_dot16(wh, __ldg(reinterpret_cast<const uint4*>(xr + 64)));
            const size_t xo = (size_t)t * S + ib * 8 + 4 * h + p;
            acc[t] = __fmaf_rn(__fmul_rn(dsc_lo, (float)lo), __ldg(dx + xo), acc[t]);
            acc[t] = __fmaf_rn(__fmul_rn(dsc_hi, (float)hi), __ldg(dx + xo + 2), acc[t]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < BT; t++) {
    if (t < B) {
      const float v = kq_tree(acc[t], 0);
      if (lane == 0) y[(size_t)t * N + row] = v;
    }
  }
}

// Q4_K for 3-32 tokens on int8 tensor-core MMA (mma.sync m16n8k32 s8 x s8 -> s32): a CTA of 4 warps takes 16 rows
// and one 8-token tile (grid.y); warp j takes the blocks ib = j mod 4 of all 16 rows. For sub-block sb of a block, one MMA gives sum(q * xq) exactly
// for the 16 rows x 8 tokens: lane (g = lane / 4, t = lane % 4) holds A = quant bytes 32c + 4t .. + 3 and 32c + 16 +
// 4t .. + 3 (nibble sb & 1, c = sb / 2) of rows g and g + 8, B = the 8-bit activations of the tile's token g at the
// same k, and C = rows g, g + 8 x the tile's tokens 2t, 2t + 1. Each (row, token) keeps one accumulator per chunk c, updated in the dp4a
// kernel's order (blocks ib = j mod 4 in order, sub-block 2c then 2c + 1) and summed in its tree: ((c0 + c1) +
// (c2 + c3)) within the warp, then ((T0 + T1) + (T2 + T3)) over the four warps. So the bits equal the dp4a kernel's.
__device__ __forceinline__ void kq_mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                          uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct KqMmaRow {
  uint32_t q[8];  // per chunk c: quant word 32c + 4t (q[2c]) and 32c + 16 + 4t (q[2c + 1])
  uint4 h;        // d, dmin, packed scales
};
__device__ __forceinline__ void kq_mma_load(KqMmaRow& r, const unsigned char* bp, int t) {
#pragma unroll
  for (int c = 0; c < 4; c++) {
    r.q[2 * c] = __ldg(reinterpret_cast<const uint32_t*>(bp + 16 + 32 * c + 4 * t));
    r.q[2 * c + 1] = __ldg(reinterpret_cast<const uint32_t*>(bp + 16 + 32 * c + 16 + 4 * t));
  }
  r.h = __ldg(reinterpret_cast<const uint4*>(bp));
}

constexpr int KQ_MMA_MIN_TOKENS = 3;  // 1-2 tokens stay on dp4a (faster there)

__global__ void __launch_bounds__(128) kq_q4k_mma_kernel(const unsigned char* __restrict__ w,
                                                         const int8_t* __restrict__ xq, const float* __restrict__ dx,
                                                         const int* __restrict__ xs, float* __restrict__ y, int N,
                                                         int K, int B) {
  __shared__ float part[4][32][4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int row0 = blockIdx.x * 16, tb = blockIdx.y * 8;  // rows, and this CTA's 8-token tile
  const int nb = K >> 8, S = K >> 5;
  const int ra = row0 + g, rb = row0 + g + 8;
  const bool va = ra < N, vb = rb < N;
  const unsigned char* pa = w + (size_t)(va ? ra : 0) * nb * 144;
  const unsigned char* pb = w + (size_t)(vb ? rb : 0) * nb * 144;
  if (warp == 0 && t == 0) {  // the 16 rows into L2 (each lane its two rows)
    if (va) kq_prefetch_row(pa, (size_t)nb * 144);
    if (vb) kq_prefetch_row(pb, (size_t)nb * 144);
  }
  KqMmaRow na, nbr;
  if (warp < nb) {
    kq_mma_load(na, pa + (size_t)warp * 144, t);
    kq_mma_load(nbr, pb + (size_t)warp * 144, t);
  }
  pdl_wait();
  pdl_trigger();
  const int t0 = tb + 2 * t, t1 = tb + 2 * t + 1, tg = tb + g;  // this lane's tokens in C, and in B
  float acc[4][4];
#pragma unroll
  for (int c = 0; c < 4; c++)
#pragma unroll
    for (int e = 0; e < 4; e++) acc[c][e] = 0.0f;
#pragma unroll 1
  for (int ib = warp; ib < nb; ib += 4) {
    const KqMmaRow qa = na, qb = nbr;
    if (ib + 4 < nb) {
      kq_mma_load(na, pa + (size_t)(ib + 4) * 144, t);
      kq_mma_load(nbr, pb + (size_t)(ib + 4) * 144, t);
    }
    const float da = kq_half(qa.h.x & 0xFFFFu), dma = kq_half(qa.h.x >> 16);
    const float db = kq_half(qb.h.x & 0xFFFFu), dmb = kq_half(qb.h.x >> 16);
    const int8_t* xr = xq + (size_t)(tg < B ? tg : 0) * K + ib * 256 + 4 * t;
#pragma unroll
    for (int c = 0; c < 4; c++) {
      int sca0, ma0, sca1, ma1, scb0, mb0, scb1, mb1;
      kq_scale_min(qa.h.y, qa.h.z, qa.h.w, 2 * c, sca0, ma0);
      kq_scale_min(qa.h.y, qa.h.z, qa.h.w, 2 * c + 1, sca1, ma1);
      kq_scale_min(qb.h.y, qb.h.z, qb.h.w, 2 * c, scb0, mb0);
      kq_scale_min(qb.h.y, qb.h.z, qb.h.w, 2 * c + 1, scb1, mb1);
#pragma unroll
      for (int n = 0; n < 2; n++) {
        const int sb = 2 * c + n;
        const uint32_t a0 = (qa.q[2 * c] >> (4 * n)) & 0x0F0F0F0Fu, a2 = (qa.q[2 * c + 1] >> (4 * n)) & 0x0F0F0F0Fu;
        const uint32_t a1 = (qb.q[2 * c] >> (4 * n)) & 0x0F0F0F0Fu, a3 = (qb.q[2 * c + 1] >> (4 * n)) & 0x0F0F0F0Fu;
        const uint32_t b0 = tg < B ? __ldg(reinterpret_cast<const uint32_t*>(xr + 32 * sb)) : 0u;
        const uint32_t b1 = tg < B ? __ldg(reinterpret_cast<const uint32_t*>(xr + 32 * sb + 16)) : 0u;
        int cc[4] = {0, 0, 0, 0};
        kq_mma_s8(cc, a0, a1, a2, a3, b0, b1);
        const float dsa = __fmul_rn(da, (float)(n ? sca1 : sca0)), dsma = __fmul_rn(dma, (float)(n ? ma1 : ma0));
        const float dsb = __fmul_rn(db, (float)(n ? scb1 : scb0)), dsmb = __fmul_rn(dmb, (float)(n ? mb1 : mb0));
        if (t0 < B) {
          const size_t xo = (size_t)t0 * S + ib * 8 + sb;
          const float xsv = (float)__ldg(xs + xo), dxv = __ldg(dx + xo);
          acc[c][0] = __fmaf_rn(__fmaf_rn(dsa, (float)cc[0], -__fmul_rn(dsma, xsv)), dxv, acc[c][0]);
          acc[c][2] = __fmaf_rn(__fmaf_rn(dsb, (float)cc[2], -__fmul_rn(dsmb, xsv)), dxv, acc[c][2]);
        }
        if (t1 < B) {
          const size_t xo = (size_t)t1 * S + ib * 8 + sb;
          const float xsv = (float)__ldg(xs + xo), dxv = __ldg(dx + xo);
          acc[c][1] = __fmaf_rn(__fmaf_rn(dsa, (float)cc[1], -__fmul_rn(dsma, xsv)), dxv, acc[c][1]);
          acc[c][3] = __fmaf_rn(__fmaf_rn(dsb, (float)cc[3], -__fmul_rn(dsmb, xsv)), dxv, acc[c][3]);
        }
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 4; e++) part[warp][lane][e] = (acc[0][e] + acc[1][e]) + (acc[2][e] + acc[3][e]);
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int e = 0; e < 4; e++) {
      const float v = (part[0][lane][e] + part[1][lane][e]) + (part[2][lane][e] + part[3][lane][e]);
      const int row = e < 2 ? ra : rb, tok = (e & 1) ? t1 : t0;
      if ((e < 2 ? va : vb) && tok < B) y[(size_t)tok * N + row] = v;
    }
  }
}

template <int BT>
static int kq_launch_bt(int type, const void* w, const int8_t* xq, const float* dx, const int* xs, float* y, int N,
                        int K, int B, cudaStream_t st) {
  const dim3 grid((unsigned)((N + KQ_WARPS - 1) / KQ_WARPS)), block(KQ_WARPS * 32);
  const unsigned char* wb = static_cast<const unsigned char*>(w);
  if (type == KQ_Q4K) return launch("kq_q4k_kernel", kq_q4k_kernel<BT>, grid, block, 0, st, wb, xq, dx, xs, y, N, K, B);
  return launch("kq_q6k_kernel", kq_q6k_kernel<BT>, grid, block, 0, st, wb, xq, dx, xs, y, N, K, B);
}

// What the kernels serve: checked before anything touches the device.
static int kq_check(const char* who, int type, int64_t N, int64_t K, int64_t B) {
  IM_REQUIRE(type == KQ_Q4K || type == KQ_Q6K, IM_UNSUPPORTED, "%s: weight type %d (12 = Q4_K and 14 = Q6_K only)",
             who, type);
  IM_REQUIRE(K > 0 && K % 256 == 0 && K <= (1 << 20), IM_UNSUPPORTED, "%s: K = %lld (a multiple of 256)", who,
             (long long)K);
  IM_REQUIRE(B >= 1 && B <= KQ_MAX_TOKENS, IM_UNSUPPORTED, "%s: %lld tokens (1 .. 32)", who, (long long)B);
  IM_REQUIRE(N >= 1 && N <= (1 << 24), IM_INVALID, "%s: N = %lld", who, (long long)N);
  return IM_OK;
}

static int kq_run(const char* who, int type, const void* w, const float* x, float* y, int64_t N, int64_t K, int64_t B,
                  void* workspace, size_t ws_bytes, cudaStream_t st) {
  if (int rc = kq_check(who, type, N, K, B)) return rc;
  IM_REQUIRE(w && x && y && workspace, IM_INVALID, "%s: null pointer", who);
  IM_REQUIRE(aligned(w, type == KQ_Q4K ? 16 : 4), IM_INVALID, "%s: weights must be %d-byte aligned", who,
             type == KQ_Q4K ? 16 : 4);
  IM_REQUIRE(aligned(workspace, 256) && ws_bytes >= kq_ws_bytes(K, B), IM_INVALID,
             "%s: workspace needs %zu bytes, 256-byte aligned", who, kq_ws_bytes(K, B));
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  int8_t* xq = reinterpret_cast<int8_t*>(ws);
  float* dx = reinterpret_cast<float*>(ws + kq_round((size_t)B * K));
  int* xs = reinterpret_cast<int*>(ws + kq_round((size_t)B * K) + kq_round((size_t)B * (K / 32) * 4));
  const int blocks = (int)(B * (K / 32));
  int rc = launch("kq_quant_kernel", kq_quant_kernel, dim3((unsigned)((blocks + 7) / 8)), dim3(256), 0, st, x, xq, dx,
                  xs, blocks);
  if (rc) return rc;
  const int n = (int)N, k = (int)K, b = (int)B;
  if (type == KQ_Q4K && B >= KQ_MMA_MIN_TOKENS)
    return launch("kq_q4k_mma_kernel", kq_q4k_mma_kernel, dim3((unsigned)((N + 15) / 16), (unsigned)((B + 7) / 8)),
                  dim3(128), 0, st,
                  static_cast<const unsigned char*>(w), xq, dx, xs, y, n, k, b);
  if (B <= 1) return kq_launch_bt<1>(type, w, xq, dx, xs, y, n, k, b, st);
  if (B <= 2) return kq_launch_bt<2>(type, w, xq, dx, xs, y, n, k, b, st);
  if (B <= 4) return kq_launch_bt<4>(type, w, xq, dx, xs, y, n, k, b, st);
  if (B <= 8) return kq_launch_bt<8>(type, w, xq, dx, xs, y, n, k, b, st);
  if (B <= 16) return kq_launch_bt<16>(type, w, xq, dx, xs, y, n, k, b, st);
  return kq_launch_bt<32>(type, w, xq, dx, xs, y, n, k, b, st);
}

// The hook's scratch: one static device array per process (per device: its own copy), found once per device.
constexpr size_t KQ_HOOK_BYTES = 2u << 20;
constexpr int KQ_HOOK_MAX_DEVICES = 64;
static __device__ __align__(256) unsigned char g_kq_hook_scratch[KQ_HOOK_BYTES];
static std::mutex g_kq_hook_mutex;
static void* g_kq_hook_ptr[KQ_HOOK_MAX_DEVICES] = {};

}  // namespace im

using namespace im;

extern "C" size_t im_kq_workspace_bytes(int64_t K, int64_t B) {
  if (K <= 0 || B <= 0) return 0;
  return kq_ws_bytes(K, B);
}

extern "C" int im_kq_gemv(int type, const void* w, const float* x, float* y, int64_t N, int64_t K, int64_t B,
                          void* workspace, size_t ws_bytes, void* stream) {
  clear_error();
  return kq_run("im_kq_gemv", type, w, x, y, N, K, B, workspace, ws_bytes, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int im_kq_mul_mat(int type, const void* w, const float* x, float* y, int64_t N, int64_t K, int64_t B,
                             void* stream) {
  clear_error();
  if (int rc = kq_check("im_kq_mul_mat", type, N, K, B)) return rc;
  IM_REQUIRE(kq_ws_bytes(K, B) <= KQ_HOOK_BYTES, IM_UNSUPPORTED, "im_kq_mul_mat: K x tokens beyond the hook's scratch");
  IM_REQUIRE(w && x && y, IM_INVALID, "im_kq_mul_mat: null pointer");
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  IM_REQUIRE(e == cudaSuccess, IM_CUDA_ERROR, "im_kq_mul_mat: cudaGetDevice: %s", cudaGetErrorString(e));
  IM_REQUIRE(dev >= 0 && dev < KQ_HOOK_MAX_DEVICES, IM_UNSUPPORTED, "im_kq_mul_mat: device %d", dev);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_kq_hook_mutex);
    if (!g_kq_hook_ptr[dev]) {
      e = cudaGetSymbolAddress(&scratch, g_kq_hook_scratch);
      IM_REQUIRE(e == cudaSuccess, IM_CUDA_ERROR, "im_kq_mul_mat: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      g_kq_hook_ptr[dev] = scratch;
    }
    scratch = g_kq_hook_ptr[dev];
  }
  return kq_run("im_kq_mul_mat", type, w, x, y, N, K, B, scratch, KQ_HOOK_BYTES, reinterpret_cast<cudaStream_t>(stream));
}

// The name llama.cpp's patched mul_mat looks up in the library IRONMULE_KG_LIB names (the reference's
// native/ggml_patches/kg1/ggml-cuda.cu.diff:6-18): the same call as im_kq_mul_mat.
extern "C" int ironmule_kg_mul_mat(int type, const void* w, const float* x, float* y, int64_t N, int64_t K, int64_t B,
                                   void* stream) {
  return im_kq_mul_mat(type, w, x, y, N, K, B, stream);
}
