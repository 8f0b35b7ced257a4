// Per-row layer math around the qGEMMs of a decode/verify pass (Qwen3 and Gemma-3 shapes):
// RMSNorm, the fused q/k RMSNorm + RoPE + paged KV write, and the 4-bit embedding gather.
//
// Every op works on one row at a time with a fixed reduction order, so a row's bits do not depend on how
// many rows share the launch (the property the reference pins for its stacked plan,
// IronMule ironmule/dense_plan.py:49-51, :438-458). bf16 rounding follows the op boundaries of the
// decode-layer math in ironmule/paired_research.py:177-215 (Gemma-3) and mlx_lm's Qwen3.
#include <math.h>

#include "common.cuh"

namespace im {

constexpr int LN_THREADS = 256;

__device__ __forceinline__ float block_sum_256(float v, float* sh) {
  // fixed-order block reduction: warp xor-tree, then the 8 warp totals in order
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < LN_THREADS / 32; w++) t += sh[w];
  return t;
}

// out[m, :] = bf16( (x * inv_rms) * w' ), w' = w (Qwen3) or 1 + w (Gemma-3), inv_rms = 1/sqrt(mean(x^2)+eps).
__global__ void __launch_bounds__(LN_THREADS)
rmsnorm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, uint16_t* __restrict__ out, int H,
               long long ldx, float eps, int gemma) {
  __shared__ float sh[LN_THREADS / 32];
  pdl_wait();
  pdl_trigger();
  const uint16_t* xr = x + (size_t)blockIdx.x * ldx;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += LN_THREADS) {
    const float v = bf(xr[i]);
    ss = fmaf(v, v, ss);
  }
  const float total = block_sum_256(ss, sh);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(total, (float)H) + eps));
  uint16_t* orow = out + (size_t)blockIdx.x * H;
  for (int i = threadIdx.x; i < H; i += LN_THREADS) {
    const float wi = gemma ? 1.0f + bf(w[i]) : bf(w[i]);
    orow[i] = to_bf((bf(xr[i]) * inv) * wi);
  }
}

// Gemma-3's output norms: h[m] = bf16(h + bf16((y * inv_rms(y)) * (1 + w))) (w' = w for Qwen3-style weights);
// with w == NULL the plain residual add h[m] = bf16(h + y) (a tensor-parallel projection whose partial sums were
// all-reduced). out_sq[m] = the new row's sum of squares (block order: thread sums, warp xor-trees, warps in
// order) for the RMSNorm that the next qGEMM fuses. One CTA per row.
__global__ void __launch_bounds__(LN_THREADS)
rmsnorm_residual_kernel(const uint16_t* __restrict__ y, const uint16_t* __restrict__ w, uint16_t* __restrict__ h,
                        int H, float eps, int gemma, float* __restrict__ out_sq) {
  __shared__ float sh[LN_THREADS / 32];
  pdl_wait();
  pdl_trigger();
  const uint16_t* yr = y + (size_t)blockIdx.x * H;
  uint16_t* hr = h + (size_t)blockIdx.x * H;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += LN_THREADS) {
    const float v = bf(yr[i]);
    ss = fmaf(v, v, ss);
  }
  const float total = block_sum_256(ss, sh);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(total, (float)H) + eps));
  float s2 = 0.f;
  for (int i = threadIdx.x; i < H; i += LN_THREADS) {
    float o = bf(yr[i]);
    if (w) {
      const float wi = gemma ? 1.0f + bf(w[i]) : bf(w[i]);
      o = round_bf((o * inv) * wi);
    }
    const uint16_t hn = to_bf(bf(hr[i]) + o);
    hr[i] = hn;
    s2 = fmaf(bf(hn), bf(hn), s2);
  }
  const float t2 = block_sum_256(s2, sh);
  if (out_sq && threadIdx.x == 0) out_sq[blockIdx.x] = t2;
}

// One CTA per (row, head) over the packed qkv row [Hq*D | Hkv*D | Hkv*D]:
//  q heads: RMSNorm over D with qn, RoPE at the row's position -> q_out[m, h, :]
//  k heads: RMSNorm with kn, RoPE -> the paged K cache; the matching v head copied to the V cache.
// RoPE is the non-interleaved form: pairs (i, i + D/2), angle = pos * inv_freq[i] (inv_freq from the host).
// KV cache layout: [pages][Hkv][16][D] bf16; the row's storage slot is row_slot[m] in its sequence
// row_seq[m], page = page_table[seq * max_pages + slot / 16].
template <int D>
__global__ void __launch_bounds__(D)
qk_rope_kv_kernel(const uint16_t* __restrict__ qkv, const uint16_t* __restrict__ qn, const uint16_t* __restrict__ kn,
                  const float* __restrict__ inv_freq, const int* __restrict__ row_pos, const int* __restrict__ row_slot,
                  const int* __restrict__ row_seq, const int* __restrict__ page_table, int max_pages, int Hq, int Hkv,
                  float eps, int gemma, uint16_t* __restrict__ q_out, uint16_t* __restrict__ kc,
                  uint16_t* __restrict__ vc) {
  __shared__ float sh[32];
  __shared__ float xn[D];
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x, h = blockIdx.y, d = threadIdx.x;
  const int stride = (Hq + 2 * Hkv) * D;
  const bool is_q = h < Hq;
  const int head = is_q ? h : h - Hq;
  const uint16_t* src = qkv + (size_t)m * stride + (is_q ? h * D : Hq * D + head * D);
  const float v = bf(src[d]);
  // RMSNorm over the head (fixed order: warp tree, then warps in order)
  float ss = warp_sum(v * v);
  if ((d & 31) == 0) sh[d >> 5] = ss;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < D / 32; w++) total += sh[w];
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(total, (float)D) + eps));
  const uint16_t* nw = is_q ? qn : kn;
  const float wd = gemma ? 1.0f + bf(nw[d]) : bf(nw[d]);
  xn[d] = round_bf((v * inv) * wd);
  __syncthreads();
  const int half = D / 2;
  const int i = d < half ? d : d - half;
  const float ang = (float)row_pos[m] * inv_freq[i];
  float sn, cs;
  sincosf(ang, &sn, &cs);
  const float x1 = xn[i], x2 = xn[i + half];
  const float r = d < half ? x1 * cs - x2 * sn : x1 * sn + x2 * cs;
  const uint16_t rb = to_bf(r);
  if (is_q) {
    q_out[((size_t)m * Hq + h) * D + d] = rb;
  } else {
    const int slot = row_slot[m];
    const int page = page_table[(size_t)row_seq[m] * max_pages + (slot >> 4)];
    const size_t off = (((size_t)page * Hkv + head) * 16 + (slot & 15)) * D + d;
    kc[off] = rb;
    vc[off] = src[(size_t)Hkv * D + d];  // v sits Hkv*D after k in the packed row
  }
}

// out[m, :] = bf16(scale_q * q + bias_q) of row tokens[m] of a 4-bit table [V, H], times `mult` (Gemma-3's
// sqrt(hidden), rounded to bf16 as the reference does) when mult != 1.
__global__ void embed_kernel(const int* __restrict__ tokens, int tstride, const uint32_t* __restrict__ wq,
                             const uint16_t* __restrict__ sc, const uint16_t* __restrict__ bi, int H, int V,
                             float mult, uint16_t* __restrict__ out, float* __restrict__ out_sq) {
  __shared__ float sh[4];
  pdl_wait();
  pdl_trigger();
  const int m = blockIdx.x;
  int tok = tokens[(size_t)m * tstride];
  tok = tok < 0 ? 0 : (tok >= V ? V - 1 : tok);
  const uint32_t* row = wq + (size_t)tok * (H / 8);
  const uint16_t* srow = sc + (size_t)tok * (H / 64);
  const uint16_t* brow = bi + (size_t)tok * (H / 64);
  const float mb = round_bf(mult);
  float sq = 0.f;
  for (int wd = threadIdx.x; wd < H / 8; wd += blockDim.x) {
    const uint32_t u = row[wd];
    const float s = bf(srow[wd >> 3]), b = bf(brow[wd >> 3]);
#pragma unroll
    for (int e = 0; e < 8; e++) {
      float val = round_bf(fmaf(s, (float)((u >> (4 * e)) & 0xFu), b));
      if (mult != 1.0f) val = val * mb;
      const uint16_t o = to_bf(val);
      out[(size_t)m * H + wd * 8 + e] = o;
      sq = fmaf(bf(o), bf(o), sq);
    }
  }
  if (out_sq) {  // the row's sum of squares for a fused RMSNorm downstream (fixed order: warps, then in order)
    sq = warp_sum(sq);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = sq;
    __syncthreads();
    if (threadIdx.x == 0) out_sq[m] = sh[0] + sh[1] + sh[2] + sh[3];
  }
}

}  // namespace im

using namespace im;

extern "C" int im_rmsnorm(const uint16_t* x, int64_t ldx, const uint16_t* weight, uint16_t* out, int64_t M,
                          int64_t H, float eps, int gemma_style, void* stream) {
  clear_error();
  IM_REQUIRE(M >= 0 && H >= 1 && H <= (1 << 20) && ldx >= H, IM_INVALID, "im_rmsnorm: bad sizes");
  if (M == 0) return IM_OK;
  IM_REQUIRE(x && weight && out, IM_INVALID, "im_rmsnorm: null pointer");
  IM_REQUIRE(M < (1ll << 31), IM_UNSUPPORTED, "im_rmsnorm: too many rows");
  return launch("rmsnorm_kernel", rmsnorm_kernel, dim3((unsigned)M), dim3(LN_THREADS), 0,
                reinterpret_cast<cudaStream_t>(stream), x, weight, out, (int)H, (long long)ldx, eps, gemma_style);
}

extern "C" int im_rmsnorm_residual(const uint16_t* y, const uint16_t* weight, uint16_t* h, int64_t M, int64_t H,
                                   float eps, int gemma_style, float* out_sq, void* stream) {
  clear_error();
  IM_REQUIRE(M >= 0 && H >= 1 && H <= (1 << 20), IM_INVALID, "im_rmsnorm_residual: bad sizes");
  if (M == 0) return IM_OK;
  IM_REQUIRE(y && h, IM_INVALID, "im_rmsnorm_residual: null pointer");
  return launch("rmsnorm_residual_kernel", rmsnorm_residual_kernel, dim3((unsigned)M), dim3(LN_THREADS), 0,
                reinterpret_cast<cudaStream_t>(stream), y, weight, h, (int)H, eps, gemma_style, out_sq);
}

extern "C" int im_qk_norm_rope_kv(const uint16_t* qkv, const uint16_t* q_norm, const uint16_t* k_norm,
                                  const float* inv_freq, const int32_t* row_pos, const int32_t* row_slot,
                                  const int32_t* row_seq, const int32_t* page_table, int64_t max_pages, int64_t M,
                                  int64_t Hq, int64_t Hkv, int64_t D, float eps, int gemma_style, uint16_t* q_out,
                                  uint16_t* k_cache, uint16_t* v_cache, void* stream) {
  clear_error();
  IM_REQUIRE(M >= 0 && Hq >= 1 && Hkv >= 1 && Hq % Hkv == 0, IM_INVALID, "im_qk_norm_rope_kv: bad head counts");
  if (M == 0) return IM_OK;
  IM_REQUIRE(D == 128 || D == 256, IM_UNSUPPORTED, "im_qk_norm_rope_kv: head_dim %lld (128 or 256 supported)",
             (long long)D);
  IM_REQUIRE(qkv && q_norm && k_norm && inv_freq && row_pos && row_slot && row_seq && page_table && q_out &&
                 k_cache && v_cache,
             IM_INVALID, "im_qk_norm_rope_kv: null pointer");
  dim3 grid((unsigned)M, (unsigned)(Hq + Hkv));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (D == 128)
    return launch("qk_rope_kv_kernel", qk_rope_kv_kernel<128>, grid, dim3(128), 0, st, qkv, q_norm, k_norm, inv_freq,
                  row_pos, row_slot, row_seq, page_table, (int)max_pages, (int)Hq, (int)Hkv, eps, gemma_style, q_out,
                  k_cache, v_cache);
  return launch("qk_rope_kv_kernel", qk_rope_kv_kernel<256>, grid, dim3(256), 0, st, qkv, q_norm, k_norm, inv_freq,
                row_pos, row_slot, row_seq, page_table, (int)max_pages, (int)Hq, (int)Hkv, eps, gemma_style, q_out,
                k_cache, v_cache);
}

extern "C" int im_embed_w4g64(const int32_t* tokens, int64_t tokens_stride, const uint32_t* wq,
                              const uint16_t* scales, const uint16_t* biases, int64_t M, int64_t V, int64_t H,
                              float mult, uint16_t* out, float* out_sq, void* stream) {
  clear_error();
  IM_REQUIRE(M >= 0 && V >= 1 && H >= 64 && H % 64 == 0 && tokens_stride >= 1, IM_INVALID,
             "im_embed_w4g64: bad sizes");
  if (M == 0) return IM_OK;
  IM_REQUIRE(tokens && wq && scales && biases && out, IM_INVALID, "im_embed_w4g64: null pointer");
  return launch("embed_kernel", embed_kernel, dim3((unsigned)M), dim3(128), 0, reinterpret_cast<cudaStream_t>(stream),
                tokens, (int)tokens_stride, wq, scales, biases, (int)H, (int)V, mult, out, out_sq);
}
