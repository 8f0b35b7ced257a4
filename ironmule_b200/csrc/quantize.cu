// MLX-affine 4-bit quantisation (group 64) on the device, for loading float weights and for the
// random-init benchmark models. Per group: scale = bf16((max - min) / 15), bias = bf16(min),
// q = clamp(rint((w - bias) / scale), 0, 15) in float32 with the rounded scale and bias (q = 0 where the
// scale rounds to 0); codes packed eight per uint32, low nibble first (the layout of
// IronMule ironmule/cuda_native.py:54-56 and ironmule/qmv_k3840.py:379-408).
#include "common.cuh"

namespace im {

__global__ void quantize_kernel(const uint16_t* __restrict__ w, int64_t groups, uint32_t* __restrict__ wq,
                                uint16_t* __restrict__ scales, uint16_t* __restrict__ biases) {
  const int64_t gidx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (gidx >= groups) return;
  const uint4* src = reinterpret_cast<const uint4*>(w + gidx * 64);
  float v[64];
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const uint4 q = src[i];
    v[8 * i + 0] = bf_lo(q.x); v[8 * i + 1] = bf_hi(q.x);
    v[8 * i + 2] = bf_lo(q.y); v[8 * i + 3] = bf_hi(q.y);
    v[8 * i + 4] = bf_lo(q.z); v[8 * i + 5] = bf_hi(q.z);
    v[8 * i + 6] = bf_lo(q.w); v[8 * i + 7] = bf_hi(q.w);
  }
  float lo = v[0], hi = v[0];
#pragma unroll
  for (int i = 1; i < 64; i++) {
    lo = fminf(lo, v[i]);
    hi = fmaxf(hi, v[i]);
  }
  const uint16_t sb = to_bf(__fdiv_rn(hi - lo, 15.0f));
  const uint16_t bb = to_bf(lo);
  const float s = bf(sb), b = bf(bb);
  scales[gidx] = sb;
  biases[gidx] = bb;
  uint32_t* dst = wq + gidx * 8;
#pragma unroll
  for (int wd = 0; wd < 8; wd++) {
    uint32_t word = 0;
#pragma unroll
    for (int e = 0; e < 8; e++) {
      float q = s == 0.f ? 0.f : rintf(__fdiv_rn(v[8 * wd + e] - b, s));
      q = fminf(fmaxf(q, 0.f), 15.f);
      word |= ((uint32_t)q) << (4 * e);
    }
    dst[wd] = word;
  }
}

}  // namespace im

using namespace im;

extern "C" int im_quantize_w4g64(const uint16_t* w, int64_t N, int64_t K, uint32_t* wq, uint16_t* scales,
                                 uint16_t* biases, void* stream) {
  clear_error();
  IM_REQUIRE(N >= 1 && K >= 64 && K % 64 == 0, IM_INVALID, "im_quantize_w4g64: bad sizes N=%lld K=%lld",
             (long long)N, (long long)K);
  IM_REQUIRE(w && wq && scales && biases, IM_INVALID, "im_quantize_w4g64: null pointer");
  IM_REQUIRE(aligned(w, 16) && aligned(wq, 16), IM_INVALID, "im_quantize_w4g64: w and wq must be 16-byte aligned");
  const int64_t groups = N * (K / 64);
  const int threads = 128;
  const int64_t blocks = (groups + threads - 1) / threads;
  IM_REQUIRE(blocks < (1ll << 31), IM_UNSUPPORTED, "im_quantize_w4g64: too many groups");
  quantize_kernel<<<(unsigned)blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(w, groups, wq, scales,
                                                                                           biases);
  return check_launch("quantize_kernel");
}
