// The split partials of the paged attention and their merge, shared by the attention kernel (which merges
// them itself) and the packed qGEMM's o-projection prologue (which merges them on the way in when the attention
// leaves them unmerged). One function does the arithmetic for both, so the two give the same bits.
#pragma once

#include <cstddef>
#include <cstdint>
#include <math.h>

#include "common.cuh"

namespace im {

constexpr int AT_KB = 64;  // keys per shared-memory block
// A split partial per query vector: D accumulators, max, sum, 2 floats of padding (16-byte rows for float4 reads).
constexpr int AT_PAD = 4;
// Workspace layout, identical for every call so calls of different shapes may share one buffer: arrival counters
// in a fixed region (kept at zero between launches), then the split partials
// part[((group * nsplit + split) * NQ + qi) * (D + AT_PAD)], group = (b * Hkv + kvh) * qblocks + qb.
constexpr size_t AT_COUNTER_BYTES = 65536;
constexpr int64_t AT_MAX_GROUPS = (int64_t)(AT_COUNTER_BYTES / 4);

// Query vectors per CTA (NQ) and query blocks per (sequence, kv head) for sequences of up to rows_per_seq rows.
inline void attn_geometry(int64_t rows_per_seq, int64_t G, int* nq, int* qblocks) {
  const int64_t qv = rows_per_seq * G;
  *nq = qv <= 8 ? 8 : 32;
  *qblocks = (int)((qv + *nq - 1) / *nq);
}

// Merges dims [d4, d4 + 4) of one query vector over splits [0, used) in split order: base points at split 0's
// partial of the vector (D accumulators, then max and sum), sstride floats apart per split. Weights
// w_s = exp(m_s - max) (0 for an empty split); the denominator sum_s l_s w_s and the numerator sum_s o_s w_s are
// both summed in split order; out = bf16(o / l), 0 when l = 0. Up to 8 splits take one round trip, more take
// two passes (their maxima first).
__device__ __forceinline__ void attn_merge4(const float* base, size_t sstride, int d4, int used, int D,
                                            uint16_t (&out)[4]) {
  constexpr int SB = 8;  // splits whose loads are in flight together
  float mx = -INFINITY, lsum = 0.f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  auto add = [&](const float4& v, float m, float l) {
    const float w = (m == -INFINITY || mx == -INFINITY) ? 0.f : expf(m - mx);
    lsum = fmaf(l, w, lsum);
    o.x = fmaf(v.x, w, o.x);
    o.y = fmaf(v.y, w, o.y);
    o.z = fmaf(v.z, w, o.z);
    o.w = fmaf(v.w, w, o.w);
  };
  if (used <= SB) {  // every split's loads in flight at once
    float4 v[SB];
    float ms[SB], ls[SB];
#pragma unroll
    for (int j = 0; j < SB; j++) {
      if (j < used) {
        const float* p = base + j * sstride;
        v[j] = __ldcg(reinterpret_cast<const float4*>(p + d4));
        ms[j] = __ldcg(p + D);
        ls[j] = __ldcg(p + D + 1);
      }
    }
#pragma unroll
    for (int j = 0; j < SB; j++)
      if (j < used) mx = fmaxf(mx, ms[j]);
#pragma unroll
    for (int j = 0; j < SB; j++)
      if (j < used) add(v[j], ms[j], ls[j]);
  } else {
    for (int s0 = 0; s0 < used; s0 += SB) {
      float ms[SB];
#pragma unroll
      for (int j = 0; j < SB; j++) ms[j] = s0 + j < used ? __ldcg(base + (s0 + j) * sstride + D) : -INFINITY;
#pragma unroll
      for (int j = 0; j < SB; j++) mx = fmaxf(mx, ms[j]);
    }
    for (int s0 = 0; s0 < used; s0 += SB) {
      float4 v[SB];
      float ms[SB], ls[SB];
#pragma unroll
      for (int j = 0; j < SB; j++) {
        if (s0 + j < used) {
          const float* p = base + (s0 + j) * sstride;
          v[j] = __ldcg(reinterpret_cast<const float4*>(p + d4));
          ms[j] = __ldcg(p + D);
          ls[j] = __ldcg(p + D + 1);
        }
      }
#pragma unroll
      for (int j = 0; j < SB; j++)
        if (s0 + j < used) add(v[j], ms[j], ls[j]);
    }
  }
  out[0] = to_bf(lsum > 0.f ? __fdiv_rn(o.x, lsum) : 0.f);
  out[1] = to_bf(lsum > 0.f ? __fdiv_rn(o.y, lsum) : 0.f);
  out[2] = to_bf(lsum > 0.f ? __fdiv_rn(o.z, lsum) : 0.f);
  out[3] = to_bf(lsum > 0.f ? __fdiv_rn(o.w, lsum) : 0.f);
}

}  // namespace im
