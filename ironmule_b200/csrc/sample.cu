// Stochastic acceptance and sampling for speculative decoding: temperature + top-p distributions over the
// vocabulary, p/q rejection of drafts with residual resampling, and token sampling, all on a counter-based
// Philox4x32-10 stream so a decision is a pure function of (seed, offset, sequence, draw).
//
// The reference accepts greedily only (IronMule ironmule/speculation.py:103-108; its product refuses
// temperature != 0 and top_p != 1, ironmule_product/worker.py:485-486). This is the published
// speculative-sampling rule (Leviathan, Kalman, Matias 2023; Chen et al. 2023): accept draft d with
// probability min(1, p(d) / q(d)); at the first rejection sample from norm(max(0, p - q)); after k accepts
// sample a bonus token from the target's next distribution.
//
// Distributions: p = softmax(logits / T) restricted to the top-p set {v : l_v >= l*} where l* is the largest
// logit whose set holds at least top_p of the mass (ties at the boundary are all kept), renormalised. The
// boundary is found over the 65536 bf16 keys with two 256-bin mass histograms (integer sums of the weights in
// units of 2^-26, independent of the order of the additions); the normaliser of the kept set is a fixed-order
// block reduction.
//
// Philox stream: key = (seed low, seed high), counter = (offset low, offset high, stream, draw), uniform =
// (word0 >> 8) * 2^-24. Acceptance uses stream = sequence, draw 2i (test of draft i), 2i+1 (resample after
// rejecting draft i), 2k (bonus). Sampling uses stream = the caller's per-row id and draw = `draw`.
#include <math.h>

#include "common.cuh"

namespace im {

constexpr int SM_THREADS = 1024;

__device__ __forceinline__ void philox_round(uint32_t (&c)[4], uint32_t k0, uint32_t k1) {
  const uint32_t lo0 = 0xD2511F53u * c[0], hi0 = __umulhi(0xD2511F53u, c[0]);
  const uint32_t lo1 = 0xCD9E8D57u * c[2], hi1 = __umulhi(0xCD9E8D57u, c[2]);
  const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
  c[0] = n0;
  c[1] = lo1;
  c[2] = n2;
  c[3] = lo0;
}

__device__ __forceinline__ void philox4x32_10(uint32_t (&c)[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; r++) {
    if (r) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    philox_round(c, k0, k1);
  }
}

__device__ __forceinline__ float philox_uniform(unsigned long long seed, unsigned long long offset, uint32_t stream,
                                                uint32_t draw) {
  uint32_t c[4] = {(uint32_t)offset, (uint32_t)(offset >> 32), stream, draw};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  return (float)(c[0] >> 8) * (1.0f / 16777216.0f);
}

// order-preserving 16-bit key of a bf16 value (NaN -> 0, excluded)
__device__ __forceinline__ uint32_t bf_key(uint16_t h) {
  if ((h & 0x7fffu) > 0x7f80u) return 0u;
  return (h & 0x8000u) ? (~h & 0xffffu) : (h | 0x8000u);
}

struct RowDist {
  float m;      // max logit
  float inv_t;  // 1 / temperature
  float s;      // sum of exp((l - m) / T) over the kept set
  uint32_t thr; // keep keys >= thr
};

__device__ __forceinline__ float block_sum_1024(float v, float* sh) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll 8
  for (int w = 0; w < SM_THREADS / 32; w++) t += sh[w];
  return t;
}

__device__ __forceinline__ float block_max_1024(float v, float* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) sh[warp] = v;
  __syncthreads();
  float t = -INFINITY;
  for (int w = 0; w < SM_THREADS / 32; w++) t = fmaxf(t, sh[w]);
  return t;
}

// Mass histograms of the top-p boundary search hold integer sums of the per-token weights exp((l - m) / T)
// (at most 1) rounded to multiples of 2^-26, so a bin's mass does not depend on the order of the additions and
// the boundary is the same on every run. A warp first adds the weights of its lanes that share a bin
// (match + reduce), then one lane per distinct bin adds that to the shared histogram.
constexpr float DIST_Q = 67108864.0f;  // 2^26

__device__ __forceinline__ void hist_add(unsigned long long* hist, uint32_t bin, uint32_t q, bool valid) {
  const uint32_t key = valid ? bin : 0xffffffffu;  // lanes without a weight form a group of their own
  const unsigned grp = __match_any_sync(0xffffffffu, key);
  const uint32_t sum = __reduce_add_sync(grp, q);  // <= 32 * 2^26
  if (valid && (int)(threadIdx.x & 31) == __ffs(grp) - 1) atomicAdd(&hist[bin], (unsigned long long)sum);
}

// One CTA per row: max, top-p boundary key, kept-set normaliser.
__global__ void __launch_bounds__(SM_THREADS)
row_dist_kernel(const uint16_t* __restrict__ logits, int V, long long ld, float temperature, float top_p,
                RowDist* __restrict__ out) {
  __shared__ float sh[32];
  __shared__ unsigned long long hist[256];
  __shared__ unsigned long long above_sh;
  __shared__ double goal_sh;
  __shared__ uint32_t sel;
  pdl_wait();
  pdl_trigger();
  const uint16_t* lp = logits + (size_t)blockIdx.x * ld;
  const float inv_t = 1.0f / temperature;
  float mx = -INFINITY;
  for (int v = threadIdx.x; v < V; v += SM_THREADS) {
    const uint16_t h = lp[v];
    if (bf_key(h)) mx = fmaxf(mx, bf(h));
  }
  const float m = block_max_1024(mx, sh);
  uint32_t thr = 0;
  if (top_p < 1.0f) {
    // level 1: mass per top key byte (every lane takes part in every step: the warp-wide match needs it)
    for (int i = threadIdx.x; i < 256; i += SM_THREADS) hist[i] = 0ull;
    __syncthreads();
    for (int base = 0; base < V; base += SM_THREADS) {
      const int v = base + threadIdx.x;
      const uint16_t h = v < V ? lp[v] : (uint16_t)0x7fffu;  // past the end: a NaN, no weight
      const uint32_t key = bf_key(h);
      const uint32_t q = key ? __float2uint_rn(expf((bf(h) - m) * inv_t) * DIST_Q) : 0u;
      hist_add(hist, key >> 8, q, key != 0u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long total = 0ull;
      for (int i = 0; i < 256; i++) total += hist[i];
      const double goal = (double)top_p * (double)total;
      unsigned long long cum = 0ull;
      uint32_t b = 0;
      for (int i = 255; i >= 0; i--) {
        cum += hist[i];
        if ((double)cum >= goal) {
          b = (uint32_t)i;
          break;
        }
      }
      sel = b;
      above_sh = cum - hist[b];  // mass strictly above the chosen bin
      goal_sh = goal;
    }
    __syncthreads();
    const uint32_t b1 = sel;
    const unsigned long long above = above_sh;
    const double goal = goal_sh;
    __syncthreads();
    // level 2: mass per low key byte inside bin b1
    for (int i = threadIdx.x; i < 256; i += SM_THREADS) hist[i] = 0ull;
    __syncthreads();
    for (int base = 0; base < V; base += SM_THREADS) {
      const int v = base + threadIdx.x;
      const uint16_t h = v < V ? lp[v] : (uint16_t)0x7fffu;
      const uint32_t key = bf_key(h);
      const bool in = key != 0u && (key >> 8) == b1;
      const uint32_t q = in ? __float2uint_rn(expf((bf(h) - m) * inv_t) * DIST_Q) : 0u;
      hist_add(hist, key & 0xffu, q, in);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      unsigned long long cum = above;
      uint32_t lo = 0;
      for (int i = 255; i >= 0; i--) {
        cum += hist[i];
        if ((double)cum >= goal) {
          lo = (uint32_t)i;
          break;
        }
      }
      sel = (b1 << 8) | lo;
    }
    __syncthreads();
    thr = sel;
  }
  // normaliser of the kept set, in a fixed order
  float s = 0.f;
  for (int v = threadIdx.x; v < V; v += SM_THREADS) {
    const uint16_t h = lp[v];
    const uint32_t key = bf_key(h);
    if (key && key >= thr) s += expf((bf(h) - m) * inv_t);
  }
  const float total = block_sum_1024(s, sh);
  if (threadIdx.x == 0) out[blockIdx.x] = RowDist{m, inv_t, total, thr};
}

__device__ __forceinline__ float dist_prob(const uint16_t* lp, const RowDist& d, int v) {
  const uint16_t h = lp[v];
  const uint32_t key = bf_key(h);
  if (!key || key < d.thr || !(d.s > 0.f)) return 0.f;
  return expf((bf(h) - d.m) * d.inv_t) / d.s;
}

// Block-wide inverse CDF over w_v, v < V (w from `weight(v)`), deterministic: per-thread contiguous
// segments summed in order, a fixed-order exclusive scan of the thread sums, then the owning thread walks
// its segment. Returns the token in every thread.
template <typename W>
__device__ int block_sample(int V, float u, W weight, float* sh_scan, int* sh_pick) {
  const int seg = (V + SM_THREADS - 1) / SM_THREADS;
  const int v0 = threadIdx.x * seg, v1 = min(V, v0 + seg);
  float local = 0.f;
  int last_pos = -1;
  for (int v = v0; v < v1; v++) {
    const float w = weight(v);
    local += w;
    if (w > 0.f) last_pos = v;
  }
  // fixed-order exclusive scan of the thread sums: warp shuffles, then the 32 warp totals in warp 0
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  float excl = __shfl_up_sync(0xffffffffu, incl, 1);
  if (lane == 0) excl = 0.f;
  if (threadIdx.x == 0) *sh_pick = -1;
  __syncthreads();
  if (lane == 31) sh_scan[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const float wt = sh_scan[lane];
    float winc = wt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, winc, o);
      if (lane >= o) winc += t;
    }
    float wex = __shfl_up_sync(0xffffffffu, winc, 1);
    if (lane == 0) wex = 0.f;
    __syncwarp();
    sh_scan[lane] = wex;
    if (lane == 31) sh_scan[SM_THREADS + 32] = winc;
  }
  __syncthreads();
  sh_scan[32 + threadIdx.x] = sh_scan[warp] + excl;  // this thread's exclusive prefix
  __syncthreads();
  const float total = sh_scan[SM_THREADS + 32];
  const float target = u * total;
  const float pre = sh_scan[32 + threadIdx.x];
  if (local > 0.f && pre <= target && (target < pre + local || threadIdx.x == SM_THREADS - 1)) {
    float acc = pre;
    int pick = last_pos;
    for (int v = v0; v < v1; v++) {
      acc += weight(v);
      if (acc > target) {
        pick = v;
        break;
      }
    }
    atomicMax(sh_pick, pick);  // at most a couple of candidates at a rounding edge: the higher segment wins
  }
  __syncthreads();
  int pick = *sh_pick;
  if (pick < 0) {
    // target at or past the total by rounding: the last token with weight
    __syncthreads();
    if (last_pos >= 0) atomicMax(sh_pick, last_pos);
    __syncthreads();
    pick = *sh_pick;
  }
  __syncthreads();
  return pick < 0 ? 0 : pick;
}

__global__ void __launch_bounds__(SM_THREADS)
accept_stochastic_kernel(const uint16_t* __restrict__ tl, const uint16_t* __restrict__ dl, int V, long long ld,
                         const RowDist* __restrict__ td, const RowDist* __restrict__ dd,
                         const int32_t* __restrict__ drafts, int drafts_ld, int k, unsigned long long seed,
                         unsigned long long offset0, const unsigned long long* __restrict__ offset_dev,
                         int32_t* __restrict__ out_tokens, int32_t* __restrict__ out_count,
                         float* __restrict__ ratios) {
  pdl_wait();
  pdl_trigger();
  const unsigned long long offset = offset0 + (offset_dev ? *offset_dev : 0ull);
  const int B = gridDim.x;
  __shared__ float scan[SM_THREADS + 33];
  __shared__ int pick;
  __shared__ int n_acc;
  const int b = blockIdx.x;
  const int32_t* dr = drafts + (size_t)b * drafts_ld;
  if (threadIdx.x == 0) {
    int n = 0;
    for (; n < k; n++) {
      const int d = dr[n];
      const int trow = b * (k + 1) + n, drow = n * B + b;
      const float p = (d >= 0 && d < V) ? dist_prob(tl + (size_t)trow * ld, td[trow], d) : 0.f;
      const float q = (d >= 0 && d < V) ? dist_prob(dl + (size_t)drow * ld, dd[drow], d) : 0.f;
      const float u = philox_uniform(seed, offset, (uint32_t)b, (uint32_t)(2 * n));
      if (ratios) ratios[(size_t)b * k + n] = q > 0.f ? p / q : (p > 0.f ? INFINITY : 0.f);
      if (!(u * q < p)) break;
    }
    n_acc = n;
  }
  __syncthreads();
  const int n = n_acc;
  int tok;
  if (n < k) {
    const int trow = b * (k + 1) + n, drow = n * B + b;
    const uint16_t* tp = tl + (size_t)trow * ld;
    const uint16_t* dp = dl + (size_t)drow * ld;
    const RowDist t = td[trow], d = dd[drow];
    const float u = philox_uniform(seed, offset, (uint32_t)b, (uint32_t)(2 * n + 1));
    tok = block_sample(V, u, [&](int v) { return fmaxf(dist_prob(tp, t, v) - dist_prob(dp, d, v), 0.f); }, scan, &pick);
    // p == q everywhere leaves no residual mass: sample from p
    __syncthreads();
    if (scan[SM_THREADS + 32] <= 0.f) tok = block_sample(V, u, [&](int v) { return dist_prob(tp, t, v); }, scan, &pick);
  } else {
    const int trow = b * (k + 1) + k;
    const uint16_t* tp = tl + (size_t)trow * ld;
    const RowDist t = td[trow];
    const float u = philox_uniform(seed, offset, (uint32_t)b, (uint32_t)(2 * k));
    tok = block_sample(V, u, [&](int v) { return dist_prob(tp, t, v); }, scan, &pick);
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < n; i++) out_tokens[(size_t)b * (k + 1) + i] = dr[i];
    out_tokens[(size_t)b * (k + 1) + n] = tok;
    for (int i = n + 1; i <= k; i++) out_tokens[(size_t)b * (k + 1) + i] = -1;
    out_count[b] = n + 1;
  }
}

__global__ void __launch_bounds__(SM_THREADS)
sample_kernel(const uint16_t* __restrict__ logits, int V, long long ld, const RowDist* __restrict__ dist,
              const uint32_t* __restrict__ streams, uint32_t draw, unsigned long long seed, unsigned long long offset0,
              const unsigned long long* __restrict__ offset_dev, int32_t* __restrict__ out, int out_stride) {
  pdl_wait();
  pdl_trigger();
  const unsigned long long offset = offset0 + (offset_dev ? *offset_dev : 0ull);
  __shared__ float scan[SM_THREADS + 33];
  __shared__ int pick;
  const int r = blockIdx.x;
  const uint16_t* lp = logits + (size_t)r * ld;
  const RowDist d = dist[r];
  const uint32_t stream = streams ? streams[r] : (uint32_t)r;
  const float u = philox_uniform(seed, offset, stream, draw);
  const int tok = block_sample(V, u, [&](int v) { return dist_prob(lp, d, v); }, scan, &pick);
  if (threadIdx.x == 0) out[(size_t)r * out_stride] = tok;
}

__global__ void philox_kernel(unsigned long long seed, unsigned long long offset, uint32_t stream, uint32_t n,
                              uint32_t* out) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  uint32_t c[4] = {(uint32_t)offset, (uint32_t)(offset >> 32), stream, i};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  out[4 * i + 0] = c[0];
  out[4 * i + 1] = c[1];
  out[4 * i + 2] = c[2];
  out[4 * i + 3] = c[3];
}

}  // namespace im

using namespace im;

extern "C" size_t im_sampling_workspace_bytes(int64_t rows) {
  return rows < 1 ? 0 : (size_t)rows * sizeof(RowDist) + 256;
}

static int check_common(const uint16_t* logits, int64_t rows, int64_t V, int64_t ld, float temperature, float top_p) {
  IM_REQUIRE(logits && rows >= 1 && rows < (1ll << 31) && V >= 1 && V < (1ll << 31) && ld >= V, IM_INVALID,
             "sampling: bad logits or sizes");
  IM_REQUIRE(temperature > 0.f && isfinite(temperature), IM_INVALID,
             "sampling: temperature must be > 0 (use the greedy kernels for temperature 0)");
  IM_REQUIRE(top_p > 0.f && top_p <= 1.f, IM_INVALID, "sampling: top_p must be in (0, 1]");
  return IM_OK;
}

extern "C" int im_sample_rows(const uint16_t* logits, int64_t rows, int64_t V, int64_t ld, float temperature,
                              float top_p, uint64_t seed, uint64_t offset, const uint64_t* offset_dev,
                              const uint32_t* streams, uint32_t draw, int32_t* out, int64_t out_stride,
                              void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  int rc = check_common(logits, rows, V, ld, temperature, top_p);
  if (rc) return rc;
  IM_REQUIRE(out && out_stride >= 1 && workspace && workspace_bytes >= im_sampling_workspace_bytes(rows),
             IM_INVALID, "im_sample_rows: null output or short workspace");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  RowDist* dist = reinterpret_cast<RowDist*>(workspace);
  rc = launch("row_dist_kernel", row_dist_kernel, dim3((unsigned)rows), dim3(SM_THREADS), 0, st, logits, (int)V,
              (long long)ld, temperature, top_p, dist);
  if (rc) return rc;
  return launch("sample_kernel", sample_kernel, dim3((unsigned)rows), dim3(SM_THREADS), 0, st, logits, (int)V,
                (long long)ld, (const RowDist*)dist, streams, draw, (unsigned long long)seed, (unsigned long long)offset,
                reinterpret_cast<const unsigned long long*>(offset_dev), out, (int)out_stride);
}

extern "C" int im_accept_stochastic(const uint16_t* target_logits, const uint16_t* draft_logits, int64_t B,
                                    int64_t k, int64_t V, int64_t ld, const int32_t* drafts, int64_t drafts_ld,
                                    float temperature, float top_p, uint64_t seed, uint64_t offset,
                                    const uint64_t* offset_dev, int32_t* out_tokens, int32_t* out_count,
                                    float* ratios, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  IM_REQUIRE(B >= 1 && B < 65536 && k >= 1 && k <= 64 && drafts && drafts_ld >= k && out_tokens && out_count,
             IM_INVALID, "im_accept_stochastic: bad sizes or null pointer");
  int rc = check_common(target_logits, B * (k + 1), V, ld, temperature, top_p);
  if (rc) return rc;
  IM_REQUIRE(draft_logits, IM_INVALID, "im_accept_stochastic: null draft logits");
  const int64_t rows = B * (k + 1) + B * k;
  IM_REQUIRE(workspace && workspace_bytes >= im_sampling_workspace_bytes(rows), IM_INVALID,
             "im_accept_stochastic: workspace of %zu bytes needed", im_sampling_workspace_bytes(rows));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  RowDist* td = reinterpret_cast<RowDist*>(workspace);
  RowDist* dd = td + B * (k + 1);
  rc = launch("row_dist_kernel", row_dist_kernel, dim3((unsigned)(B * (k + 1))), dim3(SM_THREADS), 0, st,
              target_logits, (int)V, (long long)ld, temperature, top_p, td);
  if (rc) return rc;
  rc = launch("row_dist_kernel", row_dist_kernel, dim3((unsigned)(B * k)), dim3(SM_THREADS), 0, st, draft_logits,
              (int)V, (long long)ld, temperature, top_p, dd);
  if (rc) return rc;
  return launch("accept_stochastic_kernel", accept_stochastic_kernel, dim3((unsigned)B), dim3(SM_THREADS), 0, st,
                target_logits, draft_logits, (int)V, (long long)ld, (const RowDist*)td, (const RowDist*)dd, drafts,
                (int)drafts_ld, (int)k, (unsigned long long)seed, (unsigned long long)offset,
                reinterpret_cast<const unsigned long long*>(offset_dev), out_tokens, out_count, ratios);
}

extern "C" int im_philox4x32_10(uint64_t seed, uint64_t offset, uint32_t stream_id, uint32_t n, uint32_t* out,
                                void* stream) {
  clear_error();
  IM_REQUIRE(out && n >= 1, IM_INVALID, "im_philox4x32_10: null output");
  philox_kernel<<<(n + 255) / 256, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(seed, offset, stream_id, n, out);
  return check_launch("philox_kernel");
}
