// Vocab-wide row statistics and greedy acceptance, on the device.
//
// Replaces the host numpy scans of IronMule ironmule/ggml_engine.py:669-683 (_decode_conf: argmax and
// p_top = 1 / sum exp(row - row[top])) and :848 (argmax per verified row), and the host `accept`
// (ironmule/speculation.py:103-108) that consumes them.
//
// One launch: the rows are cut into chunks; each CTA scans one chunk of one row with 128-bit loads and
// keeps (max, lowest index of the max, sum of exp(v - max)) with an online rescale; CTAs publish their
// triple and the last CTA to finish (one atomic counter) combines the chunks of every row in chunk
// order and, for greedy verification, applies the acceptance rule per sequence.
#include <math.h>

#include "common.cuh"

namespace im {

constexpr int AM_THREADS = 256;

struct RowStat {
  float m;    // running max
  int idx;    // lowest index holding m
  float s;    // sum of exp(v - m)
};

__device__ __forceinline__ void stat_push(RowStat& a, float v, int i) {
  if (v > a.m) {
    a.s = (a.m == -INFINITY ? 0.f : a.s * __expf(a.m - v)) + 1.f;
    a.m = v;
    a.idx = i;
  } else {
    if (v == a.m && i < a.idx) a.idx = i;
    if (v > -INFINITY) a.s += __expf(v - a.m);
  }
}

__device__ __forceinline__ RowStat stat_merge(const RowStat& a, const RowStat& b) {
  RowStat r;
  if (a.m > b.m || (a.m == b.m && a.idx <= b.idx)) {
    r.m = a.m;
    r.idx = a.idx;
  } else {
    r.m = b.m;
    r.idx = b.idx;
  }
  const float sa = a.m == -INFINITY ? 0.f : a.s * __expf(a.m - r.m);
  const float sb = b.m == -INFINITY ? 0.f : b.s * __expf(b.m - r.m);
  r.s = sa + sb;
  return r;
}

__device__ __forceinline__ RowStat stat_shfl(const RowStat& a, int off) {
  RowStat b;
  b.m = __shfl_xor_sync(0xffffffffu, a.m, off);
  b.idx = __shfl_xor_sync(0xffffffffu, a.idx, off);
  b.s = __shfl_xor_sync(0xffffffffu, a.s, off);
  return b;
}

struct AmWork {
  unsigned* counter;
  RowStat* part;  // [rows][chunks]
};

__global__ void __launch_bounds__(AM_THREADS)
argmax_kernel(const uint16_t* __restrict__ logits, int rows, int V, long long ld, int chunks, int chunk_len,
              int32_t* argmax, int out_stride, float* conf, AmWork work, int B, int k,
              const int32_t* __restrict__ drafts, int drafts_ld,
              int32_t* out_tokens, int32_t* out_count) {
  pdl_wait();
  pdl_trigger();
  const int chunk = blockIdx.x, row = blockIdx.y;
  const int v0 = chunk * chunk_len;
  const int v1 = min(V, v0 + chunk_len);
  const uint16_t* lp = logits + (size_t)row * ld;
  RowStat st{-INFINITY, 0x7fffffff, 0.f};
  const bool vec = ((reinterpret_cast<uintptr_t>(lp) & 15) == 0) && ((v0 & 7) == 0);
  if (vec) {
    const int nvec = (v1 - v0) >> 3;
    for (int i = threadIdx.x; i < nvec; i += AM_THREADS) {
      const uint4 q = ldg_stream_u4(lp + v0 + i * 8);
      const int base = v0 + i * 8;
      stat_push(st, bf_lo(q.x), base + 0);
      stat_push(st, bf_hi(q.x), base + 1);
      stat_push(st, bf_lo(q.y), base + 2);
      stat_push(st, bf_hi(q.y), base + 3);
      stat_push(st, bf_lo(q.z), base + 4);
      stat_push(st, bf_hi(q.z), base + 5);
      stat_push(st, bf_lo(q.w), base + 6);
      stat_push(st, bf_hi(q.w), base + 7);
    }
    for (int v = v0 + nvec * 8 + threadIdx.x; v < v1; v += AM_THREADS) stat_push(st, bf(lp[v]), v);
  } else {
    for (int v = v0 + threadIdx.x; v < v1; v += AM_THREADS) stat_push(st, bf(lp[v]), v);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) st = stat_merge(st, stat_shfl(st, off));
  __shared__ RowStat wst[AM_THREADS / 32];
  __shared__ bool last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) wst[warp] = st;
  __syncthreads();
  if (threadIdx.x == 0) {
    RowStat r = wst[0];
    for (int w = 1; w < AM_THREADS / 32; w++) r = stat_merge(r, wst[w]);
    work.part[(size_t)row * chunks + chunk] = r;
    __threadfence();
    const unsigned total = (unsigned)(gridDim.x * gridDim.y);
    last = atomicAdd(work.counter, 1u) == total - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // The last CTA: combine every row's chunks in chunk order.
  for (int r = threadIdx.x; r < rows; r += AM_THREADS) {
    RowStat acc{-INFINITY, 0x7fffffff, 0.f};
    for (int c = 0; c < chunks; c++) {
      RowStat p;
      const RowStat* src = work.part + (size_t)r * chunks + c;
      p.m = __ldcg(&src->m);
      p.idx = __ldcg(&src->idx);
      p.s = __ldcg(&src->s);
      acc = stat_merge(acc, p);
    }
    const int best = acc.idx == 0x7fffffff ? 0 : acc.idx;
    if (argmax) argmax[(size_t)r * out_stride] = best;
    if (conf) conf[r] = acc.s > 0.f ? 1.0f / acc.s : 0.f;
    if (out_count) work.part[(size_t)r * chunks].idx = best;  // hand the pick to the acceptance step
  }
  if (out_count) {
    __syncthreads();  // the picks above were written by this block; plain loads see them
    const RowStat* picks = work.part;
    for (int b = threadIdx.x; b < B; b += AM_THREADS) {
      const int base = b * (k + 1);
      int n = 0;
      while (n < k && drafts[(size_t)b * drafts_ld + n] == picks[(size_t)(base + n) * chunks].idx) n++;
      for (int i = 0; i < n; i++) out_tokens[(size_t)b * (k + 1) + i] = drafts[(size_t)b * drafts_ld + i];
      out_tokens[(size_t)b * (k + 1) + n] = picks[(size_t)(base + n) * chunks].idx;
      for (int i = n + 1; i <= k; i++) out_tokens[(size_t)b * (k + 1) + i] = -1;
      out_count[b] = n + 1;
    }
  }
  if (threadIdx.x == 0) *work.counter = 0u;
}

static void am_plan(int64_t rows, int64_t V, int* chunks, int* chunk_len) {
  int c = (int)((296 + rows - 1) / rows);
  const int cap = (int)((V + 4095) / 4096);
  c = c < 1 ? 1 : (c > cap ? cap : c);
  int len = (int)((V + c - 1) / c);
  len = (len + 7) / 8 * 8;
  *chunks = (int)((V + len - 1) / len);
  *chunk_len = len;
}

static size_t am_bytes(int64_t rows, int64_t V) {
  int chunks, len;
  am_plan(rows, V, &chunks, &len);
  return 256 + (size_t)rows * chunks * sizeof(RowStat);
}

static int am_launch(const uint16_t* logits, int64_t rows, int64_t V, int64_t ld, int32_t* argmax,
                     int64_t out_stride, float* conf, int B, int k, const int32_t* drafts, int64_t drafts_ld,
                     int32_t* out_tokens, int32_t* out_count, void* workspace,
                     size_t workspace_bytes, void* stream) {
  IM_REQUIRE(rows >= 1 && rows <= 65535 && V >= 1 && V < (1ll << 31) && ld >= V, IM_INVALID,
             "argmax: bad sizes rows=%lld V=%lld ld=%lld", (long long)rows, (long long)V, (long long)ld);
  IM_REQUIRE(logits && workspace, IM_INVALID, "argmax: null logits or workspace");
  IM_REQUIRE(aligned(logits, 2) && aligned(workspace, 256), IM_INVALID, "argmax: misaligned buffer");
  const size_t need = am_bytes(rows, V);
  IM_REQUIRE(workspace_bytes >= need, IM_INVALID, "argmax: workspace of %zu bytes needed, %zu given", need,
             workspace_bytes);
  int chunks, len;
  am_plan(rows, V, &chunks, &len);
  AmWork work{reinterpret_cast<unsigned*>(workspace),
              reinterpret_cast<RowStat*>(reinterpret_cast<char*>(workspace) + 256)};
  dim3 grid(chunks, (unsigned)rows);
  return launch("argmax_kernel", argmax_kernel, grid, dim3(AM_THREADS), 0, reinterpret_cast<cudaStream_t>(stream),
                logits, (int)rows, (int)V, (long long)ld, chunks, len, argmax, (int)out_stride, conf, work, B, k,
                drafts, (int)drafts_ld, out_tokens, out_count);
}

}  // namespace im

using namespace im;

extern "C" size_t im_argmax_workspace_bytes(int64_t rows, int64_t V) {
  if (rows < 1 || V < 1) return 0;
  return am_bytes(rows, V);
}

extern "C" int im_argmax_rows(const uint16_t* logits, int64_t rows, int64_t V, int64_t ld, int32_t* argmax,
                              int64_t argmax_stride, float* conf, void* workspace, size_t workspace_bytes,
                              void* stream) {
  clear_error();
  IM_REQUIRE(argmax && argmax_stride >= 1, IM_INVALID, "im_argmax_rows: null argmax output or bad stride");
  return am_launch(logits, rows, V, ld, argmax, argmax_stride, conf, 0, 0, nullptr, 0, nullptr, nullptr, workspace,
                   workspace_bytes, stream);
}

extern "C" int im_verify_greedy(const uint16_t* logits, int64_t B, int64_t k, int64_t V, int64_t ld,
                                const int32_t* drafts, int64_t drafts_ld, int32_t* out_tokens, int32_t* out_count,
                                int32_t* argmax_out, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  IM_REQUIRE(B >= 1 && k >= 0 && k <= 64 && drafts_ld >= k, IM_INVALID, "im_verify_greedy: bad B=%lld k=%lld",
             (long long)B, (long long)k);
  IM_REQUIRE(out_tokens && out_count && (k == 0 || drafts), IM_INVALID, "im_verify_greedy: null output");
  return am_launch(logits, B * (k + 1), V, ld, argmax_out, 1, nullptr, (int)B, (int)k, drafts, drafts_ld,
                   out_tokens, out_count, workspace, workspace_bytes, stream);
}
