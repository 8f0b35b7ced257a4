// qGEMM v4: the engine's 4-bit GEMM over weights repacked once at load into MMA-fragment order.
//
// Packed format (im_qgemm_pack_w4g64): rows padded to 32-row tiles; unit (tile, group) = 1152 contiguous bytes,
// units in tile-major, group-minor order:
//   codes, 1024 B: lane L (g = L/4, t = L%4) owns bytes [32L, 32L+32) = the 8-byte slice (words 2t, 2t+1 of the
//     group) of rows g, g+8, 16+g, 24+g of the tile -- exactly the A fragments of the lane's two 16-row MMAs;
//   scales/biases, 128 B: for g = 0..7, 16 bytes = bf16 scale of rows g, g+8, 16+g, 24+g then their biases.
// So a warp streams one contiguous 1152-byte unit per group: two 16-byte code loads and one broadcast 16-byte
// scale/bias load per lane. (MLX's own layout stays the drop-in format of im_qgemm_w4g64; the engine repacks
// its resident weights once.)
//
// The arithmetic is the warp-MMA kernel's (exact bf16 codes 128+q, fp32 group affine s*acc + (b-128 s)*sum(x)).
// A CTA is 4 warps = 4 consecutive tiles (128 rows) over a K range (CTAs split K when needed); its prologue stages
// the activation fragments and per-group sums of its K range in shared memory once, optionally applying RMSNorm
// on the way in: inv_rms of each activation row comes from per-tile sums of squares that the previous residual
// GEMM (or the embedding) wrote, summed in tile order. A residual epilogue can write those sums for the next GEMM.
// Partition (tiles x K splits) depends on (N, K) only; rows are independent: a row's bits do not depend on M.
#include "common.cuh"
#include "attention.cuh"
#include "qgemm_packed.cuh"
#include "../../include/imspec.h"

namespace im {

constexpr int Q4_WARPS = 4;
constexpr int Q4_THREADS = Q4_WARPS * 32;
constexpr int Q4_DEPTH = 3;               // units in flight per warp
static int g_q4_split_override = 0;       // sweep hook (0 = automatic)
static int g_q4_target_ctas = 148 * 4;    // split policy: at most this many CTAs (one wave at 4 per SM)
static int g_q4_max_split = Q4_MAX_SPLITS;
static int g_q4_cluster = 1;             // reduce split-K partials inside a thread-block cluster when possible
static int g_q4_path = 0;                 // 0: automatic, 1: warp MMA always, 2: tensor cores always

// The tensor-core kernel wins where an item streams many groups for many rows. Measured on B200 whole rounds,
// with the kernel's 16 epilogue warps: config 3 (Qwen3-4B verification at 160 rows) 37.5 ms from 128 rows against
// 38.6 ms from 192; config 5a (Gemma-3-27B) even. So: from 128 rows with at most 16 K splits.
static bool q4_tensor_cores(int64_t M, int splits) {
  if (g_q4_path == 2) return true;
  if (g_q4_path == 1) return false;
  return M >= 128 && splits <= 16;
}
constexpr uint32_t Q4_128 = 0x43004300u;

__device__ __forceinline__ void q4_mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void q4_codes(uint32_t u, uint32_t* p) {
  p[0] = (u & 0x000F000Fu) | Q4_128;
  p[1] = ((u >> 4) & 0x000F000Fu) | Q4_128;
  p[2] = ((u >> 8) & 0x000F000Fu) | Q4_128;
  p[3] = ((u >> 12) & 0x000F000Fu) | Q4_128;
}

__device__ __forceinline__ uint4 q4_ld_stream(const void* p) { return ldg_stream_u4(p); }
// Asks the TMA unit to bring [p, p + bytes) into L2 (p 16-byte aligned, bytes a multiple of 16); no data
// reaches the CTA and nothing waits on it.
__device__ __forceinline__ void q4_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ---- repack ---------------------------------------------------------------------------------------------
__global__ void q4_pack_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ sc,
                               const uint16_t* __restrict__ bi, int N, int K, unsigned char* __restrict__ out) {
  const int G = K >> 6;
  const long long unit = blockIdx.x;  // tile * G + group
  const int tile = (int)(unit / G), grp = (int)(unit % G);
  unsigned char* dst = out + unit * Q4_UNIT;
  const int lane = threadIdx.x;  // 32 threads
  const int g = lane >> 2, t = lane & 3;
  const int rows[4] = {g, g + 8, 16 + g, 24 + g};
  uint32_t words[8];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int r = tile * 32 + rows[j];
    if (r < N) {
      const uint32_t* src = w + (size_t)r * (K >> 3) + grp * 8 + 2 * t;
      words[2 * j] = src[0];
      words[2 * j + 1] = src[1];
    } else {
      words[2 * j] = words[2 * j + 1] = 0u;
    }
  }
  uint4* d = reinterpret_cast<uint4*>(dst + lane * 32);
  d[0] = make_uint4(words[0], words[1], words[2], words[3]);
  d[1] = make_uint4(words[4], words[5], words[6], words[7]);
  if (t == 0) {
    uint16_t sb[8];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const int r = tile * 32 + rows[j];
      sb[j] = r < N ? sc[(size_t)r * G + grp] : (uint16_t)0;
      sb[4 + j] = r < N ? bi[(size_t)r * G + grp] : (uint16_t)0;
    }
    uint4 v;
    v.x = (uint32_t)sb[0] | ((uint32_t)sb[1] << 16);
    v.y = (uint32_t)sb[2] | ((uint32_t)sb[3] << 16);
    v.z = (uint32_t)sb[4] | ((uint32_t)sb[5] << 16);
    v.w = (uint32_t)sb[6] | ((uint32_t)sb[7] << 16);
    *reinterpret_cast<uint4*>(dst + 1024 + g * 16) = v;
  }
}

// ---- the GEMM -------------------------------------------------------------------------------------------
// Dynamic shared memory, for rg = the most groups a split holds:
//   xf   [rg][NT][32 lanes][2 x 16 B]  activation fragments (the RMSNorm partial sums are staged here first)
//   sxs  [rg][NT*8]                    group sums of the activations
//   inv  [32]                          RMSNorm factors
//   part [4 warps][2*NT*4][32 lanes]   this CTA's split-K partials, read by the cluster's reducing CTA
//   xs   [8 rows][rg * 64]             merged attention output of the K range (attention-merge input only)
struct Q4Smem {
  size_t xf, sxs, inv, part, xs, total;
};
__host__ __device__ inline Q4Smem q4_smem(int nt, int rg, int norm_parts, bool am = false) {
  Q4Smem m;
  const size_t xf = (size_t)rg * nt * 32 * 32;
  const size_t nsum = (size_t)norm_parts * nt * 8 * 4;
  m.xf = 0;
  m.sxs = (xf > nsum ? xf : nsum + 15) / 16 * 16;
  m.inv = m.sxs + (size_t)rg * nt * 8 * 4;
  m.part = m.inv + 32 * 4;
  m.xs = m.part + (size_t)Q4_WARPS * 2 * nt * 4 * 32 * 4;
  m.total = m.xs + (am ? (size_t)8 * rg * 64 * 2 : 0);
  return m;
}

// ---- thread-block cluster helpers (split-K partials reduced through distributed shared memory) -------------
__device__ __forceinline__ unsigned q4_cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void q4_cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void q4_cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
// The shared::cluster address of the same shared-memory location in cluster CTA `rank`.
__device__ __forceinline__ uint32_t q4_mapa(const void* local, unsigned rank) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(local);
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
__device__ __forceinline__ float q4_ld_dsmem(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// The epilogue of one tile's warp: SwiGLU / GeGLU, or store / residual add with the per-row sums of squares of the
// written rows. rres holds the residual when it was loaded before the main loop (RES_EARLY).
template <int NT, int EPI, bool RES_EARLY>
__device__ __forceinline__ void q4_epilogue(const Q4Args& a, const float (&tot)[2][NT][4],
                                            const uint16_t (&rres)[2][NT][4], int tile, int g, int t) {
  const int rbase = tile * 32;
  if constexpr (EPI == IM_EPI_SWIGLU || EPI == IM_EPI_GEGLU) {
    const int nout = a.N >> 1;
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const int f = (rbase >> 1) + g + ((e >> 1) << 3);
        const int m = nt * 8 + 2 * t + (e & 1);
        if (m < a.M && f < nout) {
          const float ga = round_bf(tot[0][nt][e]), uu = round_bf(tot[1][nt][e]);
          float o;
          if (EPI == IM_EPI_SWIGLU) {
            const float sig = round_bf(1.0f / (1.0f + expf(-ga)));
            o = round_bf(ga * sig) * uu;
          } else {
            const float inner = 0.7978845608028654f * (ga + 0.044715f * ga * ga * ga);
            o = round_bf(0.5f * ga * (1.0f + tanhf(inner))) * uu;
          }
          a.y[(size_t)m * nout + f] = to_bf(o);
        }
      }
  } else {
    float sq[NT][2] = {};
#pragma unroll
    for (int tt = 0; tt < 2; tt++)
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int r = rbase + tt * 16 + g + ((e >> 1) << 3);
          const int m = nt * 8 + 2 * t + (e & 1);
          if (m < a.M && r < a.N) {
            const size_t o = (size_t)m * a.N + r;
            const uint16_t rv = EPI != IM_EPI_RESIDUAL ? (uint16_t)0 : (RES_EARLY ? rres[tt][nt][e] : a.res[o]);
            const uint16_t h = EPI == IM_EPI_RESIDUAL ? to_bf(bf(rv) + round_bf(tot[tt][nt][e])) : to_bf(tot[tt][nt][e]);
            a.y[o] = h;
            const float hv = bf(h);
            sq[nt][e & 1] = fmaf(hv, hv, sq[nt][e & 1]);
          }
        }
    if (a.out_sq) {
      // per activation row m: the sum over this tile's 32 rows, fixed order (lanes with the same t)
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
          float v = sq[nt][e];
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          v += __shfl_xor_sync(0xffffffffu, v, 8);
          v += __shfl_xor_sync(0xffffffffu, v, 16);
          const int m = nt * 8 + 2 * t + e;
          if (g == 0 && m < a.M) a.out_sq[(size_t)tile * a.sq_ld + m] = v;
        }
    }
  }
}

// grid (CTA columns of 4 tiles, K splits, 32-row chunks). A chunk is computed exactly as a call of its rows alone
// would be: the same plan, its own split-K counters and partials. CL: the K splits of a CTA column form one
// thread-block cluster and their partials are summed through distributed shared memory (no global atomics);
// otherwise the last split to arrive at a global counter sums them. Both sum in split order: the same bits.
// Up to 8 rows: four CTAs per SM (128 registers a thread; at five the prologue's loads spilled and the config-2
// round took 6.54 ms against 6.32), and the split plan keeps the grid within one wave of them.
// AM: the input rows are merged from attention split partials in the prologue (up to 8 rows, one merge job of
// 4 values per thread).
template <int NT, int EPI, bool CL, bool AM = false>
__global__ void __launch_bounds__(Q4_THREADS, NT == 1 ? 4 : 1)
qgemm_packed_kernel(Q4Args a) {
  extern __shared__ __align__(16) unsigned char q4_raw[];
  if (gridDim.z > 1) {  // this CTA's 32-row chunk
    const int m0 = blockIdx.z * 32;
    const int nout = (EPI == IM_EPI_SWIGLU || EPI == IM_EPI_GEGLU) ? a.N >> 1 : a.N;
    a.x += (size_t)m0 * a.K;
    a.y += (size_t)m0 * nout;
    if (a.res) a.res += (size_t)m0 * a.N;
    if (a.norm_sq) a.norm_sq += m0;
    if (a.out_sq) a.out_sq += m0;
    a.counters += (size_t)blockIdx.z * a.tiles;
    a.partial += (size_t)blockIdx.z * a.tiles * a.splits * (2 * 4 * 4 * 32);
    a.M = min(32, a.M - m0);
  }
  const Q4Smem lay = q4_smem(NT, a.rg, a.norm_w ? a.norm_parts : 0, AM);
  uint4 (*xf)[NT][32][2] = reinterpret_cast<uint4 (*)[NT][32][2]>(q4_raw + lay.xf);
  float (*sxs)[NT * 8] = reinterpret_cast<float (*)[NT * 8]>(q4_raw + lay.sxs);
  float* inv_s = reinterpret_cast<float*>(q4_raw + lay.inv);
  float* part_s = reinterpret_cast<float*>(q4_raw + lay.part);
  const int G = a.K >> 6;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int split = blockIdx.y;
  const int cg0 = (int)(((long long)G * split) / a.splits);
  const int cg1 = (int)(((long long)G * (split + 1)) / a.splits);
  const int ng = cg1 - cg0;
  const int tile = blockIdx.x * Q4_WARPS + warp;
  const bool live = tile < a.tiles;
  // the warp that finishes this tile: the last split to arrive (global counter), or in a cluster the CTA of rank
  // warp % splits (so the four tiles of a column are finished by up to four CTAs)
  const bool reducer = CL && a.splits > 1 ? (int)q4_cluster_rank() == warp % a.splits : true;

  // ---- before the dependency wait: this warp's weights (which no earlier kernel writes). Its slice is ng
  // consecutive 1152-byte units; the first Q4_DEPTH go to registers, the rest are prefetched into L2.
  const unsigned char* up = a.wp + ((size_t)(live ? tile : 0) * G + cg0) * Q4_UNIT;
  uint4 rc0[Q4_DEPTH], rc1[Q4_DEPTH], rsb[Q4_DEPTH];
  if (live) {
    if (lane == 0)
      for (int u = Q4_DEPTH; u < ng; u += 16)  // pieces of at most 16 units (18 KB)
        q4_prefetch_l2(up + (size_t)u * Q4_UNIT, (uint32_t)min(16, ng - u) * Q4_UNIT);
#pragma unroll
    for (int d = 0; d < Q4_DEPTH; d++) {
      if (d < ng) {
        const unsigned char* nu = up + (size_t)d * Q4_UNIT;
        rc0[d] = q4_ld_stream(nu + lane * 32);
        rc1[d] = q4_ld_stream(nu + lane * 32 + 16);
        rsb[d] = __ldg(reinterpret_cast<const uint4*>(nu + 1024 + g * 16));
      }
    }
  }
  // attention-merge input: this thread's merge job (row m, 4 values at K offset 4c of the CTA's range) and where
  // its partials sit, from row metadata no earlier kernel of the layer writes
  const float* am_base = nullptr;
  int am_used = 0, am_d4 = 0;
  if constexpr (AM) {
    const int m = (int)threadIdx.x / (ng * 16), c = (int)threadIdx.x % (ng * 16);
    if (m < a.M) {
      int b = 0;
      while (b + 1 < a.am.B && a.am.seq_rows[b + 1] <= m) b++;
      const int lr = m - a.am.seq_rows[b];
      am_used = min(a.am.nsplit, a.am.row_slot[m] / a.am.kpc + 1);
      const int k = cg0 * 64 + 4 * c, h = k / a.am.D, G = a.am.Hq / a.am.Hkv;
      am_d4 = k % a.am.D;
      const int flat = lr * G + h % G;
      const size_t group = ((size_t)b * a.am.Hkv + h / G) * a.am.qblocks + flat / a.am.nq;
      am_base = a.am.part + (group * a.am.nsplit * a.am.nq + flat % a.am.nq) * (size_t)(a.am.D + AT_PAD);
    }
  }
  pdl_wait();
  pdl_trigger();

  // the residual this warp's epilogue adds, loaded now so that its latency hides behind the main loop
  constexpr bool RES_EARLY = EPI == IM_EPI_RESIDUAL && NT <= 2;
  uint16_t rres[2][NT][4];
  if constexpr (RES_EARLY) {
#pragma unroll
    for (int tt = 0; tt < 2; tt++)
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) {
          const int r = tile * 32 + tt * 16 + g + ((e >> 1) << 3);
          const int m = nt * 8 + 2 * t + (e & 1);
          rres[tt][nt][e] = live && reducer && m < a.M && r < a.N ? a.res[(size_t)m * a.N + r] : (uint16_t)0;
        }
  }

  // ---- prologue: RMSNorm factors, then the activation fragments and group sums of [cg0, cg1). This thread's
  // first activation slice is loaded before the RMSNorm factors, so that the two loads are in flight together.
  uint16_t* xs = reinterpret_cast<uint16_t*>(q4_raw + lay.xs);
  if constexpr (AM) {
    // the attention output of this CTA's K range, merged from the split partials exactly as the attention's own
    // merge does it, into shared memory
    if (am_base) {
      uint16_t o4[4];
      attn_merge4(am_base, (size_t)a.am.nq * (a.am.D + AT_PAD), am_d4, am_used, a.am.D, o4);
      const int m = (int)threadIdx.x / (ng * 16), c = (int)threadIdx.x % (ng * 16);
      uint2 w;
      w.x = (uint32_t)o4[0] | ((uint32_t)o4[1] << 16);
      w.y = (uint32_t)o4[2] | ((uint32_t)o4[3] << 16);
      *reinterpret_cast<uint2*>(xs + (size_t)m * a.rg * 64 + 4 * c) = w;
    }
    __syncthreads();
  }
  uint4 pre_lo = make_uint4(0, 0, 0, 0), pre_hi = pre_lo;
  if constexpr (!AM) {
    const int job = threadIdx.x;
    const int tq = job & 3, m = (job >> 2) % (NT * 8), gl = (job >> 2) / (NT * 8);
    if (job < ng * NT * 32 && m < a.M) {
      const uint16_t* xp = a.x + (size_t)m * a.K + (size_t)(cg0 + gl) * 64 + 16 * tq;
      pre_lo = __ldg(reinterpret_cast<const uint4*>(xp));
      pre_hi = __ldg(reinterpret_cast<const uint4*>(xp + 8));
    }
  }
  if (a.norm_w) {
    // the per-tile sums of squares of every activation row, all loaded at once, then summed in tile order
    constexpr int ROWS = NT * 8;
    float* nsum = reinterpret_cast<float*>(q4_raw + lay.xf);  // the fragments are written after this
    const int total = a.norm_parts * ROWS;
    for (int i0 = 0; i0 < total; i0 += 8 * Q4_THREADS) {
      float v[8];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int i = i0 + j * Q4_THREADS + threadIdx.x;
        const int pp = i / ROWS, m = i - pp * ROWS;
        v[j] = i < total && m < a.M ? a.norm_sq[(size_t)pp * a.sq_ld + m] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const int i = i0 + j * Q4_THREADS + threadIdx.x;
        if (i < total) nsum[i] = v[j];
      }
    }
    __syncthreads();
    for (int m = threadIdx.x; m < ROWS; m += Q4_THREADS) {
      float s = 0.f;
      if (m < a.M) {
#pragma unroll 8
        for (int pp = 0; pp < a.norm_parts; pp++) s += nsum[pp * ROWS + m];
      }
      inv_s[m] = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(s, (float)a.K) + a.eps));
    }
    __syncthreads();
  }
  // one thread per (group, activation row m, quarter t): 16 values -> fragment order + partial sum
  for (int job = threadIdx.x; job < ng * NT * 32; job += Q4_THREADS) {
    const bool first = job == (int)threadIdx.x;
    const int tq = job & 3;
    const int m = (job >> 2) % (NT * 8);
    const int gl = (job >> 2) / (NT * 8);
    const int grp = cg0 + gl;
    uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
    float part = 0.f;
    if (m < a.M) {
      if constexpr (AM) {
        const uint4* xp = reinterpret_cast<const uint4*>(xs + (size_t)m * a.rg * 64 + gl * 64 + 16 * tq);
        lo = xp[0];
        hi = xp[1];
      } else if (first) {
        lo = pre_lo;
        hi = pre_hi;
      } else {
        const uint16_t* xp = a.x + (size_t)m * a.K + (size_t)grp * 64 + 16 * tq;
        lo = __ldg(reinterpret_cast<const uint4*>(xp));
        hi = __ldg(reinterpret_cast<const uint4*>(xp + 8));
      }
      if (a.norm_w) {
        const float inv = inv_s[m];
        const uint16_t* wv = a.norm_w + (size_t)grp * 64 + 16 * tq;
        uint32_t* l32 = reinterpret_cast<uint32_t*>(&lo);
        uint32_t* h32 = reinterpret_cast<uint32_t*>(&hi);
#pragma unroll
        for (int e = 0; e < 8; e++) {
          uint32_t* word = e < 4 ? &l32[e] : &h32[e - 4];
          const float w0 = a.gemma_norm ? 1.0f + bf(wv[2 * e]) : bf(wv[2 * e]);
          const float w1 = a.gemma_norm ? 1.0f + bf(wv[2 * e + 1]) : bf(wv[2 * e + 1]);
          const uint16_t n0 = to_bf((bf_lo(*word) * inv) * w0);
          const uint16_t n1 = to_bf((bf_hi(*word) * inv) * w1);
          *word = (uint32_t)n0 | ((uint32_t)n1 << 16);
        }
      }
      const uint32_t* l32 = reinterpret_cast<const uint32_t*>(&lo);
      const uint32_t* h32 = reinterpret_cast<const uint32_t*>(&hi);
#pragma unroll
      for (int e = 0; e < 4; e++) part += bf_lo(l32[e]) + bf_hi(l32[e]);
#pragma unroll
      for (int e = 0; e < 4; e++) part += bf_lo(h32[e]) + bf_hi(h32[e]);
    }
    uint4 f0, f1;
    f0.x = __byte_perm(lo.x, lo.z, 0x5410);
    f0.y = __byte_perm(lo.x, lo.z, 0x7632);
    f0.z = __byte_perm(lo.y, lo.w, 0x5410);
    f0.w = __byte_perm(lo.y, lo.w, 0x7632);
    f1.x = __byte_perm(hi.x, hi.z, 0x5410);
    f1.y = __byte_perm(hi.x, hi.z, 0x7632);
    f1.z = __byte_perm(hi.y, hi.w, 0x5410);
    f1.w = __byte_perm(hi.y, hi.w, 0x7632);
    const int nt = m >> 3, gm = m & 7;
    xf[gl][nt][gm * 4 + tq][0] = f0;
    xf[gl][nt][gm * 4 + tq][1] = f1;
    // the four quarters of (group, m) are adjacent threads: fixed-order pair sums
    part += __shfl_xor_sync(0xffffffffu, part, 1);
    part += __shfl_xor_sync(0xffffffffu, part, 2);
    if (tq == 0) sxs[gl][m] = part;
  }
  __syncthreads();
  constexpr bool CLUSTER = CL;
  if (!CLUSTER && !live) return;  // in a cluster every thread takes part in the cluster barriers

  // ---- main loop: this warp's tile over [cg0, cg1), one 1152-byte unit per group, Q4_DEPTH units in flight
  float tot[2][NT][4];
#pragma unroll
  for (int tt = 0; tt < 2; tt++)
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int e = 0; e < 4; e++) tot[tt][nt][e] = 0.f;
  const int ng_live = live ? ng : 0;
  // the register ring: Q4_DEPTH units in flight per warp (two 16-byte code loads + one scale/bias load per lane).
  // One unit: its codes and scales leave the ring, the unit Q4_DEPTH groups on is loaded in their place.
  auto unit = [&](const int gl, uint4& r0, uint4& r1, uint4& rb) {
    const uint4 c0 = r0, c1 = r1, sb = rb;
    if (gl + Q4_DEPTH < ng) {
      const unsigned char* nu = up + (size_t)(gl + Q4_DEPTH) * Q4_UNIT;
      r0 = q4_ld_stream(nu + lane * 32);
      r1 = q4_ld_stream(nu + lane * 32 + 16);
      rb = __ldg(reinterpret_cast<const uint4*>(nu + 1024 + g * 16));
    }
    uint32_t px[NT][8];
    float sx[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      const uint4 f0 = xf[gl][nt][lane][0], f1 = xf[gl][nt][lane][1];
      px[nt][0] = f0.x; px[nt][1] = f0.y; px[nt][2] = f0.z; px[nt][3] = f0.w;
      px[nt][4] = f1.x; px[nt][5] = f1.y; px[nt][6] = f1.z; px[nt][7] = f1.w;
      const float2 s2 = *reinterpret_cast<const float2*>(&sxs[gl][nt * 8 + 2 * t]);
      sx[nt][0] = s2.x;
      sx[nt][1] = s2.y;
    }
    // sb: s(g), s(g+8), s(16+g), s(24+g), b(g), b(g+8), b(16+g), b(24+g)
    const float sv[4] = {bf_lo(sb.x), bf_hi(sb.x), bf_lo(sb.y), bf_hi(sb.y)};
    const float bv[4] = {bf_lo(sb.z), bf_hi(sb.z), bf_lo(sb.w), bf_hi(sb.w)};
    const uint32_t wd[2][4] = {{c0.x, c0.y, c0.z, c0.w}, {c1.x, c1.y, c1.z, c1.w}};
#pragma unroll
    for (int tt = 0; tt < 2; tt++) {
      uint32_t pa[8], pb[8];
      q4_codes(wd[tt][0], pa);
      q4_codes(wd[tt][1], pa + 4);
      q4_codes(wd[tt][2], pb);
      q4_codes(wd[tt][3], pb + 4);
      float acc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc[nt][e] = 0.f;
#pragma unroll
      for (int q = 0; q < 4; q++)
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
          q4_mma(acc[nt], pa[2 * q], pb[2 * q], pa[2 * q + 1], pb[2 * q + 1], px[nt][2 * q], px[nt][2 * q + 1]);
      const float s0 = sv[2 * tt], s1 = sv[2 * tt + 1];
      const float b0 = fmaf(-128.f, s0, bv[2 * tt]), b1 = fmaf(-128.f, s1, bv[2 * tt + 1]);
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        tot[tt][nt][0] = fmaf(b0, sx[nt][0], fmaf(s0, acc[nt][0], tot[tt][nt][0]));
        tot[tt][nt][1] = fmaf(b0, sx[nt][1], fmaf(s0, acc[nt][1], tot[tt][nt][1]));
        tot[tt][nt][2] = fmaf(b1, sx[nt][0], fmaf(s1, acc[nt][2], tot[tt][nt][2]));
        tot[tt][nt][3] = fmaf(b1, sx[nt][1], fmaf(s1, acc[nt][3], tot[tt][nt][3]));
      }
    }
  };
  // whole rounds of Q4_DEPTH units as straight-line code (independent units' MMA chains can interleave), then
  // the last partial round
  // the last partial round (with more rows, where registers are scarcer, every round checks its units instead)
  if constexpr (NT == 1) {
    int gl0 = 0;
#pragma unroll 1
    for (; gl0 + Q4_DEPTH <= ng_live; gl0 += Q4_DEPTH) {
#pragma unroll
      for (int d = 0; d < Q4_DEPTH; d++) unit(gl0 + d, rc0[d], rc1[d], rsb[d]);
    }
#pragma unroll
    for (int d = 0; d < Q4_DEPTH - 1; d++)
      if (gl0 + d < ng_live) unit(gl0 + d, rc0[d], rc1[d], rsb[d]);
  } else {
#pragma unroll 1
    for (int gl0 = 0; gl0 < ng_live; gl0 += Q4_DEPTH) {
#pragma unroll
      for (int d = 0; d < Q4_DEPTH; d++) {
        if (gl0 + d >= ng_live) break;
        unit(gl0 + d, rc0[d], rc1[d], rsb[d]);
      }
    }
  }

  // ---- split-K: per-warp partial, summed in split order
  constexpr int NV = 2 * NT * 4;
  if (CLUSTER && a.splits > 1) {
    // each CTA of the cluster keeps its partials in its own shared memory; the reducing warp of a tile reads the
    // split partials of every CTA of the cluster in split order (CTA rank = split)
    float* mine = part_s + warp * NV * 32;
#pragma unroll
    for (int tt = 0; tt < 2; tt++)
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) mine[((tt * NT + nt) * 4 + e) * 32 + lane] = tot[tt][nt][e];
    q4_cluster_arrive();
    q4_cluster_wait();
    const bool finish = live && reducer;
    if (finish) {
#pragma unroll
      for (int tt = 0; tt < 2; tt++)
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
          for (int e = 0; e < 4; e++) tot[tt][nt][e] = 0.f;
      constexpr int SB = NV <= 8 ? 8 : (NV <= 16 ? 4 : 2);
      for (int s0 = 0; s0 < a.splits; s0 += SB) {
        float buf[SB][NV];
#pragma unroll
        for (int j = 0; j < SB; j++) {
          if (s0 + j < a.splits) {
            const uint32_t src = q4_mapa(mine, (unsigned)(s0 + j)) + (uint32_t)lane * 4u;
#pragma unroll
            for (int v = 0; v < NV; v++) buf[j][v] = q4_ld_dsmem(src + (uint32_t)v * 128u);
          }
        }
#pragma unroll
        for (int j = 0; j < SB; j++) {
          if (s0 + j < a.splits) {
#pragma unroll
            for (int tt = 0; tt < 2; tt++)
#pragma unroll
              for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int e = 0; e < 4; e++) tot[tt][nt][e] += buf[j][(tt * NT + nt) * 4 + e];
          }
        }
      }
    }
    q4_cluster_arrive();  // this CTA has read what it needs from its peers
    if (finish) q4_epilogue<NT, EPI, RES_EARLY>(a, tot, rres, tile, g, t);
    q4_cluster_wait();    // no CTA leaves while a peer may still read its partials
    return;
  }
  if (!live) return;
  if (a.splits > 1) {
    float* mine = a.partial + ((size_t)tile * a.splits + split) * NV * 32;
#pragma unroll
    for (int tt = 0; tt < 2; tt++)
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) __stcg(mine + ((tt * NT + nt) * 4 + e) * 32 + lane, tot[tt][nt][e]);
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(a.counters + tile, 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != (unsigned)(a.splits - 1)) return;
    __threadfence();
#pragma unroll
    for (int tt = 0; tt < 2; tt++)
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int e = 0; e < 4; e++) tot[tt][nt][e] = 0.f;
    // loads of SB splits at a time (64 floats per lane) are issued together; the adds stay in split order
    constexpr int SB = NV <= 8 ? 8 : (NV <= 16 ? 4 : 2);
    for (int s0 = 0; s0 < a.splits; s0 += SB) {
      float buf[SB][NV];
#pragma unroll
      for (int j = 0; j < SB; j++) {
        if (s0 + j < a.splits) {
          const float* src = a.partial + ((size_t)tile * a.splits + s0 + j) * NV * 32;
#pragma unroll
          for (int v = 0; v < NV; v++) buf[j][v] = __ldcg(src + v * 32 + lane);
        }
      }
#pragma unroll
      for (int j = 0; j < SB; j++) {
        if (s0 + j < a.splits) {
#pragma unroll
          for (int tt = 0; tt < 2; tt++)
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
              for (int e = 0; e < 4; e++) tot[tt][nt][e] += buf[j][(tt * NT + nt) * 4 + e];
        }
      }
    }
    if (lane == 0) a.counters[tile] = 0u;
  }

  q4_epilogue<NT, EPI, RES_EARLY>(a, tot, rres, tile, g, t);
}

Q4Plan q4_plan(int64_t M, int64_t N, int64_t K) {
  Q4Plan p;
  p.tiles = (int)((N + 31) / 32);
  p.ctas_x = (p.tiles + Q4_WARPS - 1) / Q4_WARPS;
  p.nt = (int)((M > 32 ? 32 : M) + 7) / 8;
  const int G = (int)(K / 64);
  const int rmax = Q4_RMAX;
  const int need = (G + rmax - 1) / rmax;                // shared-memory budget
  int s = g_q4_target_ctas / p.ctas_x;                 // the most splits that fill one wave
  if (s < 1) s = 1;
  if (s > g_q4_max_split) s = g_q4_max_split;
  const int cap = G / 4 > 0 ? G / 4 : 1;                // at least 4 groups per CTA
  if (s > cap) s = cap;
  if (s < need) s = need;
  if (g_q4_split_override > 0) s = g_q4_split_override < need ? need : (g_q4_split_override > G ? G : g_q4_split_override);
  p.splits = s;
  p.rg = (G + s - 1) / s;
  p.chunks = (int)((M + 31) / 32);
  if (q4_tensor_cores(M, s))  // the tensor-core path always needs the counter region (its error word)
    p.workspace = Q4_COUNTER_BYTES + qtc_workspace_bytes(p, M, K);
  else
    p.workspace = s > 1 ? Q4_COUNTER_BYTES + (size_t)p.chunks * p.tiles * s * 2 * 4 * 4 * 32 * sizeof(float) : 0;
  return p;
}

// Whether clusters of `splits` CTAs of this kernel can be scheduled at all (asked once per split count, before
// any launch, so a refusal never happens inside a stream capture).
template <int NT, int EPI, bool AM>
static bool q4_cluster_ok(int splits, size_t smem) {
  static int known[Q4_MAX_SPLITS + 1] = {};  // 0 unknown, 1 yes, 2 no
  if (splits < 2 || splits > Q4_MAX_SPLITS) return false;
  if (!known[splits]) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, splits, 1);
    cfg.blockDim = dim3(Q4_THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = splits;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    const cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, qgemm_packed_kernel<NT, EPI, true, AM>, &cfg);
    known[splits] = e == cudaSuccess && clusters > 0 ? 1 : 2;
    if (e != cudaSuccess) (void)cudaGetLastError();
  }
  return known[splits] == 1;
}

template <int NT, int EPI, bool AM = false>
static int q4_launch(const Q4Plan& p, const Q4Args& a, cudaStream_t st) {
  const size_t smem = q4_smem(NT, a.rg, a.norm_w ? a.norm_parts : 0, AM).total;
  static bool configured = false;
  if (!configured) {
    const int most = (int)q4_smem(NT, Q4_RMAX, Q4_MAX_NORM_PARTS, AM).total;
    cudaFuncSetAttribute(qgemm_packed_kernel<NT, EPI, false, AM>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
    cudaFuncSetAttribute(qgemm_packed_kernel<NT, EPI, true, AM>, cudaFuncAttributeMaxDynamicSharedMemorySize, most);
    cudaFuncSetAttribute(qgemm_packed_kernel<NT, EPI, true, AM>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    configured = true;
  }
  dim3 grid(p.ctas_x, p.splits, p.chunks);
  const bool cluster = g_q4_cluster && p.splits > 1 && q4_cluster_ok<NT, EPI, AM>(p.splits, smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(Q4_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (launch_overlap()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    n++;
  }
  if (cluster) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = p.splits;
    attr[n].val.clusterDim.z = 1;
    n++;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t e = cluster ? cudaLaunchKernelEx(&cfg, qgemm_packed_kernel<NT, EPI, true, AM>, a)
                                : cudaLaunchKernelEx(&cfg, qgemm_packed_kernel<NT, EPI, false, AM>, a);
  if (e != cudaSuccess) {
    set_error("qgemm_packed_kernel: %s", cudaGetErrorString(e));
    return IM_CUDA_ERROR;
  }
  return IM_OK;
}

template <int EPI>
static int q4_dispatch(const Q4Plan& p, const Q4Args& a, cudaStream_t st) {
  switch (p.nt) {
    case 1: return q4_launch<1, EPI>(p, a, st);
    case 2: return q4_launch<2, EPI>(p, a, st);
    case 3: return q4_launch<3, EPI>(p, a, st);
    default: return q4_launch<4, EPI>(p, a, st);
  }
}

}  // namespace im

using namespace im;

extern "C" int im_qgemm_packed_tune(int split_override, int target_ctas, int max_split) {
  IM_REQUIRE(split_override >= 0 && target_ctas >= 1 && max_split >= 1, IM_INVALID, "im_qgemm_packed_tune: bad value");
  g_q4_split_override = split_override;
  g_q4_target_ctas = target_ctas;
  g_q4_max_split = max_split;
  return IM_OK;
}

extern "C" int im_qgemm_packed_cluster(int on) {
  IM_REQUIRE(on == 0 || on == 1, IM_INVALID, "im_qgemm_packed_cluster: 0 or 1");
  g_q4_cluster = on;
  return IM_OK;
}

extern "C" int im_qgemm_packed_path(int path) {
  IM_REQUIRE(path >= 0 && path <= 2, IM_INVALID, "im_qgemm_packed_path: 0, 1 or 2");
  g_q4_path = path;
  return IM_OK;
}

extern "C" size_t im_qgemm_packed_bytes(int64_t N, int64_t K) {
  if (N < 1 || K < 64 || K % 64) return 0;
  return (size_t)((N + 31) / 32) * (K / 64) * Q4_UNIT;
}

extern "C" int im_qgemm_pack_w4g64(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, int64_t N,
                                   int64_t K, void* packed, void* stream) {
  clear_error();
  IM_REQUIRE(N >= 1 && K >= 64 && K % 64 == 0 && N <= (1 << 30) && K <= (1 << 24), IM_INVALID,
             "im_qgemm_pack_w4g64: bad sizes");
  IM_REQUIRE(w && scales && biases && packed, IM_INVALID, "im_qgemm_pack_w4g64: null pointer");
  IM_REQUIRE(aligned(packed, 16) && aligned(w, 4), IM_INVALID, "im_qgemm_pack_w4g64: misaligned buffer");
  const long long units = ((N + 31) / 32) * (K / 64);
  IM_REQUIRE(units < (1ll << 31), IM_UNSUPPORTED, "im_qgemm_pack_w4g64: too many units");
  q4_pack_kernel<<<(unsigned)units, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      w, scales, biases, (int)N, (int)K, reinterpret_cast<unsigned char*>(packed));
  return check_launch("q4_pack_kernel");
}

extern "C" size_t im_qgemm_packed_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (M < 1 || M > Q4_MAX_ROWS || N < 1 || K < 64 || K % 64) return 0;
  const Q4Plan p = q4_plan(M, N, K);
  return (size_t)((p.chunks + 1) / 2 * 2) * p.tiles < Q4_COUNTER_BYTES / 4 ? p.workspace : 0;
}

extern "C" int im_qgemm_packed_status(const void* workspace) {
  clear_error();
  IM_REQUIRE(workspace, IM_INVALID, "im_qgemm_packed_status: null workspace");
  unsigned word = 0;
  const cudaError_t e = cudaMemcpy(&word, reinterpret_cast<const char*>(workspace) + Q4_COUNTER_BYTES - 4, 4,
                                   cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    set_error("im_qgemm_packed_status: %s", cudaGetErrorString(e));
    return IM_CUDA_ERROR;
  }
  return (int)word;
}

extern "C" int im_qgemm_packed(const void* packed, const uint16_t* x, uint16_t* y, const uint16_t* residual,
                               int64_t M, int64_t N, int64_t K, int epilogue, const float* norm_sq,
                               int64_t norm_parts, const uint16_t* norm_weight, float eps, int gemma_norm,
                               float* out_sq, int64_t sq_ld, void* workspace, size_t workspace_bytes,
                               void* stream) {
  clear_error();
  IM_REQUIRE(M >= 0 && M <= Q4_MAX_ROWS && N >= 1 && K >= 64 && K % 64 == 0 && N <= (1 << 30) && K <= (1 << 24),
             IM_INVALID, "im_qgemm_packed: bad sizes M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (M == 0) return IM_OK;
  IM_REQUIRE(packed && x && y, IM_INVALID, "im_qgemm_packed: null pointer");
  IM_REQUIRE(aligned(packed, 16) && aligned(x, 16), IM_INVALID, "im_qgemm_packed: packed and x must be 16-byte aligned");
  IM_REQUIRE(epilogue >= IM_EPI_STORE && epilogue <= IM_EPI_GEGLU, IM_INVALID, "im_qgemm_packed: bad epilogue");
  IM_REQUIRE(epilogue != IM_EPI_RESIDUAL || residual, IM_INVALID, "im_qgemm_packed: residual epilogue needs residual");
  const bool glu = epilogue == IM_EPI_SWIGLU || epilogue == IM_EPI_GEGLU;
  IM_REQUIRE(!glu || N % 32 == 0, IM_INVALID, "im_qgemm_packed: gated epilogues need N % 32 == 0");
  IM_REQUIRE(!glu || !out_sq, IM_INVALID, "im_qgemm_packed: sums of squares come from store/residual epilogues");
  IM_REQUIRE(!norm_weight || (norm_sq && norm_parts >= 1 && aligned(norm_weight, 2)), IM_INVALID,
             "im_qgemm_packed: the RMSNorm prologue needs norm_sq partials and a weight");
  IM_REQUIRE(!norm_weight || norm_parts <= Q4_MAX_NORM_PARTS, IM_UNSUPPORTED,
             "im_qgemm_packed: %lld sum-of-squares parts exceed %d", (long long)norm_parts, Q4_MAX_NORM_PARTS);
  const int64_t ld = sq_ld > 0 ? sq_ld : (M + 31) / 32 * 32;
  IM_REQUIRE(ld >= M, IM_INVALID, "im_qgemm_packed: sq_ld %lld below M", (long long)ld);
  const Q4Plan p = q4_plan(M, N, K);
  // counters: one per (32-row chunk, tile) below 33 rows, per (64-row chunk, tile, column half) above; the
  // last word of the counter region is the tensor-core kernel's error word
  IM_REQUIRE((size_t)((p.chunks + 1) / 2 * 2) * p.tiles < Q4_COUNTER_BYTES / 4, IM_UNSUPPORTED,
             "im_qgemm_packed: N too large for split-K at %lld rows", (long long)M);
  const bool tc = q4_tensor_cores(M, p.splits);
  if (p.splits > 1 || tc)
    IM_REQUIRE(workspace && aligned(workspace, 256) && workspace_bytes >= p.workspace, IM_INVALID,
               "im_qgemm_packed: workspace of %zu bytes (256-aligned) needed, %zu given", p.workspace,
               workspace_bytes);
  Q4Args a = {};
  a.wp = reinterpret_cast<const unsigned char*>(packed);
  a.x = x;
  a.y = y;
  a.res = residual;
  a.norm_sq = norm_sq;
  a.norm_w = norm_weight;
  a.out_sq = out_sq;
  a.counters = reinterpret_cast<unsigned*>(workspace);
  a.partial = workspace ? reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + Q4_COUNTER_BYTES) : nullptr;
  a.eps = eps;
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.tiles = p.tiles;
  a.splits = p.splits;
  a.norm_parts = (int)norm_parts;
  a.gemma_norm = gemma_norm;
  a.sq_ld = (int)ld;
  a.rg = p.rg;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (tc) return qtc_launch(p, a, epilogue, workspace, st);
  switch (epilogue) {
    case IM_EPI_STORE: return q4_dispatch<IM_EPI_STORE>(p, a, st);
    case IM_EPI_RESIDUAL: return q4_dispatch<IM_EPI_RESIDUAL>(p, a, st);
    case IM_EPI_SWIGLU: return q4_dispatch<IM_EPI_SWIGLU>(p, a, st);
    default: return q4_dispatch<IM_EPI_GEGLU>(p, a, st);
  }
}

extern "C" int64_t im_qgemm_packed_attn_rows(int64_t N, int64_t K) {
  if (N < 1 || K < 64 || K % 64) return 0;
  const Q4Plan p = q4_plan(1, N, K);
  const int64_t rows = Q4_THREADS / ((int64_t)p.rg * 16);  // one merge job of 4 values per thread
  return rows > 8 ? 8 : rows;
}

extern "C" int im_qgemm_packed_attn(const void* packed, const void* attn_workspace, const int32_t* seq_rows,
                                    const int32_t* row_slot, int64_t B, int64_t max_rows_per_seq, int64_t Hq,
                                    int64_t Hkv, int64_t D, int64_t max_kv_len, int64_t keys_per_split, uint16_t* y,
                                    const uint16_t* residual, int64_t M, int64_t N, int64_t K, float* out_sq,
                                    int64_t sq_ld, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  IM_REQUIRE(M >= 0 && N >= 1 && K >= 64 && K % 64 == 0 && N <= (1 << 30) && K <= (1 << 24), IM_INVALID,
             "im_qgemm_packed_attn: bad sizes M=%lld N=%lld K=%lld", (long long)M, (long long)N, (long long)K);
  if (M == 0) return IM_OK;
  IM_REQUIRE(M <= im_qgemm_packed_attn_rows(N, K), IM_UNSUPPORTED,
             "im_qgemm_packed_attn: %lld rows exceed im_qgemm_packed_attn_rows (%lld)", (long long)M,
             (long long)im_qgemm_packed_attn_rows(N, K));
  IM_REQUIRE(packed && attn_workspace && seq_rows && row_slot && y && residual, IM_INVALID,
             "im_qgemm_packed_attn: null pointer");
  IM_REQUIRE(aligned(packed, 16) && aligned(attn_workspace, 256), IM_INVALID,
             "im_qgemm_packed_attn: packed 16-byte and the attention workspace 256-byte aligned");
  IM_REQUIRE(B >= 1 && B <= M && max_rows_per_seq >= 1 && Hkv >= 1 && Hq % Hkv == 0 && (D == 128 || D == 256) &&
                 Hq * D == K && max_kv_len >= 1 && keys_per_split >= 64 && keys_per_split % 64 == 0,
             IM_INVALID, "im_qgemm_packed_attn: attention geometry does not match K = Hq * D");
  const int64_t ld = sq_ld > 0 ? sq_ld : (M + 31) / 32 * 32;
  IM_REQUIRE(ld >= M, IM_INVALID, "im_qgemm_packed_attn: sq_ld %lld below M", (long long)ld);
  const Q4Plan p = q4_plan(M, N, K);
  if (p.splits > 1)
    IM_REQUIRE(workspace && aligned(workspace, 256) && workspace_bytes >= p.workspace, IM_INVALID,
               "im_qgemm_packed_attn: workspace of %zu bytes (256-aligned) needed, %zu given", p.workspace,
               workspace_bytes);
  int nq, qblocks;
  attn_geometry(max_rows_per_seq, Hq / Hkv, &nq, &qblocks);
  Q4Args a = {};
  a.wp = reinterpret_cast<const unsigned char*>(packed);
  a.y = y;
  a.res = residual;
  a.out_sq = out_sq;
  a.counters = reinterpret_cast<unsigned*>(workspace);
  a.partial = workspace ? reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + Q4_COUNTER_BYTES) : nullptr;
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.tiles = p.tiles;
  a.splits = p.splits;
  a.sq_ld = (int)ld;
  a.rg = p.rg;
  a.am.part = reinterpret_cast<const float*>(reinterpret_cast<const char*>(attn_workspace) + AT_COUNTER_BYTES);
  a.am.seq_rows = seq_rows;
  a.am.row_slot = row_slot;
  a.am.B = (int)B;
  a.am.Hq = (int)Hq;
  a.am.Hkv = (int)Hkv;
  a.am.D = (int)D;
  a.am.kpc = (int)keys_per_split;
  a.am.nsplit = (int)((max_kv_len + keys_per_split - 1) / keys_per_split);
  a.am.qblocks = qblocks;
  a.am.nq = nq;
  return q4_launch<1, IM_EPI_RESIDUAL, true>(p, a, reinterpret_cast<cudaStream_t>(stream));
}
