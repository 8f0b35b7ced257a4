// qGEMM v3: persistent, bulk-copy-pipelined 4-bit GEMM for small M (the default for M <= 32).
//
// Same arithmetic as the warp-MMA kernel in qgemm.cu (exact bf16 codes 128+q on the tensor pipe, the group
// affine folded into an fp32 epilogue: s*acc + (b - 128 s)*sum(x)), fed differently:
//  * one CTA per SM (persistent), 1 producer warp + 8 consumer warps;
//  * the work is the list of units (32-row tile, 16-group k-chunk) in tile-major order, split evenly across the
//    CTAs ("stream-K"): a CTA streams a contiguous run of units, so tiles may span two CTAs;
//  * the producer's lane 0 copies each unit's 32 rows x 512 bytes of codes into a 6-stage shared-memory ring
//    with cp.async.bulk (one bulk copy per row, completion counted on the stage's mbarrier); rows are padded to
//    544 bytes so the consumers' 8-byte fragment reads are bank-conflict free. Every copy targets only this CTA;
//  * consumer warp w takes groups 2w and 2w+1 of every unit for both 16-row halves, reads scales and biases
//    with 4-byte loads and activations (L1-resident) with 16-byte loads straight from global memory;
//  * at the end of a tile's run in a CTA the 8 consumers reduce in warp order; a tile covered by one CTA is
//    written directly, a tile split across CTAs publishes per-CTA partials that the last CTA to finish sums in
//    CTA order. The partition depends on (N, K, grid) only, never on M: a row gets the same bits at any M.
// Every wait on an mbarrier is bounded; a wait that runs out sets an error word in the workspace, drains the
// copies this CTA issued and leaves the CTA early (im_qgemm_tma_status reads the word).
#include <mutex>

#include "common.cuh"
#include "../../include/imspec.h"

namespace im {

constexpr int Q3_CONSUMERS = 8;
constexpr int Q3_THREADS = (Q3_CONSUMERS + 1) * 32;
constexpr int Q3_ROWS = 32;
constexpr int Q3_KC = 16;                       // groups per unit (1024 k)
constexpr int Q3_ROWB = Q3_KC * 32;             // bytes of codes per row per unit
constexpr int Q3_PITCH = Q3_ROWB + 32;          // padded shared-memory row pitch
constexpr int Q3_STAGE = Q3_ROWS * Q3_PITCH;    // 17408 bytes
constexpr int Q3_STAGES = 6;
constexpr unsigned long long Q3_WAIT_NS = 1000000000ull;  // a wait gives up after 1 s (real stalls: microseconds)
constexpr size_t Q3_COUNTER_BYTES = 65536;      // per-tile counters (16384 tiles) + the error word
constexpr uint32_t BF16X2_ONE3 = 0x3F803F80u;
constexpr uint32_t BF16X2_128_3 = 0x43004300u;

struct Q3Smem {
  unsigned char stage[Q3_STAGES][Q3_STAGE];
  float red[Q3_CONSUMERS][2 * 4 * 4][32];  // [warp][tile*NT*4 + i][lane], sized for NT <= 4
  unsigned long long full[Q3_STAGES];
  unsigned long long empty[Q3_STAGES];
  int abort;  // set when any wait of this CTA gave up; every later wait returns at once
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(unsigned long long* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: true when the phase completed; false when this CTA aborted or 1 s passed (then the CTA aborts
// and the error word records `code`).
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, uint32_t parity, volatile int* abort,
                                          unsigned* error, unsigned code) {
  if (*abort) return false;
  const unsigned long long start = global_ns();
  for (uint32_t i = 0;; i++) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      if (*abort) return false;
      if (global_ns() - start > Q3_WAIT_NS) {
        *abort = 1;
        atomicExch(error, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma16816_3(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void codes4(uint32_t u, uint32_t* p) {
  p[0] = (u & 0x000F000Fu) | BF16X2_128_3;
  p[1] = ((u >> 4) & 0x000F000Fu) | BF16X2_128_3;
  p[2] = ((u >> 8) & 0x000F000Fu) | BF16X2_128_3;
  p[3] = ((u >> 12) & 0x000F000Fu) | BF16X2_128_3;
}

__device__ __forceinline__ void frag_x(const uint4& lo, const uint4& hi, uint32_t* px) {
  px[0] = __byte_perm(lo.x, lo.z, 0x5410);
  px[1] = __byte_perm(lo.x, lo.z, 0x7632);
  px[2] = __byte_perm(lo.y, lo.w, 0x5410);
  px[3] = __byte_perm(lo.y, lo.w, 0x7632);
  px[4] = __byte_perm(hi.x, hi.z, 0x5410);
  px[5] = __byte_perm(hi.x, hi.z, 0x7632);
  px[6] = __byte_perm(hi.y, hi.w, 0x5410);
  px[7] = __byte_perm(hi.y, hi.w, 0x7632);
}

__device__ __forceinline__ float silu_mul3(float gate, float up) {
  const float a = round_bf(gate), u = round_bf(up);
  const float sig = round_bf(1.0f / (1.0f + expf(-a)));
  return round_bf(a * sig) * u;
}

__device__ __forceinline__ float gelu_mul3(float gate, float up) {
  const float a = round_bf(gate), u = round_bf(up);
  const float inner = 0.7978845608028654f * (a + 0.044715f * a * a * a);
  return round_bf(0.5f * a * (1.0f + tanhf(inner))) * u;
}

// unit index range of CTA c among C CTAs over U units
__device__ __forceinline__ long long unit_begin(int c, int C, long long U) { return (long long)c * U / C; }

// the CTA whose range holds unit u
__device__ __forceinline__ int unit_owner(long long u, int C, long long U) {
  int c = (int)((u * C) / U);
  while (c > 0 && unit_begin(c, C, U) > u) c--;
  while (c + 1 < C && unit_begin(c + 1, C, U) <= u) c++;
  return c;
}

template <int NT, int EPI>
__device__ __forceinline__ void q3_store(const float (&v)[2][NT][4], uint16_t* y, const uint16_t* res, int M, int N,
                                         int rbase, int g, int t) {
  if constexpr (EPI == IM_EPI_SWIGLU || EPI == IM_EPI_GEGLU) {
    const int nout = N >> 1;
    const int f0 = (rbase >> 1) + g;
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int f = f0 + ((i >> 1) << 3);
        const int m = nt * 8 + 2 * t + (i & 1);
        if (m < M && f < nout) {
          const float o = EPI == IM_EPI_SWIGLU ? silu_mul3(v[0][nt][i], v[1][nt][i]) : gelu_mul3(v[0][nt][i], v[1][nt][i]);
          y[(size_t)m * nout + f] = to_bf(o);
        }
      }
  } else {
#pragma unroll
    for (int tt = 0; tt < 2; tt++)
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const int r = rbase + tt * 16 + g + ((i >> 1) << 3);
          const int m = nt * 8 + 2 * t + (i & 1);
          if (m < M && r < N) {
            const size_t o = (size_t)m * N + r;
            y[o] = EPI == IM_EPI_RESIDUAL ? to_bf(bf(res[o]) + round_bf(v[tt][nt][i])) : to_bf(v[tt][nt][i]);
          }
        }
  }
}

struct Q3Args {
  const uint32_t* w;
  const uint16_t* sc;
  const uint16_t* bi;
  const uint16_t* x;
  uint16_t* y;
  const uint16_t* res;
  float* partial;       // [tiles][max parts][32 rows x NT*4 values x 32 lanes]
  unsigned* counters;   // [tiles]
  unsigned* error;      // non-zero after a wait ran out
  int M, N, K, tiles, nkc, max_parts;
};

template <int NT, int EPI>
__global__ void __launch_bounds__(Q3_THREADS, 1) qgemm_tma_kernel(Q3Args a) {
  extern __shared__ __align__(128) unsigned char q3_raw[];
  Q3Smem& sm = *reinterpret_cast<Q3Smem*>(q3_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = gridDim.x, c = blockIdx.x;
  const long long U = (long long)a.tiles * a.nkc;
  const long long u0 = unit_begin(c, C, U), u1 = unit_begin(c + 1, C, U);
  const int G = a.K >> 6;
  const size_t wrow_bytes = (size_t)a.K >> 1;

  volatile int* abort = &sm.abort;
  if (threadIdx.x == 0) {
    for (int s = 0; s < Q3_STAGES; s++) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], Q3_CONSUMERS);
    }
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == Q3_CONSUMERS) {
    // ---------------- producer ----------------
    if (lane == 0) {
      long long i = 0;
      bool ok = true;
      for (long long u = u0; u < u1; u++, i++) {
        const int s = (int)(i % Q3_STAGES);
        const uint32_t par = (uint32_t)((i / Q3_STAGES) & 1);
        if (i >= Q3_STAGES && !mbar_wait(&sm.empty[s], par ^ 1u, abort, a.error, 1u)) {
          ok = false;
          break;
        }
        const int tile = (int)(u / a.nkc), kc = (int)(u % a.nkc);
        const int g0 = kc * Q3_KC, ng = min(Q3_KC, G - g0);
        const int r0 = tile * Q3_ROWS, nrows = min(Q3_ROWS, a.N - r0);
        const uint32_t bytes = (uint32_t)(ng * 32);
        mbar_expect_tx(&sm.full[s], bytes * (uint32_t)nrows);
        const unsigned char* src = reinterpret_cast<const unsigned char*>(a.w) + (size_t)r0 * wrow_bytes + (size_t)g0 * 32;
        for (int r = 0; r < nrows; r++) bulk_g2s(&sm.stage[s][r * Q3_PITCH], src + (size_t)r * wrow_bytes, bytes, &sm.full[s]);
      }
      if (!ok) {
        // drain: wait (bounded, ignoring the abort flag) for the copies this CTA already issued
        for (long long j = (i >= Q3_STAGES ? i - Q3_STAGES : 0); j < i; j++) {
          const unsigned long long start = global_ns();
          while (!mbar_try_wait(&sm.full[j % Q3_STAGES], (uint32_t)((j / Q3_STAGES) & 1)) &&
                 global_ns() - start < Q3_WAIT_NS) {
          }
        }
      }
    }
    return;
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2, t = lane & 3;
  const uint16_t* xrow[NT];
  bool xval[NT];
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const int m = nt * 8 + g;
    xval[nt] = m < a.M;
    xrow[nt] = a.x + (size_t)(xval[nt] ? m : 0) * a.K + 16 * t;
  }
  float tot[2][NT][4];
#pragma unroll
  for (int tt = 0; tt < 2; tt++)
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int i = 0; i < 4; i++) tot[tt][nt][i] = 0.f;

  long long i = 0;
  for (long long u = u0; u < u1; u++, i++) {
    const int s = (int)(i % Q3_STAGES);
    const uint32_t par = (uint32_t)((i / Q3_STAGES) & 1);
    const int tile = (int)(u / a.nkc), kc = (int)(u % a.nkc);
    const int r0 = tile * Q3_ROWS;
    // scales and biases of my two groups for the 4 rows I touch (issued before the wait)
    const int gl0 = 2 * warp;
    const int gg0 = kc * Q3_KC + gl0;
    const bool have0 = gg0 < G, have1 = gg0 + 1 < G;
    uint32_t sv[2][2], bv[2][2];  // [tile][half] -> bf16 pair (group gg0, gg0+1)
#pragma unroll
    for (int tt = 0; tt < 2; tt++)
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int r = min(r0 + tt * 16 + g + h * 8, a.N - 1);
        const uint16_t* sp = a.sc + (size_t)r * G + gg0;
        const uint16_t* bp = a.bi + (size_t)r * G + gg0;
        if (have1) {
          sv[tt][h] = __ldg(reinterpret_cast<const unsigned int*>(sp));
          bv[tt][h] = __ldg(reinterpret_cast<const unsigned int*>(bp));
        } else if (have0) {
          sv[tt][h] = __ldg(sp);
          bv[tt][h] = __ldg(bp);
        } else {
          sv[tt][h] = bv[tt][h] = 0u;
        }
      }
    // a wait that gives up skips the math but keeps this warp in step with the others (barriers below)
    const bool have = mbar_wait(&sm.full[s], par, abort, a.error, 2u);
    const unsigned char* st = sm.stage[s];
#pragma unroll
    for (int j = 0; j < 2; j++) {
      const int gg = gg0 + j;
      if (have && gg < G) {
        uint32_t px[NT][8];
        float sx[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
          if (xval[nt]) {
            const uint16_t* xp = xrow[nt] + (size_t)gg * 64;
            frag_x(ldg_u4(xp), ldg_u4(xp + 8), px[nt]);
          } else {
#pragma unroll
            for (int e = 0; e < 8; e++) px[nt][e] = 0u;
          }
#pragma unroll
          for (int e = 0; e < 4; e++) sx[nt][e] = 0.f;
#pragma unroll
          for (int q = 0; q < 4; q++)
            mma16816_3(sx[nt], BF16X2_ONE3, BF16X2_ONE3, BF16X2_ONE3, BF16X2_ONE3, px[nt][2 * q], px[nt][2 * q + 1]);
        }
#pragma unroll
        for (int tt = 0; tt < 2; tt++) {
          const unsigned char* rowa = st + (tt * 16 + g) * Q3_PITCH + (gl0 + j) * 32 + 8 * t;
          const uint2 wa = *reinterpret_cast<const uint2*>(rowa);
          const uint2 wb = *reinterpret_cast<const uint2*>(rowa + 8 * Q3_PITCH);
          uint32_t pa[8], pb[8];
          codes4(wa.x, pa);
          codes4(wa.y, pa + 4);
          codes4(wb.x, pb);
          codes4(wb.y, pb + 4);
          float acc[NT][4];
#pragma unroll
          for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[nt][e] = 0.f;
#pragma unroll
          for (int q = 0; q < 4; q++)
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
              mma16816_3(acc[nt], pa[2 * q], pb[2 * q], pa[2 * q + 1], pb[2 * q + 1], px[nt][2 * q], px[nt][2 * q + 1]);
          const float s0 = j ? bf_hi(sv[tt][0]) : bf_lo(sv[tt][0]);
          const float s1 = j ? bf_hi(sv[tt][1]) : bf_lo(sv[tt][1]);
          const float b0 = fmaf(-128.f, s0, j ? bf_hi(bv[tt][0]) : bf_lo(bv[tt][0]));
          const float b1 = fmaf(-128.f, s1, j ? bf_hi(bv[tt][1]) : bf_lo(bv[tt][1]));
#pragma unroll
          for (int nt = 0; nt < NT; nt++) {
            tot[tt][nt][0] = fmaf(b0, sx[nt][0], fmaf(s0, acc[nt][0], tot[tt][nt][0]));
            tot[tt][nt][1] = fmaf(b0, sx[nt][1], fmaf(s0, acc[nt][1], tot[tt][nt][1]));
            tot[tt][nt][2] = fmaf(b1, sx[nt][0], fmaf(s1, acc[nt][2], tot[tt][nt][2]));
            tot[tt][nt][3] = fmaf(b1, sx[nt][1], fmaf(s1, acc[nt][3], tot[tt][nt][3]));
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[s]);

    // end of this tile's run in this CTA: reduce the 8 warps in order, then write or publish
    const bool tile_end = (kc == a.nkc - 1) || (u == u1 - 1);
    if (tile_end) {
      constexpr int NV = 2 * NT * 4;
#pragma unroll
      for (int tt = 0; tt < 2; tt++)
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
          for (int e = 0; e < 4; e++) {
            sm.red[warp][(tt * NT + nt) * 4 + e][lane] = tot[tt][nt][e];
            tot[tt][nt][e] = 0.f;
          }
      asm volatile("bar.sync 1, %0;" ::"r"(Q3_CONSUMERS * 32) : "memory");
      if (warp == 0) {
        float v[2][NT][4];
#pragma unroll
        for (int tt = 0; tt < 2; tt++)
#pragma unroll
          for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const int idx = (tt * NT + nt) * 4 + e;
              float acc = sm.red[0][idx][lane];
#pragma unroll
              for (int ww = 1; ww < Q3_CONSUMERS; ww++) acc += sm.red[ww][idx][lane];
              v[tt][nt][e] = acc;
            }
        const long long tu0 = (long long)tile * a.nkc, tu1 = tu0 + a.nkc;
        bool write = tu0 >= u0 && tu1 <= u1;  // the whole tile ran in this CTA
        if (!write) {
          const int first = unit_owner(tu0, C, U);
          const int parts = unit_owner(tu1 - 1, C, U) - first + 1;
          float* mine = a.partial + ((size_t)tile * a.max_parts + (c - first)) * NV * 32;
#pragma unroll
          for (int tt = 0; tt < 2; tt++)
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
#pragma unroll
              for (int e = 0; e < 4; e++) __stcg(mine + ((tt * NT + nt) * 4 + e) * 32 + lane, v[tt][nt][e]);
          __threadfence();
          __syncwarp();
          unsigned prev = 0;
          if (lane == 0) prev = atomicAdd(a.counters + tile, 1u);
          prev = __shfl_sync(0xffffffffu, prev, 0);
          if (prev == (unsigned)(parts - 1)) {
            __threadfence();
#pragma unroll
            for (int tt = 0; tt < 2; tt++)
#pragma unroll
              for (int nt = 0; nt < NT; nt++)
#pragma unroll
                for (int e = 0; e < 4; e++) v[tt][nt][e] = 0.f;
            for (int p = 0; p < parts; p++) {
              const float* src = a.partial + ((size_t)tile * a.max_parts + p) * NV * 32;
#pragma unroll
              for (int tt = 0; tt < 2; tt++)
#pragma unroll
                for (int nt = 0; nt < NT; nt++)
#pragma unroll
                  for (int e = 0; e < 4; e++) v[tt][nt][e] += __ldcg(src + ((tt * NT + nt) * 4 + e) * 32 + lane);
            }
            if (lane == 0) a.counters[tile] = 0u;
            write = true;
          }
        }
        if (write) q3_store<NT, EPI>(v, a.y, a.res, a.M, a.N, tile * Q3_ROWS, g, t);
      }
      asm volatile("bar.sync 1, %0;" ::"r"(Q3_CONSUMERS * 32) : "memory");
    }
  }
}

struct Q3Plan {
  int tiles, nkc, ctas, max_parts, nt;
  size_t workspace;
};

static int g_q3_sms = 0;

static Q3Plan q3_plan(int64_t M, int64_t N, int64_t K) {
  Q3Plan p;
  p.tiles = (int)((N + Q3_ROWS - 1) / Q3_ROWS);
  const int G = (int)(K / 64);
  p.nkc = (G + Q3_KC - 1) / Q3_KC;
  const long long units = (long long)p.tiles * p.nkc;
  int sms = g_q3_sms > 0 ? g_q3_sms : 148;
  p.ctas = (int)(units < sms ? units : sms);
  // a tile spans at most ceil(nkc / (units / ctas)) + 1 CTAs
  const long long per = units / p.ctas;
  p.max_parts = (int)(per > 0 ? (p.nkc + per - 1) / per + 1 : p.nkc);
  if (p.max_parts > p.ctas) p.max_parts = p.ctas;
  p.nt = (int)((M + 7) / 8);
  p.workspace = Q3_COUNTER_BYTES + (size_t)p.tiles * p.max_parts * 2 * 4 * 4 * 32 * sizeof(float);
  return p;
}

template <int NT, int EPI>
static int q3_launch(const Q3Plan& p, const Q3Args& args, cudaStream_t st) {
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(qgemm_tma_kernel<NT, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)sizeof(Q3Smem));
  });
  if (attr != cudaSuccess) {
    set_error("qgemm_tma: cannot reserve shared memory: %s", cudaGetErrorString(attr));
    return IM_CUDA_ERROR;
  }
  qgemm_tma_kernel<NT, EPI><<<p.ctas, Q3_THREADS, sizeof(Q3Smem), st>>>(args);
  return check_launch("qgemm_tma_kernel");
}

template <int EPI>
static int q3_dispatch(const Q3Plan& p, const Q3Args& args, cudaStream_t st) {
  switch (p.nt) {
    case 1: return q3_launch<1, EPI>(p, args, st);
    case 2: return q3_launch<2, EPI>(p, args, st);
    case 3: return q3_launch<3, EPI>(p, args, st);
    default: return q3_launch<4, EPI>(p, args, st);
  }
}

static void q3_init_sms() {
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
      g_q3_sms = n;
  });
}

}  // namespace im

using namespace im;

extern "C" size_t im_qgemm_tma_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (M < 1 || N < 1 || K < 64 || K % 64) return 0;
  q3_init_sms();
  const Q3Plan p = q3_plan(M, N, K);
  return p.tiles <= (int)(Q3_COUNTER_BYTES / 4) - 16 ? p.workspace : 0;
}

extern "C" int im_qgemm_tma(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const uint16_t* x,
                            uint16_t* y, const uint16_t* residual, int64_t M, int64_t N, int64_t K, int epilogue,
                            void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  IM_REQUIRE(M >= 0 && N >= 1 && K >= 64, IM_INVALID, "im_qgemm_tma: bad sizes");
  IM_REQUIRE(K % 256 == 0, IM_UNSUPPORTED, "im_qgemm_tma: K=%lld must be a multiple of 256", (long long)K);
  IM_REQUIRE(M <= 32, IM_UNSUPPORTED, "im_qgemm_tma: M=%lld exceeds 32", (long long)M);
  IM_REQUIRE(N <= (1 << 30) && K <= (1 << 24), IM_UNSUPPORTED, "im_qgemm_tma: N or K too large");
  if (M == 0) return IM_OK;
  IM_REQUIRE(w && scales && biases && x && y && workspace, IM_INVALID, "im_qgemm_tma: null pointer");
  IM_REQUIRE(aligned(w, 16) && aligned(x, 16) && aligned(scales, 4) && aligned(biases, 4) && aligned(y, 2) &&
                 aligned(workspace, 256),
             IM_INVALID, "im_qgemm_tma: misaligned buffer");
  IM_REQUIRE(epilogue >= IM_EPI_STORE && epilogue <= IM_EPI_GEGLU, IM_INVALID, "im_qgemm_tma: bad epilogue");
  IM_REQUIRE(epilogue != IM_EPI_RESIDUAL || residual, IM_INVALID, "im_qgemm_tma: residual epilogue needs residual");
  const bool glu = epilogue == IM_EPI_SWIGLU || epilogue == IM_EPI_GEGLU;
  IM_REQUIRE(!glu || N % 32 == 0, IM_INVALID, "im_qgemm_tma: gated epilogues need N % 32 == 0");
  const size_t need = im_qgemm_tma_workspace_bytes(M, N, K);
  IM_REQUIRE(need > 0 && workspace_bytes >= need, IM_INVALID, "im_qgemm_tma: workspace of %zu bytes needed, %zu given",
             need, workspace_bytes);
  const Q3Plan p = q3_plan(M, N, K);
  Q3Args args;
  args.w = w;
  args.sc = scales;
  args.bi = biases;
  args.x = x;
  args.y = y;
  args.res = residual;
  args.counters = reinterpret_cast<unsigned*>(workspace);
  args.error = reinterpret_cast<unsigned*>(workspace) + (Q3_COUNTER_BYTES / 4 - 1);
  args.partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + Q3_COUNTER_BYTES);
  args.M = (int)M;
  args.N = (int)N;
  args.K = (int)K;
  args.tiles = p.tiles;
  args.nkc = p.nkc;
  args.max_parts = p.max_parts;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (epilogue) {
    case IM_EPI_STORE: return q3_dispatch<IM_EPI_STORE>(p, args, st);
    case IM_EPI_RESIDUAL: return q3_dispatch<IM_EPI_RESIDUAL>(p, args, st);
    case IM_EPI_SWIGLU: return q3_dispatch<IM_EPI_SWIGLU>(p, args, st);
    default: return q3_dispatch<IM_EPI_GEGLU>(p, args, st);
  }
}

extern "C" int im_qgemm_tma_status(const void* workspace, uint32_t* status) {
  clear_error();
  IM_REQUIRE(workspace && status, IM_INVALID, "im_qgemm_tma_status: null pointer");
  const unsigned* word = reinterpret_cast<const unsigned*>(workspace) + (Q3_COUNTER_BYTES / 4 - 1);
  cudaError_t e = cudaMemcpy(status, word, 4, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    set_error("im_qgemm_tma_status: %s", cudaGetErrorString(e));
    return IM_CUDA_ERROR;
  }
  return IM_OK;
}
