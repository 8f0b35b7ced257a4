// W4A16 quantised GEMM for small M (speculative verify / decode), MLX-affine 4-bit, group 64.
//
// Replaces the reference's qmv kernel family (IronMule ironmule/qmv_k3840.py:133-310,
// ironmule/qmv_shared.py:66-181, ironmule/qmv_fast_shared.py:66-172, ironmule/qmv_variant.py:81-129)
// and its pre-Ampere CUDA analog (ironmule/cuda_native.py:57-168).
//
//   y[m, n] = sum_g  s[n,g] * sum_{k in g} q[n,k] x[m,k]  +  b[n,g] * sum_{k in g} x[m,k]
//
// Two kernels:
//  * qgemm_fma (v1): CUDA-core FMA, one warp per 4 output rows, 32-value chunks per lane, warp-shuffle
//    reduction, M <= 8 -- the plan the reference's own CUDA kernel follows.
//  * qgemm_mma (v2, default): warp-level bf16 tensor-core MMA (m16n8k16). A = the 4-bit codes turned
//    into exact bf16 values 128+q with one LOP3 per pair (no scale applied), B = activations, so each
//    MMA is an exact integer-weighted dot product over 16 k of one group in fp32; the group's affine is
//    applied once per group in fp32: s*acc + (b - 128 s) * sum(x). sum(x) per group comes from the same
//    MMA with A = 1. The k order inside an MMA is permuted identically for A and B, so that each lane's
//    operands come from 16 contiguous k of its own (8-byte weight load, 32-byte activation load).
//    A warp owns 32 output rows (two 16-row tiles) over a contiguous group range; the 4 warps of a CTA
//    split the CTA's group range; CTAs may split K further (S > 1), their partials summed in split order
//    by the last CTA to finish a tile. The partition depends on (N, K) only, never on M, so every
//    activation row gets the same arithmetic whatever M is (row invariance: a verify row equals a
//    one-row decode bit for bit).
#include <mutex>

#include "common.cuh"
#include "../../include/imspec.h"

namespace im {

constexpr int QG_WARPS = 4;              // warps per CTA
constexpr int QG_THREADS = QG_WARPS * 32;
constexpr int QG_ROWS = 32;              // output rows per CTA: two 16-row MMA tiles per warp
constexpr int QG_T = 2;                  // 16-row tiles per warp
constexpr uint32_t BF16X2_ONE = 0x3F803F80u;
constexpr uint32_t BF16X2_128 = 0x43004300u;  // bf16 128.0 in both halves; 128+q is exact for q < 128

static int g_split_override = 0;         // sweep hook: force the CTA-level K split (0 = automatic)
// Workspace layout, the same for every shape so that shapes may share one buffer: per-tile arrival
// counters in a fixed region at the start (kept at zero between launches), the CTA partials after it.
constexpr size_t QG_COUNTER_BYTES = 16384;
constexpr int QG_MAX_SPLIT_TILES = (int)(QG_COUNTER_BYTES / 4);

__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One packed word (8 codes, low nibble first) -> four bf16x2 registers (128+n_i, 128+n_{i+4}).
__device__ __forceinline__ void codes_to_bf16x2(uint32_t u, uint32_t* p) {
  p[0] = (u & 0x000F000Fu) | BF16X2_128;
  p[1] = ((u >> 4) & 0x000F000Fu) | BF16X2_128;
  p[2] = ((u >> 8) & 0x000F000Fu) | BF16X2_128;
  p[3] = ((u >> 12) & 0x000F000Fu) | BF16X2_128;
}

// 16 contiguous activations (8 bf16 pairs X[j] = (x_2j, x_2j+1)) -> the same pairing the codes get:
// px[4w+i] = (x_{8w+i}, x_{8w+i+4}).
__device__ __forceinline__ void acts_to_frag(const uint4& lo, const uint4& hi, uint32_t* px) {
  px[0] = __byte_perm(lo.x, lo.z, 0x5410);
  px[1] = __byte_perm(lo.x, lo.z, 0x7632);
  px[2] = __byte_perm(lo.y, lo.w, 0x5410);
  px[3] = __byte_perm(lo.y, lo.w, 0x7632);
  px[4] = __byte_perm(hi.x, hi.z, 0x5410);
  px[5] = __byte_perm(hi.x, hi.z, 0x7632);
  px[6] = __byte_perm(hi.y, hi.w, 0x5410);
  px[7] = __byte_perm(hi.y, hi.w, 0x7632);
}

__device__ __forceinline__ float silu_mul(float gate, float up) {
  // nn.silu(gate) * up with a bf16 rounding after every elementwise op: sigmoid, the product with the
  // gate, the product with up.
  const float a = round_bf(gate);
  const float u = round_bf(up);
  const float sig = round_bf(1.0f / (1.0f + expf(-a)));
  const float si = round_bf(a * sig);
  return si * u;
}

__device__ __forceinline__ float gelu_tanh_mul(float gate, float up) {
  // gelu_approx(gate) * up (Gemma-3 GeGLU): 0.5 a (1 + tanh(sqrt(2/pi) (a + 0.044715 a^3))), rounded to
  // bf16, times up.
  const float a = round_bf(gate);
  const float u = round_bf(up);
  const float inner = 0.7978845608028654f * (a + 0.044715f * a * a * a);
  const float ge = round_bf(0.5f * a * (1.0f + tanhf(inner)));
  return ge * u;
}

template <int NT, int EPI>
__device__ __forceinline__ void qgemm_mma_store(const float (&v)[QG_T][NT][4], uint16_t* y, const uint16_t* res,
                                                int M, int N, int rbase, int g, int t) {
  if constexpr (EPI == IM_EPI_SWIGLU || EPI == IM_EPI_GEGLU) {
    const int nout = N >> 1;
    const int f0 = (rbase >> 1) + g;  // tile 0 holds gate rows, tile 1 the matching up rows
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int f = f0 + ((i >> 1) << 3);
        const int m = nt * 8 + 2 * t + (i & 1);
        if (m < M && f < nout) {
          const float o = EPI == IM_EPI_SWIGLU ? silu_mul(v[0][nt][i], v[1][nt][i])
                                               : gelu_tanh_mul(v[0][nt][i], v[1][nt][i]);
          y[(size_t)m * nout + f] = to_bf(o);
        }
      }
    }
  } else {
#pragma unroll
  for (int tt = 0; tt < QG_T; tt++) {
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int r = rbase + tt * 16 + g + ((i >> 1) << 3);
        const int m = nt * 8 + 2 * t + (i & 1);
        if (m < M && r < N) {
          const size_t o = (size_t)m * N + r;
          if (EPI == IM_EPI_RESIDUAL) {
            y[o] = to_bf(bf(res[o]) + round_bf(v[tt][nt][i]));
          } else {
            y[o] = to_bf(v[tt][nt][i]);
          }
        }
      }
    }
  }
  }
}

template <int NT, int EPI, int U>
__global__ void __launch_bounds__(QG_THREADS, NT == 1 ? 4 : (NT == 2 ? 3 : 2))
qgemm_mma_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ sc, const uint16_t* __restrict__ bi,
                 const uint16_t* __restrict__ x, uint16_t* y, const uint16_t* res, int M, int N, int K, int S,
                 float* __restrict__ partial, unsigned* __restrict__ counters) {
  const int G = K >> 6;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int cg0 = (int)(((long long)G * split) / S);
  const int cg1 = (int)(((long long)G * (split + 1)) / S);
  const int span = cg1 - cg0;
  const int wg0 = cg0 + (span * warp) / QG_WARPS;
  const int wg1 = cg0 + (span * (warp + 1)) / QG_WARPS;
  const int rbase = tile * QG_ROWS;
  const size_t wstride = (size_t)(K >> 3);

  const uint32_t* wrow[QG_T][2];
  const uint16_t* srow[QG_T][2];
  const uint16_t* brow[QG_T][2];
#pragma unroll
  for (int tt = 0; tt < QG_T; tt++) {
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int r = min(rbase + tt * 16 + g + h * 8, N - 1);
      wrow[tt][h] = w + (size_t)r * wstride + 2 * t;
      srow[tt][h] = sc + (size_t)r * G;
      brow[tt][h] = bi + (size_t)r * G;
    }
  }
  const uint16_t* xrow[NT];
  bool xval[NT];
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const int m = nt * 8 + g;
    xval[nt] = m < M;
    xrow[nt] = x + (size_t)(xval[nt] ? m : 0) * K + 16 * t;
  }

  float tot[QG_T][NT][4];
#pragma unroll
  for (int tt = 0; tt < QG_T; tt++)
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int i = 0; i < 4; i++) tot[tt][nt][i] = 0.f;

  for (int gg = wg0; gg < wg1; gg += U) {
    const int cnt = min(U, wg1 - gg);
    uint2 wv[U][QG_T][2];
    uint16_t sv[U][QG_T][2], bv[U][QG_T][2];
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (u < cnt) {
#pragma unroll
        for (int tt = 0; tt < QG_T; tt++)
#pragma unroll
          for (int h = 0; h < 2; h++) {
            wv[u][tt][h] = ldg_stream_u2(wrow[tt][h] + (size_t)(gg + u) * 8);
            sv[u][tt][h] = ldg_u16(srow[tt][h] + gg + u);
            bv[u][tt][h] = ldg_u16(brow[tt][h] + gg + u);
          }
      }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      if (u < cnt) {
        uint32_t px[NT][8];
        float sx[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
          if (xval[nt]) {
            const uint16_t* xp = xrow[nt] + (size_t)(gg + u) * 64;
            const uint4 lo = ldg_u4(xp);
            const uint4 hi = ldg_u4(xp + 8);
            acts_to_frag(lo, hi, px[nt]);
          } else {
#pragma unroll
            for (int j = 0; j < 8; j++) px[nt][j] = 0u;
          }
#pragma unroll
          for (int i = 0; i < 4; i++) sx[nt][i] = 0.f;
#pragma unroll
          for (int j = 0; j < 4; j++)
            mma16816(sx[nt], BF16X2_ONE, BF16X2_ONE, BF16X2_ONE, BF16X2_ONE, px[nt][2 * j], px[nt][2 * j + 1]);
        }
#pragma unroll
        for (int tt = 0; tt < QG_T; tt++) {
          uint32_t pa[8], pb[8];
          codes_to_bf16x2(wv[u][tt][0].x, pa);
          codes_to_bf16x2(wv[u][tt][0].y, pa + 4);
          codes_to_bf16x2(wv[u][tt][1].x, pb);
          codes_to_bf16x2(wv[u][tt][1].y, pb + 4);
          float acc[NT][4];
#pragma unroll
          for (int nt = 0; nt < NT; nt++)
#pragma unroll
            for (int i = 0; i < 4; i++) acc[nt][i] = 0.f;
#pragma unroll
          for (int j = 0; j < 4; j++)
#pragma unroll
            for (int nt = 0; nt < NT; nt++)
              mma16816(acc[nt], pa[2 * j], pb[2 * j], pa[2 * j + 1], pb[2 * j + 1], px[nt][2 * j], px[nt][2 * j + 1]);
          const float s0 = bf(sv[u][tt][0]), s1 = bf(sv[u][tt][1]);
          const float b0 = fmaf(-128.f, s0, bf(bv[u][tt][0]));
          const float b1 = fmaf(-128.f, s1, bf(bv[u][tt][1]));
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
  }

  // CTA reduction over the warps' group slices, in warp order.
  constexpr int NV = QG_T * NT * 4;
  __shared__ float red[QG_WARPS][NV][32];
#pragma unroll
  for (int tt = 0; tt < QG_T; tt++)
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int i = 0; i < 4; i++) red[warp][(tt * NT + nt) * 4 + i][lane] = tot[tt][nt][i];
  __syncthreads();
  if (warp != 0) return;
  float v[QG_T][NT][4];
#pragma unroll
  for (int tt = 0; tt < QG_T; tt++)
#pragma unroll
    for (int nt = 0; nt < NT; nt++)
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int idx = (tt * NT + nt) * 4 + i;
        float a = red[0][idx][lane];
#pragma unroll
        for (int ww = 1; ww < QG_WARPS; ww++) a += red[ww][idx][lane];
        v[tt][nt][i] = a;
      }

  if (S > 1) {
    // Split-K across CTAs: publish this CTA's partial, and let the last CTA of the tile sum all partials
    // in split order (deterministic whatever order the CTAs finish in).
    float* mine = partial + ((size_t)tile * S + split) * NV * 32;
#pragma unroll
    for (int tt = 0; tt < QG_T; tt++)
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) __stcg(mine + ((tt * NT + nt) * 4 + i) * 32 + lane, v[tt][nt][i]);
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(counters + tile, 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != (unsigned)(S - 1)) return;
    __threadfence();
#pragma unroll
    for (int tt = 0; tt < QG_T; tt++)
#pragma unroll
      for (int nt = 0; nt < NT; nt++)
#pragma unroll
        for (int i = 0; i < 4; i++) v[tt][nt][i] = 0.f;
    for (int s = 0; s < S; s++) {
      const float* p = partial + ((size_t)tile * S + s) * NV * 32;
#pragma unroll
      for (int tt = 0; tt < QG_T; tt++)
#pragma unroll
        for (int nt = 0; nt < NT; nt++)
#pragma unroll
          for (int i = 0; i < 4; i++) v[tt][nt][i] += __ldcg(p + ((tt * NT + nt) * 4 + i) * 32 + lane);
    }
    if (lane == 0) counters[tile] = 0u;  // leave the workspace ready for the next launch
  }
  qgemm_mma_store<NT, EPI>(v, y, res, M, N, rbase, g, t);
}

// ---- v1: CUDA-core FMA, M <= 8 -----------------------------------------------------------------
constexpr int QF_ROWS = 4;  // output rows per warp

template <int MM, int EPI>
__global__ void __launch_bounds__(256)
qgemm_fma_kernel(const uint32_t* __restrict__ w, const uint16_t* __restrict__ sc, const uint16_t* __restrict__ bi,
                 const uint16_t* __restrict__ x, uint16_t* y, const uint16_t* res, int M, int N, int K) {
  const int wid = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  const int row0 = wid * QF_ROWS;
  if (row0 >= N) return;
  const int C = K >> 5;  // 32-value chunks per row
  const int G = K >> 6;
  float tot[QF_ROWS][MM];
#pragma unroll
  for (int r = 0; r < QF_ROWS; r++)
#pragma unroll
    for (int m = 0; m < MM; m++) tot[r][m] = 0.f;
  for (int c = lane; c < C; c += 32) {
    const int grp = c >> 1;
    uint4 wq[QF_ROWS];
#pragma unroll
    for (int r = 0; r < QF_ROWS; r++) {
      const int row = min(row0 + r, N - 1);
      wq[r] = ldg_stream_u4(w + (size_t)row * (K >> 3) + (size_t)c * 4);
    }
    float acc[QF_ROWS][MM];
    float sx[MM];
#pragma unroll
    for (int m = 0; m < MM; m++) {
      sx[m] = 0.f;
#pragma unroll
      for (int r = 0; r < QF_ROWS; r++) acc[r][m] = 0.f;
    }
#pragma unroll
    for (int sub = 0; sub < 4; sub++) {
      float xv[MM][8];
#pragma unroll
      for (int m = 0; m < MM; m++) {
        if (m < M) {
          const uint4 X = ldg_u4(x + (size_t)m * K + (size_t)c * 32 + sub * 8);
          xv[m][0] = bf_lo(X.x); xv[m][1] = bf_hi(X.x); xv[m][2] = bf_lo(X.y); xv[m][3] = bf_hi(X.y);
          xv[m][4] = bf_lo(X.z); xv[m][5] = bf_hi(X.z); xv[m][6] = bf_lo(X.w); xv[m][7] = bf_hi(X.w);
        } else {
#pragma unroll
          for (int e = 0; e < 8; e++) xv[m][e] = 0.f;
        }
#pragma unroll
        for (int e = 0; e < 8; e++) sx[m] += xv[m][e];
      }
#pragma unroll
      for (int r = 0; r < QF_ROWS; r++) {
        const uint32_t u = sub == 0 ? wq[r].x : sub == 1 ? wq[r].y : sub == 2 ? wq[r].z : wq[r].w;
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const float q = __uint_as_float(((u >> (4 * e)) & 0xFu) | 0x4B000000u) - 8388608.0f;
#pragma unroll
          for (int m = 0; m < MM; m++) acc[r][m] = fmaf(q, xv[m][e], acc[r][m]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < QF_ROWS; r++) {
      const int row = min(row0 + r, N - 1);
      const float s = bf(ldg_u16(sc + (size_t)row * G + grp));
      const float b = bf(ldg_u16(bi + (size_t)row * G + grp));
#pragma unroll
      for (int m = 0; m < MM; m++) tot[r][m] = fmaf(b, sx[m], fmaf(s, acc[r][m], tot[r][m]));
    }
  }
#pragma unroll
  for (int r = 0; r < QF_ROWS; r++)
#pragma unroll
    for (int m = 0; m < MM; m++) tot[r][m] = warp_sum(tot[r][m]);
  if (lane != 0) return;
#pragma unroll
  for (int r = 0; r < QF_ROWS; r++) {
    const int row = row0 + r;
    if (row >= N) break;
#pragma unroll
    for (int m = 0; m < MM; m++) {
      if (m < M) {
        const size_t o = (size_t)m * N + row;
        y[o] = EPI == IM_EPI_RESIDUAL ? to_bf(bf(res[o]) + round_bf(tot[r][m])) : to_bf(tot[r][m]);
      }
    }
  }
}

// ---- host side ----------------------------------------------------------------------------------
struct QgemmPlan {
  int tiles;   // 32-row CTA tiles
  int splits;  // CTA-level K split
  int nt;      // 8-row activation tiles
  size_t workspace;
};

static QgemmPlan plan_mma(int64_t M, int64_t N, int64_t K, bool have_workspace) {
  QgemmPlan p;
  p.tiles = (int)((N + QG_ROWS - 1) / QG_ROWS);
  p.nt = (int)((M + 7) / 8);
  const int G = (int)(K / 64);
  int s = 1;
  if (have_workspace) {
    // Aim for >= 8 CTAs (32 warps) per SM over 148 SMs; keep >= 2 groups per warp.
    const int target = 148 * 8;
    s = (target + p.tiles - 1) / p.tiles;
    const int cap = G / (QG_WARPS * 2);
    s = s < 1 ? 1 : (s > cap ? (cap < 1 ? 1 : cap) : s);
    if (g_split_override > 0) s = g_split_override < G ? g_split_override : G;
    if (p.tiles > QG_MAX_SPLIT_TILES) s = 1;
  }
  p.splits = s;
  // fixed counter region + partials (always sized for NT = 4)
  const size_t partials = s > 1 ? (size_t)p.tiles * s * QG_T * 4 * 4 * 32 * sizeof(float) : 0;
  p.workspace = s > 1 ? QG_COUNTER_BYTES + partials : 0;
  return p;
}

template <int NT, int EPI>
static void launch_mma(const QgemmPlan& p, const uint32_t* w, const uint16_t* s, const uint16_t* b,
                       const uint16_t* x, uint16_t* y, const uint16_t* res, int M, int N, int K, void* ws,
                       cudaStream_t st) {
  unsigned* counters = reinterpret_cast<unsigned*>(ws);
  float* partial = ws ? reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + QG_COUNTER_BYTES) : nullptr;
  dim3 grid(p.tiles, p.splits);
  qgemm_mma_kernel<NT, EPI, 4><<<grid, QG_THREADS, 0, st>>>(w, s, b, x, y, res, M, N, K, p.splits, partial, counters);
}

template <int EPI>
static void dispatch_mma(const QgemmPlan& p, const uint32_t* w, const uint16_t* s, const uint16_t* b,
                         const uint16_t* x, uint16_t* y, const uint16_t* res, int M, int N, int K, void* ws,
                         cudaStream_t st) {
  switch (p.nt) {
    case 1: launch_mma<1, EPI>(p, w, s, b, x, y, res, M, N, K, ws, st); break;
    case 2: launch_mma<2, EPI>(p, w, s, b, x, y, res, M, N, K, ws, st); break;
    case 3: launch_mma<3, EPI>(p, w, s, b, x, y, res, M, N, K, ws, st); break;
    default: launch_mma<4, EPI>(p, w, s, b, x, y, res, M, N, K, ws, st); break;
  }
}

template <int EPI>
static void dispatch_fma(const uint32_t* w, const uint16_t* s, const uint16_t* b, const uint16_t* x, uint16_t* y,
                         const uint16_t* res, int M, int N, int K, cudaStream_t st) {
  const int warps = (N + QF_ROWS - 1) / QF_ROWS;
  const int blocks = (warps * 32 + 255) / 256;
#define IM_FMA_CASE(MMV) \
  case MMV: qgemm_fma_kernel<MMV, EPI><<<blocks, 256, 0, st>>>(w, s, b, x, y, res, M, N, K); break;
  switch (M) {
    IM_FMA_CASE(1) IM_FMA_CASE(2) IM_FMA_CASE(3) IM_FMA_CASE(4)
    IM_FMA_CASE(5) IM_FMA_CASE(6) IM_FMA_CASE(7) default: IM_FMA_CASE(8)
  }
#undef IM_FMA_CASE
}

}  // namespace im

using namespace im;

extern "C" size_t im_qgemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
  if (M < 1 || N < 1 || K < 64 || K % 64) return 0;
  return plan_mma(M, N, K, true).workspace;
}

extern "C" int im_qgemm_set_splits(int splits) {
  IM_REQUIRE(splits >= 0, IM_INVALID, "im_qgemm_set_splits: negative split");
  g_split_override = splits;
  return IM_OK;
}

extern "C" int im_qgemm_w4g64_ex(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                                 const uint16_t* x, uint16_t* y, const uint16_t* residual, int64_t M, int64_t N,
                                 int64_t K, int epilogue, int variant, void* workspace, size_t workspace_bytes,
                                 void* stream) {
  clear_error();
  IM_REQUIRE(M >= 0 && N >= 1 && K >= 64, IM_INVALID, "im_qgemm: bad sizes M=%lld N=%lld K=%lld", (long long)M,
             (long long)N, (long long)K);
  IM_REQUIRE(K % 64 == 0, IM_UNSUPPORTED, "im_qgemm: K=%lld is not a multiple of the group size 64", (long long)K);
  IM_REQUIRE(N <= (1 << 30) && K <= (1 << 24), IM_UNSUPPORTED, "im_qgemm: N or K too large");
  if (M == 0) return IM_OK;
  IM_REQUIRE(w && scales && biases && x && y, IM_INVALID, "im_qgemm: null pointer");
  IM_REQUIRE(aligned(w, 16) && aligned(x, 16), IM_INVALID, "im_qgemm: w and x must be 16-byte aligned");
  IM_REQUIRE(aligned(scales, 2) && aligned(biases, 2) && aligned(y, 2), IM_INVALID, "im_qgemm: misaligned bf16");
  IM_REQUIRE(epilogue >= IM_EPI_STORE && epilogue <= IM_EPI_GEGLU, IM_INVALID, "im_qgemm: unknown epilogue %d",
             epilogue);
  IM_REQUIRE(epilogue != IM_EPI_RESIDUAL || residual, IM_INVALID, "im_qgemm: residual epilogue needs a residual");
  const bool glu = epilogue == IM_EPI_SWIGLU || epilogue == IM_EPI_GEGLU;
  IM_REQUIRE(!glu || N % 32 == 0, IM_INVALID, "im_qgemm: gated epilogues need N (gate+up rows) % 32 == 0");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int v = variant == IM_QGEMM_AUTO ? IM_QGEMM_MMA : variant;
  if (v == IM_QGEMM_FMA) {
    IM_REQUIRE(M <= 8, IM_UNSUPPORTED, "im_qgemm: the FMA variant covers M <= 8 (M=%lld)", (long long)M);
    IM_REQUIRE(!glu, IM_UNSUPPORTED, "im_qgemm: the FMA variant has no gated epilogue");
    if (epilogue == IM_EPI_RESIDUAL)
      dispatch_fma<IM_EPI_RESIDUAL>(w, scales, biases, x, y, residual, (int)M, (int)N, (int)K, st);
    else
      dispatch_fma<IM_EPI_STORE>(w, scales, biases, x, y, residual, (int)M, (int)N, (int)K, st);
    return check_launch("qgemm_fma");
  }
  IM_REQUIRE(v == IM_QGEMM_MMA, IM_INVALID, "im_qgemm: unknown variant %d", variant);
  IM_REQUIRE(M <= 32, IM_UNSUPPORTED, "im_qgemm: the warp-MMA variant covers M <= 32 (M=%lld)", (long long)M);
  QgemmPlan p = plan_mma(M, N, K, workspace != nullptr);
  if (p.splits > 1) {
    IM_REQUIRE(workspace_bytes >= p.workspace && aligned(workspace, 256), IM_INVALID,
               "im_qgemm: workspace of %zu bytes (256-aligned) needed, %zu given", p.workspace, workspace_bytes);
  }
  void* ws = p.splits > 1 ? workspace : nullptr;
  switch (epilogue) {
    case IM_EPI_STORE: dispatch_mma<IM_EPI_STORE>(p, w, scales, biases, x, y, residual, (int)M, (int)N, (int)K, ws, st); break;
    case IM_EPI_RESIDUAL: dispatch_mma<IM_EPI_RESIDUAL>(p, w, scales, biases, x, y, residual, (int)M, (int)N, (int)K, ws, st); break;
    case IM_EPI_SWIGLU: dispatch_mma<IM_EPI_SWIGLU>(p, w, scales, biases, x, y, residual, (int)M, (int)N, (int)K, ws, st); break;
    default: dispatch_mma<IM_EPI_GEGLU>(p, w, scales, biases, x, y, residual, (int)M, (int)N, (int)K, ws, st); break;
  }
  return check_launch("qgemm_mma");
}

extern "C" int im_qgemm_w4g64(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                              const uint16_t* x, uint16_t* y, int64_t M, int64_t N, int64_t K, void* stream) {
  return im_qgemm_w4g64_ex(w, scales, biases, x, y, nullptr, M, N, K, IM_EPI_STORE, IM_QGEMM_AUTO, nullptr, 0,
                           stream);
}

// ---- entry point for callers that cannot allocate device memory ---------------------------------------------
// Some callers of this library cannot call cudaMalloc: code running inside another runtime's allocator
// discipline (a host process whose device memory is owned by a pool it may not grow, a plugin loaded into an
// engine that forbids allocations on its decode path) or code that must not synchronise the device, which a
// first-use cudaMalloc can do. For them the split-K qGEMM keeps its scratch (per-tile arrival counters and CTA
// partials) in one file-scope device array instead of a caller-provided workspace.
//
// The array is allocated when the library is loaded, on every GPU that loads it, and held until the process
// exits. Its address is looked up once per device with cudaGetSymbolAddress (the host-side name of a __device__
// array is not a device address). The first call on a device does that set-up and queues a cudaMemsetAsync of
// the counters on the caller's stream, ahead of its kernel, so the zeroing is ordered before the kernel whatever
// kind of stream the caller uses; make that first call before any stream capture on the device. Calls never
// allocate. Every call shares the one array: the kernel returns its counters to zero, but calls that overlap on
// the GPU (two streams, or two host threads) race on it and must not be issued.
constexpr size_t QG_NOALLOC_BYTES = (size_t)8 << 20;  // 16 KiB of counters + ~8 MiB of partials
static __device__ __align__(256) unsigned char g_qgemm_noalloc_scratch[QG_NOALLOC_BYTES];

namespace {
constexpr int QG_NOALLOC_MAX_DEVICES = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[QG_NOALLOC_MAX_DEVICES] = {};
}  // namespace

static int noalloc_scratch(void** out, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("im_qgemm_w4g64_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
    return IM_CUDA_ERROR;
  }
  IM_REQUIRE(dev >= 0 && dev < QG_NOALLOC_MAX_DEVICES, IM_UNSUPPORTED, "im_qgemm_w4g64_noalloc: device %d", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_qgemm_noalloc_scratch);
    if (e != cudaSuccess) {
      set_error("im_qgemm_w4g64_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return IM_CUDA_ERROR;
    }
    e = cudaMemsetAsync(ptr, 0, QG_COUNTER_BYTES, stream);
    if (e != cudaSuccess) {
      set_error("im_qgemm_w4g64_noalloc: zeroing the counters: %s", cudaGetErrorString(e));
      return IM_CUDA_ERROR;
    }
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return IM_OK;
}

extern "C" size_t im_qgemm_noalloc_capacity(void) { return QG_NOALLOC_BYTES; }

extern "C" int im_qgemm_w4g64_noalloc(const uint32_t* w, const uint16_t* scales, const uint16_t* biases,
                                      const uint16_t* x, uint16_t* y, int64_t M, int64_t N, int64_t K, void* stream) {
  clear_error();
  IM_REQUIRE(M >= 0 && N >= 1 && K >= 64, IM_INVALID, "im_qgemm_w4g64_noalloc: bad sizes M=%lld N=%lld K=%lld",
             (long long)M, (long long)N, (long long)K);
  IM_REQUIRE(K % 64 == 0, IM_UNSUPPORTED, "im_qgemm_w4g64_noalloc: K=%lld is not a multiple of 64", (long long)K);
  IM_REQUIRE(N <= (1 << 30) && K <= (1 << 24), IM_UNSUPPORTED, "im_qgemm_w4g64_noalloc: N or K too large");
  IM_REQUIRE(M <= 32, IM_UNSUPPORTED, "im_qgemm_w4g64_noalloc: M=%lld exceeds 32", (long long)M);
  if (M == 0) return IM_OK;
  IM_REQUIRE(w && scales && biases && x && y, IM_INVALID, "im_qgemm_w4g64_noalloc: null pointer");
  IM_REQUIRE(aligned(w, 16) && aligned(x, 16), IM_INVALID, "im_qgemm_w4g64_noalloc: w and x must be 16-byte aligned");
  IM_REQUIRE(aligned(scales, 2) && aligned(biases, 2) && aligned(y, 2), IM_INVALID,
             "im_qgemm_w4g64_noalloc: misaligned bf16");
  const QgemmPlan p = plan_mma(M, N, K, true);
  IM_REQUIRE(p.workspace <= QG_NOALLOC_BYTES, IM_UNSUPPORTED,
             "im_qgemm_w4g64_noalloc: this shape needs %zu bytes of scratch; the static scratch holds %zu "
             "(use im_qgemm_w4g64_ex with a workspace)",
             p.workspace, QG_NOALLOC_BYTES);
  void* scratch = nullptr;
  if (p.splits > 1) {
    const int rc = noalloc_scratch(&scratch, reinterpret_cast<cudaStream_t>(stream));
    if (rc) return rc;
  }
  dispatch_mma<IM_EPI_STORE>(p, w, scales, biases, x, y, nullptr, (int)M, (int)N, (int)K, scratch,
                             reinterpret_cast<cudaStream_t>(stream));
  return check_launch("qgemm_mma (no-alloc)");
}
