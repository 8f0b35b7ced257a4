// qGEMM v6: the packed 4-bit GEMM for more than 32 activation rows, on the 5th-generation tensor cores
// (tcgen05.mma with the accumulators in tensor memory).
//
// The arithmetic is the warp-MMA kernel's (qgemm_packed.cu), bit for bit, as if the rows were computed in
// 32-row calls: per (weight row, activation row, 64-wide group) the exact bf16 codes 128+q times the activations
// summed on the tensor pipe in four K=16 steps whose k-sets (and column order) are those of the warp-MMA
// fragments, the fp32 group affine tot = fmaf(b - 128 s, sum(x), fmaf(s, acc, tot)) in group order, the same
// K splits summed in split order, the same epilogues. A tcgen05 K=16 step over a given 16-column slice returns
// the same fp32 bits as the m16n8k16 warp MMA over the same slice; the GPU tests hold every path to that.
//
// Machinery:
//  * qtc_prep_kernel (grid: groups x 64-row chunks) applies the optional RMSNorm, computes the per-group
//    activation sums in the warp-MMA kernel's order, and writes each (chunk, group) as an 8 KB tensor-core
//    tile: 64 rows of 128 bytes, K-major, 128-byte swizzled (16-byte column c of row r at (c ^ r%8)), columns
//    permuted to the fragment k-sets; plus the 64 group sums.
//  * qtc_kernel: a CTA owns 4 tiles (128 weight rows) x one K range of the split plan x one 64-row chunk;
//    9 warps. The MMA warp copies the chunk's activation tiles of the whole K range into shared memory with
//    bulk copies (one mbarrier per group), then per group issues 4 MMAs (M = 128, N = 64, K = 16) into one of two
//    tensor-memory accumulators and commits to the stage and accumulator barriers. Math warp w (0..7) owns tile
//    w%4 and the weight-code half w/4 of every unit: it expands the codes to bf16 into a 4-stage A ring (two
//    groups ahead), and per group loads accumulator columns [32 (w/4), +32) of its tile's 32 rows (tensor-memory
//    lane quadrant w%4) and applies the group affine into 32 fp32 totals per thread.
//  * Split-K: per (chunk, tile, column half) partials; the last split to arrive sums them in split order and
//    runs the epilogue (store / residual (+ sums of squares) / SwiGLU / GeGLU) in the warp-MMA kernel's order.
// Every mbarrier wait is bounded (1 s); a wait that runs out sets the error word (the last word of the counter
// region, read by im_qgemm_packed_status) and an abort flag that every later wait of the CTA honours, and the
// CTA still waits (bounded) for its issued MMAs before it frees its tensor memory.
#include "common.cuh"
#include "qgemm_packed.cuh"
#include "../../include/imspec.h"

namespace im {

constexpr int QT_MATH = 8;                       // math warps
constexpr int QT_THREADS = (QT_MATH + 1) * 32;   // + the MMA warp
constexpr int QT_ROWS = 64;                      // activation rows per CTA (one chunk) = MMA N
constexpr int QT_STAGES = 4;                     // A ring
constexpr int QT_AHEAD = 2;                      // groups expanded ahead of the epilogue
constexpr int QT_A = 128 * 128;                  // bytes of one A stage: 128 rows x 64 bf16
constexpr int QT_B = QT_ROWS * 128;              // bytes of one activation tile: 64 rows x 64 bf16
constexpr int QT_SX = QT_ROWS * 4;               // bytes of one tile's group sums
constexpr uint32_t QT_TMEM_COLS = 2 * QT_ROWS;   // two accumulators
constexpr int QT_BARS = 2 * QT_STAGES + 4 + Q4_RMAX;
constexpr unsigned long long QT_WAIT_NS = 1000000000ull;
constexpr uint32_t QT_128 = 0x43004300u;
// instruction descriptor: f32 accumulate, bf16 A and B, both K-major, N = 64, M = 128
constexpr uint32_t QT_IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(QT_ROWS >> 3) << 17) | ((128u >> 4) << 24);

struct QtArgs {
  const unsigned char* wp;  // packed units
  const unsigned char* xt;  // [chunks][G] activation tiles (QT_B bytes each)
  const float* sxt;         // [chunks][G][64] group sums
  uint16_t* y;
  const uint16_t* res;
  float* out_sq;
  float* partial;
  unsigned* counters;
  unsigned* error;
  int M, N, K, tiles, splits, sq_ld, gmax;
};

__host__ __device__ constexpr size_t qtc_smem_bytes(int gmax) {
  return 1024 + (size_t)QT_STAGES * QT_A + (size_t)gmax * (QT_B + QT_SX) + QT_BARS * 8 + 16;
}

__device__ __forceinline__ uint32_t qt_smem(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool qt_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

__device__ __forceinline__ unsigned long long qt_clock() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase of `parity`; false when this CTA has given up (now or earlier).
__device__ __forceinline__ bool qt_wait(unsigned long long* bar, uint32_t parity, volatile int* abort_flag,
                                        unsigned* error) {
  const uint32_t b = qt_smem(bar);
  if (*abort_flag) return false;
  if (qt_try_wait(b, parity)) return true;
  const unsigned long long t0 = qt_clock();
  while (true) {
    if (qt_try_wait(b, parity)) return true;
    if (*abort_flag) return false;
    if (qt_clock() - t0 > QT_WAIT_NS) {
      *abort_flag = 1;
      atomicExch(error, 1u);
      return false;
    }
  }
}

__device__ __forceinline__ void qt_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(qt_smem(bar)) : "memory");
}

__device__ __forceinline__ uint64_t qt_desc(uint32_t saddr) {
  // K-major, 128-byte swizzle: 8-row groups 1024 bytes apart (SBO), leading offset 1 (unused), version 1
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void qt_codes(uint32_t u, uint32_t* p) {
  p[0] = (u & 0x000F000Fu) | QT_128;
  p[1] = ((u >> 4) & 0x000F000Fu) | QT_128;
  p[2] = ((u >> 8) & 0x000F000Fu) | QT_128;
  p[3] = ((u >> 12) & 0x000F000Fu) | QT_128;
}

// Byte offset of the 4-byte pair at (row r, column pair 2t of 16-byte chunk c) in a 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t qt_sw(int r, int c, int t) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4) + 4 * t);
}

// ---- prologue: activation tiles -------------------------------------------------------------------------
// grid (G, chunks), 256 threads = 64 rows x 4 quarters of a group; the warp-MMA kernel's prologue arithmetic.
__global__ void __launch_bounds__(256)
qtc_prep_kernel(const uint16_t* __restrict__ x, int M, int K, const float* __restrict__ norm_sq, int norm_parts,
                int sq_ld, const uint16_t* __restrict__ norm_w, float eps, int gemma_norm,
                unsigned char* __restrict__ xt, float* __restrict__ sxt) {
  pdl_wait();
  pdl_trigger();
  const int grp = blockIdx.x, chunk = blockIdx.y, G = K >> 6;
  const int m = threadIdx.x >> 2, tq = threadIdx.x & 3;
  const int row = chunk * QT_ROWS + m;
  uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
  float part = 0.f;
  if (row < M) {
    const uint16_t* xp = x + (size_t)row * K + (size_t)grp * 64 + 16 * tq;
    lo = __ldg(reinterpret_cast<const uint4*>(xp));
    hi = __ldg(reinterpret_cast<const uint4*>(xp + 8));
    if (norm_w) {
      float s = 0.f;
      for (int p = 0; p < norm_parts; p++) s += norm_sq[(size_t)p * sq_ld + row];
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(s, (float)K) + eps));
      const uint16_t* wv = norm_w + (size_t)grp * 64 + 16 * tq;
      uint32_t* l32 = reinterpret_cast<uint32_t*>(&lo);
      uint32_t* h32 = reinterpret_cast<uint32_t*>(&hi);
#pragma unroll
      for (int e = 0; e < 8; e++) {
        uint32_t* word = e < 4 ? &l32[e] : &h32[e - 4];
        const float w0 = gemma_norm ? 1.0f + bf(wv[2 * e]) : bf(wv[2 * e]);
        const float w1 = gemma_norm ? 1.0f + bf(wv[2 * e + 1]) : bf(wv[2 * e + 1]);
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
  // fragment pairs: (k, k+4) of each 8-wide half, in the order of the warp-MMA kernel's B fragments
  const uint32_t w[8] = {__byte_perm(lo.x, lo.z, 0x5410), __byte_perm(lo.x, lo.z, 0x7632),
                         __byte_perm(lo.y, lo.w, 0x5410), __byte_perm(lo.y, lo.w, 0x7632),
                         __byte_perm(hi.x, hi.z, 0x5410), __byte_perm(hi.x, hi.z, 0x7632),
                         __byte_perm(hi.y, hi.w, 0x5410), __byte_perm(hi.y, hi.w, 0x7632)};
  // pair i belongs to K=16 step i/2, 16-byte chunk 2 (i/2) + i%2 of the row, column pair tq
  unsigned char* tile = xt + ((size_t)chunk * G + grp) * QT_B;
#pragma unroll
  for (int i = 0; i < 8; i++) *reinterpret_cast<uint32_t*>(tile + qt_sw(m, i, tq)) = w[i];
  part += __shfl_xor_sync(0xffffffffu, part, 1);
  part += __shfl_xor_sync(0xffffffffu, part, 2);
  if (tq == 0) sxt[((size_t)chunk * G + grp) * QT_ROWS + m] = part;
}

// ---- the GEMM -------------------------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(QT_THREADS, 2)
qtc_kernel(QtArgs a) {
  extern __shared__ unsigned char qt_raw[];
  const uint32_t raw = qt_smem(qt_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* sbase = qt_raw + (base - raw);
  const uint32_t sA = base, sB = base + QT_STAGES * QT_A;
  float* sxs = reinterpret_cast<float*>(sbase + QT_STAGES * QT_A + (size_t)a.gmax * QT_B);
  unsigned long long* bars =
      reinterpret_cast<unsigned long long*>(sbase + QT_STAGES * QT_A + (size_t)a.gmax * (QT_B + QT_SX));
  unsigned long long* a_full = bars;
  unsigned long long* a_empty = bars + QT_STAGES;
  unsigned long long* t_full = bars + 2 * QT_STAGES;
  unsigned long long* t_empty = t_full + 2;
  unsigned long long* b_full = t_empty + 2;
  uint32_t* holder = reinterpret_cast<uint32_t*>(bars + QT_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(holder + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.K >> 6, split = blockIdx.y, chunk = blockIdx.z;
  const int cg0 = (int)(((long long)G * split) / a.splits);
  const int cg1 = (int)(((long long)G * (split + 1)) / a.splits);
  const int ng = cg1 - cg0;
  const int mrows = min(QT_ROWS, a.M - chunk * QT_ROWS);

  if (warp == QT_MATH) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(qt_smem(holder)),
                 "r"(QT_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < QT_STAGES; s++) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(qt_smem(&a_full[s])), "r"((uint32_t)QT_MATH));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(qt_smem(&a_empty[s])), "r"(1u));
    }
    for (int b = 0; b < 2; b++) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(qt_smem(&t_full[b])), "r"(1u));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(qt_smem(&t_empty[b])), "r"((uint32_t)QT_MATH));
    }
    for (int g = 0; g < Q4_RMAX; g++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(qt_smem(&b_full[g])), "r"(1u));
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *holder;

  if (warp == QT_MATH) {
    // ---- MMA warp: activation tiles of the K range, then 4 MMAs per group -------------------------------
    int issued = -1;
    if (lane == 0) {
      pdl_wait();
      pdl_trigger();
      for (int gl = 0; gl < ng; gl++) {
        const size_t t = (size_t)chunk * G + cg0 + gl;
        const uint32_t bar = qt_smem(&b_full[gl]);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"((uint32_t)(QT_B + QT_SX))
                     : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         sB + (uint32_t)(gl * QT_B)),
                     "l"(a.xt + t * QT_B), "r"((uint32_t)QT_B), "r"(bar)
                     : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         qt_smem(sxs + gl * QT_ROWS)),
                     "l"(a.sxt + t * QT_ROWS), "r"((uint32_t)QT_SX), "r"(bar)
                     : "memory");
      }
      for (int gl = 0; gl < ng; gl++) {
        const int s = gl % QT_STAGES, buf = gl & 1;
        if (!qt_wait(&a_full[s], (uint32_t)((gl / QT_STAGES) & 1), abort_flag, a.error)) break;
        if (!qt_wait(&b_full[gl], 0u, abort_flag, a.error)) break;
        if (gl >= 2 && !qt_wait(&t_empty[buf], (uint32_t)(((gl >> 1) - 1) & 1), abort_flag, a.error)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + (uint32_t)(buf * QT_ROWS);
#pragma unroll
        for (int k4 = 0; k4 < 4; k4++) {
          const uint64_t ad = qt_desc(sA + (uint32_t)(s * QT_A + 32 * k4));
          const uint64_t bd = qt_desc(sB + (uint32_t)(gl * QT_B + 32 * k4));
          asm volatile(
              "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
              "l"(ad), "l"(bd), "r"(QT_IDESC), "r"((uint32_t)(k4 > 0)));
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         qt_smem(&a_empty[s]))
                     : "memory");
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         qt_smem(&t_full[buf]))
                     : "memory");
        issued = gl;
      }
      if (*abort_flag && issued >= 0) {
        // the MMAs already issued finish before their tensor memory is freed
        const unsigned long long t0 = qt_clock();
        const uint32_t b = qt_smem(&t_full[issued & 1]);
        while (!qt_try_wait(b, (uint32_t)((issued >> 1) & 1)) && qt_clock() - t0 < QT_WAIT_NS) {
        }
      }
    } else {
      pdl_wait();
      pdl_trigger();
    }
    __syncwarp();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(QT_TMEM_COLS));
    return;
  }

  // ---- math warps ----------------------------------------------------------------------------------------
  const int q = warp & 3, h = warp >> 2;
  const int tile = blockIdx.x * 4 + q;
  const bool live = tile < a.tiles;
  const int g8 = lane >> 2, t4 = lane & 3;
  const unsigned char* up = a.wp + ((size_t)(live ? tile : 0) * G + cg0) * Q4_UNIT;
  if (live && h == 0 && lane == 0)
    for (int u = 0; u < ng; u += 16)
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(up + (size_t)u * Q4_UNIT),
                   "r"((uint32_t)min(16, ng - u) * Q4_UNIT)
                   : "memory");
  auto load_codes = [&](int gl) -> uint4 {
    if (!live || gl >= ng) return make_uint4(0, 0, 0, 0);
    return ldg_stream_u4(up + (size_t)gl * Q4_UNIT + lane * 32 + h * 16);
  };
  // scale and bias of this thread's row (tile row `lane`) in group gl
  auto load_sb = [&](int gl) -> uint32_t {
    if (!live || gl >= ng) return 0u;
    const unsigned char* sb = up + (size_t)gl * Q4_UNIT + 1024 + (lane & 7) * 16 + (lane >> 3) * 2;
    const uint32_t sv = __ldg(reinterpret_cast<const uint16_t*>(sb));
    const uint32_t bv = __ldg(reinterpret_cast<const uint16_t*>(sb + 8));
    return sv | (bv << 16);
  };
  // codes of group gl -> A stage gl % QT_STAGES: this warp writes rows 32q + 16h + {g, g + 8}
  auto expand = [&](int gl, uint4 c) -> bool {
    const int s = gl % QT_STAGES;
    if (gl >= QT_STAGES && !qt_wait(&a_empty[s], (uint32_t)(((gl / QT_STAGES) - 1) & 1), abort_flag, a.error))
      return false;
    if (live) {
      unsigned char* st = sbase + (size_t)s * QT_A;
      const uint32_t words[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
      for (int wi = 0; wi < 4; wi++) {
        const int r = 32 * q + 16 * h + g8 + 8 * (wi >> 1), hw = wi & 1;
        uint32_t p[4];
        qt_codes(words[wi], p);
#pragma unroll
        for (int n = 0; n < 4; n++) {
          const int step = 2 * hw + (n >> 1);  // K=16 step of nibbles (n, n + 4)
          *reinterpret_cast<uint32_t*>(st + qt_sw(r, 2 * step + (n & 1), t4)) = p[n];
        }
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) qt_arrive(&a_full[s]);
    return true;
  };

  float tot[32];
#pragma unroll
  for (int j = 0; j < 32; j++) tot[j] = 0.f;
  bool ok = true;
  // before the dependency wait: the first groups' codes (weights only)
  uint4 cur = load_codes(0);
  for (int d = 0; d < QT_AHEAD && d < ng && ok; d++) {
    const uint4 nxt = load_codes(d + 1);
    ok = expand(d, cur);
    cur = nxt;
  }
  pdl_wait();
  pdl_trigger();
  uint32_t sb_cur = load_sb(0);
  for (int gl = 0; gl < ng && ok; gl++) {
    const int dq = gl + QT_AHEAD;
    if (dq < ng) {
      const uint4 nxt = load_codes(dq + 1);
      ok = expand(dq, cur);
      cur = nxt;
      if (!ok) break;
    }
    const uint32_t sb_next = load_sb(gl + 1);
    const int buf = gl & 1;
    if (!qt_wait(&t_full[buf], (uint32_t)((gl >> 1) & 1), abort_flag, a.error) ||
        !qt_wait(&b_full[gl], 0u, abort_flag, a.error)) {
      ok = false;
      break;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    uint32_t acc[32];
    const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * QT_ROWS + 32 * h);
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(acc[0]), "=r"(acc[1]), "=r"(acc[2]), "=r"(acc[3]), "=r"(acc[4]), "=r"(acc[5]), "=r"(acc[6]),
          "=r"(acc[7]), "=r"(acc[8]), "=r"(acc[9]), "=r"(acc[10]), "=r"(acc[11]), "=r"(acc[12]), "=r"(acc[13]),
          "=r"(acc[14]), "=r"(acc[15]), "=r"(acc[16]), "=r"(acc[17]), "=r"(acc[18]), "=r"(acc[19]), "=r"(acc[20]),
          "=r"(acc[21]), "=r"(acc[22]), "=r"(acc[23]), "=r"(acc[24]), "=r"(acc[25]), "=r"(acc[26]), "=r"(acc[27]),
          "=r"(acc[28]), "=r"(acc[29]), "=r"(acc[30]), "=r"(acc[31])
        : "r"(ta));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncwarp();
    if (lane == 0) qt_arrive(&t_empty[buf]);
    const float s0 = bf_lo(sb_cur), b0 = fmaf(-128.f, s0, bf_hi(sb_cur));
    const float4* sx4 = reinterpret_cast<const float4*>(sxs + gl * QT_ROWS + 32 * h);
#pragma unroll
    for (int j4 = 0; j4 < 8; j4++) {
      const float4 sx = sx4[j4];
      tot[4 * j4 + 0] = fmaf(b0, sx.x, fmaf(s0, __uint_as_float(acc[4 * j4 + 0]), tot[4 * j4 + 0]));
      tot[4 * j4 + 1] = fmaf(b0, sx.y, fmaf(s0, __uint_as_float(acc[4 * j4 + 1]), tot[4 * j4 + 1]));
      tot[4 * j4 + 2] = fmaf(b0, sx.z, fmaf(s0, __uint_as_float(acc[4 * j4 + 2]), tot[4 * j4 + 2]));
      tot[4 * j4 + 3] = fmaf(b0, sx.w, fmaf(s0, __uint_as_float(acc[4 * j4 + 3]), tot[4 * j4 + 3]));
    }
    sb_cur = sb_next;
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();  // every MMA of this CTA has completed: the MMA warp frees the tensor memory
  if (!ok || *abort_flag || !live) return;

  // ---- split-K: per (chunk, tile, half) partials; the last split sums them in split order
  const size_t slot = ((size_t)chunk * a.tiles + tile) * 2 + h;
  if (a.splits > 1) {
    float* mine = a.partial + (slot * a.splits + split) * 1024;
#pragma unroll
    for (int j = 0; j < 32; j++) __stcg(mine + j * 32 + lane, tot[j]);
    __threadfence();
    __syncwarp();
    unsigned prev = 0;
    if (lane == 0) prev = atomicAdd(a.counters + slot, 1u);
    prev = __shfl_sync(0xffffffffu, prev, 0);
    if (prev != (unsigned)(a.splits - 1)) return;
    __threadfence();
#pragma unroll
    for (int j = 0; j < 32; j++) tot[j] = 0.f;
    for (int sp = 0; sp < a.splits; sp++) {
      const float* src = a.partial + (slot * a.splits + sp) * 1024;
      float buf[32];
#pragma unroll
      for (int j = 0; j < 32; j++) buf[j] = __ldcg(src + j * 32 + lane);
#pragma unroll
      for (int j = 0; j < 32; j++) tot[j] += buf[j];
    }
    if (lane == 0) a.counters[slot] = 0u;
  }

  // ---- epilogue: this thread's weight row (tile row `lane`) x activation rows 32h .. 32h + 31 of the chunk
  const int rbase = tile * 32;
  const int m0 = chunk * QT_ROWS + 32 * h;
  if constexpr (EPI == IM_EPI_SWIGLU || EPI == IM_EPI_GEGLU) {
    // tile rows 0-15 are gate features, rows 16-31 the matching up features
    const int nout = a.N >> 1;
    const int f = (rbase >> 1) + lane;
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const float up_v = __shfl_down_sync(0xffffffffu, tot[j], 16);
      if (lane < 16 && 32 * h + j < mrows && f < nout) {
        const float ga = round_bf(tot[j]), uu = round_bf(up_v);
        float o;
        if (EPI == IM_EPI_SWIGLU) {
          const float sig = round_bf(1.0f / (1.0f + expf(-ga)));
          o = round_bf(ga * sig) * uu;
        } else {
          const float inner = 0.7978845608028654f * (ga + 0.044715f * ga * ga * ga);
          o = round_bf(0.5f * ga * (1.0f + tanhf(inner))) * uu;
        }
        a.y[(size_t)(m0 + j) * nout + f] = to_bf(o);
      }
    }
  } else {
    const int r = rbase + lane;
#pragma unroll
    for (int j = 0; j < 32; j++) {
      const bool valid = 32 * h + j < mrows && r < a.N;
      float hv = 0.f;
      if (valid) {
        const size_t o = (size_t)(m0 + j) * a.N + r;
        const uint16_t hq = EPI == IM_EPI_RESIDUAL ? to_bf(bf(a.res[o]) + round_bf(tot[j])) : to_bf(tot[j]);
        a.y[o] = hq;
        hv = bf(hq);
      }
      if (a.out_sq) {
        // the warp-MMA kernel's order: rows g, g + 8, g + 16, g + 24 chained per g, then a butterfly over g
        const float x8 = __shfl_sync(0xffffffffu, hv, (lane + 8) & 31);
        const float x16 = __shfl_sync(0xffffffffu, hv, (lane + 16) & 31);
        const float x24 = __shfl_sync(0xffffffffu, hv, (lane + 24) & 31);
        float v = fmaf(x24, x24, fmaf(x16, x16, fmaf(x8, x8, fmaf(hv, hv, 0.f))));
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        if (lane == 0 && 32 * h + j < mrows) a.out_sq[(size_t)tile * a.sq_ld + m0 + j] = v;
      }
    }
  }
}

template <int EPI>
static int qtc_launch_gemm(const QtArgs& a, const Q4Plan& p, int chunks, cudaStream_t st) {
  static bool configured = false;
  const size_t smem = qtc_smem_bytes(a.gmax);
  if (!configured) {
    const cudaError_t e = cudaFuncSetAttribute(qtc_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)qtc_smem_bytes(Q4_RMAX));
    if (e != cudaSuccess) {
      set_error("qGEMM (tensor cores): cannot reserve shared memory: %s", cudaGetErrorString(e));
      return IM_CUDA_ERROR;
    }
    configured = true;
  }
  dim3 grid(p.ctas_x, p.splits, chunks);
  return launch("qtc_kernel", qtc_kernel<EPI>, grid, dim3(QT_THREADS), smem, st, a);
}

static size_t qtc_partials(const Q4Plan& p, int chunks) {
  return p.splits > 1 ? (size_t)chunks * p.tiles * 2 * p.splits * 1024 * sizeof(float) : 0;
}

size_t qtc_workspace_bytes(const Q4Plan& p, int64_t M, int64_t K) {
  const int chunks = (int)((M + QT_ROWS - 1) / QT_ROWS);
  const size_t G = (size_t)(K / 64);
  const size_t part = (qtc_partials(p, chunks) + 1023) / 1024 * 1024;
  return part + (size_t)chunks * G * (QT_B + QT_SX);
}

int qtc_launch(const Q4Plan& p, const Q4Args& a4, int epilogue, void* workspace, cudaStream_t st) {
  const int chunks = (a4.M + QT_ROWS - 1) / QT_ROWS;
  const int G = a4.K / 64;
  IM_REQUIRE((size_t)chunks * p.tiles * 2 < Q4_COUNTER_BYTES / 4, IM_UNSUPPORTED,
             "im_qgemm_packed: N too large at %d rows", a4.M);
  const int gmax = (G + p.splits - 1) / p.splits;
  IM_REQUIRE(gmax <= Q4_RMAX, IM_UNSUPPORTED, "im_qgemm_packed: %d groups per split", gmax);
  char* ws = reinterpret_cast<char*>(workspace);
  const size_t part = (qtc_partials(p, chunks) + 1023) / 1024 * 1024;
  unsigned char* xt = reinterpret_cast<unsigned char*>(ws + Q4_COUNTER_BYTES + part);
  float* sxt = reinterpret_cast<float*>(xt + (size_t)chunks * G * QT_B);
  int rc = launch("qtc_prep_kernel", qtc_prep_kernel, dim3((unsigned)G, (unsigned)chunks), dim3(256), 0, st, a4.x,
                  a4.M, a4.K, a4.norm_sq, a4.norm_parts, a4.sq_ld, a4.norm_w, a4.eps, a4.gemma_norm, xt, sxt);
  if (rc) return rc;
  QtArgs a;
  a.wp = a4.wp;
  a.xt = xt;
  a.sxt = sxt;
  a.y = a4.y;
  a.res = a4.res;
  a.out_sq = a4.out_sq;
  a.partial = reinterpret_cast<float*>(ws + Q4_COUNTER_BYTES);
  a.counters = reinterpret_cast<unsigned*>(ws);
  a.error = reinterpret_cast<unsigned*>(ws + Q4_COUNTER_BYTES - 4);
  a.M = a4.M;
  a.N = a4.N;
  a.K = a4.K;
  a.tiles = p.tiles;
  a.splits = p.splits;
  a.sq_ld = a4.sq_ld;
  a.gmax = gmax;
  switch (epilogue) {
    case IM_EPI_STORE: return qtc_launch_gemm<IM_EPI_STORE>(a, p, chunks, st);
    case IM_EPI_RESIDUAL: return qtc_launch_gemm<IM_EPI_RESIDUAL>(a, p, chunks, st);
    case IM_EPI_SWIGLU: return qtc_launch_gemm<IM_EPI_SWIGLU>(a, p, chunks, st);
    default: return qtc_launch_gemm<IM_EPI_GEGLU>(a, p, chunks, st);
  }
}

}  // namespace im
