// qGEMM v8: the packed 4-bit GEMM for more than 32 activation rows on the 5th-generation tensor cores
// (tcgen05.mma, accumulators in tensor memory): persistent and warp-specialised.
//
// The arithmetic is the warp-MMA kernel's (qgemm_packed.cu), bit for bit, as if the rows were computed in calls
// of at most 32 rows: per (weight row, activation row, 64-wide group) the exact bf16 codes 128+q times the
// activations summed on the tensor pipe in four K=16 steps whose k-sets and column order are those of the
// warp-MMA fragments (a tcgen05 K=16 step over a 16-column slice returns the same fp32 bits as the m16n8k16 warp
// MMA over it), the fp32 group affine tot = fmaf(b - 128 s, sum(x), fmaf(s, acc, tot)) in group order, the same
// RMSNorm prologue and group sums, the same K splits summed in split order, the same epilogues.
//
// qtc_prep_kernel (grid: groups x chunks) applies the optional RMSNorm, computes the per-group activation sums
// in the warp-MMA kernel's order and writes each (chunk, group) as a tensor-core tile: the chunk's rows of 128
// bytes, K-major, 128-byte swizzled (16-byte column c of row r at c ^ r%8), columns permuted to the fragment
// k-sets, rows past M zero; plus the group sums.
//
// qtc_kernel: items (4 tiles = 128 weight rows, one K range of the split plan, one chunk of <= 128 rows); a
// persistent grid (one CTA per SM) walks items blockIdx.x, + gridDim.x, ... Its warps run concurrently, coupled
// only by mbarriers:
//  * warp 0, the producer: per group, the four 1152-byte weight units and the activation tile into a load stage
//    (cp.async.bulk, one mbarrier per stage), and the group sums into a ring of their own. Weights depend on no
//    earlier kernel: the first stages' weight copies are issued before the programmatic-dependency wait;
//  * warps 2-3, the transform warps: tiles 2 (w-2) and 2 (w-2) + 1's codes -> bf16 128+q in the A ring (128 x 64,
//    K-major, swizzled);
//  * warp 1, the MMA warp: 4 MMAs (M = 128, N = the chunk's rows rounded up to 16, K = 16) per group into one of
//    four tensor-memory accumulators, committed to the A, load-stage and accumulator barriers;
//  * warps 4-19, the epilogue warps (lane quadrant = tile w%4, columns [32 ((w-4)/4), +32)): per group the accumulator and
//    group sums into 32 fp32 totals per thread; at an item's last group the split-K partials (the last split to
//    arrive sums them in split order) and the epilogue (store / residual (+ sums of squares) / SwiGLU / GeGLU) in
//    the warp-MMA kernel's order.
// Every mbarrier wait is bounded (1 s). A wait that runs out sets the error word (the last word of the counter
// region, read by im_qgemm_packed_status) and the CTA's abort flag, which every later wait honours; the CTA
// then waits (bounded) for its own bulk copies and MMAs in flight before it frees its tensor memory and exits.
#include "common.cuh"
#include "qgemm_packed.cuh"
#include "../../include/imspec.h"

namespace im {

constexpr int QT_WBYTES = 4 * Q4_UNIT;  // one group of an item's 4 tiles
constexpr int QT_A = 128 * 128;         // bf16 codes of 128 rows x 64
constexpr int QT_N = 128;               // activation rows per chunk at most (MMA N)
constexpr int QT_B = QT_N * 128;        // one activation tile
constexpr int QT_LS = 4;                // load stages (weights + activation tile)
constexpr int QT_AS = 3;                // A stages
constexpr int QT_TB = 4;                // tensor-memory accumulators
constexpr int QT_SR = 16;               // group-sum ring entries
constexpr int QT_CW = 32;               // accumulator columns per epilogue warp
constexpr int QT_PARTS = QT_N / QT_CW;  // epilogue warps per tile (column parts of an accumulator)
constexpr int QT_TRANSFORM = 2, QT_EPI = 4 * QT_PARTS;
constexpr int QT_W_TRANSFORM = 2, QT_W_EPI = 2 + QT_TRANSFORM;
constexpr int QT_THREADS = (2 + QT_TRANSFORM + QT_EPI) * 32;
constexpr uint32_t QT_TMEM_COLS = QT_TB * QT_N;
constexpr int QT_BARS = 2 * QT_LS + 2 * QT_AS + 2 * QT_TB + 2 * QT_SR;
constexpr size_t QT_OFF_A = (size_t)QT_LS * QT_B;
constexpr size_t QT_OFF_W = QT_OFF_A + (size_t)QT_AS * QT_A;
constexpr size_t QT_OFF_SX = QT_OFF_W + (size_t)QT_LS * QT_WBYTES;
constexpr int QT_SBB = 4 * 128;           // a group's scales and biases of the item's 4 tiles
constexpr size_t QT_OFF_SB = QT_OFF_SX + (size_t)QT_SR * QT_N * 4;
constexpr size_t QT_OFF_BAR = QT_OFF_SB + (size_t)QT_SR * QT_SBB;
constexpr size_t QT_SMEM = 1024 + QT_OFF_BAR + (size_t)QT_BARS * 8 + 16;
constexpr unsigned long long QT_WAIT_NS = 1000000000ull;
constexpr uint32_t QT_128 = 0x43004300u;

struct QtArgs {
  const unsigned char* wp;
  const unsigned char* xt;  // [chunks][G] activation tiles (QT_B bytes each)
  const float* sxt;         // [chunks][G][QT_N] group sums
  uint16_t* y;
  const uint16_t* res;
  float* out_sq;
  float* partial;
  unsigned* counters;
  unsigned* error;
  int M, N, K, tiles, ctas_x, splits, sq_ld;
  int nmma;   // MMA N: rows per chunk, a multiple of 16
  int items;  // ctas_x * splits * chunks
};

// An item and the position of a group in the CTA's sequence of groups.
struct QtCursor {
  int item, gl, ng, cg0, x, split, chunk;
};

__device__ __forceinline__ void qt_item(const QtArgs& a, int item, QtCursor& c) {
  c.item = item;
  c.gl = 0;
  c.x = item % a.ctas_x;
  const int rest = item / a.ctas_x;
  c.split = rest % a.splits;
  c.chunk = rest / a.splits;
  const int G = a.K >> 6;
  c.cg0 = (int)(((long long)G * c.split) / a.splits);
  c.ng = (int)(((long long)G * (c.split + 1)) / a.splits) - c.cg0;
}

__device__ __forceinline__ bool qt_next(const QtArgs& a, QtCursor& c) {
  if (++c.gl < c.ng) return true;
  const int nxt = c.item + (int)gridDim.x;
  if (nxt >= a.items) return false;
  qt_item(a, nxt, c);
  return true;
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

// The same with a suspend-time hint: the thread sleeps (up to 20 us) instead of spinning until the phase completes.
__device__ __forceinline__ bool qt_try_wait_sleep(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(bar), "r"(parity), "r"(20000u)
      : "memory");
  return done != 0;
}

// d = a * b + d on two fp32 lanes at once, each rounded once to nearest (the same bits as two fmaf).
__device__ __forceinline__ void qt_fma2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rd, {%0, %1};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rd;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
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
    if (qt_try_wait_sleep(b, parity)) return true;
    if (*abort_flag) return false;
    if (qt_clock() - t0 > QT_WAIT_NS) {
      *abort_flag = 1;
      atomicExch(error, 1u);
      return false;
    }
  }
}

// Bounded wait that ignores the abort flag (draining copies and MMAs already in flight).
__device__ __forceinline__ void qt_drain(unsigned long long* bar, uint32_t parity) {
  const uint32_t b = qt_smem(bar);
  const unsigned long long t0 = qt_clock();
  while (!qt_try_wait(b, parity) && qt_clock() - t0 < QT_WAIT_NS) {
  }
}

__device__ __forceinline__ void qt_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(qt_smem(bar)) : "memory");
}

__device__ __forceinline__ void qt_init(unsigned long long* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(qt_smem(bar)), "r"(count));
}

__device__ __forceinline__ uint64_t qt_desc(uint32_t saddr) {
  // K-major, 128-byte swizzle: 8-row groups 1024 bytes apart (SBO), leading offset 1 (unused), version 1
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// instruction descriptor: f32 accumulate, bf16 A and B, both K-major, N = n, M = 128
__device__ __forceinline__ uint32_t qt_idesc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((128u >> 4) << 24);
}

__device__ __forceinline__ void qt_codes(uint32_t u, uint32_t* p) {
  p[0] = (u & 0x000F000Fu) | QT_128;
  p[1] = ((u >> 4) & 0x000F000Fu) | QT_128;
  p[2] = ((u >> 8) & 0x000F000Fu) | QT_128;
  p[3] = ((u >> 12) & 0x000F000Fu) | QT_128;
}

// Byte offset of the 4-byte pair at (row r, column pair t of 16-byte chunk c) in a 128-byte-swizzled tile.
__device__ __forceinline__ uint32_t qt_sw(int r, int c, int t) {
  return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4) + 4 * t);
}


// ---- prologue: activation tiles -------------------------------------------------------------------------
// grid (G, chunks), 4 nmma threads = nmma rows x 4 quarters of a group; the warp-MMA kernel's prologue arithmetic.
__global__ void __launch_bounds__(4 * QT_N)
qtc_prep_kernel(const uint16_t* __restrict__ x, int M, int K, int nmma, const float* __restrict__ norm_sq,
                int norm_parts, int sq_ld, const uint16_t* __restrict__ norm_w, float eps, int gemma_norm,
                unsigned char* __restrict__ xt, float* __restrict__ sxt) {
  pdl_wait();
  pdl_trigger();
  const int grp = blockIdx.x, chunk = blockIdx.y, G = K >> 6;
  const int m = threadIdx.x >> 2, tq = threadIdx.x & 3;
  const int row = chunk * nmma + m;
  uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
  float part = 0.f;
  if (row < M && m < nmma) {
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
  // fragment pairs (k, k+4) in the order of the warp-MMA kernel's B fragments: pair i belongs to K=16 step i/2,
  // 16-byte chunk i of the row, column pair tq
  const uint32_t w[8] = {__byte_perm(lo.x, lo.z, 0x5410), __byte_perm(lo.x, lo.z, 0x7632),
                         __byte_perm(lo.y, lo.w, 0x5410), __byte_perm(lo.y, lo.w, 0x7632),
                         __byte_perm(hi.x, hi.z, 0x5410), __byte_perm(hi.x, hi.z, 0x7632),
                         __byte_perm(hi.y, hi.w, 0x5410), __byte_perm(hi.y, hi.w, 0x7632)};
  unsigned char* tile = xt + ((size_t)chunk * G + grp) * QT_B;
#pragma unroll
  for (int i = 0; i < 8; i++) *reinterpret_cast<uint32_t*>(tile + qt_sw(m, i, tq)) = w[i];
  part += __shfl_xor_sync(0xffffffffu, part, 1);
  part += __shfl_xor_sync(0xffffffffu, part, 2);
  if (tq == 0) sxt[((size_t)chunk * G + grp) * QT_N + m] = part;
}

// ---- the GEMM -------------------------------------------------------------------------------------------
template <int EPI>
__global__ void __launch_bounds__(QT_THREADS, 1)
qtc_kernel(QtArgs a) {
  extern __shared__ unsigned char qt_raw[];
  const uint32_t raw = qt_smem(qt_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  unsigned char* sbase = qt_raw + (base - raw);
  unsigned long long* bars = reinterpret_cast<unsigned long long*>(sbase + QT_OFF_BAR);
  unsigned long long* ld_full = bars;
  unsigned long long* ld_empty = ld_full + QT_LS;
  unsigned long long* a_full = ld_empty + QT_LS;
  unsigned long long* a_empty = a_full + QT_AS;
  unsigned long long* t_full = a_empty + QT_AS;
  unsigned long long* t_empty = t_full + QT_TB;
  unsigned long long* sx_full = t_empty + QT_TB;
  unsigned long long* sx_empty = sx_full + QT_SR;
  uint32_t* holder = reinterpret_cast<uint32_t*>(bars + QT_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(holder + 1);
  const float* sx_ring = reinterpret_cast<const float*>(sbase + QT_OFF_SX);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = a.K >> 6;

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(qt_smem(holder)),
                 "r"(QT_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < QT_LS; s++) {
      qt_init(&ld_full[s], 1u);
      qt_init(&ld_empty[s], (uint32_t)QT_TRANSFORM + 1u);
    }
    for (int s = 0; s < QT_AS; s++) {
      qt_init(&a_full[s], (uint32_t)QT_TRANSFORM);
      qt_init(&a_empty[s], 1u);
    }
    for (int b = 0; b < QT_TB; b++) {
      qt_init(&t_full[b], 1u);
      qt_init(&t_empty[b], (uint32_t)QT_EPI);
    }
    for (int r = 0; r < QT_SR; r++) {
      qt_init(&sx_full[r], 1u);
      qt_init(&sx_empty[r], (uint32_t)QT_EPI);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *holder;

  if (warp == 0) {
    // ---- producer ----------------------------------------------------------------------------------------
    if (lane == 0) {
      const uint32_t bbytes = (uint32_t)a.nmma * 128u, sbytes = (uint32_t)a.nmma * 4u;
      auto copy = [&](uint32_t dst, const void* src, uint32_t bytes, unsigned long long* bar) {
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         dst),
                     "l"(src), "r"(bytes), "r"(qt_smem(bar))
                     : "memory");
      };
      auto weights = [&](int ls, const QtCursor& c) {
        const uint32_t dst = base + (uint32_t)(QT_OFF_W + (size_t)ls * QT_WBYTES);
#pragma unroll
        for (int t = 0; t < 4; t++) {
          const int tile = min(4 * c.x + t, a.tiles - 1);  // a missing tile copies a real one (never used)
          copy(dst + (uint32_t)(t * Q4_UNIT), a.wp + ((size_t)tile * G + c.cg0 + c.gl) * Q4_UNIT, (uint32_t)Q4_UNIT,
               &ld_full[ls]);
        }
      };
      auto expect = [&](unsigned long long* bar, uint32_t bytes) {
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(qt_smem(bar)), "r"(bytes)
                     : "memory");
      };
      QtCursor c;
      qt_item(a, blockIdx.x, c);
      // the first stages' weights before the dependency wait
      int pre = 0;
      {
        QtCursor cw = c;
        bool more = true;
        for (; pre < QT_LS && more; pre++) {
          expect(&ld_full[pre], (uint32_t)QT_WBYTES + bbytes);
          weights(pre, cw);
          more = qt_next(a, cw);
        }
      }
      pdl_wait();
      int k = 0;
      for (;; k++) {
        const int ls = k % QT_LS, r = k % QT_SR;
        if (k >= pre) {
          if (!qt_wait(&ld_empty[ls], (uint32_t)(((k / QT_LS) - 1) & 1), abort_flag, a.error)) break;
          expect(&ld_full[ls], (uint32_t)QT_WBYTES + bbytes);
          weights(ls, c);
        }
        const size_t t = (size_t)c.chunk * G + c.cg0 + c.gl;
        copy(base + (uint32_t)(ls * QT_B), a.xt + t * QT_B, bbytes, &ld_full[ls]);
        if (k >= QT_SR && !qt_wait(&sx_empty[r], (uint32_t)(((k / QT_SR) - 1) & 1), abort_flag, a.error)) {
          k++;
          break;
        }
        expect(&sx_full[r], sbytes + (uint32_t)QT_SBB);
        copy(base + (uint32_t)(QT_OFF_SX + (size_t)r * QT_N * 4), a.sxt + t * QT_N, sbytes, &sx_full[r]);
#pragma unroll
        for (int tt = 0; tt < 4; tt++) {  // the group's scales and biases (bytes 1024.. of each tile's unit)
          const int tile = min(4 * c.x + tt, a.tiles - 1);
          copy(base + (uint32_t)(QT_OFF_SB + (size_t)r * QT_SBB + tt * 128),
               a.wp + ((size_t)tile * G + c.cg0 + c.gl) * Q4_UNIT + 1024, 128u, &sx_full[r]);
        }
        if (!qt_next(a, c)) {
          k++;
          break;
        }
      }
      if (*abort_flag) {  // copies still landing in this CTA's shared memory finish before it exits
        const int kk = k > pre ? k : pre;
        for (int j = (kk > QT_LS ? kk - QT_LS : 0); j < kk; j++) qt_drain(&ld_full[j % QT_LS], (uint32_t)((j / QT_LS) & 1));
        for (int j = (k > QT_SR ? k - QT_SR : 0); j < k; j++) qt_drain(&sx_full[j % QT_SR], (uint32_t)((j / QT_SR) & 1));
      }
    }
    __syncwarp();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    return;
  }

  if (warp == 1) {
    // ---- MMA issue ------------------------------------------------------------------------------------
    if (lane == 0) {
      QtCursor c;
      qt_item(a, blockIdx.x, c);
      const uint32_t idesc = qt_idesc(a.nmma);
      int issued = -1;
      for (int k = 0;; k++) {
        const int ls = k % QT_LS, as = k % QT_AS, tb = k % QT_TB;
        if (!qt_wait(&a_full[as], (uint32_t)((k / QT_AS) & 1), abort_flag, a.error)) break;
        if (!qt_wait(&ld_full[ls], (uint32_t)((k / QT_LS) & 1), abort_flag, a.error)) break;
        if (k >= QT_TB && !qt_wait(&t_empty[tb], (uint32_t)(((k / QT_TB) - 1) & 1), abort_flag, a.error)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + (uint32_t)(tb * QT_N);
        const uint32_t sa = base + (uint32_t)(QT_OFF_A + (size_t)as * QT_A), sb = base + (uint32_t)(ls * QT_B);
#pragma unroll
        for (int k4 = 0; k4 < 4; k4++) {
          const uint64_t ad = qt_desc(sa + (uint32_t)(32 * k4));
          const uint64_t bd = qt_desc(sb + (uint32_t)(32 * k4));
          asm volatile(
              "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
              "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
              "l"(ad), "l"(bd), "r"(idesc), "r"((uint32_t)(k4 > 0)));
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         qt_smem(&a_empty[as]))
                     : "memory");
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         qt_smem(&ld_empty[ls]))
                     : "memory");
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                         qt_smem(&t_full[tb]))
                     : "memory");
        issued = k;
        if (!qt_next(a, c)) break;
      }
      if (*abort_flag && issued >= 0) qt_drain(&t_full[issued % QT_TB], (uint32_t)((issued / QT_TB) & 1));
    }
    __syncwarp();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(QT_TMEM_COLS));
    return;
  }

  const int g8 = lane >> 2, t4 = lane & 3;
  if (warp < QT_W_EPI) {
    // ---- transform: tile (warp - 2)'s codes -> bf16 128+q in the A ring ----------------------------------
    const int t0 = 2 * (warp - QT_W_TRANSFORM);  // tiles t0 and t0 + 1
    // byte offset in an A stage of (tile t0, row slot 0, 16-byte chunk c, this lane's column pair)
    uint32_t xo[8];
#pragma unroll
    for (int c = 0; c < 8; c++) xo[c] = (uint32_t)(t0 * 4096 + g8 * 128 + ((c ^ g8) << 4) + 4 * t4);
    QtCursor c;
    qt_item(a, blockIdx.x, c);
    for (int k = 0;; k++) {
      const int ls = k % QT_LS, as = k % QT_AS;
      if (!qt_wait(&ld_full[ls], (uint32_t)((k / QT_LS) & 1), abort_flag, a.error)) break;
      if (k >= QT_AS && !qt_wait(&a_empty[as], (uint32_t)(((k / QT_AS) - 1) & 1), abort_flag, a.error)) break;
      unsigned char* st = sbase + QT_OFF_A + (size_t)as * QT_A;
#pragma unroll
      for (int tt = 0; tt < 2; tt++) {
        const unsigned char* wsrc = sbase + QT_OFF_W + (size_t)ls * QT_WBYTES + (t0 + tt) * Q4_UNIT + lane * 32;
        const uint4 c0 = *reinterpret_cast<const uint4*>(wsrc), c1 = *reinterpret_cast<const uint4*>(wsrc + 16);
        const uint32_t words[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
        for (int wd = 0; wd < 8; wd++) {  // row g + 8 (wd / 2) of the tile, word 2t + wd % 2 of the group
          const int j = wd >> 1, hw = wd & 1;
          uint32_t p[4];
          qt_codes(words[wd], p);
          // nibbles (n, n + 4) of word half hw belong to K=16 step 2 hw + n / 2, 16-byte chunk 4 hw + n
#pragma unroll
          for (int n = 0; n < 4; n++)
            *reinterpret_cast<uint32_t*>(st + tt * 4096 + j * 1024 + xo[4 * hw + n]) = p[n];
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        qt_arrive(&a_full[as]);
        qt_arrive(&ld_empty[ls]);
      }
      if (!qt_next(a, c)) break;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    return;
  }

  // ---- epilogue warps ------------------------------------------------------------------------------------
  // a warp reads tensor-memory lanes [32 (warp % 4), +32) only: quadrant = tile = warp % 4
  const int q = warp & 3, part = (warp - QT_W_EPI) >> 2;
  const int col0 = QT_CW * part;
  const int ncols = max(0, min(QT_CW, a.nmma - col0));  // accumulator columns of this warp holding chunk rows
  pdl_wait();
  pdl_trigger();
  // this thread's row (tile row `lane`) in a group's scale/bias block: scales of rows g, g+8, 16+g, 24+g, then
  // their biases, 16 bytes per g
  const uint32_t sb_off = (uint32_t)(q * 128 + (lane & 7) * 16 + (lane >> 3) * 2);
  float tot[QT_CW];
#pragma unroll
  for (int j = 0; j < QT_CW; j++) tot[j] = 0.f;
  QtCursor ce, cn;
  qt_item(a, blockIdx.x, ce);
  cn = ce;
  bool has_next = qt_next(a, cn);
  for (int k = 0;; k++) {
    const int tb = k % QT_TB, r = k % QT_SR;
    if (!qt_wait(&t_full[tb], (uint32_t)((k / QT_TB) & 1), abort_flag, a.error)) break;
    if (!qt_wait(&sx_full[r], (uint32_t)((k / QT_SR) & 1), abort_flag, a.error)) break;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned char* sbp = sbase + QT_OFF_SB + (size_t)r * QT_SBB + sb_off;
    const float s0 = bf(*reinterpret_cast<const uint16_t*>(sbp));
    const float b0 = fmaf(-128.f, s0, bf(*reinterpret_cast<const uint16_t*>(sbp + 8)));
    // the warp's accumulator columns, every load in flight before one wait
    uint32_t acc[QT_CW];
#pragma unroll
    for (int h = 0; h < QT_CW / 16; h++) {
      const uint32_t ta = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(tb * QT_N + col0 + 16 * h);
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(acc[16 * h + 0]), "=r"(acc[16 * h + 1]), "=r"(acc[16 * h + 2]), "=r"(acc[16 * h + 3]),
            "=r"(acc[16 * h + 4]), "=r"(acc[16 * h + 5]), "=r"(acc[16 * h + 6]), "=r"(acc[16 * h + 7]),
            "=r"(acc[16 * h + 8]), "=r"(acc[16 * h + 9]), "=r"(acc[16 * h + 10]), "=r"(acc[16 * h + 11]),
            "=r"(acc[16 * h + 12]), "=r"(acc[16 * h + 13]), "=r"(acc[16 * h + 14]), "=r"(acc[16 * h + 15])
          : "r"(ta));
    }
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int h = 0; h < QT_CW / 16; h++) {
      if (16 * h < ncols) {
        const float4* sx4 = reinterpret_cast<const float4*>(sx_ring + (size_t)r * QT_N + col0 + 16 * h);
#pragma unroll
        for (int j4 = 0; j4 < 4; j4++) {
          const float4 sx = sx4[j4];
          float* tt = tot + 16 * h + 4 * j4;
          const uint32_t* ac = acc + 16 * h + 4 * j4;
          // tot = fmaf(b', sx, fmaf(s, acc, tot)), two columns per instruction
          qt_fma2(tt[0], tt[1], s0, s0, __uint_as_float(ac[0]), __uint_as_float(ac[1]));
          qt_fma2(tt[2], tt[3], s0, s0, __uint_as_float(ac[2]), __uint_as_float(ac[3]));
          qt_fma2(tt[0], tt[1], b0, b0, sx.x, sx.y);
          qt_fma2(tt[2], tt[3], b0, b0, sx.z, sx.w);
        }
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
      qt_arrive(&t_empty[tb]);
      qt_arrive(&sx_empty[r]);
    }

    if (ce.gl == ce.ng - 1) {
      // ---- the item's last group: split-K, then the epilogue
      const int tile = 4 * ce.x + q;
      if (tile < a.tiles && ncols > 0) {
        bool last = true;
        if (a.splits > 1) {
          const size_t slot = ((size_t)ce.chunk * a.tiles + tile) * QT_PARTS + part;
          float* mine = a.partial + (slot * a.splits + ce.split) * (QT_CW * 32);
#pragma unroll
          for (int j = 0; j < QT_CW; j++) __stcg(mine + j * 32 + lane, tot[j]);
          __threadfence();
          __syncwarp();
          unsigned prev = 0;
          if (lane == 0) prev = atomicAdd(a.counters + slot, 1u);
          prev = __shfl_sync(0xffffffffu, prev, 0);
          last = prev == (unsigned)(a.splits - 1);
          if (last) {
            __threadfence();
#pragma unroll
            for (int j = 0; j < QT_CW; j++) tot[j] = 0.f;
            for (int sp = 0; sp < a.splits; sp++) {
              const float* src = a.partial + (slot * a.splits + sp) * (QT_CW * 32);
#pragma unroll
              for (int j = 0; j < QT_CW; j++) tot[j] += __ldcg(src + j * 32 + lane);
            }
            if (lane == 0) a.counters[slot] = 0u;
          }
        }
        if (last) {
          const int rbase = tile * 32;
          const int m0 = ce.chunk * a.nmma + col0;  // this warp's first activation row
          const int mrows = min(a.nmma, a.M - ce.chunk * a.nmma);
          if constexpr (EPI == IM_EPI_SWIGLU || EPI == IM_EPI_GEGLU) {
            const int nout = a.N >> 1;
            const int f = (rbase >> 1) + lane;  // tile rows 0-15 gate features, 16-31 the matching up features
#pragma unroll
            for (int j = 0; j < QT_CW; j++) {
              const float up_v = __shfl_down_sync(0xffffffffu, tot[j], 16);
              if (lane < 16 && col0 + j < mrows && f < nout) {
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
            const int row = rbase + lane;
#pragma unroll
            for (int j = 0; j < QT_CW; j++) {
              const bool valid = col0 + j < mrows && row < a.N;
              float hv = 0.f;
              if (valid) {
                const size_t o = (size_t)(m0 + j) * a.N + row;
                const uint16_t hq =
                    EPI == IM_EPI_RESIDUAL ? to_bf(bf(a.res[o]) + round_bf(tot[j])) : to_bf(tot[j]);
                a.y[o] = hq;
                hv = bf(hq);
              }
              if (a.out_sq) {
                // the warp-MMA kernel's order: rows g, g + 8, g + 16, g + 24 chained per g, then over g
                const float x8 = __shfl_sync(0xffffffffu, hv, (lane + 8) & 31);
                const float x16 = __shfl_sync(0xffffffffu, hv, (lane + 16) & 31);
                const float x24 = __shfl_sync(0xffffffffu, hv, (lane + 24) & 31);
                float v = fmaf(x24, x24, fmaf(x16, x16, fmaf(x8, x8, fmaf(hv, hv, 0.f))));
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                v += __shfl_xor_sync(0xffffffffu, v, 4);
                if (lane == 0 && col0 + j < mrows) a.out_sq[(size_t)tile * a.sq_ld + m0 + j] = v;
              }
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < QT_CW; j++) tot[j] = 0.f;
    }
    if (!has_next) break;
    ce = cn;
    has_next = qt_next(a, cn);
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();  // every MMA of this CTA has completed (or been drained): the MMA warp frees tensor memory
}

static int g_qt_sms = 0;

template <int EPI>
static int qtc_launch_gemm(const QtArgs& a, cudaStream_t st) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(qtc_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)QT_SMEM);
    int dev = 0;
    if (e == cudaSuccess) e = cudaGetDevice(&dev);
    if (e == cudaSuccess && g_qt_sms == 0) e = cudaDeviceGetAttribute(&g_qt_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
      set_error("qGEMM (tensor cores): cannot configure the kernel: %s", cudaGetErrorString(e));
      return IM_CUDA_ERROR;
    }
    configured = true;
  }
  const int grid = min(a.items, g_qt_sms);  // one CTA per SM: its tensor memory is the SM's 512 columns
  return launch("qtc_kernel", qtc_kernel<EPI>, dim3((unsigned)grid), dim3(QT_THREADS), QT_SMEM, st, a);
}

// chunks of at most 128 rows, as even as multiples of 16 allow
static void qtc_shape(int64_t M, int* chunks, int* nmma) {
  *chunks = (int)((M + QT_N - 1) / QT_N);
  const int per = (int)((M + *chunks - 1) / *chunks);
  *nmma = (per + 15) / 16 * 16;
}

static size_t qtc_partials(const Q4Plan& p, int chunks) {
  return p.splits > 1 ? (size_t)chunks * p.tiles * QT_PARTS * p.splits * QT_CW * 32 * sizeof(float) : 0;
}

size_t qtc_workspace_bytes(const Q4Plan& p, int64_t M, int64_t K) {
  int chunks, nmma;
  qtc_shape(M, &chunks, &nmma);
  const size_t G = (size_t)(K / 64);
  const size_t part = (qtc_partials(p, chunks) + 1023) / 1024 * 1024;
  return part + (size_t)chunks * G * (QT_B + QT_N * 4);
}

int qtc_launch(const Q4Plan& p, const Q4Args& a4, int epilogue, void* workspace, cudaStream_t st) {
  int chunks, nmma;
  qtc_shape(a4.M, &chunks, &nmma);
  const int G = a4.K / 64;
  IM_REQUIRE((size_t)chunks * p.tiles * QT_PARTS < Q4_COUNTER_BYTES / 4 - 1, IM_UNSUPPORTED,
             "im_qgemm_packed: N too large at %d rows", a4.M);
  IM_REQUIRE(workspace, IM_INVALID, "im_qgemm_packed: the tensor-core path needs the workspace");
  char* ws = reinterpret_cast<char*>(workspace);
  const size_t part = (qtc_partials(p, chunks) + 1023) / 1024 * 1024;
  unsigned char* xt = reinterpret_cast<unsigned char*>(ws + Q4_COUNTER_BYTES + part);
  float* sxt = reinterpret_cast<float*>(xt + (size_t)chunks * G * QT_B);
  int rc = launch("qtc_prep_kernel", qtc_prep_kernel, dim3((unsigned)G, (unsigned)chunks), dim3(4 * QT_N), 0, st,
                  a4.x, a4.M, a4.K, nmma, a4.norm_sq, a4.norm_parts, a4.sq_ld, a4.norm_w, a4.eps, a4.gemma_norm, xt,
                  sxt);
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
  a.ctas_x = p.ctas_x;
  a.splits = p.splits;
  a.sq_ld = a4.sq_ld;
  a.nmma = nmma;
  a.items = p.ctas_x * p.splits * chunks;
  switch (epilogue) {
    case IM_EPI_STORE: return qtc_launch_gemm<IM_EPI_STORE>(a, st);
    case IM_EPI_RESIDUAL: return qtc_launch_gemm<IM_EPI_RESIDUAL>(a, st);
    case IM_EPI_SWIGLU: return qtc_launch_gemm<IM_EPI_SWIGLU>(a, st);
    default: return qtc_launch_gemm<IM_EPI_GEGLU>(a, st);
  }
}

}  // namespace im
