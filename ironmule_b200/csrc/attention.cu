// Paged verification attention for speculative decoding: every query row of a sequence attends to that
// sequence's KV pages under a causal limit, an optional sliding window and an optional tree mask.
//
// Replaces the reference's decode/verify attention: FA2 over a slot pool with per-row lengths
// (IronMule ironmule/dense_plan.py:111-195 partial, :258-274 combine -- the per-row length
// `positions + 1` of :345 is the causal verify mask) and its Gemma-3 form with head_dim 256 and a sliding
// window (ironmule/dense_gemma.py:47-300).
//
// Layout: K and V caches [pages][Hkv][16][D] bf16 (16-token pages); page_table [B][max_pages];
// q [M][Hq][D] with the rows of sequence b at [seq_rows[b], seq_rows[b+1]); row_slot[r] is the KV slot the
// row was written to (its causal limit). Tree mode: slots >= tree_base[b] are draft-tree nodes and row r sees
// node j only if bit j of tree_mask[r] is set.
//
// Two entry points share one kernel. im_attention_paged reads q and every key from memory.
// im_attention_qkv_paged starts from the packed qkv rows of the projection: each CTA applies the q RMSNorm
// + RoPE to its own query vectors and the k RMSNorm + RoPE to the new rows' keys of its split (the same
// arithmetic, in the same order, as im_qk_norm_rope_kv), uses them from shared memory, and one CTA per
// (row, kv head) writes them to the cache. Keys that no row of this launch writes are staged with cp.async
// before the kernel waits for the previous kernel, so their loads overlap it.
//
// Work split: grid (CTAs per group, kv heads, sequences x query blocks). A CTA owns up to NQ query vectors
// (rows x the kv head's query heads) and walks splits of `kpc` keys at fixed absolute positions (split x, x +
// gridDim.x, ...), each in 64-key blocks staged in shared memory with an online softmax started afresh per
// split. Every split publishes its (acc, max, sum) partial; the last CTA of a (sequence, kv head, query block)
// to finish merges the splits in split order. The host picks the CTAs per group from the occupancy and the
// number of groups (one CTA per split for a single sequence, several splits per CTA for large batches). A row's result depends
// only on its own query, its mask and the KV -- not on how many rows or sequences share the launch.
#include <climits>
#include <math.h>

#include "common.cuh"
#include "attention.cuh"

namespace im {

constexpr int AT_MAXNEW = 32;   // new (written by this launch) keys per split at most: rows per sequence <= 32
constexpr int AT_MW = 64;       // splits whose merge weights are kept in shared memory

struct AttnArgs {
  const uint16_t* q;          // plain mode: [M][Hq][D]
  const uint16_t* qkv;        // fused mode: [M][(Hq + 2 Hkv) D] packed q | k | v rows
  const uint16_t* q_norm;     // fused: [D]
  const uint16_t* k_norm;     // fused: [D]
  const float* inv_freq;      // fused: [D/2]
  const int* row_pos;         // fused: RoPE position per row
  uint16_t* kc;
  uint16_t* vc;
  const int* page_table;
  const int* seq_rows;
  const int* seq_slot;  // page-table row of each sequence group (NULL: group b uses row b)
  const int* row_slot;
  const unsigned long long* tree_mask;
  const int* tree_base;
  uint16_t* out;
  float* part;
  unsigned* counters;
  int max_pages, Hq, Hkv, kpc, nsplit, qblocks, window, gemma;
  int defer;  // publish the split partials only: the o-projection merges them (out is not written)
  float scale, eps;
};

template <int D, int NQ, bool FUSED, int NBUF>
struct AttnSmem {
  // new keys one CTA may hold: a query block of at most 8 vectors comes from at most 8 rows per sequence
  static constexpr int NEW = FUSED ? (NQ <= 8 ? 8 : AT_MAXNEW) : 1;
  static constexpr int QM = NQ < 16 ? 16 : NQ;  // rows of the m16 MMA tiles (rows >= nq stay zero)
  // key blocks staged at once: with two, a 128-key split is staged whole before the kernel waits for the previous
  // one and later blocks load while the block before them is computed (for launches of few groups, where the
  // second buffer costs no occupancy that matters)
  static constexpr int NB = NBUF;
  // Row strides are padded by 16 bytes so the MMA fragment loads (and ldmatrix rows) hit distinct banks.
  uint16_t qs[QM][D + 8];         // bf16 queries
  uint32_t ks[NB][AT_KB][D / 2 + 4];  // keys as bf16 pairs
  uint16_t vs[NB][AT_KB][D + 8];      // values
  float s[NQ][AT_KB + 4];         // scores; in the merge, the splits' sums
  uint16_t ph[QM][AT_KB + 8];     // probabilities split into bf16 high and low parts: p = ph + pl
  uint16_t pl[QM][AT_KB + 8];
  uint16_t nk[NEW][D];  // fused: keys (normed, roped) and values of the rows this launch writes in this split
  uint16_t nv[NEW][D];
  float m[NQ], l[NQ], alpha[QM];
  int row_slot[NQ];
  unsigned long long tmask[NQ];
  int new_row[NEW], new_slot[NEW];
  int nnew, kv_len;
  int page[NB][AT_KB / 16];  // pages of the blocks being staged
  int newidx[NB][AT_KB];  // per key of the blocks being staged: index into nk/nv, or -1
  float mw[NQ][AT_MW];  // merge: per (query vector, split) weights
  int last;
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const unsigned dst = (unsigned)__cvta_generic_to_shared(smem);
  const int n = valid ? 16 : 0;  // 0 source bytes: the 16 bytes are zero-filled
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Four 8x8 bf16 matrices from shared memory, transposed: rows given by lanes 0-7, 8-15, 16-23, 24-31.
__device__ __forceinline__ void ldsm_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  const unsigned addr = (unsigned)__cvta_generic_to_shared(p);
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// RMSNorm (weight w: w or 1 + w) + RoPE of one head vector by one warp; lane owns elements lane + 32 e.
// The sum of squares is the per-32-element xor-tree sums added in element order, and the RoPE pairs
// (i, i + D/2) sit in the same lane: the arithmetic of qk_rope_kv_kernel, value for value.
// wd[e] = the norm weight of element lane + 32 e (w or 1 + w), fq[e] = inv_freq[lane + 32 e]: loaded by the caller
// (before the kernel waits for the qkv projection: neither depends on it).
template <int D>
__device__ __forceinline__ void norm_rope_vals(const float (&v)[D / 32], const float (&wd)[D / 32], float eps, int pos,
                                               const float (&fq)[D / 64], uint16_t (&outv)[D / 32]) {
  constexpr int E = D / 32, H = E / 2;
  float total = 0.f;
#pragma unroll
  for (int e = 0; e < E; e++) total += warp_sum(v[e] * v[e]);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fdiv_rn(total, (float)D) + eps));
  float xn[E];
#pragma unroll
  for (int e = 0; e < E; e++) xn[e] = round_bf((v[e] * inv) * wd[e]);
#pragma unroll
  for (int e = 0; e < H; e++) {
    const float ang = (float)pos * fq[e];
    float sn, cs;
    sincosf(ang, &sn, &cs);
    const float x1 = xn[e], x2 = xn[e + H];
    outv[e] = to_bf(x1 * cs - x2 * sn);
    outv[e + H] = to_bf(x1 * sn + x2 * cs);
  }
}

template <int D, int NQ, bool FUSED, int W, int NB>
__global__ void __launch_bounds__(32 * W, W == 4 ? 4 : 2)
attn_kernel(AttnArgs a) {
  constexpr int TH = 32 * W;  // W warps
  extern __shared__ __align__(16) unsigned char smem_raw[];
  using Smem = AttnSmem<D, NQ, FUSED, NB>;
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  if constexpr (!FUSED) {
    pdl_wait();  // q and every key were written by earlier kernels
    pdl_trigger();
  }
  // Before the wait (fused mode) only data that the previous kernel (the qkv projection) does not write is
  // read: the row metadata, the page table and the keys of slots no row of this launch writes.
  // The CTA walks splits blockIdx.x, blockIdx.x + gridDim.x, ... of its (sequence, kv head, query block); each
  // split is computed and published exactly as if it had a CTA of its own.
  const int kvh = blockIdx.y;
  const int b = blockIdx.z / a.qblocks, qb = blockIdx.z % a.qblocks;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int G = a.Hq / a.Hkv;
  const int r0 = a.seq_rows[b], nr = a.seq_rows[b + 1] - r0;
  const int prow = a.seq_slot ? a.seq_slot[b] : b;
  const int q0 = qb * NQ;
  const int nq = max(0, min(NQ, nr * G - q0));
  const int stride_x = gridDim.x;

  const int tbase = a.tree_mask ? a.tree_base[b] : 0;
  // Row metadata with every load in flight at once: warp 0 reads the rows' slots (kv length = one past the
  // largest; the rows whose slot falls in one of this CTA's splits are this launch's new keys there), the
  // other threads the query vectors' limits and masks.
  if (warp == 0) {
    int mx = -1, n = 0;
    for (int r0l = 0; r0l < nr; r0l += 32) {
      const int r = r0l + lane;
      const int slot = r < nr ? a.row_slot[r0 + r] : -1;
      int m2 = slot;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m2 = max(m2, __shfl_xor_sync(0xffffffffu, m2, o));
      mx = max(mx, m2);
      if constexpr (FUSED) {
        const bool isnew = slot >= 0 && (slot / a.kpc) % stride_x == (int)blockIdx.x;
        const unsigned ball = __ballot_sync(0xffffffffu, isnew);
        const int idx = n + __popc(ball & ((1u << lane) - 1u));
        if (isnew && idx < Smem::NEW) {
          sm.new_row[idx] = r0 + r;
          sm.new_slot[idx] = slot;
        }
        n += __popc(ball);
      }
    }
    if (lane == 0) {
      sm.kv_len = mx + 1;
      sm.nnew = min(n, Smem::NEW);
    }
  }
  for (int i = tid; i < Smem::QM * (D + 8) / 2; i += TH) reinterpret_cast<uint32_t*>(&sm.qs[0][0])[i] = 0u;
  for (int i = tid; i < Smem::QM * (AT_KB + 8) / 2; i += TH) {
    reinterpret_cast<uint32_t*>(&sm.ph[0][0])[i] = 0u;
    reinterpret_cast<uint32_t*>(&sm.pl[0][0])[i] = 0u;
  }
  for (int i = tid; i < Smem::QM; i += TH) sm.alpha[i] = 0.f;
  for (int i = tid; i < NQ; i += TH) {
    sm.m[i] = -INFINITY;
    sm.l[i] = 0.f;
    if (i < nq) {
      const int row = r0 + (q0 + i) / G;
      sm.row_slot[i] = a.row_slot[row];
      sm.tmask[i] = a.tree_mask ? a.tree_mask[row] : 0ull;
    }
  }
  __syncthreads();
  const int kv_len = sm.kv_len;
  const bool any = nq > 0 && (int)blockIdx.x * a.kpc < kv_len;  // this CTA has at least one non-empty split
  // A CTA without a split leaves now, before the wait, and frees its slot for one that has work; the merge
  // counts only the CTAs of the group that have a split.
  if (!any) return;
  const int live_ctas = min(stride_x, (kv_len + a.kpc - 1) / a.kpc);
  // keys below min_vis are visible to every query vector of this CTA (no window; below the tree slots)
  int min_vis = 0;
  if (a.window <= 0 && nq > 0) {
    int lo = INT_MAX;
    for (int i = 0; i < nq; i++) lo = min(lo, sm.row_slot[i] + 1);
    if (a.tree_mask) lo = min(lo, tbase);
    min_vis = lo;
  }
  int k_begin = blockIdx.x * a.kpc;
  int k_end = min(kv_len, k_begin + a.kpc);

  // stage keys [kb0, kb0 + 64): K as bf16 pairs and V; slots written by this launch come from nk/nv later
  auto stage_old = [&](int kb0, int buf) {
    if (tid < AT_KB / 16) {
      const int slot = kb0 + tid * 16;
      sm.page[buf][tid] = slot < k_end ? a.page_table[(size_t)prow * a.max_pages + (slot >> 4)] : 0;
    }
    if constexpr (FUSED) {
      for (int j = tid; j < AT_KB; j += TH) {
        int idx = -1;
        for (int n = 0; n < sm.nnew; n++)
          if (sm.new_slot[n] == kb0 + j) idx = n;
        sm.newidx[buf][j] = idx;
      }
    }
    __syncthreads();
    constexpr int PER = AT_KB * (D / 8) / TH;
#pragma unroll
    for (int t = 0; t < PER; t++) {
      const int i = tid + t * TH;
      const int j = i / (D / 8), c = i % (D / 8);
      const int slot = kb0 + j;
      bool skip = false;
      if constexpr (FUSED) skip = sm.newidx[buf][j] >= 0;  // filled from nk/nv by plain stores: no async copy here
      if (!skip) {
        const bool load = slot < k_end;  // past the end: zero-filled
        const size_t off = load ? (((size_t)sm.page[buf][j >> 4] * a.Hkv + kvh) * 16 + (slot & 15)) * D + c * 8 : 0;
        cp_async16(&sm.ks[buf][j][c * 4], a.kc + off, load);
        cp_async16(&sm.vs[buf][j][c * 8], a.vc + off, load);
      }
    }
    cp_async_commit();
  };
  auto fill_new = [&](int buf) {
    if constexpr (FUSED) {
      for (int i = tid; i < AT_KB * (D / 8); i += TH) {
        const int j = i / (D / 8), c = i % (D / 8);
        const int idx = sm.newidx[buf][j];
        if (idx >= 0) {
          *reinterpret_cast<uint4*>(&sm.ks[buf][j][c * 4]) = *reinterpret_cast<const uint4*>(&sm.nk[idx][c * 8]);
          *reinterpret_cast<uint4*>(&sm.vs[buf][j][c * 8]) = *reinterpret_cast<const uint4*>(&sm.nv[idx][c * 8]);
        }
      }
    }
  };

  // the split's first block (and its second, with two buffers) before the wait: no earlier kernel writes them
  bool second = false;
  if (any) {
    stage_old(k_begin, 0);
    second = Smem::NB > 1 && k_begin + AT_KB < k_end;
    if (second) stage_old(k_begin + AT_KB, Smem::NB - 1);
  }

  if constexpr (FUSED) {
    // Before the wait: the norm weights, RoPE frequencies, positions and cache pages (no earlier kernel of the
    // layer writes them). After it, every element of this warp's query vectors and of its first new row is
    // loaded at once, then normed and roped.
    constexpr int E = D / 32, H = E / 2, VPW = NQ / (TH / 32);
    const int stride = (a.Hq + 2 * a.Hkv) * D;
    uint32_t qwp[H], kwp[H];  // the norm weights of elements lane + 32 e, two bf16 per word (e = 2i, 2i + 1)
    float fq[H];
    int qpos[VPW], kpos = 0, kpage = 0;
    const int n0 = warp;  // this warp's first new row (later ones, if any, go one at a time below)
    if (any) {
#pragma unroll
      for (int i = 0; i < H; i++) {
        qwp[i] = (uint32_t)a.q_norm[lane + 64 * i] | ((uint32_t)a.q_norm[lane + 64 * i + 32] << 16);
        kwp[i] = (uint32_t)a.k_norm[lane + 64 * i] | ((uint32_t)a.k_norm[lane + 64 * i + 32] << 16);
      }
#pragma unroll
      for (int e = 0; e < H; e++) fq[e] = a.inv_freq[lane + 32 * e];
#pragma unroll
      for (int t = 0; t < VPW; t++) {
        const int qi = warp + t * (TH / 32);
        qpos[t] = qi < nq ? a.row_pos[r0 + (q0 + qi) / G] : 0;
      }
      if (n0 < sm.nnew) {
        kpos = a.row_pos[sm.new_row[n0]];
        kpage = a.page_table[(size_t)prow * a.max_pages + (sm.new_slot[n0] >> 4)];
      }
    }
    pdl_wait();
    pdl_trigger();
    if (any) {
      float qw[E], kw[E];
#pragma unroll
      for (int e = 0; e < E; e++) {
        const float q1 = (e & 1) ? bf_hi(qwp[e >> 1]) : bf_lo(qwp[e >> 1]);
        const float k1 = (e & 1) ? bf_hi(kwp[e >> 1]) : bf_lo(kwp[e >> 1]);
        qw[e] = a.gemma ? 1.0f + q1 : q1;
        kw[e] = a.gemma ? 1.0f + k1 : k1;
      }
      float v[VPW][E], kv[E];
      uint16_t vv[E];
#pragma unroll
      for (int t = 0; t < VPW; t++) {
        const int qi = warp + t * (TH / 32);
        if (qi < nq) {
          const int row = r0 + (q0 + qi) / G, head = kvh * G + (q0 + qi) % G;
          const uint16_t* src = a.qkv + (size_t)row * stride + head * D;
#pragma unroll
          for (int e = 0; e < E; e++) v[t][e] = bf(src[lane + 32 * e]);
        }
      }
      if (n0 < sm.nnew) {
        const uint16_t* src = a.qkv + (size_t)sm.new_row[n0] * stride + (a.Hq + kvh) * D;
#pragma unroll
        for (int e = 0; e < E; e++) {
          kv[e] = bf(src[lane + 32 * e]);
          vv[e] = src[(size_t)a.Hkv * D + lane + 32 * e];
        }
      }
      // this CTA's query vectors: RMSNorm + RoPE, rounded to bf16 as the unfused path stores them
#pragma unroll
      for (int t = 0; t < VPW; t++) {
        const int qi = warp + t * (TH / 32);
        if (qi < nq) {
          uint16_t o[E];
          norm_rope_vals<D>(v[t], qw, a.eps, qpos[t], fq, o);
#pragma unroll
          for (int e = 0; e < E; e++) sm.qs[qi][lane + 32 * e] = o[e];
        }
      }
      // the new rows' keys and values of this CTA's splits (the first query block's CTA also writes them out)
      auto put_new = [&](int n, const float (&kin)[E], const uint16_t (&vin)[E], int pos, int page) {
        uint16_t o[E];
        norm_rope_vals<D>(kin, kw, a.eps, pos, fq, o);
        const int slot = sm.new_slot[n];
        const size_t off = (((size_t)page * a.Hkv + kvh) * 16 + (slot & 15)) * D;
#pragma unroll
        for (int e = 0; e < E; e++) {
          const int d = lane + 32 * e;
          sm.nk[n][d] = o[e];
          sm.nv[n][d] = vin[e];
          if (qb == 0) {
            a.kc[off + d] = o[e];
            a.vc[off + d] = vin[e];
          }
        }
      };
      if (n0 < sm.nnew) put_new(n0, kv, vv, kpos, kpage);
      for (int n = n0 + TH / 32; n < sm.nnew; n += TH / 32) {
        const int row = sm.new_row[n];
        const uint16_t* src = a.qkv + (size_t)row * stride + (a.Hq + kvh) * D;
        float k2[E];
        uint16_t v2[E];
#pragma unroll
        for (int e = 0; e < E; e++) {
          k2[e] = bf(src[lane + 32 * e]);
          v2[e] = src[(size_t)a.Hkv * D + lane + 32 * e];
        }
        put_new(n, k2, v2, a.row_pos[row], a.page_table[(size_t)prow * a.max_pages + (sm.new_slot[n] >> 4)]);
      }
      __syncthreads();
      fill_new(0);
      if (second) fill_new(Smem::NB - 1);
    }
  } else {
    for (int i = tid; i < nq * D; i += TH) {
      const int qi = i / D, d = i % D;
      const int row = r0 + (q0 + qi) / G, head = kvh * G + (q0 + qi) % G;
      sm.qs[qi][d] = a.q[((size_t)row * a.Hq + head) * D + d];
    }
  }

  // Tensor-core tiles (mma.sync m16n8k16, bf16 in, fp32 accumulate). Scores S[q][key] = Q K^T: warp w owns
  // keys 16w..16w+15 (two n8 tiles) for all query rows. Output O[q][d] = P V: warp w owns dims
  // [w D/4, (w+1) D/4); P enters as two bf16 operands (high and low parts), so it keeps ~16 bits.
  constexpr int MT = Smem::QM / 16;     // m16 tiles of query rows
  constexpr int DW = D / W;             // output dims per warp
  constexpr int KPW = AT_KB / W;        // keys per warp in the scores
  constexpr int NTK = KPW / 8;          // n8 tiles of keys per warp
  constexpr int NTO = DW / 8;           // n8 tiles of output dims per warp
  float o_acc[MT][NTO][4];
#pragma unroll
  for (int mt = 0; mt < MT; mt++)
#pragma unroll
    for (int nt = 0; nt < NTO; nt++)
#pragma unroll
      for (int e = 0; e < 4; e++) o_acc[mt][nt][e] = 0.f;
  const int g = lane >> 2, t = lane & 3;
  const size_t group = ((size_t)b * a.Hkv + kvh) * a.qblocks + qb;

  for (int split = blockIdx.x; any && split * a.kpc < kv_len; split += stride_x) {
    if (split != (int)blockIdx.x) {
      // the previous split's probabilities, K/V and statistics are consumed and published
      __syncthreads();
      k_begin = split * a.kpc;
      k_end = min(kv_len, k_begin + a.kpc);
      for (int i = tid; i < NQ; i += TH) {
        sm.m[i] = -INFINITY;
        sm.l[i] = 0.f;
      }
      for (int i = tid; i < Smem::QM; i += TH) sm.alpha[i] = 0.f;
#pragma unroll
      for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int nt = 0; nt < NTO; nt++)
#pragma unroll
          for (int e = 0; e < 4; e++) o_acc[mt][nt][e] = 0.f;
      stage_old(k_begin, 0);
      second = Smem::NB > 1 && k_begin + AT_KB < k_end;
      if (second) stage_old(k_begin + AT_KB, Smem::NB - 1);
      fill_new(0);
      if (second) fill_new(Smem::NB - 1);
    }
    int bi = 0;
    for (int kb0 = k_begin; kb0 < k_end; kb0 += AT_KB, bi++) {
      const int buf = bi % Smem::NB;
      bool ahead = false;  // the next block's copies are in flight behind this block's
      if (Smem::NB > 1) {
        if (bi == 0) {
          ahead = second;
        } else {
          __syncthreads();  // block bi - 1 is consumed: its buffer takes block bi + 1
          if (kb0 + AT_KB < k_end) {
            stage_old(kb0 + AT_KB, (bi + 1) % Smem::NB);
            fill_new((bi + 1) % Smem::NB);
            ahead = true;
          }
        }
      } else if (bi > 0) {
        __syncthreads();  // the previous block's K/V and probabilities are consumed
        stage_old(kb0, 0);
        fill_new(0);
      }
      if (ahead)
        cp_async_wait<1>();
      else
        cp_async_wait<0>();
      __syncthreads();
      // scores
      {
        float sacc[MT][NTK][4];
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
          for (int nt = 0; nt < NTK; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) sacc[mt][nt][e] = 0.f;
        const int n0 = warp * KPW;
#pragma unroll 4
        for (int kk = 0; kk < D / 16; kk++) {
          uint32_t bk[NTK][2];
#pragma unroll
          for (int nt = 0; nt < NTK; nt++) {
            bk[nt][0] = sm.ks[buf][n0 + nt * 8 + g][kk * 8 + t];
            bk[nt][1] = sm.ks[buf][n0 + nt * 8 + g][kk * 8 + 4 + t];
          }
#pragma unroll
          for (int mt = 0; mt < MT; mt++) {
            const uint32_t* q0r = reinterpret_cast<const uint32_t*>(&sm.qs[mt * 16 + g][kk * 16 + 2 * t]);
            const uint32_t* q8r = reinterpret_cast<const uint32_t*>(&sm.qs[mt * 16 + g + 8][kk * 16 + 2 * t]);
            const uint32_t a0 = q0r[0], a1 = q8r[0], a2 = q0r[4], a3 = q8r[4];
#pragma unroll
            for (int nt = 0; nt < NTK; nt++) mma_bf16(sacc[mt][nt], a0, a1, a2, a3, bk[nt][0], bk[nt][1]);
          }
        }
        // scale and mask into sm.s; a block that every row sees whole (below every row's limit and the tree, no
      // window) skips the per-key tests
      if (kb0 + AT_KB <= min_vis) {
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
          for (int nt = 0; nt < NTK; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const int qi = mt * 16 + g + (e >> 1) * 8;
              if (qi < nq) sm.s[qi][n0 + nt * 8 + 2 * t + (e & 1)] = sacc[mt][nt][e] * a.scale;
            }
      } else {
#pragma unroll
        for (int mt = 0; mt < MT; mt++)
#pragma unroll
          for (int nt = 0; nt < NTK; nt++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
              const int qi = mt * 16 + g + (e >> 1) * 8;
              const int j = n0 + nt * 8 + 2 * t + (e & 1);
              if (qi < nq) {
                const int slot = kb0 + j;
                const int lim = sm.row_slot[qi];
                bool vis = slot < k_end && slot <= lim;
                if (a.window > 0) vis = vis && slot > lim - a.window;
                if (a.tree_mask && slot >= tbase) {
                  const int node = slot - tbase;
                  vis = vis && node < 64 && ((sm.tmask[qi] >> node) & 1ull);
                }
                sm.s[qi][j] = vis ? sacc[mt][nt][e] * a.scale : -INFINITY;
              }
            }
      }
      }
      __syncthreads();
      // online softmax per query vector: warp w takes w, w+4, ...; p goes out as bf16 high + low parts
      for (int qi = warp; qi < nq; qi += TH / 32) {
        const float s0 = sm.s[qi][lane], s1 = sm.s[qi][lane + 32];
        float bm = fmaxf(s0, s1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
        const float mo = sm.m[qi];
        const float mn = fmaxf(mo, bm);
        const float p0 = mn == -INFINITY ? 0.f : expf(s0 - mn);
        const float p1 = mn == -INFINITY ? 0.f : expf(s1 - mn);
        const float ps = warp_sum(p0 + p1);
        const uint16_t h0 = to_bf(p0), h1 = to_bf(p1);
        sm.ph[qi][lane] = h0;
        sm.ph[qi][lane + 32] = h1;
        sm.pl[qi][lane] = to_bf(p0 - bf(h0));
        sm.pl[qi][lane + 32] = to_bf(p1 - bf(h1));
        if (lane == 0) {
          const float al = mo == -INFINITY ? 0.f : expf(mo - mn);
          sm.alpha[qi] = al;
          sm.l[qi] = sm.l[qi] * al + ps;
          sm.m[qi] = mn;
        }
      }
      __syncthreads();
      // O = alpha O + P V
#pragma unroll
      for (int mt = 0; mt < MT; mt++) {
        const float al0 = sm.alpha[mt * 16 + g], al8 = sm.alpha[mt * 16 + g + 8];
#pragma unroll
        for (int nt = 0; nt < NTO; nt++) {
          o_acc[mt][nt][0] *= al0;
          o_acc[mt][nt][1] *= al0;
          o_acc[mt][nt][2] *= al8;
          o_acc[mt][nt][3] *= al8;
        }
      }
#pragma unroll
      for (int kk = 0; kk < AT_KB / 16; kk++) {
        uint32_t bv[NTO][2];
#pragma unroll
        for (int nt = 0; nt < NTO; nt += 2) {
          const int key = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
          const int d0 = warp * DW + nt * 8 + (lane >> 4) * 8;
          ldsm_x4_trans(bv[nt][0], bv[nt][1], bv[nt + 1][0], bv[nt + 1][1], &sm.vs[buf][key][d0]);
        }
#pragma unroll
        for (int mt = 0; mt < MT; mt++) {
          const int r0w = mt * 16 + g;
          const uint32_t h0 = *reinterpret_cast<const uint32_t*>(&sm.ph[r0w][kk * 16 + 2 * t]);
          const uint32_t h1 = *reinterpret_cast<const uint32_t*>(&sm.ph[r0w + 8][kk * 16 + 2 * t]);
          const uint32_t h2 = *reinterpret_cast<const uint32_t*>(&sm.ph[r0w][kk * 16 + 2 * t + 8]);
          const uint32_t h3 = *reinterpret_cast<const uint32_t*>(&sm.ph[r0w + 8][kk * 16 + 2 * t + 8]);
          const uint32_t l0 = *reinterpret_cast<const uint32_t*>(&sm.pl[r0w][kk * 16 + 2 * t]);
          const uint32_t l1 = *reinterpret_cast<const uint32_t*>(&sm.pl[r0w + 8][kk * 16 + 2 * t]);
          const uint32_t l2 = *reinterpret_cast<const uint32_t*>(&sm.pl[r0w][kk * 16 + 2 * t + 8]);
          const uint32_t l3 = *reinterpret_cast<const uint32_t*>(&sm.pl[r0w + 8][kk * 16 + 2 * t + 8]);
#pragma unroll
          for (int nt = 0; nt < NTO; nt++) {
            mma_bf16(o_acc[mt][nt], h0, h1, h2, h3, bv[nt][0], bv[nt][1]);
            mma_bf16(o_acc[mt][nt], l0, l1, l2, l3, bv[nt][0], bv[nt][1]);
          }
        }
      }
    }

    // publish this split's partial (empty splits publish nothing: the merge stops at the last non-empty one)
    {
      float* mine = a.part + (group * a.nsplit + split) * (size_t)NQ * (D + AT_PAD);
#pragma unroll
      for (int mt = 0; mt < MT; mt++)
#pragma unroll
        for (int nt = 0; nt < NTO; nt++)
#pragma unroll
          for (int h = 0; h < 2; h++) {
            const int qi = mt * 16 + g + h * 8;
            if (qi < nq) {
              const int d = warp * DW + nt * 8 + 2 * t;
              __stcg(reinterpret_cast<float2*>(mine + (size_t)qi * (D + AT_PAD) + d),
                     make_float2(o_acc[mt][nt][2 * h], o_acc[mt][nt][2 * h + 1]));
            }
          }
      for (int i = tid; i < nq; i += TH) {
        __stcg(mine + (size_t)i * (D + AT_PAD) + D, sm.m[i]);
        __stcg(mine + (size_t)i * (D + AT_PAD) + D + 1, sm.l[i]);
      }
    }
  }
  if (a.defer) return;  // the partials are merged by their consumer
  __threadfence();
  __syncthreads();
  if (tid == 0) sm.last = atomicAdd(a.counters + group, 1u) == (unsigned)(live_ctas - 1);
  __syncthreads();
  if (!sm.last) return;
  __threadfence();
  // merge the splits in split order, in one pass: every thread owns (query vector, 4 dims)
  int used = a.nsplit;
  while (used > 1 && (used - 1) * a.kpc >= kv_len) used--;
  constexpr int C4 = D / 4;
  for (int job = tid; job < nq * C4; job += TH) {
    const int i = job / C4, d4 = (job % C4) * 4;
    const float* base = a.part + (group * a.nsplit * NQ + i) * (size_t)(D + AT_PAD);
    uint16_t o4[4];
    attn_merge4(base, (size_t)NQ * (D + AT_PAD), d4, used, D, o4);
    const int row = r0 + (q0 + i) / G, head = kvh * G + (q0 + i) % G;
    uint16_t* dst = a.out + ((size_t)row * a.Hq + head) * D + d4;
    dst[0] = o4[0];
    dst[1] = o4[1];
    dst[2] = o4[2];
    dst[3] = o4[3];
  }
  if (tid == 0) a.counters[group] = 0u;
}

// CTAs per (sequence, kv head, query block): enough for `g_attn_waves` waves of resident CTAs over the whole
// GPU, at most one per split. Only the scheduling changes with it: every split is computed and merged the same
// way whichever CTA walks it.
static int g_attn_waves = 2;

template <int D, int NQ, bool FUSED, int W, int NB>
static int launch_attn(const AttnArgs& args, int B, cudaStream_t st) {
  const size_t smem = sizeof(AttnSmem<D, NQ, FUSED, NB>);
  static bool configured = false;  // per instantiation
  static int resident = 1, sms = 148;
  if (!configured) {
    cudaError_t e =
        cudaFuncSetAttribute(attn_kernel<D, NQ, FUSED, W, NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int dev = 0;
    if (e == cudaSuccess) e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess)
      e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, attn_kernel<D, NQ, FUSED, W, NB>, 32 * W, smem);
    if (e != cudaSuccess) {
      set_error("attention: cannot configure the kernel for %zu bytes of shared memory: %s", smem,
                cudaGetErrorString(e));
      return IM_CUDA_ERROR;
    }
    resident = resident < 1 ? 1 : resident;
    configured = true;
  }
  const long long groups = (long long)B * args.Hkv * args.qblocks;
  const long long want = ((long long)sms * resident * g_attn_waves + groups - 1) / groups;
  const int per_group = (int)(want < 1 ? 1 : (want > args.nsplit ? args.nsplit : want));
  dim3 grid(per_group, args.Hkv, B * args.qblocks);
  return launch("attn_kernel", attn_kernel<D, NQ, FUSED, W, NB>, grid, dim3(32 * W), smem, st, args);
}

template <bool FUSED>
static int dispatch_attn(const AttnArgs& args, int64_t D, int nq, int B, cudaStream_t st) {
  // 8 warps for query blocks of 32 vectors (more warps in flight where shared memory limits the CTAs per SM) and
  // for small blocks of head_dim 128 when the (sequence, kv head) groups are fewer than the SMs (one sequence:
  // each split's chain is shorter); 4 warps for small blocks of large batches (more CTAs per SM). Every score and
  // output element is computed the same way whatever the warp count.
  const long long groups = (long long)B * args.Hkv * args.qblocks;
  if (D == 128) {
    if (nq != 8)
      return groups < 148 ? launch_attn<128, 32, FUSED, 8, 2>(args, B, st) : launch_attn<128, 32, FUSED, 8, 1>(args, B, st);
    return groups < 148 ? launch_attn<128, 8, FUSED, 8, 2>(args, B, st) : launch_attn<128, 8, FUSED, 4, 1>(args, B, st);
  }
  return nq == 8 ? launch_attn<256, 8, FUSED, 4, 1>(args, B, st) : launch_attn<256, 32, FUSED, 8, 1>(args, B, st);
}

// Shared argument checks and setup of both entry points.
static int attn_setup(const char* who, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* page_table,
                      int64_t max_pages, const int32_t* seq_rows, const int32_t* seq_slot, const int32_t* row_slot,
                      const uint64_t* tree_mask, const int32_t* tree_base, int64_t B, int64_t max_rows_per_seq,
                      int64_t Hq, int64_t Hkv, int64_t D, int64_t max_kv_len, int64_t keys_per_split, int64_t window,
                      float scale, uint16_t* out, void* workspace, size_t workspace_bytes, AttnArgs* args, int* nq);

}  // namespace im

using namespace im;

extern "C" size_t im_attention_workspace_bytes(int64_t B, int64_t max_rows_per_seq, int64_t Hq, int64_t Hkv,
                                               int64_t D, int64_t max_kv_len, int64_t keys_per_split) {
  if (B < 1 || max_rows_per_seq < 1 || Hkv < 1 || Hq % Hkv || keys_per_split < AT_KB || keys_per_split % AT_KB)
    return 0;
  int nq, qblocks;
  attn_geometry(max_rows_per_seq, Hq / Hkv, &nq, &qblocks);
  const int64_t nsplit = (max_kv_len + keys_per_split - 1) / keys_per_split;
  const int64_t groups = B * Hkv * qblocks;
  if (groups > AT_MAX_GROUPS) return 0;
  return AT_COUNTER_BYTES + (size_t)groups * nsplit * nq * (D + AT_PAD) * sizeof(float);
}

extern "C" int im_attention_tune(int waves) {
  IM_REQUIRE(waves >= 1 && waves <= 64, IM_INVALID, "im_attention_tune: waves %d", waves);
  g_attn_waves = waves;
  return IM_OK;
}

namespace im {
static int attn_setup(const char* who, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* page_table,
                      int64_t max_pages, const int32_t* seq_rows, const int32_t* seq_slot, const int32_t* row_slot,
                      const uint64_t* tree_mask, const int32_t* tree_base, int64_t B, int64_t max_rows_per_seq,
                      int64_t Hq, int64_t Hkv, int64_t D, int64_t max_kv_len, int64_t keys_per_split, int64_t window,
                      float scale, uint16_t* out, void* workspace, size_t workspace_bytes, AttnArgs* args, int* nq) {
  IM_REQUIRE(B >= 1 && max_rows_per_seq >= 1 && Hq >= 1 && Hkv >= 1 && Hq % Hkv == 0, IM_INVALID, "%s: bad sizes",
             who);
  IM_REQUIRE(D == 128 || D == 256, IM_UNSUPPORTED, "%s: head_dim %lld", who, (long long)D);
  IM_REQUIRE(keys_per_split >= AT_KB && keys_per_split % AT_KB == 0, IM_INVALID,
             "%s: keys_per_split must be a positive multiple of 64", who);
  IM_REQUIRE(max_kv_len >= 1 && max_kv_len <= max_pages * 16, IM_INVALID, "%s: max_kv_len %lld exceeds the page table",
             who, (long long)max_kv_len);
  IM_REQUIRE(k_cache && v_cache && page_table && seq_rows && row_slot && workspace, IM_INVALID,
             "%s: null pointer", who);
  IM_REQUIRE(!tree_mask || tree_base, IM_INVALID, "%s: tree_mask needs tree_base", who);
  IM_REQUIRE(aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(workspace, 256), IM_INVALID,
             "%s: caches must be 16-byte and the workspace 256-byte aligned", who);
  const size_t need = im_attention_workspace_bytes(B, max_rows_per_seq, Hq, Hkv, D, max_kv_len, keys_per_split);
  IM_REQUIRE(need > 0, IM_UNSUPPORTED, "%s: too many (sequence, kv head, query block) groups", who);
  IM_REQUIRE(workspace_bytes >= need, IM_INVALID, "%s: workspace of %zu bytes needed, %zu given", who, need,
             workspace_bytes);
  int qblocks;
  attn_geometry(max_rows_per_seq, Hq / Hkv, nq, &qblocks);
  AttnArgs& A = *args;
  A = AttnArgs{};
  A.kc = const_cast<uint16_t*>(k_cache);
  A.vc = const_cast<uint16_t*>(v_cache);
  A.page_table = page_table;
  A.seq_rows = seq_rows;
  A.seq_slot = seq_slot;
  A.row_slot = row_slot;
  A.tree_mask = reinterpret_cast<const unsigned long long*>(tree_mask);
  A.tree_base = tree_base;
  A.out = out;
  A.counters = reinterpret_cast<unsigned*>(workspace);
  A.part = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + AT_COUNTER_BYTES);
  A.max_pages = (int)max_pages;
  A.Hq = (int)Hq;
  A.Hkv = (int)Hkv;
  A.kpc = (int)keys_per_split;
  A.nsplit = (int)((max_kv_len + keys_per_split - 1) / keys_per_split);
  A.qblocks = qblocks;
  A.window = (int)window;
  A.scale = scale;
  return IM_OK;
}
}  // namespace im

extern "C" int im_attention_paged(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                  const int32_t* page_table, int64_t max_pages, const int32_t* seq_rows,
                                  const int32_t* seq_slot, const int32_t* row_slot, const uint64_t* tree_mask,
                                  const int32_t* tree_base, int64_t B, int64_t max_rows_per_seq, int64_t Hq,
                                  int64_t Hkv, int64_t D, int64_t max_kv_len, int64_t keys_per_split, int64_t window,
                                  float scale, uint16_t* out, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  AttnArgs args;
  int nq;
  int rc = attn_setup("im_attention_paged", k_cache, v_cache, page_table, max_pages, seq_rows, seq_slot, row_slot,
                      tree_mask, tree_base, B, max_rows_per_seq, Hq, Hkv, D, max_kv_len, keys_per_split, window, scale,
                      out, workspace, workspace_bytes, &args, &nq);
  if (rc) return rc;
  IM_REQUIRE(q && out, IM_INVALID, "im_attention_paged: null q or out");
  args.q = q;
  return dispatch_attn<false>(args, D, nq, (int)B, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int im_attention_qkv_paged(const uint16_t* qkv, const uint16_t* q_norm, const uint16_t* k_norm,
                                      const float* inv_freq, const int32_t* row_pos, float eps, int gemma_style,
                                      uint16_t* k_cache, uint16_t* v_cache, const int32_t* page_table,
                                      int64_t max_pages, const int32_t* seq_rows, const int32_t* seq_slot,
                                      const int32_t* row_slot, const uint64_t* tree_mask, const int32_t* tree_base,
                                      int64_t B, int64_t max_rows_per_seq, int64_t Hq, int64_t Hkv, int64_t D,
                                      int64_t max_kv_len, int64_t keys_per_split, int64_t window, float scale,
                                      uint16_t* out, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  AttnArgs args;
  int nq;
  int rc = attn_setup("im_attention_qkv_paged", k_cache, v_cache, page_table, max_pages, seq_rows, seq_slot,
                      row_slot, tree_mask, tree_base, B, max_rows_per_seq, Hq, Hkv, D, max_kv_len, keys_per_split,
                      window, scale, out, workspace, workspace_bytes, &args, &nq);
  if (rc) return rc;
  IM_REQUIRE(max_rows_per_seq <= AT_MAXNEW, IM_UNSUPPORTED, "im_attention_qkv_paged: at most %d rows per sequence",
             AT_MAXNEW);
  IM_REQUIRE(qkv && q_norm && k_norm && inv_freq && row_pos, IM_INVALID, "im_attention_qkv_paged: null pointer");
  args.qkv = qkv;
  args.q_norm = q_norm;
  args.k_norm = k_norm;
  args.inv_freq = inv_freq;
  args.row_pos = row_pos;
  args.eps = eps;
  args.gemma = gemma_style;
  args.defer = out == nullptr;
  return dispatch_attn<true>(args, D, nq, (int)B, reinterpret_cast<cudaStream_t>(stream));
}
