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
// Work split: grid (key splits, kv heads, sequences x query blocks). A CTA owns up to NQ query vectors
// (rows x the kv head's query heads) and one split of `kpc` keys at fixed absolute positions, walked in
// 64-key blocks staged in shared memory with an online softmax. CTAs publish (acc, max, sum) partials; the
// last CTA of a (sequence, kv head, query block) merges the splits in split order. A row's result depends
// only on its own query, its mask and the KV -- not on how many rows or sequences share the launch.
#include <math.h>

#include "common.cuh"

namespace im {

constexpr int AT_THREADS = 128;
constexpr int AT_KB = 64;  // keys per shared-memory block
// Workspace layout, identical for every call so calls of different shapes may share one buffer: arrival
// counters in a fixed region (kept at zero between launches), then the split partials.
constexpr size_t AT_COUNTER_BYTES = 65536;
constexpr int64_t AT_MAX_GROUPS = (int64_t)(AT_COUNTER_BYTES / 4);

struct AttnArgs {
  const uint16_t* q;
  const uint16_t* kc;
  const uint16_t* vc;
  const int* page_table;
  const int* seq_rows;
  const int* seq_slot;  // page-table row of each sequence group (NULL: group b uses row b)
  const int* row_slot;
  const unsigned long long* tree_mask;
  const int* tree_base;
  uint16_t* out;
  float* part;
  unsigned* counters;
  int max_pages, Hq, Hkv, kpc, nsplit, qblocks, window;
  float scale;
};

template <int D, int NQ>
struct AttnSmem {
  float qs[NQ][D];
  uint32_t ks[AT_KB][D / 2 + 1];  // bf16 pairs, odd row stride in words: conflict-free per-key reads
  uint16_t vs[AT_KB][D];
  float s[NQ][AT_KB];
  float m[NQ], l[NQ], alpha[NQ];
  int row_slot[NQ];
  unsigned long long tmask[NQ];
  int last;
};

template <int D, int NQ>
__global__ void __launch_bounds__(AT_THREADS)
attn_kernel(AttnArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  AttnSmem<D, NQ>& sm = *reinterpret_cast<AttnSmem<D, NQ>*>(smem_raw);
  pdl_wait();
  pdl_trigger();
  const int split = blockIdx.x, kvh = blockIdx.y;
  const int b = blockIdx.z / a.qblocks, qb = blockIdx.z % a.qblocks;
  const int tid = threadIdx.x;
  const int G = a.Hq / a.Hkv;
  const int r0 = a.seq_rows[b], nr = a.seq_rows[b + 1] - r0;
  const int prow = a.seq_slot ? a.seq_slot[b] : b;
  const int q0 = qb * NQ;
  const int nq = max(0, min(NQ, nr * G - q0));

  // kv length of the sequence: one past the largest slot any of its rows was written to
  int kv_len = 0;
  for (int r = 0; r < nr; r++) kv_len = max(kv_len, a.row_slot[r0 + r] + 1);
  const int tbase = a.tree_mask ? a.tree_base[b] : 0;

  for (int i = tid; i < NQ; i += AT_THREADS) {
    sm.m[i] = -INFINITY;
    sm.l[i] = 0.f;
    if (i < nq) {
      const int row = r0 + (q0 + i) / G;
      sm.row_slot[i] = a.row_slot[row];
      sm.tmask[i] = a.tree_mask ? a.tree_mask[row] : 0ull;
    }
  }
  for (int i = tid; i < nq * D; i += AT_THREADS) {
    const int qi = i / D, d = i % D;
    const int row = r0 + (q0 + qi) / G, head = kvh * G + (q0 + qi) % G;
    sm.qs[qi][d] = bf(a.q[((size_t)row * a.Hq + head) * D + d]);
  }
  constexpr int DPT = D / AT_THREADS;  // output dims per thread in the P.V step
  float acc[NQ][DPT];
#pragma unroll
  for (int i = 0; i < NQ; i++)
#pragma unroll
    for (int e = 0; e < DPT; e++) acc[i][e] = 0.f;

  const int k_begin = split * a.kpc;
  const int k_end = min(kv_len, k_begin + a.kpc);
  for (int kb0 = k_begin; kb0 < k_end && nq > 0; kb0 += AT_KB) {
    __syncthreads();
    // stage K (as bf16 pairs) and V for keys [kb0, kb0 + 64)
    for (int i = tid; i < AT_KB * (D / 8); i += AT_THREADS) {
      const int j = i / (D / 8), c = i % (D / 8);
      const int slot = kb0 + j;
      uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (slot < k_end) {
        const int page = a.page_table[(size_t)prow * a.max_pages + (slot >> 4)];
        const size_t off = (((size_t)page * a.Hkv + kvh) * 16 + (slot & 15)) * D + c * 8;
        kv = ldg_u4(a.kc + off);
        vv = ldg_u4(a.vc + off);
      }
      sm.ks[j][c * 4 + 0] = kv.x;
      sm.ks[j][c * 4 + 1] = kv.y;
      sm.ks[j][c * 4 + 2] = kv.z;
      sm.ks[j][c * 4 + 3] = kv.w;
      *reinterpret_cast<uint4*>(&sm.vs[j][c * 8]) = vv;
    }
    __syncthreads();
    // scores: thread -> key j, query vectors h, h+2, h+4, ...
    {
      const int j = tid & (AT_KB - 1), h = tid >> 6;
      constexpr int PER = NQ / 2;
      float sc[PER];
#pragma unroll
      for (int i = 0; i < PER; i++) sc[i] = 0.f;
#pragma unroll 4
      for (int d2 = 0; d2 < D / 2; d2++) {
        const uint32_t kk = sm.ks[j][d2];
        const float k0 = bf_lo(kk), k1 = bf_hi(kk);
#pragma unroll
        for (int i = 0; i < PER; i++) {
          const float2 qq = *reinterpret_cast<const float2*>(&sm.qs[h + 2 * i][2 * d2]);
          sc[i] = fmaf(qq.y, k1, fmaf(qq.x, k0, sc[i]));
        }
      }
      const int slot = kb0 + j;
#pragma unroll
      for (int i = 0; i < PER; i++) {
        const int qi = h + 2 * i;
        if (qi < nq) {
          const int lim = sm.row_slot[qi];
          bool vis = slot < k_end && slot <= lim;
          if (a.window > 0) vis = vis && slot > lim - a.window;
          if (a.tree_mask && slot >= tbase) {
            const int node = slot - tbase;
            vis = vis && node < 64 && ((sm.tmask[qi] >> node) & 1ull);
          }
          sm.s[qi][j] = vis ? sc[i] * a.scale : -INFINITY;
        }
      }
    }
    __syncthreads();
    // online softmax per query vector: warp w takes w, w+4, ...
    {
      const int warp = tid >> 5, lane = tid & 31;
      for (int qi = warp; qi < nq; qi += AT_THREADS / 32) {
        const float s0 = sm.s[qi][lane], s1 = sm.s[qi][lane + 32];
        float bm = fmaxf(s0, s1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
        const float mo = sm.m[qi];
        const float mn = fmaxf(mo, bm);
        const float p0 = mn == -INFINITY ? 0.f : expf(s0 - mn);
        const float p1 = mn == -INFINITY ? 0.f : expf(s1 - mn);
        const float ps = warp_sum(p0 + p1);
        sm.s[qi][lane] = p0;
        sm.s[qi][lane + 32] = p1;
        if (lane == 0) {
          const float al = mo == -INFINITY ? 0.f : expf(mo - mn);
          sm.alpha[qi] = al;
          sm.l[qi] = sm.l[qi] * al + ps;
          sm.m[qi] = mn;
        }
      }
    }
    __syncthreads();
    // P.V: thread owns dims tid, tid + 128, ...
#pragma unroll
    for (int i = 0; i < NQ; i++) {
      if (i < nq) {
        const float al = sm.alpha[i];
#pragma unroll
        for (int e = 0; e < DPT; e++) acc[i][e] *= al;
      }
    }
    for (int j = 0; j < AT_KB; j += 4) {
      float v[4][DPT];
#pragma unroll
      for (int jj = 0; jj < 4; jj++)
#pragma unroll
        for (int e = 0; e < DPT; e++) v[jj][e] = bf(sm.vs[j + jj][tid + e * AT_THREADS]);
#pragma unroll
      for (int i = 0; i < NQ; i++) {
        if (i < nq) {
          const float4 p = *reinterpret_cast<const float4*>(&sm.s[i][j]);
#pragma unroll
          for (int e = 0; e < DPT; e++)
            acc[i][e] = fmaf(p.w, v[3][e], fmaf(p.z, v[2][e], fmaf(p.y, v[1][e], fmaf(p.x, v[0][e], acc[i][e]))));
        }
      }
    }
  }
  __syncthreads();

  // publish this split's partial: acc[D], max, sum per query vector
  const size_t group = ((size_t)b * a.Hkv + kvh) * a.qblocks + qb;
  float* mine = a.part + (group * a.nsplit + split) * (size_t)NQ * (D + 2);
#pragma unroll
  for (int i = 0; i < NQ; i++) {
    if (i < nq) {
#pragma unroll
      for (int e = 0; e < DPT; e++) __stcg(mine + (size_t)i * (D + 2) + tid + e * AT_THREADS, acc[i][e]);
    }
  }
  for (int i = tid; i < nq; i += AT_THREADS) {
    __stcg(mine + (size_t)i * (D + 2) + D, sm.m[i]);
    __stcg(mine + (size_t)i * (D + 2) + D + 1, sm.l[i]);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) sm.last = atomicAdd(a.counters + group, 1u) == (unsigned)(a.nsplit - 1);
  __syncthreads();
  if (!sm.last) return;
  __threadfence();
  // merge the splits in split order: warp w takes query vectors w, w+4, ...; lane owns D/32 dims
  {
    const int warp = tid >> 5, lane = tid & 31;
    constexpr int DPL = D / 32;
    int used = a.nsplit;
    while (used > 1 && (used - 1) * a.kpc >= kv_len) used--;
    for (int i = warp; i < nq; i += AT_THREADS / 32) {
      float mx = -INFINITY;
      for (int s0 = lane; s0 < used; s0 += 32)
        mx = fmaxf(mx, __ldcg(a.part + ((group * a.nsplit + s0) * NQ + i) * (D + 2) + D));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      float L = 0.f, O[DPL];
#pragma unroll
      for (int e = 0; e < DPL; e++) O[e] = 0.f;
#pragma unroll 4
      for (int s = 0; s < used; s++) {
        const float* p = a.part + ((group * a.nsplit + s) * NQ + i) * (D + 2);
        const float ms = __ldcg(p + D);
        const float ls = __ldcg(p + D + 1);
        float v[DPL];
#pragma unroll
        for (int e = 0; e < DPL; e++) v[e] = __ldcg(p + lane + 32 * e);
        const float w = (ms == -INFINITY || mx == -INFINITY) ? 0.f : expf(ms - mx);
        L = fmaf(ls, w, L);
#pragma unroll
        for (int e = 0; e < DPL; e++) O[e] = fmaf(v[e], w, O[e]);
      }
      const int row = r0 + (q0 + i) / G, head = kvh * G + (q0 + i) % G;
#pragma unroll
      for (int e = 0; e < DPL; e++)
        a.out[((size_t)row * a.Hq + head) * D + lane + 32 * e] = to_bf(L > 0.f ? __fdiv_rn(O[e], L) : 0.f);
    }
  }
  if (tid == 0) a.counters[group] = 0u;
}

template <int D, int NQ>
static int launch_attn(const AttnArgs& args, int B, cudaStream_t st) {
  const size_t smem = sizeof(AttnSmem<D, NQ>);
  static bool configured = false;  // per instantiation
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attn_kernel<D, NQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) {
      set_error("attention: cannot reserve %zu bytes of shared memory: %s", smem, cudaGetErrorString(e));
      return IM_CUDA_ERROR;
    }
    configured = true;
  }
  dim3 grid(args.nsplit, args.Hkv, B * args.qblocks);
  return launch("attn_kernel", attn_kernel<D, NQ>, grid, dim3(AT_THREADS), smem, st, args);
}

static void attn_geometry(int64_t rows_per_seq, int64_t G, int* nq, int* qblocks) {
  const int64_t qv = rows_per_seq * G;
  *nq = qv <= 8 ? 8 : 32;
  *qblocks = (int)((qv + *nq - 1) / *nq);
}

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
  return AT_COUNTER_BYTES + (size_t)groups * nsplit * nq * (D + 2) * sizeof(float);
}

extern "C" int im_attention_paged(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                                  const int32_t* page_table, int64_t max_pages, const int32_t* seq_rows,
                                  const int32_t* seq_slot, const int32_t* row_slot, const uint64_t* tree_mask, const int32_t* tree_base,
                                  int64_t B, int64_t max_rows_per_seq, int64_t Hq, int64_t Hkv, int64_t D,
                                  int64_t max_kv_len, int64_t keys_per_split, int64_t window, float scale,
                                  uint16_t* out, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  IM_REQUIRE(B >= 1 && max_rows_per_seq >= 1 && Hq >= 1 && Hkv >= 1 && Hq % Hkv == 0, IM_INVALID,
             "im_attention_paged: bad sizes");
  IM_REQUIRE(D == 128 || D == 256, IM_UNSUPPORTED, "im_attention_paged: head_dim %lld", (long long)D);
  IM_REQUIRE(keys_per_split >= AT_KB && keys_per_split % AT_KB == 0, IM_INVALID,
             "im_attention_paged: keys_per_split must be a positive multiple of 64");
  IM_REQUIRE(max_kv_len >= 1 && max_kv_len <= max_pages * 16, IM_INVALID,
             "im_attention_paged: max_kv_len %lld exceeds the page table", (long long)max_kv_len);
  IM_REQUIRE(q && k_cache && v_cache && page_table && seq_rows && row_slot && out && workspace, IM_INVALID,
             "im_attention_paged: null pointer");
  IM_REQUIRE(!tree_mask || tree_base, IM_INVALID, "im_attention_paged: tree_mask needs tree_base");
  IM_REQUIRE(aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(workspace, 256), IM_INVALID,
             "im_attention_paged: caches must be 16-byte and the workspace 256-byte aligned");
  const size_t need = im_attention_workspace_bytes(B, max_rows_per_seq, Hq, Hkv, D, max_kv_len, keys_per_split);
  IM_REQUIRE(need > 0, IM_UNSUPPORTED, "im_attention_paged: too many (sequence, kv head, query block) groups");
  IM_REQUIRE(workspace_bytes >= need, IM_INVALID, "im_attention_paged: workspace of %zu bytes needed, %zu given",
             need, workspace_bytes);
  int nq, qblocks;
  attn_geometry(max_rows_per_seq, Hq / Hkv, &nq, &qblocks);
  AttnArgs args;
  args.q = q;
  args.kc = k_cache;
  args.vc = v_cache;
  args.page_table = page_table;
  args.seq_rows = seq_rows;
  args.seq_slot = seq_slot;
  args.row_slot = row_slot;
  args.tree_mask = reinterpret_cast<const unsigned long long*>(tree_mask);
  args.tree_base = tree_base;
  args.out = out;
  args.counters = reinterpret_cast<unsigned*>(workspace);
  args.part = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + AT_COUNTER_BYTES);
  args.max_pages = (int)max_pages;
  args.Hq = (int)Hq;
  args.Hkv = (int)Hkv;
  args.kpc = (int)keys_per_split;
  args.nsplit = (int)((max_kv_len + keys_per_split - 1) / keys_per_split);
  args.qblocks = qblocks;
  args.window = (int)window;
  args.scale = scale;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (D == 128) return nq == 8 ? launch_attn<128, 8>(args, (int)B, st) : launch_attn<128, 32>(args, (int)B, st);
  return nq == 8 ? launch_attn<256, 8>(args, (int)B, st) : launch_attn<256, 32>(args, (int)B, st);
}
