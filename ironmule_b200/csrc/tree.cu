// Tree speculation on the device: top-k drafting, the tree's row bookkeeping, greedy acceptance of the longest
// path the target agrees with, and compaction of the accepted nodes' K/V into the committed slots.
//
// The tree is static in shape: `levels` levels below the root with branching branch[0..levels-1]; nodes are
// numbered level by level, the children of node i of level L being consecutive in level L + 1. Node j of a
// sequence whose committed length is n sits in KV slot n + j (tree_base = n) at RoPE position n - 1 + depth(j);
// verify row 0 is the root (the last committed token, slot n - 1) and row 1 + j is node j. A node's mask has the
// bits of its ancestors and itself, so attention sees the committed prefix plus its own path -- the keys a
// linear decode of that path would see, which is why an accepted path's K/V equal the linear decode's bit for
// bit and tree speculation returns exactly the greedy tokens.
//
// No reference code exists for trees (the reference's speculation is linear,
// ironmule/speculation.py:39-108). Greedy acceptance follows its rule, applied along the tree.
#include <math.h>

#include "common.cuh"

namespace im {

constexpr int TK_MAX = 8;          // top-k at most
constexpr int TK_THREADS = 256;
constexpr int TK_CHUNK = 4096;     // logits per CTA
constexpr int TR_MAX_LEVELS = 4;
constexpr int TR_MAX_NODES = 63;   // mask bits

struct TkCand {
  float v;
  int i;
};
// a before b: larger value, then smaller index (NaN counts as -inf)
__device__ __forceinline__ bool tk_before(const TkCand& a, const TkCand& b) {
  return a.v > b.v || (a.v == b.v && a.i < b.i);
}
template <int K>
__device__ __forceinline__ void tk_insert(TkCand (&list)[K], TkCand c) {
  if (!tk_before(c, list[K - 1])) return;
  int p = K - 1;
  while (p > 0 && tk_before(c, list[p - 1])) {
    list[p] = list[p - 1];
    p--;
  }
  list[p] = c;
}

// grid (chunks, rows): each CTA keeps the top K of its chunk (threads' own lists, then a fixed-order tree of
// list merges in shared memory); the last CTA of a row merges the chunks' lists in chunk order.
template <int K>
__global__ void __launch_bounds__(TK_THREADS)
topk_kernel(const uint16_t* __restrict__ logits, int V, long long ld, int chunks, int32_t* __restrict__ out,
            int out_stride, TkCand* __restrict__ part, unsigned* __restrict__ counters) {
  __shared__ TkCand sh[TK_THREADS][K];
  __shared__ int last;
  pdl_wait();
  pdl_trigger();
  const int chunk = blockIdx.x, row = blockIdx.y;
  const uint16_t* lp = logits + (size_t)row * ld;
  TkCand mine[K];
#pragma unroll
  for (int j = 0; j < K; j++) mine[j] = TkCand{-INFINITY, 0x7fffffff};
  const int v0 = chunk * TK_CHUNK, v1 = min(V, v0 + TK_CHUNK);
  for (int v = v0 + threadIdx.x; v < v1; v += TK_THREADS) {
    float x = bf(lp[v]);
    if (x != x) x = -INFINITY;
    tk_insert<K>(mine, TkCand{x, v});
  }
#pragma unroll
  for (int j = 0; j < K; j++) sh[threadIdx.x][j] = mine[j];
  __syncthreads();
  for (int stride = TK_THREADS / 2; stride > 0; stride >>= 1) {
    if (threadIdx.x < stride) {
      TkCand a[K];
#pragma unroll
      for (int j = 0; j < K; j++) a[j] = sh[threadIdx.x][j];
#pragma unroll
      for (int j = 0; j < K; j++) tk_insert<K>(a, sh[threadIdx.x + stride][j]);
#pragma unroll
      for (int j = 0; j < K; j++) sh[threadIdx.x][j] = a[j];
    }
    __syncthreads();
  }
  TkCand* mine_part = part + ((size_t)row * chunks + chunk) * K;
  if (threadIdx.x < K) mine_part[threadIdx.x] = sh[0][threadIdx.x];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(counters + row, 1u) == (unsigned)(chunks - 1);
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  TkCand best[K];
#pragma unroll
  for (int j = 0; j < K; j++) best[j] = TkCand{-INFINITY, 0x7fffffff};
  for (int c = 0; c < chunks; c++)
#pragma unroll
    for (int j = 0; j < K; j++) {
      const TkCand* p = part + ((size_t)row * chunks + c) * K + j;
      tk_insert<K>(best, TkCand{__ldcg(&p->v), __ldcg(&p->i)});
    }
#pragma unroll
  for (int j = 0; j < K; j++) out[(size_t)row * out_stride + j] = best[j].i < V ? best[j].i : 0;
  counters[row] = 0u;
}

struct TreeShape {
  int levels;
  int branch[TR_MAX_LEVELS];
  int count[TR_MAX_LEVELS];   // nodes per level
  int first[TR_MAX_LEVELS];   // first node index of each level
  int total;
};

__device__ __forceinline__ int tree_level(const TreeShape& t, int j) {
  int L = 0;
  while (L + 1 < t.levels && j >= t.first[L + 1]) L++;
  return L;
}
__device__ __forceinline__ int tree_parent(const TreeShape& t, int j) {  // -1: the root
  const int L = tree_level(t, j);
  if (L == 0) return -1;
  return t.first[L - 1] + (j - t.first[L]) / t.branch[L];
}

// Per sequence: the two re-fed rows of the first draft pass, and the verify rows (root + nodes): slot,
// position and mask; the node tokens are written by the top-k passes.
__global__ void tree_prepare_kernel(const int* __restrict__ hist, int cap, const int* __restrict__ n, int B,
                                    TreeShape t, int slot_cap, int* __restrict__ d0_tok, int* __restrict__ d0_pos,
                                    int* __restrict__ v_tok, int* __restrict__ v_pos, int* __restrict__ v_slot,
                                    unsigned long long* __restrict__ v_mask, int* __restrict__ tbase) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  if (b >= B) return;
  int nb = n[b];
  nb = max(2, min(nb, min(cap, slot_cap - t.total)));
  const int* h = hist + (size_t)b * cap;
  const int rows = 1 + t.total;
  if (threadIdx.x == 0) {
    d0_tok[2 * b] = h[nb - 2];
    d0_tok[2 * b + 1] = h[nb - 1];
    d0_pos[2 * b] = nb - 2;
    d0_pos[2 * b + 1] = nb - 1;
    v_tok[(size_t)b * rows] = h[nb - 1];
    v_pos[(size_t)b * rows] = nb - 1;
    v_slot[(size_t)b * rows] = nb - 1;
    v_mask[(size_t)b * rows] = 0ull;
    tbase[b] = nb;
  }
  for (int j = threadIdx.x; j < t.total; j += blockDim.x) {
    unsigned long long m = 0ull;
    int depth = 0;
    for (int a = j; a >= 0; a = tree_parent(t, a)) {
      m |= 1ull << a;
      depth++;
    }
    const size_t r = (size_t)b * rows + 1 + j;
    v_pos[r] = nb - 1 + depth;
    v_slot[r] = nb + j;
    v_mask[r] = m;
  }
}

// Greedy acceptance along the tree: from the root, follow the child whose token equals the target's argmax at
// the current row; emit the accepted tokens and the target's token at the last accepted row. acc_node gets
// the accepted node indices (depth order), -1 past the end.
__global__ void tree_accept_kernel(const int* __restrict__ argmax, const int* __restrict__ v_tok, int B, TreeShape t,
                                   int* __restrict__ out_tokens, int* __restrict__ out_count, int* __restrict__ acc_node) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int rows = 1 + t.total;
  const int* am = argmax + (size_t)b * rows;
  const int* tok = v_tok + (size_t)b * rows;
  int row = 0, depth = 0, child0 = t.first[0], nchild = t.count[0];
  while (depth < t.levels) {
    const int want = am[row];
    int hit = -1;
    for (int c = 0; c < nchild; c++)
      if (tok[1 + child0 + c] == want) {
        hit = child0 + c;
        break;
      }
    if (hit < 0) break;
    out_tokens[(size_t)b * (t.levels + 1) + depth] = want;
    acc_node[(size_t)b * t.levels + depth] = hit;
    depth++;
    row = 1 + hit;
    if (depth < t.levels) {
      nchild = t.branch[depth];
      child0 = t.first[depth] + (hit - t.first[depth - 1]) * nchild;
    }
  }
  out_tokens[(size_t)b * (t.levels + 1) + depth] = am[row];
  out_count[b] = depth + 1;
  for (int d = depth; d < t.levels; d++) acc_node[(size_t)b * t.levels + d] = -1;
}

// Move the accepted nodes' K/V (tree slots tbase + node) to the committed slots tbase + depth, for every layer
// and kv head; depths in order (a destination never holds a deeper accepted node: tbase + d < first node of
// level d + 1). Nodes deeper than max_depth are skipped (the draft model never computed the leaves).
__global__ void tree_compact_kernel(uint16_t* __restrict__ kc, uint16_t* __restrict__ vc, long long layer_stride,
                                    const int* __restrict__ page_table, int max_pages, const int* __restrict__ tbase,
                                    const int* __restrict__ acc_node, int levels, int max_depth, int Hkv, int D) {
  pdl_wait();
  pdl_trigger();
  const int layer = blockIdx.x, head = blockIdx.y, b = blockIdx.z;
  const int base = tbase[b];
  uint16_t* K = kc + (size_t)layer * layer_stride;
  uint16_t* Vv = vc + (size_t)layer * layer_stride;
  for (int d = 0; d < levels && d < max_depth; d++) {
    const int node = acc_node[(size_t)b * levels + d];
    if (node < 0) break;
    const int src = base + node, dst = base + d;
    if (src != dst) {
      const int ps = page_table[(size_t)b * max_pages + (src >> 4)], pd = page_table[(size_t)b * max_pages + (dst >> 4)];
      const size_t os = (((size_t)ps * Hkv + head) * 16 + (src & 15)) * D;
      const size_t od = (((size_t)pd * Hkv + head) * 16 + (dst & 15)) * D;
      for (int i = threadIdx.x; i < D; i += blockDim.x) {
        K[od + i] = K[os + i];
        Vv[od + i] = Vv[os + i];
      }
    }
    __syncthreads();
  }
}

static int tree_shape(const int32_t* branch, int64_t levels, TreeShape* t) {
  IM_REQUIRE(branch && levels >= 1 && levels <= TR_MAX_LEVELS, IM_INVALID, "tree: 1 to %d levels", TR_MAX_LEVELS);
  *t = TreeShape{};
  t->levels = (int)levels;
  int count = 1, first = 0;
  for (int L = 0; L < levels; L++) {
    IM_REQUIRE(branch[L] >= 1 && branch[L] <= TK_MAX, IM_INVALID, "tree: branching 1 to %d", TK_MAX);
    t->branch[L] = branch[L];
    count *= branch[L];
    t->count[L] = count;
    t->first[L] = first;
    first += count;
  }
  t->total = first;
  IM_REQUIRE(t->total <= TR_MAX_NODES, IM_UNSUPPORTED, "tree: %d nodes (at most %d)", t->total, TR_MAX_NODES);
  return IM_OK;
}

}  // namespace im

using namespace im;

extern "C" size_t im_topk_workspace_bytes(int64_t rows, int64_t V, int64_t k) {
  if (rows < 1 || V < 1 || k < 1 || k > TK_MAX) return 0;
  const int64_t chunks = (V + TK_CHUNK - 1) / TK_CHUNK;
  return (size_t)((rows * 4 + 255) / 256) * 256 + (size_t)rows * chunks * TK_MAX * sizeof(TkCand);
}

extern "C" int im_topk_rows(const uint16_t* logits, int64_t rows, int64_t V, int64_t ld, int64_t k, int32_t* out,
                            int64_t out_stride, void* workspace, size_t workspace_bytes, void* stream) {
  clear_error();
  IM_REQUIRE(rows >= 1 && rows <= 65535 && V >= 1 && V < (1ll << 31) && ld >= V && k >= 1 && k <= TK_MAX &&
                 out_stride >= k,
             IM_INVALID, "im_topk_rows: bad sizes");
  IM_REQUIRE(logits && out && workspace, IM_INVALID, "im_topk_rows: null pointer");
  IM_REQUIRE(aligned(workspace, 256), IM_INVALID, "im_topk_rows: workspace must be 256-byte aligned");
  const size_t need = im_topk_workspace_bytes(rows, V, k);
  IM_REQUIRE(workspace_bytes >= need, IM_INVALID, "im_topk_rows: workspace of %zu bytes needed", need);
  const int chunks = (int)((V + TK_CHUNK - 1) / TK_CHUNK);
  // counters first (kept at zero between launches), then the chunk lists
  unsigned* counters = reinterpret_cast<unsigned*>(workspace);
  TkCand* part = reinterpret_cast<TkCand*>(reinterpret_cast<char*>(workspace) + ((rows * 4 + 255) / 256) * 256);
  dim3 grid(chunks, (unsigned)rows);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (k) {
#define IM_TK(KK) \
  case KK: return launch("topk_kernel", topk_kernel<KK>, grid, dim3(TK_THREADS), 0, st, logits, (int)V, (long long)ld, chunks, out, (int)out_stride, part, counters);
    IM_TK(1) IM_TK(2) IM_TK(3) IM_TK(4) IM_TK(5) IM_TK(6) IM_TK(7) IM_TK(8)
#undef IM_TK
    default: return IM_INVALID;
  }
}

extern "C" int im_tree_prepare(const int32_t* hist, int64_t cap, const int32_t* n, int64_t B, const int32_t* branch,
                               int64_t levels, int64_t slot_cap, int32_t* d0_tok, int32_t* d0_pos, int32_t* v_tok,
                               int32_t* v_pos, int32_t* v_slot, uint64_t* v_mask, int32_t* tree_base, void* stream) {
  clear_error();
  TreeShape t;
  int rc = tree_shape(branch, levels, &t);
  if (rc) return rc;
  IM_REQUIRE(B >= 1 && cap >= 2 && slot_cap >= t.total + 2, IM_INVALID, "im_tree_prepare: bad sizes");
  IM_REQUIRE(hist && n && d0_tok && d0_pos && v_tok && v_pos && v_slot && v_mask && tree_base, IM_INVALID,
             "im_tree_prepare: null pointer");
  return launch("tree_prepare_kernel", tree_prepare_kernel, dim3((unsigned)B), dim3(64), 0,
                reinterpret_cast<cudaStream_t>(stream), hist, (int)cap, n, (int)B, t, (int)slot_cap, d0_tok, d0_pos,
                v_tok, v_pos, v_slot, reinterpret_cast<unsigned long long*>(v_mask), tree_base);
}

extern "C" int im_tree_accept(const int32_t* argmax, const int32_t* v_tok, int64_t B, const int32_t* branch,
                              int64_t levels, int32_t* out_tokens, int32_t* out_count, int32_t* acc_node,
                              void* stream) {
  clear_error();
  TreeShape t;
  int rc = tree_shape(branch, levels, &t);
  if (rc) return rc;
  IM_REQUIRE(B >= 1 && argmax && v_tok && out_tokens && out_count && acc_node, IM_INVALID,
             "im_tree_accept: bad arguments");
  return launch("tree_accept_kernel", tree_accept_kernel, dim3((unsigned)((B + 63) / 64)), dim3(64), 0,
                reinterpret_cast<cudaStream_t>(stream), argmax, v_tok, (int)B, t, out_tokens, out_count, acc_node);
}

extern "C" int im_tree_compact(uint16_t* k_cache, uint16_t* v_cache, int64_t layers, int64_t layer_stride,
                               const int32_t* page_table, int64_t max_pages, const int32_t* tree_base,
                               const int32_t* acc_node, int64_t levels, int64_t max_depth, int64_t B, int64_t Hkv,
                               int64_t D, void* stream) {
  clear_error();
  IM_REQUIRE(layers >= 1 && layer_stride >= 1 && B >= 1 && Hkv >= 1 && D >= 1 && D <= 1024 && levels >= 1 &&
                 levels <= TR_MAX_LEVELS && max_depth >= 0,
             IM_INVALID, "im_tree_compact: bad sizes");
  IM_REQUIRE(k_cache && v_cache && page_table && tree_base && acc_node, IM_INVALID, "im_tree_compact: null pointer");
  if (max_depth == 0) return IM_OK;
  return launch("tree_compact_kernel", tree_compact_kernel, dim3((unsigned)layers, (unsigned)Hkv, (unsigned)B),
                dim3(128), 0, reinterpret_cast<cudaStream_t>(stream), k_cache, v_cache, (long long)layer_stride,
                page_table, (int)max_pages, tree_base, acc_node, (int)levels, (int)max_depth, (int)Hkv, (int)D);
}
