// On-device bookkeeping of a speculative round, so that a whole draft -> verify -> accept round is a fixed
// sequence of launches (capturable in one CUDA graph) that never returns to the host.
//
// Replaces the host loop of IronMule ironmule/ggml_engine.py:1155-1343 (build `[last] + drafts` rows per
// request, decode, accept, roll the KV back with llama_memory_seq_rm at :1340) and the draft model's slot
// bookkeeping of ironmule/draft_model.py:203-274 (catch-up of new tokens, one draft row per call, trimming
// on rejection) for a fixed draft length k.
//
// Per sequence b the device holds the committed tokens hist[b][0..n_b) and n_b. Both models' KV caches hold
// slots 0..n_b-2; the last committed token is fed again at the start of each round. A round:
//   prepare:  draft pass 0 rows = (hist[n-2] @ n-2, hist[n-1] @ n-1) -- the first re-feeds a slot whose KV
//             is already right (same token, same prefix) so the pass always has two rows, whatever was
//             accepted last round; draft pass i (1..k-1) row = (d_i @ n-1+i); verify rows =
//             (hist[n-1] @ n-1, d_1 @ n, ..., d_k @ n-1+k). The draft tokens d_i are written straight into
//             the verify row buffer by the argmax of the draft passes.
//   commit:   append the accepted tokens (verify_greedy / stochastic acceptance output) to hist and
//             advance n. KV rollback needs no work: attention reads each row's slots up to its own
//             position, and the stale slots past n are rewritten by the next round.
// Sequences that reached their target length stop committing; their rows are still computed (the round has
// a fixed shape) on clamped positions.
#include "common.cuh"

namespace im {

__global__ void spec_prepare_kernel(const int* __restrict__ hist, int cap, const int* __restrict__ n,
                                    const int* __restrict__ target, int B, int k, int slot_cap,
                                    int* __restrict__ d0_tok, int* __restrict__ d0_pos, int* __restrict__ d_pos,
                                    int* __restrict__ v_tok, int* __restrict__ v_pos) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  int nb = n[b];
  nb = max(2, min(nb, min(cap, slot_cap - k)));  // keep every slot of the round inside the cache
  const int* h = hist + (size_t)b * cap;
  d0_tok[2 * b] = h[nb - 2];
  d0_tok[2 * b + 1] = h[nb - 1];
  d0_pos[2 * b] = nb - 2;
  d0_pos[2 * b + 1] = nb - 1;
  for (int i = 1; i < k; i++) d_pos[(size_t)(i - 1) * B + b] = nb - 1 + i;
  v_tok[(size_t)b * (k + 1)] = h[nb - 1];
  for (int j = 0; j <= k; j++) v_pos[(size_t)b * (k + 1) + j] = nb - 1 + j;
  (void)target;
}

__global__ void spec_commit_kernel(int* __restrict__ hist, int cap, int* __restrict__ n,
                                   const int* __restrict__ target, int B, int k, const int* __restrict__ out_tokens,
                                   const int* __restrict__ out_count, long long* __restrict__ stats) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int nb = n[b];
  if (nb >= target[b]) return;
  const int c = out_count[b];
  int* h = hist + (size_t)b * cap;
  int put = 0;
  for (int j = 0; j < c && nb + j < cap; j++, put++) h[nb + j] = out_tokens[(size_t)b * (k + 1) + j];
  n[b] = nb + put;
  if (stats) {
    stats[3 * b] += 1;          // rounds
    stats[3 * b + 1] += put;    // tokens committed
    stats[3 * b + 2] += c - 1;  // drafts accepted
  }
}

}  // namespace im

using namespace im;

extern "C" int im_spec_prepare(const int32_t* hist, int64_t cap, const int32_t* n, const int32_t* target, int64_t B,
                               int64_t k, int64_t slot_cap, int32_t* d0_tok, int32_t* d0_pos, int32_t* d_pos,
                               int32_t* v_tok, int32_t* v_pos, void* stream) {
  clear_error();
  IM_REQUIRE(B >= 1 && k >= 1 && cap >= 2 && slot_cap >= k + 2, IM_INVALID, "im_spec_prepare: bad sizes");
  IM_REQUIRE(hist && n && target && d0_tok && d0_pos && v_tok && v_pos && (k == 1 || d_pos), IM_INVALID,
             "im_spec_prepare: null pointer");
  const int threads = 128;
  return launch("spec_prepare_kernel", spec_prepare_kernel, dim3((unsigned)((B + threads - 1) / threads)), dim3(threads),
                0, reinterpret_cast<cudaStream_t>(stream), hist, (int)cap, n, target, (int)B, (int)k, (int)slot_cap,
                d0_tok, d0_pos, d_pos, v_tok, v_pos);
}

extern "C" int im_spec_commit(int32_t* hist, int64_t cap, int32_t* n, const int32_t* target, int64_t B, int64_t k,
                              const int32_t* out_tokens, const int32_t* out_count, int64_t* stats, void* stream) {
  clear_error();
  IM_REQUIRE(B >= 1 && k >= 0 && cap >= 1, IM_INVALID, "im_spec_commit: bad sizes");
  IM_REQUIRE(hist && n && target && out_tokens && out_count, IM_INVALID, "im_spec_commit: null pointer");
  const int threads = 128;
  return launch("spec_commit_kernel", spec_commit_kernel, dim3((unsigned)((B + threads - 1) / threads)), dim3(threads),
                0, reinterpret_cast<cudaStream_t>(stream), hist, (int)cap, n, target, (int)B, (int)k, out_tokens,
                out_count, reinterpret_cast<long long*>(stats));
}
