/*
 * libimspec -- B200 (sm_100a) kernels for IronMule's speculative-decoding hot path, behind a C ABI.
 *
 * Conventions (modelled on the reference's own native hook, IronMule ironmule/kernel_gen.py:803-862):
 *  - every pointer is a caller-owned device pointer unless a comment says otherwise; sizes are int64;
 *  - bf16 values are passed as uint16_t bit patterns, 4-bit weights as uint32_t words (8 codes, low
 *    nibble first), MLX-affine with group size 64: w = scale * q + bias;
 *  - `stream` is a cudaStream_t (NULL = the legacy default stream); every call is stream-ordered and
 *    returns without synchronising;
 *  - the return value is IM_OK (0) when the work was enqueued, non-zero otherwise; nothing is launched
 *    on a non-zero return, and im_last_error() describes why (thread-local). No C++ exception crosses
 *    the boundary.
 */
#ifndef IMSPEC_H
#define IMSPEC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IM_ABI_VERSION 1

enum {
  IM_OK = 0,
  IM_UNSUPPORTED = 1, /* a shape or mode this build does not handle */
  IM_INVALID = 2,     /* null pointer, bad size or misaligned buffer */
  IM_CUDA_ERROR = 3   /* a CUDA runtime error (message from cudaGetErrorString) */
};

/* qGEMM epilogues */
enum {
  IM_EPI_STORE = 0,    /* y = bf16(acc) */
  IM_EPI_RESIDUAL = 1, /* y = bf16(residual + bf16(acc)); residual may alias y */
  IM_EPI_SWIGLU = 2,   /* rows come as 16 gate rows then the matching 16 up rows; y[m, N/2] = silu(gate)*up */
  IM_EPI_GEGLU = 3     /* as SWIGLU with gelu_approx(gate)*up (Gemma-3) */
};

/* qGEMM kernel variants */
enum {
  IM_QGEMM_AUTO = 0, /* the warp-MMA kernel */
  IM_QGEMM_MMA = 1,  /* warp-level bf16 tensor-core MMA on exact 4-bit codes, M <= 32 */
  IM_QGEMM_FMA = 2   /* CUDA-core FMA with warp-shuffle reduction, M <= 8 */
};

/* The ABI revision this library implements (IM_ABI_VERSION). */
int im_abi_version(void);
/* Decode-path kernels (the packed qGEMM, embedding, q/k norm + RoPE, attention, argmax/verify, sampling and
 * the round bookkeeping) are launched with programmatic dependent launch: a kernel's CTAs may start while the
 * previous kernel on the stream runs, load weights, and wait for the previous kernel's results before reading
 * activations. Results are the same either way. on = 0 turns this off process-wide; returns the previous
 * setting. */
int im_set_launch_overlap(int on);

/* The message of the last non-zero return on this thread ("" when the last call succeeded). */
const char* im_last_error(void);

/*
 * y[M, N] = x[M, K] . dequantize(w, scales, biases)[N, K]^T, bf16 in and out, float32 accumulation.
 * w uint32 [N, K/8] (16-byte aligned), scales/biases bf16 [N, K/64], x bf16 [M, K] (16-byte aligned),
 * y bf16 [M, N]. K % 64 == 0, 1 <= M <= 32. Row-invariant: a row of x gets the same bits whatever M is.
 * Replaces the reference's qmv kernels and their `run` dispatchers:
 *   ironmule/qmv_k3840.py:299-310 (run), ironmule/qmv_shared.py:169-181 (run_shared),
 *   ironmule/qmv_fast_shared.py:161-172 (run_fast), ironmule/qmv_variant.py:116-129,
 *   and the library fallback mx.quantized_matmul at ironmule/qmv_k3840.py:336-339.
 */
int im_qgemm_w4g64(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const uint16_t* x,
                   uint16_t* y, int64_t M, int64_t N, int64_t K, void* stream);

/*
 * im_qgemm_w4g64 with a fused epilogue (IM_EPI_*), a kernel variant (IM_QGEMM_*) and an optional
 * workspace that lets CTAs split K (more parallelism for small N). `workspace` must be 256-byte aligned,
 * at least im_qgemm_workspace_bytes(M, N, K) bytes and zero-filled before its first use; the kernel
 * leaves it zeroed. Calls that share one workspace must not overlap on the GPU. With workspace == NULL
 * the CTAs do not split K. The gated epilogues write y[M, N/2].
 * Same reference interfaces as im_qgemm_w4g64, plus the fused decode-layer math of
 * ironmule/paired_research.py:177-215 (residual adds, GeGLU) and mlx_lm's Qwen3 SwiGLU.
 */
int im_qgemm_w4g64_ex(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const uint16_t* x,
                      uint16_t* y, const uint16_t* residual, int64_t M, int64_t N, int64_t K, int epilogue,
                      int variant, void* workspace, size_t workspace_bytes, void* stream);

/*
 * im_qgemm_w4g64 for callers that cannot allocate device memory (an engine that owns all device memory through
 * its own pool, a plugin that may not call cudaMalloc or synchronise on its decode path). No reference
 * counterpart: it is an addition of this library. It splits K across CTAs with the same plan as
 * im_qgemm_w4g64_ex given a workspace (so the results are bit-identical), keeping the scratch in one static
 * device array of im_qgemm_noalloc_capacity() bytes that every GPU loading the library holds until exit.
 * Shapes whose scratch would exceed it return IM_UNSUPPORTED. The first call on a device looks the array up and
 * queues the zeroing of its counters on the caller's stream, ahead of its kernel; make it before any stream
 * capture. Calls share the array: calls that overlap on the GPU race and must not be issued.
 */
int im_qgemm_w4g64_noalloc(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, const uint16_t* x,
                           uint16_t* y, int64_t M, int64_t N, int64_t K, void* stream);
size_t im_qgemm_noalloc_capacity(void);

/* Workspace bytes im_qgemm_w4g64_ex needs for this shape (0: it does not split K). */
size_t im_qgemm_workspace_bytes(int64_t M, int64_t N, int64_t K);

/* Sweep hook: force the CTA-level K split (0 restores the automatic choice). Process-wide. */
int im_qgemm_set_splits(int splits);

/*
 * qGEMM v4 over weights repacked once into MMA-fragment order (the engine's resident format).
 * im_qgemm_pack_w4g64 converts MLX-layout w/scales/biases [N, K] into `packed` (16-byte aligned,
 * im_qgemm_packed_bytes(N, K) bytes): rows padded to 32-row tiles, one contiguous 1152-byte unit per
 * (tile, 64-group) holding that tile's codes in lane order and its 32 scales/biases.
 * im_qgemm_packed computes the same product and epilogues as im_qgemm_w4g64_ex from it for M <= 320 rows (every
 * row exactly as a call of at most 32 rows computes it, on the warp MMA in 32-row chunks or on the tcgen05
 * tensor cores with the same k-steps and fp32 order, activations staged as tiles in the workspace),
 * and can fuse the RMSNorm that precedes a
 * projection: with norm_weight != NULL, x is the raw residual stream and each row is normalised on the way in
 * (x * 1/sqrt(sum(x^2)/K + eps) * w', w' = w or 1 + w when gemma_norm), its sum of squares taken from
 * norm_sq[p * sq_ld + m] summed over p < norm_parts (per-tile partial sums). With out_sq != NULL, a
 * store/residual epilogue writes those per-tile partial sums of its own output rows (out_sq[tile * sq_ld + m],
 * ceil(N/32) tiles) for the next normalised GEMM. sq_ld = 0 means M rounded up to 32. workspace >= im_qgemm_packed_workspace_bytes(M, N, K)
 * (256-byte aligned, zero-filled before first use) when that is non-zero; calls sharing it must not overlap.
 * Replaces the same reference interfaces as im_qgemm_w4g64, plus the RMSNorm before each projection of the
 * decode layer (ironmule/paired_research.py:177-215).
 */
size_t im_qgemm_packed_bytes(int64_t N, int64_t K);
int im_qgemm_pack_w4g64(const uint32_t* w, const uint16_t* scales, const uint16_t* biases, int64_t N, int64_t K,
                        void* packed, void* stream);
size_t im_qgemm_packed_workspace_bytes(int64_t M, int64_t N, int64_t K);
/* Tuning hook of the K-split policy: a forced split (0 = automatic), the most CTAs the automatic policy fills
 * (default 592: one wave at four CTAs per SM) and its largest split. Process-wide; changes workspace sizes, so set
 * it before sizing workspaces. */
int im_qgemm_packed_tune(int split_override, int target_ctas, int max_split);
/* Kernel choice: 0 (default) = automatic (tcgen05 tensor cores from 128 rows when the K split is at most 16, the
 * warp MMA otherwise), 1 = warp MMA always, 2 = tensor cores always. Process-wide; every choice gives the same
 * bits; changes workspace sizes, so set it before sizing workspaces. */
int im_qgemm_packed_path(int path);
/* Split-K reduction of the warp-MMA kernel: 1 (default) = the K splits of a CTA column run as one thread-block
 * cluster and their partials are summed through distributed shared memory (when the device can schedule the
 * cluster), 0 = through the workspace and a global arrival counter. Process-wide; both give the same bits. */
int im_qgemm_packed_cluster(int on);
/* The error word of a workspace last used by a call of more than 32 rows (the tensor-core kernel): 0 when
 * every bounded wait of that kernel completed, 1 when one ran out. Synchronous (reads device memory). */
int im_qgemm_packed_status(const void* workspace);
int im_qgemm_packed(const void* packed, const uint16_t* x, uint16_t* y, const uint16_t* residual, int64_t M, int64_t N,
                    int64_t K, int epilogue, const float* norm_sq, int64_t norm_parts, const uint16_t* norm_weight,
                    float eps, int gemma_norm, float* out_sq, int64_t sq_ld, void* workspace, size_t workspace_bytes,
                    void* stream);
/*
 * The o-projection fused with the attention's split merge: im_qgemm_packed's residual epilogue
 * (y = residual + x . W^T, out_sq as there) where x, the attention output [M][Hq * D], is merged in the
 * prologue from the split partials that im_attention_qkv_paged left in attn_workspace when called with
 * out = NULL (same B, max_rows_per_seq, Hq, Hkv, D, max_kv_len, keys_per_split and seq_rows; row_slot is that
 * call's row_slot). Row r merges splits [0, row_slot[r] / keys_per_split + 1) with the attention's own merge
 * arithmetic: the same bits as merging in the attention and calling im_qgemm_packed. Takes
 * M <= im_qgemm_packed_attn_rows(N, K) rows (0: the shape has no fused form); K = Hq * D.
 */
int64_t im_qgemm_packed_attn_rows(int64_t N, int64_t K);
int im_qgemm_packed_attn(const void* packed, const void* attn_workspace, const int32_t* seq_rows,
                         const int32_t* row_slot, int64_t B, int64_t max_rows_per_seq, int64_t Hq, int64_t Hkv,
                         int64_t D, int64_t max_kv_len, int64_t keys_per_split, uint16_t* y, const uint16_t* residual,
                         int64_t M, int64_t N, int64_t K, float* out_sq, int64_t sq_ld, void* workspace,
                         size_t workspace_bytes, void* stream);

/*
 * Row statistics over a logits matrix: for each row r of logits[rows, V] (bf16, row stride ld elements)
 * writes argmax[r * argmax_stride] (lowest index among equal maxima) and, if conf != NULL, the top-1 probability
 * conf[r] = 1 / sum_v exp(l_v - l_max). Replaces the host numpy scan of
 * ironmule/ggml_engine.py:669-683 (_decode_conf) and the per-row argmax at ggml_engine.py:848.
 * `workspace` >= im_argmax_workspace_bytes(rows, V) bytes, 256-byte aligned, zero-filled before first use.
 */
int im_argmax_rows(const uint16_t* logits, int64_t rows, int64_t V, int64_t ld, int32_t* argmax,
                   int64_t argmax_stride, float* conf, void* workspace, size_t workspace_bytes, void* stream);
size_t im_argmax_workspace_bytes(int64_t rows, int64_t V);

/*
 * Greedy verification of B sequences with k drafts each, in one launch: argmax over each of the
 * B*(k+1) logits rows (row b*(k+1)+i scores the token after draft i-1), then per sequence the drafts the
 * target agrees with followed by the target's own next token -- IronMule's `accept`
 * (ironmule/speculation.py:103-108) applied to the argmax of ironmule/ggml_engine.py:1316-1332.
 * drafts int32 [B, k] with row stride drafts_ld; out_tokens int32 [B, k+1] (entries past out_count[b] are -1);
 * out_count int32 [B] (1..k+1); argmax_out int32 [B*(k+1)] may be NULL.
 * `workspace` as for im_argmax_rows with rows = B*(k+1).
 */
int im_verify_greedy(const uint16_t* logits, int64_t B, int64_t k, int64_t V, int64_t ld, const int32_t* drafts,
                     int64_t drafts_ld, int32_t* out_tokens, int32_t* out_count, int32_t* argmax_out, void* workspace,
                     size_t workspace_bytes, void* stream);

/*
 * MLX-affine 4-bit quantisation of bf16 weights w[N, K] (16-byte aligned), group 64: scale = bf16((max-min)/15),
 * bias = bf16(min), q = clamp(rint((w - bias)/scale), 0, 15); writes wq uint32 [N, K/8] (low nibble first),
 * scales/biases bf16 [N, K/64]. The format nn.QuantizedLinear.from_linear produces for the reference
 * (tests/runtime/test_qmv_k3840_integration.py:17-21; layout checked at ironmule/qmv_k3840.py:379-408).
 */
int im_quantize_w4g64(const uint16_t* w, int64_t N, int64_t K, uint32_t* wq, uint16_t* scales, uint16_t* biases,
                      void* stream);

/*
 * RMSNorm over rows (input row stride ldx elements, output rows contiguous):
 * out[m, :] = bf16((x[m, :] * inv_rms) * w'), inv_rms = 1/sqrt(mean(x^2) + eps), with
 * w' = weight (gemma_style = 0, Qwen3) or 1 + weight (gemma_style = 1, Gemma-3). One fixed reduction order per
 * row. The norms of the verify forward: ironmule/paired_research.py:177-215 (Gemma-3 pre/post norms) and
 * mlx_lm's Qwen3 input/post-attention/final norms called from ironmule/runtime.py:505-545.
 */
int im_rmsnorm(const uint16_t* x, int64_t ldx, const uint16_t* weight, uint16_t* out, int64_t M, int64_t H,
               float eps, int gemma_style, void* stream);
/*
 * Gemma-3's post-attention / post-feedforward norm fused with its residual add: per row m < M,
 * h[m] = bf16(h[m] + bf16((y[m] * inv_rms(y[m])) * w')), w' = 1 + weight (gemma_style) or weight, and, when
 * out_sq != NULL, out_sq[m] = the sum of squares of the new h[m] for the RMSNorm that the next
 * im_qgemm_packed fuses (norm_parts = 1). y, h [M, H] bf16. weight == NULL: the plain residual add
 * h[m] = bf16(h[m] + y[m]) (after an all-reduce of tensor-parallel partial projections). Replaces the post_attention_layernorm /
 * post_feedforward_layernorm steps of the Gemma-3 decode layer (ironmule/paired_research.py:177-215).
 */
int im_rmsnorm_residual(const uint16_t* y, const uint16_t* weight, uint16_t* h, int64_t M, int64_t H, float eps,
                        int gemma_style, float* out_sq, void* stream);

/*
 * The per-head step between the qkv projection and attention, fused: for each row m of the packed projection
 * qkv[M, (Hq + 2 Hkv) D] (q heads, then k heads, then v heads): q/k RMSNorm over D (q_norm, k_norm; 1 + w when
 * gemma_style), non-interleaved RoPE at row_pos[m] with angle = pos * inv_freq[i] (inv_freq float [D/2]),
 * q -> q_out[M, Hq, D]; k and v -> the paged caches [pages][Hkv][16][D] at slot row_slot[m] of sequence
 * row_seq[m] (page = page_table[seq * max_pages + slot / 16]). D is 128 or 256.
 * Reference: the q/k norm + RoPE of ironmule/paired_research.py:177-215 and ironmule/dense_plan.py:365-370,
 * and the KV slot writes of the stacked plan's forward, ironmule/dense_plan.py:337-363.
 */
int im_qk_norm_rope_kv(const uint16_t* qkv, const uint16_t* q_norm, const uint16_t* k_norm, const float* inv_freq,
                       const int32_t* row_pos, const int32_t* row_slot, const int32_t* row_seq,
                       const int32_t* page_table, int64_t max_pages, int64_t M, int64_t Hq, int64_t Hkv, int64_t D,
                       float eps, int gemma_style, uint16_t* q_out, uint16_t* k_cache, uint16_t* v_cache,
                       void* stream);

/*
 * Embedding gather from a 4-bit table: out[m, :] = bf16(scale * q + bias) of row tokens[m * tokens_stride] (int32;
 * clamped to [0, V)), times bf16(mult) when mult != 1 (Gemma-3 scales by sqrt(hidden)); out_sq (M floats, may
 * be NULL) receives each row's sum of squares, the norm_sq input of a fused-RMSNorm im_qgemm_packed. The tied table
 * doubles as the LM head through im_qgemm_w4g64 (nn.QuantizedEmbedding / as_linear,
 * ironmule/cuda_native.py:227-229).
 */
int im_embed_w4g64(const int32_t* tokens, int64_t tokens_stride, const uint32_t* wq, const uint16_t* scales,
                   const uint16_t* biases, int64_t M, int64_t V, int64_t H, float mult, uint16_t* out, float* out_sq,
                   void* stream);

/*
 * Paged verification attention: out[M, Hq, D] for q[M, Hq, D] whose rows are grouped by sequence (rows of
 * sequence b are seq_rows[b] .. seq_rows[b+1]-1, int32 [B+1]); row r sees the KV slots s <= row_slot[r] of its
 * sequence (causal verify mask), also s > row_slot[r] - window when window > 0 (sliding window), and, when
 * tree_mask != NULL, a slot s >= tree_base[b] only if bit (s - tree_base[b]) of tree_mask[r] is set (draft
 * tree). GQA with Hq/Hkv query heads per KV head; scores scaled by `scale`; softmax in float32.
 * KV keys are split at fixed absolute multiples of keys_per_split (a multiple of 64) -- keep it fixed for a
 * model so a row's bits never depend on the launch. max_kv_len bounds every sequence's kv length (the grid
 * size; larger slots are not read). `workspace` >= im_attention_workspace_bytes(...), 256-byte aligned,
 * zero-filled before first use; calls sharing it must not overlap on the GPU.
 * Replaces FA2 partial + combine of ironmule/dense_plan.py:111-195, :258-274 (causal by per-row length,
 * :345) and the sliding-window Gemma form of ironmule/dense_gemma.py:47-300.
 */
int im_attention_paged(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                       const int32_t* page_table, int64_t max_pages, const int32_t* seq_rows, const int32_t* seq_slot,
                       const int32_t* row_slot,
                       const uint64_t* tree_mask, const int32_t* tree_base, int64_t B, int64_t max_rows_per_seq,
                       int64_t Hq, int64_t Hkv, int64_t D, int64_t max_kv_len, int64_t keys_per_split, int64_t window,
                       float scale, uint16_t* out, void* workspace, size_t workspace_bytes, void* stream);
size_t im_attention_workspace_bytes(int64_t B, int64_t max_rows_per_seq, int64_t Hq, int64_t Hkv, int64_t D,
                                    int64_t max_kv_len, int64_t keys_per_split);
/* Tuning hook of the attention launch: the waves of resident CTAs it aims for when it gives a (sequence,
 * kv head) group several CTAs. Process-wide; scheduling only -- every result is the same at any value. */
int im_attention_tune(int waves);
/*
 * The same attention starting from the packed projection rows qkv [M, (Hq + 2 Hkv) D] (q heads, k heads,
 * v heads): q and the new keys get RMSNorm (q_norm / k_norm; w or 1 + w when gemma_style) and RoPE at
 * row_pos[r] inside the kernel -- bit-identical to im_qk_norm_rope_kv followed by im_attention_paged -- and
 * every row's K and V are written to the caches at row_slot[r] of its sequence's pages. At most 32 rows
 * per sequence. Replaces the q/k norm, RoPE and cache write of the decode step together with its
 * attention (ironmule/paired_research.py:177-215, ironmule/dense_plan.py:337-370 then :111-195, :258-274).
 * With out = NULL the kernel only writes the split partials into the workspace and leaves their merge to
 * im_qgemm_packed_attn.
 */
int im_attention_qkv_paged(const uint16_t* qkv, const uint16_t* q_norm, const uint16_t* k_norm,
                           const float* inv_freq, const int32_t* row_pos, float eps, int gemma_style,
                           uint16_t* k_cache, uint16_t* v_cache, const int32_t* page_table, int64_t max_pages,
                           const int32_t* seq_rows, const int32_t* seq_slot, const int32_t* row_slot,
                           const uint64_t* tree_mask, const int32_t* tree_base, int64_t B, int64_t max_rows_per_seq,
                           int64_t Hq, int64_t Hkv, int64_t D, int64_t max_kv_len, int64_t keys_per_split,
                           int64_t window, float scale, uint16_t* out, void* workspace, size_t workspace_bytes,
                           void* stream);

/*
 * Tree speculation (the reference's speculation is linear, ironmule/speculation.py:39-108,
 * so these have no reference counterpart beyond its greedy rule). The tree has `levels` levels below the root
 * with branching branch[0..levels-1] (total nodes <= 63), nodes numbered level by level, children of a node
 * consecutive. Node j of a sequence with n committed tokens sits in KV slot n + j (tree_base[b] = n) at RoPE
 * position n - 1 + depth(j); verify row 0 is the root (slot n - 1), row 1 + j node j, with tree_mask bits of the
 * node's ancestors and itself (im_attention_paged's tree mode).
 *
 * im_topk_rows: the k (<= 8) largest of each row (ties: lower index first; NaN lowest), row r's indices at
 * out[r * out_stride ..]; workspace >= im_topk_workspace_bytes, 256-byte aligned, zero-filled once.
 * im_tree_prepare: the first draft pass's two re-fed rows (d0_*) and the verify rows' slot, position, mask
 * (v_*, [B][1 + nodes]; v_tok[b][0] = the root token, node tokens come from im_topk_rows) and tree_base.
 * im_tree_accept: from the target's argmax of each verify row, the longest path whose node tokens equal the
 * argmax of their parent's row, then the target's token there: out_tokens [B][levels + 1], out_count [B],
 * acc_node [B][levels] (accepted node per depth, -1 after).
 * im_tree_compact: copies the accepted nodes' K/V (depth < max_depth) to slots tree_base + depth, for every layer
 * of a [layers][pages][Hkv][16][D] cache (layer_stride elements apart).
 */
size_t im_topk_workspace_bytes(int64_t rows, int64_t V, int64_t k);
int im_topk_rows(const uint16_t* logits, int64_t rows, int64_t V, int64_t ld, int64_t k, int32_t* out,
                 int64_t out_stride, void* workspace, size_t workspace_bytes, void* stream);
int im_tree_prepare(const int32_t* hist, int64_t cap, const int32_t* n, int64_t B, const int32_t* branch,
                    int64_t levels, int64_t slot_cap, int32_t* d0_tok, int32_t* d0_pos, int32_t* v_tok, int32_t* v_pos,
                    int32_t* v_slot, uint64_t* v_mask, int32_t* tree_base, void* stream);
int im_tree_accept(const int32_t* argmax, const int32_t* v_tok, int64_t B, const int32_t* branch, int64_t levels,
                   int32_t* out_tokens, int32_t* out_count, int32_t* acc_node, void* stream);
int im_tree_compact(uint16_t* k_cache, uint16_t* v_cache, int64_t layers, int64_t layer_stride,
                    const int32_t* page_table, int64_t max_pages, const int32_t* tree_base, const int32_t* acc_node,
                    int64_t levels, int64_t max_depth, int64_t B, int64_t Hkv, int64_t D, void* stream);

/*
 * Device bookkeeping of one speculative round with k drafts for B sequences (no host round trip).
 * hist int32 [B, cap] holds each sequence's committed tokens, n int32 [B] their count, target int32 [B] the
 * length at which a sequence stops committing; slot_cap = pages * 16 bounds every KV slot.
 * im_spec_prepare fills the round's row buffers: d0_tok/d0_pos [B*2] (draft pass 0: the last two committed
 * tokens), d_pos [(k-1), B] (draft pass i at slot n-1+i), v_tok/v_pos [B*(k+1)] (verify rows: the last
 * committed token then the k drafts, which the draft passes' argmax writes into v_tok[b*(k+1)+i]).
 * im_spec_commit appends out_tokens[b, :out_count[b]] (from im_verify_greedy or im_accept_stochastic) to
 * hist and advances n; stats int64 [B, 3] (rounds, tokens committed, drafts accepted) accumulates if non-NULL.
 * Reference: the per-step row building, accept and KV rollback of ironmule/ggml_engine.py:1155-1343 and the
 * draft slot bookkeeping of ironmule/draft_model.py:203-274.
 */
int im_spec_prepare(const int32_t* hist, int64_t cap, const int32_t* n, const int32_t* target, int64_t B, int64_t k,
                    int64_t slot_cap, int32_t* d0_tok, int32_t* d0_pos, int32_t* d_pos, int32_t* v_tok,
                    int32_t* v_pos, void* stream);
int im_spec_commit(int32_t* hist, int64_t cap, int32_t* n, const int32_t* target, int64_t B, int64_t k,
                   const int32_t* out_tokens, const int32_t* out_count, int64_t* stats, void* stream);

/*
 * Stochastic speculative decoding on a Philox4x32-10 stream (no counterpart in the reference's code, which
 * accepts greedily only, ironmule/speculation.py:103-108; this is the published speculative-sampling rule that
 * the north-star configuration asks for). Distributions are softmax(logits / temperature) restricted to the
 * top-p set {v : logit_v >= l*} (l* the largest logit whose set holds >= top_p of the mass; boundary ties kept)
 * and renormalised. Philox key = (seed low, seed high), counter = (off low, off high, stream, draw) with
 * off = offset + (*offset_dev when offset_dev != NULL: a device counter a captured CUDA graph can advance);
 * uniform = (word0 >> 8) * 2^-24.
 *
 * im_accept_stochastic: target_logits [B, k+1, V] (row b*(k+1)+i scores the token after draft i-1), draft_logits
 * [k, B, V] (pass-major: row i*B+b is the distribution draft i of sequence b was sampled from), drafts int32 [B, k]
 * (row stride drafts_ld). Draft i is accepted iff u(stream b, draw 2i) * q(d) < p(d); at the first rejection the
 * token is drawn from norm(max(0, p - q)) with u(b, 2i+1); after k accepts the bonus token is drawn from the
 * target's row k with u(b, 2k). Writes out_tokens [B, k+1] (-1 padded) and out_count [B]; ratios [B, k] (p/q per
 * tested draft) when non-NULL. workspace >= im_sampling_workspace_bytes(B*(2k+1)).
 * im_sample_rows: one token per row of logits [rows, V] from its filtered distribution with u(streams[r] (or r),
 * draw), written at out[r * out_stride]; workspace >= im_sampling_workspace_bytes(rows).
 * im_philox4x32_10: the raw stream, out[4i..4i+3] = Philox4x32-10(counter (offset lo, hi, stream_id, i), seed).
 */
size_t im_sampling_workspace_bytes(int64_t rows);
int im_accept_stochastic(const uint16_t* target_logits, const uint16_t* draft_logits, int64_t B, int64_t k, int64_t V,
                         int64_t ld, const int32_t* drafts, int64_t drafts_ld, float temperature, float top_p,
                         uint64_t seed, uint64_t offset, const uint64_t* offset_dev, int32_t* out_tokens,
                         int32_t* out_count, float* ratios, void* workspace, size_t workspace_bytes, void* stream);
int im_sample_rows(const uint16_t* logits, int64_t rows, int64_t V, int64_t ld, float temperature, float top_p,
                   uint64_t seed, uint64_t offset, const uint64_t* offset_dev, const uint32_t* streams, uint32_t draw,
                   int32_t* out, int64_t out_stride, void* workspace, size_t workspace_bytes, void* stream);
int im_philox4x32_10(uint64_t seed, uint64_t offset, uint32_t stream_id, uint32_t n, uint32_t* out, void* stream);

/* ---- GGUF k-quant matmul (the ggml path) ------------------------------------------------------------------
 *
 * y[B][N] = x[B][K] . W^T for W in llama.cpp's GGUF blocks of 256 weights: type 12 = Q4_K (144-byte blocks, W 16-byte
 * aligned) or 14 = Q6_K (210-byte blocks, W 2-byte aligned), N rows of K/256 blocks each; x and y float32 on the
 * device; 1 <= B <= 32 tokens, K a multiple of 256. The activations are rounded to 8 bits per 32 values and each
 * sub-block's dot product is exact in integers, as llama.cpp's own quantized matmuls compute; a token's results do
 * not depend on B or on the other tokens.
 *
 * im_kq_mul_mat replaces the reference's llama.cpp hook ironmule_kg_mul_mat (ironmule/kernel_gen.py:803-862) with the
 * same arguments and contract: IM_OK (0) when it computed y, non-zero (IM_UNSUPPORTED for a type, K or token count it
 * does not serve) when llama.cpp's own kernel should run. Its scratch is one static device array per GPU (B x K up to
 * about 1.5 M), looked up on the first call on a device: overlapping calls race and must not be issued.
 * im_kq_gemv takes a caller workspace of im_kq_workspace_bytes(K, B) bytes, 256-byte aligned, instead.
 */
int im_kq_mul_mat(int type, const void* w, const float* x, float* y, int64_t N, int64_t K, int64_t B, void* stream);
/* im_kq_mul_mat under the name llama.cpp's patched mul_mat looks up (dlsym) in the library IRONMULE_KG_LIB names
 * (the reference's native/ggml_patches/kg1/ggml-cuda.cu.diff:6-18), so this library loads there as it is. */
int ironmule_kg_mul_mat(int type, const void* w, const float* x, float* y, int64_t N, int64_t K, int64_t B,
                        void* stream);
int im_kq_gemv(int type, const void* w, const float* x, float* y, int64_t N, int64_t K, int64_t B, void* workspace,
               size_t workspace_bytes, void* stream);
size_t im_kq_workspace_bytes(int64_t K, int64_t B);

#ifdef __cplusplus
}
#endif

#endif /* IMSPEC_H */
