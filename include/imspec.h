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

/* Workspace bytes im_qgemm_w4g64_ex needs for this shape (0: it does not split K). */
size_t im_qgemm_workspace_bytes(int64_t M, int64_t N, int64_t K);

/* Sweep hook: force the CTA-level K split (0 restores the automatic choice). Process-wide. */
int im_qgemm_set_splits(int splits);

/*
 * Row statistics over a logits matrix: for each row r of logits[rows, V] (bf16, row stride ld elements)
 * writes argmax[r] (lowest index among equal maxima) and, if conf != NULL, the top-1 probability
 * conf[r] = 1 / sum_v exp(l_v - l_max). Replaces the host numpy scan of
 * ironmule/ggml_engine.py:669-683 (_decode_conf) and the per-row argmax at ggml_engine.py:848.
 * `workspace` >= im_argmax_workspace_bytes(rows, V) bytes, 256-byte aligned, zero-filled before first use.
 */
int im_argmax_rows(const uint16_t* logits, int64_t rows, int64_t V, int64_t ld, int32_t* argmax, float* conf,
                   void* workspace, size_t workspace_bytes, void* stream);
size_t im_argmax_workspace_bytes(int64_t rows, int64_t V);

/*
 * Greedy verification of B sequences with k drafts each, in one launch: argmax over each of the
 * B*(k+1) logits rows (row b*(k+1)+i scores the token after draft i-1), then per sequence the drafts the
 * target agrees with followed by the target's own next token -- IronMule's `accept`
 * (ironmule/speculation.py:103-108) applied to the argmax of ironmule/ggml_engine.py:1316-1332.
 * drafts int32 [B, k]; out_tokens int32 [B, k+1] (entries past out_count[b] are -1);
 * out_count int32 [B] (1..k+1); argmax_out int32 [B*(k+1)] may be NULL.
 * `workspace` as for im_argmax_rows with rows = B*(k+1).
 */
int im_verify_greedy(const uint16_t* logits, int64_t B, int64_t k, int64_t V, int64_t ld, const int32_t* drafts,
                     int32_t* out_tokens, int32_t* out_count, int32_t* argmax_out, void* workspace,
                     size_t workspace_bytes, void* stream);

/*
 * MLX-affine 4-bit quantisation of bf16 weights w[N, K] (16-byte aligned), group 64: scale = bf16((max-min)/15),
 * bias = bf16(min), q = clamp(rint((w - bias)/scale), 0, 15); writes wq uint32 [N, K/8] (low nibble first),
 * scales/biases bf16 [N, K/64]. The format nn.QuantizedLinear.from_linear produces for the reference
 * (tests/runtime/test_qmv_k3840_integration.py:17-21; layout checked at ironmule/qmv_k3840.py:379-408).
 */
int im_quantize_w4g64(const uint16_t* w, int64_t N, int64_t K, uint32_t* wq, uint16_t* scales, uint16_t* biases,
                      void* stream);

#ifdef __cplusplus
}
#endif

#endif /* IMSPEC_H */
