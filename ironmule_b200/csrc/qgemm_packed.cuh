// Shared by the two kernels behind im_qgemm_packed: the warp-MMA kernel for up to 32 activation rows
// (qgemm_packed.cu) and the tensor-core kernel for more (qgemm_tc.cu). Both use the same packed units, the same
// K-split plan and the same arithmetic, so a row's bits do not depend on which kernel computed it.
#pragma once

#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

namespace im {

constexpr int Q4_UNIT = 1152;                // packed bytes per (32-row tile, 64-wide group)
constexpr int Q4_RMAX = 24;                  // groups per CTA K range (the split plan never exceeds it)
constexpr int Q4_MAX_SPLITS = 16;            // K splits per tile: one thread-block cluster reduces them
constexpr int Q4_MAX_NORM_PARTS = 256;       // partial sums of squares per activation row (RMSNorm prologue)
constexpr size_t Q4_COUNTER_BYTES = 524288;  // split-K arrival counters; the last word is the error word
constexpr int Q4_MAX_ROWS = 320;             // activation rows per call

// The o-projection's input taken from the attention's unmerged split partials (part == NULL: from x). Row r of
// sequence b (seq_rows[b] <= r < seq_rows[b + 1]) merges, per head, splits [0, row_slot[r] / kpc + 1): the
// splits past its own slot hold no key it sees.
struct Q4Attn {
  const float* part;      // the attention workspace's split partials
  const int* seq_rows;    // [B + 1]
  const int* row_slot;    // [M]
  int B, Hq, Hkv, D, kpc, nsplit, qblocks, nq;
};

struct Q4Args {
  const unsigned char* wp;  // packed units
  const uint16_t* x;        // [M, K] activations (raw residual when norm_w != NULL)
  uint16_t* y;
  const uint16_t* res;
  const float* norm_sq;     // [norm_parts][sq_ld] sums of squares of x rows (RMSNorm prologue) or NULL
  const uint16_t* norm_w;   // [K]
  float* out_sq;            // [tiles][sq_ld] sums of squares of the written rows (residual epilogue) or NULL
  float* partial;
  unsigned* counters;
  float eps;
  int M, N, K, tiles, splits, norm_parts, gemma_norm, sq_ld;
  int rg;                   // the most groups any split holds (sizes the activation staging)
  Q4Attn am;                // attention-merge input (am.part != NULL)
};

struct Q4Plan {
  int tiles, ctas_x, splits, nt, chunks;
  int rg;  // the most groups one split holds
  size_t workspace;
};

// The K-split plan: depends on (N, K) only, never on M.
Q4Plan q4_plan(int64_t M, int64_t N, int64_t K);

// Tensor-core path (M > 32): workspace bytes past the counters for M rows, and the launch (prologue kernel +
// GEMM kernel) on `workspace` laid out as [counters][partials][activation tiles].
size_t qtc_workspace_bytes(const Q4Plan& p, int64_t M, int64_t K);
int qtc_launch(const Q4Plan& p, const Q4Args& a, int epilogue, void* workspace, cudaStream_t st);

}  // namespace im
