// calib_layer.cuh — host-side interface of the fused calibration-layer
// kernel (calib_layer.cu), used by the C entry points of pool_scores.cu and
// calib_layer.cu.
#pragma once

#include "sa_common.cuh"

namespace sa {
namespace calib {

// One launch: block means of Q and K (128-token blocks, D = 128), pooled
// logits, per-batch softmax, batch mean, and optionally the calibrator's
// running sums and the coverage mask of every row.
struct LayerArgs {
  const void* q;
  const void* k;
  const int64_t* q_strides;  // [4] elements: b, h, s, d (d == 1)
  const int64_t* k_strides;
  int B, H, S;
  float scale;
  float* scores;      // nullable [B,H,nb,nb]
  float* batch_mean;  // nullable [H,nb,nb]
  float* acc_sum;     // nullable [H,nb,nb], with acc_sumsq
  float* acc_sumsq;
  int acc_first;      // 1: the sums are set (first record), 0: added to
  uint8_t* mask;      // nullable [H,nb,nb]
  int32_t* row_flags; // nullable [H,nb] (only with mask)
  int mode;           // SA_COVERAGE_*
  float coverage;
  int keep_diagonal;
  int text_blocks;
  int force_sink_col;
  void* workspace;
  size_t ws_bytes;
  int32_t* status;    // nullable device word for SA_DEV_WAIT_TIMEOUT
};

// Bytes of the launch's work counters at the start of the workspace, and of
// the per-(head, row group) flags that follow them.
size_t counter_bytes(int H);
size_t flag_bytes(int H, int nb);
// Workspace bytes of one launch: counters, flags, pooled Q and K, and a
// batch-mean scratch for callers that want the mask only.
size_t workspace_bytes(int B, int H, int S);

// Whether the fused kernel takes this shape and these pointers (D = 128,
// block = 128, at most 256 blocks and 128 heads, TMA-compatible strides and
// alignment).
bool eligible(const void* q, const void* k, const int64_t* q_strides, const int64_t* k_strides,
              int B, int H, int S, int D, int block);

// Launches the kernel on a workspace of workspace_bytes() (any contents):
// counters, flags, the pooled Q [B,H,nb,128] and transposed pooled K
// [B,H,128,nb] in fp32, and the batch-mean scratch [H,nb,nb].
int launch(const LayerArgs& a, cudaStream_t stream);

}  // namespace calib
}  // namespace sa
