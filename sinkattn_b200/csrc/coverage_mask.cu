// coverage_mask.cu — per-row minimal-coverage block mask on the GPU.
//
// Restates _build_direct_mean_coverage_mask (sinkattention/sparse_attention.py:268-376)
// and _build_offline_required_mask (sparse_attention.py:241-265) with one warp
// per (head, query-block row):
//
//   joint mode (lines 334-376)
//     total    = max(sum_j s[j], 1e-6)                   (fp32)
//     req[j]   = j < T || row < T || (force_sink_col && j == 0)
//     selected = sum_j s[j] * req[j]
//     target   = max(coverage * total - selected, 0)      (fp32 multiply, line 340-341)
//     sort non-required scores descending (required -> -inf -> 0 after sort)
//     cum      = cumsum(sorted) accumulated in fp64, each prefix rounded to fp32
//     k        = target > 1e-6 ? (any(cum >= target) ? first + 1 : #candidates) : 0
//     keep sorted[0:k] | req | diagonal ; empty row keeps sorted[0]
//   video_residual mode (lines 286-332), T > 0
//     rows < T and columns < T are required; rows >= T run the rule above on
//     columns >= T with total over those columns and no `selected`; no diagonal;
//     an empty row keeps argmax over the full row.
//
// Exactness: CPU torch.cumsum accumulates fp32 input in fp64 and rounds each
// prefix, so the cumulative sums here are the sequential fp64 sums. They are
// computed in parallel only when every addition is exact in fp64 (all values
// non-negative multiples of 2^q whose total stays below 2^(q+52)); otherwise
// one lane runs the sequential loop. The sort is stable (value descending,
// index ascending); torch's CPU sort is not, so a row whose cut separates
// equal scores is reported with SA_ROW_TIE_AT_CUT. When the caller does not
// supply the row totals they are computed in fp64 and rounded, and rows whose
// crossing lies within 2 ulp of the target get SA_ROW_NEAR_TARGET.

#include <float.h>
#include <math.h>

#include "coverage_row.cuh"

namespace sa {
namespace cov {

struct Params {
  const float* scores;
  int64_t ss0, ss1;  // head, row strides (elements); column stride is 1
  int H, nq, nk, mode, T, keep_diag, force_sink;
  float coverage;
  const float* row_total;
  const float* row_selected;
  uint8_t* mask;
  int32_t* flags;
};

template <int NPAD>
__global__ void coverage_mask_kernel(const Params p) {
  extern __shared__ uint8_t smem_raw[];
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // per warp: sorted value keys, then the candidate value of every column
  uint32_t* skey = reinterpret_cast<uint32_t*>(smem_raw) + (size_t)warp * 2 * NPAD;
  float* cval = reinterpret_cast<float*>(skey + NPAD);

  const int64_t grow = (int64_t)blockIdx.x * warps + warp;  // (head, row) flattened
  if (grow >= (int64_t)p.H * p.nq) return;
  const int h = (int)(grow / p.nq);
  const int row = (int)(grow % p.nq);
  const float* s = p.scores + (int64_t)h * p.ss0 + (int64_t)row * p.ss1;
  RowSpec rs;
  rs.nk = p.nk;
  rs.T = p.T;
  rs.mode = p.mode;
  rs.keep_diag = p.keep_diag;
  rs.force_sink = p.force_sink;
  rs.coverage = p.coverage;
  coverage_row<NPAD>(s, row, rs, p.row_total != nullptr ? p.row_total + grow : nullptr,
                     p.row_selected != nullptr ? p.row_selected + grow : nullptr, skey, cval,
                     p.mask + grow * p.nk, p.flags != nullptr ? p.flags + grow : nullptr, lane);
}

template <int NPAD>
int launch(const Params& p, cudaStream_t stream) {
  const int warps = NPAD <= 1024 ? 8 : (NPAD == 2048 ? 4 : 2);
  const size_t smem = (size_t)warps * NPAD * 2 * sizeof(uint32_t);
  // max shared carveout: lets this kernel share SMs with the pooling kernel
  SA_CUDA_TRY(cudaFuncSetAttribute(coverage_mask_kernel<NPAD>,
                                   cudaFuncAttributePreferredSharedMemoryCarveout,
                                   cudaSharedmemCarveoutMaxShared));
  if (smem > 48 * 1024) {
    SA_CUDA_TRY(cudaFuncSetAttribute(coverage_mask_kernel<NPAD>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  const int64_t rows = (int64_t)p.H * p.nq;
  const int64_t blocks = (rows + warps - 1) / warps;
  coverage_mask_kernel<NPAD><<<(unsigned)blocks, warps * 32, smem, stream>>>(p);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

}  // namespace cov
}  // namespace sa

extern "C" int sa_coverage_mask(const float* scores, const int64_t s_strides[3], int H, int nq,
                                int nk, int mode, float coverage, int keep_diagonal,
                                int text_blocks, int force_sink_col, const float* row_total,
                                const float* row_selected, uint8_t* mask_out, int32_t* row_flags,
                                cudaStream_t stream) {
  using namespace sa::cov;
  SA_CHECK_ARG(scores && mask_out && s_strides, "sa_coverage_mask: null pointer argument");
  SA_CHECK_ARG(H >= 1 && nq >= 1 && nk >= 1, "sa_coverage_mask: H, nq, nk must be >= 1");
  SA_CHECK_ARG(nk <= 4096, "sa_coverage_mask: nk=%d exceeds 4096", nk);
  SA_CHECK_ARG(s_strides[2] == 1, "sa_coverage_mask: scores need stride(-1) == 1");
  SA_CHECK_ARG(mode == SA_COVERAGE_JOINT || mode == SA_COVERAGE_VIDEO_RESIDUAL,
               "sa_coverage_mask: unknown mode %d", mode);
  SA_CHECK_ARG(text_blocks >= 0, "sa_coverage_mask: text_blocks must be >= 0");
  SA_CHECK_ARG(!(coverage != coverage), "sa_coverage_mask: coverage is NaN");
  Params p;
  p.scores = scores;
  p.ss0 = s_strides[0];
  p.ss1 = s_strides[1];
  p.H = H; p.nq = nq; p.nk = nk;
  p.T = text_blocks < nq ? (text_blocks < nk ? text_blocks : nk) : (nq < nk ? nq : nk);
  // video_residual only applies with text blocks (line 286-290); else joint.
  p.mode = (mode == SA_COVERAGE_VIDEO_RESIDUAL && p.T > 0) ? mode : SA_COVERAGE_JOINT;
  p.keep_diag = keep_diagonal != 0;
  p.force_sink = force_sink_col != 0;
  p.coverage = coverage;
  p.row_total = row_total;
  p.row_selected = row_selected;
  p.mask = mask_out;
  p.flags = row_flags;
  if (nk <= 32) return launch<32>(p, stream);
  if (nk <= 64) return launch<64>(p, stream);
  if (nk <= 128) return launch<128>(p, stream);
  if (nk <= 256) return launch<256>(p, stream);
  if (nk <= 512) return launch<512>(p, stream);
  if (nk <= 1024) return launch<1024>(p, stream);
  if (nk <= 2048) return launch<2048>(p, stream);
  return launch<4096>(p, stream);
}
