// calib_layer.cu — one calibration layer of the `mean` score mode in a
// single persistent launch:
//
//   q_pool = block means of Q, k_pool = block means of K  (128-token blocks,
//            the last partial block replicate-padded; sparse_attention.py:79-94)
//   logits = q_pool k_pool^T * scale                        (lines 138-141)
//   scores = softmax(logits) per batch element               (line 142)
//   mean   = scores.mean(dim=0)                              (record, line 580)
//   [sum += mean, sumsq += mean^2]                           (_accumulate_score, 537-549)
//   [mask  = coverage rule on mean]                          (lines 241-376)
//
// The pooling is HBM-bound and the rest is small, so the two overlap inside
// the launch instead of running as a chain of kernels after it. Each CTA
// (one per SM) has
//   * 3 pooling warps. Each takes (head, batch, q|k, block) items from a
//     launch-wide counter in head-major order, streams the item's
//     128 x 128 bf16 tile through its own two TMA stages, writes the fp32
//     block mean (Q row-major [B,H,nb,128], K transposed [B,H,128,nb]) and
//     counts the item against its head.
//   * 8 score warps. Together they take (head, 8 query rows) items from a
//     second counter, wait (bounded) until every pooling item of that head
//     has been counted, and compute the rows' logits (thread = key column),
//     softmax per batch element (warp = row), batch mean, optional running
//     sums, and optional coverage mask (warp = row, coverage_row.cuh).
// Heads complete in order while later heads are still being pooled, so only
// the last head's score items run after the HBM read ends.
//
// Both counters hand out items in order to CTAs that are running, so a score
// item only ever waits on pooling items that running warps hold or will
// take: the launch needs no co-residency guarantee. The last CTA to finish
// returns every counter to zero for the next launch on the workspace.
//
// The floating-point operations are those of the three-kernel chain in
// pool_scores.cu, in the same order (per-lane column sums of the TMA tile,
// one fmaf per channel in channel order, the scale multiply after, the
// lane-strided softmax sum, the batch sum from 0), so both give the same bits.

#include <math.h>

#include "calib_layer.cuh"
#include "coverage_row.cuh"

namespace sa {
namespace calib {

constexpr int kPoolWarps = 3;
constexpr int kScoreWarps = 8;
constexpr int kScoreThreads = kScoreWarps * 32;
constexpr int kThreads = (kPoolWarps + kScoreWarps) * 32;
constexpr int kRows = kScoreWarps;          // query rows per score item
constexpr int kD = 128;
constexpr int kStageBytes = 128 * 128 * 2;  // one bf16 128 x 128 tile
constexpr int kMaxBlocks = 256;

// counters: [0] pooling items taken, [1] score items taken, [2] CTAs done,
// [3 + h] pooling items finished of head h
size_t counter_bytes(int H) { return (((size_t)(4 + H) * 4) + 255) & ~size_t(255); }

template <int NPAD>
struct Layout {
  static constexpr size_t stages = 0;
  static constexpr size_t bars = stages + (size_t)kPoolWarps * 2 * kStageBytes;
  static constexpr size_t qs = bars + 64;                               // [kRows][128] fp32
  static constexpr size_t ebuf = qs + (size_t)kRows * kD * 4;           // [kRows][NPAD] fp32
  static constexpr size_t cov = ebuf + (size_t)kRows * NPAD * 4;        // [warps][2*NPAD] u32
  static constexpr size_t ctl = cov + (size_t)kScoreWarps * 2 * NPAD * 4;
  static constexpr size_t total = ctl + 16 + 1024;                      // + base alignment
};
static_assert(Layout<256>::total <= 232448, "shared memory layout exceeds 227 KB");

struct Params {
  int B, H, S, nb, G;   // G = score items per head
  float scale;
  float* qp;            // [B,H,nb,128]
  float* kpt;           // [B,H,128,nb]
  int* ctr;
  float* scores;
  float* bmean;
  float* sum;
  float* sumsq;
  int first;
  uint8_t* mask;
  int32_t* flags;
  cov::RowSpec spec;
  int32_t* status;
};

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void score_bar() {
  asm volatile("bar.sync 1, %0;" ::"r"(kScoreThreads) : "memory");
}

// Bounded wait until *cnt >= target; gives up (false) on timeout, recording
// SA_DEV_WAIT_TIMEOUT, or as soon as another wait of the launch gave up.
__device__ bool wait_count(const int* cnt, int target, int32_t* status) {
  if (ld_acquire(cnt) >= target) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (ld_acquire(cnt) >= target) return true;
    __nanosleep(32);
    if ((it & 63u) == 0u) {
      if (status != nullptr && *reinterpret_cast<volatile int32_t*>(status) != 0) return false;
      if (global_timer_ns() - t0 > kWaitNs) {
        if (status != nullptr) atomicExch(status, SA_DEV_WAIT_TIMEOUT);
        return false;
      }
    }
  }
}

template <int NPAD>
__global__ void __launch_bounds__(kThreads, 1)
    calib_layer_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k, const Params p) {
  using L = Layout<NPAD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::bars);
  float* qs = reinterpret_cast<float*>(smem + L::qs);
  float* ebuf = reinterpret_cast<float*>(smem + L::ebuf);
  uint32_t* covs = reinterpret_cast<uint32_t*>(smem + L::cov);
  volatile int* ctl = reinterpret_cast<volatile int*>(smem + L::ctl);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < kPoolWarps && lane == 0) {
    mbar_init(&bars[2 * warp], 1);
    mbar_init(&bars[2 * warp + 1], 1);
    fence_barrier_init();
  }
  __syncthreads();

  const int nb = p.nb;
  const int per_head = 2 * p.B * nb;  // pooling items of one head
  const int n_pool = p.H * per_head;

  if (warp < kPoolWarps) {
    // ---------------------------------------------------------------- pooling
    uint8_t* stage0 = smem + L::stages + (size_t)warp * 2 * kStageBytes;
    uint64_t* full = &bars[2 * warp];
    if (lane == 0) {
      prefetch_tensormap(&tm_q);
      prefetch_tensormap(&tm_k);
    }
    auto fetch = [&]() -> int {
      int it = 0;
      if (lane == 0) it = atomicAdd(&p.ctr[0], 1);
      return __shfl_sync(0xffffffffu, it, 0);
    };
    auto issue = [&](int it, int st) {
      const int h = it / per_head;
      const int r = it - h * per_head;
      const int b = r / (2 * nb);
      const int r2 = r - b * 2 * nb;
      const int t = r2 / nb;
      const int j = r2 - t * nb;
      mbar_arrive_expect_tx(&full[st], kStageBytes);
      tma_load_4d(t ? &tm_k : &tm_q, &full[st], stage0 + (size_t)st * kStageBytes, 0, j * 128, h,
                  b);
    };
    int item = fetch();
    if (lane == 0 && item < n_pool) issue(item, 0);
    for (int k = 0; item < n_pool; ++k) {
      const int st = k & 1;
      const int next = fetch();
      if (lane == 0 && next < n_pool) {
        fence_proxy_async_smem();
        issue(next, st ^ 1);
      }
      if (!mbar_wait_drain(&full[st], (uint32_t)(k >> 1) & 1u)) {
        if (lane == 0 && p.status != nullptr) atomicExch(p.status, SA_DEV_WAIT_TIMEOUT);
        break;
      }
      const uint8_t* tile = stage0 + (size_t)st * kStageBytes + lane * 8;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      float b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
#pragma unroll 8
      for (int r = 0; r < 128; r += 2) {
        const uint2 u = *reinterpret_cast<const uint2*>(tile + r * 256);
        const uint2 w = *reinterpret_cast<const uint2*>(tile + (r + 1) * 256);
        a0 += __uint_as_float(u.x << 16); a1 += __uint_as_float(u.x & 0xffff0000u);
        a2 += __uint_as_float(u.y << 16); a3 += __uint_as_float(u.y & 0xffff0000u);
        b0 += __uint_as_float(w.x << 16); b1 += __uint_as_float(w.x & 0xffff0000u);
        b2 += __uint_as_float(w.y << 16); b3 += __uint_as_float(w.y & 0xffff0000u);
      }
      a0 += b0; a1 += b1; a2 += b2; a3 += b3;
      const int h = item / per_head;
      const int r = item - h * per_head;
      const int b = r / (2 * nb);
      const int r2 = r - b * 2 * nb;
      const int t = r2 / nb;
      const int j = r2 - t * nb;
      const int valid = min(128, p.S - j * 128);
      if (valid < 128) {
        // rows past S arrived zero-filled; the final token stands in for them
        const uint2 u = *reinterpret_cast<const uint2*>(tile + (valid - 1) * 256);
        const float wgt = (float)(128 - valid);
        a0 += wgt * __uint_as_float(u.x << 16); a1 += wgt * __uint_as_float(u.x & 0xffff0000u);
        a2 += wgt * __uint_as_float(u.y << 16); a3 += wgt * __uint_as_float(u.y & 0xffff0000u);
      }
      const float inv = 1.0f / 128.0f;
      const int64_t bh = (int64_t)b * p.H + h;
      if (t == 0) {
        float* outp = p.qp + (bh * nb + j) * kD + lane * 4;
        *reinterpret_cast<float4*>(outp) = make_float4(a0 * inv, a1 * inv, a2 * inv, a3 * inv);
      } else {
        float* col = p.kpt + (bh * kD + lane * 4) * nb + j;
        col[0] = a0 * inv;
        col[nb] = a1 * inv;
        col[2 * nb] = a2 * inv;
        col[3 * nb] = a3 * inv;
      }
      __threadfence();
      __syncwarp();
      if (lane == 0) atomicAdd(&p.ctr[3 + h], 1);
      item = next;
    }
  } else {
    // ----------------------------------------------------------------- scores
    const int tid = threadIdx.x - kPoolWarps * 32;  // 0..255: key column j
    const int sw = warp - kPoolWarps;               // 0..7: row of the item
    const int j = tid;
    const int n_score = p.H * p.G;
    const float invb = 1.0f / (float)p.B;
    for (;;) {
      if (tid == 0) {
        const int s = atomicAdd(&p.ctr[1], 1);
        int ok = 0;
        if (s < n_score) ok = wait_count(&p.ctr[3 + s / p.G], per_head, p.status) ? 1 : 0;
        ctl[0] = s;
        ctl[1] = ok;
      }
      score_bar();
      const int s = ctl[0];
      const int ok = ctl[1];
      score_bar();
      if (s >= n_score) break;
      const int h = s / p.G;
      const int i0 = (s - h * p.G) * kRows;
      const int nrows = min(kRows, nb - i0);
      if (!ok) {
        // a wait gave up (status set): the item's outputs are marked invalid
        for (int r = 0; r < nrows; ++r) {
          if (j >= nb) continue;
          const int64_t hi = ((int64_t)h * nb + i0 + r) * nb + j;
          if (p.bmean != nullptr) p.bmean[hi] = __int_as_float(0x7fc00000);
          if (p.mask != nullptr) p.mask[hi] = 1;
          for (int b = 0; b < p.B && p.scores != nullptr; ++b)
            p.scores[(((int64_t)b * p.H + h) * nb + i0 + r) * nb + j] = __int_as_float(0x7fc00000);
        }
        continue;
      }
      float bacc[kRows];
#pragma unroll
      for (int r = 0; r < kRows; ++r) bacc[r] = 0.f;
      for (int b = 0; b < p.B; ++b) {
        const int64_t bh = (int64_t)b * p.H + h;
        {  // stage the item's pooled query rows: one float4 per thread
          const int r = tid >> 5;
          const int c = (tid & 31) * 4;
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if (r < nrows)
            v = __ldcg(reinterpret_cast<const float4*>(p.qp + (bh * nb + i0 + r) * kD + c));
          *reinterpret_cast<float4*>(qs + r * kD + c) = v;
        }
        score_bar();
        float acc[kRows];
#pragma unroll
        for (int r = 0; r < kRows; ++r) acc[r] = 0.f;
        if (j < nb) {
          const float* kcol = p.kpt + bh * kD * nb + j;
#pragma unroll 2
          for (int d = 0; d < kD; d += 4) {
            const float k0 = __ldcg(kcol + (int64_t)(d + 0) * nb);
            const float k1 = __ldcg(kcol + (int64_t)(d + 1) * nb);
            const float k2 = __ldcg(kcol + (int64_t)(d + 2) * nb);
            const float k3 = __ldcg(kcol + (int64_t)(d + 3) * nb);
#pragma unroll
            for (int r = 0; r < kRows; ++r) {
              const float4 q4 = *reinterpret_cast<const float4*>(qs + r * kD + d);
              acc[r] = fmaf(q4.x, k0, acc[r]);
              acc[r] = fmaf(q4.y, k1, acc[r]);
              acc[r] = fmaf(q4.z, k2, acc[r]);
              acc[r] = fmaf(q4.w, k3, acc[r]);
            }
          }
#pragma unroll
          for (int r = 0; r < kRows; ++r) ebuf[r * NPAD + j] = acc[r] * p.scale;
        }
        score_bar();
        if (sw < nrows) {  // softmax of row sw, lanes over the columns
          float* x = ebuf + sw * NPAD;
          float m = -INFINITY;
          for (int c = lane; c < nb; c += 32) m = fmaxf(m, x[c]);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
          float ssum = 0.f;
          for (int c = lane; c < nb; c += 32) ssum += expf(x[c] - m);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ssum += __shfl_xor_sync(0xffffffffu, ssum, o);
          const float inv = 1.0f / ssum;
          for (int c = lane; c < nb; c += 32) x[c] = expf(x[c] - m) * inv;
        }
        score_bar();
        if (j < nb) {
#pragma unroll
          for (int r = 0; r < kRows; ++r) {
            if (r >= nrows) break;
            const float pv = ebuf[r * NPAD + j];
            if (p.scores != nullptr) p.scores[(bh * nb + i0 + r) * nb + j] = pv;
            bacc[r] += pv;
          }
        }
        score_bar();
      }
      if (j < nb) {
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          if (r >= nrows) break;
          const float bm = p.B == 1 ? bacc[r] : bacc[r] * invb;
          const int64_t hi = ((int64_t)h * nb + i0 + r) * nb + j;
          if (p.bmean != nullptr) p.bmean[hi] = bm;
          if (p.sum != nullptr) {
            // separate roundings, as `sums += s; sq_sums += s.square()`
            const float sq = __fmul_rn(bm, bm);
            if (p.first) {
              p.sum[hi] = bm;
              p.sumsq[hi] = sq;
            } else {
              p.sum[hi] = __fadd_rn(p.sum[hi], bm);
              p.sumsq[hi] = __fadd_rn(p.sumsq[hi], sq);
            }
          }
          ebuf[r * NPAD + j] = bm;
        }
      }
      if (p.mask != nullptr) {
        score_bar();
        if (sw < nrows) {
          const int row = i0 + sw;
          uint32_t* skey = covs + (size_t)sw * 2 * NPAD;
          cov::coverage_row<NPAD>(ebuf + sw * NPAD, row, p.spec, nullptr, nullptr, skey,
                                  reinterpret_cast<float*>(skey + NPAD),
                                  p.mask + ((int64_t)h * nb + row) * nb,
                                  p.flags != nullptr ? p.flags + (int64_t)h * nb + row : nullptr,
                                  lane);
        }
      }
      score_bar();
    }
  }

  // the last CTA to finish returns the counters to zero
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&p.ctr[2], 1) == (int)gridDim.x - 1) {
      __threadfence();
      volatile int* c = p.ctr;
      c[0] = 0;
      c[1] = 0;
      for (int h = 0; h < p.H; ++h) c[3 + h] = 0;
      c[2] = 0;
      __threadfence();
    }
  }
}

bool eligible(const void* q, const void* k, const int64_t* q_strides, const int64_t* k_strides,
              int B, int H, int S, int D, int block) {
  if (D != kD || block != 128 || B < 1 || H < 1 || S < 1) return false;
  if ((S + 127) / 128 > kMaxBlocks) return false;
  if (((uintptr_t)q | (uintptr_t)k) % 16 != 0) return false;
  for (int i = 0; i < 3; ++i)
    if (q_strides[i] % 8 != 0 || k_strides[i] % 8 != 0 || q_strides[i] <= 0 || k_strides[i] <= 0)
      return false;
  return q_strides[3] == 1 && k_strides[3] == 1;
}

template <int NPAD>
int launch_t(const CUtensorMap& mq, const CUtensorMap& mk, const Params& p, int grid,
             cudaStream_t stream) {
  const int smem = (int)Layout<NPAD>::total;
  if (int rc = func_attr_once((const void*)calib_layer_kernel<NPAD>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      rc != SA_OK)
    return rc;
  calib_layer_kernel<NPAD><<<grid, kThreads, smem, stream>>>(mq, mk, p);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

int launch(const LayerArgs& a, cudaStream_t stream) {
  const int nb = (a.S + 127) / 128;
  const size_t ctr_bytes = counter_bytes(a.H);
  const size_t need = ctr_bytes + 2 * (size_t)a.B * a.H * nb * kD * sizeof(float);
  SA_CHECK_ARG(a.workspace != nullptr && a.ws_bytes >= need,
               "calibration layer: workspace of %zu bytes required, got %zu", need, a.ws_bytes);
  SA_CHECK_ARG(((uintptr_t)a.workspace) % 256 == 0,
               "calibration layer: workspace must be 256-byte aligned");
  EncodeTiledFn enc = encode_tiled_fn();
  if (enc == nullptr) return SA_ECUDA;
  CUtensorMap maps[2];
  const void* bases[2] = {a.q, a.k};
  const int64_t* strides[2] = {a.q_strides, a.k_strides};
  for (int t = 0; t < 2; ++t) {
    cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)a.S, (cuuint64_t)a.H, (cuuint64_t)a.B};
    cuuint64_t gst[3] = {(cuuint64_t)strides[t][2] * 2, (cuuint64_t)strides[t][1] * 2,
                         (cuuint64_t)strides[t][0] * 2};
    cuuint32_t box[4] = {128, 128, 1, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(&maps[t], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(bases[t]),
                     dims, gst, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled (calibration layer) failed (CUresult %d)", (int)r);
      return SA_ECUDA;
    }
  }
  Params p;
  p.B = a.B;
  p.H = a.H;
  p.S = a.S;
  p.nb = nb;
  p.G = (nb + kRows - 1) / kRows;
  p.scale = a.scale;
  p.ctr = reinterpret_cast<int*>(a.workspace);
  p.qp = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(a.workspace) + ctr_bytes);
  p.kpt = p.qp + (size_t)a.B * a.H * nb * kD;
  p.scores = a.scores;
  p.bmean = a.batch_mean;
  p.sum = a.acc_sum;
  p.sumsq = a.acc_sumsq;
  p.first = a.acc_first != 0;
  p.mask = a.mask;
  p.flags = a.mask != nullptr ? a.row_flags : nullptr;
  const int T = a.text_blocks < nb ? a.text_blocks : nb;
  p.spec.nk = nb;
  p.spec.T = T > 0 ? T : 0;
  p.spec.mode = (a.mode == SA_COVERAGE_VIDEO_RESIDUAL && p.spec.T > 0) ? a.mode
                                                                        : SA_COVERAGE_JOINT;
  p.spec.keep_diag = a.keep_diagonal != 0;
  p.spec.force_sink = a.force_sink_col != 0;
  p.spec.coverage = a.coverage;
  p.status = a.status;
  const int sms = sm_count_current_device();
  const int64_t n_pool = 2LL * a.B * a.H * nb;
  const int64_t n_score = (int64_t)a.H * p.G;
  int64_t want = (n_pool + kPoolWarps - 1) / kPoolWarps;
  if (n_score > want) want = n_score;
  const int grid = (int)(want < sms ? want : sms);
  if (nb <= 32) return launch_t<32>(maps[0], maps[1], p, grid, stream);
  if (nb <= 64) return launch_t<64>(maps[0], maps[1], p, grid, stream);
  if (nb <= 128) return launch_t<128>(maps[0], maps[1], p, grid, stream);
  return launch_t<256>(maps[0], maps[1], p, grid, stream);
}

}  // namespace calib
}  // namespace sa

extern "C" size_t sa_calibration_layer_workspace_size(int B, int H, int S) {
  if (B < 1 || H < 1 || S < 1) return 0;
  const size_t nb = (size_t)((S + 127) / 128);
  return sa::calib::counter_bytes(H) + 2 * (size_t)B * H * nb * 128 * sizeof(float);
}

extern "C" int sa_calibration_layer(const void* q, const void* k, const int64_t q_strides[4],
                                    const int64_t k_strides[4], int B, int H, int S, int D,
                                    float scale, float* scores, float* batch_mean, float* acc_sum,
                                    float* acc_sumsq, int acc_first, uint8_t* mask_out,
                                    int32_t* row_flags, int mode, float coverage,
                                    int keep_diagonal, int text_blocks, int force_sink_col,
                                    void* workspace, size_t ws_bytes, int32_t* status,
                                    cudaStream_t stream) {
  SA_CHECK_ARG(q && k && q_strides && k_strides, "sa_calibration_layer: null pointer argument");
  SA_CHECK_ARG(B >= 1 && H >= 1 && S >= 1, "sa_calibration_layer: B, H, S must be >= 1");
  SA_CHECK_ARG((acc_sum == nullptr) == (acc_sumsq == nullptr),
               "sa_calibration_layer: acc_sum and acc_sumsq go together");
  SA_CHECK_ARG(scores || batch_mean || acc_sum || mask_out,
               "sa_calibration_layer: no output requested");
  SA_CHECK_ARG(row_flags == nullptr || mask_out != nullptr,
               "sa_calibration_layer: row_flags needs mask_out");
  SA_CHECK_ARG(mode == SA_COVERAGE_JOINT || mode == SA_COVERAGE_VIDEO_RESIDUAL,
               "sa_calibration_layer: unknown mode %d", mode);
  SA_CHECK_ARG(text_blocks >= 0, "sa_calibration_layer: text_blocks must be >= 0");
  SA_CHECK_ARG(!(coverage != coverage), "sa_calibration_layer: coverage is NaN");
  SA_CHECK_ARG(D == 128, "sa_calibration_layer: D must be 128, got %d", D);
  SA_CHECK_ARG((S + 127) / 128 <= 256, "sa_calibration_layer: at most 256 blocks (S <= 32768)");
  SA_CHECK_ARG(q_strides[3] == 1 && k_strides[3] == 1,
               "sa_calibration_layer: stride(dim) must be 1");
  for (int i = 0; i < 3; ++i)
    SA_CHECK_ARG(q_strides[i] > 0 && k_strides[i] > 0 && q_strides[i] % 8 == 0 &&
                     k_strides[i] % 8 == 0,
                 "sa_calibration_layer: strides must be positive multiples of 8 elements");
  SA_CHECK_ARG(((uintptr_t)q | (uintptr_t)k) % 16 == 0,
               "sa_calibration_layer: q/k must be 16-byte aligned");
  sa::calib::LayerArgs a;
  a.q = q;
  a.k = k;
  a.q_strides = q_strides;
  a.k_strides = k_strides;
  a.B = B;
  a.H = H;
  a.S = S;
  a.scale = scale > 0.f ? scale : 1.0f / sqrtf(128.0f);
  a.scores = scores;
  a.batch_mean = batch_mean;
  a.acc_sum = acc_sum;
  a.acc_sumsq = acc_sumsq;
  a.acc_first = acc_first;
  a.mask = mask_out;
  a.row_flags = row_flags;
  a.mode = mode;
  a.coverage = coverage;
  a.keep_diagonal = keep_diagonal;
  a.text_blocks = text_blocks;
  a.force_sink_col = force_sink_col;
  a.workspace = workspace;
  a.ws_bytes = ws_bytes;
  a.status = status;
  return sa::calib::launch(a, stream);
}
