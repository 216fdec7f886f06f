// pool_scores.cu — pooled block scores of the `mean` calibration mode.
//
// Restates _compute_pooled_qk_block_scores with pooling_mode="mean"
// (sinkattention/sparse_attention.py:138-142):
//   q_pool = _mean_pool_sequence(q.float(), block)   (lines 88-94; the last
//            partial block is replicate-padded with the final token, line 85)
//   k_pool = _mean_pool_sequence(k.float(), block)
//   scores = softmax(q_pool @ k_pool^T * (1/sqrt(D)), dim=-1)
// and the batch mean SinkMaskCalibrator.record takes next (line 580-581).
//
// At the calibration shapes (D = 128, 128-token blocks, at most 256 blocks,
// TMA-compatible strides) sa_pool_scores runs the fused calibration-layer
// kernel of calib_layer.cu: one launch whose score work overlaps its HBM-bound
// pooling. Other shapes, and the two halves sa_pool_means / sa_pooled_softmax,
// run three kernels, stream-ordered:
//   pool_rows     HBM-bound: reads Q and K once with 16-byte loads (or TMA
//                 tiles at D = 128, block = 128), writes fp32 block means
//                 [B,H,nb,D] to the workspace
//   pooled_logits fp32 SIMT GEMM, 64x64 tiles: logits = q_pool k_pool^T, then
//                 the scale multiply (a separate rounding, as torch does)
//   row_softmax   one warp per (head, query block): softmax of every batch's
//                 row, optional per-batch output and the batch mean
// Both forms take the same floating-point steps and agree to within one ulp.
// fp32 throughout so the scores track the reference's fp32 matmul closely
// (the coverage mask downstream is decided on these values).

#include <math.h>

#include "calib_layer.cuh"
#include "sa_common.cuh"

namespace sa {
namespace pool {

constexpr int kPoolThreads = 256;

// grid: (nb, B*H, 2 [q|k]); block: 256 threads.
__global__ void __launch_bounds__(kPoolThreads)
    pool_rows_kernel(const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
                     int64_t qs0, int64_t qs1, int64_t qs2, int64_t ks0, int64_t ks1,
                     int64_t ks2, int H, int S, int D, int block, int nb,
                     float* __restrict__ qp, float* __restrict__ kp) {
  __shared__ float red[kPoolThreads * 8];
  const int j = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const bool is_k = blockIdx.z != 0;
  const __nv_bfloat16* x = is_k ? k : q;
  const int64_t s0 = is_k ? ks0 : qs0, s1 = is_k ? ks1 : qs1, s2 = is_k ? ks2 : qs2;
  float* outp = (is_k ? kp : qp) + ((int64_t)bh * nb + j) * D;

  const int tpr = D >> 3;            // threads per token row (8 bf16 each)
  const int rpp = kPoolThreads / tpr; // token rows per pass
  const int t = threadIdx.x;
  const int c = t % tpr;
  const int r0 = t / tpr;
  const int row_lo = j * block;
  const int valid = min(block, S - row_lo);
  const __nv_bfloat16* base = x + (int64_t)b * s0 + (int64_t)h * s1 + (int64_t)c * 8;

  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  if (r0 < rpp) {
    int r = r0;
    // 4 independent 16-byte loads in flight per iteration
    for (; r + 3 * rpp < valid; r += 4 * rpp) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        v[u] = __ldg(reinterpret_cast<const uint4*>(base + (int64_t)(row_lo + r + u * rpp) * s2));
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const __nv_bfloat162* pv = reinterpret_cast<const __nv_bfloat162*>(&v[u]);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(pv[e]);
          acc[2 * e] += f.x;
          acc[2 * e + 1] += f.y;
        }
      }
    }
    for (; r < valid; r += rpp) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(base + (int64_t)(row_lo + r) * s2));
      const __nv_bfloat162* pv = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(pv[e]);
        acc[2 * e] += f.x;
        acc[2 * e + 1] += f.y;
      }
    }
    // Replicate padding: the final token stands in for the missing rows.
    if (valid < block && r0 == 0) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(base + (int64_t)(S - 1) * s2));
      const __nv_bfloat162* pv = reinterpret_cast<const __nv_bfloat162*>(&v);
      const float w = (float)(block - valid);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __bfloat1622float2(pv[e]);
        acc[2 * e] += w * f.x;
        acc[2 * e + 1] += w * f.y;
      }
    }
  }
  // red[r0][c*8 + e]
  if (r0 < rpp) {
#pragma unroll
    for (int e = 0; e < 8; ++e) red[r0 * D + c * 8 + e] = acc[e];
  }
  __syncthreads();
  const float inv = 1.0f / (float)block;
  for (int d = t; d < D; d += kPoolThreads) {
    float s = 0.f;
    for (int r = 0; r < rpp; ++r) s += red[r * D + d];
    outp[d] = s * inv;
  }
}

// TMA-staged variant of pool_rows for D == 128, block == 128 (the
// calibration shape). Persistent: one CTA per SM, 3 warps; each warp owns two
// 32 KB shared-memory stages and streams its own sequence of (tensor, b, h,
// block) items through them: the TMA load of item k+1 is in flight while the
// warp sums item k. Lane l sums columns 4l..4l+3 over the block's 128 rows
// (rows past S arrive zero-filled and the final token is added for them,
// the replicate padding of sparse_attention.py:79-85).
constexpr int kTmaWarps = 3;
constexpr int kTmaStageBytes = 128 * 128 * 2;
constexpr size_t kTmaSmem = 1024 + (size_t)kTmaWarps * 2 * kTmaStageBytes + 64;

__global__ void __launch_bounds__(kTmaWarps * 32, 1)
    pool_rows_tma_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k, int BH, int H, int S, int nb,
                         float* __restrict__ qp, float* __restrict__ kp) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* stage0 = smem + (size_t)warp * 2 * kTmaStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kTmaWarps * 2 * kTmaStageBytes) +
                   warp * 2;
  if (lane == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    fence_barrier_init();
  }
  __syncwarp();
  const int64_t n_items = 2LL * BH * nb;
  const int64_t stride = (int64_t)gridDim.x * kTmaWarps;
  int64_t item = (int64_t)blockIdx.x * kTmaWarps + warp;
  auto issue = [&](int64_t it, int st) {
    const int t = (int)(it / ((int64_t)BH * nb));
    const int rem = (int)(it - (int64_t)t * BH * nb);
    const int bh = rem / nb, j = rem - (rem / nb) * nb;
    mbar_arrive_expect_tx(&full[st], kTmaStageBytes);
    tma_load_4d(t ? &tm_k : &tm_q, &full[st], stage0 + (size_t)st * kTmaStageBytes, 0, j * 128,
                bh % H, bh / H);
  };
  if (lane == 0 && item < n_items) issue(item, 0);
  for (int k = 0; item < n_items; ++k, item += stride) {
    const int st = k & 1;
    const int64_t next = item + stride;
    if (lane == 0 && next < n_items) {
      fence_proxy_async_smem();
      issue(next, st ^ 1);
    }
    if (!mbar_wait_drain(&full[st], (uint32_t)(k >> 1) & 1u)) break;
    const uint8_t* tile = stage0 + (size_t)st * kTmaStageBytes + lane * 8;
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
    const int t = (int)(item / ((int64_t)BH * nb));
    const int rem = (int)(item - (int64_t)t * BH * nb);
    const int j = rem % nb;
    const int valid = min(128, S - j * 128);
    if (valid < 128) {
      const uint2 u = *reinterpret_cast<const uint2*>(tile + (valid - 1) * 256);
      const float wgt = (float)(128 - valid);
      a0 += wgt * __uint_as_float(u.x << 16); a1 += wgt * __uint_as_float(u.x & 0xffff0000u);
      a2 += wgt * __uint_as_float(u.y << 16); a3 += wgt * __uint_as_float(u.y & 0xffff0000u);
    }
    const float inv = 1.0f / 128.0f;
    float* outp = (t ? kp : qp) + (int64_t)rem * 128 + lane * 4;
    *reinterpret_cast<float4*>(outp) = make_float4(a0 * inv, a1 * inv, a2 * inv, a3 * inv);
    __syncwarp();
  }
}

// logits[bh, i, j] = scale * sum_d qp[bh, i, d] * kp[bh, j, d]
// grid: (ceil(nb/64), ceil(nb/64), B*H); block 256 = 16x16 threads, 4x4 each.
constexpr int kT = 64, kKC = 32;
__global__ void __launch_bounds__(256)
    pooled_logits_kernel(const float* __restrict__ qp, const float* __restrict__ kp, int nb, int D,
                         float scale, float* __restrict__ logits) {
  __shared__ float As[kKC][kT + 4];
  __shared__ float Bs[kKC][kT + 4];
  const int bh = blockIdx.z;
  const int i0 = blockIdx.y * kT, j0 = blockIdx.x * kT;
  const float* A = qp + (int64_t)bh * nb * D;
  const float* Bm = kp + (int64_t)bh * nb * D;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[a][c] = 0.f;

  for (int k0 = 0; k0 < D; k0 += kKC) {
    // 64 rows x 32 k per operand = 512 float4 → 2 per thread each
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int idx = threadIdx.x + u * 256;  // 0..511
      const int r = idx >> 3;                 // row 0..63
      const int kc = (idx & 7) * 4;           // k offset 0..28
      float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = va;
      if (i0 + r < nb && k0 + kc < D)
        va = *reinterpret_cast<const float4*>(A + (int64_t)(i0 + r) * D + k0 + kc);
      if (j0 + r < nb && k0 + kc < D)
        vb = *reinterpret_cast<const float4*>(Bm + (int64_t)(j0 + r) * D + k0 + kc);
      As[kc + 0][r] = va.x; As[kc + 1][r] = va.y; As[kc + 2][r] = va.z; As[kc + 3][r] = va.w;
      Bs[kc + 0][r] = vb.x; Bs[kc + 1][r] = vb.y; Bs[kc + 2][r] = vb.z; Bs[kc + 3][r] = vb.w;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kKC; ++kk) {
      const float4 a = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
      const float4 bv = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float bw[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
      for (int x = 0; x < 4; ++x)
#pragma unroll
        for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(av[x], bw[y], acc[x][y]);
    }
    __syncthreads();
  }
  float* out = logits + (int64_t)bh * nb * nb;
#pragma unroll
  for (int x = 0; x < 4; ++x) {
    const int i = i0 + ty * 4 + x;
    if (i >= nb) continue;
#pragma unroll
    for (int y = 0; y < 4; ++y) {
      const int j = j0 + tx * 4 + y;
      if (j < nb) out[(int64_t)i * nb + j] = acc[x][y] * scale;
    }
  }
}

// One warp per (h, i). For every batch b: p = exp(x - max) * (1/sum).
// scores (nullable) [B,H,nb,nb]; batch_mean (nullable) [H,nb,nb].
// L stacked layers: logits [L,B,H,nb,nb], batch_mean [L,H,nb,nb] (per layer).
__global__ void row_softmax_kernel(const float* __restrict__ logits, int L, int B, int H, int nb,
                                   float* __restrict__ scores, float* __restrict__ batch_mean) {
  extern __shared__ float accs[];
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * warps + warp;  // (l*H + h)*nb + i
  if (r >= (int64_t)L * H * nb) return;
  const int l = (int)(r / ((int64_t)H * nb));
  const int rh = (int)(r % ((int64_t)H * nb));
  const int h = rh / nb, i = rh % nb;
  float* acc = accs + (size_t)warp * nb;
  for (int j = lane; j < nb; j += 32) acc[j] = 0.f;
  for (int b = 0; b < B; ++b) {
    const int64_t off = ((((int64_t)l * B + b) * H + h) * nb + i) * nb;
    const float* x = logits + off;
    float m = -INFINITY;
    for (int j = lane; j < nb; j += 32) m = fmaxf(m, x[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float s = 0.f;
    for (int j = lane; j < nb; j += 32) s += expf(x[j] - m);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float inv = 1.0f / s;
    for (int j = lane; j < nb; j += 32) {
      const float pv = expf(x[j] - m) * inv;
      if (scores != nullptr) scores[off + j] = pv;
      acc[j] += pv;
    }
  }
  if (batch_mean != nullptr) {
    const float invb = 1.0f / (float)B;
    float* out = batch_mean + r * nb;
    for (int j = lane; j < nb; j += 32) out[j] = B == 1 ? acc[j] : acc[j] * invb;
  }
}

}  // namespace pool
}  // namespace sa


namespace sa {
namespace pool {

// All calibration kernels prefer the maximum shared-memory carveout, so the
// small score kernels of one layer can share SMs with the pooling kernel of
// the next layer (launched on another stream) instead of waiting for a
// carveout change.
int prefer_max_shared_carveout() {
  const void* fns[3] = {(const void*)pool_rows_tma_kernel, (const void*)pooled_logits_kernel,
                        (const void*)row_softmax_kernel};
  for (const void* f : fns)
    if (int rc = func_attr_once(f, cudaFuncAttributePreferredSharedMemoryCarveout,
                                cudaSharedmemCarveoutMaxShared);
        rc != SA_OK)
      return rc;
  return SA_OK;
}

// The row-softmax kernel's dynamic shared memory (8 warps x nb fp32) may
// exceed the 48 KB default; the limit is raised once to the largest size
// the entry points accept (200 KB).
constexpr int kSoftmaxSmemMax = 200 * 1024;
int allow_softmax_smem(size_t smem) {
  if (smem <= 48 * 1024) return SA_OK;
  return func_attr_once((const void*)row_softmax_kernel,
                        cudaFuncAttributeMaxDynamicSharedMemorySize, kSoftmaxSmemMax);
}

// Pools Q and K into qp / kp, through TMA staging when the shape allows.
int launch_pool_rows(const void* q, const void* k, const int64_t q_strides[4],
                     const int64_t k_strides[4], int B, int H, int S, int D, int block, int nb,
                     float* qp, float* kp, cudaStream_t stream) {
  const bool tma_ok = D == 128 && block == 128 && ((uintptr_t)q % 16 == 0) &&
                      ((uintptr_t)k % 16 == 0);
  if (int rc0 = prefer_max_shared_carveout(); rc0 != SA_OK) return rc0;
  if (tma_ok) {
    EncodeTiledFn enc = encode_tiled_fn();
    if (enc == nullptr) return SA_ECUDA;
    CUtensorMap maps[2];
    const void* bases[2] = {q, k};
    const int64_t* strides[2] = {q_strides, k_strides};
    for (int t = 0; t < 2; ++t) {
      cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
      cuuint64_t gst[3] = {(cuuint64_t)strides[t][2] * 2, (cuuint64_t)strides[t][1] * 2,
                           (cuuint64_t)strides[t][0] * 2};
      cuuint32_t box[4] = {128, 128, 1, 1};
      cuuint32_t estr[4] = {1, 1, 1, 1};
      CUresult r = enc(&maps[t], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(bases[t]),
                       dims, gst, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                       CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled (pool) failed (CUresult %d)", (int)r);
        return SA_ECUDA;
      }
    }
    if (int rc = func_attr_once((const void*)pool_rows_tma_kernel,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTmaSmem);
        rc != SA_OK)
      return rc;
    const int64_t items = 2LL * B * H * nb;
    const int sms = sm_count_current_device();
    const int64_t warps_needed = (items + 0) / 1;
    int grid = (int)((warps_needed + kTmaWarps - 1) / kTmaWarps);
    if (grid > sms) grid = sms;
    if (grid < 1) grid = 1;
    pool_rows_tma_kernel<<<grid, kTmaWarps * 32, kTmaSmem, stream>>>(maps[0], maps[1], B * H, H, S,
                                                                     nb, qp, kp);
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
  }
  pool_rows_kernel<<<dim3(nb, B * H, 2), kPoolThreads, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k),
      q_strides[0], q_strides[1], q_strides[2], k_strides[0], k_strides[1], k_strides[2], H, S, D,
      block, nb, qp, kp);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

}  // namespace pool
}  // namespace sa

extern "C" size_t sa_pool_scores_workspace_size(int B, int H, int S, int D, int block) {
  if (B < 1 || H < 1 || S < 1 || D < 1 || block < 1) return 0;
  const size_t nb = (size_t)((S + block - 1) / block);
  return sa::calib::counter_bytes(H) + sa::calib::flag_bytes(H, (int)nb) +
         2 * (size_t)B * H * nb * D * sizeof(float) + (size_t)B * H * nb * nb * sizeof(float);
}

namespace sa {
namespace pool {

// sa_pool_scores after its argument checks: the fused kernel where it
// applies, else the three-kernel chain. The workspace starts with the fused
// kernel's counters in both cases.
int pool_scores_impl(const void* q, const void* k, const int64_t q_strides[4],
                     const int64_t k_strides[4], int B, int H, int S, int D, int block,
                     float scale, float* scores, float* batch_mean, void* workspace,
                     size_t ws_bytes, cudaStream_t stream) {
  const int nb = (S + block - 1) / block;
  if (scale <= 0.f) scale = 1.0f / sqrtf((float)D);
  if (calib::eligible(q, k, q_strides, k_strides, B, H, S, D, block)) {
    calib::LayerArgs a = {};
    a.q = q;
    a.k = k;
    a.q_strides = q_strides;
    a.k_strides = k_strides;
    a.B = B;
    a.H = H;
    a.S = S;
    a.scale = scale;
    a.scores = scores;
    a.batch_mean = batch_mean;
    a.mode = SA_COVERAGE_JOINT;
    a.workspace = workspace;
    a.ws_bytes = ws_bytes;
    return calib::launch(a, stream);
  }
  float* qp = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) +
                                       calib::counter_bytes(H) + calib::flag_bytes(H, nb));
  float* kp = qp + (size_t)B * H * nb * D;
  float* logits = kp + (size_t)B * H * nb * D;

  int rc = launch_pool_rows(q, k, q_strides, k_strides, B, H, S, D, block, nb, qp, kp, stream);
  if (rc != SA_OK) return rc;
  const int tiles = (nb + kT - 1) / kT;
  pooled_logits_kernel<<<dim3(tiles, tiles, B * H), 256, 0, stream>>>(qp, kp, nb, D, scale, logits);
  SA_CUDA_TRY(cudaGetLastError());
  const int warps = 8;
  const size_t smem = (size_t)warps * nb * sizeof(float);
  SA_CHECK_ARG(smem <= kSoftmaxSmemMax, "sa_pool_scores: nb=%d too large", nb);
  if (int rc2 = allow_softmax_smem(smem); rc2 != SA_OK) return rc2;
  const int64_t rows = (int64_t)H * nb;
  row_softmax_kernel<<<(unsigned)((rows + warps - 1) / warps), warps * 32, smem, stream>>>(
      logits, 1, B, H, nb, scores, batch_mean);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

}  // namespace pool
}  // namespace sa

extern "C" int sa_pool_scores(const void* q, const void* k, const int64_t q_strides[4],
                              const int64_t k_strides[4], int B, int H, int S, int D, int block,
                              float scale, float* scores, float* batch_mean, void* workspace,
                              size_t ws_bytes, cudaStream_t stream) {
  using namespace sa::pool;
  SA_CHECK_ARG(q && k && q_strides && k_strides, "sa_pool_scores: null pointer argument");
  SA_CHECK_ARG(scores || batch_mean, "sa_pool_scores: scores and batch_mean are both NULL");
  SA_CHECK_ARG(B >= 1 && H >= 1 && S >= 1 && block >= 1,
               "sa_pool_scores: B, H, S, block must be >= 1");
  SA_CHECK_ARG(D >= 8 && D <= 256 && D % 8 == 0, "sa_pool_scores: D must be a multiple of 8 in [8,256]");
  SA_CHECK_ARG(q_strides[3] == 1 && k_strides[3] == 1, "sa_pool_scores: stride(dim) must be 1");
  for (int i = 0; i < 3; ++i)
    SA_CHECK_ARG(q_strides[i] % 8 == 0 && k_strides[i] % 8 == 0,
                 "sa_pool_scores: strides must be multiples of 8 elements (16-byte loads)");
  SA_CHECK_ARG(((uintptr_t)q | (uintptr_t)k) % 16 == 0, "sa_pool_scores: q/k must be 16-byte aligned");
  const size_t need = sa_pool_scores_workspace_size(B, H, S, D, block);
  SA_CHECK_ARG(workspace != nullptr && ws_bytes >= need,
               "sa_pool_scores: workspace of %zu bytes required, got %zu", need, ws_bytes);
  SA_CHECK_ARG(((uintptr_t)workspace) % 256 == 0,
               "sa_pool_scores: workspace must be 256-byte aligned");
  SA_CHECK_ARG((int64_t)B * H <= 65535, "sa_pool_scores: B*H too large");
  return pool_scores_impl(q, k, q_strides, k_strides, B, H, S, D, block, scale, scores,
                          batch_mean, workspace, ws_bytes, stream);
}

extern "C" int sa_pool_means(const void* q, const void* k, const int64_t q_strides[4],
                             const int64_t k_strides[4], int B, int H, int S, int D, int block,
                             float* qp, float* kp, cudaStream_t stream) {
  using namespace sa::pool;
  SA_CHECK_ARG(q && k && q_strides && k_strides && qp && kp, "sa_pool_means: null pointer argument");
  SA_CHECK_ARG(B >= 1 && H >= 1 && S >= 1 && block >= 1, "sa_pool_means: B, H, S, block must be >= 1");
  SA_CHECK_ARG(D >= 8 && D <= 256 && D % 8 == 0, "sa_pool_means: D must be a multiple of 8 in [8,256]");
  SA_CHECK_ARG(q_strides[3] == 1 && k_strides[3] == 1, "sa_pool_means: stride(dim) must be 1");
  for (int i = 0; i < 3; ++i)
    SA_CHECK_ARG(q_strides[i] % 8 == 0 && k_strides[i] % 8 == 0,
                 "sa_pool_means: strides must be multiples of 8 elements (16-byte loads)");
  SA_CHECK_ARG(((uintptr_t)q | (uintptr_t)k) % 16 == 0, "sa_pool_means: q/k must be 16-byte aligned");
  SA_CHECK_ARG(((uintptr_t)qp | (uintptr_t)kp) % 16 == 0, "sa_pool_means: qp/kp must be 16-byte aligned");
  SA_CHECK_ARG((int64_t)B * H <= 65535, "sa_pool_means: B*H too large");
  const int nb = (S + block - 1) / block;
  return launch_pool_rows(q, k, q_strides, k_strides, B, H, S, D, block, nb, qp, kp, stream);
}

extern "C" int sa_pooled_softmax(const float* qp, const float* kp, int B, int H, int nb, int D,
                                 float scale, float* scores, float* batch_mean, float* logits_ws,
                                 cudaStream_t stream) {
  using namespace sa::pool;
  SA_CHECK_ARG(qp && kp && logits_ws, "sa_pooled_softmax: null pointer argument");
  SA_CHECK_ARG(scores || batch_mean, "sa_pooled_softmax: scores and batch_mean are both NULL");
  SA_CHECK_ARG(B >= 1 && H >= 1 && nb >= 1, "sa_pooled_softmax: B, H, nb must be >= 1");
  SA_CHECK_ARG(D >= 8 && D <= 256 && D % 8 == 0, "sa_pooled_softmax: D must be a multiple of 8 in [8,256]");
  SA_CHECK_ARG((int64_t)B * H <= 65535, "sa_pooled_softmax: B*H too large");
  SA_CHECK_ARG(((uintptr_t)qp | (uintptr_t)kp) % 16 == 0, "sa_pooled_softmax: qp/kp must be 16-byte aligned");
  if (scale <= 0.f) scale = 1.0f / sqrtf((float)D);
  if (int rc0 = prefer_max_shared_carveout(); rc0 != SA_OK) return rc0;
  const int tiles = (nb + kT - 1) / kT;
  pooled_logits_kernel<<<dim3(tiles, tiles, B * H), 256, 0, stream>>>(qp, kp, nb, D, scale, logits_ws);
  SA_CUDA_TRY(cudaGetLastError());
  const int warps = 8;
  const size_t smem = (size_t)warps * nb * sizeof(float);
  SA_CHECK_ARG(smem <= kSoftmaxSmemMax, "sa_pooled_softmax: nb=%d too large", nb);
  if (int rc = allow_softmax_smem(smem); rc != SA_OK) return rc;
  const int64_t rows = (int64_t)H * nb;
  row_softmax_kernel<<<(unsigned)((rows + warps - 1) / warps), warps * 32, smem, stream>>>(
      logits_ws, 1, B, H, nb, scores, batch_mean);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

// Pooled softmax and per-layer batch mean of L stacked layers in two launches
// (a calibration pass over many layers): qp, kp [L,B,H,nb,D] fp32.
extern "C" int sa_pooled_softmax_layers(const float* qp, const float* kp, int L, int B, int H,
                                        int nb, int D, float scale, float* batch_means,
                                        float* logits_ws, cudaStream_t stream) {
  using namespace sa::pool;
  SA_CHECK_ARG(qp && kp && logits_ws && batch_means,
               "sa_pooled_softmax_layers: null pointer argument");
  SA_CHECK_ARG(L >= 1 && B >= 1 && H >= 1 && nb >= 1,
               "sa_pooled_softmax_layers: L, B, H, nb must be >= 1");
  SA_CHECK_ARG(D >= 8 && D <= 256 && D % 8 == 0,
               "sa_pooled_softmax_layers: D must be a multiple of 8 in [8,256]");
  SA_CHECK_ARG((int64_t)L * B * H <= 65535, "sa_pooled_softmax_layers: L*B*H too large");
  SA_CHECK_ARG(((uintptr_t)qp | (uintptr_t)kp) % 16 == 0,
               "sa_pooled_softmax_layers: qp/kp must be 16-byte aligned");
  if (scale <= 0.f) scale = 1.0f / sqrtf((float)D);
  if (int rc0 = prefer_max_shared_carveout(); rc0 != SA_OK) return rc0;
  const int tiles = (nb + kT - 1) / kT;
  pooled_logits_kernel<<<dim3(tiles, tiles, L * B * H), 256, 0, stream>>>(qp, kp, nb, D, scale,
                                                                          logits_ws);
  SA_CUDA_TRY(cudaGetLastError());
  const int warps = 8;
  const size_t smem = (size_t)warps * nb * sizeof(float);
  SA_CHECK_ARG(smem <= kSoftmaxSmemMax, "sa_pooled_softmax_layers: nb=%d too large", nb);
  if (int rc = allow_softmax_smem(smem); rc != SA_OK) return rc;
  const int64_t rows = (int64_t)L * H * nb;
  row_softmax_kernel<<<(unsigned)((rows + warps - 1) / warps), warps * 32, smem, stream>>>(
      logits_ws, L, B, H, nb, nullptr, batch_means);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

// ---------------------------------------------------------------------------
// sa_pool_scores_noalloc: the same computation with library-owned scratch.
//
// Some callers cannot hand this library a workspace: a plain C or FFI host
// that binds the .so without any device allocator of its own, or a serving
// loop that reserved all device memory when it started and may not call
// cudaMalloc on its hot path (cudaMalloc can synchronise the device and can
// fail once memory is committed). For them the scratch of sa_pool_scores
// (work counters, pooled Q/K, logits) lives in one file-scope device array of
// kNoAllocScratchBytes (16 MiB), which every GPU that loads this module keeps
// until the process exits. That covers the Wan calibration shape (B=2, H=12,
// S=32768, D=128 needs 12.6 MB); larger requests are rejected with SA_EINVAL.
// The call runs exactly what sa_pool_scores runs for the same arguments.
//
// The first call on a device looks up the array's device address with
// cudaGetSymbolAddress (host code only sees a host-side stand-in for the
// symbol); make that first call before any stream capture begins. The
// address is kept for the life of the process, so no call may follow a
// cudaDeviceReset of that device. All calls share the one array and it keeps
// the last call's contents. Nothing in it has to start at zero: the fused
// kernel's work counters carry a per-launch tag (a counter holding another
// launch's tag counts as zero), and every other byte a call reads it writes
// first. Calls whose kernels overlap on the GPU (different streams, or
// several host threads, on one device) race on it and must be serialised by
// the caller.
// ---------------------------------------------------------------------------
#include <mutex>

namespace sa {
namespace pool {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64] = {};

// Device address of g_noalloc_scratch on the current device (looked up once).
int noalloc_scratch(void** out) {
  int dev = 0;
  SA_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) {
    sa::set_error("sa_pool_scores_noalloc: device index %d out of range", dev);
    return SA_EUNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    SA_CUDA_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return SA_OK;
}

}  // namespace pool
}  // namespace sa

extern "C" int sa_pool_scores_noalloc(const void* q, const void* k, const int64_t q_strides[4],
                                      const int64_t k_strides[4], int B, int H, int S, int D,
                                      int block, float scale, float* scores, float* batch_mean,
                                      cudaStream_t stream) {
  using namespace sa::pool;
  SA_CHECK_ARG(q && k && q_strides && k_strides, "sa_pool_scores_noalloc: null pointer argument");
  SA_CHECK_ARG(scores || batch_mean, "sa_pool_scores_noalloc: scores and batch_mean are both NULL");
  SA_CHECK_ARG(B >= 1 && H >= 1 && S >= 1 && block >= 1,
               "sa_pool_scores_noalloc: B, H, S, block must be >= 1");
  SA_CHECK_ARG(D >= 8 && D <= 256 && D % 8 == 0,
               "sa_pool_scores_noalloc: D must be a multiple of 8 in [8,256]");
  SA_CHECK_ARG(q_strides[3] == 1 && k_strides[3] == 1,
               "sa_pool_scores_noalloc: stride(dim) must be 1");
  for (int i = 0; i < 3; ++i)
    SA_CHECK_ARG(q_strides[i] % 8 == 0 && k_strides[i] % 8 == 0,
                 "sa_pool_scores_noalloc: strides must be multiples of 8 elements");
  SA_CHECK_ARG(((uintptr_t)q | (uintptr_t)k) % 16 == 0,
               "sa_pool_scores_noalloc: q/k must be 16-byte aligned");
  SA_CHECK_ARG((int64_t)B * H <= 65535, "sa_pool_scores_noalloc: B*H too large");
  const size_t need = sa_pool_scores_workspace_size(B, H, S, D, block);
  SA_CHECK_ARG(need <= kNoAllocScratchBytes,
               "sa_pool_scores_noalloc: this shape needs %zu bytes of scratch but the "
               "built-in scratch holds %zu bytes (16 MiB); use sa_pool_scores with a "
               "caller-provided workspace",
               need, kNoAllocScratchBytes);
  const int nb = (S + block - 1) / block;
  SA_CHECK_ARG((size_t)8 * nb * sizeof(float) <= kSoftmaxSmemMax,
               "sa_pool_scores_noalloc: nb=%d too large", nb);

  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != SA_OK) return rc;
  return pool_scores_impl(q, k, q_strides, k_strides, B, H, S, D, block, scale, scores,
                          batch_mean, scratch, kNoAllocScratchBytes, stream);
}
