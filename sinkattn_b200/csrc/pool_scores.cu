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
// Three kernels, stream-ordered:
//   pool_rows     HBM-bound: reads Q and K once with 16-byte loads, writes
//                 fp32 block means [B,H,nb,D] to the workspace
//   pooled_logits fp32 SIMT GEMM, 64x64 tiles: logits = q_pool k_pool^T, then
//                 the scale multiply (a separate rounding, as torch does)
//   row_softmax   one warp per (head, query block): softmax of every batch's
//                 row, optional per-batch output and the batch mean
// fp32 throughout so the scores track the reference's fp32 matmul closely
// (the coverage mask downstream is decided on these values).

#include <math.h>

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
__global__ void row_softmax_kernel(const float* __restrict__ logits, int B, int H, int nb,
                                   float* __restrict__ scores, float* __restrict__ batch_mean) {
  extern __shared__ float accs[];
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * warps + warp;  // h*nb + i
  if (r >= (int64_t)H * nb) return;
  const int h = (int)(r / nb), i = (int)(r % nb);
  float* acc = accs + (size_t)warp * nb;
  for (int j = lane; j < nb; j += 32) acc[j] = 0.f;
  for (int b = 0; b < B; ++b) {
    const int64_t off = (((int64_t)b * H + h) * nb + i) * nb;
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

extern "C" size_t sa_pool_scores_workspace_size(int B, int H, int S, int D, int block) {
  if (B < 1 || H < 1 || S < 1 || D < 1 || block < 1) return 0;
  const size_t nb = (size_t)((S + block - 1) / block);
  return 2 * (size_t)B * H * nb * D * sizeof(float) + (size_t)B * H * nb * nb * sizeof(float);
}

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
  SA_CHECK_ARG(((uintptr_t)workspace) % 16 == 0, "sa_pool_scores: workspace must be 16-byte aligned");
  const int nb = (S + block - 1) / block;
  SA_CHECK_ARG((int64_t)B * H <= 65535, "sa_pool_scores: B*H too large");
  if (scale <= 0.f) scale = 1.0f / sqrtf((float)D);

  float* qp = reinterpret_cast<float*>(workspace);
  float* kp = qp + (size_t)B * H * nb * D;
  float* logits = kp + (size_t)B * H * nb * D;

  pool_rows_kernel<<<dim3(nb, B * H, 2), kPoolThreads, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k),
      q_strides[0], q_strides[1], q_strides[2], k_strides[0], k_strides[1], k_strides[2], H, S,
      D, block, nb, qp, kp);
  SA_CUDA_TRY(cudaGetLastError());
  const int tiles = (nb + kT - 1) / kT;
  pooled_logits_kernel<<<dim3(tiles, tiles, B * H), 256, 0, stream>>>(qp, kp, nb, D, scale, logits);
  SA_CUDA_TRY(cudaGetLastError());
  const int warps = 8;
  const size_t smem = (size_t)warps * nb * sizeof(float);
  if (smem > 48 * 1024) {
    SA_CHECK_ARG(smem <= 200 * 1024, "sa_pool_scores: nb=%d too large", nb);
    SA_CUDA_TRY(cudaFuncSetAttribute(row_softmax_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  const int64_t rows = (int64_t)H * nb;
  row_softmax_kernel<<<(unsigned)((rows + warps - 1) / warps), warps * 32, smem, stream>>>(
      logits, B, H, nb, scores, batch_mean);
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
// fail once memory is committed). For them the pooled Q/K and logits live in
// one file-scope device array of kNoAllocScratchBytes (16 MiB), which every
// GPU that loads this module keeps until the process exits. That covers the
// Wan calibration shape (B=2, H=12, S=32768, D=128 needs 12.6 MB); larger
// requests are rejected with SA_EINVAL.
//
// The first call on a device looks up the array's device address with
// cudaGetSymbolAddress (host code only sees a host-side stand-in for the
// symbol); make that first call before any stream capture begins. All calls
// share the one array and it keeps the last call's contents: every byte a
// call reads is written earlier in the same call, so nothing needs clearing,
// but calls whose kernels overlap on the GPU (different streams, or several
// host threads, on one device) race on it and must be serialised by the
// caller.
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
  const size_t smem = (size_t)8 * nb * sizeof(float);
  SA_CHECK_ARG(smem <= 200 * 1024, "sa_pool_scores_noalloc: nb=%d too large", nb);
  if (scale <= 0.f) scale = 1.0f / sqrtf((float)D);

  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != SA_OK) return rc;
  float* qp = reinterpret_cast<float*>(scratch);
  float* kp = qp + (size_t)B * H * nb * D;
  float* logits = kp + (size_t)B * H * nb * D;

  pool_rows_kernel<<<dim3(nb, B * H, 2), kPoolThreads, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(q), reinterpret_cast<const __nv_bfloat16*>(k),
      q_strides[0], q_strides[1], q_strides[2], k_strides[0], k_strides[1], k_strides[2], H, S,
      D, block, nb, qp, kp);
  SA_CUDA_TRY(cudaGetLastError());
  const int tiles = (nb + kT - 1) / kT;
  pooled_logits_kernel<<<dim3(tiles, tiles, B * H), 256, 0, stream>>>(qp, kp, nb, D, scale, logits);
  SA_CUDA_TRY(cudaGetLastError());
  if (smem > 48 * 1024)
    SA_CUDA_TRY(cudaFuncSetAttribute(row_softmax_kernel,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  const int64_t rows = (int64_t)H * nb;
  row_softmax_kernel<<<(unsigned)((rows + 7) / 8), 256, smem, stream>>>(logits, B, H, nb, scores,
                                                                         batch_mean);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}
