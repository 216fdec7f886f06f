// misc_kernels.cu — the small kernels either side of the two hot paths:
// device-resident score accumulation and finalisation of the calibrator,
// sequence mean pooling for the pooled-K/V dynamic branch, and the adaptive
// LSE mix of the sink and dynamic branches.

#include <math.h>

#include "sa_common.cuh"

namespace sa {
namespace misc {

// SinkMaskCalibrator._accumulate_score (sinkattention/sparse_attention.py:537-549)
__global__ void accumulate_kernel(const float* __restrict__ x, int64_t n, float* __restrict__ sum,
                                  float* __restrict__ sumsq, int first) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    // separate roundings (no FMA contraction), as the reference's
    // `sums += scores; sq_sums += scores.square()` on fp32 tensors
    const float v = x[i];
    const float sq = __fmul_rn(v, v);
    if (first) {
      sum[i] = v;
      sumsq[i] = sq;
    } else {
      sum[i] = __fadd_rn(sum[i], v);
      sumsq[i] = __fadd_rn(sumsq[i], sq);
    }
  }
}

// SinkMaskCalibrator._build_mean_and_masks (sparse_attention.py:563-566) and the
// presence-weighted variant of zimg/runtime/sink_sparse_zimage.py:330-334.
// With clamp_count the per-element counts are first raised to >= 1 in place,
// as the Z-Image calibrator's `presence_sums.clamp_min_(1.0)` does.
// With emit_variance the second output receives the clamped variance (no
// square root), for hosts that take the root themselves.
__global__ void finalize_kernel(const float* __restrict__ sum, const float* __restrict__ sumsq,
                                float* __restrict__ count, float scalar_count, int64_t n,
                                float* __restrict__ mean, float* __restrict__ std_out,
                                int clamp_count, int emit_variance) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float c = count != nullptr ? count[i] : scalar_count;
    if (clamp_count && c < 1.0f) {
      c = 1.0f;
      count[i] = c;
    }
    // IEEE division and separate roundings, as the reference's CPU tensors
    const float m = __fdiv_rn(sum[i], c);
    mean[i] = m;
    if (std_out != nullptr) {
      const float second = __fdiv_rn(sumsq[i], c);
      const float var = fmaxf(__fsub_rn(second, __fmul_rn(m, m)), 0.f);
      std_out[i] = emit_variance ? var : __fsqrt_rn(var);
    }
  }
}

// ZImageSinkMaskCalibrator.record's alignment and accumulation
// (zimg/runtime/sink_sparse_zimage.py:140-186, 262-278, 300-319): the scores of
// one sample, [H, n, n] with n = image blocks + this sample's text blocks,
// are placed in the fixed [H, T, T] layout (image blocks first, text blocks
// at the end), and sum, sum of squares and presence (1 where a score landed)
// accumulate there. Absent entries add 0, as the reference's zero-filled
// aligned tensor does. One thread per target entry.
__global__ void accumulate_aligned_kernel(const float* __restrict__ scores, int H, int n,
                                          int image_blocks, int text_start, int T,
                                          float* __restrict__ sum, float* __restrict__ sumsq,
                                          float* __restrict__ presence, int first) {
  const int64_t total = (int64_t)H * T * T;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int h = (int)(e / ((int64_t)T * T));
    const int ti = (int)((e / T) % T), tj = (int)(e % T);
    const int si = ti < image_blocks ? ti : (ti >= text_start ? image_blocks + (ti - text_start) : -1);
    const int sj = tj < image_blocks ? tj : (tj >= text_start ? image_blocks + (tj - text_start) : -1);
    const bool present = si >= 0 && sj >= 0;
    const float v = present ? scores[((int64_t)h * n + si) * n + sj] : 0.f;
    const float sq = __fmul_rn(v, v);
    const float pr = present ? 1.f : 0.f;
    if (first) {
      sum[e] = v;
      sumsq[e] = sq;
      presence[e] = pr;
    } else {
      sum[e] = __fadd_rn(sum[e], v);
      sumsq[e] = __fadd_rn(sumsq[e], sq);
      presence[e] = __fadd_rn(presence[e], pr);
    }
  }
}

// _mean_pool_sequence_preserve_prefix (sparse_attention.py:97-115).
// grid: (out_rows, B*H); block: D/8 threads x 8 token groups.
__global__ void mean_pool_seq_kernel(const __nv_bfloat16* __restrict__ x, int64_t xs0, int64_t xs1,
                                     int64_t xs2, int H, int S, int D, int pool, int prefix,
                                     __nv_bfloat16* __restrict__ out, int64_t os0, int64_t os1,
                                     int64_t os2) {
  __shared__ float red[8][256];
  const int orow = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int tpr = D >> 3;
  const int c = threadIdx.x % tpr;
  const int g = threadIdx.x / tpr;  // 0..7
  const __nv_bfloat16* base = x + (int64_t)b * xs0 + (int64_t)h * xs1 + (int64_t)c * 8;
  __nv_bfloat16* obase = out + (int64_t)b * os0 + (int64_t)h * os1 + (int64_t)orow * os2 + c * 8;
  if (orow < prefix) {
    if (g == 0)
      *reinterpret_cast<uint4*>(obase) =
          __ldg(reinterpret_cast<const uint4*>(base + (int64_t)orow * xs2));
    return;
  }
  const int lo = prefix + (orow - prefix) * pool;
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc[e] = 0.f;
  for (int r = g; r < pool; r += 8) {
    const int t = min(lo + r, S - 1);  // replicate padding of the final token
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(base + (int64_t)t * xs2));
    const __nv_bfloat162* pv = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(pv[e]);
      acc[2 * e] += f.x;
      acc[2 * e + 1] += f.y;
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) red[g][c * 8 + e] = acc[e];
  __syncthreads();
  if (g == 0) {
    const float inv = 1.0f / (float)pool;
    uint4 w;
    uint32_t* pw = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        s0 += red[q][c * 8 + 2 * e];
        s1 += red[q][c * 8 + 2 * e + 1];
      }
      pw[e] = pack_bf16x2(s0 * inv, s1 * inv);
    }
    *reinterpret_cast<uint4*>(obase) = w;
  }
}

// The same pooling for D = 128 through TMA, reading memory in order: an item
// is one pooled row of hb heads of one batch element (all heads where a
// stage holds them), a box {128, hb, pool} over the (d, h, s) axes, which is
// one contiguous stretch of the processors' [B, S, H, D] storage. A producer
// warp loads the next box while consumer warp w sums head w's pool rows of
// the current one (lane l: columns 4l .. 4l+3) and writes the pooled row.
// At the Wan shape (gap 30, 12 heads: 92 KB boxes) 38 us against 44 us for
// mean_pool_seq_kernel; boxes of 6, 4 or 3 heads measured 39, 44 and 56 us.
// The prefix rows are copied first with plain 16-byte loads. A pooled row that
// runs past the end adds the final token for each missing row, as line 111's
// padding does; heads past H in the last head group are skipped.
constexpr int kMpStages = 2;
constexpr int kMpStageBytes = 96 * 1024;
constexpr int kMpMaxHeads = 12;  // consumer warps
constexpr size_t kMpSmem = 1024 + (size_t)kMpStages * kMpStageBytes + 256;

__global__ void __launch_bounds__((kMpMaxHeads + 1) * 32, 1)
    mean_pool_seq_tma_kernel(const __grid_constant__ CUtensorMap tm_x,
                             const __nv_bfloat16* __restrict__ x, int64_t xs0, int64_t xs1,
                             int64_t xs2, int H, int S, int pool, int prefix, int hb, int pooled,
                             int B, __nv_bfloat16* __restrict__ out, int64_t os0, int64_t os1,
                             int64_t os2) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // prefix rows, copied
  const int64_t n_pre = (int64_t)B * H * prefix * 16;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_pre;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int piece = (int)(i & 15);
    const int64_t r = i >> 4;
    const int row = (int)(r % prefix), bh = (int)(r / prefix);
    const int b = bh / H, h = bh - (bh / H) * H;
    *reinterpret_cast<uint4*>(out + b * os0 + h * os1 + (int64_t)row * os2 + piece * 8) =
        __ldg(reinterpret_cast<const uint4*>(x + b * xs0 + h * xs1 + (int64_t)row * xs2 +
                                             piece * 8));
  }
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kMpStages * kMpStageBytes);
  uint64_t* empty = full + kMpStages;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kMpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], hb);  // one arrival per consumer warp
    }
    fence_barrier_init();
  }
  __syncthreads();
  const int hgroups = (H + hb - 1) / hb;
  const int64_t n_items = (int64_t)B * pooled * hgroups;
  const uint32_t box_bytes = (uint32_t)hb * pool * 256;
  if (warp == hb) {  // producer
    if (lane == 0) {
      int k = 0;
      for (int64_t it = blockIdx.x; it < n_items; it += gridDim.x, ++k) {
        const int st = k % kMpStages;
        if (!mbar_wait_drain(&empty[st], ((uint32_t)(k / kMpStages) & 1u) ^ 1u)) break;
        const int hg = (int)(it % hgroups);
        const int64_t r = it / hgroups;
        const int orow = (int)(r % pooled), b = (int)(r / pooled);
        mbar_arrive_expect_tx(&full[st], box_bytes);
        tma_load_4d(&tm_x, &full[st], smem + (size_t)st * kMpStageBytes, 0, hg * hb,
                    prefix + orow * pool, b);
      }
      // this CTA's copies in flight complete before it exits
      for (int j = (k > kMpStages ? k - kMpStages : 0); j < k; ++j)
        mbar_wait_drain(&full[j % kMpStages], (uint32_t)(j / kMpStages) & 1u);
    }
    return;
  }
  if (warp > hb) return;
  const float inv = 1.0f / (float)pool;
  int k = 0;
  for (int64_t it = blockIdx.x; it < n_items; it += gridDim.x, ++k) {
    const int st = k % kMpStages;
    if (!mbar_wait_drain(&full[st], (uint32_t)(k / kMpStages) & 1u)) break;
    const int hg = (int)(it % hgroups);
    const int64_t r = it / hgroups;
    const int orow = (int)(r % pooled), b = (int)(r / pooled);
    const int h = hg * hb + warp;
    if (h < H) {
      const int lo = prefix + orow * pool;
      const int valid = min(pool, S - lo);
      // row t of head w sits at (t * hb + w) * 256 bytes
      const uint8_t* rows = smem + (size_t)st * kMpStageBytes + (size_t)warp * 256 + lane * 8;
      const size_t rstride = (size_t)hb * 256;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
      float b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
      int t = 0;
      for (; t + 1 < valid; t += 2) {
        const uint2 u = *reinterpret_cast<const uint2*>(rows + t * rstride);
        const uint2 w = *reinterpret_cast<const uint2*>(rows + (t + 1) * rstride);
        a0 += __uint_as_float(u.x << 16); a1 += __uint_as_float(u.x & 0xffff0000u);
        a2 += __uint_as_float(u.y << 16); a3 += __uint_as_float(u.y & 0xffff0000u);
        b0 += __uint_as_float(w.x << 16); b1 += __uint_as_float(w.x & 0xffff0000u);
        b2 += __uint_as_float(w.y << 16); b3 += __uint_as_float(w.y & 0xffff0000u);
      }
      if (t < valid) {
        const uint2 u = *reinterpret_cast<const uint2*>(rows + t * rstride);
        a0 += __uint_as_float(u.x << 16); a1 += __uint_as_float(u.x & 0xffff0000u);
        a2 += __uint_as_float(u.y << 16); a3 += __uint_as_float(u.y & 0xffff0000u);
      }
      a0 += b0; a1 += b1; a2 += b2; a3 += b3;
      if (valid < pool) {  // the final token stands in for each missing row
        const uint2 u = *reinterpret_cast<const uint2*>(rows + (valid - 1) * rstride);
        const float wgt = (float)(pool - valid);
        a0 += wgt * __uint_as_float(u.x << 16); a1 += wgt * __uint_as_float(u.x & 0xffff0000u);
        a2 += wgt * __uint_as_float(u.y << 16); a3 += wgt * __uint_as_float(u.y & 0xffff0000u);
      }
      uint2 o;
      o.x = pack_bf16x2(a0 * inv, a1 * inv);
      o.y = pack_bf16x2(a2 * inv, a3 * inv);
      *reinterpret_cast<uint2*>(out + b * os0 + h * os1 + (int64_t)(prefix + orow) * os2 +
                                lane * 4) = o;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
}

// _mix_attention_outputs, adaptive mode (sparse_attention.py:898-919).
// One thread per 8 output elements.
__global__ void mix_kernel(const __nv_bfloat16* __restrict__ os, int64_t a0, int64_t a1, int64_t a2,
                           const float* __restrict__ lse_s, const __nv_bfloat16* __restrict__ od,
                           int64_t b0, int64_t b1, int64_t b2, const float* __restrict__ lse_d,
                           int H, int S, int D, float log_gap, __nv_bfloat16* __restrict__ out,
                           int64_t c0, int64_t c1, int64_t c2, int64_t total_vec) {
  const int vpr = D >> 3;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total_vec;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int vc = (int)(i % vpr);
    const int64_t r = i / vpr;  // (b*H + h)*S + s
    const int s = (int)(r % S);
    const int64_t bh = r / S;
    const int h = (int)(bh % H);
    const int b = (int)(bh / H);
    const float ws = lse_s[r];
    const float wd = lse_d[r] + log_gap;
    const float m = fmaxf(ws, wd);
    const float es = expf(ws - m), ed = expf(wd - m);
    const float alpha = es / (es + ed);
    const uint4 va = __ldg(reinterpret_cast<const uint4*>(os + b * a0 + h * a1 + s * a2 + vc * 8));
    const uint4 vb = __ldg(reinterpret_cast<const uint4*>(od + b * b0 + h * b1 + s * b2 + vc * 8));
    const __nv_bfloat162* pa = reinterpret_cast<const __nv_bfloat162*>(&va);
    const __nv_bfloat162* pb = reinterpret_cast<const __nv_bfloat162*>(&vb);
    uint4 w;
    uint32_t* pw = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 fa = __bfloat1622float2(pa[e]);
      const float2 fb = __bfloat1622float2(pb[e]);
      pw[e] = pack_bf16x2(fa.x * alpha + fb.x * (1.f - alpha), fa.y * alpha + fb.y * (1.f - alpha));
    }
    *reinterpret_cast<uint4*>(out + b * c0 + h * c1 + s * c2 + vc * 8) = w;
  }
}

inline unsigned grid_for(int64_t n, int threads) {
  const int64_t g = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)sa::sm_count_current_device() * 16;
  return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

bool strides4_ok(const int64_t s[4]) {
  return s[3] == 1 && s[0] % 8 == 0 && s[1] % 8 == 0 && s[2] % 8 == 0;
}

}  // namespace misc
}  // namespace sa

extern "C" int sa_score_accumulate(const float* x, int64_t n, float* sum, float* sumsq, int first,
                                   cudaStream_t stream) {
  SA_CHECK_ARG(x && sum && sumsq, "sa_score_accumulate: null pointer argument");
  SA_CHECK_ARG(n >= 0, "sa_score_accumulate: n must be >= 0");
  if (n == 0) return SA_OK;
  sa::misc::accumulate_kernel<<<sa::misc::grid_for(n, 256), 256, 0, stream>>>(x, n, sum, sumsq,
                                                                              first);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_score_finalize(const float* sum, const float* sumsq, const float* count,
                                 float scalar_count, int64_t n, float* mean, float* std_out,
                                 int emit_variance, cudaStream_t stream) {
  SA_CHECK_ARG(sum && mean, "sa_score_finalize: null pointer argument");
  SA_CHECK_ARG(std_out == nullptr || sumsq != nullptr, "sa_score_finalize: std needs sumsq");
  SA_CHECK_ARG(count != nullptr || scalar_count > 0.f, "sa_score_finalize: count must be > 0");
  SA_CHECK_ARG(n >= 0, "sa_score_finalize: n must be >= 0");
  if (n == 0) return SA_OK;
  sa::misc::finalize_kernel<<<sa::misc::grid_for(n, 256), 256, 0, stream>>>(
      sum, sumsq, const_cast<float*>(count), scalar_count, n, mean, std_out, 0, emit_variance);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_score_accumulate_aligned(const float* scores, int H, int n_blocks,
                                           int image_blocks, int text_blocks, int total_blocks,
                                           float* sum, float* sumsq, float* presence, int first,
                                           cudaStream_t stream) {
  SA_CHECK_ARG(scores && sum && sumsq && presence,
               "sa_score_accumulate_aligned: null pointer argument");
  SA_CHECK_ARG(H >= 1 && image_blocks >= 0 && text_blocks >= 0,
               "sa_score_accumulate_aligned: bad sizes");
  SA_CHECK_ARG(n_blocks == image_blocks + text_blocks,
               "Unexpected Z-Image block score shape. Expected %dx%d, got %dx%d.",
               image_blocks + text_blocks, image_blocks + text_blocks, n_blocks, n_blocks);
  SA_CHECK_ARG(image_blocks + text_blocks <= total_blocks,
               "sa_score_accumulate_aligned: %d image + %d text blocks exceed the %d-block layout",
               image_blocks, text_blocks, total_blocks);
  const int64_t total = (int64_t)H * total_blocks * total_blocks;
  if (total == 0) return SA_OK;
  sa::misc::accumulate_aligned_kernel<<<sa::misc::grid_for(total, 256), 256, 0, stream>>>(
      scores, H, n_blocks, image_blocks, total_blocks - text_blocks, total_blocks, sum, sumsq,
      presence, first);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_score_finalize_presence(const float* sum, const float* sumsq, float* presence,
                                          int64_t n, float* mean, float* std_out,
                                          int emit_variance, cudaStream_t stream) {
  SA_CHECK_ARG(sum && sumsq && presence && mean,
               "sa_score_finalize_presence: null pointer argument");
  SA_CHECK_ARG(n >= 0, "sa_score_finalize_presence: n must be >= 0");
  if (n == 0) return SA_OK;
  sa::misc::finalize_kernel<<<sa::misc::grid_for(n, 256), 256, 0, stream>>>(
      sum, sumsq, presence, 0.f, n, mean, std_out, 1, emit_variance);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_mean_pool_seq(const void* x, const int64_t x_strides[4], int B, int H, int S,
                                int D, int pool, int prefix, void* out,
                                const int64_t o_strides[4], cudaStream_t stream) {
  SA_CHECK_ARG(x && out && x_strides && o_strides, "sa_mean_pool_seq: null pointer argument");
  SA_CHECK_ARG(B >= 1 && H >= 1 && S >= 1 && pool >= 1, "sa_mean_pool_seq: bad sizes");
  SA_CHECK_ARG(D >= 8 && D <= 256 && D % 8 == 0, "sa_mean_pool_seq: D must be a multiple of 8 in [8,256]");
  SA_CHECK_ARG(sa::misc::strides4_ok(x_strides) && sa::misc::strides4_ok(o_strides),
               "sa_mean_pool_seq: stride(dim) must be 1 and other strides multiples of 8");
  SA_CHECK_ARG(((uintptr_t)x | (uintptr_t)out) % 16 == 0, "sa_mean_pool_seq: 16-byte alignment");
  SA_CHECK_ARG((int64_t)B * H <= 65535, "sa_mean_pool_seq: B*H too large");
  prefix = prefix < 0 ? 0 : (prefix > S ? S : prefix);
  const int out_rows = (prefix >= S) ? S : prefix + (S - prefix + pool - 1) / pool;
  const int threads = (D / 8) * 8;
  // prefix >= S means "no pooling" (line 108-109): every row is a prefix row.
  const int eff_prefix = prefix >= S ? S : prefix;
  // heads per box: as many as fit a stage, at most one warp each
  const int hb = D == 128 ? min(min(H, sa::misc::kMpMaxHeads),
                                sa::misc::kMpStageBytes / (pool * 256))
                          : 0;
  // (a box is at most 256 rows, and no taller than the sequence)
  if (D == 128 && pool <= 256 && pool <= S && hb >= 1 && prefix < S) {
    sa::EncodeTiledFn enc = sa::encode_tiled_fn();
    if (enc == nullptr) return SA_ECUDA;
    const int pooled = (S - prefix + pool - 1) / pool;
    CUtensorMap map;
    cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)B};
    cuuint64_t gst[3] = {(cuuint64_t)x_strides[1] * 2, (cuuint64_t)x_strides[2] * 2,
                         (cuuint64_t)x_strides[0] * 2};
    cuuint32_t box[4] = {128, (cuuint32_t)hb, (cuuint32_t)pool, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(x), dims, gst,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      sa::set_error("cuTensorMapEncodeTiled (mean pool) failed (CUresult %d)", (int)r);
      return SA_ECUDA;
    }
    if (int rc = sa::func_attr_once((const void*)sa::misc::mean_pool_seq_tma_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)sa::misc::kMpSmem);
        rc != SA_OK)
      return rc;
    const int64_t items = (int64_t)B * pooled * ((H + hb - 1) / hb);
    const int sms = sa::sm_count_current_device();
    const int grid = (int)(items < sms ? (items > 0 ? items : 1) : sms);
    sa::misc::mean_pool_seq_tma_kernel<<<grid, (hb + 1) * 32, sa::misc::kMpSmem, stream>>>(
        map, reinterpret_cast<const __nv_bfloat16*>(x), x_strides[0], x_strides[1], x_strides[2],
        H, S, pool, prefix, hb, pooled, B, reinterpret_cast<__nv_bfloat16*>(out), o_strides[0],
        o_strides[1], o_strides[2]);
    SA_CUDA_TRY(cudaGetLastError());
    return SA_OK;
  }
  sa::misc::mean_pool_seq_kernel<<<dim3(out_rows, B * H), threads, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(x), x_strides[0], x_strides[1], x_strides[2], H, S, D,
      pool, eff_prefix, reinterpret_cast<__nv_bfloat16*>(out), o_strides[0], o_strides[1],
      o_strides[2]);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_mix_outputs(const void* o_s, const int64_t os_strides[4], const float* lse_s,
                              const void* o_d, const int64_t od_strides[4], const float* lse_d,
                              int B, int H, int S, int D, float log_gap, void* out,
                              const int64_t o_strides[4], cudaStream_t stream) {
  SA_CHECK_ARG(o_s && o_d && lse_s && lse_d && out && os_strides && od_strides && o_strides,
               "sa_mix_outputs: null pointer argument");
  SA_CHECK_ARG(B >= 1 && H >= 1 && S >= 1 && D % 8 == 0 && D >= 8, "sa_mix_outputs: bad sizes");
  SA_CHECK_ARG(sa::misc::strides4_ok(os_strides) && sa::misc::strides4_ok(od_strides) &&
                   sa::misc::strides4_ok(o_strides),
               "sa_mix_outputs: stride(dim) must be 1 and other strides multiples of 8");
  SA_CHECK_ARG(((uintptr_t)o_s | (uintptr_t)o_d | (uintptr_t)out) % 16 == 0,
               "sa_mix_outputs: 16-byte alignment");
  const int64_t total_vec = (int64_t)B * H * S * (D / 8);
  sa::misc::mix_kernel<<<sa::misc::grid_for(total_vec, 256), 256, 0, stream>>>(
      reinterpret_cast<const __nv_bfloat16*>(o_s), os_strides[0], os_strides[1], os_strides[2],
      lse_s, reinterpret_cast<const __nv_bfloat16*>(o_d), od_strides[0], od_strides[1],
      od_strides[2], lse_d, H, S, D, log_gap, reinterpret_cast<__nv_bfloat16*>(out), o_strides[0],
      o_strides[1], o_strides[2], total_vec);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}
