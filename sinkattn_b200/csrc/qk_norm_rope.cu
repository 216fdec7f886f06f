// qk_norm_rope.cu — the producer of Q and K for the sink attention: RMSNorm
// over the full hidden dimension followed by the rotary embedding, for Q and
// K in one pass over HBM.
//
// Replaces the two steps of the Wan attention processor
// (wanx/runtime/sink_sparse_wan.py:300-315, wanx/runtime/fast_misc.py:834-864
// and 216-234):
//   y = bf16( (x * rstd) * w ),  rstd = 1 / sqrt(sum(x^2) / hidden + eps)
//       (the RMSNorm of fast_misc.py:306-340, computed on fp32 values)
//   per head and per pair p = (2i, 2i+1) of its D channels, at position s:
//   out_2i   = bf16( y_2i * cos[s,i] - y_2i+1 * sin[s,i] )
//   out_2i+1 = bf16( y_2i * sin[s,i] + y_2i+1 * cos[s,i] )
//       (the complex product of fast_misc.py:173-194 and 432-500)
// The normalised value is rounded to bf16 before the rotation, as it is
// between the reference's two kernels.
//
// One warp per token row: the Q and K rows (hidden bf16 values each, 3 KB for
// Wan) are held in registers as 16-byte vectors, the sums of squares are warp
// reductions, and both rows are written back with 16-byte stores.
// Memory-bound: 2 x (read + write) hidden x 2 bytes per token.

#include <math.h>

#include "sa_common.cuh"

namespace sa {
namespace qkrope {

constexpr int kMaxVecPerLane = 16;  // hidden <= 32 lanes x 16 vectors x 8 = 4096

template <int VPL>
__device__ __forceinline__ float row_rstd(const uint4 (&raw)[VPL], int count, int hidden,
                                          float eps) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if (i >= count) continue;
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw[i]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(p[e]);
      ss = fmaf(f.x, f.x, ss);
      ss = fmaf(f.y, f.y, ss);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hidden), eps)));
}

__device__ __forceinline__ void load_w8(const void* w, int w_is_bf16, int c0, float* out) {
  if (w == nullptr) {
#pragma unroll
    for (int e = 0; e < 8; ++e) out[e] = 1.f;
  } else if (w_is_bf16) {
    const uint4 v = reinterpret_cast<const uint4*>(w)[c0 >> 3];
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(p[e]);
      out[2 * e] = f.x;
      out[2 * e + 1] = f.y;
    }
  } else {
    const float4 a = reinterpret_cast<const float4*>(w)[c0 >> 2];
    const float4 b = reinterpret_cast<const float4*>(w)[(c0 >> 2) + 1];
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
  }
}

// Normalise, round to bf16 and rotate 8 channels (4 pairs) of one row.
__device__ __forceinline__ uint4 norm_rope8(const uint4 raw, float rstd, const float* w,
                                            const float* cs, const float* sn) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw);
  uint4 res;
  uint32_t* r32 = reinterpret_cast<uint32_t*>(&res);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(p[e]);
    // the RMSNorm output as the reference stores it (bf16)
    float y0 = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(f.x, rstd), w[2 * e])));
    float y1 = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(f.y, rstd), w[2 * e + 1])));
    if (cs != nullptr) {
      const float o0 = fmaf(y0, cs[e], -__fmul_rn(y1, sn[e]));
      const float o1 = fmaf(y0, sn[e], __fmul_rn(y1, cs[e]));
      y0 = o0;
      y1 = o1;
    }
    const __nv_bfloat162 ob = __floats2bfloat162_rn(y0, y1);
    r32[e] = *reinterpret_cast<const uint32_t*>(&ob);
  }
  return res;
}

// grid: ceil(rows / 8) CTAs of 8 warps; warp w of CTA c handles token row
// 8c + w of Q and of K. Both rows are loaded before either is reduced, and
// the weights and the position's cos/sin are read as 16-byte vectors shared
// by the two tensors.
template <int VPL>
__global__ void __launch_bounds__(256)
    qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ q_in, const __nv_bfloat16* __restrict__ k_in,
                        int64_t qs_in, int64_t ks_in, int rows, int S, int hidden, int D,
                        const void* __restrict__ wq, const void* __restrict__ wk, int w_is_bf16,
                        float eps, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                        int64_t fs, __nv_bfloat16* __restrict__ q_out,
                        __nv_bfloat16* __restrict__ k_out, int64_t qs_out, int64_t ks_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int nvec = hidden >> 3;
  const int count = (nvec - lane + 31) >> 5;  // vectors of this lane
  const uint4* qv = reinterpret_cast<const uint4*>(q_in + row * qs_in);
  const uint4* kv = reinterpret_cast<const uint4*>(k_in + row * ks_in);
  uint4 rq[VPL], rk[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if (i < count) {
      rq[i] = qv[lane + 32 * i];
      rk[i] = kv[lane + 32 * i];
    }
  }
  const float rstd_q = row_rstd<VPL>(rq, count, hidden, eps);
  const float rstd_k = row_rstd<VPL>(rk, count, hidden, eps);
  const int s = (int)(row % S);
  const float* crow = cos_t != nullptr ? cos_t + (int64_t)s * fs : nullptr;
  const float* srow = sin_t != nullptr ? sin_t + (int64_t)s * fs : nullptr;
  uint4* qo = reinterpret_cast<uint4*>(q_out + row * qs_out);
  uint4* ko = reinterpret_cast<uint4*>(k_out + row * ks_out);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if (i >= count) continue;
    const int v = lane + 32 * i;
    const int c0 = v * 8;
    float cs[4], sn[4];
    const float* csp = nullptr;
    const float* snp = nullptr;
    if (crow != nullptr) {
      const int p0 = (c0 % D) >> 1;  // 4 consecutive pairs, 16-byte aligned
      const float4 c4 = *reinterpret_cast<const float4*>(crow + p0);
      const float4 s4 = *reinterpret_cast<const float4*>(srow + p0);
      cs[0] = c4.x; cs[1] = c4.y; cs[2] = c4.z; cs[3] = c4.w;
      sn[0] = s4.x; sn[1] = s4.y; sn[2] = s4.z; sn[3] = s4.w;
      csp = cs;
      snp = sn;
    }
    float w8[8];
    load_w8(wq, w_is_bf16, c0, w8);
    qo[v] = norm_rope8(rq[i], rstd_q, w8, csp, snp);
    load_w8(wk, w_is_bf16, c0, w8);
    ko[v] = norm_rope8(rk[i], rstd_k, w8, csp, snp);
  }
}

}  // namespace qkrope
}  // namespace sa

extern "C" int sa_qk_norm_rope(const void* q_in, const void* k_in, int64_t q_in_row_stride,
                               int64_t k_in_row_stride, int rows, int S, int hidden, int D,
                               const void* w_q, const void* w_k, int w_is_bf16, float eps,
                               const float* cos_table, const float* sin_table,
                               int64_t freq_row_stride, void* q_out, void* k_out,
                               int64_t q_out_row_stride, int64_t k_out_row_stride,
                               cudaStream_t stream) {
  using namespace sa::qkrope;
  SA_CHECK_ARG(q_in && k_in && q_out && k_out, "sa_qk_norm_rope: null tensor pointer");
  SA_CHECK_ARG(rows >= 0 && S >= 1 && D >= 8 && D % 8 == 0,
               "sa_qk_norm_rope: bad sizes (D must be a multiple of 8)");
  SA_CHECK_ARG(hidden >= 8 && hidden % 8 == 0 && hidden % D == 0 && hidden <= 32 * 8 * kMaxVecPerLane,
               "sa_qk_norm_rope: hidden (%d) must be a multiple of 8 and of D (%d), at most %d",
               hidden, D, 32 * 8 * kMaxVecPerLane);
  SA_CHECK_ARG((cos_table == nullptr) == (sin_table == nullptr),
               "sa_qk_norm_rope: cos and sin tables go together");
  SA_CHECK_ARG(cos_table == nullptr ||
                   (freq_row_stride >= D / 2 && freq_row_stride % 4 == 0 &&
                    (((uintptr_t)cos_table | (uintptr_t)sin_table) & 15) == 0),
               "sa_qk_norm_rope: frequency rows need D/2 entries, a stride that is a multiple "
               "of 4 and 16-byte aligned tables");
  SA_CHECK_ARG(((q_in_row_stride | k_in_row_stride | q_out_row_stride | k_out_row_stride) & 7) == 0,
               "sa_qk_norm_rope: row strides must be multiples of 8 elements");
  SA_CHECK_ARG((((uintptr_t)q_in | (uintptr_t)k_in | (uintptr_t)q_out | (uintptr_t)k_out) & 15) == 0,
               "sa_qk_norm_rope: tensors must be 16-byte aligned");
  SA_CHECK_ARG(w_q == nullptr || (((uintptr_t)w_q | (uintptr_t)w_k) & 15) == 0,
               "sa_qk_norm_rope: weights must be 16-byte aligned");
  SA_CHECK_ARG((w_q == nullptr) == (w_k == nullptr), "sa_qk_norm_rope: weights go together");
  if (rows == 0) return SA_OK;
  const int vpl = (hidden / 8 + 31) / 32;
  const dim3 grid((unsigned)((rows + 7) / 8));
  const auto* qi = reinterpret_cast<const __nv_bfloat16*>(q_in);
  const auto* ki = reinterpret_cast<const __nv_bfloat16*>(k_in);
  auto* qo = reinterpret_cast<__nv_bfloat16*>(q_out);
  auto* ko = reinterpret_cast<__nv_bfloat16*>(k_out);
#define SA_QKROPE_LAUNCH(V)                                                                    \
  qk_norm_rope_kernel<V><<<grid, 256, 0, stream>>>(qi, ki, q_in_row_stride, k_in_row_stride,   \
                                                   rows, S, hidden, D, w_q, w_k, w_is_bf16, eps, \
                                                   cos_table, sin_table, freq_row_stride, qo,  \
                                                   ko, q_out_row_stride, k_out_row_stride)
  if (vpl <= 2) SA_QKROPE_LAUNCH(2);
  else if (vpl <= 6) SA_QKROPE_LAUNCH(6);
  else if (vpl <= 8) SA_QKROPE_LAUNCH(8);
  else SA_QKROPE_LAUNCH(16);
#undef SA_QKROPE_LAUNCH
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}
