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

// bf16 pair (low half = even channel) -> two fp32 values, exact.
__device__ __forceinline__ uint64_t bf16x2_to_f2(uint32_t w) {
  return f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

template <int VPL>
__device__ __forceinline__ float row_rstd(const uint4 (&raw)[VPL], int count, int hidden,
                                          float eps) {
  // even and odd channels accumulate in the two halves of one f32x2 sum
  uint64_t ss2 = f2_pack(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if (i >= count) continue;
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&raw[i]);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const uint64_t x2 = bf16x2_to_f2(w[e]);
      ss2 = f2_fma(x2, x2, ss2);
    }
  }
  float s0, s1;
  f2_unpack(ss2, s0, s1);
  float ss = s0 + s1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hidden), eps)));
}

// Weights of channels c0..c0+7 as four f32x2 pairs (all 1 without weights).
__device__ __forceinline__ void load_w8(const void* w, int w_is_bf16, int c0, uint64_t (&out)[4]) {
  if (w == nullptr) {
#pragma unroll
    for (int e = 0; e < 4; ++e) out[e] = f2_pack(1.f, 1.f);
  } else if (w_is_bf16) {
    const uint4 v = reinterpret_cast<const uint4*>(w)[c0 >> 3];
    const uint32_t* p = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int e = 0; e < 4; ++e) out[e] = bf16x2_to_f2(p[e]);
  } else {
    const float4 a = reinterpret_cast<const float4*>(w)[c0 >> 2];
    const float4 b = reinterpret_cast<const float4*>(w)[(c0 >> 2) + 1];
    out[0] = f2_pack(a.x, a.y); out[1] = f2_pack(a.z, a.w);
    out[2] = f2_pack(b.x, b.y); out[3] = f2_pack(b.z, b.w);
  }
}

// Normalise, round to bf16 and rotate 8 channels (4 pairs) of one row, on
// f32x2 pairs. Per lane this is the scalar arithmetic
//   y = bf16((x * rstd) * w),
//   out_even = fma(y_even, cos, -(y_odd * sin)), out_odd = fma(y_even, sin, y_odd * cos),
// with csn[e] = (cos, sin) and nsc[e] = (-sin, cos): -(y_odd*sin) = y_odd*(-sin)
// exactly, so the packed products round exactly as the scalar ones.
__device__ __forceinline__ uint4 norm_rope8(const uint4 raw, uint64_t rstd2,
                                            const uint64_t (&w2)[4], bool rope,
                                            const uint64_t (&csn)[4], const uint64_t (&nsc)[4]) {
  const uint32_t* p = reinterpret_cast<const uint32_t*>(&raw);
  uint4 res;
  uint32_t* r32 = reinterpret_cast<uint32_t*>(&res);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float a0, a1;
    f2_unpack(f2_mul(f2_mul(bf16x2_to_f2(p[e]), rstd2), w2[e]), a0, a1);
    // the RMSNorm output as the reference stores it (bf16)
    const uint32_t yb = pack_bf16x2(a0, a1);
    if (rope) {
      const float y0 = __uint_as_float(yb << 16);
      const float y1 = __uint_as_float(yb & 0xffff0000u);
      const uint64_t u = f2_mul(f2_pack(y1, y1), nsc[e]);
      float o0, o1;
      f2_unpack(f2_fma(f2_pack(y0, y0), csn[e], u), o0, o1);
      r32[e] = pack_bf16x2(o0, o1);
    } else {
      r32[e] = yb;
    }
  }
  return res;
}

// grid: one single-warp CTA per token row, which handles that row of Q and
// of K. Both rows are loaded (streaming, evict-first) before either is
// reduced, and the weights and the position's cos/sin are read as 16-byte
// vectors shared by the two tensors. Up to hidden = 1536 (6 vectors per lane)
// the register budget is capped for 24 resident warps per SM: the extra rows
// in flight are worth more than the few spilled registers, and single-warp
// CTAs retire and refill the SM without waiting for slower sibling warps.
template <int VPL>
__global__ void __launch_bounds__(32, (VPL <= 6 ? 24 : 1))
    qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ q_in, const __nv_bfloat16* __restrict__ k_in,
                        int64_t qs_in, int64_t ks_in, int rows, int S, int hidden, int D,
                        const void* __restrict__ wq, const void* __restrict__ wk, int w_is_bf16,
                        float eps, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                        int64_t fs, __nv_bfloat16* __restrict__ q_out,
                        __nv_bfloat16* __restrict__ k_out, int64_t qs_out, int64_t ks_out) {
  const int lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x;
  if (row >= rows) return;
  const int nvec = hidden >> 3;
  const int count = (nvec - lane + 31) >> 5;  // vectors of this lane
  const uint4* qv = reinterpret_cast<const uint4*>(q_in + row * qs_in);
  const uint4* kv = reinterpret_cast<const uint4*>(k_in + row * ks_in);
  uint4 rq[VPL], rk[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if (i < count) {
      rq[i] = __ldcs(qv + lane + 32 * i);
      rk[i] = __ldcs(kv + lane + 32 * i);
    }
  }
  const uint64_t rstd_q = [&] { const float r = row_rstd<VPL>(rq, count, hidden, eps); return f2_pack(r, r); }();
  const uint64_t rstd_k = [&] { const float r = row_rstd<VPL>(rk, count, hidden, eps); return f2_pack(r, r); }();
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
    uint64_t csn[4], nsc[4];
    const bool rope = crow != nullptr;
    if (rope) {
      const int p0 = (c0 % D) >> 1;  // 4 consecutive pairs, 16-byte aligned
      const float4 c4 = *reinterpret_cast<const float4*>(crow + p0);
      const float4 s4 = *reinterpret_cast<const float4*>(srow + p0);
      csn[0] = f2_pack(c4.x, s4.x); csn[1] = f2_pack(c4.y, s4.y);
      csn[2] = f2_pack(c4.z, s4.z); csn[3] = f2_pack(c4.w, s4.w);
      nsc[0] = f2_pack(-s4.x, c4.x); nsc[1] = f2_pack(-s4.y, c4.y);
      nsc[2] = f2_pack(-s4.z, c4.z); nsc[3] = f2_pack(-s4.w, c4.w);
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) csn[e] = nsc[e] = 0ull;
    }
    uint64_t w2[4];
    load_w8(wq, w_is_bf16, c0, w2);
    __stcs(qo + v, norm_rope8(rq[i], rstd_q, w2, rope, csn, nsc));
    load_w8(wk, w_is_bf16, c0, w2);
    __stcs(ko + v, norm_rope8(rk[i], rstd_k, w2, rope, csn, nsc));
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
  const dim3 grid((unsigned)rows);
  const auto* qi = reinterpret_cast<const __nv_bfloat16*>(q_in);
  const auto* ki = reinterpret_cast<const __nv_bfloat16*>(k_in);
  auto* qo = reinterpret_cast<__nv_bfloat16*>(q_out);
  auto* ko = reinterpret_cast<__nv_bfloat16*>(k_out);
#define SA_QKROPE_LAUNCH(V)                                                                    \
  qk_norm_rope_kernel<V><<<grid, 32, 0, stream>>>(qi, ki, q_in_row_stride, k_in_row_stride,   \
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
