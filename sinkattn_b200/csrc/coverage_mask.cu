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

#include "sa_common.cuh"

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

__device__ __forceinline__ uint32_t float_to_ordered(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ordered_to_float(uint32_t o) {
  const uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
  return __uint_as_float(u);
}

__device__ __forceinline__ double warp_sum_f64(double x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}
__device__ __forceinline__ int warp_min_i(int x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = min(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}
__device__ __forceinline__ int warp_max_i(int x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x = max(x, __shfl_xor_sync(0xffffffffu, x, o));
  return x;
}

// ulp exponent of a positive finite float: the value is a multiple of 2^q.
__device__ __forceinline__ int ulp_exp(float v) {
  const int e = (int)((__float_as_uint(v) >> 23) & 0xff);
  return (e == 0 ? -126 : e - 127) - 23;
}

__device__ __forceinline__ float ulp_of(float v) {
  const float a = fabsf(v);
  return nextafterf(a, INFINITY) - a;
}

template <int NPAD>
__global__ void coverage_mask_kernel(const Params p) {
  constexpr int E = NPAD / 32;  // sorted positions per lane (contiguous chunk)
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
  uint8_t* out = p.mask + grow * p.nk;
  const int nk = p.nk;
  const int T = p.T;
  const bool video = p.mode == SA_COVERAGE_VIDEO_RESIDUAL;

  // Rows fully required by the text rule: all ones.
  if (T > 0 && row < T) {
    for (int j = lane; j < nk; j += 32) out[j] = 1;
    if (p.flags != nullptr && lane == 0) p.flags[grow] = 0;
    return;
  }
  const int c_lo = video ? T : 0;  // first column taking part in the coverage step

  // ---- load, required set, row sums ---------------------------------------
  // Participating columns (j >= c_lo) get a sort key ~ordered(candidate);
  // required columns enter as -inf (joint mode). Others get key 0xFFFFFFFF
  // (sorted last) and candidate value NaN.
  double tot = 0.0, sel = 0.0;
  int n_cand_local = 0;  // non-required participating columns (candidate_counts, line 348)
  for (int j = lane; j < NPAD; j += 32) {
    uint32_t key = 0xFFFFFFFFu;
    float cv = __int_as_float(0x7fc00000);
    if (j < nk && j >= c_lo) {
      const float v = s[j];
      const bool req = (j < T) || (p.force_sink && j == 0);
      tot += (double)v;
      if (!video && req) sel += (double)v;
      if (video || !req) ++n_cand_local;
      cv = (!video && req) ? -INFINITY : v;
      key = ~float_to_ordered(cv);
    }
    skey[j] = key;
    cval[j] = cv;
  }
  tot = warp_sum_f64(tot);
  sel = warp_sum_f64(sel);
  float total = p.row_total != nullptr ? p.row_total[grow] : (float)tot;
  const float selected = video ? 0.f : (p.row_selected != nullptr ? p.row_selected[grow] : (float)sel);
  total = fmaxf(total, 1e-6f);
  const float cov = fminf(fmaxf(p.coverage, 0.f), 1.f);
  float target = __fmul_rn(cov, total);
  if (!video) target = fmaxf(__fsub_rn(target, selected), 0.f);
  const int n_cand = __reduce_add_sync(0xffffffffu, (unsigned)n_cand_local);
  __syncwarp();

  // ---- sort the 32-bit value keys ascending (= values descending) ----------
  // Equal values may land in any order: the cumulative sums do not depend on
  // it, and the kept set below is chosen by value and index, not position.
  if constexpr (NPAD <= 256) {
    constexpr int R = NPAD / 32;
    uint32_t reg[R];
#pragma unroll
    for (int i = 0; i < R; ++i) reg[i] = skey[lane + 32 * i];
#pragma unroll
    for (int k = 2; k <= NPAD; k <<= 1) {
#pragma unroll
      for (int j = k >> 1; j > 0; j >>= 1) {
        if (j >= 32) {
          const int js = j >> 5;
#pragma unroll
          for (int i = 0; i < R; ++i) {
            const int i2 = i ^ js;
            if (i2 > i) {
              const bool up = (((lane + 32 * i) & k) == 0);
              const uint32_t a = reg[i], c = reg[i2];
              const uint32_t lo = min(a, c), hi = max(a, c);
              reg[i] = up ? lo : hi;
              reg[i2] = up ? hi : lo;
            }
          }
        } else {
          const bool lower = (lane & j) == 0;
#pragma unroll
          for (int i = 0; i < R; ++i) {
            const uint32_t a = reg[i];
            const uint32_t c = __shfl_xor_sync(0xffffffffu, a, j);
            const bool up = (((lane + 32 * i) & k) == 0);
            reg[i] = (lower == up) ? min(a, c) : max(a, c);
          }
        }
      }
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < R; ++i) skey[lane + 32 * i] = reg[i];
    __syncwarp();
  } else {
#pragma unroll 1
    for (int k = 2; k <= NPAD; k <<= 1) {
#pragma unroll 1
      for (int j = k >> 1; j > 0; j >>= 1) {
        for (int i = lane; i < NPAD; i += 32) {
          const int partner = i ^ j;
          if (partner > i) {
            const uint32_t a = skey[i], b = skey[partner];
            const bool up = (i & k) == 0;
            if ((a > b) == up) {
              skey[i] = b;
              skey[partner] = a;
            }
          }
        }
        __syncwarp();
      }
    }
  }

  // sorted value at position r (0 for padding / non-finite, as line 345 does)
  auto sorted_val0 = [&](int r) -> float {
    const uint32_t key = skey[r];
    if (key == 0xFFFFFFFFu) return 0.f;
    const float v = ordered_to_float(~key);
    return isfinite(v) ? v : 0.f;
  };

  // ---- exactness test, cumulative sums ---------------------------------------
  // Lane owns sorted positions [lane*E, lane*E + E).
  int min_q = INT_MAX;
  bool nonneg = true;
  double local = 0.0;
  for (int e = 0; e < E; ++e) {
    const float v = sorted_val0(lane * E + e);
    if (v < 0.f) nonneg = false;
    if (v > 0.f) min_q = min(min_q, ulp_exp(v));
    local += (double)v;
  }
  const bool all_nonneg = __all_sync(0xffffffffu, nonneg);
  min_q = warp_min_i(min_q);
  const double sum_all = warp_sum_f64(local);
  // Exact when every partial sum is representable: all terms multiples of 2^q
  // and the (upper-bounded) total below 2^(q+52).
  const bool exact =
      all_nonneg && (min_q == INT_MAX || (sum_all < ldexp(1.0, min_q + 52)));

  int first = INT_MAX;  // first sorted position with cum >= target
  float cum_at_first = 0.f, cum_before_first = 0.f;
  if (exact) {
    // exclusive prefix of the lane sums (exact, so order does not matter)
    double pre = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double t = __shfl_up_sync(0xffffffffu, pre, o);
      if (lane >= o) pre += t;
    }
    double run = pre - local;
    float prev_f = lane == 0 ? 0.f : (float)run;
    for (int e = 0; e < E; ++e) {
      const int r = lane * E + e;
      run += (double)sorted_val0(r);
      const float cf = (float)run;
      if (cf >= target && first == INT_MAX) {
        first = r;
        cum_at_first = cf;
        cum_before_first = prev_f;
      }
      prev_f = cf;
    }
    const int f = warp_min_i(first);
    const int owner = __ffs(__ballot_sync(0xffffffffu, first == f && f != INT_MAX)) - 1;
    if (f != INT_MAX && owner >= 0) {
      cum_at_first = __shfl_sync(0xffffffffu, cum_at_first, owner);
      cum_before_first = __shfl_sync(0xffffffffu, cum_before_first, owner);
    }
    first = f;
  } else {
    if (lane == 0) {
      double run = 0.0;
      float prev_f = 0.f;
      for (int r = 0; r < NPAD; ++r) {
        run += (double)sorted_val0(r);
        const float cf = (float)run;
        if (cf >= target) {
          first = r;
          cum_at_first = cf;
          cum_before_first = prev_f;
          break;
        }
        prev_f = cf;
      }
    }
    first = __shfl_sync(0xffffffffu, first, 0);
    cum_at_first = __shfl_sync(0xffffffffu, cum_at_first, 0);
    cum_before_first = __shfl_sync(0xffffffffu, cum_before_first, 0);
  }

  const int n_sortable = video ? (nk - c_lo) : nk;  // k is clamped to this
  int kcut;
  if (target > 1e-6f) {
    kcut = first != INT_MAX ? first + 1 : n_cand;
  } else {
    kcut = 0;
  }
  kcut = max(0, min(kcut, n_sortable));

  // ---- assemble the row ------------------------------------------------
  // The first kcut positions of the stable (value desc, index asc) order are
  // every candidate above the cut value plus, among candidates equal to it,
  // the lowest indices.
  uint32_t key_cut = 0xFFFFFFFFu;
  int m_eq = 0;
  if (kcut > 0) {
    key_cut = skey[kcut - 1];
    int gt = 0;
    for (int j = lane; j < nk; j += 32) {
      const float cv = cval[j];
      if (cv == cv && ~float_to_ordered(cv) < key_cut) ++gt;
    }
    gt = __reduce_add_sync(0xffffffffu, (unsigned)gt);
    m_eq = kcut - gt;
  }
  int any = 0;
  int eq_seen = 0;
  for (int base = 0; base < nk; base += 32) {
    const int j = base + lane;
    bool keep = false;
    bool eq = false;
    if (j < nk) {
      const bool req = (j < T) || (!video && p.force_sink && j == 0);
      const float cv = cval[j];
      const bool part = (cv == cv) && cv != -INFINITY;
      if (part && kcut > 0) {
        const uint32_t key = ~float_to_ordered(cv);
        eq = key == key_cut;
        keep = key < key_cut;
      }
      keep = keep || req;
      if (!video && p.keep_diag && j == row) keep = true;
    }
    const uint32_t bal = __ballot_sync(0xffffffffu, eq);
    if (eq && eq_seen + __popc(bal & ((1u << lane) - 1u)) < m_eq) keep = true;
    eq_seen += __popc(bal);
    if (j < nk) out[j] = keep ? 1 : 0;
    any |= keep ? 1 : 0;
  }
  any = __any_sync(0xffffffffu, any);
  uint32_t flags = 0;
  if (!any) {
    flags |= SA_ROW_EMPTY_FALLBACK;
    // video mode: argmax over the full row (line 329); joint: the first entry
    // of the candidate sort (line 373), lowest index among equal maxima.
    float best = -INFINITY;
    int top = INT_MAX;
    for (int j = lane; j < nk; j += 32) {
      const float v = video ? s[j] : cval[j];
      if (v == v && (top == INT_MAX || v > best)) {
        best = v;
        top = j;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int ot = __shfl_xor_sync(0xffffffffu, top, o);
      if (ot != INT_MAX && (top == INT_MAX || ob > best || (ob == best && ot < top))) {
        best = ob;
        top = ot;
      }
    }
    if (top == INT_MAX) top = 0;
    if (lane == 0) out[top] = 1;
  }

  if (p.flags != nullptr && lane == 0) {
    auto sorted_val = [&](int r) -> float {
      const uint32_t key = skey[r];
      if (key == 0xFFFFFFFFu) return NAN;
      return ordered_to_float(~key);
    };
    // A tie straddling the cut (or the top-1 fallback) makes torch's order matter.
    const int cut = (flags & SA_ROW_EMPTY_FALLBACK) ? 1 : kcut;
    if (cut > 0 && cut < n_sortable) {
      const float a = sorted_val(cut - 1), b = sorted_val(cut);
      if (a == b && a != -INFINITY) flags |= SA_ROW_TIE_AT_CUT;
    }
    if (p.row_total == nullptr && target > 1e-6f && first != INT_MAX) {
      const float u = 2.f * ulp_of(target);
      if (cum_at_first - target <= u || (first > 0 && target - cum_before_first <= u))
        flags |= SA_ROW_NEAR_TARGET;
    }
    p.flags[grow] = (int32_t)flags;
  }
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
