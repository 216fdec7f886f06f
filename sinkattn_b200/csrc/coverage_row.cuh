// coverage_row.cuh — one row of the minimal-coverage block mask, run by one
// warp. Shared by the standalone coverage kernel (coverage_mask.cu) and the
// fused calibration-layer kernel (pool_scores.cu), so both take the same
// decisions bit for bit. The rule, its exactness argument and the row flags
// are described at the top of coverage_mask.cu
// (sinkattention/sparse_attention.py:241-376).
#pragma once

#include <float.h>
#include <limits.h>
#include <math.h>

#include "sa_common.cuh"

namespace sa {
namespace cov {

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

// What a row needs to know about the rule.
struct RowSpec {
  int nk;          // columns
  int T;           // text blocks (required rows / columns), already clamped
  int mode;        // SA_COVERAGE_JOINT or SA_COVERAGE_VIDEO_RESIDUAL (only with T > 0)
  int keep_diag;   // keep (row, row) in joint mode
  int force_sink;  // key block 0 joins the required set (joint mode)
  float coverage;  // unclamped; clamped to [0, 1] here as line 340 does
};

// Row `row` of the rule, executed by all 32 lanes of one warp.
//   s            the row's nk fp32 scores (global or shared memory)
//   total_in     the caller's fp32 row total (torch's sum order), or nullptr
//                to take the fp64 sum rounded to fp32
//   selected_in  the caller's fp32 sum over required columns, or nullptr
//   skey, cval   NPAD words each of this warp's shared-memory scratch
//   out          nk bytes of the mask row
//   flag         nullable; receives the row's SA_ROW_* bits
template <int NPAD>
__device__ __forceinline__ void coverage_row(const float* s, int row, const RowSpec& p,
                                             const float* total_in, const float* selected_in,
                                             uint32_t* skey, float* cval, uint8_t* out,
                                             int32_t* flag, int lane) {
  constexpr int E = NPAD / 32;  // sorted positions per lane (contiguous chunk)
  const int nk = p.nk;
  const int T = p.T;
  const bool video = p.mode == SA_COVERAGE_VIDEO_RESIDUAL;

  // Rows fully required by the text rule: all ones.
  if (T > 0 && row < T) {
    for (int j = lane; j < nk; j += 32) out[j] = 1;
    if (flag != nullptr && lane == 0) *flag = 0;
    return;
  }
  const int c_lo = video ? T : 0;  // first column taking part in the coverage step

  // ---- load, required set, row sums ---------------------------------------
  // Participating columns (j >= c_lo) get a sort key ~ordered(candidate);
  // required columns enter as -inf (joint mode). Others get key 0xFFFFFFFF
  // (sorted last) and candidate value NaN.
  double tot = 0.0, sel = 0.0;
  int n_cand_local = 0;  // non-required participating columns (candidate_counts, line 348)
  // The row's values are loaded eight at a time, each eight before the first
  // shared-memory store of their batch: loads and stores in one loop made
  // each load wait for the previous iteration's stores (the compiler cannot
  // tell the row from the scratch).
  constexpr int kBatch = NPAD / 32 < 8 ? NPAD / 32 : 8;
  static_assert((NPAD / 32) % kBatch == 0, "row batches");
#pragma unroll
  for (int q0 = 0; q0 < NPAD / 32; q0 += kBatch) {
  float vin[kBatch];
#pragma unroll
  for (int u = 0; u < kBatch; ++u) {
    const int j = lane + 32 * (q0 + u);
    vin[u] = (j < nk && j >= c_lo) ? s[j] : 0.f;
  }
#pragma unroll
  for (int u = 0; u < kBatch; ++u) {
    const int j = lane + 32 * (q0 + u);
    uint32_t key = 0xFFFFFFFFu;
    float cv = __int_as_float(0x7fc00000);
    if (j < nk && j >= c_lo) {
      const float v = vin[u];
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
  }
  tot = warp_sum_f64(tot);
  sel = warp_sum_f64(sel);
  float total = total_in != nullptr ? *total_in : (float)tot;
  const float selected = video ? 0.f : (selected_in != nullptr ? *selected_in : (float)sel);
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

  if (flag != nullptr && lane == 0) {
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
    if (total_in == nullptr && target > 1e-6f && first != INT_MAX) {
      const float u = 2.f * ulp_of(target);
      if (cum_at_first - target <= u || (first > 0 && target - cum_before_first <= u))
        flags |= SA_ROW_NEAR_TARGET;
    }
    *flag = (int32_t)flags;
  }
}


}  // namespace cov
}  // namespace sa
