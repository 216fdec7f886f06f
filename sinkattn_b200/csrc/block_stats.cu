// block_stats.cu — dense per-(query row, key block) statistics of Q K^T on
// tcgen05 tensor cores, for the two other calibration score modes:
//
//   EXACT  _compute_exact_block_mass_scores (sinkattention/sparse_attention.py:145-227)
//          score[qb, kb] = mean over the query rows r of block qb of
//            sum_{n in kb} exp(s_rn - m_r) / max(sum_n exp(s_rn - m_r), 1e-6),
//          s = q k^T / sqrt(D), m_r the row maximum over all keys.
//          One sweep over the keys: every block's mass is taken under the
//          block's own row maximum R_j (c_j = sum_{n in j} exp2(s_rn - R_j),
//          each term at most 1), and the scratch slot keeps c_j and R_j. The
//          epilogue rescales by exp2(R_j - m_r) once the row maximum m_r is
//          known, sums the row total from the same products in block order,
//          and normalises and averages: one exponential per (row, key) and one
//          per (row, block), where two sweeps needed the keys' QK twice.
//   MAX    the Triton pooling kernel attn_with_pooling (sinkattention/pooling_kernel.py:
//          11-248), whose statistics are maxima (the "pooled" name notwithstanding):
//            R[r, kb] = bf16( max_{n in kb} s_rn * log2(e) )         (line 45-48)
//            m_r      = max_kb of the unrounded values                  (line 46)
//            Po[qb,kb]= bf16( max_{r in qb} exp2(R[r,kb] - m_r) )      (lines 65-75)
//          and the row normalisation Po / sum(Po) in bf16 (lines 243-244).
//          For S not a multiple of 128 the Triton kernel reads query rows past
//          the end of the head (its block pointers carry no boundary check);
//          here rows past S take no part in the column maxima and keys past S
//          are masked, as the Triton kernel masks its last key block.
//
// Persistent grid (one CTA per SM) looping over pairs of 128-row query tiles
// of one head: every K tile brought into shared memory serves both query
// tiles, which halves the L2 -> shared-memory traffic per MMA. Max mode runs
// 384 threads (below); exact mode 640, its statistics warps 4-19 each owning
// 64 columns of a row (warps 4-7 and 8-11 the two halves of tile 0, 12-15 and
// 16-19 of tile 1), so that four warps per SMSP feed MUFU and each loads and
// reduces half as much per block before its exponentials (two whole-row warps
// per SMSP loaded and reduced in step while MUFU idled); each half keeps its
// own (mass, maximum) per block and the epilogue combines them.
//   warp 0      TMA producer: K tiles into a 5-slot ring
//   warp 1      MMA issuer of query tile 0: S = Q_0 K^T (Q_0 from TMEM, K
//               from shared memory) into its two TMEM buffers in turn
//   warp 3      MMA issuer of query tile 1, into its one TMEM buffer
//               (two issuing threads halve the per-MMA-group waits and
//               commits that a single thread serialises)
//   warp 2      TMEM allocator
//   warps 4-7   statistics of query tile 0 (thread t owns query row t);
//               exact mode: columns 0-63 of tile 0, warps 8-11 its columns
//               64-127
//   warps 8-11  statistics of query tile 1 (exact mode: warps 12-19, the
//               two halves as for tile 0)
//   Each statistics group writes its tile's Q into TMEM. Every K tile is
//   released by both issuers (by a commit after its MMAs, or an arrival when
//   the work item has no second tile).
// TMEM: S buffers [0,128) and [256,384) of tile 0, [128,256) of tile 1;
// Q_0 [384,448), Q_1 [448,512) (bf16 pairs, the A-operand layout). Each CTA
// owns one scratch slot per query tile: nk x 128 fp32 values (the bf16-rounded
// block maxima) in max mode, 2 x nk x 2 x 128 (block masses of both halves,
// then their maxima) in exact mode, written with one coalesced store per
// block and warp.

#include <math.h>

#include "sa_common.cuh"

namespace sa {
namespace stats {

constexpr int kBM = 128, kBN = 128, kHD = 128;
constexpr int kStages = 5;
constexpr int kSBuf = 3;  // TMEM S buffers of 128 columns
constexpr int kGroups = 2;  // query tiles per work item
// threads of a launch whose statistics warps each own 128 / kHalves columns
// of a row (kHalves = 2: four statistics warps per SMSP)
template <int kHalves>
constexpr int threads_of() { return 128 + kGroups * 128 * kHalves; }
constexpr int kTileBytes = kBN * kHD * 2;
constexpr int kBoxBytes = kTileBytes / 2;
constexpr int kMaxNB = 1024;
constexpr uint32_t kColQ = 384;  // Q of tile a at kColQ + 64 a

enum Mode { kExact = 0, kMax = 1 };

struct Params {
  int B, H, S, nq, nk, mode, pairs;
  float scale_log2;
  const __nv_bfloat16* q;
  int64_t qs0, qs1, qs2;
  float* scores;          // [B,H,nq,nk] fp32
  float* scratch;         // [gridDim.x][kGroups][slot] fp32 (slot layout above)
  int32_t* status;
};

struct __align__(8) SmemCtl {
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t s_full[kSBuf];   // per TMEM buffer; each buffer belongs to one query tile
  uint64_t s_empty[kSBuf];  // 128 arrivals: the statistics group that owns the buffer
  uint64_t q_ready[kGroups]; // one phase per work item of the group, 128 arrivals
  uint64_t mma_drain;
  uint32_t tmem_base;
  int abort_flag;
  float red[kGroups][4][kMaxNB];  // per-warp column partials
  float po[kGroups][kMaxNB];      // MAX: bf16 column maxima before normalisation
  float psum[kGroups][4];
  float mxh[kGroups][2][kBM];  // exact mode, two halves: each half's row maximum
  float lxh[kGroups][2][kBM];  // ... and its part of the row total
};

constexpr size_t kSmemBytes = 1024 + kStages * kTileBytes + sizeof(SmemCtl);

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Named barrier of one statistics group (ids 1 and 2, 128 threads each).
__device__ __forceinline__ void stats_bar_sync(int group, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(group + 1), "r"(threads) : "memory");
}

// Epilogue: the scratch values of kEpi consecutive blocks of one row, loaded
// before any of them is used (blocks past nk repeat the last one).
constexpr int kEpi = 8;
__device__ __forceinline__ void epi_load(const float* c, const float* r, int nk, int j0, int row,
                                         float (&cv)[kEpi], float (&rv)[kEpi]) {
#pragma unroll
  for (int u = 0; u < kEpi; ++u) {
    const int64_t e = (int64_t)min(j0 + u, nk - 1) * kBM + row;
    cv[u] = c[e];
    rv[u] = r != nullptr ? r[e] : 0.f;
  }
}

// Work item t: query tiles 2 qp and 2 qp + 1 (if it exists) of head (b, h).
__device__ __forceinline__ void pair_coords(const Params& p, int t, int& qp, int& h, int& b,
                                            int& ntp) {
  const int nqp = (p.nq + 1) >> 1;
  qp = t % nqp;
  const int bh = t / nqp;
  h = bh % p.H;
  b = bh / p.H;
  ntp = min(kGroups, p.nq - 2 * qp);
}


// TMEM S buffers of query tile a: tile 0 owns two of them, tile 1 one.
constexpr int kNB0 = 2;
__device__ __forceinline__ int nbuf_of(int a) { return a == 0 ? kNB0 : 1; }
// physical buffer (columns [128 id, 128 id + 128)) of tile a's i-th buffer
__device__ __forceinline__ int buf_id(int a, int i) { return a == 0 ? (i == 0 ? 0 : 2) : 1; }
template <int kHalves>
__global__ void __launch_bounds__(threads_of<kHalves>(), 1)
    block_stats_kernel(const __grid_constant__ CUtensorMap tm_k, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ring = smem;
  SmemCtl* ctl = reinterpret_cast<SmemCtl*>(ring + kStages * kTileBytes);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int items = p.nk;  // K tiles per work item

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&ctl->kv_full[i], 1);
      mbar_init(&ctl->kv_empty[i], kGroups);  // one release per issuer
    }
    for (int i = 0; i < kSBuf; ++i) {
      mbar_init(&ctl->s_full[i], 1);
      mbar_init(&ctl->s_empty[i], kBM * kHalves);
    }
    for (int a = 0; a < kGroups; ++a) mbar_init(&ctl->q_ready[a], kBM * kHalves);
    mbar_init(&ctl->mma_drain, kGroups);  // both issuers' MMAs
    ctl->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) prefetch_tensormap(&tm_k);
  if (warp == 2) {
    tmem_alloc(&ctl->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  volatile int* abort_flag = &ctl->abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;  // K tiles produced by this CTA
      bool ok = true;
      for (int t = blockIdx.x; t < p.pairs && ok; t += gridDim.x) {
        int qp, h, b, ntp;
        pair_coords(p, t, qp, h, b, ntp);
        for (int it = 0; it < items; ++it, ++g) {
          const int stage = g % kStages;
          if (!mbar_wait(&ctl->kv_empty[stage], ((uint32_t)(g / kStages) & 1u) ^ 1u, p.status,
                         abort_flag)) {
            ok = false;
            break;
          }
          const int j = it % p.nk;
          uint8_t* dst = ring + stage * kTileBytes;
          mbar_arrive_expect_tx(&ctl->kv_full[stage], kTileBytes);
          tma_load_4d(&tm_k, &ctl->kv_full[stage], dst, 0, j * kBN, h, b);
          tma_load_4d(&tm_k, &ctl->kv_full[stage], dst + kBoxBytes, 64, j * kBN, h, b);
        }
      }
      for (int k = (g > kStages ? g - kStages : 0); k < g; ++k)
        mbar_wait_drain(&ctl->kv_full[k % kStages], (uint32_t)(k / kStages) & 1u);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 3) {
    // one MMA issuer per query tile: warp 1 tile 0, warp 3 tile 1
    const int ta = warp == 3 ? 1 : 0;
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(kBM, kBN, 0, 0);
      const uint32_t ring_base = smem_u32(ring);
      const int nb = nbuf_of(ta);
      int stage = 0, bi = 0;
      uint32_t kv_ph = 0, se_ph = 0;
      int qc = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.pairs && ok; t += gridDim.x) {
        int qp, h, b, ntp;
        pair_coords(p, t, qp, h, b, ntp);
        const bool mine = ta < ntp;
        if (mine) {
          ok = mbar_wait(&ctl->q_ready[ta], (uint32_t)qc & 1u, p.status, abort_flag);
          ++qc;
          if (!ok) break;
          tc_fence_after();
        }
        for (int it = 0; it < items && ok; ++it) {
          if (!mbar_wait(&ctl->kv_full[stage], kv_ph, p.status, abort_flag)) {
            ok = false;
            break;
          }
          if (mine) {
            const int buf = buf_id(ta, bi);
            if (!mbar_wait(&ctl->s_empty[buf], se_ph ^ 1u, p.status, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint64_t desc0 = make_sdesc_sw128(ring_base + stage * kTileBytes, 16, 1024);
#pragma unroll
            for (int kk = 0; kk < kHD / 16; ++kk)
              mma_ts(tmem + buf * 128, tmem + kColQ + ta * 64 + kk * 8,
                     desc0 + (uint64_t)((((kk >> 2) * kBoxBytes) + (kk & 3) * 32) >> 4), idesc,
                     kk > 0 ? 1u : 0u);
            mma_commit(&ctl->s_full[buf]);
            mma_commit(&ctl->kv_empty[stage]);
            if (++bi == nb) {
              bi = 0;
              se_ph ^= 1u;
            }
          } else {
            mbar_arrive(&ctl->kv_empty[stage]);  // this issuer does not read the tile
          }
          if (++stage == kStages) {
            stage = 0;
            kv_ph ^= 1u;
          }
        }
      }
      mma_commit(&ctl->mma_drain);
      mbar_wait_drain(&ctl->mma_drain, 0);
    }
    __syncwarp();
  } else if (warp >= 4) {
    constexpr int kCh = 4 / kHalves;     // 32-column chunks of S per warp
    constexpr int kCols = 32 * kCh;      // columns of S per warp
    constexpr int kGT = kBM * kHalves;   // threads of one statistics group
    const int sw = warp - 4;
    const int grp = sw / (4 * kHalves);                 // query tile of the work item
    const int hf = kHalves == 2 ? ((sw >> 2) & 1) : 0;  // this warp's half of the columns
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const int gt = hf * kBM + row;  // thread of the group
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    // scratch: [block][half][row] masses (exact) or bf16-rounded maxima (max),
    // then in exact mode [block][half][row] maxima
    const int slot_words = (p.mode == kExact ? 2 : 1) * kHalves * p.nk * kBM;
    float* slot = p.scratch + ((int64_t)blockIdx.x * kGroups + grp) * slot_words;
    float* slot_r = slot + (int64_t)kHalves * p.nk * kBM;
    float* red = ctl->red[grp][0];    // red[wq][j] at red[wq * kMaxNB + j]
    float* po_s = ctl->po[grp];
    float* psum = ctl->psum[grp];
    bool ok = true;
    // S items this group has consumed: its buffers are used round robin, and
    // a buffer is refilled only after this group has released it, so the
    // phase parity of s_full[buf] cannot alias.
    int cnt = 0;
    for (int t = blockIdx.x; t < p.pairs; t += gridDim.x) {
      int qp, h, b, ntp;
      pair_coords(p, t, qp, h, b, ntp);
      if (grp >= ntp) continue;
      const int qb = 2 * qp + grp;
      const int grow = qb * kBM + row;
      const bool row_valid = grow < p.S;
      const int rows_valid = min(kBM, p.S - qb * kBM);
      // Q row -> TMEM (all S of this group's previous work item has been read,
      // so the MMAs that read Q_grp are complete); with two halves each warp
      // writes its half of the row. Rows past S are zero.
      {
        const uint4* src = reinterpret_cast<const uint4*>(
            p.q + (int64_t)b * p.qs0 + (int64_t)h * p.qs1 + (int64_t)grow * p.qs2);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          if (kHalves == 2 && half != hf) continue;
          uint32_t qv[32];
#pragma unroll
          for (int v = 0; v < 8; ++v) {
            const uint4 w = row_valid ? src[half * 8 + v] : make_uint4(0, 0, 0, 0);
            qv[4 * v] = w.x; qv[4 * v + 1] = w.y; qv[4 * v + 2] = w.z; qv[4 * v + 3] = w.w;
          }
          tmem_st32(tmem + lane_off + kColQ + grp * 64 + half * 32, qv);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&ctl->q_ready[grp]);
      }
      float m = -INFINITY;
      for (int it = 0; it < items; ++it) {
        const int nbg = nbuf_of(grp);
        const int buf = buf_id(grp, cnt % nbg);
        const uint32_t sph = (uint32_t)(cnt / nbg) & 1u;
        ++cnt;
        const int j = it;
        if (ok)
          ok = __all_sync(0xffffffffu, mbar_wait(&ctl->s_full[buf], sph, p.status, abort_flag));
        if (!ok) continue;
        tc_fence_after();
        uint32_t r[kCh][32];
        const uint32_t s_addr = tmem + lane_off + buf * 128 + hf * kCols;
#pragma unroll
        for (int c = 0; c < kCh; ++c) tmem_ld32(s_addr + 32 * c, r[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < kCh; ++c) reg_fence32(r[c]);
        tc_fence_before();
        mbar_arrive(&ctl->s_empty[buf]);  // S copied out: the buffer may be refilled
        // valid keys among this warp's columns (none, in the second half of a
        // last block with at most 64 keys)
        const int valid = min(kBN, p.S - j * kBN) - hf * kCols;
        if (valid < kCols) {
#pragma unroll
          for (int c = 0; c < kCols; ++c)
            if (c >= valid) r[c >> 5][c & 31] = __float_as_uint(-INFINITY);
        }
        float mxp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mxp[u] = __uint_as_float(r[0][u]);
#pragma unroll
        for (int c = 8; c + 16 <= kCols; c += 16) {  // columns 8 .. kCols - 9
#pragma unroll
          for (int u = 0; u < 8; ++u)
            mxp[u] = fmax3(mxp[u], __uint_as_float(r[(c + u) >> 5][(c + u) & 31]),
                           __uint_as_float(r[(c + 8 + u) >> 5][(c + 8 + u) & 31]));
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) mxp[u] = fmaxf(mxp[u], __uint_as_float(r[kCh - 1][24 + u]));
        const float bmax = fmax3(fmax3(mxp[0], mxp[1], mxp[2]), fmax3(mxp[3], mxp[4], mxp[5]),
                                 fmaxf(mxp[6], mxp[7]));
        const float R = bmax * p.scale_log2;
        m = fmaxf(m, R);
        const int64_t e = ((int64_t)j * kHalves + hf) * kBM + row;
        // MAX: the block maximum rounded as the Triton kernel stores it
        // (pooling_kernel.py:45-48).
        if (p.mode == kMax) {
          slot[e] = bf16_round(R);
          continue;
        }
        // EXACT: this block's (half's) mass under its own maximum R, kept with
        // R; a half with no valid key has mass 0 and maximum -inf
        float cs = 0.f;
        if (R != -INFINITY) {
          const float negR = -R;
          float sp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int c = 0; c < kCols; ++c)
            sp[c & 3] += ex2_approx(fmaf(__uint_as_float(r[c >> 5][c & 31]), p.scale_log2, negR));
          cs = (sp[0] + sp[1]) + (sp[2] + sp[3]);
        }
        slot[e] = cs;
        slot_r[e] = R;
      }
      __syncwarp();
      float* out = p.scores + ((int64_t)(b * p.H + h) * p.nq + qb) * p.nk;
      if (p.mode == kExact) {
        // the row maximum m over both halves; then the masses under m and the
        // row total l from them (this warp's blocks j = hf, hf + kHalves, ...);
        // then the sum over the tile's rows of mass / max(l, 1e-6)
        // (sparse_attention.py:224), divided by the number of valid rows (the
        // mean of line 225). The masses are recomputed in the second pass
        // rather than stored back, and each pass loads kEpi blocks' values
        // before using any: a store into the scratch inside the loop kept every
        // iteration's loads from being issued before the previous store, and
        // the epilogue ran at one L2 round trip per block (~25% of the kernel).
        if (kHalves == 2) {
          ctl->mxh[grp][hf][row] = m;
          stats_bar_sync(grp, kGT);
          m = fmaxf(ctl->mxh[grp][0][row], ctl->mxh[grp][1][row]);
        }
        auto masses = [&](int j0, float (&w)[kEpi]) {
          float cv[kHalves][kEpi], rv[kHalves][kEpi];
#pragma unroll
          for (int u = 0; u < kEpi; ++u) {
            const int jj = min(j0 + u * kHalves, p.nk - 1);
#pragma unroll
            for (int hh = 0; hh < kHalves; ++hh) {
              const int64_t ee = ((int64_t)jj * kHalves + hh) * kBM + row;
              cv[hh][u] = slot[ee];
              rv[hh][u] = slot_r[ee];
            }
          }
#pragma unroll
          for (int u = 0; u < kEpi; ++u) {
            float x = 0.f;
#pragma unroll
            for (int hh = 0; hh < kHalves; ++hh) x += cv[hh][u] * ex2_approx(rv[hh][u] - m);
            w[u] = x;
          }
        };
        float l = 0.f;
        for (int j0 = hf; j0 < p.nk; j0 += kEpi * kHalves) {
          float w[kEpi];
          masses(j0, w);
#pragma unroll
          for (int u = 0; u < kEpi; ++u)
            if (j0 + u * kHalves < p.nk) l += row_valid ? w[u] : 0.f;
        }
        if (kHalves == 2) {
          ctl->lxh[grp][hf][row] = l;
          stats_bar_sync(grp, kGT);
          l = ctl->lxh[grp][0][row] + ctl->lxh[grp][1][row];
        }
        const float lc = fmaxf(l, 1e-6f);
        for (int j0 = hf; j0 < p.nk; j0 += kEpi * kHalves) {
          float w[kEpi];
          masses(j0, w);
#pragma unroll
          for (int u = 0; u < kEpi; ++u) {
            const int jj = j0 + u * kHalves;
            if (jj >= p.nk) break;
            float v = row_valid ? __fdiv_rn(w[u], lc) : 0.f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) red[wq * kMaxNB + jj] = v;
          }
        }
        stats_bar_sync(grp, kGT);
        const float inv_rows = 1.0f / (float)rows_valid;
        for (int jj = gt; jj < p.nk; jj += kGT)
          out[jj] = ((red[jj] + red[kMaxNB + jj]) + (red[2 * kMaxNB + jj] + red[3 * kMaxNB + jj])) *
                    inv_rows;
      } else if constexpr (kHalves == 1) {
        // Po[qb, kb] = bf16(max over the tile's rows of exp2(R - m_r)); l_i = 1
        // in the Triton kernel, so there is no division (pooling_kernel.py:65-75).
        for (int j0 = 0; j0 < p.nk; j0 += kEpi) {
          float cv[kEpi], rv[kEpi];
          epi_load(slot, nullptr, p.nk, j0, row, cv, rv);
#pragma unroll
          for (int u = 0; u < kEpi; ++u) {
            const int jj = j0 + u;
            if (jj >= p.nk) break;
            float x = row_valid ? ex2_approx(cv[u] - m) : 0.f;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, o));
            if (lane == 0) red[wq * kMaxNB + jj] = x;
          }
        }
        stats_bar_sync(grp, kGT);
        float part = 0.f;
        for (int jj = row; jj < p.nk; jj += kBM) {
          const float po = bf16_round(fmaxf(fmaxf(red[jj], red[kMaxNB + jj]),
                                            fmaxf(red[2 * kMaxNB + jj], red[3 * kMaxNB + jj])));
          po_s[jj] = po;
          part += po;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if (lane == 0) psum[wq] = part;
        stats_bar_sync(grp, kGT);
        // Po / sum(Po) with bf16 tensors (pooling_kernel.py:243-244): the sum is
        // accumulated in fp32 and rounded to bf16, the quotient rounded to bf16.
        const float sum = bf16_round((psum[0] + psum[1]) + (psum[2] + psum[3]));
        for (int jj = row; jj < p.nk; jj += kBM) out[jj] = bf16_round(__fdiv_rn(po_s[jj], sum));
      }
      stats_bar_sync(grp, kGT);  // red / po / mxh / lxh are rewritten by the next work item
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, 512);
}

}  // namespace stats
}  // namespace sa

namespace {

int make_map_bhsd(CUtensorMap* map, const void* base, const int64_t st[4], int B, int H, int S,
                  int D) {
  sa::EncodeTiledFn enc = sa::encode_tiled_fn();
  if (enc == nullptr) return SA_ECUDA;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)st[2] * 2, (cuuint64_t)st[1] * 2, (cuuint64_t)st[0] * 2};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    sa::set_error("cuTensorMapEncodeTiled (block stats) failed (CUresult %d)", (int)r);
    return SA_ECUDA;
  }
  return SA_OK;
}

bool stats_strides_ok(const int64_t st[4]) {
  if (st[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (st[i] < 0 || st[i] % 8 != 0) return false;
  return true;
}

// CTAs of the persistent grid: one per SM, at most one per work item (pair
// of query tiles of one head).
int stats_grid(int B, int H, int S) {
  const int64_t nq = (S + 127) / 128;
  const int64_t pairs = (int64_t)B * H * ((nq + 1) / 2);
  const int sms = sa::sm_count_current_device();
  return (int)(pairs < sms ? pairs : sms);
}

}  // namespace

extern "C" size_t sa_block_stats_workspace_size(int B, int H, int S, int mode) {
  if (B < 1 || H < 1 || S < 1) return 0;
  if (mode != sa::stats::kExact && mode != sa::stats::kMax) return 0;
  const size_t nk = (size_t)((S + 127) / 128);
  // per query tile: [block][half][row] values (two halves in exact mode),
  // and the same again for the maxima in exact mode
  const size_t words = (mode == sa::stats::kExact ? 2 * 2 : 1) * nk * 128;
  return (size_t)stats_grid(B, H, S) * sa::stats::kGroups * words * sizeof(float);
}

extern "C" int sa_block_stats(const void* q, const void* k, const int64_t q_strides[4],
                              const int64_t k_strides[4], int B, int H, int S, int D, int mode,
                              float softmax_scale, float* scores, void* workspace, size_t ws_bytes,
                              int32_t* status, cudaStream_t stream) {
  using namespace sa::stats;
  SA_CHECK_ARG(q && k && q_strides && k_strides && scores, "sa_block_stats: null pointer argument");
  SA_CHECK_ARG(mode == kExact || mode == kMax, "sa_block_stats: unknown mode %d", mode);
  SA_CHECK_ARG(D == kHD, "sa_block_stats: head dim must be 128, got %d", D);
  SA_CHECK_ARG(B >= 1 && H >= 1 && S >= 1, "sa_block_stats: B, H, S must be >= 1");
  const int nq = (S + kBM - 1) / kBM, nk = nq;
  SA_CHECK_ARG(nk <= kMaxNB, "sa_block_stats: S=%d exceeds %d blocks", S, kMaxNB);
  SA_CHECK_ARG((int64_t)B * H * nq <= 0x7fffffff, "sa_block_stats: too many query tiles");
  SA_CHECK_ARG(stats_strides_ok(q_strides) && stats_strides_ok(k_strides),
               "sa_block_stats: q/k need stride(dim)=1 and strides multiple of 8 elements");
  SA_CHECK_ARG(((uintptr_t)q | (uintptr_t)k) % 16 == 0, "sa_block_stats: q/k must be 16-byte aligned");
  const size_t need = sa_block_stats_workspace_size(B, H, S, mode);
  SA_CHECK_ARG(workspace != nullptr && ws_bytes >= need,
               "sa_block_stats: workspace of %zu bytes required, got %zu", need, ws_bytes);
  SA_CHECK_ARG((uintptr_t)workspace % 16 == 0, "sa_block_stats: workspace must be 16-byte aligned");

  CUtensorMap tk;
  int rc;
  if ((rc = make_map_bhsd(&tk, k, k_strides, B, H, S, D)) != SA_OK) return rc;
  Params p;
  p.B = B; p.H = H; p.S = S; p.nq = nq; p.nk = nk; p.mode = mode;
  p.pairs = B * H * ((nq + 1) / 2);
  // 1/sqrt(D) in double then fp32, as a Python float passed to fp32 math
  const float scale = softmax_scale > 0.f ? softmax_scale : (float)(1.0 / sqrt((double)D));
  p.scale_log2 = scale * 1.4426950408889634f;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.qs0 = q_strides[0]; p.qs1 = q_strides[1]; p.qs2 = q_strides[2];
  p.scores = scores;
  p.scratch = reinterpret_cast<float*>(workspace);
  p.status = status;
  // exact mode: four statistics warps per SMSP (each 64 columns of a row);
  // max mode: two (each a whole row)
  auto* kern = mode == kExact ? block_stats_kernel<2> : block_stats_kernel<1>;
  const int threads = mode == kExact ? threads_of<2>() : threads_of<1>();
  if (int rc = sa::func_attr_once((const void*)kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)kSmemBytes);
      rc != SA_OK)
    return rc;
  kern<<<stats_grid(B, H, S), threads, kSmemBytes, stream>>>(tk, p);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}
