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
// The pooling reads the layer's Q and K once and is HBM-bound; the rest is
// small but latency-bound, so it runs on other SMs and warps while the
// pooling streams, head by head. CTAs (one per SM) take a role by the order
// in which they start:
//   * pooling CTAs (the first to start). Warps 0-2 each own a fixed share of
//     the (head, batch, q|k, block) items, in head-major order, stream each
//     item's 128 x 128 bf16 tile through two 32 KB TMA stages, write its fp32
//     block mean (Q row-major [B,H,nb,128], K transposed [B,H,128,nb]) and
//     count it in shared memory (a CTA-scope release only). Warp 3 publishes
//     those counts per head to global memory about every half microsecond
//     behind one GPU-scope fence: the fence sits in a warp with no TMA load
//     in flight, so the streaming warps never wait on it. Warps 4-10 take
//     coverage rows whose batch mean is already published. When the CTA's
//     items are done, warps 3-10 join the score work below.
//   * score CTAs (the rest, about a fifth). Warps 3-10 take (head, 16 query
//     rows) items once every item of the head is counted, bulk-copy the
//     head's pooled K (four 32 KB channel chunks) and the rows' pooled Q into
//     shared memory, and compute the logits (each thread 4 rows x 4 keys),
//     the softmax per batch element (warp = row), the batch mean and the
//     optional running sums, then publish the 16 rows' batch mean. When no
//     item is left they take coverage rows (warp = row, coverage_row.cuh).
// So only the last head's score items and coverage rows run after the HBM
// read ends, spread over every SM. Roles go by start order, so a score CTA
// never holds an SM that a pooling CTA still has to start on; pooling warps
// never wait on other CTAs, and coverage rows taken while pooling are only
// rows that are already published, so every wait ends.
//
// Counters live in the caller's workspace, each on its own 128-byte line.
// The work counters are 64-bit words whose high half is the launch's epoch
// (drawn by the host per launch) and whose low half is the count: a counter
// left at another epoch (a fresh workspace, an earlier launch) counts as zero,
// and the first taker moves it into this launch's epoch with one
// compare-and-swap. The first CTA to start clears the per-head counts and
// then publishes the epoch in a `ready` word; the per-group "batch mean
// published" flags hold the epoch once set. The last CTA to finish returns
// everything to zero, so a launch replayed with the same epoch (a CUDA graph)
// starts clean too.
//
// The floating-point steps are those of the three-kernel chain in
// pool_scores.cu (per-lane column sums of the TMA tile, one fmaf per channel
// in channel order, the scale multiply after, the lane-strided softmax sum,
// the batch sum from 0); the two agree to within one ulp (measured: about a
// fifth of the entries differ, by one ulp).

#include <math.h>
#include <stdlib.h>
#include <unistd.h>

#include <atomic>
#include <chrono>

#include "calib_layer.cuh"
#include "coverage_row.cuh"

namespace sa {
namespace calib {

constexpr int kPoolWarps = 3;               // warps 0-2 of a pooling CTA
constexpr int kScoreWarp0 = 3;              // warps 3-10: signal / score / coverage
constexpr int kScoreWarps = 8;
constexpr int kScoreThreads = kScoreWarps * 32;
constexpr int kThreads = (kPoolWarps + kScoreWarps) * 32;
constexpr int kRows = 16;                   // query rows per score item
constexpr int kD = 128;
constexpr int kStageBytes = 128 * 128 * 2;  // one bf16 128 x 128 tile
constexpr int kMaxBlocks = 256;
constexpr int kMaxHeads = 128;
constexpr int kKChunks = 4;                 // pooled-K channel chunks of a score item
constexpr int kKChunkD = kD / kKChunks;     // 32 channels = 32 KB at 256 blocks

// counters, one per 128-byte line; [0..3] epoch-tagged, [4] holds the epoch
// once the head counts are cleared, [5 + h] pooling items finished of head h
constexpr int kCtrStride = 128 / 8;  // 64-bit words per line
constexpr int kRoleCtr = 0, kScoreCtr = 1, kCovCtr = 2, kDoneCtr = 3, kReady = 4, kHead0 = 5;
size_t counter_bytes(int H) { return (((size_t)(kHead0 + H) * 128) + 255) & ~size_t(255); }
// "batch mean published" flag of every (head, group of kRows rows)
size_t flag_bytes(int H, int nb) {
  return (((size_t)H * ((nb + kRows - 1) / kRows) * 8) + 255) & ~size_t(255);
}

// Shared memory. The pooling stages and the score items' pooled-K chunks and
// pooled-Q rows share the first 192 KB (a CTA pools first, then scores).
template <int NPAD>
struct Layout {
  static constexpr size_t stages = 0;                                   // pooling: 6 x 32 KB
  static constexpr size_t kslots = 0;                                   // scores: 4 x 32 KB
  static constexpr size_t qs = kslots + (size_t)kKChunks * kKChunkD * kMaxBlocks * 4;  // [2][16][128]
  static constexpr size_t bars = stages + (size_t)kPoolWarps * 2 * kStageBytes;
  static constexpr size_t ebuf = bars + 128;                            // [16][NPAD] fp32
  static constexpr size_t cov = ebuf + (size_t)kRows * NPAD * 4;        // [8][2*NPAD] u32
  static constexpr size_t hcnt = cov + (size_t)kScoreWarps * 2 * NPAD * 4;  // [kMaxHeads] int
  static constexpr size_t hpub = hcnt + (size_t)kMaxHeads * 4;          // [kMaxHeads] int
  static constexpr size_t ctl = hpub + (size_t)kMaxHeads * 4;           // 16 ints
  static constexpr size_t total = ctl + 64 + 1024;                      // + base alignment
};
static_assert(Layout<256>::total <= 232448, "shared memory layout exceeds 227 KB");
static_assert(Layout<256>::qs + (size_t)2 * kRows * kD * 4 <= Layout<256>::bars,
              "pooled-Q buffers overlap the barriers");
// barriers: [2w, 2w+1] pooling warp w's stages, [6 + c] pooled-K chunk slot
// c, [10 + q] pooled-Q buffer q
// ctl: [0] score item, [1] its head is complete, [2] role (1 = pool),
//      [3] pooling warps done, [4] ticket, [5] pooling published

struct Params {
  int B, H, S, nb, G;   // G = score items (groups of kRows rows) per head
  int pool_ctas;        // CTAs that pool first (the first to start)
  float scale;
  float* qp;            // [B,H,nb,128]
  float* kpt;           // [B,H,128,nb]
  float* bm_scratch;    // [H,nb,nb] batch mean when the caller wants a mask only
  unsigned long long* ctr;
  unsigned long long* gflag;  // [H*G]
  uint32_t epoch;
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

__device__ __forceinline__ unsigned long long ld_acquire(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Count of an epoch-tagged counter in this launch (another epoch reads 0).
__device__ __forceinline__ uint32_t epoch_count(unsigned long long v, uint32_t epoch) {
  return (uint32_t)(v >> 32) == epoch ? (uint32_t)v : 0u;
}

// Adds 1 to an epoch-tagged counter and returns this launch's count before
// the add. A counter left at another epoch is claimed for this one; only the
// claimer sees 0.
__device__ __forceinline__ uint32_t epoch_add(unsigned long long* c, uint32_t epoch) {
  unsigned long long cur = atomicAdd(c, 1ull);
  while ((uint32_t)(cur >> 32) != epoch) {
    // another epoch: this add went to the stale value cur + 1
    const unsigned long long stale = cur + 1ull;
    const unsigned long long prev =
        atomicCAS(c, stale, ((unsigned long long)epoch << 32) | 1ull);
    if (prev == stale) return 0u;
    cur = (uint32_t)(prev >> 32) == epoch ? atomicAdd(c, 1ull) : prev - 1ull;
  }
  return (uint32_t)cur;
}

__device__ __forceinline__ void score_bar() {
  asm volatile("bar.sync 1, %0;" ::"r"(kScoreThreads) : "memory");
}

// Bounded spin until pred() holds; gives up (false) on timeout, recording
// SA_DEV_WAIT_TIMEOUT, or as soon as another wait of the launch gave up.
template <class Pred>
__device__ bool spin_until(Pred pred, int32_t* status, uint32_t sleep_ns) {
  if (pred()) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    __nanosleep(sleep_ns);
    if (pred()) return true;
    if ((it & 63u) == 0u) {
      if (status_set(status)) return false;
      if (global_timer_ns() - t0 > kWaitNs) {
        report_timeout(status);
        return false;
      }
    }
  }
}

// One coverage row, run by a whole warp (coverage_row is warp-collective):
// the row's batch mean is copied into this warp's shared buffer first.
template <int NPAD>
__device__ __forceinline__ void coverage_of_row(const Params& p, int r, float* rowbuf,
                                                uint32_t* skey, int lane, bool ok) {
  const int nb = p.nb;
  const int h = r / nb, i = r - (r / nb) * nb;
  uint8_t* mrow = p.mask + (int64_t)r * nb;
  if (!ok) {  // a wait gave up (status set): the row keeps every block
    for (int c = lane; c < nb; c += 32) mrow[c] = 1;
    return;
  }
  const float* bm = (p.bmean != nullptr ? p.bmean : p.bm_scratch) + (int64_t)r * nb;
  for (int c = lane; c < nb; c += 32) rowbuf[c] = __ldcg(bm + c);
  __syncwarp();
  cov::coverage_row<NPAD>(rowbuf, i, p.spec, nullptr, nullptr, skey,
                          reinterpret_cast<float*>(skey + NPAD), mrow,
                          p.flags != nullptr ? p.flags + (int64_t)h * nb + i : nullptr, lane);
  __syncwarp();
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
  int* hcnt = reinterpret_cast<int*>(smem + L::hcnt);
  int* hpub = reinterpret_cast<int*>(smem + L::hpub);
  volatile int* ctl = reinterpret_cast<volatile int*>(smem + L::ctl);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.nb;
  const int per_head = 2 * p.B * nb;  // pooling items of one head
  const int n_pool = p.H * per_head;
  const int n_score = p.H * p.G;
  const int n_rows = p.H * nb;        // coverage rows

  for (int i = threadIdx.x; i < p.H; i += kThreads) {
    hcnt[i] = 0;
    hpub[i] = 0;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 12; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
    const uint32_t ticket = epoch_add(&p.ctr[kRoleCtr * kCtrStride], p.epoch);
    if (ticket == 0u) {
      // the first CTA clears the head counts, then publishes the epoch
      volatile unsigned long long* c = p.ctr;
      for (int h = 0; h < p.H; ++h) c[(kHead0 + h) * kCtrStride] = 0ull;
      __threadfence();
      c[kReady * kCtrStride] = (unsigned long long)p.epoch;
    }
    ctl[2] = ticket < (uint32_t)p.pool_ctas ? 1 : 0;
    ctl[3] = 0;
    ctl[4] = (int)ticket;
    ctl[5] = 0;
  }
  __syncthreads();
  const bool pool_role = ctl[2] != 0;

  if (warp < kPoolWarps) {
    if (pool_role) {
      // ------------------------------------------------------------- pooling
      uint8_t* stage0 = smem + L::stages + (size_t)warp * 2 * kStageBytes;
      uint64_t* full = &bars[2 * warp];
      if (lane == 0) {
        prefetch_tensormap(&tm_q);
        prefetch_tensormap(&tm_k);
      }
      // this warp's share: items first, first + stride, ... (head-major order)
      const int stride = p.pool_ctas * kPoolWarps;
      auto issue = [&](int it, int st) {
        const int h = it / per_head;
        const int r = it - h * per_head;
        const int b = r / (2 * nb);
        const int r2 = r - b * 2 * nb;
        const int t = r2 / nb;
        const int j = r2 - t * nb;
        mbar_arrive_expect_tx(&full[st], kStageBytes);
        tma_load_4d(t ? &tm_k : &tm_q, &full[st], stage0 + (size_t)st * kStageBytes, 0, j * 128,
                    h, b);
      };
      int item = ctl[4] * kPoolWarps + warp;
      int next = item + stride;
      if (lane == 0 && item < n_pool) issue(item, 0);
      for (int k = 0; item < n_pool; ++k) {
        const int st = k & 1;
        __syncwarp();  // every lane is done reading stage st ^ 1 (item k - 1)
        if (lane == 0 && next < n_pool) {
          fence_proxy_async_smem();
          issue(next, st ^ 1);
        }
        if (!mbar_wait_drain(&full[st], (uint32_t)(k >> 1) & 1u)) {
          if (lane == 0) report_timeout(p.status);
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
        // count the item in shared memory (CTA-scope release); warp 3
        // publishes the counts with the GPU-scope fence
        __syncwarp();
        if (lane == 0) {
          __threadfence_block();
          atomicAdd(&hcnt[h], 1);
        }
        item = next;
        next += stride;
      }
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        atomicAdd(const_cast<int*>(&ctl[3]), 1);
      }
    }
  } else {
    const int sw = warp - kScoreWarp0;  // 0..7
    const int tid = threadIdx.x - kScoreWarp0 * 32;
    float* rowbuf = ebuf + (size_t)sw * NPAD;
    uint32_t* skey = covs + (size_t)sw * 2 * NPAD;
    if (pool_role) {
      if (warp == kScoreWarp0) {
        // ----------------------------------------------- publish head counts
        if (lane == 0) {
          spin_until([&] { return ld_acquire(&p.ctr[kReady * kCtrStride]) ==
                                  (unsigned long long)p.epoch; },
                     p.status, 64);
          for (;;) {
            const int done = ctl[3];
            __threadfence();  // acquire the counts (and the pooled values behind them)
            bool any = false;
            for (int h = 0; h < p.H; ++h)
              any |= *reinterpret_cast<volatile int*>(&hcnt[h]) != hpub[h];
            if (any) {
              __threadfence();
              for (int h = 0; h < p.H; ++h) {
                const int c = *reinterpret_cast<volatile int*>(&hcnt[h]);
                if (c != hpub[h]) {
                  atomicAdd(&p.ctr[(kHead0 + h) * kCtrStride], (unsigned long long)(c - hpub[h]));
                  hpub[h] = c;
                }
              }
            }
            if (done == kPoolWarps) break;
            __nanosleep(400);
          }
          ctl[5] = 1;
        }
        __syncwarp();
      } else if (p.mask != nullptr) {
        // ------------------------------ coverage rows that are published already
        for (;;) {
          int r = -1;
          int ok = 0;
          if (lane == 0) {
            unsigned long long* c = &p.ctr[kCovCtr * kCtrStride];
            unsigned long long cur = ld_acquire(c);
            for (int tries = 0; tries < 8 && ctl[5] == 0; ++tries) {
              const uint32_t row = epoch_count(cur, p.epoch);
              if (row >= (uint32_t)n_rows) break;
              const int g = (int)(row / nb) * p.G + (int)(row % nb) / kRows;
              if (ld_acquire(&p.gflag[g]) != (unsigned long long)p.epoch) break;
              const unsigned long long want = ((unsigned long long)p.epoch << 32) | (row + 1u);
              const unsigned long long prev = atomicCAS(c, cur, want);
              if (prev == cur) {
                r = (int)row;
                ok = 1;
                break;
              }
              cur = prev;
            }
          }
          // the row and its verdict go to the whole warp: coverage_row is
          // warp-collective
          r = __shfl_sync(0xffffffffu, r, 0);
          ok = __shfl_sync(0xffffffffu, ok, 0);
          if (r < 0) {
            // nothing published yet: look again later, or stop once pooling is done
            if (__shfl_sync(0xffffffffu, (int)ctl[5], 0) != 0) break;
            __nanosleep(1000);
            continue;
          }
          coverage_of_row<NPAD>(p, r, rowbuf, skey, lane, ok != 0);
        }
      }
      // warps 3-10 turn to score items once this CTA's pooling is published
      asm volatile("bar.sync 2, %0;" ::"r"(kScoreThreads) : "memory");
    }

    // ------------------------------------------------------------ score items
    uint64_t* kbar = &bars[6];
    uint64_t* qbar = &bars[10];
    uint32_t kpar = 0u, qpar = 0u;  // parity of the next completion of each slot / buffer
    const uint32_t kbytes = (uint32_t)(kKChunkD * nb * 4);
    const float invb = 1.0f / (float)p.B;
    // thread tile: rows r0 .. r0 + 3 and keys kb .. kb + 3
    const int r0 = 4 * (sw >> 1);
    const int kb = 4 * (32 * (sw & 1) + lane);
    const bool vec4 = (nb & 3) == 0;
    auto kslot = [&](int c) -> float* {
      return reinterpret_cast<float*>(smem + L::kslots + (size_t)c * kKChunkD * kMaxBlocks * 4);
    };
    auto wait_copy = [&](uint64_t* bar, uint32_t parity) {
      if (!mbar_wait_drain(bar, parity) && tid == 0) report_timeout(p.status);
    };
    // the stage region was last written by TMA and read by generic loads
    if (tid == 0) fence_proxy_async_all();
    for (;;) {
      if (tid == 0) {
        const int s = (int)epoch_add(&p.ctr[kScoreCtr * kCtrStride], p.epoch);
        int ok = 0;
        if (s < n_score) {
          const unsigned long long* cnt = &p.ctr[(kHead0 + s / p.G) * kCtrStride];
          ok = spin_until([&] {
                 return ld_acquire(&p.ctr[kReady * kCtrStride]) == (unsigned long long)p.epoch &&
                        ld_acquire(cnt) >= (unsigned long long)per_head;
               }, p.status, 256) ? 1 : 0;
        }
        ctl[0] = s;
        ctl[1] = ok;
      }
      score_bar();
      const int s = ctl[0];
      const int ok = ctl[1];
      score_bar();
      if (s >= n_score) break;
      const int h = s / p.G;
      const int g = s - h * p.G;
      const int i0 = g * kRows;
      const int nrows = min(kRows, nb - i0);
      if (!ok) {
        // a wait gave up (status set): the item's outputs are marked invalid
        for (int e = tid; e < nrows * nb; e += kScoreThreads) {
          const int64_t hi = ((int64_t)h * nb + i0 + e / nb) * nb + e % nb;
          if (p.bmean != nullptr) p.bmean[hi] = __int_as_float(0x7fc00000);
          for (int b = 0; b < p.B && p.scores != nullptr; ++b)
            p.scores[hi + (int64_t)b * p.H * nb * nb] = __int_as_float(0x7fc00000);
        }
        score_bar();
        if (tid == 0) {
          __threadfence();
          *reinterpret_cast<volatile unsigned long long*>(&p.gflag[s]) = p.epoch;
        }
        continue;
      }
      const uint32_t qbytes = (uint32_t)nrows * kD * 4;
      auto issue_q = [&](int b) {
        const int64_t bh = (int64_t)b * p.H + h;
        mbar_arrive_expect_tx(&qbar[b & 1], qbytes);
        bulk_load(qs + (b & 1) * kRows * kD, p.qp + (bh * nb + i0) * kD, qbytes, &qbar[b & 1]);
      };
      auto issue_k = [&](int b, int c) {
        const int64_t bh = (int64_t)b * p.H + h;
        mbar_arrive_expect_tx(&kbar[c], kbytes);
        bulk_load(kslot(c), p.kpt + (bh * kD + c * kKChunkD) * nb, kbytes, &kbar[c]);
      };
      if (tid == 0) {
        // the head's data was written by other CTAs (generic stores, seen
        // through the acquire above); the slots were last read by this CTA's
        // generic loads
        fence_proxy_async_all();
        issue_q(0);
        for (int c = 0; c < kKChunks; ++c) issue_k(0, c);
      }
      float bacc[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int e = 0; e < 4; ++e) bacc[a][e] = 0.f;
      for (int b = 0; b < p.B; ++b) {
        const int64_t bh = (int64_t)b * p.H + h;
        if (tid == 0 && b + 1 < p.B) {
          fence_proxy_async_all();
          issue_q(b + 1);  // its buffer was last read by batch element b - 1
        }
        wait_copy(&qbar[b & 1], (qpar >> (b & 1)) & 1u);
        qpar ^= 1u << (b & 1);
        const float* q0 = qs + (b & 1) * kRows * kD + r0 * kD;
        float acc[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[a][e] = 0.f;
        for (int c = 0; c < kKChunks; ++c) {
          wait_copy(&kbar[c], (kpar >> c) & 1u);
          kpar ^= 1u << c;
          if (kb < nb) {
            const float* ks = kslot(c) + kb;
#pragma unroll 2
            for (int dd = 0; dd < kKChunkD; dd += 4) {
              const int d = c * kKChunkD + dd;
              float qv[4][4];
#pragma unroll
              for (int a = 0; a < 4; ++a) {
                const float4 q4 = *reinterpret_cast<const float4*>(q0 + a * kD + d);
                qv[a][0] = q4.x; qv[a][1] = q4.y; qv[a][2] = q4.z; qv[a][3] = q4.w;
              }
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                float kv[4];
                if (vec4) {
                  const float4 k4 = *reinterpret_cast<const float4*>(ks + (dd + i) * nb);
                  kv[0] = k4.x; kv[1] = k4.y; kv[2] = k4.z; kv[3] = k4.w;
                } else {
#pragma unroll
                  for (int e = 0; e < 4; ++e) kv[e] = ks[(dd + i) * nb + e];
                }
#pragma unroll
                for (int a = 0; a < 4; ++a)
#pragma unroll
                  for (int e = 0; e < 4; ++e) acc[a][e] = fmaf(qv[a][i], kv[e], acc[a][e]);
              }
            }
          }
          score_bar();  // every thread is done with slot c
          if (tid == 0 && b + 1 < p.B) {
            fence_proxy_async_all();
            issue_k(b + 1, c);
          }
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (kb + e < nb) ebuf[(r0 + a) * NPAD + kb + e] = acc[a][e] * p.scale;
        score_bar();
        for (int rr = sw; rr < nrows; rr += kScoreWarps) {  // softmax of row rr
          float* x = ebuf + rr * NPAD;
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
#pragma unroll
        for (int a = 0; a < 4; ++a) {
          if (r0 + a >= nrows) continue;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            if (kb + e >= nb) continue;
            const float pv = ebuf[(r0 + a) * NPAD + kb + e];
            if (p.scores != nullptr) p.scores[(bh * nb + i0 + r0 + a) * nb + kb + e] = pv;
            bacc[a][e] += pv;
          }
        }
        score_bar();
      }
      float* bmo = p.bmean != nullptr ? p.bmean : (p.mask != nullptr ? p.bm_scratch : nullptr);
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        if (r0 + a >= nrows) continue;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (kb + e >= nb) continue;
          const float bm = p.B == 1 ? bacc[a][e] : bacc[a][e] * invb;
          const int64_t hi = ((int64_t)h * nb + i0 + r0 + a) * nb + kb + e;
          if (bmo != nullptr) bmo[hi] = bm;
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
        }
      }
      if (p.mask != nullptr) {
        // publish the group's batch mean for the coverage rows
        score_bar();
        if (tid == 0) {
          __threadfence();
          *reinterpret_cast<volatile unsigned long long*>(&p.gflag[s]) = p.epoch;
        }
      }
    }

    // ------------------------------------------------ coverage rows, any left
    if (p.mask != nullptr) {
      for (;;) {
        int r = 0, ok = 0;
        if (lane == 0) {
          r = (int)epoch_add(&p.ctr[kCovCtr * kCtrStride], p.epoch);
          if (r < n_rows) {
            const int g = (r / nb) * p.G + (r % nb) / kRows;
            ok = spin_until([&] { return ld_acquire(&p.gflag[g]) == (unsigned long long)p.epoch; },
                            p.status, 128) ? 1 : 0;
          }
        }
        r = __shfl_sync(0xffffffffu, r, 0);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (r >= n_rows) break;
        coverage_of_row<NPAD>(p, r, rowbuf, skey, lane, ok != 0);
      }
    }
  }

  // the last CTA to finish returns the counters and flags to zero
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (epoch_add(&p.ctr[kDoneCtr * kCtrStride], p.epoch) == gridDim.x - 1) {
      __threadfence();
      volatile unsigned long long* c = p.ctr;
      c[kRoleCtr * kCtrStride] = 0ull;
      c[kScoreCtr * kCtrStride] = 0ull;
      c[kCovCtr * kCtrStride] = 0ull;
      c[kReady * kCtrStride] = 0ull;
      for (int h = 0; h < p.H; ++h) c[(kHead0 + h) * kCtrStride] = 0ull;
      volatile unsigned long long* f = p.gflag;
      for (int i = 0; i < n_score; ++i) f[i] = 0ull;
      c[kDoneCtr * kCtrStride] = 0ull;
      __threadfence();
    }
  }
}

// Epochs of successive launches: a per-process sequence started from the
// clock and the process id, never 0 (the value of a cleared counter).
uint32_t next_epoch() {
  static std::atomic<uint32_t> seq{(uint32_t)std::chrono::steady_clock::now()
                                       .time_since_epoch()
                                       .count() ^
                                   ((uint32_t)getpid() << 16)};
  uint32_t e = seq.fetch_add(1, std::memory_order_relaxed);
  if (e == 0) e = seq.fetch_add(1, std::memory_order_relaxed);
  return e;
}

size_t workspace_bytes(int B, int H, int S) {
  const size_t nb = (size_t)((S + 127) / 128);
  return counter_bytes(H) + flag_bytes(H, (int)nb) + 2 * (size_t)B * H * nb * kD * sizeof(float) +
         (size_t)H * nb * nb * sizeof(float);
}

bool eligible(const void* q, const void* k, const int64_t* q_strides, const int64_t* k_strides,
              int B, int H, int S, int D, int block) {
  if (D != kD || block != 128 || B < 1 || H < 1 || S < 1 || H > kMaxHeads) return false;
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
  const size_t need = workspace_bytes(a.B, a.H, a.S);
  SA_CHECK_ARG(a.workspace != nullptr && a.ws_bytes >= need,
               "calibration layer: workspace of %zu bytes required, got %zu", need, a.ws_bytes);
  SA_CHECK_ARG(((uintptr_t)a.workspace) % 256 == 0,
               "calibration layer: workspace must be 256-byte aligned");
  SA_CHECK_ARG(a.H <= kMaxHeads, "calibration layer: at most %d heads, got %d", kMaxHeads, a.H);
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
  uint8_t* ws = reinterpret_cast<uint8_t*>(a.workspace);
  p.ctr = reinterpret_cast<unsigned long long*>(ws);
  ws += counter_bytes(a.H);
  p.gflag = reinterpret_cast<unsigned long long*>(ws);
  ws += flag_bytes(a.H, nb);
  p.qp = reinterpret_cast<float*>(ws);
  p.kpt = p.qp + (size_t)a.B * a.H * nb * kD;
  p.bm_scratch = p.kpt + (size_t)a.B * a.H * nb * kD;
  p.epoch = next_epoch();
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
  // score CTAs: about a fifth of the grid (SINKATTN_CALIB_SCORE_CTAS sets the
  // number, for tuning); at least one CTA pools
  int score_ctas = (grid * 22 + 50) / 100;
  if (const char* env = getenv("SINKATTN_CALIB_SCORE_CTAS")) score_ctas = atoi(env);
  if (score_ctas > grid - 1) score_ctas = grid - 1;
  if (score_ctas < 0) score_ctas = 0;
  p.pool_ctas = grid - score_ctas;
  if (nb <= 32) return launch_t<32>(maps[0], maps[1], p, grid, stream);
  if (nb <= 64) return launch_t<64>(maps[0], maps[1], p, grid, stream);
  if (nb <= 128) return launch_t<128>(maps[0], maps[1], p, grid, stream);
  return launch_t<256>(maps[0], maps[1], p, grid, stream);
}

}  // namespace calib
}  // namespace sa

extern "C" size_t sa_calibration_layer_workspace_size(int B, int H, int S) {
  if (B < 1 || H < 1 || S < 1) return 0;
  return sa::calib::workspace_bytes(B, H, S);
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
