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
// small but latency-bound, so it runs beside the pooling on every SM while
// the pooling streams, head by head. One CTA per SM, all alike:
//   * warps 0-2 pool. The (head, batch, q|k, block) items, in head-major
//     order, are dealt round robin to the pooling warps of all CTAs; each
//     block streams as two 64-token halves through the warp's two 16 KB TMA
//     stages. A copy engine moves about 60 GB/s into one SM's shared memory,
//     so the HBM stream needs the TMA units of (nearly) every SM. The warp
//     writes the fp32 block mean (row-major [B,H,nb,128], one float4 per
//     lane) and counts it in shared memory (a CTA-scope release only).
//   * warp 3 publishes those counts per head to global memory about every
//     half microsecond behind one GPU-scope fence: the fence sits in a warp
//     with no TMA load in flight, so the streaming warps never wait on it.
//   * warps 4-11 take, as a group, (head, 16 query rows) score items in
//     order, each once every item of its head is counted, and after the last
//     item is taken, coverage tasks of eight rows, each once its rows' batch
//     mean is published. An item streams the head's pooled K (TMA,
//     16-channel chunks) and the rows' pooled Q into shared memory and computes the
//     logits (each thread 8 rows x 4 keys), the softmax per batch element
//     (warp = row), the batch mean and the optional running sums, then
//     publishes the rows' batch mean. A coverage row is one warp
//     (coverage_row.cuh).
// So only the last head's score items and coverage rows run after the HBM
// read ends. Pooling warps never wait on other CTAs, and the task warps take
// only work whose inputs are complete or in progress, so every wait ends.
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

constexpr int kPoolWarps = 3;               // warps 0-2: pooling
constexpr int kSignalWarp = 3;              // warp 3: publishes the head counts
constexpr int kScoreWarp0 = 4;              // warps 4-11: score items and coverage rows
constexpr int kScoreWarps = 8;
constexpr int kScoreThreads = kScoreWarps * 32;
constexpr int kThreads = (kScoreWarp0 + kScoreWarps) * 32;
constexpr int kRows = 16;                   // query rows per score item
constexpr int kD = 128;
constexpr int kHalf = 64;                   // tokens per pooling stage
constexpr int kStageBytes = kHalf * 128 * 2;  // 64 x 128 bf16 = 16 KB
constexpr int kMaxBlocks = 256;
constexpr int kMaxHeads = 128;
constexpr int kKChunks = 8;                 // pooled-K channel chunks of one batch element
constexpr int kKChunkD = kD / kKChunks;     // 16 channels = 16 KB at 256 blocks
constexpr int kKBufs = 2;                   // chunk buffers per batch element of a pair
constexpr int kKBufBytes = kKChunkD * kMaxBlocks * 4;

// counters, one per 128-byte line; [0..3] epoch-tagged, [4] holds the epoch
// once the head counts are cleared, [5 + h] pooling items finished of head h
constexpr int kCtrStride = 128 / 8;  // 64-bit words per line
constexpr int kStartCtr = 0, kScoreCtr = 1, kCovCtr = 2, kDoneCtr = 3, kReady = 4, kHead0 = 5;
size_t counter_bytes(int H) { return (((size_t)(kHead0 + H) * 128) + 255) & ~size_t(255); }
// "batch mean published" flag of every (head, group of kRows rows)
size_t flag_bytes(int H, int nb) {
  return (((size_t)H * ((nb + kRows - 1) / kRows) * 8) + 255) & ~size_t(255);
}

// Shared memory of one CTA (NPAD = keys rounded up to a power of two).
template <int NPAD>
struct Layout {
  static constexpr size_t stages = 0;                                      // [3][2] x 16 KB
  static constexpr size_t kslots = stages + (size_t)kPoolWarps * 2 * kStageBytes;  // [2][2] x 16 KB
  static constexpr size_t qs = kslots + (size_t)2 * kKBufs * kKBufBytes;  // [2][16][128] fp32
  // logits / probabilities of a pair [2][16][NPAD] fp32; coverage rows use
  // the same bytes between items: [8][NPAD] fp32 values, [8][2*NPAD] words
  static constexpr size_t lbuf = qs + (size_t)2 * kRows * kD * 4;
  static constexpr size_t rowbuf = lbuf;
  static constexpr size_t cov = rowbuf + (size_t)kScoreWarps * NPAD * 4;
  static constexpr size_t bars = lbuf + (size_t)2 * kRows * 256 * 4;
  static constexpr size_t hcnt = bars + 128;                               // [kMaxHeads] int
  static constexpr size_t hpub = hcnt + (size_t)kMaxHeads * 4;             // [kMaxHeads] int
  static constexpr size_t ctl = hpub + (size_t)kMaxHeads * 4;              // 16 ints
  static constexpr size_t total = ctl + 64 + 1024;                         // + base alignment
};
static_assert(Layout<256>::total <= 232448, "shared memory layout exceeds 227 KB");
static_assert(Layout<256>::cov + (size_t)kScoreWarps * 2 * 256 * 4 <= Layout<256>::bars,
              "coverage scratch overlaps the barriers");
static_assert(Layout<256>::kslots % 1024 == 0, "swizzled pooled-K buffers need 1 KB alignment");
// barriers: [2w, 2w+1] pooling warp w's stages, [6 + 2 bsel + buf] pooled-K
// buffer buf of the pair's batch element bsel, [10 + bsel] its pooled-Q rows
// ctl: [0] claimed item or task, [1] its inputs are complete, [3] pooling
//      warps done, [5] pooling published

struct Params {
  int B, H, S, nb, G;   // G = score items (groups of kRows rows) per head
  float scale;
  float* qp;            // [B,H,nb,128]
  float* kp;            // [B,H,nb,128]
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
// claimer sees 0. The add is split so that a caller can issue the atomic
// early and look at its result (epoch_add_finish) only where it needs it.
__device__ __forceinline__ uint32_t epoch_add_finish(unsigned long long* c, uint32_t epoch,
                                                     unsigned long long cur) {
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
__device__ __forceinline__ uint32_t epoch_add(unsigned long long* c, uint32_t epoch) {
  return epoch_add_finish(c, epoch, atomicAdd(c, 1ull));
}

__device__ __forceinline__ void score_bar() {
  asm volatile("bar.sync 1, %0;" ::"r"(kScoreThreads) : "memory");
}

// Bounded spin until pred() holds; gives up (false) on timeout, recording
// SA_DEV_WAIT_TIMEOUT. It does not read the status word (possibly host memory).
template <class Pred>
__device__ bool spin_until(Pred pred, int32_t* status, uint32_t sleep_ns) {
  if (pred()) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    __nanosleep(sleep_ns);
    if (pred()) return true;
    if ((it & 63u) == 0u) {
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
  // eight loads issued before the first store of their batch (see coverage_row)
  constexpr int kBatch = NPAD / 32 < 8 ? NPAD / 32 : 8;
#pragma unroll
  for (int q0 = 0; q0 < NPAD / 32; q0 += kBatch) {
    float v[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int c = lane + 32 * (q0 + u);
      v[u] = c < nb ? __ldcg(bm + c) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int c = lane + 32 * (q0 + u);
      if (c < nb) rowbuf[c] = v[u];
    }
  }
  __syncwarp();
  cov::coverage_row<NPAD>(rowbuf, i, p.spec, nullptr, nullptr, skey,
                          reinterpret_cast<float*>(skey + NPAD), mrow,
                          p.flags != nullptr ? p.flags + (int64_t)h * nb + i : nullptr, lane);
  __syncwarp();
}

template <int NPAD>
__global__ void __launch_bounds__(kThreads, 1)
    calib_layer_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_kp, const Params p) {
  using L = Layout<NPAD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::bars);
  float* qs = reinterpret_cast<float*>(smem + L::qs);
  int* hcnt = reinterpret_cast<int*>(smem + L::hcnt);
  int* hpub = reinterpret_cast<int*>(smem + L::hpub);
  volatile int* ctl = reinterpret_cast<volatile int*>(smem + L::ctl);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.nb;
  const int per_head = 2 * p.B * nb;  // pooling items of one head
  const int n_pool = p.H * per_head;
  const int n_score = p.H * p.G;

  for (int i = threadIdx.x; i < p.H; i += kThreads) {
    hcnt[i] = 0;
    hpub[i] = 0;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 12; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
    if (epoch_add(&p.ctr[kStartCtr * kCtrStride], p.epoch) == 0u) {
      // the first CTA to start clears the head counts, then publishes the epoch
      volatile unsigned long long* c = p.ctr;
      for (int h = 0; h < p.H; ++h) c[(kHead0 + h) * kCtrStride] = 0ull;
      __threadfence();
      c[kReady * kCtrStride] = (unsigned long long)p.epoch;
    }
    ctl[3] = 0;
    ctl[5] = 0;
  }
  __syncthreads();

  if (warp < kPoolWarps) {
    // --------------------------------------------------------------- pooling
    // Items (head, batch, q|k, block) in head-major order, dealt to the warps
    // of all CTAs round robin; each block streams as two 64-token halves
    // through this warp's two 16 KB stages.
    uint8_t* stage0 = smem + L::stages + (size_t)warp * 2 * kStageBytes;
    uint64_t* full = &bars[2 * warp];
    if (lane == 0) {
      prefetch_tensormap(&tm_q);
      prefetch_tensormap(&tm_k);
    }
    const int stride = gridDim.x * kPoolWarps;
    const int first = blockIdx.x * kPoolWarps + warp;
    auto issue = [&](int it, int half, int st) {
      const int h = it / per_head;
      const int r = it - h * per_head;
      const int b = r / (2 * nb);
      const int r2 = r - b * 2 * nb;
      const int t = r2 / nb;
      const int j = r2 - t * nb;
      mbar_arrive_expect_tx(&full[st], kStageBytes);
      tma_load_4d(t ? &tm_k : &tm_q, &full[st], stage0 + (size_t)st * kStageBytes, 0,
                  j * 128 + half * kHalf, h, b);
    };
    // halves n = 0, 1, 2, ...: item first + (n / 2) * stride, half n % 2
    const int n_mine = first < n_pool ? 2 * ((n_pool - 1 - first) / stride + 1) : 0;
    if (lane == 0 && n_mine > 0) issue(first, 0, 0);
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    float b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
    uint2 last = make_uint2(0u, 0u);  // the block's final token (ragged blocks)
    for (int n = 0; n < n_mine; ++n) {
      const int st = n & 1;
      const int item = first + (n >> 1) * stride;
      const int half = n & 1;
      __syncwarp();  // every lane is done reading stage st ^ 1 (half n - 1)
      if (lane == 0 && n + 1 < n_mine) {
        fence_proxy_async_smem();
        issue(first + ((n + 1) >> 1) * stride, (n + 1) & 1, st ^ 1);
      }
      if (!mbar_wait_drain(&full[st], (uint32_t)(n >> 1) & 1u)) {
        if (lane == 0) report_timeout(p.status);
        break;
      }
      const int h = item / per_head;
      const int r = item - h * per_head;
      const int b = r / (2 * nb);
      const int r2 = r - b * 2 * nb;
      const int t = r2 / nb;
      const int j = r2 - t * nb;
      const int valid = min(128, p.S - j * 128);
      const uint8_t* tile = stage0 + (size_t)st * kStageBytes + lane * 8;
      // even rows into a*, odd rows into b*, in row order across both halves
#pragma unroll 8
      for (int rr = 0; rr < kHalf; rr += 2) {
        const uint2 u = *reinterpret_cast<const uint2*>(tile + rr * 256);
        const uint2 w = *reinterpret_cast<const uint2*>(tile + (rr + 1) * 256);
        a0 += __uint_as_float(u.x << 16); a1 += __uint_as_float(u.x & 0xffff0000u);
        a2 += __uint_as_float(u.y << 16); a3 += __uint_as_float(u.y & 0xffff0000u);
        b0 += __uint_as_float(w.x << 16); b1 += __uint_as_float(w.x & 0xffff0000u);
        b2 += __uint_as_float(w.y << 16); b3 += __uint_as_float(w.y & 0xffff0000u);
      }
      if (valid < 128 && (valid - 1) / kHalf == half)
        last = *reinterpret_cast<const uint2*>(tile + ((valid - 1) % kHalf) * 256);
      if (half == 0) continue;
      a0 += b0; a1 += b1; a2 += b2; a3 += b3;
      if (valid < 128) {
        // rows past S arrived zero-filled; the final token stands in for them
        const float wgt = (float)(128 - valid);
        a0 += wgt * __uint_as_float(last.x << 16); a1 += wgt * __uint_as_float(last.x & 0xffff0000u);
        a2 += wgt * __uint_as_float(last.y << 16); a3 += wgt * __uint_as_float(last.y & 0xffff0000u);
      }
      const float inv = 1.0f / 128.0f;
      const int64_t bh = (int64_t)b * p.H + h;
      float* outp = (t ? p.kp : p.qp) + (bh * nb + j) * kD + lane * 4;
      *reinterpret_cast<float4*>(outp) = make_float4(a0 * inv, a1 * inv, a2 * inv, a3 * inv);
      a0 = a1 = a2 = a3 = b0 = b1 = b2 = b3 = 0.f;
      // count the item in shared memory (CTA-scope release); the signal warp
      // publishes the counts with the GPU-scope fence
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        atomicAdd(&hcnt[h], 1);
      }
    }
    __syncwarp();
    if (lane == 0) {
      __threadfence_block();
      atomicAdd(const_cast<int*>(&ctl[3]), 1);
    }
  } else if (warp == kSignalWarp) {
    // ----------------------------------------------------- publish head counts
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
  } else {
    const int sw = warp - kScoreWarp0;  // 0..7
    const int tid = threadIdx.x - kScoreWarp0 * 32;
    float* rowbuf = reinterpret_cast<float*>(smem + L::rowbuf) + (size_t)sw * NPAD;
    uint32_t* skey = reinterpret_cast<uint32_t*>(smem + L::cov) + (size_t)sw * 2 * NPAD;
    // ---------------------------------------------------------------- tasks
    // A score item is (head h, kRows query rows) over every batch element,
    // a pair of batch elements at a time. Score warp w computes logits of
    // batch element w / 4 of the pair, rows 8 ((w / 2) % 2) .. +7, and keys
    // lane + 32 (w % 2 + 2 j): per 4 channels a lane reads 8 broadcast Q
    // float4 and 4 K float4 for 128 fmaf, each sum in channel order. Pooled K
    // ([B,H,nb,128] fp32, the layout the pooling writes with whole-sector
    // stores) streams through kKBufs TMA buffers of kKChunkD channels per
    // batch element, each [nb keys][16 channels] with the 64-byte swizzle,
    // so the lanes' key rows fall in distinct banks.
    constexpr int KJ = NPAD >= 64 ? NPAD / 64 : 1;  // keys per lane
    uint64_t* kbar = &bars[6];                 // [bsel * kKBufs + buf]
    uint64_t* qbar = &bars[6 + 2 * kKBufs];    // [bsel]
    uint32_t kpar = 0u, qpar = 0u;  // parity of the next completion of each buffer
    const uint32_t kbytes = (uint32_t)(kKChunkD * nb * 4);
    const float invb = 1.0f / (float)p.B;
    const int npairs = (p.B + 1) / 2;
    const int gb = sw >> 2;                // logits: batch element of the pair
    const int grow = 8 * ((sw >> 1) & 1);  // logits: first of the 8 rows
    const int kh = sw & 1;                 // logits: key interleave
    // output thread tile: rows r0 .. r0 + 3 and keys kb .. kb + 3
    const int r0 = 4 * (sw >> 1);
    const int kb = 4 * (32 * (sw & 1) + lane);
    float* lbuf = reinterpret_cast<float*>(smem + L::lbuf);
    auto kslot = [&](int bsel, int buf) -> uint8_t* {
      return smem + L::kslots + (size_t)(bsel * kKBufs + buf) * kKBufBytes;
    };
    auto wait_copy = [&](uint64_t* bar, uint32_t parity) {
      if (!mbar_wait_drain(bar, parity) && lane == 0) report_timeout(p.status);
    };
    auto item_rows = [&](int s, int& h, int& i0, int& nrows) {
      h = s / p.G;
      i0 = (s - h * p.G) * kRows;
      nrows = min(kRows, nb - i0);
    };
    auto head_ready = [&](int s) {
      return ld_acquire(&p.ctr[(kHead0 + s / p.G) * kCtrStride]) >=
             (unsigned long long)per_head;
    };
    auto issue_k = [&](int h, int b, int bsel, int c) {
      uint64_t* bar = &kbar[bsel * kKBufs + c % kKBufs];
      mbar_arrive_expect_tx(bar, kbytes);
      tma_load_2d(&tm_kp, bar, kslot(bsel, c % kKBufs), c * kKChunkD, (b * p.H + h) * nb);
    };
    // Q rows and the first kKBufs K chunks of pair bp. The head's data was
    // written by other CTAs (generic stores, seen through an acquire of its
    // count). The buffers were last read by this CTA's generic loads before a
    // barrier, as in a producer / consumer pipeline.
    auto issue_pair = [&](int s, int bp) {
      int h, i0, nrows;
      item_rows(s, h, i0, nrows);
      fence_proxy_async_global();
      for (int bsel = 0; bsel < 2; ++bsel) {
        const int b = 2 * bp + bsel;
        if (b >= p.B) break;
        const int64_t bh = (int64_t)b * p.H + h;
        const uint32_t qbytes = (uint32_t)nrows * kD * 4;
        mbar_arrive_expect_tx(&qbar[bsel], qbytes);
        bulk_load(qs + bsel * kRows * kD, p.qp + (bh * nb + i0) * kD, qbytes, &qbar[bsel]);
        for (int c = 0; c < kKBufs; ++c) issue_k(h, b, bsel, c);
      }
    };
    if (tid == 0) prefetch_tensormap(&tm_kp);
    // phase 1: score items, claimed in order with one fetch-and-add each
    for (;;) {
      if (tid == 0) {
        const int s = (int)epoch_add(&p.ctr[kScoreCtr * kCtrStride], p.epoch);
        int ok = 1;
        if (s < n_score)
          ok = spin_until([&] {
                 return ld_acquire(&p.ctr[kReady * kCtrStride]) ==
                            (unsigned long long)p.epoch && head_ready(s);
               }, p.status, 256) ? 1 : 0;
        ctl[0] = s;
        ctl[1] = ok;
      }
      score_bar();
      const int s = ctl[0];
      const int ok = ctl[1];
      score_bar();
      if (s >= n_score) break;
      int h, i0, nrows;
      item_rows(s, h, i0, nrows);
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
      // ------------------------------------------------------- score item
      if (tid == 0) issue_pair(s, 0);
      float bacc[4][4];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int e = 0; e < 4; ++e) bacc[a][e] = 0.f;
      for (int bp = 0; bp < npairs; ++bp) {
        // ---------------------------------------------------- logits of the pair
        const bool active = 2 * bp + gb < p.B;
        float acc[8][KJ];
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
          for (int j = 0; j < KJ; ++j) acc[r][j] = 0.f;
        if (active) {
          wait_copy(&qbar[gb], (qpar >> gb) & 1u);
          qpar ^= 1u << gb;
        }
        const float* qrow = qs + (gb * kRows + grow) * kD;
        for (int c = 0; c < kKChunks; ++c) {
          const int slot = gb * kKBufs + c % kKBufs;
          if (active) {
            wait_copy(&kbar[slot], (kpar >> slot) & 1u);
            kpar ^= 1u << slot;
            const uint8_t* ks = kslot(gb, c % kKBufs);
#pragma unroll
            for (int cq = 0; cq < kKChunkD / 4; ++cq) {
              float kv[KJ][4];
#pragma unroll
              for (int j = 0; j < KJ; ++j) {
                const int key = lane + 32 * (kh + 2 * j);
                const float4 x = *reinterpret_cast<const float4*>(
                    ks + key * (kKChunkD * 4) + ((cq ^ ((key >> 1) & 3)) << 4));
                kv[j][0] = x.x; kv[j][1] = x.y; kv[j][2] = x.z; kv[j][3] = x.w;
              }
              const int d = c * kKChunkD + cq * 4;
#pragma unroll
              for (int r = 0; r < 8; ++r) {
                const float4 q4 = *reinterpret_cast<const float4*>(qrow + r * kD + d);
                const float qv[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
                for (int i = 0; i < 4; ++i)
#pragma unroll
                  for (int j = 0; j < KJ; ++j) acc[r][j] = fmaf(qv[i], kv[j][i], acc[r][j]);
              }
            }
          }
          score_bar();  // every warp is done with this chunk's buffers
          if (tid == 0) {
            if (c + kKBufs < kKChunks) {
              for (int bsel = 0; bsel < 2 && 2 * bp + bsel < p.B; ++bsel)
                issue_k(h, 2 * bp + bsel, bsel, c + kKBufs);
            } else if (c == kKChunks - 1 && bp + 1 < npairs) {
              issue_pair(s, bp + 1);
            }
          }
        }
        if (active) {
          float* lrow = lbuf + (gb * kRows + grow) * NPAD;
#pragma unroll
          for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int j = 0; j < KJ; ++j) {
              const int key = lane + 32 * (kh + 2 * j);
              if (key < nb) lrow[r * NPAD + key] = acc[r][j] * p.scale;
            }
        }
        score_bar();
        // ------------------- softmax of every row of the pair (warp = row)
        // a warp's four rows go together, so their reduction chains overlap
        {
          constexpr int E = NPAD / 32;
          constexpr int RW = 2 * kRows / kScoreWarps;  // rows per warp
          float v[RW][E];
          float m[RW], ssum[RW];
          bool act[RW];
#pragma unroll
          for (int q = 0; q < RW; ++q) {
            const int x = sw + kScoreWarps * q;
            act[q] = 2 * bp + x / kRows < p.B && x % kRows < nrows;
            const float* row = lbuf + (size_t)x * NPAD;
            m[q] = -INFINITY;
#pragma unroll
            for (int j = 0; j < E; ++j) {
              const int c = lane + 32 * j;
              v[q][j] = (act[q] && c < nb) ? row[c] : -INFINITY;
              m[q] = fmaxf(m[q], v[q][j]);
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int q = 0; q < RW; ++q) m[q] = fmaxf(m[q], __shfl_xor_sync(0xffffffffu, m[q], o));
#pragma unroll
          for (int q = 0; q < RW; ++q) {
            ssum[q] = 0.f;
#pragma unroll
            for (int j = 0; j < E; ++j) {
              if (act[q] && lane + 32 * j < nb) {
                v[q][j] = expf(v[q][j] - m[q]);
                ssum[q] += v[q][j];
              }
            }
          }
#pragma unroll
          for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int q = 0; q < RW; ++q) ssum[q] += __shfl_xor_sync(0xffffffffu, ssum[q], o);
#pragma unroll
          for (int q = 0; q < RW; ++q) {
            if (!act[q]) continue;
            float* row = lbuf + (size_t)(sw + kScoreWarps * q) * NPAD;
            const float inv = 1.0f / ssum[q];
#pragma unroll
            for (int j = 0; j < E; ++j)
              if (lane + 32 * j < nb) row[lane + 32 * j] = v[q][j] * inv;
          }
        }
        score_bar();
        // ------------------------------------ probabilities out, batch sum
        for (int bsel = 0; bsel < 2; ++bsel) {
          const int b = 2 * bp + bsel;
          if (b >= p.B) break;
          const int64_t bh = (int64_t)b * p.H + h;
#pragma unroll
          for (int a = 0; a < 4; ++a) {
            if (r0 + a >= nrows) continue;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if (kb + e >= nb) continue;
              const float pv = lbuf[(bsel * kRows + r0 + a) * NPAD + kb + e];
              if (p.scores != nullptr) p.scores[(bh * nb + i0 + r0 + a) * nb + kb + e] = pv;
              bacc[a][e] += pv;
            }
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
    // phase 2: coverage tasks of up to kScoreWarps rows of one group, once
    // every score item is taken (each is then finished by its taker, which
    // waits only on the pooling), so every wait below ends
    if (p.mask != nullptr) {
      const int tph = (nb + kScoreWarps - 1) / kScoreWarps;  // tasks per head
      const int n_tasks = p.H * tph;
      for (;;) {
        if (tid == 0) {
          const int t = (int)epoch_add(&p.ctr[kCovCtr * kCtrStride], p.epoch);
          int ok = 1;
          if (t < n_tasks) {
            const int h = t / tph, row0 = (t - h * tph) * kScoreWarps;
            const int g = h * p.G + row0 / kRows;
            ok = spin_until([&] { return ld_acquire(&p.gflag[g]) ==
                                         (unsigned long long)p.epoch; },
                            p.status, 128) ? 1 : 0;
          }
          ctl[0] = t;
          ctl[1] = ok;
        }
        score_bar();
        const int t = ctl[0];
        const int ok = ctl[1];
        score_bar();
        if (t >= n_tasks) break;
        const int h = t / tph, row0 = (t - h * tph) * kScoreWarps;
        if (row0 + sw < nb)
          coverage_of_row<NPAD>(p, h * nb + row0 + sw, rowbuf, skey, lane, ok != 0);
        score_bar();  // the scratch is shared with the next task's reads
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
      c[kStartCtr * kCtrStride] = 0ull;
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
int launch_t(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mkp,
             const Params& p, int grid, cudaStream_t stream) {
  const int smem = (int)Layout<NPAD>::total;
  if (int rc = func_attr_once((const void*)calib_layer_kernel<NPAD>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      rc != SA_OK)
    return rc;
  calib_layer_kernel<NPAD><<<grid, kThreads, smem, stream>>>(mq, mk, mkp, p);
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
    cuuint32_t box[4] = {128, (cuuint32_t)kHalf, 1, 1};
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
  // pooled K [B*H*nb rows][128] fp32 in the workspace, read by the score
  // items in boxes of 16 channels x nb keys with the 64-byte swizzle
  CUtensorMap mkp;
  {
    const size_t off = counter_bytes(a.H) + flag_bytes(a.H, nb) + (size_t)a.B * a.H * nb * kD * 4;
    cuuint64_t dims[2] = {(cuuint64_t)kD, (cuuint64_t)a.B * a.H * nb};
    cuuint64_t gst[1] = {(cuuint64_t)kD * 4};
    cuuint32_t box[2] = {(cuuint32_t)kKChunkD, (cuuint32_t)nb};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(&mkp, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
                     reinterpret_cast<uint8_t*>(a.workspace) + off, dims, gst, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
      set_error("cuTensorMapEncodeTiled (calibration layer, pooled K) failed (CUresult %d)",
                (int)r);
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
  p.kp = p.qp + (size_t)a.B * a.H * nb * kD;
  p.bm_scratch = p.kp + (size_t)a.B * a.H * nb * kD;
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
  if (nb <= 32) return launch_t<32>(maps[0], maps[1], mkp, p, grid, stream);
  if (nb <= 64) return launch_t<64>(maps[0], maps[1], mkp, p, grid, stream);
  if (nb <= 128) return launch_t<128>(maps[0], maps[1], mkp, p, grid, stream);
  return launch_t<256>(maps[0], maps[1], mkp, p, grid, stream);
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
