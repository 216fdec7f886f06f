// bsattn_fwd.cu — block-sparse attention forward for sm_100a.
//
// Computes, per (batch b, head h, 128-row query tile i), softmax(Q K^T * scale)
// V over the key blocks j whose mask bit (b, hm(h), i, j) is set, plus the
// natural-log logsumexp of every query row. This is the operation the
// reference obtains from the external block_sparse_attn_func
// (sinkattention/sparse_attention.py:735-771): 128x128 blocks, no dropout,
// not causal, scale 1/sqrt(D) by default.
//
// Kernel structure (persistent: one CTA per SM looping over query tiles
// taken from a per-launch tile counter, 512 threads):
//   warp 0       TMA producer: K/V tiles into a 6-slot ring
//   warp 1       QK issuer (one thread): S = Q K^T
//   warp 2       TMEM allocator; then fetches the next tiles and builds their
//                kept-block lists, two tiles ahead
//   warp 3       PV issuer (one thread): O[h] += P[h] V
//   warps 4-7    softmax stream 0: keys 0-63 of every kept block
//   warps 8-11   softmax stream 1: keys 64-127 of every kept block
//   warps 12-15  epilogue: writes the next tile's Q into TMEM and merges the
//                finished tile's two (max, sum, O), writing its output rows
// Each kept 128-key block is split into two 64-key halves. Stream h owns half
// h of every block with its own running maximum, row sum and O accumulator,
// so a stream's thread holds one query row and needs no exchange with the
// other stream until the end of the tile.
//
// Q lives in TMEM, so S = Q K^T is a TS MMA that reads only K from shared
// memory, and shared memory holds nothing but the K/V ring: per block the
// tensor core reads 64 KB of it and TMA writes 64 KB. P has its own TMEM
// columns, and QK and PV come from two issuing threads, so QK of block j+1 is
// issued as soon as both streams have copied S of block j to registers
// (whatever PV is waiting for), and the next S is computed while the softmax
// still works on the current one. The same holds across tiles: the next
// tile's Q is written as soon as the last QK of the current tile completes.
//
// TMEM (512 columns x 128 lanes, 32-bit):
//   S [0,128) (stream h: columns 64h..64h+63)   P[h] [128+32h, 160+32h)
//   Q [192,256) (bf16 pairs)   O[0] [256,384)   O[1] [384,512)
//
// Shared memory: a ring of 6 x 32 KB K/V tiles in the 128-byte-swizzled
// layout TMA writes and UMMA reads (two 64-column boxes per 128x128 tile).
//
// Online softmax uses base-2 exponentials with a lazily updated row maximum:
// the running maximum is only raised (and O, l rescaled) when a block's
// maximum exceeds it by more than 8 (a factor 256), which keeps every P
// value <= 256 and leaves the result exact up to rounding.

#include <math.h>

#include <atomic>

#include "sa_common.cuh"

namespace sa {
namespace attn {

constexpr int kBM = 128;      // query rows per tile
constexpr int kBN = 128;      // keys per block
constexpr int kHalf = 64;     // keys per stream per block
constexpr int kHD = 128;      // head dim
constexpr int kStages = 6;    // K/V ring slots
constexpr int kThreads = 512;  // 4 role warps + 2 softmax warpgroups + 1 epilogue warpgroup
constexpr int kTileBytes = kBM * kHD * 2;   // 32 KB bf16 tile
constexpr int kBoxBytes = kTileBytes / 2;   // one 64-column box
constexpr int kHalfRowsBytes = kHalf * 128; // 64 rows of a box: 8 KB
constexpr int kMaxBlocks = 1024;            // max key blocks per row (S <= 131072)
constexpr float kRescaleThreshold = 8.0f;   // log2 units
// readers of a kept-block list slot: TMA, QK and PV threads, 256 softmax and
// 128 epilogue threads
constexpr int kListReaders = 3 + 256 + 128;
// TMEM columns
constexpr uint32_t kColS = 0, kColP = 128, kColQ = 192, kColO = 256;

struct Params {
  int B, H, Sq, Sk, nq, nk;
  int Sk2, nk2;      // pooled (dynamic-branch) keys appended to every row; 0 if none
  float bias_log2;   // logit bias of the pooled keys, log2 units (ln(gap) * log2(e))
  const uint8_t* mask;
  int64_t ms0, ms1, ms2, ms3;
  const int32_t* head_mask_type;
  float scale_log2;  // softmax_scale * log2(e)
  const __nv_bfloat16* q;
  int64_t qs0, qs1, qs2;
  __nv_bfloat16* out;
  int64_t os0, os1, os2;
  float* lse;
  int32_t* status;
  int tiles;         // nq * H * B
  int sched;         // tile-counter slot of this launch
};

// Dynamic tile scheduler: per launch slot, [0] the next tile to hand out and
// [1] the CTAs that have finished. The last CTA of a launch resets both, so
// the slot is zero for the next launch that uses it; launches take slots
// round robin, so concurrent launches on different streams use different
// slots.
constexpr int kSchedSlots = 1024;  // 8 KB per device
__device__ int g_sched[kSchedSlots][2];

struct __align__(8) SmemCtl {
  uint64_t kv_full[kStages];
  uint64_t kv_empty[kStages];
  uint64_t list_full[2];   // [slot] kept-block list of a tile written, 1 arrival
  uint64_t list_empty[2];  // [slot] released by every reader, kListReaders arrivals
  uint64_t q_ready;        // Q of a tile written to TMEM (epilogue group), 128 arrivals
  uint64_t q_free;         // the last QK of a tile is complete (commit)
  uint64_t s_full;         // S of a block computed (commit)
  uint64_t s_free;         // S of a block copied out by both streams, 256 arrivals
  uint64_t p_full[2];      // [stream], 128 arrivals per phase
  uint64_t pv_done[2];     // [stream], committed after each PV
  uint64_t o_final[2];     // [stream], committed after a tile's last PV
  uint64_t x_ready[2];     // [tile parity] both streams' (max, sum) written, 256 arrivals
  uint64_t o_free;         // the epilogue has read O of a tile, 128 arrivals
  uint64_t mma_drain[2];   // [0] QK issuer, [1] PV issuer
  uint32_t tmem_base;
  int abort_flag;
  int n_blocks[2];         // [slot]
  int tile_id[2];          // [slot] tile of the list, -1: no more tiles
  uint16_t list[2][kMaxBlocks];  // [slot] key blocks; bit 15 marks a pooled-key block
  float xm[2][2][kBM];     // [tile parity][stream][row]
  float xl[2][2][kBM];
};

constexpr size_t kSmemBytes = 1024 /*align slack*/ + kStages * kTileBytes + sizeof(SmemCtl);

// The order in which K/V tiles are produced and consumed:
//   K(0), then for every j: K(j+1) (if any), V(j)
// so QK of block j+1 is issued before PV of block j.
template <typename F>
__device__ __forceinline__ void for_each_item(const int n, F&& f) {
  if (n <= 0) return;
  if (!f(0, 0)) return;
  for (int j = 0; j < n; ++j) {
    if (j + 1 < n && !f(j + 1, 0)) return;
    if (!f(j, 1)) return;
  }
}

__device__ __forceinline__ void tile_coords(const Params& p, int t, int& qt, int& h, int& b) {
  qt = t % p.nq;
  const int bh = t / p.nq;
  h = bh % p.H;
  b = bh / p.H;
}

// Persistent grid, one CTA per SM. Warp 2 takes the CTA's next tile from the
// launch's tile counter (tile t = query tile t % nq of head t / nq) and
// publishes it with its kept-block list, two tiles ahead, in one of two list
// slots; every role walks that same sequence. The barriers of the per-block
// pipeline (ring slots, S, P, PV) count blocks over all of the CTA's tiles,
// so the pipeline runs from one tile into the next without draining; the
// per-tile barriers count the tiles that have kept blocks.
__global__ void __launch_bounds__(kThreads, 1)
    bsattn_fwd_kernel(const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v,
                      const __grid_constant__ CUtensorMap tm_k2,
                      const __grid_constant__ CUtensorMap tm_v2, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* ring = smem;
  SmemCtl* ctl = reinterpret_cast<SmemCtl*>(ring + kStages * kTileBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // The status word is written on failure and never read here: it lives in
  // mapped host memory, and one read of it per CTA at entry cost 60-90 us per
  // launch (148 PCIe round trips).

  // ---- set-up: barriers, TMEM ----------------------------------------------
  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&ctl->kv_full[i], 1);
      mbar_init(&ctl->kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->list_full[i], 1);
      mbar_init(&ctl->list_empty[i], kListReaders);
      mbar_init(&ctl->p_full[i], kBM);
      mbar_init(&ctl->pv_done[i], 1);
      mbar_init(&ctl->o_final[i], 1);
      mbar_init(&ctl->x_ready[i], 2 * kBM);
      mbar_init(&ctl->mma_drain[i], 1);
    }
    mbar_init(&ctl->q_ready, kBM);
    mbar_init(&ctl->q_free, 1);
    mbar_init(&ctl->s_full, 1);
    mbar_init(&ctl->s_free, 2 * kBM);
    mbar_init(&ctl->o_free, kBM);
    ctl->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tensormap(&tm_k);
    prefetch_tensormap(&tm_v);
    if (p.nk2 > 0) {
      prefetch_tensormap(&tm_k2);
      prefetch_tensormap(&tm_v2);
    }
  }
  if (warp == 2) {
    tmem_alloc(&ctl->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const uint32_t tmem = ctl->tmem_base;
  volatile int* abort_flag = &ctl->abort_flag;

  if (warp == 2) {
    // ---------------- kept-block lists, two tiles ahead ----------------
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int slot = k & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&ctl->list_empty[slot],
                                             ((uint32_t)(k >> 1) & 1u) ^ 1u, p.status,
                                             abort_flag));
      if (!ok) break;
      // the next tile from the launch's counter (tiles are handed out in
      // order, so the CTAs work on neighbouring tiles of one head at a time)
      int t = 0;
      if (lane == 0) t = atomicAdd(&g_sched[p.sched][0], 1);
      t = __shfl_sync(0xffffffffu, t, 0);
      if (t >= p.tiles) {
        if (lane == 0) {
          ctl->tile_id[slot] = -1;
          ctl->n_blocks[slot] = 0;
          mbar_arrive(&ctl->list_full[slot]);
        }
        break;
      }
      int qt, h, b;
      tile_coords(p, t, qt, h, b);
      int mh = h;
      bool dense = false;
      if (p.head_mask_type != nullptr) {
        const int ty = p.head_mask_type[h];
        if (ty > 0) mh = ty - 1; else dense = true;
      }
      const uint8_t* row =
          p.mask + (int64_t)b * p.ms0 + (int64_t)mh * p.ms1 + (int64_t)qt * p.ms2;
      // all mask bytes of the row are loaded before any is used: bit i of
      // `bits` is block 32 i + lane
      const int nw = (p.nk + 31) >> 5;  // <= 32 (nk <= kMaxBlocks)
      uint32_t bits = 0;
#pragma unroll 8
      for (int i = 0; i < nw; ++i) {
        const int c = i * 32 + lane;
        const bool keep = c < p.nk && (dense || row[(int64_t)c * p.ms3] != 0);
        bits |= (uint32_t)keep << i;
      }
      uint16_t* list = ctl->list[slot];
      int count = 0;
      for (int i = 0; i < nw; ++i) {
        const bool keep = (bits >> i) & 1u;
        const uint32_t bal = __ballot_sync(0xffffffffu, keep);
        if (keep) list[count + __popc(bal & ((1u << lane) - 1u))] = (uint16_t)(i * 32 + lane);
        count += __popc(bal);
      }
      // the dynamic branch: every pooled-key block, after the kept sink blocks
      for (int u = lane; u < p.nk2; u += 32) list[count + u] = (uint16_t)(0x8000u | u);
      count += p.nk2;
      if (lane == 0) {
        ctl->n_blocks[slot] = count;
        ctl->tile_id[slot] = t;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&ctl->list_full[slot]);
    }
  } else if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int slot = k & 1;
        if (!mbar_wait(&ctl->list_full[slot], (uint32_t)(k >> 1) & 1u, p.status, abort_flag)) {
          ok = false;
          break;
        }
        const int t = ctl->tile_id[slot];
        if (t < 0) break;
        int qt, h, b;
        tile_coords(p, t, qt, h, b);
        (void)qt;
        const int n = ctl->n_blocks[slot];
        const uint16_t* list = ctl->list[slot];
        for_each_item(n, [&](const int j, const int is_v) -> bool {
          const int stage = it % kStages;
          const uint32_t phase = (uint32_t)(it / kStages) & 1u;
          if (!mbar_wait(&ctl->kv_empty[stage], phase ^ 1u, p.status, abort_flag)) {
            ok = false;
            return false;
          }
          uint8_t* dst = ring + stage * kTileBytes;
          const uint32_t ent = list[j];
          const int kb = (int)(ent & 0x7fffu);
          const bool pooled = (ent & 0x8000u) != 0;
          const CUtensorMap* map = is_v ? (pooled ? &tm_v2 : &tm_v) : (pooled ? &tm_k2 : &tm_k);
          mbar_arrive_expect_tx(&ctl->kv_full[stage], kTileBytes);
          tma_load_4d(map, &ctl->kv_full[stage], dst, 0, kb * kBN, h, b);
          tma_load_4d(map, &ctl->kv_full[stage], dst + kBoxBytes, 64, kb * kBN, h, b);
          ++it;
          return true;
        });
        if (ok) mbar_arrive(&ctl->list_empty[slot]);
      }
      // Drain: make sure no TMA write is still in flight before the CTA exits.
      for (int i = (it > kStages ? it - kStages : 0); i < it; ++i)
        mbar_wait_drain(&ctl->kv_full[i % kStages], (uint32_t)(i / kStages) & 1u);
    }
    __syncwarp();
  } else if (warp == 1 || warp == 3) {
    // ---------------- MMA issuers: warp 1 QK, warp 3 PV ----------------
    // Both walk the K/V sequence to find the ring stage of each item and
    // take only their own kind (K tiles for QK, V tiles for PV).
    const int role_v = warp == 3 ? 1 : 0;
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_bf16(kBM, kBN, 0, 0);
      constexpr uint32_t idesc_pv = make_idesc_bf16(kBM, kHD, 0, 1);
      const uint32_t ring_base = smem_u32(ring);
      int it = 0;   // ring items walked
      int jg = 0;   // blocks of earlier tiles
      int e = 0;    // earlier tiles with kept blocks
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int slot = k & 1;
        if (!mbar_wait(&ctl->list_full[slot], (uint32_t)(k >> 1) & 1u, p.status, abort_flag)) {
          ok = false;
          break;
        }
        if (ctl->tile_id[slot] < 0) break;
        const int n = ctl->n_blocks[slot];
        if (n > 0 && !role_v) {
          // Q of this tile in TMEM (the epilogue group writes it once the
          // previous tile's last QK has completed)
          if (!mbar_wait(&ctl->q_ready, (uint32_t)e & 1u, p.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        for_each_item(n, [&](const int j, const int is_v) -> bool {
          if (is_v != role_v) {
            ++it;
            return true;
          }
          const int J = jg + j;
          const int stage = it % kStages;
          const uint32_t phase = (uint32_t)(it / kStages) & 1u;
          if (!is_v && J > 0) {
            // S is single-buffered: both streams have copied S(J-1) out
            if (!mbar_wait(&ctl->s_free, (uint32_t)(J - 1) & 1u, p.status, abort_flag)) {
              ok = false;
              return false;
            }
          }
          if (is_v && j == 0 && e > 0) {
            // the first PV of a tile overwrites O: the epilogue group has read
            // the previous tile's O
            if (!mbar_wait(&ctl->o_free, (uint32_t)(e - 1) & 1u, p.status, abort_flag)) {
              ok = false;
              return false;
            }
          }
          if (!mbar_wait(&ctl->kv_full[stage], phase, p.status, abort_flag)) {
            ok = false;
            return false;
          }
          const uint32_t tile = ring_base + stage * kTileBytes;
          if (!is_v) {
            tc_fence_after();
            // S = Q (TMEM) . K^T (shared memory), all 128 keys of the block
#pragma unroll
            for (int kk = 0; kk < kHD / 16; ++kk) {
              const uint32_t off = (kk >> 2) * kBoxBytes + (kk & 3) * 32;
              mma_ts(tmem + kColS, tmem + kColQ + kk * 8, make_sdesc_sw128(tile + off, 16, 1024),
                     idesc_qk, kk > 0 ? 1u : 0u);
            }
            mma_commit(&ctl->s_full);
            mma_commit(&ctl->kv_empty[stage]);
            if (j == n - 1) mma_commit(&ctl->q_free);  // Q columns may be rewritten
          } else {
#pragma unroll
            for (int st = 0; st < 2; ++st) {
              if (!mbar_wait(&ctl->p_full[st], (uint32_t)J & 1u, p.status, abort_flag)) {
                ok = false;
                return false;
              }
              tc_fence_after();
              // O[st] += P[st] (128 x 64, bf16 in TMEM) . V[keys 64st .. 64st+63]
#pragma unroll
              for (int kk = 0; kk < kHalf / 16; ++kk) {
                const uint64_t bd =
                    make_sdesc_sw128(tile + st * kHalfRowsBytes + kk * 2048, kBoxBytes, 1024);
                mma_ts(tmem + kColO + st * 128, tmem + kColP + st * 32 + kk * 8, bd, idesc_pv,
                       (j > 0 || kk > 0) ? 1u : 0u);
              }
              mma_commit(&ctl->pv_done[st]);
              if (j == n - 1) mma_commit(&ctl->o_final[st]);
            }
            mma_commit(&ctl->kv_empty[stage]);
          }
          ++it;
          return true;
        });
        if (!ok) break;
        if (n > 0) {
          jg += n;
          ++e;
        }
        mbar_arrive(&ctl->list_empty[slot]);
      }
      // Drain every MMA this thread issued before TMEM can be released.
      mma_commit(&ctl->mma_drain[role_v]);
      mbar_wait_drain(&ctl->mma_drain[role_v], 0);
    }
    __syncwarp();
  } else if (warp < 12) {
    // ---------------- softmax streams ----------------
    // Stream st = 0/1 (warps 4-7 / 8-11) owns keys 64st..64st+63 of every
    // kept block. Thread (warp quarter wq, lane) owns query row wq*32+lane,
    // which is TMEM lane wq*32+lane.
    const int st = (warp - 4) >> 2;
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    bool ok = true;
    int jg = 0, e = 0;
    for (int k = 0; ok; ++k) {
      const int slot = k & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&ctl->list_full[slot], (uint32_t)(k >> 1) & 1u,
                                             p.status, abort_flag));
      if (!ok) break;
      if (ctl->tile_id[slot] < 0) break;
      const int n = ctl->n_blocks[slot];
      const uint16_t* list = ctl->list[slot];
      float m_used = -INFINITY;
      float l = 0.f;
      for (int j = 0; j < n && ok; ++j) {
        const int J = jg + j;
        // the block's list entry, read before the wait (the list is complete
        // once list_full has passed; after the wait's memory clobber the
        // read would sit on the block's path)
        const uint32_t ent = list[j];
        // warp-uniform outcome: the TMEM loads below are warp-collective
        if (!__all_sync(0xffffffffu,
                        mbar_wait(&ctl->s_full, (uint32_t)J & 1u, p.status, abort_flag))) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r[2][32];
        tmem_ld32(tmem + lane_off + kColS + st * kHalf + 0, r[0]);
        tmem_ld32(tmem + lane_off + kColS + st * kHalf + 32, r[1]);
        tmem_wait_ld();
        reg_fence32(r[0]);
        reg_fence32(r[1]);
        tc_fence_before();
        mbar_arrive(&ctl->s_free);  // S may be overwritten by the next QK
        const int kb = (int)(ent & 0x7fffu);
        const bool pooled = (ent & 0x8000u) != 0;
        const int valid = min(kHalf, (pooled ? p.Sk2 : p.Sk) - kb * kBN - st * kHalf);
        const float bias = pooled ? p.bias_log2 : 0.f;
        if (valid < kHalf) {
#pragma unroll
          for (int c = 0; c < kHalf; ++c)
            if (c >= valid) r[c >> 5][c & 31] = __float_as_uint(-INFINITY);
        }
        // Row maximum over this stream's 64 columns: 8 chains of 3-input max.
        float mxp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mxp[u] = __uint_as_float(r[0][u]);
#pragma unroll
        for (int c = 8; c + 16 <= kHalf; c += 16) {
#pragma unroll
          for (int u = 0; u < 8; ++u)
            mxp[u] = fmax3(mxp[u], __uint_as_float(r[(c + u) >> 5][(c + u) & 31]),
                           __uint_as_float(r[(c + 8 + u) >> 5][(c + 8 + u) & 31]));
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) mxp[u] = fmaxf(mxp[u], __uint_as_float(r[1][24 + u]));
        const float mx_raw = fmax3(fmax3(mxp[0], mxp[1], mxp[2]), fmax3(mxp[3], mxp[4], mxp[5]),
                                   fmaxf(mxp[6], mxp[7]));
        const float mx = fmaf(mx_raw, p.scale_log2, bias);  // -inf stays -inf
        float alpha = 1.0f;
        const bool rescale = mx > m_used + kRescaleThreshold;
        if (rescale) {
          alpha = ex2_approx(m_used - mx);  // 0 when m_used = -inf
          l *= alpha;
          m_used = mx;
        }
        // P = exp2(S*scale*log2e + bias - m); a row that has seen no valid key
        // yet (m = -inf) gets P = 0 from its -inf inputs.
        const float negm = m_used == -INFINITY ? 0.f : -m_used;
        const uint64_t scale2 = f2_pack(p.scale_log2, p.scale_log2);
        const uint64_t negm2 = f2_pack(bias + negm, bias + negm);
        uint64_t lp2[4] = {0ull, 0ull, 0ull, 0ull};
        uint32_t pk[32];
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          const int c = 2 * u;
          const uint64_t x2 = f2_fma(f2_pack(__uint_as_float(r[c >> 5][c & 31]),
                                             __uint_as_float(r[(c + 1) >> 5][(c + 1) & 31])),
                                     scale2, negm2);
          float x0, x1;
          f2_unpack(x2, x0, x1);
          const float p0 = ex2_approx(x0);
          const float p1 = ex2_approx(x1);
          lp2[u & 3] = f2_add(lp2[u & 3], f2_pack(p0, p1));
          pk[u] = pack_bf16x2(p0, p1);
        }
        {
          const uint64_t t2 = f2_add(f2_add(lp2[0], lp2[1]), f2_add(lp2[2], lp2[3]));
          float a0, a1;
          f2_unpack(t2, a0, a1);
          l += a0 + a1;
        }
        // P[st] (and O[st]) are free once the previous PV has completed, which
        // may belong to the previous tile.
        if (J > 0) {
          if (!__all_sync(0xffffffffu, mbar_wait(&ctl->pv_done[st], (uint32_t)(J - 1) & 1u,
                                                 p.status, abort_flag))) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        tmem_st32(tmem + lane_off + kColP + st * 32, pk);
        // Rescale O when the maximum moved after the tile's first block.
        // tcgen05.ld/st are warp-collective (.sync.aligned): the whole warp
        // takes this branch when any of its rows rescales; other rows use 1.
        if (__any_sync(0xffffffffu, rescale && j > 0)) {
          if (!(rescale && j > 0)) alpha = 1.0f;
          const uint32_t o_self = tmem + lane_off + kColO + st * 128;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(o_self + c * 32, o);
            tmem_wait_ld();
            reg_fence32(o);
#pragma unroll
            for (int u = 0; u < 32; ++u) o[u] = __float_as_uint(__uint_as_float(o[u]) * alpha);
            tmem_st32(o_self + c * 32, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&ctl->p_full[st]);
      }
      if (!ok) break;
      if (n > 0) {
        // this stream's (max, sum) of the row, for the epilogue group
        ctl->xm[e & 1][st][row] = m_used;
        ctl->xl[e & 1][st][row] = l;
        mbar_arrive(&ctl->x_ready[e & 1]);
        jg += n;
        ++e;
      }
      mbar_arrive(&ctl->list_empty[slot]);
    }
  } else {
    // ---------------- epilogue group (warps 12-15) ----------------
    // For each tile with kept blocks: write its Q into TMEM as soon as the
    // previous tile's last QK has completed, then finish the previous tile
    // (merge the two streams' max, sum and O; write the output rows and LSE)
    // while the softmax streams already work on this one.
    const int wq = warp & 3;
    const int row = wq * 32 + lane;
    const uint32_t lane_off = (uint32_t)(wq * 32) << 16;
    bool ok = true;
    int e = 0;
    int prev_t = -1;  // the last tile with kept blocks whose output is pending

    auto finish = [&](const int tp, const int ep) {
      int qt, h, b;
      tile_coords(p, tp, qt, h, b);
      const int grow = qt * kBM + row;
      if (ok)
        ok = __all_sync(0xffffffffu,
                        mbar_wait(&ctl->o_final[0], (uint32_t)ep & 1u, p.status, abort_flag) &&
                            mbar_wait(&ctl->o_final[1], (uint32_t)ep & 1u, p.status,
                                      abort_flag) &&
                            mbar_wait(&ctl->x_ready[ep & 1], (uint32_t)(ep >> 1) & 1u,
                                      p.status, abort_flag));
      if (!ok) return;
      tc_fence_after();
      const float m0 = ctl->xm[ep & 1][0][row], m1 = ctl->xm[ep & 1][1][row];
      const float l0 = ctl->xl[ep & 1][0][row], l1 = ctl->xl[ep & 1][1][row];
      const float m = fmaxf(m0, m1);
      const float a0 = m0 == -INFINITY ? 0.f : ex2_approx(m0 - m);
      const float a1 = m1 == -INFINITY ? 0.f : ex2_approx(m1 - m);
      const float L = l0 * a0 + l1 * a1;
      const float inv_l = 1.0f / L;
      const float w0 = a0 * inv_l, w1 = a1 * inv_l;
      const bool write = grow < p.Sq;
      __nv_bfloat16* orow =
          p.out + (int64_t)b * p.os0 + (int64_t)h * p.os1 + (int64_t)grow * p.os2;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t o0[32], o1[32];
        tmem_ld32(tmem + lane_off + kColO + c * 32, o0);
        tmem_ld32(tmem + lane_off + kColO + 128 + c * 32, o1);
        tmem_wait_ld();
        reg_fence32(o0);
        reg_fence32(o1);
        if (write) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint32_t w[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const int i0 = 8 * v + 2 * u;
              w[u] = pack_bf16x2(
                  fmaf(__uint_as_float(o0[i0]), w0, __uint_as_float(o1[i0]) * w1),
                  fmaf(__uint_as_float(o0[i0 + 1]), w0, __uint_as_float(o1[i0 + 1]) * w1));
            }
            dst[v] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&ctl->o_free);  // O may be overwritten by the next tile's first PV
      if (write && p.lse != nullptr)
        p.lse[((int64_t)b * p.H + h) * p.Sq + grow] = (m + __log2f(L)) * 0.69314718055994531f;
    };

    for (int k = 0; ok; ++k) {
      const int slot = k & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&ctl->list_full[slot], (uint32_t)(k >> 1) & 1u,
                                             p.status, abort_flag));
      if (!ok) break;
      const int t = ctl->tile_id[slot];
      if (t < 0) break;
      const int n = ctl->n_blocks[slot];
      mbar_arrive(&ctl->list_empty[slot]);  // only t and n are needed from the slot
      int qt, h, b;
      tile_coords(p, t, qt, h, b);
      const int grow = qt * kBM + row;
      if (n == 0) {
        // no kept block: zero output, LSE -inf
        if (grow < p.Sq) {
          uint4* dst = reinterpret_cast<uint4*>(p.out + (int64_t)b * p.os0 + (int64_t)h * p.os1 +
                                                (int64_t)grow * p.os2);
          for (int v = 0; v < 16; ++v) dst[v] = make_uint4(0, 0, 0, 0);
          if (p.lse != nullptr) p.lse[((int64_t)b * p.H + h) * p.Sq + grow] = -INFINITY;
        }
        continue;
      }
      // Q row of this tile -> TMEM columns [kColQ, kColQ+64) as bf16 pairs
      // (the A-operand layout of the QK MMA). Rows past Sq are 0.
      uint32_t qv[2][32];
      if (grow < p.Sq) {
        const uint4* src = reinterpret_cast<const uint4*>(
            p.q + (int64_t)b * p.qs0 + (int64_t)h * p.qs1 + (int64_t)grow * p.qs2);
#pragma unroll
        for (int v = 0; v < 16; ++v) {
          const uint4 w = src[v];
          qv[v >> 3][4 * (v & 7)] = w.x; qv[v >> 3][4 * (v & 7) + 1] = w.y;
          qv[v >> 3][4 * (v & 7) + 2] = w.z; qv[v >> 3][4 * (v & 7) + 3] = w.w;
        }
      } else {
#pragma unroll
        for (int u = 0; u < 32; ++u) qv[0][u] = qv[1][u] = 0u;
      }
      if (e > 0)
        ok = __all_sync(0xffffffffu, mbar_wait(&ctl->q_free, (uint32_t)(e - 1) & 1u, p.status,
                                               abort_flag));
      if (!ok) break;
      tc_fence_after();
      tmem_st32(tmem + lane_off + kColQ, qv[0]);
      tmem_st32(tmem + lane_off + kColQ + 32, qv[1]);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&ctl->q_ready);
      if (prev_t >= 0) finish(prev_t, e - 1);
      prev_t = t;
      ++e;
    }
    if (ok && prev_t >= 0) finish(prev_t, e - 1);
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 2) tmem_dealloc(tmem, 512);
  if (threadIdx.x == 0) {
    // every tile fetch of this CTA is done: the last CTA resets the slot
    __threadfence();
    if (atomicAdd(&g_sched[p.sched][1], 1) == (int)gridDim.x - 1) {
      g_sched[p.sched][0] = 0;
      g_sched[p.sched][1] = 0;
      __threadfence();
    }
  }
}

}  // namespace attn
}  // namespace sa

// ---------------------------------------------------------------------------
// Host entry point
// ---------------------------------------------------------------------------
namespace {

int make_map_bshd(CUtensorMap* map, const void* base, const int64_t st[4], int B, int H, int S,
                  int D) {
  sa::EncodeTiledFn enc = sa::encode_tiled_fn();
  if (enc == nullptr) return SA_ECUDA;
  // dims innermost first: (D, S, H, B); strides in bytes for dims 1..3.
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)st[2] * 2, (cuuint64_t)st[1] * 2, (cuuint64_t)st[0] * 2};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    sa::set_error("cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return SA_ECUDA;
  }
  return SA_OK;
}

bool strides_ok(const int64_t st[4]) {
  if (st[3] != 1) return false;
  for (int i = 0; i < 3; ++i)
    if (st[i] < 0 || (st[i] % 8) != 0) return false;
  return true;
}

}  // namespace

namespace {

// Shared by sa_bsattn_fwd (k2 == nullptr) and sa_sink_dynamic_attn_fwd.
int launch_attention(const char* fn, const void* q, const void* k, const void* v,
                     const int64_t q_strides[4], const int64_t k_strides[4],
                     const int64_t v_strides[4], int B, int H, int Sq, int Sk, int D,
                     const uint8_t* block_mask, const int64_t m_strides[4], int Hm,
                     const int32_t* head_mask_type, const void* k2, const void* v2,
                     const int64_t* k2_strides, const int64_t* v2_strides, int Sk2,
                     float log_bias, float softmax_scale, void* out, const int64_t o_strides[4],
                     float* lse, int32_t* status, cudaStream_t stream) {
  using namespace sa::attn;
  SA_CHECK_ARG(q && k && v && out && block_mask, "%s: null tensor pointer", fn);
  SA_CHECK_ARG(q_strides && k_strides && v_strides && o_strides && m_strides,
               "%s: null stride array", fn);
  SA_CHECK_ARG(D == kHD, "%s: head dim must be 128, got %d", fn, D);
  SA_CHECK_ARG(B >= 1 && H >= 1 && Sq >= 1 && Sk >= 1,
               "%s: B, H, Sq, Sk must be >= 1 (got %d, %d, %d, %d)", fn, B, H, Sq, Sk);
  const int nq = (Sq + kBM - 1) / kBM;
  const int nk = (Sk + kBN - 1) / kBN;
  const bool dual = k2 != nullptr;
  const int nk2 = dual ? (Sk2 + kBN - 1) / kBN : 0;
  SA_CHECK_ARG(!dual || (v2 && k2_strides && v2_strides && Sk2 >= 1),
               "%s: pooled keys need k2, v2, their strides and Sk2 >= 1", fn);
  SA_CHECK_ARG(nk + nk2 <= kMaxBlocks && nk2 < 0x8000,
               "%s: %d + %d key blocks exceed %d", fn, nk, nk2, kMaxBlocks);
  SA_CHECK_ARG((int64_t)nq * H * B <= 0x7fffffff, "%s: too many query tiles", fn);
  SA_CHECK_ARG(strides_ok(q_strides) && strides_ok(k_strides) && strides_ok(v_strides) &&
                   strides_ok(o_strides) && (!dual || (strides_ok(k2_strides) && strides_ok(v2_strides))),
               "%s: q/k/v/out need stride(dim)=1 and other strides multiple of 8 "
               "elements (16 bytes)", fn);
  SA_CHECK_ARG(((uintptr_t)q | (uintptr_t)k | (uintptr_t)v | (uintptr_t)out |
                (uintptr_t)(dual ? k2 : q) | (uintptr_t)(dual ? v2 : q)) % 16 == 0,
               "%s: tensor base pointers must be 16-byte aligned", fn);
  SA_CHECK_ARG(head_mask_type != nullptr || Hm == H,
               "%s: mask has %d heads but H=%d and no head_mask_type", fn, Hm, H);
  SA_CHECK_ARG(Hm >= 1, "%s: mask heads must be >= 1", fn);

  CUtensorMap tk, tv, tk2, tv2;
  int rc;
  if ((rc = make_map_bshd(&tk, k, k_strides, B, H, Sk, D)) != SA_OK) return rc;
  if ((rc = make_map_bshd(&tv, v, v_strides, B, H, Sk, D)) != SA_OK) return rc;
  if (dual) {
    if ((rc = make_map_bshd(&tk2, k2, k2_strides, B, H, Sk2, D)) != SA_OK) return rc;
    if ((rc = make_map_bshd(&tv2, v2, v2_strides, B, H, Sk2, D)) != SA_OK) return rc;
  } else {
    tk2 = tk;  // unused
    tv2 = tv;
  }

  Params p;
  p.B = B; p.H = H; p.Sq = Sq; p.Sk = Sk; p.nq = nq; p.nk = nk;
  p.Sk2 = dual ? Sk2 : 0;
  p.nk2 = nk2;
  p.bias_log2 = dual ? log_bias * 1.4426950408889634f : 0.f;
  p.mask = block_mask;
  p.ms0 = m_strides[0]; p.ms1 = m_strides[1]; p.ms2 = m_strides[2]; p.ms3 = m_strides[3];
  p.head_mask_type = head_mask_type;
  const float scale = softmax_scale > 0.f ? softmax_scale : 1.0f / sqrtf((float)D);
  p.scale_log2 = scale * 1.4426950408889634f;
  p.q = reinterpret_cast<const __nv_bfloat16*>(q);
  p.qs0 = q_strides[0]; p.qs1 = q_strides[1]; p.qs2 = q_strides[2];
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.os0 = o_strides[0]; p.os1 = o_strides[1]; p.os2 = o_strides[2];
  p.lse = lse;
  p.status = status;
  p.tiles = nq * H * B;
  static std::atomic<unsigned> launch_seq{0};
  p.sched = (int)(launch_seq.fetch_add(1, std::memory_order_relaxed) % kSchedSlots);

  if (int rc = sa::func_attr_once((const void*)bsattn_fwd_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
      rc != SA_OK)
    return rc;
  // persistent grid: one CTA per SM (at most one per tile)
  const int sms = sa::sm_count_current_device();
  const int grid = p.tiles < sms ? p.tiles : sms;
  bsattn_fwd_kernel<<<grid, kThreads, kSmemBytes, stream>>>(tk, tv, tk2, tv2, p);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

}  // namespace

extern "C" int sa_bsattn_fwd(const void* q, const void* k, const void* v,
                             const int64_t q_strides[4], const int64_t k_strides[4],
                             const int64_t v_strides[4], int B, int H, int Sq, int Sk, int D,
                             const uint8_t* block_mask, const int64_t m_strides[4], int Hm,
                             const int32_t* head_mask_type, float softmax_scale, void* out,
                             const int64_t o_strides[4], float* lse, int32_t* status,
                             cudaStream_t stream) {
  return launch_attention("sa_bsattn_fwd", q, k, v, q_strides, k_strides, v_strides, B, H, Sq,
                          Sk, D, block_mask, m_strides, Hm, head_mask_type, nullptr, nullptr,
                          nullptr, nullptr, 0, 0.f, softmax_scale, out, o_strides, lse, status,
                          stream);
}

extern "C" int sa_sink_dynamic_attn_fwd(
    const void* q, const void* k, const void* v, const int64_t q_strides[4],
    const int64_t k_strides[4], const int64_t v_strides[4], int B, int H, int Sq, int Sk, int D,
    const uint8_t* block_mask, const int64_t m_strides[4], int Hm, const int32_t* head_mask_type,
    const void* k_pool, const void* v_pool, const int64_t kp_strides[4],
    const int64_t vp_strides[4], int Sk_pool, float log_gap, float softmax_scale, void* out,
    const int64_t o_strides[4], float* lse, int32_t* status, cudaStream_t stream) {
  if (k_pool == nullptr || v_pool == nullptr) {
    sa::set_error("sa_sink_dynamic_attn_fwd: k_pool and v_pool are required");
    return SA_EINVAL;
  }
  return launch_attention("sa_sink_dynamic_attn_fwd", q, k, v, q_strides, k_strides, v_strides,
                          B, H, Sq, Sk, D, block_mask, m_strides, Hm, head_mask_type, k_pool,
                          v_pool, kp_strides, vp_strides, Sk_pool, log_gap, softmax_scale, out,
                          o_strides, lse, status, stream);
}
