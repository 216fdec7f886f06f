// exchange.cu — the Ulysses sequence-parallel exchange over NVLink peer
// memory, and the CUDA IPC helpers that give each rank its peers' buffers.
//
// In a sequence-parallel DiT every rank holds a [B, S/P, H, D] shard of Q, K
// and V; attention needs whole sequences. The (batch, head) pairs ("units")
// are split over the ranks, n_per each, and:
//   dispatch: every rank writes each row of its shard straight into the
//     receive buffer of the unit's owner, at the row's place in the whole
//     sequence. The receive buffer is [T][n_per][S][D], so each unit's
//     sequence is contiguous and the attention kernel reads it as it lies.
//   combine: every rank writes the output rows and LSE of its units straight
//     into the [B, S/P, H, D] output and [B, H, S/P] LSE of the rank that owns
//     that stretch of the sequence.
// One pass over the data each way, with 16-byte loads and 16-byte stores
// (NVLink for remote rows, HBM for the rank's own), and no pack or unpack
// copies. The kernels do not wait on other ranks: the caller orders them
// against the peers' use of the same buffers with stream-ordered
// collectives (sinkattn_b200/sharding.py). Every thread ends with a
// system-scope fence, so its remote stores are performed before the kernel
// completes.

#include <string.h>

#include "sa_common.cuh"

namespace sa {
namespace xchg {

constexpr int kD = 128;
constexpr int kMaxRanks = 8;
constexpr int kMaxTensors = 3;
constexpr int kRowBytes = kD * 2;     // one bf16 row
constexpr int kPieces = kRowBytes / 16;  // 16-byte pieces of one row

// One piece of a row: 32 bytes moved with one 256-bit load and store where
// every address allows it (half the stores, over NVLink included), else 16.
template <int kBytes>
struct Piece;
template <>
struct Piece<16> {
  uint4 v;
  __device__ __forceinline__ void load(const uint8_t* a) { v = *reinterpret_cast<const uint4*>(a); }
  __device__ __forceinline__ void store(uint8_t* a) const { *reinterpret_cast<uint4*>(a) = v; }
};
template <>
struct Piece<32> {
  uint32_t r[8];
  __device__ __forceinline__ void load(const uint8_t* a) {
    asm volatile("ld.global.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "l"(a));
  }
  __device__ __forceinline__ void store(uint8_t* a) const {
    asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(a), "r"(r[0]),
                 "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
  }
};

struct DispatchParams {
  const uint8_t* src[kMaxTensors];
  int64_t st[kMaxTensors][3];  // element strides of b, s, h (d is unit stride)
  uint8_t* dst[kMaxRanks];     // each rank's receive buffer [T][n_per][S][D]
  int T, B, Sr, H, P, rank, n_per;
  int j0, nj;                  // the owners' unit slots j0 .. j0 + nj - 1
};

// 128-thread CTAs at no more than 32 registers a thread: one fits on an SM
// beside a persistent attention CTA (512 threads, up to 120 registers), so the
// exchange of one group of units can run while attention works on another.
constexpr int kXThreads = 128;
constexpr int kXMinBlocks = 16;

// Thread i moves piece (i mod n) of row i / n, n = 256 / kBytes; rows are
// ordered (t, slot, s, owner) with the owner fastest, so that every stretch
// of the grid-stride loop stores to every owner (NVLink and local HBM at
// once), and each warp moves whole 256-byte rows.
template <int kBytes>
__global__ void __launch_bounds__(kXThreads, kXMinBlocks) dispatch_kernel(const DispatchParams p) {
  constexpr int kN = kRowBytes / kBytes;
  const int U = p.B * p.H;
  const int64_t S = (int64_t)p.P * p.Sr;
  const uint32_t rows = (uint32_t)p.T * p.P * p.nj * p.Sr;
  const uint32_t n = rows * kN;
  for (uint32_t i = blockIdx.x * kXThreads + threadIdx.x; i < n; i += gridDim.x * kXThreads) {
    const int piece = (int)(i & (kN - 1));
    uint32_t r = i / kN;
    const int owner = (int)(r % (uint32_t)p.P);
    r /= (uint32_t)p.P;
    const int s = (int)(r % (uint32_t)p.Sr);
    r /= (uint32_t)p.Sr;
    const int j = p.j0 + (int)(r % (uint32_t)p.nj);
    const int t = (int)(r / (uint32_t)p.nj);
    const int u = owner * p.n_per + j;
    if (u >= U) continue;  // a padding unit
    const int b = u / p.H, h = u - b * p.H;
    Piece<kBytes> v;
    v.load(p.src[t] + ((b * p.st[t][0] + s * p.st[t][1] + h * p.st[t][2]) * 2 + piece * kBytes));
    v.store(p.dst[owner] + ((((int64_t)t * p.n_per + j) * S + (int64_t)p.rank * p.Sr + s) *
                                kRowBytes +
                            piece * kBytes));
  }
  __threadfence_system();
}

struct CombineParams {
  const uint8_t* out;    // [n_per][S][D] bf16, this rank's units
  const float* lse;      // [n_per][S] fp32
  uint8_t* out_dst[kMaxRanks];  // each rank's [B][Sr][H][D] bf16
  float* lse_dst[kMaxRanks];    // each rank's [B][H][Sr] fp32 (nullable as a whole)
  int B, Sr, H, P, rank, n_per;
  int j0, nj;                   // this rank's unit slots j0 .. j0 + nj - 1
  int lse_w;                    // LSE values per store: 4 (16 bytes) when Sr % 4 == 0, else 1
};

// Threads i < n_out move 16-byte piece (i mod 16) of output row i / 16; rows
// are (slot, s mod Sr, s div Sr) with the receiving rank s div Sr fastest, so
// that every stretch of the loop stores to every rank. The threads after them
// move the LSE, lse_w consecutive rows of one rank per store (a 4-byte store
// per row would be one NVLink write of 4 bytes).
template <int kBytes>
__global__ void __launch_bounds__(kXThreads, kXMinBlocks) combine_kernel(const CombineParams p) {
  constexpr int kN = kRowBytes / kBytes;
  const int U = p.B * p.H;
  const uint32_t S = (uint32_t)p.P * p.Sr;
  const uint32_t n_out = (uint32_t)p.nj * S * kN;
  const uint32_t n_lse = p.lse_dst[0] != nullptr ? (uint32_t)p.nj * S / (uint32_t)p.lse_w : 0u;
  for (uint32_t i = blockIdx.x * kXThreads + threadIdx.x; i < n_out + n_lse;
       i += gridDim.x * kXThreads) {
    const bool is_out = i < n_out;
    const uint32_t w = is_out ? 1u : (uint32_t)p.lse_w;
    uint32_t rr = is_out ? i / kN : (i - n_out);  // output row, or LSE group
    const int piece = is_out ? (int)(i & (kN - 1)) : 0;
    const int owner = (int)(rr % (uint32_t)p.P);
    rr /= (uint32_t)p.P;
    const uint32_t per_owner = (uint32_t)p.Sr / w;  // rows (or LSE groups) per rank
    const int sl = (int)((rr % per_owner) * w);
    const int j = p.j0 + (int)(rr / per_owner);
    const int u = p.rank * p.n_per + j;
    if (u >= U) continue;  // a padding unit
    const int b = u / p.H, h = u - b * p.H;
    const int64_t row = (int64_t)j * S + (int64_t)owner * p.Sr + sl;
    if (is_out) {
      Piece<kBytes> v;
      v.load(p.out + (row * kRowBytes + piece * kBytes));
      v.store(p.out_dst[owner] +
              ((((int64_t)b * p.Sr + sl) * p.H + h) * kRowBytes + piece * kBytes));
    } else {
      float* to = p.lse_dst[owner] + ((int64_t)b * p.H + h) * p.Sr + sl;
      if (w == 4u)
        *reinterpret_cast<float4*>(to) = *reinterpret_cast<const float4*>(p.lse + row);
      else
        *to = p.lse[row];
    }
  }
  __threadfence_system();
}

int grid_for(int64_t work) {
  const int64_t want = (work + kXThreads - 1) / kXThreads;
  const int64_t cap = (int64_t)sm_count_current_device() * kXMinBlocks;
  return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

}  // namespace xchg
}  // namespace sa

using sa::xchg::kD;
using sa::xchg::kMaxRanks;
using sa::xchg::kMaxTensors;

extern "C" int sa_ipc_alloc(size_t bytes, void** ptr) {
  SA_CHECK_ARG(ptr != nullptr && bytes > 0, "sa_ipc_alloc: null pointer or zero size");
  *ptr = nullptr;
  SA_CUDA_TRY(cudaMalloc(ptr, bytes));
  return SA_OK;
}

extern "C" int sa_ipc_free(void* ptr) {
  if (ptr == nullptr) return SA_OK;
  SA_CUDA_TRY(cudaFree(ptr));
  return SA_OK;
}

extern "C" int sa_ipc_get_handle(void* ptr, uint8_t handle[64]) {
  SA_CHECK_ARG(ptr != nullptr && handle != nullptr, "sa_ipc_get_handle: null pointer argument");
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  cudaIpcMemHandle_t h;
  SA_CUDA_TRY(cudaIpcGetMemHandle(&h, ptr));
  memcpy(handle, &h, 64);
  return SA_OK;
}

extern "C" int sa_ipc_open_handle(const uint8_t handle[64], void** ptr) {
  SA_CHECK_ARG(ptr != nullptr && handle != nullptr, "sa_ipc_open_handle: null pointer argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, 64);
  *ptr = nullptr;
  SA_CUDA_TRY(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return SA_OK;
}

extern "C" int sa_ipc_close(void* ptr) {
  if (ptr == nullptr) return SA_OK;
  SA_CUDA_TRY(cudaIpcCloseMemHandle(ptr));
  return SA_OK;
}

extern "C" int sa_ulysses_dispatch_units(int T, const void* const* src,
                                         const int64_t* src_strides, int B, int Sr, int H, int D,
                                         int P, int rank, int n_per, int j0, int j1,
                                         void* const* dst, cudaStream_t stream) {
  SA_CHECK_ARG(src != nullptr && src_strides != nullptr && dst != nullptr,
               "sa_ulysses_dispatch: null pointer argument");
  SA_CHECK_ARG(T >= 1 && T <= kMaxTensors, "sa_ulysses_dispatch: 1 to %d tensors, got %d",
               kMaxTensors, T);
  SA_CHECK_ARG(D == kD, "sa_ulysses_dispatch: head dim must be 128, got %d", D);
  SA_CHECK_ARG(P >= 1 && P <= kMaxRanks, "sa_ulysses_dispatch: 1 to %d ranks, got %d",
               kMaxRanks, P);
  SA_CHECK_ARG(rank >= 0 && rank < P, "sa_ulysses_dispatch: rank %d outside 0..%d", rank, P - 1);
  SA_CHECK_ARG(B >= 1 && Sr >= 1 && H >= 1, "sa_ulysses_dispatch: empty shard");
  SA_CHECK_ARG(n_per >= 1 && (int64_t)n_per * P >= (int64_t)B * H,
               "sa_ulysses_dispatch: %d units per rank cannot hold %d units", n_per, B * H);
  SA_CHECK_ARG(0 <= j0 && j0 < j1 && j1 <= n_per,
               "sa_ulysses_dispatch: unit slots [%d, %d) not a non-empty range of 0..%d", j0, j1,
               n_per);
  SA_CHECK_ARG((int64_t)T * P * (j1 - j0) * Sr * sa::xchg::kPieces < ((int64_t)1 << 32),
               "sa_ulysses_dispatch: too many rows in one call");
  sa::xchg::DispatchParams p = {};
  for (int t = 0; t < T; ++t) {
    SA_CHECK_ARG(src[t] != nullptr && ((uintptr_t)src[t] % 16) == 0,
                 "sa_ulysses_dispatch: tensor %d null or not 16-byte aligned", t);
    const int64_t* st = src_strides + 4 * t;  // [B, S, H, D] element strides
    SA_CHECK_ARG(st[3] == 1 && st[0] % 8 == 0 && st[1] % 8 == 0 && st[2] % 8 == 0,
                 "sa_ulysses_dispatch: tensor %d needs stride(dim) 1 and strides multiple "
                 "of 8 elements", t);
    p.src[t] = reinterpret_cast<const uint8_t*>(src[t]);
    p.st[t][0] = st[0];
    p.st[t][1] = st[1];
    p.st[t][2] = st[2];
  }
  for (int r = 0; r < P; ++r) {
    SA_CHECK_ARG(dst[r] != nullptr && ((uintptr_t)dst[r] % 16) == 0,
                 "sa_ulysses_dispatch: receive buffer of rank %d null or not 16-byte aligned", r);
    p.dst[r] = reinterpret_cast<uint8_t*>(dst[r]);
  }
  p.T = T;
  p.B = B;
  p.Sr = Sr;
  p.H = H;
  p.P = P;
  p.rank = rank;
  p.n_per = n_per;
  p.j0 = j0;
  p.nj = j1 - j0;
  bool wide = true;  // every row and destination 32-byte aligned
  for (int t = 0; t < T; ++t)
    wide = wide && ((uintptr_t)src[t] % 32) == 0 && p.st[t][0] % 16 == 0 &&
           p.st[t][1] % 16 == 0 && p.st[t][2] % 16 == 0;
  for (int r = 0; r < P; ++r) wide = wide && ((uintptr_t)dst[r] % 32) == 0;
  const int64_t rows = (int64_t)T * P * p.nj * Sr;
  if (wide)
    sa::xchg::dispatch_kernel<32><<<sa::xchg::grid_for(rows * (sa::xchg::kRowBytes / 32)),
                                    sa::xchg::kXThreads, 0, stream>>>(p);
  else
    sa::xchg::dispatch_kernel<16><<<sa::xchg::grid_for(rows * (sa::xchg::kRowBytes / 16)),
                                    sa::xchg::kXThreads, 0, stream>>>(p);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_ulysses_dispatch(int T, const void* const* src, const int64_t* src_strides,
                                   int B, int Sr, int H, int D, int P, int rank, int n_per,
                                   void* const* dst, cudaStream_t stream) {
  return sa_ulysses_dispatch_units(T, src, src_strides, B, Sr, H, D, P, rank, n_per, 0,
                                   n_per > 0 ? n_per : 1, dst, stream);
}

extern "C" int sa_ulysses_combine_units(const void* out_units, const float* lse_units, int B,
                                        int Sr, int H, int D, int P, int rank, int n_per, int j0,
                                        int j1, void* const* out_dst, float* const* lse_dst,
                                        cudaStream_t stream) {
  SA_CHECK_ARG(out_units != nullptr && out_dst != nullptr,
               "sa_ulysses_combine: null pointer argument");
  SA_CHECK_ARG((lse_units == nullptr) == (lse_dst == nullptr),
               "sa_ulysses_combine: lse_units and lse_dst go together");
  SA_CHECK_ARG(D == kD, "sa_ulysses_combine: head dim must be 128, got %d", D);
  SA_CHECK_ARG(P >= 1 && P <= kMaxRanks, "sa_ulysses_combine: 1 to %d ranks, got %d",
               kMaxRanks, P);
  SA_CHECK_ARG(rank >= 0 && rank < P, "sa_ulysses_combine: rank %d outside 0..%d", rank, P - 1);
  SA_CHECK_ARG(B >= 1 && Sr >= 1 && H >= 1, "sa_ulysses_combine: empty shard");
  SA_CHECK_ARG(n_per >= 1 && (int64_t)n_per * P >= (int64_t)B * H,
               "sa_ulysses_combine: %d units per rank cannot hold %d units", n_per, B * H);
  SA_CHECK_ARG(0 <= j0 && j0 < j1 && j1 <= n_per,
               "sa_ulysses_combine: unit slots [%d, %d) not a non-empty range of 0..%d", j0, j1,
               n_per);
  SA_CHECK_ARG((int64_t)(j1 - j0) * P * Sr * (sa::xchg::kPieces + 1) < ((int64_t)1 << 32),
               "sa_ulysses_combine: too many rows in one call");
  SA_CHECK_ARG(((uintptr_t)lse_units % 16) == 0,
               "sa_ulysses_combine: lse_units not 16-byte aligned");
  SA_CHECK_ARG(((uintptr_t)out_units % 16) == 0, "sa_ulysses_combine: out_units not 16-byte aligned");
  sa::xchg::CombineParams p = {};
  p.out = reinterpret_cast<const uint8_t*>(out_units);
  p.lse = lse_units;
  for (int r = 0; r < P; ++r) {
    SA_CHECK_ARG(out_dst[r] != nullptr && ((uintptr_t)out_dst[r] % 16) == 0,
                 "sa_ulysses_combine: output of rank %d null or not 16-byte aligned", r);
    p.out_dst[r] = reinterpret_cast<uint8_t*>(out_dst[r]);
    if (lse_dst != nullptr) {
      SA_CHECK_ARG(lse_dst[r] != nullptr && ((uintptr_t)lse_dst[r] % 16) == 0,
                   "sa_ulysses_combine: LSE of rank %d null or not 16-byte aligned", r);
      p.lse_dst[r] = lse_dst[r];
    }
  }
  p.B = B;
  p.Sr = Sr;
  p.H = H;
  p.P = P;
  p.rank = rank;
  p.n_per = n_per;
  p.j0 = j0;
  p.nj = j1 - j0;
  p.lse_w = Sr % 4 == 0 ? 4 : 1;
  bool wide = ((uintptr_t)out_units % 32) == 0;
  for (int r = 0; r < P; ++r) wide = wide && ((uintptr_t)out_dst[r] % 32) == 0;
  const int64_t rows = (int64_t)p.nj * P * Sr;
  const int64_t lse_work = lse_dst != nullptr ? rows / p.lse_w : 0;
  if (wide)
    sa::xchg::combine_kernel<32><<<sa::xchg::grid_for(rows * (sa::xchg::kRowBytes / 32) +
                                                      lse_work),
                                   sa::xchg::kXThreads, 0, stream>>>(p);
  else
    sa::xchg::combine_kernel<16><<<sa::xchg::grid_for(rows * (sa::xchg::kRowBytes / 16) +
                                                      lse_work),
                                   sa::xchg::kXThreads, 0, stream>>>(p);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}

extern "C" int sa_ulysses_combine(const void* out_units, const float* lse_units, int B, int Sr,
                                  int H, int D, int P, int rank, int n_per,
                                  void* const* out_dst, float* const* lse_dst,
                                  cudaStream_t stream) {
  return sa_ulysses_combine_units(out_units, lse_units, B, Sr, H, D, P, rank, n_per, 0,
                                  n_per > 0 ? n_per : 1, out_dst, lse_dst, stream);
}
