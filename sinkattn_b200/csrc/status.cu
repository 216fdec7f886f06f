// status.cu — the device status word that kernels write when a bounded wait
// gives up, kept in mapped page-locked host memory so that the host reads it
// at any time without synchronising; and a kernel whose only job is to let a
// bounded wait run out, so that failure detection can be tested without any
// GPU fault.

#include "sa_common.cuh"

namespace sa {
namespace status {

// One warp: an mbarrier that expects one arrival gets none, and the warp
// waits on it with the given limit. The wait gives up, records
// SA_DEV_WAIT_TIMEOUT in *status, and the kernel returns. Nothing else is in
// flight (no copy, no MMA), so the kernel leaves no work behind.
__global__ void unanswered_wait_kernel(int32_t* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncwarp();
  mbar_wait(&bar, 0u, status, nullptr, limit_ns);
}

}  // namespace status
}  // namespace sa

extern "C" int32_t* sa_status_create(void) {
  void* p = nullptr;
  const cudaError_t e = cudaHostAlloc(&p, sizeof(int32_t), cudaHostAllocMapped |
                                                              cudaHostAllocPortable);
  if (e != cudaSuccess) {
    sa::cuda_fail(e, "cudaHostAlloc (status word)");
    return nullptr;
  }
  *reinterpret_cast<volatile int32_t*>(p) = SA_DEV_OK;
  return reinterpret_cast<int32_t*>(p);
}

extern "C" int sa_status_device_pointer(int32_t* status, int32_t** device_ptr) {
  SA_CHECK_ARG(status && device_ptr, "sa_status_device_pointer: null pointer argument");
  void* d = nullptr;
  SA_CUDA_TRY(cudaHostGetDevicePointer(&d, status, 0));
  *device_ptr = reinterpret_cast<int32_t*>(d);
  return SA_OK;
}

extern "C" int sa_status_destroy(int32_t* status) {
  if (status == nullptr) return SA_OK;
  SA_CUDA_TRY(cudaFreeHost(status));
  return SA_OK;
}

extern "C" int sa_check_status(int32_t* status) {
  SA_CHECK_ARG(status, "sa_check_status: null pointer argument");
  const int32_t v = *reinterpret_cast<volatile int32_t*>(status);
  if (v == SA_DEV_OK) return SA_OK;
  *reinterpret_cast<volatile int32_t*>(status) = SA_DEV_OK;
  sa::set_error(
      "a bounded wait in a kernel gave up (device status %d): the outputs of the launches "
      "that shared this status word since the last check are not valid",
      (int)v);
  return SA_ETIMEOUT;
}

extern "C" int sa_selftest_wait_timeout(int32_t* status, uint64_t limit_ns, cudaStream_t stream) {
  SA_CHECK_ARG(status, "sa_selftest_wait_timeout: null status");
  SA_CHECK_ARG(limit_ns >= 1000ull && limit_ns <= 1000000000ull,
               "sa_selftest_wait_timeout: limit must be in [1 us, 1 s], got %llu ns",
               (unsigned long long)limit_ns);
  sa::status::unanswered_wait_kernel<<<1, 32, 0, stream>>>(status, limit_ns);
  SA_CUDA_TRY(cudaGetLastError());
  return SA_OK;
}
