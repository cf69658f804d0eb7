// libcab_b200.so: single translation unit holding every kernel of the library and the
// utility entry points of cab_capi.h (version, errors, device checks, device status).

#include "cab_host.h"
#include "cab_ptx.cuh"

#include "coarsen.cu"
#include "frc.cu"
#include "topk.cu"
#include "sparse_attn.cu"
#include "noalloc.cu"
#include "prefill_host.cu"
#include "node_frc.cu"
#include "evict.cu"

extern "C" int cab_get_version(void) { return CAB_API_VERSION; }

extern "C" const char* cab_last_error_string(void) { return cab::last_error().c_str(); }

extern "C" int cab_device_supported(int device) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return (major == 10 && minor == 0) ? 1 : 0;
}

namespace cab {
// Failure-detection self-test: one thread waits on an mbarrier that nothing arrives at,
// with the bounded-wait pattern of every kernel in this library but a caller-chosen limit;
// when the limit runs out it records CAB_DEVICE_TIMEOUT and returns. Nothing faults, traps
// or hangs, and the context stays usable.
__global__ void wait_timeout_selftest_kernel(uint64_t limit_ns, int* gave_up) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_barrier_init();
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(&bar, 0)) {  // never completes: nothing arrives
      *gave_up = 0;
      return;
    }
    if ((i & 255u) == 0u && globaltimer_ns() - t0 > limit_ns) {
      atomicOr(&g_device_status, CAB_DEVICE_TIMEOUT);
      *gave_up = 1;
      return;
    }
  }
}
}  // namespace cab

extern "C" int cab_selftest_wait_timeout(int64_t limit_us, int* gave_up_device, void* stream) {
  if (!gave_up_device) return cab::fail(CAB_ERR_INVALID_ARG, "selftest: NULL output");
  if (limit_us <= 0 || limit_us > 10000000) return cab::fail(CAB_ERR_INVALID_ARG, "selftest: limit outside (0, 10 s]");
  cab::wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint64_t>(limit_us) * 1000ull, gave_up_device);
  return cab::check_launch("wait_timeout_selftest_kernel");
}

namespace cab {
// The status word is read and cleared in one atomic exchange on the device, so a bit that
// a kernel on another stream sets meanwhile is either returned now or kept for the next
// read, never lost between a read and a separate clear.
__device__ int g_status_taken = 0;
__global__ void status_take_kernel() { g_status_taken = atomicExch(&g_device_status, 0); }
}  // namespace cab

extern "C" int cab_device_status(void* stream, int* status) {
  if (!status) return cab::fail(CAB_ERR_INVALID_ARG, "device_status: NULL output");
  static std::mutex mu;  // one exchange-and-read at a time (g_status_taken is shared)
  std::lock_guard<std::mutex> lock(mu);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cab::fail(CAB_ERR_LAUNCH, "device_status: %s", cudaGetErrorString(e));
  cab::status_take_kernel<<<1, 1, 0, st>>>();
  if (int rc = cab::check_launch("status_take_kernel")) return rc;
  int value = 0;
  e = cudaMemcpyFromSymbolAsync(&value, cab::g_status_taken, sizeof(int), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cab::fail(CAB_ERR_LAUNCH, "device_status: %s", cudaGetErrorString(e));
  *status = (value & cab::CAB_DEVICE_TIMEOUT) ? CAB_ERR_TIMEOUT
           : (value & cab::CAB_DEVICE_LAYOUT) ? CAB_ERR_LAUNCH
                                               : CAB_OK;
  return CAB_OK;
}
