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

extern "C" int cab_device_status(void* stream, int* status) {
  if (!status) return cab::fail(CAB_ERR_INVALID_ARG, "device_status: NULL output");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return cab::fail(CAB_ERR_LAUNCH, "device_status: %s", cudaGetErrorString(e));
  int value = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&value, cab::g_device_status, sizeof(int));
  if (e == cudaSuccess) e = cudaMemcpyToSymbol(cab::g_device_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cab::fail(CAB_ERR_LAUNCH, "device_status: %s", cudaGetErrorString(e));
  *status = (value & cab::CAB_DEVICE_TIMEOUT) ? CAB_ERR_TIMEOUT
           : (value & cab::CAB_DEVICE_LAYOUT) ? CAB_ERR_LAUNCH
                                               : CAB_OK;
  return CAB_OK;
}
