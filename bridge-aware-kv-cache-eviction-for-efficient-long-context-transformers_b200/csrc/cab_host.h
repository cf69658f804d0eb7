// Host-side helpers shared by the entry points: error reporting, argument checks,
// tensor-map encoding through the driver entry point, launch checks.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <string>

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "../../include/cab_capi.h"

namespace cab {

inline std::string& last_error() {
  static thread_local std::string err;
  return err;
}

inline int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  last_error() = buf;
  return code;
}

inline int ok() { return CAB_OK; }

inline int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(CAB_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
  return CAB_OK;
}

inline size_t dtype_size(int dtype) {
  switch (dtype) {
    case CAB_DTYPE_F32: return 4;
    case CAB_DTYPE_F16: return 2;
    case CAB_DTYPE_BF16: return 2;
    default: return 0;
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int current_sm_count() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

inline PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Encodes a tiled tensor map. dims/strides are innermost-first; strides exclude dim 0
// and are in bytes. Returns CAB_OK or an error code with the message set.
inline int make_tensor_map(CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base,
                           const uint64_t* dims, const uint64_t* strides_bytes,
                           const uint32_t* box, CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return fail(CAB_ERR_LAUNCH, "cuTensorMapEncodeTiled is not available from the driver");
  uint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, type, static_cast<cuuint32_t>(rank), const_cast<void*>(base),
                  reinterpret_cast<const cuuint64_t*>(dims),
                  reinterpret_cast<const cuuint64_t*>(strides_bytes),
                  reinterpret_cast<const cuuint32_t*>(box),
                  reinterpret_cast<const cuuint32_t*>(elem_strides),
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(CAB_ERR_INVALID_ARG, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return CAB_OK;
}

inline CUtensorMapDataType tma_type(int dtype) {
  switch (dtype) {
    case CAB_DTYPE_F32: return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    case CAB_DTYPE_F16: return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    default: return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  }
}

}  // namespace cab
