// cab_sparse_attn_fwd_noalloc: block-sparse attention for callers that cannot allocate
// device memory.
//
// Some hosts of this library cannot call cudaMalloc themselves: a serving engine or
// framework whose caching allocator owns all device memory and forbids side allocations,
// a language binding (cgo, JNI, ctypes) that links no CUDA allocator, or a caller with a
// fixed device-memory budget decided at start-up. cab_sparse_attn_fwd asks such callers
// for a workspace (the merged key-block lists of each pair of query blocks); this entry
// point instead uses a scratch buffer that lives inside the library itself.
//
// The scratch is a file-scope static __device__ array of kScratchBytes (16 MiB). Every GPU
// that loads the library's device code holds those 16 MiB until the process exits.
// Host code cannot use the array's name as a device address (on the host it names a
// stand-in object), so the first call on each device, with that device current, resolves
// the real address with cudaGetSymbolAddress and caches it; make that first call before
// any stream capture. Calls share the one buffer: two calls whose kernels overlap on the
// GPU (different streams, or concurrent host threads) race on it. Each call rewrites every
// scratch location it later reads, so nothing has to be cleared between calls.
//
// Sizes whose scratch need exceeds kScratchBytes are rejected with CAB_ERR_UNSUPPORTED;
// the need is cab_sparse_attn_workspace_size() (about 4 * B * Hq * ceil(M/2) *
// (2 * kmax + 3) bytes; 13 MB for B2 H8 N128000 kmax 100). No allocation happens here:
// the call resolves the address (first call per device) and forwards to
// cab_sparse_attn_fwd with the static buffer as its workspace.

#include "cab_host.h"

#include <mutex>

namespace cab {
namespace noalloc {

constexpr size_t kScratchBytes = static_cast<size_t>(16) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_attn_scratch[kScratchBytes];

static std::mutex g_mu;
static void* g_addr[kMaxDevices] = {};

static int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(CAB_ERR_LAUNCH, "attn_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(CAB_ERR_UNSUPPORTED, "attn_noalloc: device %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);
    if (e != cudaSuccess || !p)
      return fail(CAB_ERR_LAUNCH, "attn_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return CAB_OK;
}

}  // namespace noalloc
}  // namespace cab

extern "C" int cab_sparse_attn_fwd_noalloc(const void* q, const void* k, const void* v,
                                           const int32_t* kv_idx, const int32_t* kv_num, void* out,
                                           float* lse, int64_t B, int64_t Hq, int64_t Hkv, int64_t N,
                                           int64_t D, int64_t block_size, int64_t kmax,
                                           const int64_t* q_strides, const int64_t* k_strides,
                                           const int64_t* v_strides, const int64_t* o_strides,
                                           float softmax_scale, int causal, int dtype, void* stream) {
  using namespace cab;
  size_t need = 0;
  if (int rc = cab_sparse_attn_workspace_size(B, Hq, N, D, block_size, kmax, dtype, &need)) return rc;
  if (need > noalloc::kScratchBytes)
    return fail(CAB_ERR_UNSUPPORTED,
                "attn_noalloc: these sizes need %zu bytes of scratch; the library's static buffer "
                "holds %zu (16 MiB). Use cab_sparse_attn_fwd with a caller workspace.",
                need, noalloc::kScratchBytes);
  void* ws = nullptr;
  if (need > 0) {
    if (int rc = noalloc::scratch_address(&ws)) return rc;
  }
  return cab_sparse_attn_fwd(q, k, v, kv_idx, kv_num, out, lse, B, Hq, Hkv, N, D, block_size, kmax,
                             q_strides, k_strides, v_strides, o_strides, softmax_scale, causal, dtype,
                             ws, need, stream);
}
