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
// stand-in object), so the first call in each CUDA context, with that context current,
// resolves the real address with cudaGetSymbolAddress and caches it against the context's
// unique ID; make that first call before any stream capture. A new context on the device
// (after cudaDeviceReset, or a driver-API context made current) holds its own copy of the
// array, so its first call resolves the address again. Calls share the one buffer: two
// calls whose kernels overlap on the GPU (different streams, or concurrent host threads)
// race on it. Each call rewrites every scratch location it later reads, so nothing has to
// be cleared between calls.
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
struct CachedAddress {
  unsigned long long ctx_id;  // context the address belongs to (0 = none yet)
  void* addr;
};
static CachedAddress g_addr[kMaxDevices] = {};

// Unique ID of the calling thread's current context (0 if none is current or the driver
// entry points are missing). cuCtxGetId (CUDA 12) never repeats within a process, unlike a
// context handle, whose address a later context may reuse.
static unsigned long long current_context_id() {
  static PFN_cuCtxGetCurrent_v4000 get_current = nullptr;
  static PFN_cuCtxGetId_v12000 get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PFN_cuCtxGetId_v12000>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
  if (get_id && get_id(ctx, &id) == CUDA_SUCCESS) return id;
  return reinterpret_cast<unsigned long long>(ctx);
}

static int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(CAB_ERR_LAUNCH, "attn_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(CAB_ERR_UNSUPPORTED, "attn_noalloc: device %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_mu);
  const unsigned long long ctx = current_context_id();
  if (ctx == 0 || g_addr[dev].ctx_id != ctx || !g_addr[dev].addr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attn_scratch);  // makes the device's context current if none is
    if (e != cudaSuccess || !p)
      return fail(CAB_ERR_LAUNCH, "attn_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_addr[dev].ctx_id = current_context_id();
    g_addr[dev].addr = p;
  }
  *out = g_addr[dev].addr;
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
