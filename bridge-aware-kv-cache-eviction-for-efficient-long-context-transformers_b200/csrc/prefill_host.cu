// Host-buffer prefill: the whole path (coarsen -> FRC -> top-k -> block-sparse attention)
// for inputs and outputs held in page-locked host memory, streamed through the GPU one
// (batch, KV head) unit at a time.
//
// Every unit is independent through the whole path (a KV head and the G = Hq / Hkv query
// heads that read it), so the units form a three-stage pipeline over two device slots:
//
//   copy-in stream  : H2D q/k/v of unit u into slot u % 2 (after unit u-2's compute)
//   caller's stream : the four entry points on slot u % 2 (after its copy-in, and after
//                     unit u-2's copy-out released the slot's output buffers)
//   copy-out stream : D2H out (and the block lists) of unit u (after its compute)
//
// H2D and D2H use the two PCIe directions at once and the compute of unit u hides under
// the copy-in of unit u+1, so a layer costs about max(H2D bytes, D2H bytes) / PCIe
// bandwidth plus one unit of compute, instead of the sum of all three.
// No counterpart in the reference: its callers move whole tensors between host and device
// around the layer (`.to(device)` / `.cpu()`, e.g. examples/demo_cab_attention.py:82,142).

#include "cab_host.h"

#include <map>

namespace cab {
namespace prefill {

constexpr int kSlots = 2;

struct SlotLayout {
  size_t q, k, v, out, qc, kc, frc, idx, num, frc_ws, attn_ws;
  size_t frc_ws_bytes, attn_ws_bytes, total;
};

inline size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Device buffers of one slot (one unit: G query heads and one KV head).
inline int slot_layout(int64_t G, int64_t N, int64_t D, int64_t bs, int64_t keep, int dtype,
                       int normalization, SlotLayout* L) {
  const size_t es = dtype_size(dtype);
  const int64_t M = (N + bs - 1) / bs;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align256(off + bytes);
    return o;
  };
  L->q = take(static_cast<size_t>(G * N * D) * es);
  L->k = take(static_cast<size_t>(N * D) * es);
  L->v = take(static_cast<size_t>(N * D) * es);
  L->out = take(static_cast<size_t>(G * N * D) * es);
  L->qc = take(static_cast<size_t>(G * M * D) * es);
  L->kc = take(static_cast<size_t>(M * D) * es);
  L->frc = take(static_cast<size_t>(G * M * M) * 4);
  L->idx = take(static_cast<size_t>(G * M * keep) * 4);
  L->num = take(static_cast<size_t>(G * M) * 4);
  size_t fb = 0, ab = 0;
  int rc = cab_frc_workspace_size(1, G, M, D, dtype, normalization, &fb);
  if (rc != CAB_OK) return rc;
  rc = cab_sparse_attn_workspace_size(1, G, N, D, bs, keep, dtype, &ab);
  if (rc != CAB_OK) return rc;
  L->frc_ws = take(fb);
  L->frc_ws_bytes = fb;
  L->attn_ws = take(ab);
  L->attn_ws_bytes = ab;
  L->total = off;
  return CAB_OK;
}

// The copy-in and copy-out streams of the current device, created on first use and kept
// for the life of the process (non-blocking, so they never serialise with the legacy
// default stream; every ordering is an explicit event).
struct CopyStreams {
  cudaStream_t h2d = nullptr;
  cudaStream_t d2h = nullptr;
};

inline int copy_streams(CopyStreams* out) {
  static std::mutex mu;
  static std::map<int, CopyStreams> per_device;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    cudaGetLastError();
    return fail(CAB_ERR_LAUNCH, "prefill_host: no current CUDA device");
  }
  std::lock_guard<std::mutex> guard(mu);
  auto it = per_device.find(dev);
  if (it == per_device.end()) {
    CopyStreams s;
    if (cudaStreamCreateWithFlags(&s.h2d, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&s.d2h, cudaStreamNonBlocking) != cudaSuccess) {
      cudaGetLastError();
      return fail(CAB_ERR_LAUNCH, "prefill_host: cannot create the copy streams");
    }
    it = per_device.emplace(dev, s).first;
  }
  *out = it->second;
  return CAB_OK;
}

// True if [p, p + bytes) lies in page-locked host memory known to CUDA.
inline bool page_locked(const void* p, size_t bytes) {
  for (const char* a : {static_cast<const char*>(p), static_cast<const char*>(p) + bytes - 1}) {
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, a) != cudaSuccess) {
      cudaGetLastError();
      return false;
    }
    if (attr.type != cudaMemoryTypeHost) return false;
  }
  return true;
}

// Events of one call: per slot, copy-in done / compute done / copy-out done; plus the
// call's start and the two copy streams' ends. Destroyed at the end of the call (CUDA
// releases an event's resources once its pending work completes).
struct Events {
  cudaEvent_t in_done[kSlots] = {}, comp_done[kSlots] = {}, out_done[kSlots] = {};
  cudaEvent_t start = nullptr, h2d_end = nullptr, d2h_end = nullptr;
  bool ok = true;
  Events() {
    for (int s = 0; s < kSlots; ++s) {
      ok &= cudaEventCreateWithFlags(&in_done[s], cudaEventDisableTiming) == cudaSuccess;
      ok &= cudaEventCreateWithFlags(&comp_done[s], cudaEventDisableTiming) == cudaSuccess;
      ok &= cudaEventCreateWithFlags(&out_done[s], cudaEventDisableTiming) == cudaSuccess;
    }
    ok &= cudaEventCreateWithFlags(&start, cudaEventDisableTiming) == cudaSuccess;
    ok &= cudaEventCreateWithFlags(&h2d_end, cudaEventDisableTiming) == cudaSuccess;
    ok &= cudaEventCreateWithFlags(&d2h_end, cudaEventDisableTiming) == cudaSuccess;
    if (!ok) cudaGetLastError();
  }
  ~Events() {
    for (int s = 0; s < kSlots; ++s) {
      if (in_done[s]) cudaEventDestroy(in_done[s]);
      if (comp_done[s]) cudaEventDestroy(comp_done[s]);
      if (out_done[s]) cudaEventDestroy(out_done[s]);
    }
    if (start) cudaEventDestroy(start);
    if (h2d_end) cudaEventDestroy(h2d_end);
    if (d2h_end) cudaEventDestroy(d2h_end);
  }
};

}  // namespace prefill
}  // namespace cab

using namespace cab;

static int prefill_check_sizes(int64_t B, int64_t Hq, int64_t Hkv, int64_t N, int64_t D,
                               int64_t block_size, int64_t keep, int dtype) {
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || N <= 0 || D <= 0 || block_size <= 0)
    return fail(CAB_ERR_INVALID_ARG, "prefill_host: non-positive size");
  if (Hq % Hkv != 0) return fail(CAB_ERR_INVALID_ARG, "prefill_host: Hq %% Hkv != 0");
  const int64_t M = (N + block_size - 1) / block_size;
  if (keep < 1 || keep > M)
    return fail(CAB_ERR_INVALID_ARG, "prefill_host: keep=%lld outside [1, M=%lld]", (long long)keep, (long long)M);
  if (!dtype_size(dtype)) return fail(CAB_ERR_UNSUPPORTED, "prefill_host: unknown dtype %d", dtype);
  return CAB_OK;
}

extern "C" int cab_prefill_host_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t N,
                                               int64_t D, int64_t block_size, int64_t keep,
                                               int dtype, int normalization, size_t* bytes) {
  if (!bytes) return fail(CAB_ERR_INVALID_ARG, "prefill_host_workspace_size: NULL output");
  int rc = prefill_check_sizes(B, Hq, Hkv, N, D, block_size, keep, dtype);
  if (rc != CAB_OK) return rc;
  prefill::SlotLayout L;
  rc = prefill::slot_layout(Hq / Hkv, N, D, block_size, keep, dtype, normalization, &L);
  if (rc != CAB_OK) return rc;
  *bytes = prefill::kSlots * L.total;
  return CAB_OK;
}

extern "C" int cab_prefill_host(const void* q, const void* k, const void* v, void* out,
                                int32_t* kv_idx, int32_t* kv_num, int64_t B, int64_t Hq,
                                int64_t Hkv, int64_t N, int64_t D, int64_t block_size,
                                int64_t keep, float temperature, float lambda_redundancy,
                                int normalization, int formula, int redundancy_scale,
                                int select_high, int keep_diagonal, int causal,
                                float softmax_scale, int dtype, void* workspace,
                                size_t workspace_bytes, void* stream) {
  using namespace prefill;
  if (!q || !k || !v || !out) return fail(CAB_ERR_INVALID_ARG, "prefill_host: NULL pointer");
  int rc = prefill_check_sizes(B, Hq, Hkv, N, D, block_size, keep, dtype);
  if (rc != CAB_OK) return rc;
  if (!(softmax_scale > 0.f)) return fail(CAB_ERR_INVALID_ARG, "prefill_host: softmax_scale must be > 0");
  const int64_t G = Hq / Hkv;
  const int64_t M = (N + block_size - 1) / block_size;
  const size_t es = dtype_size(dtype);
  const size_t q_unit = static_cast<size_t>(G * N * D) * es;  // q / out bytes per unit
  const size_t k_unit = static_cast<size_t>(N * D) * es;      // k / v bytes per unit
  const size_t idx_unit = static_cast<size_t>(G * M * keep) * 4;
  const size_t num_unit = static_cast<size_t>(G * M) * 4;
  const int64_t U = B * Hkv;
  if (!page_locked(q, U * q_unit) || !page_locked(k, U * k_unit) || !page_locked(v, U * k_unit) ||
      !page_locked(out, U * q_unit) || (kv_idx && !page_locked(kv_idx, U * idx_unit)) ||
      (kv_num && !page_locked(kv_num, U * num_unit)))
    return fail(CAB_ERR_INVALID_ARG,
                "prefill_host: q, k, v, out (and kv_idx / kv_num if given) must be page-locked "
                "host memory (cudaHostAlloc / cudaHostRegister)");
  SlotLayout L;
  rc = slot_layout(G, N, D, block_size, keep, dtype, normalization, &L);
  if (rc != CAB_OK) return rc;
  if (!workspace || workspace_bytes < kSlots * L.total)
    return fail(CAB_ERR_WORKSPACE, "prefill_host: workspace %zu B < %zu B", workspace_bytes,
                kSlots * L.total);
  if (!aligned16(workspace)) return fail(CAB_ERR_INVALID_ARG, "prefill_host: workspace must be 16-byte aligned");
  CopyStreams cp;
  rc = copy_streams(&cp);
  if (rc != CAB_OK) return rc;
  Events ev;
  if (!ev.ok) return fail(CAB_ERR_LAUNCH, "prefill_host: cannot create events");

  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  const int64_t qs[3] = {G * N * D, N * D, D};
  const int64_t ks[3] = {N * D, N * D, D};
  auto* const ws = static_cast<char*>(workspace);
  const char* const hq = static_cast<const char*>(q);
  const char* const hk = static_cast<const char*>(k);
  const char* const hv = static_cast<const char*>(v);
  char* const ho = static_cast<char*>(out);
  cudaError_t ce = cudaSuccess;
  auto cuda_ok = [&](cudaError_t e) {
    if (e != cudaSuccess && ce == cudaSuccess) ce = e;
    return e == cudaSuccess;
  };

  cuda_ok(cudaEventRecord(ev.start, cs));
  cuda_ok(cudaStreamWaitEvent(cp.h2d, ev.start, 0));
  cuda_ok(cudaStreamWaitEvent(cp.d2h, ev.start, 0));
  for (int64_t u = 0; u < U && rc == CAB_OK && ce == cudaSuccess; ++u) {
    const int s = static_cast<int>(u % kSlots);
    char* const base = ws + s * L.total;
    // copy-in: the slot's inputs are free once unit u - kSlots has been computed
    if (u >= kSlots) cuda_ok(cudaStreamWaitEvent(cp.h2d, ev.comp_done[s], 0));
    cuda_ok(cudaMemcpyAsync(base + L.q, hq + u * q_unit, q_unit, cudaMemcpyHostToDevice, cp.h2d));
    cuda_ok(cudaMemcpyAsync(base + L.k, hk + u * k_unit, k_unit, cudaMemcpyHostToDevice, cp.h2d));
    cuda_ok(cudaMemcpyAsync(base + L.v, hv + u * k_unit, k_unit, cudaMemcpyHostToDevice, cp.h2d));
    cuda_ok(cudaEventRecord(ev.in_done[s], cp.h2d));
    // compute: after the copy-in, and after unit u - kSlots's outputs have left the slot
    cuda_ok(cudaStreamWaitEvent(cs, ev.in_done[s], 0));
    if (u >= kSlots) cuda_ok(cudaStreamWaitEvent(cs, ev.out_done[s], 0));
    if (ce != cudaSuccess) break;
    rc = cab_coarsen_maxl2(base + L.q, base + L.k, base + L.qc, base + L.kc, nullptr, nullptr, 1,
                           G, 1, N, D, block_size, qs, ks, dtype, cs);
    if (rc == CAB_OK)
      rc = cab_frc(base + L.qc, base + L.kc, reinterpret_cast<float*>(base + L.frc), nullptr,
                   nullptr, 1, G, 1, M, D, dtype, temperature, lambda_redundancy, normalization,
                   formula, redundancy_scale, L.frc_ws_bytes ? base + L.frc_ws : nullptr,
                   L.frc_ws_bytes, cs);
    if (rc == CAB_OK)
      rc = cab_topk_blocks(reinterpret_cast<const float*>(base + L.frc),
                           reinterpret_cast<int32_t*>(base + L.idx),
                           reinterpret_cast<int32_t*>(base + L.num), nullptr, G, M, keep,
                           select_high, keep_diagonal, causal, cs);
    if (rc == CAB_OK)
      rc = cab_sparse_attn_fwd(base + L.q, base + L.k, base + L.v,
                               reinterpret_cast<const int32_t*>(base + L.idx),
                               reinterpret_cast<const int32_t*>(base + L.num), base + L.out,
                               nullptr, 1, G, 1, N, D, block_size, keep, qs, ks, ks, qs,
                               softmax_scale, causal, dtype,
                               L.attn_ws_bytes ? base + L.attn_ws : nullptr, L.attn_ws_bytes, cs);
    if (rc != CAB_OK) break;
    cuda_ok(cudaEventRecord(ev.comp_done[s], cs));
    // copy-out
    cuda_ok(cudaStreamWaitEvent(cp.d2h, ev.comp_done[s], 0));
    cuda_ok(cudaMemcpyAsync(ho + u * q_unit, base + L.out, q_unit, cudaMemcpyDeviceToHost, cp.d2h));
    if (kv_idx)
      cuda_ok(cudaMemcpyAsync(reinterpret_cast<char*>(kv_idx) + u * idx_unit, base + L.idx,
                              idx_unit, cudaMemcpyDeviceToHost, cp.d2h));
    if (kv_num)
      cuda_ok(cudaMemcpyAsync(reinterpret_cast<char*>(kv_num) + u * num_unit, base + L.num,
                              num_unit, cudaMemcpyDeviceToHost, cp.d2h));
    cuda_ok(cudaEventRecord(ev.out_done[s], cp.d2h));
  }
  // Join both copy streams back into the caller's stream on every path, so that whatever
  // was queued (including after an error) completes before later work on `stream`.
  cudaEventRecord(ev.h2d_end, cp.h2d);
  cudaEventRecord(ev.d2h_end, cp.d2h);
  cudaStreamWaitEvent(cs, ev.h2d_end, 0);
  cudaStreamWaitEvent(cs, ev.d2h_end, 0);
  if (rc != CAB_OK) return rc;
  if (ce != cudaSuccess) {
    cudaGetLastError();
    return fail(CAB_ERR_LAUNCH, "prefill_host: %s", cudaGetErrorString(ce));
  }
  return CAB_OK;
}
