// Three-component KV-cache eviction selection (ThreeComponentEvictionPolicy.select_indices,
// cab_attention/eviction/policy.py:40-210): keep the local window, the most important
// tokens, and "bridge" tokens, and return the kept positions sorted.
//
//   budgets: local = int(K * local_ratio), bridge = int(K * bridge_ratio),
//            importance = K - local - bridge, each clipped to the cache length L
//   local:      [L - local, L)
//   importance: the `importance` largest scores among the rest (padded with zeros /
//               truncated to L); without scores the range just before the local window
//   bridge:     with an attention matrix A and at least one important token: the largest
//               (sum_{i in imp} A[i, j]) * (sum_{i in imp} A[j, i]) among the rest;
//               else with scores: the smallest |score - median| among the rest, the median
//               being the lower median of the scores still unselected; else the positions
//               from one third into the unselected ones
//   ties go to the lower position (torch.topk leaves their order unspecified).
//
// One CTA per sequence keeps the selection bitmap in shared memory and runs the top-k and
// median selections as CTA-wide MSB-first radix selects over keys recomputed from global
// memory on each pass (the score vectors stay in L2). With an attention matrix the work
// is split in four launches so the connectivity sums run grid-wide.

#include "cab_host.h"

#include <algorithm>

namespace cab {
namespace evict {

constexpr int kThreads = 1024;
constexpr int kMaxLen = 1 << 19;  // two bitmaps of kMaxLen bits = 128 KB of shared memory

struct Params {
  const float* imp;   // [batch, imp_len] or null
  int64_t imp_len;
  const float* attn;  // [batch, L, L] or null
  int64_t L;
  int32_t local_b, imp_b, bridge_b, keep_size;
  int64_t* keep;      // [batch, keep_size] sorted kept positions, -1 padded
  int32_t* counts;    // [batch, 4] kept, local, importance, bridge
  uint32_t* bitmap;   // workspace [batch, words]: selection between launches
  uint32_t* impmap;   // workspace [batch, words]: the importance selection
  float* from;        // workspace [batch, L]: connectivity from the important set
  float* score;       // workspace [batch, L]: bridge connectivity scores
  int32_t words;
};

__device__ __forceinline__ uint32_t key_of(float f) {  // order-preserving, NaN least
  if (f != f) f = -__int_as_float(0x7f800000);
  if (f == 0.0f) f = 0.0f;
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float unkey(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

__device__ __forceinline__ bool bit(const uint32_t* m, int64_t j) { return (m[j >> 5] >> (j & 31)) & 1u; }

// Block-wide sum of v (every thread gets it); `red` holds 32 words of shared memory.
__device__ __forceinline__ uint32_t block_sum(uint32_t v, uint32_t* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  uint32_t t = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0u;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
  return t;
}

// Exclusive block-wide prefix of v in thread order (and the total).
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, uint32_t* red, uint32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  __syncthreads();
  if (lane == 31) red[warp] = incl;
  __syncthreads();
  uint32_t wsum = lane < static_cast<int>(blockDim.x >> 5) ? red[lane] : 0u;
  uint32_t wincl = wsum;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t o = __shfl_up_sync(0xffffffffu, wincl, off);
    if (lane >= off) wincl += o;
  }
  const uint32_t before = __shfl_sync(0xffffffffu, wincl - wsum, warp);
  *total = __shfl_sync(0xffffffffu, wincl, (blockDim.x >> 5) - 1);
  return before + incl - v;
}

// Keys of the candidates of one selection: key(j) for unselected j, 0 (never taken) for
// selected ones. Source: scores (larger preferred), or -|x - center| (closer preferred).
struct KeySource {
  const float* x;
  int64_t n;           // valid length of x (positions >= n read as 0)
  int mode;            // 0: x, 1: -|x - center|
  float center;
  __device__ __forceinline__ uint32_t operator()(int64_t j) const {
    const float v = j < n ? x[j] : 0.0f;
    return mode == 0 ? key_of(v) : key_of(-fabsf(v - center));
  }
};

// CTA-wide radix select: the key `tau` and tie count `take_eq` such that the keys > tau
// plus the `take_eq` lowest-position keys == tau are the `r` largest unselected keys.
// With `exact`, tau is always the exact key of rank r (take_eq >= 1).
__device__ void radix_select(const KeySource& ks, const uint32_t* sel, int64_t L, uint32_t r, bool exact,
                             uint32_t* hist, uint32_t* red, uint32_t& tau, uint32_t& take_eq) {
  uint32_t prefix = 0, pmask = 0;
  int hi = 31;
  uint32_t remaining = r;
#pragma unroll 1
  while (true) {
    const int width = min(8, hi + 1);
    const int lo = hi + 1 - width;
    const uint32_t dmask = (1u << width) - 1u;
    for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0u;
    __syncthreads();
    for (int64_t j = threadIdx.x; j < L; j += blockDim.x) {
      if (bit(sel, j)) continue;
      const uint32_t k = ks(j);
      if ((k & pmask) == prefix) atomicAdd(&hist[(k >> lo) & dmask], 1u);
    }
    __syncthreads();
    // find the digit holding rank `remaining` (highest digit first), one warp
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      uint32_t c[8], tot = 0;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        c[t] = hist[255 - 8 * lane - t];
        tot += c[t];
      }
      uint32_t incl = tot;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      uint32_t running = incl - tot;
      int fd = -1;
      uint32_t fa = 0, fc = 0;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        if (fd < 0 && running < remaining && running + c[t] >= remaining) {
          fd = 255 - 8 * lane - t;
          fa = running;
          fc = c[t];
        }
        running += c[t];
      }
      const uint32_t who = __ballot_sync(0xffffffffu, fd >= 0);
      const int src = __ffs(who) - 1;
      const uint32_t d0 = static_cast<uint32_t>(__shfl_sync(0xffffffffu, fd, src));
      const uint32_t d1 = __shfl_sync(0xffffffffu, fa, src);
      const uint32_t d2 = __shfl_sync(0xffffffffu, fc, src);
      if (lane == 0) {
        red[0] = d0;
        red[1] = d1;
        red[2] = d2;
      }
    }
    __syncthreads();
    const uint32_t digit = red[0], above = red[1], count = red[2];
    __syncthreads();
    prefix |= digit << lo;
    pmask |= dmask << lo;
    remaining -= above;
    if (!exact && remaining == count) {
      tau = prefix == 0u ? 0u : prefix - 1u;  // whole bin taken
      take_eq = 0;
      return;
    }
    if (lo == 0) {
      tau = prefix;
      take_eq = remaining;
      return;
    }
    hi = lo - 1;
  }
}

// Marks (in `mark`, and in `sel` if different) the unselected keys > tau and the
// `take_eq` lowest-position unselected keys == tau. Returns how many were marked.
__device__ uint32_t mark_selected(const KeySource& ks, uint32_t* sel, uint32_t* mark, int64_t L, uint32_t tau,
                                  uint32_t take_eq, uint32_t* red) {
  uint32_t eq_seen = 0, marked = 0;
  for (int64_t base = 0; base < L; base += blockDim.x) {
    const int64_t j = base + threadIdx.x;
    bool cand = j < L && !bit(sel, j);
    const uint32_t k = cand ? ks(j) : 0u;
    const bool gt = cand && k > tau;
    const bool eq = cand && k == tau;
    uint32_t eq_total;
    const uint32_t eq_rank = eq_seen + block_excl_scan(eq ? 1u : 0u, red, &eq_total);
    eq_seen += eq_total;
    const bool take = gt || (eq && eq_rank < take_eq);
    __syncthreads();
    if (take) {
      atomicOr(&mark[j >> 5], 1u << (j & 31));
      if (mark != sel) atomicOr(&sel[j >> 5], 1u << (j & 31));
    }
    marked += block_sum(take ? 1u : 0u, red);
    __syncthreads();
  }
  return marked;
}

// Top-r selection among the unselected positions (marks into sel and mark).
__device__ uint32_t select_top(const KeySource& ks, uint32_t* sel, uint32_t* mark, int64_t L, uint32_t r,
                               uint32_t* hist, uint32_t* red) {
  if (r == 0) return 0;
  uint32_t tau, take_eq;
  radix_select(ks, sel, L, r, false, hist, red, tau, take_eq);
  return mark_selected(ks, sel, mark, L, tau, take_eq, red);
}

__device__ uint32_t count_unselected(const uint32_t* sel, int64_t L, uint32_t* red) {
  uint32_t c = 0;
  for (int64_t j = threadIdx.x; j < L; j += blockDim.x) c += bit(sel, j) ? 0u : 1u;
  return block_sum(c, red);
}

// Phase 1: local window and importance selection.
__global__ void __launch_bounds__(kThreads) phase1_kernel(const Params p) {
  extern __shared__ uint32_t sm[];
  uint32_t* sel = sm;                   // [words]
  uint32_t* imp_m = sel + p.words;      // [words]
  uint32_t* hist = imp_m + p.words;     // [256]
  uint32_t* red = hist + 256;           // [32]
  const int64_t b = blockIdx.x;
  const int64_t L = p.L;
  for (int w = threadIdx.x; w < p.words; w += blockDim.x) {
    sel[w] = 0u;
    imp_m[w] = 0u;
  }
  __syncthreads();
  for (int64_t j = L - p.local_b + threadIdx.x; j < L; j += blockDim.x) atomicOr(&sel[j >> 5], 1u << (j & 31));
  __syncthreads();
  uint32_t n_imp = 0;
  if (p.imp && p.imp_b > 0) {
    const uint32_t unsel = static_cast<uint32_t>(L - p.local_b);
    const uint32_t r = min(static_cast<uint32_t>(p.imp_b), unsel);
    KeySource ks{p.imp + b * p.imp_len, p.imp_len, 0, 0.f};
    n_imp = select_top(ks, sel, imp_m, L, r, hist, red);
  } else {
    const int64_t end = L - p.local_b;
    const int64_t start = end - p.imp_b > 0 ? end - p.imp_b : 0;
    for (int64_t j = start + threadIdx.x; j < end; j += blockDim.x) {
      atomicOr(&sel[j >> 5], 1u << (j & 31));
      atomicOr(&imp_m[j >> 5], 1u << (j & 31));
    }
    n_imp = static_cast<uint32_t>(end - start);
  }
  __syncthreads();
  for (int w = threadIdx.x; w < p.words; w += blockDim.x) {
    p.bitmap[b * p.words + w] = sel[w];
    p.impmap[b * p.words + w] = imp_m[w];
  }
  if (threadIdx.x == 0) {
    p.counts[b * 4 + 1] = p.local_b;
    p.counts[b * 4 + 2] = static_cast<int32_t>(n_imp);
  }
}

// Connectivity of every position with the important set: from[j] = sum_{i in imp} A[i, j]
// (one thread per j: the rows of the important positions are read coalesced), then
// score[j] = from[j] * sum_{i in imp} A[j, i] (one warp per j: a walk along row j).
__global__ void __launch_bounds__(256) connectivity_from_kernel(const Params p) {
  const int64_t b = blockIdx.y;
  const int64_t L = p.L;
  const uint32_t* im = p.impmap + b * p.words;
  const float* A = p.attn + b * L * L;
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < L;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float from = 0.f;
    for (int64_t i = 0; i < L; ++i)
      if (bit(im, i)) from += A[i * L + j];
    p.from[b * L + j] = from;
  }
}

__global__ void __launch_bounds__(256) connectivity_score_kernel(const Params p) {
  const int64_t b = blockIdx.y;
  const int64_t L = p.L;
  const uint32_t* im = p.impmap + b * p.words;
  const float* A = p.attn + b * L * L;
  const int lane = threadIdx.x & 31;
  for (int64_t j = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; j < L;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x / 32) {
    float to = 0.f;
    for (int64_t i = lane; i < L; i += 32)
      if (bit(im, i)) to += A[j * L + i];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) to += __shfl_xor_sync(0xffffffffu, to, off);
    if (lane == 0) p.score[b * L + j] = p.from[b * L + j] * to;
  }
}

// Phase 2: bridge selection and the sorted output.
__global__ void __launch_bounds__(kThreads) phase2_kernel(const Params p, int use_attention) {
  extern __shared__ uint32_t sm[];
  uint32_t* sel = sm;
  uint32_t* hist = sel + p.words;
  uint32_t* red = hist + 256;
  const int64_t b = blockIdx.x;
  const int64_t L = p.L;
  for (int w = threadIdx.x; w < p.words; w += blockDim.x) sel[w] = p.bitmap[b * p.words + w];
  __syncthreads();
  uint32_t n_bridge = 0;
  if (p.bridge_b > 0) {
    const uint32_t unsel = count_unselected(sel, L, red);
    const uint32_t r = min(static_cast<uint32_t>(p.bridge_b), unsel);
    // the attention rule needs at least one important position (else the reference falls
    // back to the median / positional rules)
    if (use_attention && p.counts[b * 4 + 2] > 0) {
      KeySource ks{p.score + b * L, L, 0, 0.f};
      n_bridge = select_top(ks, sel, sel, L, r, hist, red);
    } else if (p.imp) {
      if (unsel > 0) {
        // lower median of the unselected scores: the element of ascending rank
        // (unsel - 1) / 2, i.e. descending rank unsel - (unsel - 1) / 2
        KeySource vs{p.imp + b * p.imp_len, p.imp_len, 0, 0.f};
        uint32_t tau, teq;
        radix_select(vs, sel, L, unsel - (unsel - 1) / 2, true, hist, red, tau, teq);
        KeySource ks{p.imp + b * p.imp_len, p.imp_len, 1, unkey(tau)};
        n_bridge = select_top(ks, sel, sel, L, r, hist, red);
      }
    } else {
      // positions from one third into the unselected ones
      const uint32_t start = unsel / 3;
      const uint32_t take = min(r, unsel - start);
      uint32_t seen = 0;
      for (int64_t base = 0; base < L; base += blockDim.x) {
        const int64_t j = base + threadIdx.x;
        const bool cand = j < L && !bit(sel, j);
        uint32_t total;
        const uint32_t rank = seen + block_excl_scan(cand ? 1u : 0u, red, &total);
        seen += total;
        __syncthreads();
        if (cand && rank >= start && rank < start + take) atomicOr(&sel[j >> 5], 1u << (j & 31));
        __syncthreads();
      }
      n_bridge = take;
    }
  }
  __syncthreads();
  // sorted kept positions
  uint32_t written = 0;
  int64_t* out = p.keep + b * p.keep_size;
  for (int64_t base = 0; base < L; base += blockDim.x) {
    const int64_t j = base + threadIdx.x;
    const bool kept = j < L && bit(sel, j);
    uint32_t total;
    const uint32_t pos = written + block_excl_scan(kept ? 1u : 0u, red, &total);
    if (kept && pos < static_cast<uint32_t>(p.keep_size)) out[pos] = j;
    written += total;
    __syncthreads();
  }
  for (int64_t q = written + threadIdx.x; q < p.keep_size; q += blockDim.x) out[q] = -1;
  if (threadIdx.x == 0) {
    p.counts[b * 4 + 0] = static_cast<int32_t>(written);
    p.counts[b * 4 + 3] = static_cast<int32_t>(n_bridge);
  }
}

}  // namespace evict
}  // namespace cab

extern "C" int cab_evict_workspace_size(int64_t batch, int64_t L, int with_attention, size_t* bytes) {
  using namespace cab;
  if (!bytes) return fail(CAB_ERR_INVALID_ARG, "evict_workspace_size: NULL output");
  if (batch <= 0 || L <= 0) return fail(CAB_ERR_INVALID_ARG, "evict_workspace_size: non-positive size");
  const size_t words = static_cast<size_t>((L + 31) / 32);
  size_t b = 2 * static_cast<size_t>(batch) * words * 4;
  b = (b + 255) & ~static_cast<size_t>(255);
  if (with_attention) b += 2 * static_cast<size_t>(batch) * L * 4;
  *bytes = b;
  return CAB_OK;
}

extern "C" int cab_evict_select(const float* importance, int64_t imp_len, const float* attention, int64_t batch,
                                int64_t L, int64_t keep_size, double local_ratio, double bridge_ratio,
                                int64_t* keep_indices, int32_t* counts, void* workspace, size_t workspace_bytes,
                                void* stream) {
  using namespace cab;
  using namespace cab::evict;
  if (!keep_indices || !counts) return fail(CAB_ERR_INVALID_ARG, "evict: NULL output");
  if (batch <= 0 || L <= 0 || keep_size <= 0) return fail(CAB_ERR_INVALID_ARG, "evict: non-positive size");
  if (importance && imp_len <= 0) return fail(CAB_ERR_INVALID_ARG, "evict: imp_len must be positive");
  if (L > kMaxLen) return fail(CAB_ERR_UNSUPPORTED, "evict: cache length %lld > %d", (long long)L, kMaxLen);
  if (!(local_ratio >= 0.0 && bridge_ratio >= 0.0 && local_ratio + bridge_ratio <= 1.0 + 1e-6))
    return fail(CAB_ERR_INVALID_ARG, "evict: ratios must be >= 0 with local + bridge <= 1");
  size_t need = 0;
  cab_evict_workspace_size(batch, L, attention != nullptr, &need);
  if (!workspace || workspace_bytes < need)
    return fail(CAB_ERR_WORKSPACE, "evict: workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  // budgets as the reference computes them (Python int() of a double product)
  int64_t lb = static_cast<int64_t>(static_cast<double>(keep_size) * local_ratio);
  int64_t bb = static_cast<int64_t>(static_cast<double>(keep_size) * bridge_ratio);
  int64_t ib = keep_size - lb - bb;
  lb = std::min(lb, L);
  bb = std::min(bb, L);
  ib = std::min(ib, L);
  Params p{};
  p.imp = importance;
  p.imp_len = importance ? imp_len : 0;
  p.attn = attention;
  p.L = L;
  p.local_b = static_cast<int32_t>(lb);
  p.imp_b = static_cast<int32_t>(ib);
  p.bridge_b = static_cast<int32_t>(bb);
  p.keep_size = static_cast<int32_t>(keep_size);
  p.keep = keep_indices;
  p.counts = counts;
  p.words = static_cast<int32_t>((L + 31) / 32);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.bitmap = reinterpret_cast<uint32_t*>(ws);
  p.impmap = p.bitmap + batch * p.words;
  const size_t maps = (2 * static_cast<size_t>(batch) * p.words * 4 + 255) & ~static_cast<size_t>(255);
  p.from = attention ? reinterpret_cast<float*>(ws + maps) : nullptr;
  p.score = attention ? p.from + batch * L : nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t sm1 = (2 * static_cast<size_t>(p.words) + 256 + 32) * 4;
  const size_t sm2 = (static_cast<size_t>(p.words) + 256 + 32) * 4;
  cudaFuncSetAttribute(phase1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm1);
  cudaFuncSetAttribute(phase2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2);
  phase1_kernel<<<static_cast<unsigned>(batch), kThreads, sm1, st>>>(p);
  if (int rc = check_launch("evict phase1_kernel")) return rc;
  // the attention rule needs at least one important position; that count is known only on
  // the device, so the connectivity runs whenever a matrix is given and phase 2 decides
  // per sequence
  const bool use_attention = attention != nullptr && bb > 0;
  if (use_attention) {
    dim3 gf(static_cast<unsigned>(std::min<int64_t>((L + 255) / 256, 65535)), static_cast<unsigned>(batch));
    connectivity_from_kernel<<<gf, 256, 0, st>>>(p);
    if (int rc = check_launch("evict connectivity_from_kernel")) return rc;
    dim3 gs(static_cast<unsigned>(std::min<int64_t>((L + 7) / 8, 65535)), static_cast<unsigned>(batch));
    connectivity_score_kernel<<<gs, 256, 0, st>>>(p);
    if (int rc = check_launch("evict connectivity_score_kernel")) return rc;
  }
  phase2_kernel<<<static_cast<unsigned>(batch), kThreads, sm2, st>>>(p, use_attention ? 1 : 0);
  return check_launch("evict phase2_kernel");
}
