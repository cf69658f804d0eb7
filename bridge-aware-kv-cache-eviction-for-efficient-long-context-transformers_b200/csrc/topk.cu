// K3: per-row top-k block selection (HBM-bound on reading the score matrix).
//
// One warp owns one row (b, h, i) of the [BH, M, M] score matrix at a time. It reads the
// row once (coalesced, 16-byte loads when M % 4 == 0, four per lane in flight) and stores
// it in shared memory as order-preserving 32-bit keys: the preferred direction
// (select_high or not) maps to "larger key", NaN to the least preferred real key, -0 to
// +0, excluded (causal j > i) candidates to 0 and the forced diagonal to 0xFFFFFFFF. An
// MSB-first radix select over the ordinary keys (8-bit digits, 256-bin shared-memory
// histogram) starts at the highest bit in which the row's keys differ and stops as soon
// as the boundary bin is taken whole, which gives the threshold tau. A final pass in index order (128 keys per step, four
// consecutive keys per lane) takes every key > tau and the lowest-index keys == tau until
// k_i are taken, compacting with warp prefix sums so kv_idx comes out ascending, and
// writes the dense 0/1 mask of the row.
//
// Selection rule: per-(b,h,row) top-k of the Forman-Ricci score (generate_block_mask,
// called with select_high / keep_diagonal / causal at experiments/longbench_qa/
// methods.py:339-345; k = max(1, int((1 - sparsity) * M)) as at methods.py:252).

#include "cab_host.h"
#include "cab_ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

namespace cab {
namespace topk {

struct Params {
  const float* scores;  // [rows, M] score matrix (FRC), preferred direction select_high
  const float* mag;     // hybrid: [rows, M] magnitude scores (larger preferred), or null
  int32_t* kv_idx;
  int32_t* kv_num;
  uint8_t* dense;
  int64_t rows;  // BH * M
  int32_t M, k;
  int32_t select_high, keep_diagonal, causal;
  int32_t warps;
  double mag_ratio;  // hybrid: share of the non-diagonal budget taken by magnitude
};

__device__ __forceinline__ uint32_t to_key(float f, bool high) {
  float g = high ? f : -f;
  if (g != g) g = -__int_as_float(0x7f800000);  // NaN -> -inf (least preferred)
  if (g == 0.0f) g = 0.0f;                       // -0 -> +0
  const uint32_t bits = __float_as_uint(g);
  return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}

// Exclusive warp prefix sum of v (and the warp total in *total).
__device__ __forceinline__ uint32_t warp_excl_scan(uint32_t v, int lane, uint32_t* total) {
  uint32_t incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += o;
  }
  *total = __shfl_sync(0xffffffffu, incl, 31);
  return incl - v;
}

// Key of candidate j of row i. diag: 0 = ordinary, 1 = forced (always taken), 2 = excluded.
// `taken` (a bitmap, or null) excludes candidates already chosen by an earlier phase.
// kCheckN: candidates j >= ncand (causal rows) are excluded; without it every j < M is one.
template <bool kCheckN>
__device__ __forceinline__ uint32_t key_at(float f, int j, int i, int ncand, bool high, int diag,
                                           const uint32_t* taken) {
  uint32_t key = to_key(f, high);
  if (kCheckN && j >= ncand) key = 0u;
  if (taken && ((taken[j >> 5] >> (j & 31)) & 1u)) key = 0u;
  if (diag != 0 && j == i) key = diag == 1 ? 0xFFFFFFFFu : 0u;
  return key;
}

// Loads row `src` into the warp's key buffer (four 16-byte loads per lane in flight when
// M % 4 == 0; the tail of the last 4-key group is excluded) and returns the warp-reduced
// range [kmin, kmax] of the ordinary keys (neither excluded nor forced).
template <bool kCheckN>
__device__ __forceinline__ void load_row(const float* src, uint32_t* keys, int M, int row_words, int i,
                                         int ncand, bool high, int diag, const uint32_t* taken, int lane,
                                         uint32_t& kmin, uint32_t& kmax) {
  kmin = 0xFFFFFFFFu;
  kmax = 0u;
  const int M4 = row_words >> 2;
  auto track = [&](uint32_t key) {
    if (key != 0u && key != 0xFFFFFFFFu) {
      kmin = min(kmin, key);
      kmax = max(kmax, key);
    }
  };
  if ((M & 3) == 0) {
    const float4* src4 = reinterpret_cast<const float4*>(src);
    uint4* keys4 = reinterpret_cast<uint4*>(keys);
    for (int base = lane; base < M4; base += 32 * 4) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (base + 32 * u < M4) v[u] = __ldg(src4 + base + 32 * u);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int j4 = base + 32 * u;
        if (j4 < M4) {
          uint4 kv;
          kv.x = key_at<kCheckN>(v[u].x, 4 * j4 + 0, i, ncand, high, diag, taken);
          kv.y = key_at<kCheckN>(v[u].y, 4 * j4 + 1, i, ncand, high, diag, taken);
          kv.z = key_at<kCheckN>(v[u].z, 4 * j4 + 2, i, ncand, high, diag, taken);
          kv.w = key_at<kCheckN>(v[u].w, 4 * j4 + 3, i, ncand, high, diag, taken);
          track(kv.x);
          track(kv.y);
          track(kv.z);
          track(kv.w);
          keys4[j4] = kv;
        }
      }
    }
  } else {
    for (int base = lane; base < row_words; base += 32 * 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = base + 32 * u;
        v[u] = j < M ? __ldg(src + j) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = base + 32 * u;
        if (j < row_words) {
          const uint32_t key = j < M ? key_at<kCheckN>(v[u], j, i, ncand, high, diag, taken) : 0u;
          track(key);
          keys[j] = key;
        }
      }
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, off));
    kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, off));
  }
  __syncwarp();
}

// MSB-first radix select over the ordinary keys: the threshold such that taking every
// key > tau, and among keys == tau the lowest `take_eq` indices, takes exactly `remaining`
// ordinary keys. Starts at the highest bit in which the ordinary keys differ; stops as
// soon as the boundary bin is taken whole.
__device__ __forceinline__ void radix_threshold(const uint32_t* keys, int M4, uint32_t* hist, uint32_t kmin,
                                                uint32_t kmax, int remaining, int lane, uint32_t& tau,
                                                int& take_eq) {
  const uint4* keys4 = reinterpret_cast<const uint4*>(keys);
  tau = 0xFFFFFFFEu;  // only the forced key (0xFFFFFFFF) is above this
  take_eq = 0;
  if (remaining <= 0) return;
  const uint32_t diff = kmin ^ kmax;
  if (diff == 0u) {
    tau = kmin;
    take_eq = remaining;
    return;
  }
  int hi = 31 - __clz(diff);  // highest differing bit; bits above it are shared
  uint32_t prefix = hi == 31 ? 0u : (kmin & ~((2u << hi) - 1u));
  uint32_t pmask = hi == 31 ? 0u : ~((2u << hi) - 1u);
#pragma unroll 1
  while (true) {
    const int width = min(8, hi + 1);
    const int lo = hi + 1 - width;
    const uint32_t dmask = (1u << width) - 1u;
    for (int b = lane; b < 256; b += 32) hist[b] = 0u;
    __syncwarp();
    for (int j4 = lane; j4 < M4; j4 += 32) {
      const uint4 kv = keys4[j4];
      const uint32_t ks[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
      for (int t = 0; t < 4; ++t)
        if (ks[t] != 0u && ks[t] != 0xFFFFFFFFu && (ks[t] & pmask) == prefix)
          atomicAdd(&hist[(ks[t] >> lo) & dmask], 1u);
    }
    __syncwarp();
    // lane l owns bins 255-8l .. 248-8l (highest first)
    uint32_t c[8];
    uint32_t tot = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      c[t] = hist[255 - 8 * lane - t];
      tot += c[t];
    }
    uint32_t all;
    uint32_t running = warp_excl_scan(tot, lane, &all);
    int found_digit = -1;
    uint32_t found_above = 0, found_count = 0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      if (found_digit < 0 && running < static_cast<uint32_t>(remaining) &&
          running + c[t] >= static_cast<uint32_t>(remaining)) {
        found_digit = 255 - 8 * lane - t;
        found_above = running;
        found_count = c[t];
      }
      running += c[t];
    }
    const uint32_t who = __ballot_sync(0xffffffffu, found_digit >= 0);
    const int src_lane = __ffs(who) - 1;
    const uint32_t digit = static_cast<uint32_t>(__shfl_sync(0xffffffffu, found_digit, src_lane));
    const uint32_t above = __shfl_sync(0xffffffffu, found_above, src_lane);
    const uint32_t count = __shfl_sync(0xffffffffu, found_count, src_lane);
    prefix |= digit << lo;
    pmask |= dmask << lo;
    remaining -= static_cast<int>(above);
    __syncwarp();
    if (static_cast<uint32_t>(remaining) == count) {
      // the whole boundary bin is taken: every ordinary key >= prefix (low bits zero).
      // Ordinary keys are >= 0x007FFFFF, so tau = 0 still leaves the excluded keys out.
      tau = prefix == 0u ? 0u : prefix - 1u;
      take_eq = 0;
      return;
    }
    if (lo == 0) {
      tau = prefix;  // exact boundary key; ties by index
      take_eq = remaining;
      return;
    }
    hi = lo - 1;
  }
}

// The index-order pass, 128 keys per step (four consecutive keys per lane): a key is
// taken if > tau, or == tau among the lowest `take_eq` such indices, or (when `or_bits`
// is given) marked there. Taken keys are added to `set_bits` (if given), written
// ascending to `out_idx` (if given) with warp prefix sums, and to the dense row (if given).
__device__ __forceinline__ int select_pass(const uint32_t* keys, int M, int M4, uint32_t tau, int take_eq,
                                           const uint32_t* or_bits, uint32_t* set_bits, int32_t* out_idx,
                                           uint8_t* out_dense, int lane) {
  const uint4* keys4 = reinterpret_cast<const uint4*>(keys);
  uint32_t eq_seen = 0, taken = 0;
  for (int base = 0; base < M4; base += 32) {
    const int j4 = base + lane;
    const uint4 kv = j4 < M4 ? keys4[j4] : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t ks[4] = {kv.x, kv.y, kv.z, kv.w};
    uint32_t take_bits = 0;
    if (take_eq == 0) {  // warp-uniform: no ties at tau to split by index
#pragma unroll
      for (int t = 0; t < 4; ++t) take_bits |= (ks[t] > tau ? 1u : 0u) << t;
    } else {
      uint32_t n_eq = 0;
#pragma unroll
      for (int t = 0; t < 4; ++t) n_eq += (ks[t] == tau) ? 1u : 0u;
      uint32_t eq_total;
      uint32_t eq_rank = eq_seen + warp_excl_scan(n_eq, lane, &eq_total);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        bool take = ks[t] > tau;
        if (ks[t] == tau) {
          take = eq_rank < static_cast<uint32_t>(take_eq);
          ++eq_rank;
        }
        take_bits |= (take ? 1u : 0u) << t;
      }
      eq_seen += eq_total;
    }
    if (j4 >= M4) take_bits = 0u;
    if (or_bits && j4 < M4) take_bits |= (or_bits[j4 >> 3] >> (4 * (j4 & 7))) & 0xFu;
    if (set_bits && take_bits) atomicOr(&set_bits[j4 >> 3], take_bits << (4 * (j4 & 7)));
    uint32_t take_total;
    uint32_t pos = taken + warp_excl_scan(__popc(take_bits), lane, &take_total);
    if (out_idx) {
#pragma unroll
      for (int t = 0; t < 4; ++t)
        if ((take_bits >> t) & 1u) out_idx[pos++] = 4 * j4 + t;
    }
    taken += take_total;
    if (out_dense && j4 < M4) {
      if ((M & 3) == 0) {
        reinterpret_cast<uchar4*>(out_dense)[j4] =
            make_uchar4(take_bits & 1u, (take_bits >> 1) & 1u, (take_bits >> 2) & 1u, (take_bits >> 3) & 1u);
      } else {
#pragma unroll
        for (int t = 0; t < 4; ++t)
          if (4 * j4 + t < M) out_dense[4 * j4 + t] = (take_bits >> t) & 1u;
      }
    }
  }
  __syncwarp();
  return static_cast<int>(taken);
}

// kHybrid: a magnitude phase before the score phase; kCausal: row i has i + 1 candidates.
template <bool kHybrid, bool kCausal>
__global__ void __launch_bounds__(256, 3) topk_kernel(const Params p) {
  extern __shared__ __align__(16) uint32_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = p.M;
  const int row_words = (M + 3) & ~3;
  const int M4 = row_words >> 2;  // 4-key groups (the tail group is padded with excluded keys)
  // per-warp layout: keys [row_words] | histogram [256] | bitmap [bm_words]; every part a
  // multiple of 4 words so each warp's keys stay 16-byte aligned for the uint4 accesses
  const int bm_words = (((row_words + 31) / 32) + 3) & ~3;
  uint32_t* keys = smem + static_cast<size_t>(warp) * (row_words + 256 + bm_words);
  uint32_t* hist = keys + row_words;
  uint32_t* bits = hist + 256;  // hybrid: candidates taken by magnitude
  const bool high = p.select_high != 0;
  constexpr bool hybrid = kHybrid;

  for (int64_t row = static_cast<int64_t>(blockIdx.x) * p.warps + warp; row < p.rows;
       row += static_cast<int64_t>(gridDim.x) * p.warps) {
    const int i = static_cast<int>(row % M);
    const int ncand = kCausal ? i + 1 : M;
    const int kk = min(p.k, ncand);
    const int forced = (p.keep_diagonal && i < ncand) ? 1 : 0;
    int rest = kk - forced;  // budget beyond the forced diagonal
    uint32_t kmin, kmax, tau;
    int take_eq;
    if (hybrid) {
      // phase 1: floor(rest * ratio) candidates with the largest magnitude score (the
      // forced diagonal is not one of them), marked in the bitmap
      const int k_mag = static_cast<int>(static_cast<double>(rest) * p.mag_ratio);
      for (int w = lane; w < bm_words; w += 32) bits[w] = 0u;
      __syncwarp();
      if (k_mag > 0) {
        load_row<kCausal>(p.mag + row * M, keys, M, row_words, i, ncand, true, forced ? 2 : 0, nullptr, lane, kmin, kmax);
        radix_threshold(keys, M4, hist, kmin, kmax, k_mag, lane, tau, take_eq);
        select_pass(keys, M, M4, tau, take_eq, nullptr, bits, nullptr, nullptr, lane);
      }
      rest -= k_mag;
    }
    // phase 2 (the only phase without magnitude scores): the rest by score, among the
    // candidates not yet taken, plus the forced diagonal
    load_row<kCausal>(p.scores + row * M, keys, M, row_words, i, ncand, high, p.keep_diagonal ? 1 : 0,
             hybrid ? bits : nullptr, lane, kmin, kmax);
    radix_threshold(keys, M4, hist, kmin, kmax, rest, lane, tau, take_eq);
    int32_t* out_idx = p.kv_idx + row * p.k;
    uint8_t* out_dense = p.dense ? p.dense + row * M : nullptr;
    select_pass(keys, M, M4, tau, take_eq, hybrid ? bits : nullptr, nullptr, out_idx, out_dense, lane);
    for (int pos = kk + lane; pos < p.k; pos += 32) out_idx[pos] = -1;
    if (lane == 0) p.kv_num[row] = kk;
    __syncwarp();
  }
}

// ---------------------------------------------------------------- block max-pool
// out[bh, I, J] = max over the block_size x block_size tile (I, J) of attn[bh]; a partial
// last block also sees the zero padding (the reference pads with 0 before pooling).
// One CTA per (bh, I): every thread keeps the running maxima of its column chunks (8
// consecutive elements) over the tile's rows, then the chunks of one column block meet
// through shared memory.
__device__ __forceinline__ float to_float(float x) { return x; }
__device__ __forceinline__ float to_float(__half x) { return __half2float(x); }
__device__ __forceinline__ float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }

// Eight consecutive elements from a 16-byte aligned address.
__device__ __forceinline__ void load8(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <typename H>
__device__ __forceinline__ void load8(const H* p, float (&v)[8]) {
  const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
  const H* h = reinterpret_cast<const H*>(&a);
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = to_float(h[e]);
}

template <typename T>
__global__ void __launch_bounds__(256) block_maxpool_kernel(const T* attn, float* out, int64_t N, int bs,
                                                            int Mb, bool vec) {
  extern __shared__ float part[];  // [256 threads][chunks per thread] running maxima
  const int64_t bh = blockIdx.y;
  const int I = blockIdx.x;
  const int64_t r0 = static_cast<int64_t>(I) * bs;
  const int64_t r1 = (r0 + bs < N) ? r0 + bs : N;
  const bool pad_rows = (r1 - r0) < bs;
  const int chunks = static_cast<int>((N + 7) / 8);
  const T* base = attn + bh * N * N;
  for (int c0 = 0; c0 < chunks; c0 += blockDim.x * 16) {
    float mx[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) mx[u] = -INFINITY;
    for (int64_t r = r0; r < r1; ++r) {
      const T* rowp = base + r * N;
#pragma unroll
      for (int u = 0; u < 16; ++u) {
        const int c = c0 + threadIdx.x + u * blockDim.x;
        if (c < chunks) {
          const int64_t j0 = static_cast<int64_t>(c) * 8;
          float v[8];
          if (vec && j0 + 8 <= N) {
            load8(rowp + j0, v);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = j0 + e < N ? to_float(rowp[j0 + e]) : -INFINITY;
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) mx[u] = fmaxf(mx[u], v[e]);
        }
      }
    }
    // column chunk c covers columns 8c .. 8c+7 of column block (8c) / bs
#pragma unroll
    for (int u = 0; u < 16; ++u) part[threadIdx.x * 16 + u] = mx[u];
    __syncthreads();
    const int per_block = bs / 8;  // chunks per column block (bs is a multiple of 8)
    const int cb0 = c0 / per_block;
    const int cb1 = min(Mb, (c0 + static_cast<int>(blockDim.x) * 16 + per_block - 1) / per_block);
    for (int J = cb0 + threadIdx.x; J < cb1; J += blockDim.x) {
      float m = -INFINITY;
      bool partial = pad_rows || static_cast<int64_t>(J + 1) * bs > N;
      for (int q = 0; q < per_block; ++q) {
        const int c = J * per_block + q;
        if (c < c0 || c >= c0 + static_cast<int>(blockDim.x) * 16 || c >= chunks) continue;
        const int rel = c - c0;
        m = fmaxf(m, part[(rel % blockDim.x) * 16 + rel / blockDim.x]);
      }
      if (partial) m = fmaxf(m, 0.f);
      out[(bh * Mb + I) * Mb + J] = m;
    }
    __syncthreads();
  }
}

}  // namespace topk
}  // namespace cab

using namespace cab;

static int launch_topk(const float* scores, const float* mag, double ratio, int32_t* kv_idx, int32_t* kv_num,
                       uint8_t* dense_mask, int64_t BH, int64_t M, int64_t k, int select_high,
                       int keep_diagonal, int causal, void* stream) {
  if (!scores || !kv_idx || !kv_num) return fail(CAB_ERR_INVALID_ARG, "topk: NULL pointer");
  if (BH <= 0 || M <= 0) return fail(CAB_ERR_INVALID_ARG, "topk: non-positive size");
  if (k < 1 || k > M) return fail(CAB_ERR_INVALID_ARG, "topk: k=%lld outside [1, M=%lld]", (long long)k, (long long)M);
  if (M > 49152) return fail(CAB_ERR_UNSUPPORTED, "topk: M=%lld > 49152", (long long)M);
  if (!(ratio >= 0.0 && ratio <= 1.0)) return fail(CAB_ERR_INVALID_ARG, "topk: magnitude_ratio outside [0, 1]");
  topk::Params p{};
  p.scores = scores;
  p.mag = mag;
  p.mag_ratio = ratio;
  p.kv_idx = kv_idx;
  p.kv_num = kv_num;
  p.dense = dense_mask;
  p.rows = BH * M;
  p.M = static_cast<int32_t>(M);
  p.k = static_cast<int32_t>(k);
  p.select_high = select_high != 0;
  p.keep_diagonal = keep_diagonal != 0;
  p.causal = causal != 0;
  const size_t row_words = static_cast<size_t>((M + 3) & ~3);
  const size_t per_warp = (row_words + 256 + ((((row_words + 31) / 32) + 3) & ~static_cast<size_t>(3))) * sizeof(uint32_t);
  int warps = static_cast<int>(std::min<size_t>(8, (200 * 1024) / per_warp));
  if (warps < 1) warps = 1;
  p.warps = warps;
  const size_t smem = per_warp * warps;
  const int64_t ctas_needed = (p.rows + warps - 1) / warps;
  const int per_sm = std::max<int>(1, static_cast<int>((227 * 1024) / (smem + 1024)));
  const int grid = static_cast<int>(std::min<int64_t>(ctas_needed, (int64_t)current_sm_count() * per_sm));
  auto kern = mag ? (p.causal ? topk::topk_kernel<true, true> : topk::topk_kernel<true, false>)
                 : (p.causal ? topk::topk_kernel<false, true> : topk::topk_kernel<false, false>);
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  kern<<<grid, 32 * warps, smem, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("topk_kernel");
}

extern "C" int cab_topk_blocks(const float* scores, int32_t* kv_idx, int32_t* kv_num,
                               uint8_t* dense_mask, int64_t BH, int64_t M, int64_t k,
                               int select_high, int keep_diagonal, int causal, void* stream) {
  return launch_topk(scores, nullptr, 0.0, kv_idx, kv_num, dense_mask, BH, M, k, select_high, keep_diagonal,
                     causal, stream);
}

extern "C" int cab_topk_blocks_hybrid(const float* scores, const float* magnitude, int32_t* kv_idx,
                                      int32_t* kv_num, uint8_t* dense_mask, int64_t BH, int64_t M, int64_t k,
                                      double magnitude_ratio, int select_high, int keep_diagonal, int causal,
                                      void* stream) {
  if (!magnitude) return fail(CAB_ERR_INVALID_ARG, "topk_hybrid: NULL magnitude scores");
  return launch_topk(scores, magnitude, magnitude_ratio, kv_idx, kv_num, dense_mask, BH, M, k, select_high,
                     keep_diagonal, causal, stream);
}

extern "C" int cab_block_maxpool(const void* attn, float* out, int64_t BH, int64_t N, int64_t block_size,
                                 int dtype, void* stream) {
  if (!attn || !out) return fail(CAB_ERR_INVALID_ARG, "block_maxpool: NULL pointer");
  if (BH <= 0 || N <= 0) return fail(CAB_ERR_INVALID_ARG, "block_maxpool: non-positive size");
  if (block_size < 8 || block_size > 1024 || (block_size & (block_size - 1)) != 0)
    return fail(CAB_ERR_UNSUPPORTED, "block_maxpool: block_size %lld (a power of two in [8, 1024])",
                (long long)block_size);
  if (BH > 65535) return fail(CAB_ERR_UNSUPPORTED, "block_maxpool: BH=%lld > 65535", (long long)BH);
  const int64_t Mb = (N + block_size - 1) / block_size;
  const size_t es = dtype_size(dtype);
  if (!es) return fail(CAB_ERR_UNSUPPORTED, "block_maxpool: unknown dtype %d", dtype);
  const bool vec = (N % 8 == 0) && aligned16(attn);
  dim3 grid(static_cast<unsigned>(Mb), static_cast<unsigned>(BH));
  const size_t smem = 256 * 16 * sizeof(float);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int bs = static_cast<int>(block_size), mb = static_cast<int>(Mb);
  switch (dtype) {
    case CAB_DTYPE_F32:
      topk::block_maxpool_kernel<float><<<grid, 256, smem, st>>>(static_cast<const float*>(attn), out, N, bs, mb, vec);
      break;
    case CAB_DTYPE_F16:
      topk::block_maxpool_kernel<__half><<<grid, 256, smem, st>>>(static_cast<const __half*>(attn), out, N, bs, mb, vec);
      break;
    default:
      topk::block_maxpool_kernel<__nv_bfloat16><<<grid, 256, smem, st>>>(static_cast<const __nv_bfloat16*>(attn), out, N, bs, mb, vec);
      break;
  }
  return check_launch("block_maxpool_kernel");
}
