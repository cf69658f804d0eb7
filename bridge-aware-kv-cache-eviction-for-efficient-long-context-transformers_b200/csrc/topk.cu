// K3: per-row top-k block selection (HBM-bound on reading the score matrix).
//
// One warp owns one row (b, h, i) of the [BH, M, M] score matrix at a time. It reads the
// row once (coalesced, 16-byte loads when M % 4 == 0, eight per lane in flight) and stores
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

#include <algorithm>

namespace cab {
namespace topk {

struct Params {
  const float* scores;
  int32_t* kv_idx;
  int32_t* kv_num;
  uint8_t* dense;
  int64_t rows;  // BH * M
  int32_t M, k;
  int32_t select_high, keep_diagonal, causal;
  int32_t warps;
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

__device__ __forceinline__ uint32_t key_at(const Params& p, float f, int j, int i, int ncand, bool high) {
  uint32_t key = to_key(f, high);
  if (j >= ncand) key = 0u;
  if (p.keep_diagonal && j == i) key = 0xFFFFFFFFu;
  return key;
}

__global__ void __launch_bounds__(256) topk_kernel(const Params p) {
  extern __shared__ __align__(16) uint32_t smem[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = p.M;
  const int row_words = (M + 3) & ~3;
  const int M4 = row_words >> 2;  // 4-key groups (the tail group is padded with excluded keys)
  uint32_t* keys = smem + static_cast<size_t>(warp) * (row_words + 256);
  uint4* keys4 = reinterpret_cast<uint4*>(keys);
  uint32_t* hist = keys + row_words;
  const bool high = p.select_high != 0;

  for (int64_t row = static_cast<int64_t>(blockIdx.x) * p.warps + warp; row < p.rows;
       row += static_cast<int64_t>(gridDim.x) * p.warps) {
    const int i = static_cast<int>(row % M);
    const int ncand = p.causal ? i + 1 : M;
    const int kk = min(p.k, ncand);
    const float* src = p.scores + row * M;

    // ---- load the row as keys (eight loads in flight per lane), tracking the range of
    // the ordinary keys (neither excluded nor forced)
    uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
    if ((M & 3) == 0) {
      const float4* src4 = reinterpret_cast<const float4*>(src);
      for (int base = lane; base < M4; base += 32 * 8) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (base + 32 * u < M4) v[u] = __ldg(src4 + base + 32 * u);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int j4 = base + 32 * u;
          if (j4 < M4) {
            uint4 kv;
            kv.x = key_at(p, v[u].x, 4 * j4 + 0, i, ncand, high);
            kv.y = key_at(p, v[u].y, 4 * j4 + 1, i, ncand, high);
            kv.z = key_at(p, v[u].z, 4 * j4 + 2, i, ncand, high);
            kv.w = key_at(p, v[u].w, 4 * j4 + 3, i, ncand, high);
            const uint32_t ks[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
            for (int t = 0; t < 4; ++t)
              if (ks[t] != 0u && ks[t] != 0xFFFFFFFFu) {
                kmin = min(kmin, ks[t]);
                kmax = max(kmax, ks[t]);
              }
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
            const uint32_t key = j < M ? key_at(p, v[u], j, i, ncand, high) : 0u;
            if (key != 0u && key != 0xFFFFFFFFu) {
              kmin = min(kmin, key);
              kmax = max(kmax, key);
            }
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

    // ---- radix select among the ordinary keys (the forced diagonal is always taken,
    // excluded candidates never are). Passes start at the highest bit in which the
    // row's ordinary keys differ, so bits every key shares cost nothing.
    const int forced = (p.keep_diagonal && i < ncand) ? 1 : 0;
    int remaining = kk - forced;
    // Selection rule applied below: take key > tau, and among keys == tau the lowest
    // `take_eq` indices.
    uint32_t tau = 0xFFFFFFFEu;  // only the forced key (0xFFFFFFFF) is above this
    int take_eq = 0;
    if (remaining > 0) {
      const uint32_t diff = kmin ^ kmax;
      if (diff == 0u) {
        tau = kmin;
        take_eq = remaining;
      } else {
        int hi = 31 - __clz(diff);  // highest differing bit; bits above it are shared
        uint32_t prefix = hi == 31 ? 0u : (kmin & ~((2u << hi) - 1u));
        uint32_t pmask = hi == 31 ? 0u : ~((2u << hi) - 1u);
        bool resolved = false;
#pragma unroll 1
        while (!resolved) {
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
            // the whole boundary bin is taken: every ordinary key >= prefix (low bits
            // zero). Ordinary keys are >= 0x007FFFFF, so tau = 0 still leaves the
            // excluded candidates (key 0) out.
            tau = prefix == 0u ? 0u : prefix - 1u;
            take_eq = 0;
            resolved = true;
          } else if (lo == 0) {
            tau = prefix;  // exact boundary key; ties by index
            take_eq = remaining;
            resolved = true;
          } else {
            hi = lo - 1;
          }
        }
      }
    }
    // ---- select in index order, 128 keys per step (4 consecutive keys per lane),
    // compact with warp scans, write outputs
    int32_t* out_idx = p.kv_idx + row * p.k;
    uint8_t* out_dense = p.dense ? p.dense + row * M : nullptr;
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
      uint32_t take_total;
      uint32_t pos = taken + warp_excl_scan(__popc(take_bits), lane, &take_total);
#pragma unroll
      for (int t = 0; t < 4; ++t)
        if ((take_bits >> t) & 1u) out_idx[pos++] = 4 * j4 + t;
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
    for (int pos = kk + lane; pos < p.k; pos += 32) out_idx[pos] = -1;
    if (lane == 0) p.kv_num[row] = kk;
    __syncwarp();
  }
}

}  // namespace topk
}  // namespace cab

using namespace cab;

extern "C" int cab_topk_blocks(const float* scores, int32_t* kv_idx, int32_t* kv_num,
                               uint8_t* dense_mask, int64_t BH, int64_t M, int64_t k,
                               int select_high, int keep_diagonal, int causal, void* stream) {
  if (!scores || !kv_idx || !kv_num) return fail(CAB_ERR_INVALID_ARG, "topk: NULL pointer");
  if (BH <= 0 || M <= 0) return fail(CAB_ERR_INVALID_ARG, "topk: non-positive size");
  if (k < 1 || k > M) return fail(CAB_ERR_INVALID_ARG, "topk: k=%lld outside [1, M=%lld]", (long long)k, (long long)M);
  if (M > 49152) return fail(CAB_ERR_UNSUPPORTED, "topk: M=%lld > 49152", (long long)M);
  topk::Params p{};
  p.scores = scores; p.kv_idx = kv_idx; p.kv_num = kv_num; p.dense = dense_mask;
  p.rows = BH * M;
  p.M = static_cast<int32_t>(M);
  p.k = static_cast<int32_t>(k);
  p.select_high = select_high != 0;
  p.keep_diagonal = keep_diagonal != 0;
  p.causal = causal != 0;
  const size_t per_warp = (static_cast<size_t>((M + 3) & ~3) + 256) * sizeof(uint32_t);
  int warps = static_cast<int>(std::min<size_t>(8, (200 * 1024) / per_warp));
  if (warps < 1) warps = 1;
  p.warps = warps;
  const size_t smem = per_warp * warps;
  const int64_t ctas_needed = (p.rows + warps - 1) / warps;
  const int per_sm = std::max<int>(1, static_cast<int>((227 * 1024) / (smem + 1024)));
  const int grid = static_cast<int>(std::min<int64_t>(ctas_needed, (int64_t)current_sm_count() * per_sm));
  cudaFuncSetAttribute(topk::topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  topk::topk_kernel<<<grid, 32 * warps, smem, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("topk_kernel");
}
