// K1: Max-L2 block coarsening (HBM-bound).
//
// One warp owns one token block at a time. Each warp keeps a private ring of shared
// memory stages; lane 0 fills them with TMA tiled loads (box = block_size rows x D
// columns of one head), so every byte of Q and K is read from HBM exactly once and the
// warp's next blocks are in flight while it reduces the current one. In a stage, lane l
// owns rows l, l+32, ...: it accumulates each row's squared L2 norm in fp32 (FFMA),
// reading its 16-byte chunks in a lane-rotated order so the 8 lanes of a shared-memory
// phase hit distinct banks, and a warp arg-max picks the best row. Every row whose fp32
// norm lies within the fp32 error bound of that maximum is then re-scored in fp64, which
// is exact for bf16/f16 inputs, so the chosen token (lowest index on exact ties) is the
// one exact arithmetic picks. Its row is copied from shared memory to the dense output.
//
// Semantics follow the reference's Max-L2 pooling (README.md:30-32;
// CAB_Attention_Colab.ipynb cells 5-7: one representative token per block chosen by L2
// norm, output equal to the selected input rows).

#include "cab_host.h"
#include "cab_ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

namespace cab {
namespace coarsen {

struct Params {
  void* qc;
  void* kc;
  int32_t* qidx;
  int32_t* kidx;
  int64_t units_q;  // B*Hq*M (0 if Q is skipped)
  int64_t units_k;  // B*Hkv*M
  int32_t Hq, Hkv, M, N, bs;
  int32_t row_bytes;    // D * elem size
  int32_t stage_bytes;  // bs * row_bytes
  int32_t stages;       // stages per warp
  int32_t warps;        // consumer warps per CTA (each is its own producer)
};

__device__ __forceinline__ double sq_bf16x2(uint32_t w, double acc) {
  float lo = __uint_as_float(w << 16);
  float hi = __uint_as_float(w & 0xFFFF0000u);
  double a = static_cast<double>(lo), b = static_cast<double>(hi);
  acc = fma(a, a, acc);
  return fma(b, b, acc);
}

__device__ __forceinline__ double sq_f16x2(uint32_t w, double acc) {
  __half2 h = *reinterpret_cast<__half2*>(&w);
  float2 f = __half22float2(h);
  double a = static_cast<double>(f.x), b = static_cast<double>(f.y);
  acc = fma(a, a, acc);
  return fma(b, b, acc);
}

__device__ __forceinline__ double sq_f32(uint32_t w, double acc) {
  double a = static_cast<double>(__uint_as_float(w));
  return fma(a, a, acc);
}

template <int kDtype>
__device__ __forceinline__ double accumulate_chunk(const uint4& v, double acc) {
  if constexpr (kDtype == CAB_DTYPE_BF16) {
    acc = sq_bf16x2(v.x, acc);
    acc = sq_bf16x2(v.y, acc);
    acc = sq_bf16x2(v.z, acc);
    acc = sq_bf16x2(v.w, acc);
  } else if constexpr (kDtype == CAB_DTYPE_F16) {
    acc = sq_f16x2(v.x, acc);
    acc = sq_f16x2(v.y, acc);
    acc = sq_f16x2(v.z, acc);
    acc = sq_f16x2(v.w, acc);
  } else {
    acc = sq_f32(v.x, acc);
    acc = sq_f32(v.y, acc);
    acc = sq_f32(v.z, acc);
    acc = sq_f32(v.w, acc);
  }
  return acc;
}

// fp32 variant: bf16 / f16 squares are exact in fp32 and only the additions round.
template <int kDtype>
__device__ __forceinline__ float accumulate_chunk32(const uint4& v, float acc) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (kDtype == CAB_DTYPE_BF16) {
      const float lo = __uint_as_float(w[i] << 16), hi = __uint_as_float(w[i] & 0xFFFF0000u);
      acc = fmaf(lo, lo, acc);
      acc = fmaf(hi, hi, acc);
    } else if constexpr (kDtype == CAB_DTYPE_F16) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      acc = fmaf(f.x, f.x, acc);
      acc = fmaf(f.y, f.y, acc);
    } else {
      const float a = __uint_as_float(w[i]);
      acc = fmaf(a, a, acc);
    }
  }
  return acc;
}

// Exact (fp64) squared norm of one row; chunk order rotated by `start`.
template <int kDtype>
__device__ __forceinline__ double row_norm64(const uint4* row, int chunks, int start) {
  double acc[4] = {0.0, 0.0, 0.0, 0.0};
  int c = start, n = 0;
  for (; n + 4 <= chunks; n += 4) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      acc[u] = accumulate_chunk<kDtype>(row[c], acc[u]);
      c = (c + 1 == chunks) ? 0 : c + 1;
    }
  }
  for (; n < chunks; ++n) {
    acc[0] = accumulate_chunk<kDtype>(row[c], acc[0]);
    c = (c + 1 == chunks) ? 0 : c + 1;
  }
  return (acc[0] + acc[1]) + (acc[2] + acc[3]);
}

// Candidate margin of the fp32 pass: each fp32 norm is a sum of at most 512 / 4 + 3
// rounded terms (D * elem <= 1024 bytes, four partial sums), so its relative error is
// below gamma = 131 * 2^-24 < 8e-6 while no square under- or overflows; a row can only
// match or beat the fp32 arg-max exactly if its fp32 norm is >= (1 - 2 gamma) of it.
constexpr float kCandidateMargin = 4e-5f;
constexpr int kMaxRowsPerLane = 8;  // block_size <= 256

template <int kDtype>
__global__ void __launch_bounds__(256) coarsen_kernel(const __grid_constant__ CUtensorMap qmap,
                                                      const __grid_constant__ CUtensorMap kmap,
                                                      const Params p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= p.warps) return;

  uint8_t* ring = smem_raw + static_cast<size_t>(warp) * p.stages * p.stage_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_raw + static_cast<size_t>(p.warps) *
                                                              p.stages * p.stage_bytes) +
                   warp * p.stages;

  const int64_t total = p.units_q + p.units_k;
  const int64_t first = static_cast<int64_t>(blockIdx.x) * p.warps + warp;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * p.warps;

  if (lane == 0) {
    if (p.units_q) prefetch_tensormap(&qmap);
    if (p.units_k) prefetch_tensormap(&kmap);
    for (int s = 0; s < p.stages; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncwarp();

  auto issue = [&](int64_t u, int s) {
    const CUtensorMap* map;
    int64_t idx;
    int H;
    if (u < p.units_q) {
      map = &qmap; idx = u; H = p.Hq;
    } else {
      map = &kmap; idx = u - p.units_q; H = p.Hkv;
    }
    const int m = static_cast<int>(idx % p.M);
    const int h = static_cast<int>((idx / p.M) % H);
    const int b = static_cast<int>(idx / (static_cast<int64_t>(p.M) * H));
    mbar_arrive_expect_tx(&bars[s], static_cast<uint32_t>(p.stage_bytes));
    tma_load_4d(ring + static_cast<size_t>(s) * p.stage_bytes, map, &bars[s], 0, m * p.bs, h, b);
  };

  if (lane == 0) {
    for (int s = 0; s < p.stages; ++s) {
      const int64_t u = first + s * stride;
      if (u < total) issue(u, s);
    }
  }
  __syncwarp();

  const int chunks = p.row_bytes >> 4;
  int64_t it = 0;
  bool aborted = false;
  for (int64_t u = first; u < total; u += stride, ++it) {
    const int s = static_cast<int>(it % p.stages);
    const uint32_t parity = static_cast<uint32_t>((it / p.stages) & 1);
    const bool ok = mbar_wait(&bars[s], parity);
    if (!__all_sync(0xffffffffu, ok)) { aborted = true; break; }

    const uint8_t* stage = ring + static_cast<size_t>(s) * p.stage_bytes;
    int64_t idx;
    int H;
    bool is_q = u < p.units_q;
    if (is_q) { idx = u; H = p.Hq; } else { idx = u - p.units_q; H = p.Hkv; }
    const int m = static_cast<int>(idx % p.M);
    const int nvalid = min(p.bs, p.N - m * p.bs);

    // Pass 1: fp32 norms (FFMA), arg-max with the lowest index on ties.
    const int start = lane % chunks;
    float n32[kMaxRowsPerLane];
    float best32 = -1.0f;
    int best_row = 0x7fffffff;
#pragma unroll
    for (int x = 0; x < kMaxRowsPerLane; ++x) {
      const int r = lane + 32 * x;
      n32[x] = -1.0f;
      if (r < nvalid) {
        const uint4* row = reinterpret_cast<const uint4*>(stage + static_cast<size_t>(r) * p.row_bytes);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        int c = start, n = 0;
        for (; n + 4 <= chunks; n += 4) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            acc[u] = accumulate_chunk32<kDtype>(row[c], acc[u]);
            c = (c + 1 == chunks) ? 0 : c + 1;
          }
        }
        for (; n < chunks; ++n) {
          acc[0] = accumulate_chunk32<kDtype>(row[c], acc[0]);
          c = (c + 1 == chunks) ? 0 : c + 1;
        }
        const float tot = (acc[0] + acc[1]) + (acc[2] + acc[3]);
        n32[x] = tot;
        if (tot > best32) { best32 = tot; best_row = r; }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best32, off);
      const int orow = __shfl_xor_sync(0xffffffffu, best_row, off);
      if (ob > best32 || (ob == best32 && orow < best_row)) { best32 = ob; best_row = orow; }
    }
    // Pass 2: rows within the fp32 error margin of the arg-max (all rows when the norms
    // are not safely inside fp32 range) are re-scored exactly in fp64.
    const bool safe = best32 >= 1e-30f && best32 <= 3.0e38f;
    const float thr = safe ? best32 * (1.0f - kCandidateMargin) : -2.0f;
    uint32_t cand = 0u;
#pragma unroll
    for (int x = 0; x < kMaxRowsPerLane; ++x)
      if (lane + 32 * x < nvalid && !(n32[x] < thr)) cand |= 1u << x;
    const int ncand = __reduce_add_sync(0xffffffffu, static_cast<unsigned>(__popc(cand)));
    if (ncand > 1) {
      double best = -1.0;
      best_row = 0x7fffffff;
#pragma unroll 1
      for (int x = 0; x < kMaxRowsPerLane; ++x) {
        if (!((cand >> x) & 1u)) continue;
        const int r = lane + 32 * x;
        // same chunk order in every lane, so identical rows get identical sums even for
        // fp32 inputs (whose fp64 sums of squares are not exact)
        const double tot = row_norm64<kDtype>(
            reinterpret_cast<const uint4*>(stage + static_cast<size_t>(r) * p.row_bytes), chunks, 0);
        if (tot > best) { best = tot; best_row = r; }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const double ob = __shfl_xor_sync(0xffffffffu, best, off);
        const int orow = __shfl_xor_sync(0xffffffffu, best_row, off);
        if (ob > best || (ob == best && orow < best_row)) { best = ob; best_row = orow; }
      }
    }
    if (best_row >= nvalid) best_row = 0;  // every valid row was NaN: keep the first

    uint8_t* out = static_cast<uint8_t*>(is_q ? p.qc : p.kc) + idx * static_cast<int64_t>(p.row_bytes);
    const uint4* src = reinterpret_cast<const uint4*>(stage + static_cast<size_t>(best_row) * p.row_bytes);
    for (int c = lane; c < chunks; c += 32) reinterpret_cast<uint4*>(out)[c] = src[c];
    int32_t* idx_out = is_q ? p.qidx : p.kidx;
    if (lane == 0 && idx_out) idx_out[idx] = m * p.bs + best_row;
    __syncwarp();

    const int64_t next = u + static_cast<int64_t>(p.stages) * stride;
    if (lane == 0 && next < total) {
      fence_proxy_async_smem();
      issue(next, s);
    }
    __syncwarp();
  }
  if (aborted && lane == 0) {
    // Give loads still in flight a bounded chance to land before the CTA exits.
    for (int s = 0; s < p.stages; ++s) {
      const int64_t k_it = it + s;
      const int64_t u = first + k_it * stride;
      if (u < total) (void)mbar_wait(&bars[k_it % p.stages], static_cast<uint32_t>((k_it / p.stages) & 1));
    }
  }
}

static int make_map(CUtensorMap* map, const void* base, int dtype, int64_t B, int64_t H, int64_t N,
                    int64_t D, int64_t bs, const int64_t* strides) {
  const size_t es = dtype_size(dtype);
  uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(N), static_cast<uint64_t>(H),
                      static_cast<uint64_t>(B)};
  uint64_t str[3] = {static_cast<uint64_t>(strides[2]) * es, static_cast<uint64_t>(strides[1]) * es,
                     static_cast<uint64_t>(strides[0]) * es};
  uint32_t box[4] = {static_cast<uint32_t>(D), static_cast<uint32_t>(bs), 1, 1};
  return make_tensor_map(map, tma_type(dtype), 4, base, dims, str, box, CU_TENSOR_MAP_SWIZZLE_NONE);
}

}  // namespace coarsen
}  // namespace cab

using namespace cab;

extern "C" int cab_coarsen_maxl2(const void* q, const void* k, void* q_coarse, void* k_coarse,
                                 int32_t* q_idx, int32_t* k_idx, int64_t B, int64_t Hq,
                                 int64_t Hkv, int64_t N, int64_t D, int64_t block_size,
                                 const int64_t* q_strides, const int64_t* k_strides, int dtype,
                                 void* stream) {
  const size_t es = dtype_size(dtype);
  if (!es) return fail(CAB_ERR_UNSUPPORTED, "coarsen: unknown dtype %d", dtype);
  if (!q && !k) return fail(CAB_ERR_INVALID_ARG, "coarsen: both q and k are NULL");
  if ((q && !q_coarse) || (k && !k_coarse))
    return fail(CAB_ERR_INVALID_ARG, "coarsen: missing output pointer");
  if (B <= 0 || N <= 0 || D <= 0 || block_size <= 0 || (q && Hq <= 0) || (k && Hkv <= 0))
    return fail(CAB_ERR_INVALID_ARG, "coarsen: non-positive size");
  if (block_size > 256) return fail(CAB_ERR_UNSUPPORTED, "coarsen: block_size %lld > 256", (long long)block_size);
  const int64_t row_bytes = D * static_cast<int64_t>(es);
  if (row_bytes % 16 != 0 || row_bytes > 1024)
    return fail(CAB_ERR_UNSUPPORTED, "coarsen: D*elem_size = %lld must be a multiple of 16 and <= 1024",
                (long long)row_bytes);
  if (N > (int64_t)1 << 31 || B * std::max(Hq, Hkv) > (int64_t)1 << 31)
    return fail(CAB_ERR_UNSUPPORTED, "coarsen: sizes exceed int32 coordinates");
  const int64_t M = (N + block_size - 1) / block_size;

  CUtensorMap qmap{}, kmap{};
  for (int side = 0; side < 2; ++side) {
    const void* x = side ? k : q;
    if (!x) continue;
    const int64_t* s = side ? k_strides : q_strides;
    void* out = side ? k_coarse : q_coarse;
    if (!s) return fail(CAB_ERR_INVALID_ARG, "coarsen: strides are NULL");
    if (!aligned16(x) || !aligned16(out))
      return fail(CAB_ERR_INVALID_ARG, "coarsen: pointers must be 16-byte aligned");
    for (int i = 0; i < 3; ++i)
      if ((s[i] * static_cast<int64_t>(es)) % 16 != 0 || s[i] <= 0)
        return fail(CAB_ERR_INVALID_ARG, "coarsen: stride %d (%lld elements) is not a positive multiple of 16 bytes",
                    i, (long long)s[i]);
    int rc = coarsen::make_map(side ? &kmap : &qmap, x, dtype, B, side ? Hkv : Hq, N, D, block_size, s);
    if (rc) return rc;
  }

  coarsen::Params p{};
  p.qc = q_coarse; p.kc = k_coarse; p.qidx = q_idx; p.kidx = k_idx;
  p.units_q = q ? B * Hq * M : 0;
  p.units_k = k ? B * Hkv * M : 0;
  p.Hq = static_cast<int32_t>(q ? Hq : 1);
  p.Hkv = static_cast<int32_t>(k ? Hkv : 1);
  p.M = static_cast<int32_t>(M);
  p.N = static_cast<int32_t>(N);
  p.bs = static_cast<int32_t>(block_size);
  p.row_bytes = static_cast<int32_t>(row_bytes);
  p.stage_bytes = static_cast<int32_t>(row_bytes * block_size);

  // Shared-memory budget: as many stages as fit in ~200 KB (at most 16), spread over up
  // to 8 warps with two stages each so every warp keeps one block in flight while it
  // reduces another.
  const int64_t budget = 200 * 1024;
  int64_t total_stages = std::min<int64_t>(16, budget / p.stage_bytes);
  if (total_stages < 1) return fail(CAB_ERR_UNSUPPORTED, "coarsen: block tile of %d bytes does not fit", p.stage_bytes);
  p.warps = static_cast<int32_t>(std::max<int64_t>(1, std::min<int64_t>(8, total_stages / 2)));
  p.stages = static_cast<int32_t>(std::max<int64_t>(1, total_stages / p.warps));
  const size_t smem = static_cast<size_t>(p.warps) * p.stages * p.stage_bytes +
                      static_cast<size_t>(p.warps) * p.stages * sizeof(uint64_t);

  const int64_t units = p.units_q + p.units_k;
  const int64_t ctas_needed = (units + p.warps - 1) / p.warps;
  const int sms = current_sm_count();
  const int64_t per_sm = std::max<int64_t>(1, (227 * 1024) / static_cast<int64_t>(smem + 1024));
  const int grid = static_cast<int>(std::min<int64_t>(ctas_needed, sms * per_sm));
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  switch (dtype) {
#define CAB_LAUNCH_COARSEN(DT)                                                                  \
  case DT: {                                                                                    \
    auto kern = coarsen::coarsen_kernel<DT>;                                                    \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);         \
    kern<<<grid, 32 * p.warps, smem, st>>>(qmap, kmap, p);                                      \
    break;                                                                                      \
  }
    CAB_LAUNCH_COARSEN(CAB_DTYPE_BF16)
    CAB_LAUNCH_COARSEN(CAB_DTYPE_F16)
    CAB_LAUNCH_COARSEN(CAB_DTYPE_F32)
#undef CAB_LAUNCH_COARSEN
  }
  return check_launch("coarsen_kernel");
}
