// K2: coarse Forman-Ricci score on tcgen05 tensor cores.
//
//   A      = Qc Kc^T / sqrt(D) / temperature           (GEMM 1, K = D)
//   Direct = |A| | A | min-max(A)                      (GEMM 1 epilogue / normalise pass)
//   T      = Direct Direct  (optionally / M)           (GEMM 2, K = M)
//   F      = Direct - lambda T  |  Direct / (1 + lambda T / (Direct + 1e-8))
//                                                       (GEMM 2 epilogue)
//
// Both GEMMs run in one persistent, warp-specialised kernel template: warp 0 issues TMA
// loads into a shared-memory ring (128-byte swizzle; 2 stages for GEMM 1, 4 for GEMM 2),
// one thread of warp 1 issues tcgen05.mma (M=128, N=256, K=16) into a double-buffered TMEM
// accumulator (2 x 256 columns), and warps 2-9 (two per TMEM lane quadrant) drain the other
// accumulator buffer through tcgen05.ld and run the epilogue, so the epilogue of one
// 128x256 tile overlaps the main loop of the next. The epilogues stage Direct (GEMM 1) and
// F (GEMM 2) in swizzled shared-memory boxes and write them with TMA stores.
// GEMM 2 reads Direct through two tensor maps of the same buffer: K-major for the A
// operand, MN-major (N contiguous) for the B operand, so no transpose is materialised.
//
// Operand precision: GEMM 1 takes the bf16/f16 inputs as they are (exact products, f32
// accumulation). GEMM 2 takes Direct rounded to f16 (10-bit mantissa, f32 accumulation).
// For f32 inputs GEMM 1 runs on CUDA cores in f32 and GEMM 2 uses an f16 hi/lo split of
// Direct (three products: hi*hi + hi*lo + lo*hi), which restores ~f32 accuracy.
//
// Formulas: affinity kernel_benchmark.py:135-137 and methods.py:330-336 (temperature);
// |A| CAB_Attention_Colab.ipynb cell 17; min-max cell 11 and config.py:466; T = Direct
// Direct kernel_benchmark.py:143-144; /M cell 19; additive README.md:34-38; multiplicative
// cell 11.

#include "cab_host.h"
#include "cab_ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

namespace cab {
namespace frc {

constexpr int kTileM = 128;
constexpr int kTileN = 256;
constexpr int kTileK = 64;
constexpr int kStages = 4;
constexpr int kEpiWarps = 8;  // two per TMEM lane quadrant, each drains half the columns
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kABytes = kTileM * kTileK * 2;  // 16 KB
constexpr int kBBytes = kTileN * kTileK * 2;  // 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr float kEps = 1e-8f;

enum Mode { kAffinity = 0, kTriangle = 1 };

// Shared memory per mode. Both epilogues leave through TMA stores staged in 4 KB boxes of
// 32 rows x 128 bytes (128-byte swizzle). GEMM 1 (K = D <= 128, one or two K blocks per
// tile) runs a 2-stage ring and gives each epilogue warp two f16 Direct boxes (32 x 64);
// GEMM 2 runs 4 stages and gives each epilogue warp one f32 F box (32 x 32), reused per
// 32-column chunk once its previous store has read it.
template <int kMode>
struct Ring {
  static constexpr int kStages = kMode == kAffinity ? 2 : frc::kStages;
  static constexpr int kBoxBytes = 32 * 128;
  static constexpr int kStagingBytes = kEpiWarps * (kMode == kAffinity ? 2 : 1) * kBoxBytes;
  static constexpr int kSmem = kStages * kStageBytes + kStagingBytes + 1024 /*align slack*/ + 256 /*barriers*/;
  static_assert(kSmem <= 232448, "shared memory per CTA exceeded");
};

struct Params {
  int32_t BH, Hq, Hkv, M, D, Mp;  // Mp: leading dimension (elements) of the Direct buffers
  int32_t tiles_m, tiles_n, kblocks, segments;
  float alpha;       // GEMM 1: 1/sqrt(D)/temperature; GEMM 2: redundancy scale
  float lambda;
  int32_t normalization, formula;
  __half* direct_hi;  // [BH, M, Mp]
  __half* direct_lo;  // [BH, M, Mp] (split mode only)
  float* raw;         // [BH, M, M] min-max mode: scaled A before normalisation
  uint32_t* minmax;   // [BH, 2] ordered encodings of max(A) and max(-A)
  float* frc;         // [BH, M, M]
  float* affinity;    // [BH, M, M] or null
  float* redundancy;  // [BH, M, M] or null
  int32_t direct_tma;  // GEMM 1: Direct (hi only) leaves through staged TMA stores
  int32_t frc_tma;     // GEMM 2: F leaves through staged TMA stores (M % 4 == 0)
};

__device__ __forceinline__ uint32_t ordered(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float unordered(uint32_t u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7FFFFFFFu) : ~u);
}

__device__ __forceinline__ float direct_of(float v, int normalization) {
  return normalization == CAB_NORM_ABS ? fabsf(v) : v;
}

__device__ __forceinline__ float frc_of(float d, float t, float lambda, int formula) {
  if (formula == CAB_FORMULA_ADDITIVE) return d - lambda * t;
  const float f = d * (1.0f / (1.0f + lambda * t / (d + kEps)));
  return isfinite(f) ? f : 0.0f;
}

// Epilogue of one 32-column chunk of one accumulator row.
template <int kMode>
__device__ __forceinline__ void epilogue_chunk(const Params& p, int bh, int row, int col0,
                                               const uint32_t (&acc)[32], float& vmin_neg,
                                               float& vmax) {
  const int64_t rbase = (static_cast<int64_t>(bh) * p.M + row);
  if constexpr (kMode == kAffinity) {
    __align__(16) __half hv[32];
    __align__(16) __half lv[32];
    __align__(16) float dv[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const float v = __uint_as_float(acc[c]) * p.alpha;
      const float d = direct_of(v, p.normalization);
      dv[c] = d;
      const __half h = __float2half_rn(d);
      hv[c] = h;
      lv[c] = __float2half_rn(d - __half2float(h));
      if (col0 + c < p.M) {
        vmax = fmaxf(vmax, v);
        vmin_neg = fmaxf(vmin_neg, -v);
      }
    }
    const bool full = col0 + 32 <= p.M;
    if (p.normalization == CAB_NORM_MINMAX) {
      float* dst = p.raw + rbase * p.M + col0;
      if (full && (p.M % 4 == 0)) {
#pragma unroll
        for (int c = 0; c < 32; c += 4)
          *reinterpret_cast<float4*>(dst + c) = *reinterpret_cast<float4*>(&dv[c]);
      } else {
        for (int c = 0; c < 32; ++c)
          if (col0 + c < p.M) dst[c] = dv[c];
      }
      return;
    }
    __half* dh = p.direct_hi + rbase * p.Mp + col0;
    __half* dl = p.direct_lo ? p.direct_lo + rbase * p.Mp + col0 : nullptr;
    if (full) {
#pragma unroll
      for (int c = 0; c < 32; c += 8) {
        *reinterpret_cast<uint4*>(dh + c) = *reinterpret_cast<uint4*>(&hv[c]);
        if (dl) *reinterpret_cast<uint4*>(dl + c) = *reinterpret_cast<uint4*>(&lv[c]);
      }
    } else {
      for (int c = 0; c < 32; ++c)
        if (col0 + c < p.M) {
          dh[c] = hv[c];
          if (dl) dl[c] = lv[c];
        }
    }
    if (p.affinity) {
      float* dst = p.affinity + rbase * p.M + col0;
      if (full && (p.M % 4 == 0)) {
#pragma unroll
        for (int c = 0; c < 32; c += 4)
          *reinterpret_cast<float4*>(dst + c) = *reinterpret_cast<float4*>(&dv[c]);
      } else {
        for (int c = 0; c < 32; ++c)
          if (col0 + c < p.M) dst[c] = dv[c];
      }
    }
  } else {
    const __half* dh = p.direct_hi + rbase * p.Mp + col0;
    const __half* dl = p.direct_lo ? p.direct_lo + rbase * p.Mp + col0 : nullptr;
    __align__(16) __half hv[32];
    __align__(16) __half lv[32];
    const bool full = col0 + 32 <= p.M;
    if (full) {
#pragma unroll
      for (int c = 0; c < 32; c += 8) {
        *reinterpret_cast<uint4*>(&hv[c]) = *reinterpret_cast<const uint4*>(dh + c);
        if (dl) *reinterpret_cast<uint4*>(&lv[c]) = *reinterpret_cast<const uint4*>(dl + c);
      }
    } else {
      for (int c = 0; c < 32; ++c) {
        hv[c] = (col0 + c < p.M) ? dh[c] : __float2half(0.f);
        lv[c] = (dl && col0 + c < p.M) ? dl[c] : __float2half(0.f);
      }
    }
    __align__(16) float fv[32];
    __align__(16) float tv[32];
#pragma unroll
    for (int c = 0; c < 32; ++c) {
      const float t = __uint_as_float(acc[c]) * p.alpha;
      float d = __half2float(hv[c]);
      if (dl) d += __half2float(lv[c]);
      tv[c] = t;
      fv[c] = frc_of(d, t, p.lambda, p.formula);
    }
    float* fdst = p.frc + rbase * p.M + col0;
    float* tdst = p.redundancy ? p.redundancy + rbase * p.M + col0 : nullptr;
    if (full && (p.M % 4 == 0)) {
#pragma unroll
      for (int c = 0; c < 32; c += 4) {
        *reinterpret_cast<float4*>(fdst + c) = *reinterpret_cast<float4*>(&fv[c]);
        if (tdst) *reinterpret_cast<float4*>(tdst + c) = *reinterpret_cast<float4*>(&tv[c]);
      }
    } else {
      for (int c = 0; c < 32; ++c)
        if (col0 + c < p.M) {
          fdst[c] = fv[c];
          if (tdst) tdst[c] = tv[c];
        }
    }
  }
}

// GEMM 1 epilogue with the Direct tile staged for a TMA store: this thread's 32 Direct
// values (row `lane` of the warp's box, 16-byte chunks 4h .. 4h + 3 of the 128-byte box row,
// placed at chunk ^ (lane & 7) as the 128-byte swizzle lays them out); the optional f32
// affinity output is written directly. Min-max normalisation and the f16 hi/lo split use
// epilogue_chunk instead.
__device__ __forceinline__ void affinity_staged(const Params& p, int bh, int row, int col0, const uint32_t (&acc)[32],
                                                uint8_t* box, int h, int lane) {
  __align__(16) __half hv[32];
  __align__(16) float dv[32];
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    const float d = direct_of(__uint_as_float(acc[c]) * p.alpha, p.normalization);
    dv[c] = d;
    hv[c] = __float2half_rn(d);
  }
#pragma unroll
  for (int q = 0; q < 4; ++q)
    *reinterpret_cast<uint4*>(box + lane * 128 + 16 * ((4 * h + q) ^ (lane & 7))) =
        *reinterpret_cast<const uint4*>(&hv[8 * q]);
  if (p.affinity && row < p.M && col0 < p.M) {
    float* dst = p.affinity + (static_cast<int64_t>(bh) * p.M + row) * p.M + col0;
    if (col0 + 32 <= p.M && (p.M % 4 == 0)) {
#pragma unroll
      for (int c = 0; c < 32; c += 4) *reinterpret_cast<float4*>(dst + c) = *reinterpret_cast<float4*>(&dv[c]);
    } else {
      for (int c = 0; c < 32; ++c)
        if (col0 + c < p.M) dst[c] = dv[c];
    }
  }
}

// GEMM 2 epilogue with the F chunk staged for a TMA store: F = frc_of(Direct, T) of this
// thread's 32 columns (row `lane` of the warp's 32 x 32 f32 box, 16-byte chunk q placed at
// q ^ (lane & 7)); the optional T output is written directly.
__device__ __forceinline__ void triangle_staged(const Params& p, int bh, int row, int col0, const uint32_t (&acc)[32],
                                                uint8_t* box, int lane) {
  const bool live = row < p.M && col0 < p.M;
  const int64_t rbase = static_cast<int64_t>(bh) * p.M + row;
  __align__(16) __half hv[32];
  if (live && col0 + 32 <= p.M) {
    const __half* dh = p.direct_hi + rbase * p.Mp + col0;
#pragma unroll
    for (int c = 0; c < 32; c += 8) *reinterpret_cast<uint4*>(&hv[c]) = *reinterpret_cast<const uint4*>(dh + c);
  } else {
    const __half* dh = p.direct_hi + rbase * p.Mp + col0;
    for (int c = 0; c < 32; ++c) hv[c] = (live && col0 + c < p.M) ? dh[c] : __float2half(0.f);
  }
  __align__(16) float fv[32];
  __align__(16) float tv[32];
#pragma unroll
  for (int c = 0; c < 32; ++c) {
    const float t = __uint_as_float(acc[c]) * p.alpha;
    tv[c] = t;
    fv[c] = frc_of(__half2float(hv[c]), t, p.lambda, p.formula);
  }
#pragma unroll
  for (int q = 0; q < 8; ++q)
    *reinterpret_cast<uint4*>(box + lane * 128 + 16 * (q ^ (lane & 7))) = *reinterpret_cast<const uint4*>(&fv[4 * q]);
  if (p.redundancy && live) {
    float* tdst = p.redundancy + rbase * p.M + col0;
    for (int c = 0; c < 32; ++c)
      if (col0 + c < p.M) tdst[c] = tv[c];
  }
}

// Persistent tcgen05 GEMM. kMode = kAffinity: A = Qc (K-major), B = Kc (K-major).
// kMode = kTriangle: A = Direct (K-major), B = Direct (MN-major), `segments` = 1 or 3.
template <int kMode>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a0, const __grid_constant__ CUtensorMap map_a1,
                const __grid_constant__ CUtensorMap map_b0, const __grid_constant__ CUtensorMap map_b1,
                const __grid_constant__ CUtensorMap map_d, const Params p, uint32_t idesc) {
  using R = Ring<kMode>;
  constexpr int kStages = R::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* staging = smem + kStages * kStageBytes;  // epilogue store boxes (1024-aligned)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes + R::kStagingBytes);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles = p.BH * p.tiles_m * p.tiles_n;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&map_a0);
    prefetch_tensormap(&map_b0);
    if ((kMode == kAffinity && p.direct_tma) || (kMode == kTriangle && p.frc_tma)) prefetch_tensormap(&map_d);
    if (kMode == kTriangle && p.segments > 1) {
      prefetch_tensormap(&map_a1);
      prefetch_tensormap(&map_b1);
    }
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int kiters = p.kblocks * p.segments;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, last_parity = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int bh = t / (p.tiles_m * p.tiles_n);
        const int rem = t % (p.tiles_m * p.tiles_n);
        const int tm = rem / p.tiles_n, tn = rem % p.tiles_n;
        const int bh_b = (kMode == kAffinity) ? (bh / p.Hq) * p.Hkv + (bh % p.Hq) / (p.Hq / p.Hkv) : bh;
        for (int it = 0; it < kiters; ++it) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag)) { ok = false; break; }
          const int seg = it / p.kblocks, kb = it % p.kblocks;
          const CUtensorMap* ma = (seg == 2) ? &map_a1 : &map_a0;
          const CUtensorMap* mb = (seg == 1) ? &map_b1 : &map_b0;
          uint8_t* sa = smem + stage * kStageBytes;
          uint8_t* sb = sa + kABytes;
          mbar_arrive_expect_tx(&full[stage], kStageBytes);
          tma_load_3d(sa, ma, &full[stage], kb * kTileK, tm * kTileM, bh);
          if (kMode == kAffinity) {
            tma_load_3d(sb, mb, &full[stage], kb * kTileK, tn * kTileN, bh_b);
          } else {
#pragma unroll
            for (int c = 0; c < kTileN / 64; ++c)
              tma_load_3d(sb + c * (kTileK * 128), mb, &full[stage], tn * kTileN + 64 * c, kb * kTileK, bh);
          }
          issued |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        for (int s = 0; s < kStages; ++s)
          if (issued & (1u << s)) (void)mbar_wait(&full[s], (last_parity >> s) & 1u);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const uint64_t desc_a = make_smem_desc(smem_u32(smem), 16, 1024, 2);
      const uint64_t desc_b = (kMode == kAffinity) ? make_smem_desc(smem_u32(smem + kABytes), 16, 1024, 2)
                                                   : make_smem_desc(smem_u32(smem + kABytes), kTileK * 128, 1024, 2);
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag)) { ok = false; break; }
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * kTileN;
        for (int it = 0; it < kiters; ++it) {
          if (!mbar_wait(&full[stage], phase, abort_flag)) { ok = false; break; }
          tc_fence_after_sync();
          const uint64_t soff = static_cast<uint64_t>((stage * kStageBytes) >> 4);
          const uint64_t da0 = desc_a + soff, db0 = desc_b + soff;
#pragma unroll
          for (int kk = 0; kk < kTileK / 16; ++kk) {
            // advance only the 16-byte-unit start address: 32 B per K step (K-major), 16
            // rows x 128 B per K step (MN-major B)
            const uint64_t da = da0 + static_cast<uint64_t>(kk * (32 >> 4));
            const uint64_t db = db0 + static_cast<uint64_t>(kMode == kAffinity ? kk * (32 >> 4) : kk * (2048 >> 4));
            mma_f16_ss(d_tmem, da, db, idesc, (it > 0 || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
      // All MMAs issued by this thread have completed once `drain` flips.
      mma_commit(drain);
      (void)mbar_wait(drain, 0);
    }
    __syncwarp();
  } else {
    const int quad = warp & 3;              // TMEM lane quadrant this warp may access
    const int colhalf = (warp - 2) >> 2;    // which 128 of the tile's 256 columns it drains
    int acc = 0;
    uint32_t acc_phase = 0;
    float vmax = -INFINITY, vmin_neg = -INFINITY;
    int cur_bh = -1;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      const int bh = t / (p.tiles_m * p.tiles_n);
      const int rem = t % (p.tiles_m * p.tiles_n);
      const int tm = rem / p.tiles_n, tn = rem % p.tiles_n;
      if (kMode == kAffinity && p.normalization == CAB_NORM_MINMAX && bh != cur_bh) {
        if (cur_bh >= 0) {
          float a = vmax, b = vmin_neg;
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) {
            a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
            b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, off));
          }
          if (lane == 0) {
            atomicMax(&p.minmax[2 * cur_bh], ordered(a));
            atomicMax(&p.minmax[2 * cur_bh + 1], ordered(b));
          }
        }
        cur_bh = bh;
        vmax = -INFINITY;
        vmin_neg = -INFINITY;
      }
      const bool ok = mbar_wait(&tfull[acc], acc_phase, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after_sync();
      const int row = tm * kTileM + quad * 32 + lane;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * kTileN;
      constexpr int kChunks = kTileN / 32 / 2;
      // staged epilogue: this warp's boxes are free once the stores of its previous tile
      // have read them
      const bool staged = kMode == kAffinity ? p.direct_tma != 0 : p.frc_tma != 0;
      uint8_t* wbox = staging + (warp - 2) * (kMode == kAffinity ? 2 : 1) * R::kBoxBytes;
      if (staged) {
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
      }
#pragma unroll 1
      for (int c = colhalf * kChunks; c < (colhalf + 1) * kChunks; ++c) {
        uint32_t r[32];
        tmem_ld32(taddr + c * 32, r);
        tmem_wait_ld();
        const int col0 = tn * kTileN + c * 32;
        if constexpr (kMode == kAffinity) {
          if (staged) {
            uint8_t* box = wbox + ((c & 3) >> 1) * R::kBoxBytes;
            affinity_staged(p, bh, row, col0, r, box, c & 1, lane);
            if (c & 1) {
              // rows and columns past M are clipped by the tensor map
              fence_proxy_async_smem();
              __syncwarp();
              const int brow = tm * kTileM + quad * 32, bcol = tn * kTileN + (c >> 1) * 64;
              if (lane == 0 && brow < p.M && bcol < p.M) {  // boxes wholly past M are skipped
                tma_store_3d(&map_d, box, bcol, brow, bh);
                bulk_commit_group();
              }
            }
            continue;
          }
        } else {
          if (staged) {
            if (c != colhalf * kChunks) {  // the box is reused: its previous store must have read it
              if (lane == 0) bulk_wait_read_all();
              __syncwarp();
            }
            triangle_staged(p, bh, row, col0, r, wbox, lane);
            fence_proxy_async_smem();
            __syncwarp();
            const int brow = tm * kTileM + quad * 32;
            if (lane == 0 && brow < p.M && col0 < p.M) {  // clipped at M by the tensor map
              tma_store_3d(&map_d, wbox, col0, brow, bh);
              bulk_commit_group();
            }
            continue;
          }
        }
        if (row < p.M && col0 < p.M) epilogue_chunk<kMode>(p, bh, row, col0, r, vmin_neg, vmax);
      }
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (((kMode == kAffinity && p.direct_tma) || (kMode == kTriangle && p.frc_tma)) && lane == 0)
      bulk_wait_all();  // boxes stay valid until stored
    if (kMode == kAffinity && p.normalization == CAB_NORM_MINMAX && cur_bh >= 0) {
      float a = vmax, b = vmin_neg;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, off));
        b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, off));
      }
      if (lane == 0) {
        atomicMax(&p.minmax[2 * cur_bh], ordered(a));
        atomicMax(&p.minmax[2 * cur_bh + 1], ordered(b));
      }
    }
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, 512);
  }
}

// A = Qc Kc^T on CUDA cores for f32 inputs (64x64 tile per CTA, f32 accumulation), with
// the same epilogue as the tensor-core affinity GEMM.
__global__ void __launch_bounds__(256) affinity_f32_kernel(const float* qc, const float* kc, const Params p) {
  __shared__ float sq[64][33];
  __shared__ float sk[64][33];
  const int bh = blockIdx.z;
  const int bh_b = (bh / p.Hq) * p.Hkv + (bh % p.Hq) / (p.Hq / p.Hkv);
  const int i0 = blockIdx.y * 64, j0 = blockIdx.x * 64;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // 16 x 16 threads, 4x4 outputs each
  float acc[4][4] = {};
  const float* qb = qc + static_cast<int64_t>(bh) * p.M * p.D;
  const float* kb = kc + static_cast<int64_t>(bh_b) * p.M * p.D;
  for (int d0 = 0; d0 < p.D; d0 += 32) {
    for (int e = threadIdx.x; e < 64 * 32; e += 256) {
      const int r = e >> 5, c = e & 31;
      sq[r][c] = (i0 + r < p.M && d0 + c < p.D) ? qb[static_cast<int64_t>(i0 + r) * p.D + d0 + c] : 0.f;
      sk[r][c] = (j0 + r < p.M && d0 + c < p.D) ? kb[static_cast<int64_t>(j0 + r) * p.D + d0 + c] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int c = 0; c < 32; ++c) {
      float a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        a[u] = sq[ty + 16 * u][c];
        b[u] = sk[tx + 16 * u][c];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
#pragma unroll
        for (int w = 0; w < 4; ++w) acc[u][w] = fmaf(a[u], b[w], acc[u][w]);
    }
    __syncthreads();
  }
  float vmax = -INFINITY, vmin_neg = -INFINITY;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = i0 + ty + 16 * u;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int j = j0 + tx + 16 * w;
      if (i >= p.M || j >= p.M) continue;
      const float v = acc[u][w] * p.alpha;
      const int64_t o = (static_cast<int64_t>(bh) * p.M + i);
      vmax = fmaxf(vmax, v);
      vmin_neg = fmaxf(vmin_neg, -v);
      if (p.normalization == CAB_NORM_MINMAX) {
        p.raw[o * p.M + j] = v;
      } else {
        const float d = direct_of(v, p.normalization);
        const __half h = __float2half_rn(d);
        p.direct_hi[o * p.Mp + j] = h;
        p.direct_lo[o * p.Mp + j] = __float2half_rn(d - __half2float(h));
        if (p.affinity) p.affinity[o * p.M + j] = d;
      }
    }
  }
  if (p.normalization == CAB_NORM_MINMAX) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, off));
      vmin_neg = fmaxf(vmin_neg, __shfl_xor_sync(0xffffffffu, vmin_neg, off));
    }
    if ((threadIdx.x & 31) == 0) {
      atomicMax(&p.minmax[2 * bh], ordered(vmax));
      atomicMax(&p.minmax[2 * bh + 1], ordered(vmin_neg));
    }
  }
}

// Min-max normalisation: Direct = (A - min) / (max - min + 1e-8) per (b,h) when max > min.
__global__ void __launch_bounds__(256) minmax_normalize_kernel(const Params p) {
  const int64_t rows = static_cast<int64_t>(p.BH) * p.M;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const int bh = static_cast<int>(r / p.M);
    const float mx = unordered(p.minmax[2 * bh]);
    const float mn = -unordered(p.minmax[2 * bh + 1]);
    const bool scale = mx > mn;
    const float inv = 1.0f / (mx - mn + kEps);
    for (int j = threadIdx.x; j < p.M; j += blockDim.x) {
      const float v = p.raw[r * p.M + j];
      const float d = scale ? (v - mn) * inv : v;
      const __half h = __float2half_rn(d);
      p.direct_hi[r * p.Mp + j] = h;
      if (p.direct_lo) p.direct_lo[r * p.Mp + j] = __float2half_rn(d - __half2float(h));
      if (p.affinity) p.affinity[r * p.M + j] = d;
    }
  }
}

struct Layout {
  size_t hi_off, lo_off, raw_off, mm_off, total;
  int64_t Mp;
};

static Layout layout_for(int64_t BH, int64_t M, int dtype, int normalization) {
  Layout L{};
  L.Mp = (M + 7) / 8 * 8;
  const size_t direct_bytes = static_cast<size_t>(BH) * M * L.Mp * 2;
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  L.hi_off = 0;
  L.lo_off = up(direct_bytes);
  const bool split = dtype == CAB_DTYPE_F32;
  L.raw_off = L.lo_off + (split ? up(direct_bytes) : 0);
  const bool minmax = normalization == CAB_NORM_MINMAX;
  L.mm_off = L.raw_off + (minmax ? up(static_cast<size_t>(BH) * M * M * 4) : 0);
  L.total = L.mm_off + (minmax ? up(static_cast<size_t>(BH) * 2 * 4) : 0);
  return L;
}

}  // namespace frc
}  // namespace cab

using namespace cab;

extern "C" int cab_frc_workspace_size(int64_t B, int64_t Hq, int64_t M, int64_t D, int dtype,
                                      int normalization, size_t* bytes) {
  (void)D;
  if (!bytes) return fail(CAB_ERR_INVALID_ARG, "frc_workspace_size: NULL output");
  if (B <= 0 || Hq <= 0 || M <= 0) return fail(CAB_ERR_INVALID_ARG, "frc_workspace_size: non-positive size");
  *bytes = frc::layout_for(B * Hq, M, dtype, normalization).total;
  return CAB_OK;
}

extern "C" int cab_frc(const void* q_coarse, const void* k_coarse, float* frc_out, float* affinity,
                       float* redundancy, int64_t B, int64_t Hq, int64_t Hkv, int64_t M, int64_t D,
                       int dtype, float temperature, float lambda_redundancy, int normalization,
                       int formula, int redundancy_scale, void* workspace, size_t workspace_bytes,
                       void* stream) {
  using namespace frc;
  if (!q_coarse || !k_coarse || !frc_out) return fail(CAB_ERR_INVALID_ARG, "frc: NULL pointer");
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || M <= 0 || D <= 0) return fail(CAB_ERR_INVALID_ARG, "frc: non-positive size");
  if (Hq % Hkv != 0) return fail(CAB_ERR_INVALID_ARG, "frc: Hq=%lld not a multiple of Hkv=%lld", (long long)Hq, (long long)Hkv);
  if (normalization < 0 || normalization > 2) return fail(CAB_ERR_INVALID_ARG, "frc: normalization %d", normalization);
  if (formula < 0 || formula > 1) return fail(CAB_ERR_INVALID_ARG, "frc: formula %d", formula);
  if (redundancy_scale < 0 || redundancy_scale > 1) return fail(CAB_ERR_INVALID_ARG, "frc: redundancy_scale %d", redundancy_scale);
  if (!(temperature > 0.f)) return fail(CAB_ERR_INVALID_ARG, "frc: temperature must be > 0");
  const size_t es = dtype_size(dtype);
  if (!es) return fail(CAB_ERR_UNSUPPORTED, "frc: unknown dtype %d", dtype);
  if (M > (1 << 20)) return fail(CAB_ERR_UNSUPPORTED, "frc: M=%lld too large", (long long)M);
  if (dtype != CAB_DTYPE_F32 && (D * 2) % 16 != 0) return fail(CAB_ERR_UNSUPPORTED, "frc: D=%lld must be a multiple of 8", (long long)D);
  if (!aligned16(q_coarse) || !aligned16(k_coarse) || !aligned16(frc_out) ||
      (affinity && !aligned16(affinity)) || (redundancy && !aligned16(redundancy)))
    return fail(CAB_ERR_INVALID_ARG, "frc: pointers must be 16-byte aligned");
  const int64_t BH = B * Hq;
  const Layout L = layout_for(BH, M, dtype, normalization);
  if (!workspace || workspace_bytes < L.total)
    return fail(CAB_ERR_WORKSPACE, "frc: workspace of %zu bytes needed, %zu given", L.total, workspace_bytes);
  if (!aligned16(workspace)) return fail(CAB_ERR_INVALID_ARG, "frc: workspace must be 16-byte aligned");

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  Params p{};
  p.BH = static_cast<int32_t>(BH);
  p.Hq = static_cast<int32_t>(Hq);
  p.Hkv = static_cast<int32_t>(Hkv);
  p.M = static_cast<int32_t>(M);
  p.D = static_cast<int32_t>(D);
  p.Mp = static_cast<int32_t>(L.Mp);
  p.lambda = lambda_redundancy;
  p.normalization = normalization;
  p.formula = formula;
  p.direct_hi = reinterpret_cast<__half*>(ws + L.hi_off);
  const bool split = dtype == CAB_DTYPE_F32;
  p.direct_lo = split ? reinterpret_cast<__half*>(ws + L.lo_off) : nullptr;
  p.raw = normalization == CAB_NORM_MINMAX ? reinterpret_cast<float*>(ws + L.raw_off) : nullptr;
  p.minmax = normalization == CAB_NORM_MINMAX ? reinterpret_cast<uint32_t*>(ws + L.mm_off) : nullptr;
  p.frc = frc_out;
  p.affinity = affinity;
  p.redundancy = redundancy;
  p.tiles_m = static_cast<int32_t>((M + kTileM - 1) / kTileM);
  p.tiles_n = static_cast<int32_t>((M + kTileN - 1) / kTileN);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int sms = current_sm_count();

  if (p.minmax) cudaMemsetAsync(p.minmax, 0, static_cast<size_t>(BH) * 2 * 4, st);

  // ---- GEMM 1: affinity + Direct
  p.alpha = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D)) / temperature);
  if (dtype == CAB_DTYPE_F32) {
    dim3 grid(static_cast<unsigned>((M + 63) / 64), static_cast<unsigned>((M + 63) / 64), static_cast<unsigned>(BH));
    affinity_f32_kernel<<<grid, 256, 0, st>>>(static_cast<const float*>(q_coarse),
                                              static_cast<const float*>(k_coarse), p);
    if (int rc = check_launch("affinity_f32_kernel")) return rc;
  } else {
    CUtensorMap ma{}, mb{};
    uint64_t dq[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(M), static_cast<uint64_t>(BH)};
    uint64_t sq[2] = {static_cast<uint64_t>(D) * es, static_cast<uint64_t>(M * D) * es};
    uint32_t boxa[3] = {kTileK, kTileM, 1};
    if (int rc = make_tensor_map(&ma, tma_type(dtype), 3, q_coarse, dq, sq, boxa, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    uint64_t dk[3] = {static_cast<uint64_t>(D), static_cast<uint64_t>(M), static_cast<uint64_t>(B * Hkv)};
    uint32_t boxb[3] = {kTileK, kTileN, 1};
    if (int rc = make_tensor_map(&mb, tma_type(dtype), 3, k_coarse, dk, sq, boxb, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    p.kblocks = static_cast<int32_t>((D + kTileK - 1) / kTileK);
    p.segments = 1;
    // Direct (f16) leaves through staged TMA stores unless min-max normalisation needs the
    // raw values first; boxes of 64 columns x 32 rows, clipped at M
    CUtensorMap md{};
    p.direct_tma = normalization != CAB_NORM_MINMAX ? 1 : 0;
    if (p.direct_tma) {
      uint64_t dd[3] = {static_cast<uint64_t>(M), static_cast<uint64_t>(M), static_cast<uint64_t>(BH)};
      uint64_t sd[2] = {static_cast<uint64_t>(L.Mp) * 2, static_cast<uint64_t>(M * L.Mp) * 2};
      uint32_t boxd[3] = {64, 32, 1};
      if (int rc = make_tensor_map(&md, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, p.direct_hi, dd, sd, boxd, CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
    }
    const int tiles = p.BH * p.tiles_m * p.tiles_n;
    const int grid = std::min(tiles, sms);
    const uint32_t idesc = make_idesc_f16(kTileM, kTileN, dtype == CAB_DTYPE_BF16 ? 1 : 0, 0, 0);
    cudaFuncSetAttribute(gemm_kernel<kAffinity>, cudaFuncAttributeMaxDynamicSharedMemorySize, Ring<kAffinity>::kSmem);
    gemm_kernel<kAffinity><<<grid, kThreads, Ring<kAffinity>::kSmem, st>>>(ma, ma, mb, mb, md, p, idesc);
    if (int rc = check_launch("gemm_kernel<affinity>")) return rc;
  }
  if (p.minmax) {
    const int grid = static_cast<int>(std::min<int64_t>(BH * M, (int64_t)sms * 8));
    minmax_normalize_kernel<<<grid, 256, 0, st>>>(p);
    if (int rc = check_launch("minmax_normalize_kernel")) return rc;
  }

  // ---- GEMM 2: T = Direct Direct, F epilogue
  {
    CUtensorMap a0{}, a1{}, b0{}, b1{};
    uint64_t dims[3] = {static_cast<uint64_t>(M), static_cast<uint64_t>(M), static_cast<uint64_t>(BH)};
    uint64_t str[2] = {static_cast<uint64_t>(L.Mp) * 2, static_cast<uint64_t>(M * L.Mp) * 2};
    uint32_t boxa[3] = {kTileK, kTileM, 1};
    uint32_t boxb[3] = {64, kTileK, 1};
    if (int rc = make_tensor_map(&a0, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, p.direct_hi, dims, str, boxa, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    if (int rc = make_tensor_map(&b0, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, p.direct_hi, dims, str, boxb, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    if (split) {
      if (int rc = make_tensor_map(&a1, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, p.direct_lo, dims, str, boxa, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
      if (int rc = make_tensor_map(&b1, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, p.direct_lo, dims, str, boxb, CU_TENSOR_MAP_SWIZZLE_128B)) return rc;
    } else {
      a1 = a0;
      b1 = b0;
    }
    p.kblocks = static_cast<int32_t>((M + kTileK - 1) / kTileK);
    p.segments = split ? 3 : 1;
    p.alpha = redundancy_scale == CAB_RED_SCALE_INV_M ? 1.0f / static_cast<float>(M) : 1.0f;
    // F leaves through staged TMA stores (32 x 32 f32 boxes, clipped at M) when its rows are
    // 16-byte multiples and there is no f16 lo part to add
    CUtensorMap mf{};
    p.frc_tma = (M % 4 == 0 && !split) ? 1 : 0;
    if (p.frc_tma) {
      uint64_t df[3] = {static_cast<uint64_t>(M), static_cast<uint64_t>(M), static_cast<uint64_t>(BH)};
      uint64_t sf[2] = {static_cast<uint64_t>(M) * 4, static_cast<uint64_t>(M * M) * 4};
      uint32_t boxf[3] = {32, 32, 1};
      if (int rc = make_tensor_map(&mf, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, frc_out, df, sf, boxf, CU_TENSOR_MAP_SWIZZLE_128B))
        return rc;
    }
    const int tiles = p.BH * p.tiles_m * p.tiles_n;
    const int grid = std::min(tiles, sms);
    const uint32_t idesc = make_idesc_f16(kTileM, kTileN, 0, 0, 1);
    cudaFuncSetAttribute(gemm_kernel<kTriangle>, cudaFuncAttributeMaxDynamicSharedMemorySize, Ring<kTriangle>::kSmem);
    gemm_kernel<kTriangle><<<grid, kThreads, Ring<kTriangle>::kSmem, st>>>(a0, a1, b0, b1, p.frc_tma ? mf : a0, p, idesc);
    if (int rc = check_launch("gemm_kernel<triangle>")) return rc;
  }
  return CAB_OK;
}
