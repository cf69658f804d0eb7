// Node-level Forman-Ricci curvature of an attention graph (HBM-bound, two passes over A).
//
//   S_i = sum_j A_ij                      (node strength)
//   T_i = sum_j sum_k A_ij A_jk = sum_j A_ij S_j   (weighted triangles through i)
//   F_i = 4 w_i - 2 S_i + 3 T_i with w_i = S_i, i.e. 2 S_i + 3 T_i
//
// The reference computes T with an O(N^3) scalar loop (cab_attention/kernels/
// frc_triton.py:68-118) or as (A @ A).sum(1) (:243-259); both equal A @ S, two
// matrix-vector passes here. Pass 1: one warp per row, 16-byte loads, fp32 partial sums per
// lane and a warp reduction. Pass 2: the same row walk against S (read through L1: every
// warp of a batch reads the same vector) and the fused F epilogue. Chunks of matrices that
// fit in L2 go through both passes before the next chunk, so A crosses HBM once.

#include "cab_host.h"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

namespace cab {
namespace nodefrc {

__device__ __forceinline__ float f32(float x) { return x; }
__device__ __forceinline__ float f32(__half x) { return __half2float(x); }
__device__ __forceinline__ float f32(__nv_bfloat16 x) { return __bfloat162float(x); }

// Dot product of row `a` (N elements of T) with `s` (N floats, or all ones when null),
// across one warp; 16-byte loads when `vec`.
template <typename T>
__device__ __forceinline__ float row_dot(const T* a, const float* s, int64_t N, bool vec, int lane) {
  constexpr int kPer = 16 / sizeof(T);  // elements per 16-byte load
  float acc[2] = {0.f, 0.f};
  int64_t j0 = 0;
  if (vec) {
    const int64_t nv = N / kPer;
    for (int64_t v = lane; v < nv; v += 32) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4*>(a) + v);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int t = 0; t < kPer; ++t) {
        const float w = f32(e[t]);
        acc[t & 1] = s ? fmaf(w, __ldg(s + v * kPer + t), acc[t & 1]) : acc[t & 1] + w;
      }
    }
    j0 = nv * kPer;
  }
  for (int64_t j = j0 + lane; j < N; j += 32) {
    const float w = f32(a[j]);
    acc[0] = s ? fmaf(w, __ldg(s + j), acc[0]) : acc[0] + w;
  }
  float v = acc[0] + acc[1];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

template <typename T>
__global__ void __launch_bounds__(256) strengths_kernel(const T* A, float* S, int64_t rows, int64_t N, bool vec) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; r < rows;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x / 32) {
    const float v = row_dot<T>(A + r * N, nullptr, N, vec, lane);
    if (lane == 0) S[r] = v;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) frc_kernel(const T* A, const float* S, float* F, float* Tri, int64_t rows,
                                                  int64_t N, bool vec) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32; r < rows;
       r += static_cast<int64_t>(gridDim.x) * blockDim.x / 32) {
    const int64_t b = r / N;
    const float t = row_dot<T>(A + r * N, S + b * N, N, vec, lane);
    if (lane == 0) {
      if (Tri) Tri[r] = t;
      F[r] = 2.0f * S[r] + 3.0f * t;
    }
  }
}

// The matrices are processed in chunks of at most kL2Chunk bytes, both passes per chunk,
// so the second pass over a chunk reads it from L2 (126 MB) instead of HBM.
constexpr int64_t kL2Chunk = 48ll << 20;

template <typename T>
static int launch(const void* attn, float* F, float* S, float* Tri, int64_t batch, int64_t N, cudaStream_t st) {
  const T* A = static_cast<const T*>(attn);
  const bool vec = aligned16(attn) && (N * static_cast<int64_t>(sizeof(T))) % 16 == 0;
  const int64_t mat_bytes = N * N * static_cast<int64_t>(sizeof(T));
  const int64_t per_chunk = std::max<int64_t>(1, kL2Chunk / std::max<int64_t>(1, mat_bytes));
  for (int64_t b0 = 0; b0 < batch; b0 += per_chunk) {
    const int64_t nb = std::min(per_chunk, batch - b0);
    const int64_t rows = nb * N;
    const int grid = static_cast<int>(std::min<int64_t>((rows + 7) / 8, (int64_t)current_sm_count() * 8));
    const T* Ab = A + b0 * N * N;
    float* Sb = S + b0 * N;
    strengths_kernel<T><<<grid, 256, 0, st>>>(Ab, Sb, rows, N, vec);
    if (int rc = check_launch("node_frc strengths_kernel")) return rc;
    frc_kernel<T><<<grid, 256, 0, st>>>(Ab, Sb, F + b0 * N, Tri ? Tri + b0 * N : nullptr, rows, N, vec);
    if (int rc = check_launch("node_frc frc_kernel")) return rc;
  }
  return CAB_OK;
}

}  // namespace nodefrc
}  // namespace cab

extern "C" int cab_node_frc(const void* attention, float* frc, float* strengths, float* triangles, int64_t batch,
                            int64_t N, int dtype, void* stream) {
  using namespace cab;
  if (!attention || !frc || !strengths) return fail(CAB_ERR_INVALID_ARG, "node_frc: NULL pointer");
  if (batch <= 0 || N <= 0) return fail(CAB_ERR_INVALID_ARG, "node_frc: non-positive size");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case CAB_DTYPE_F32: return nodefrc::launch<float>(attention, frc, strengths, triangles, batch, N, st);
    case CAB_DTYPE_F16: return nodefrc::launch<__half>(attention, frc, strengths, triangles, batch, N, st);
    case CAB_DTYPE_BF16: return nodefrc::launch<__nv_bfloat16>(attention, frc, strengths, triangles, batch, N, st);
    default: return fail(CAB_ERR_UNSUPPORTED, "node_frc: unknown dtype %d", dtype);
  }
}
