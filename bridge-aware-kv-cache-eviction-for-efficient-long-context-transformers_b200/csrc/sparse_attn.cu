// K4: block-sparse attention forward over the kept key blocks.
//
// Tensor-core path (bf16/f16, block_size 64, D in {64, 128}):
//  * Work item = (b, query head h, pair p): the 128 query rows of query blocks 2p and
//    2p+1, the M=128 shape of tcgen05.mma. The two rows' kept-block lists are merged by
//    `pair_union_kernel` into one ascending list whose entries carry two flags (kept by
//    block 2p / by block 2p+1); key blocks are consumed two at a time (a 128-key tile).
//    A block kept by only one of the two query blocks is masked for the other 64 rows.
//  * Warp 0 streams each item's Q tile (double-buffered, so the next item's Q lands while
//    this item finishes) and the K and V tiles with TMA (128-byte swizzle) into
//    shared-memory rings. One thread of warp 1 issues S = Q K^T (M=128, N=128, K=D; both
//    operands K-major from shared memory) into one of three TMEM S buffers; one thread of
//    warp 2 issues O += P V (P from TMEM where the softmax wrote it over its S, V read
//    MN-major from its natural [keys, D] layout; M=128, N=D, K=128). Three buffers keep
//    S(g+1), S(g+2) and PV(g-1) in flight while tile g is in the softmax. Warp 3 consumes
//    the PV completions in order and publishes their count.
//  * Warps 4-11, two per row (one per 64-key block of the tile): tcgen05.ld of the S row
//    half, exact masking (union flags, causal token mask, sequence end), online softmax
//    in the exp2 domain with a lazy rescale of O (only when the running max grows by more
//    than 2^8), P stored to TMEM over the S columns it came from, and the final O / l
//    epilogue.
//  * Items run (b, h, p)-major so the CTAs in flight share one head's K/V in L2.
//
// CUDA-core path: one CTA per query block, fp32 arithmetic, any dtype, block <= 128,
// D <= 128.
//
// Semantics: softmax over the kept blocks' keys with -inf elsewhere, fully masked rows
// -> 0 (manual sparse path of the reference: experiments/longbench_qa/methods.py:103-119
// expands the block mask, :348-356 masks, softmaxes and applies nan_to_num).

#include "cab_host.h"
#include "cab_ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

namespace cab {
namespace attn {

constexpr uint32_t kIdxMask = 0x3FFFFFFFu;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed two-wide fp32 arithmetic (one instruction for two lanes of work).
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// ------------------------------------------------------------------ pair union lists
struct UnionParams {
  const int32_t* kv_idx;
  const int32_t* kv_num;
  uint32_t* ulist;   // [items, stride]
  int32_t* ntiles;   // [items]
  int64_t items;     // B*Hq*P
  int32_t M, P, kmax, stride, words;
};

__global__ void __launch_bounds__(128) pair_union_kernel(const UnionParams p) {
  extern __shared__ uint32_t bm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t* b0 = bm + static_cast<size_t>(warp) * 2 * p.words;
  uint32_t* b1 = b0 + p.words;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * 4 + warp; item < p.items;
       item += static_cast<int64_t>(gridDim.x) * 4) {
    const int64_t bh = item / p.P;
    const int pr = static_cast<int>(item % p.P);
    for (int w = lane; w < 2 * p.words; w += 32) b0[w] = 0u;
    __syncwarp();
    for (int half = 0; half < 2; ++half) {
      const int i = 2 * pr + half;
      if (i >= p.M) continue;
      const int64_t row = bh * p.M + i;
      const int n = min(max(p.kv_num[row], 0), p.kmax);
      uint32_t* bits = half ? b1 : b0;
      for (int x = lane; x < n; x += 32) {
        const int j = p.kv_idx[row * p.kmax + x];
        if (j >= 0 && j < p.M) atomicOr(&bits[j >> 5], 1u << (j & 31));
      }
    }
    __syncwarp();
    uint32_t* out = p.ulist + item * p.stride;
    int total = 0;
    for (int base = 0; base < p.words; base += 32) {
      const int w = base + lane;
      const uint32_t x0 = w < p.words ? b0[w] : 0u, x1 = w < p.words ? b1[w] : 0u;
      uint32_t u = x0 | x1;
      const int cnt = __popc(u);
      int incl = cnt;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      int pos = total + incl - cnt;
      while (u) {
        const int bit = __ffs(u) - 1;
        u &= u - 1;
        out[pos++] = static_cast<uint32_t>(32 * w + bit) | (((x0 >> bit) & 1u) << 30) |
                     (((x1 >> bit) & 1u) << 31);
      }
      total += __shfl_sync(0xffffffffu, incl, 31);
    }
    __syncwarp();
    if (lane == 0) {
      if (total & 1) out[total] = out[total - 1] & kIdxMask;  // padding block, masked for all rows
      p.ntiles[item] = (total + 1) / 2;
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------------ tensor-core kernel
// kDense: every item is one 128-row query block against all key tiles in order (the
// flash-attention forward with optional column scores); one Q buffer suffices there (items
// are long), and the space holds the column-score exchange slots.
template <int D, bool kDense = false>
struct Cfg {
  static constexpr int kAtoms = D / 64;
  static constexpr int kQBytes = 128 * D * 2;
  static constexpr int kKBytes = 128 * D * 2;  // one tile = two 64-key blocks
  static constexpr int kVBytes = 128 * D * 2;
  static constexpr int kQStages = kDense ? 1 : 2;  // sparse: the next item's Q lands while this item finishes
  static constexpr int kKStages = D == 128 ? 2 : 5;
  static constexpr int kVStages = D == 128 ? 3 : 5;
  static constexpr int kTileBytes = kQStages * kQBytes + kKStages * kKBytes + kVStages * kVBytes;
  // sparse epilogue: each softmax warp stages its 32 rows x D/2 columns of O (one TMA store
  // box) in the item's Q buffer; the eight boxes fill it exactly
  static constexpr int kWarpOBytes = 32 * (D / 2) * 2;
  static_assert(8 * kWarpOBytes == kQBytes, "O staging must fill the Q buffer");
  static constexpr int kSlotBytes = kDense ? 2 * 2 * 4 * 32 * 8 : 0;  // column sums [parity][kb][quad][lane] float2
  static constexpr int kXchgBytes = 2 * 2 * 128 * 4 + kSlotBytes;  // + row-max / row-sum exchange [parity][kb][row]
  static constexpr int kAuxBytes = kXchgBytes + 512;   // + mbarriers (<= 54), TMEM slot, abort flag, counter
  // Tiles start at the first 1024-byte boundary of the dynamic shared memory; the kernel
  // checks at run time that tiles + aux fit in what it was given.
  static constexpr int kSmemWanted = kTileBytes + kAuxBytes + 1024;
  static constexpr int kSmem = kSmemWanted < 232448 ? kSmemWanted : 232448;
};

// TMEM columns: three S buffers at 0, 128, 256 (fp32; the P of a tile overwrites the S
// columns it came from: the thread owning keys 64*kb..+63 of a row writes their 32 packed
// columns at S column 64*kb), O at 384..384+D-1 (fp32). Three S/P buffers keep three tiles
// in flight: S(g) may start once PV(g - 3), the last reader of its buffer, has finished.
constexpr int kSBufs = 3;
constexpr uint32_t kTmemO = 384;

// One completion signal per MMA group where the rings allow it. After the first
// tcgen05.commit of a group every further commit costs the tensor pipe time (about 86
// clocks measured on B200), so:
//  * with at most kSBufs K stages the producer frees a K stage on s_full (S(g) completed)
//    instead of a separate k_empty commit: S(g + 3), the next phase of the same barrier,
//    needs K(g + 3), which is loaded after that wait, so the producer never falls a phase
//    behind;
//  * with exactly kSBufs V stages, V stage, S/P buffer and PV-completion barrier coincide:
//    buf_free[g % 3] (PV(g) completed) also frees V stage g % 3 and feeds the completion
//    tracker, replacing the v_empty and o_ready commits.
template <class C>
struct Signals {
  static constexpr bool kKOnSFull = C::kKStages <= kSBufs;
  static constexpr bool kPvOneCommit = C::kVStages == kSBufs;
};

// Warp 0: TMA producer; warp 1: issues S = Q K^T; warps 2-9: softmax; warp 10: issues
// O += P V; warp 11: PV completion tracker. Two issuing threads keep the tensor pipe
// queued: while one blocks on a full MMA queue, the other's group is already waiting
// behind it.
//
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void named_bar_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Barrier discipline. Every mbarrier wait is a parity wait, which is only sound while the
// barrier is at most one phase past the phase waited for, and an arrival count is only
// sound while no arrival for a later phase can overtake one for the current phase. Each
// barrier below is therefore waited phase after phase by one consumer, or made safe by a
// dependency: P(g) arrives on p_full[g % 3], and a warp can only reach tile g + 3 after
// PV(g) consumed p_full(g). PV completions are consumed in order by warp 11 alone, which
// publishes their count in `pv_seen`: on buf_free[g % 3] where that barrier is the only
// PV signal (the PV issuer then starts PV(g) once PV(g - 3) has been seen), else on
// o_ready[g & 1] (PV(g) once PV(g - 2) has been seen), so the barrier never runs two
// phases ahead of warp 11 while consecutive PVs can still be queued together. The
// producer's waits on s_full and buf_free are safe for the same reason: the next phase
// of the barrier needs the very tile it is about to load. Softmax threads wait on the
// count only when they must rescale O (rare) and in the epilogue.
constexpr int kSoftmaxWarps = 8;
constexpr int kPvWarp = 2;
constexpr int kTrackWarp = 3;
constexpr int kFirstSoftmaxWarp = 4;
constexpr int kAttnThreads = 32 * (kFirstSoftmaxWarp + kSoftmaxWarps);
// Register split (setmaxnreg, both modes): warpgroup 0 (producer, issuers, tracker) hands
// registers to the two softmax warpgroups (measured on B200 against the even 168 / 168
// split: sparse 4-5 % faster, dense 7 % without and 2 % with column scores). 128 x (kRegsLow + 2 x kRegsHigh) must not exceed the
// launch's 384 x 168; the host checks the kernel's register count before each launch.
constexpr int kRegsLow = 72, kRegsHigh = 216;
constexpr int kRegsNeeded = (128 * (kRegsLow + 2 * kRegsHigh) + kAttnThreads - 1) / kAttnThreads;
static_assert(kRegsNeeded <= 168, "register split exceeds the launch's registers");

struct Params {
  int32_t B, Hq, Hkv, Nq, Nk, M, P;  // sparse: Nq == Nk == N; dense: P = query blocks of 128 rows
  int32_t Tk;                        // dense: key tiles (128 keys) per query block
  int64_t items;
  const void* q;
  int64_t q_s0, q_s1, q_s2;
  int64_t o_s0, o_s1, o_s2;
  void* out;
  float* lse;
  const uint32_t* ulist;
  const int32_t* ntiles;
  int32_t stride;
  float scale_log2;
  int32_t causal;
  float* colsum;      // dense: [B, Hq, Nk] column scores, accumulated (may be null)
  int64_t cs_s0, cs_s1;
  float* partial;     // dense + colsum: per-CTA private column sums [gridDim.x, pstride], zeroed
  int64_t pstride;
};

// Tiles of an item: the merged list length (sparse) or the key tiles up to the causal
// limit (dense).
template <bool kDense>
__device__ __forceinline__ int item_tiles(const Params& p, int64_t item) {
  if constexpr (kDense) {
    const int pr = static_cast<int>(item % p.P);
    return p.causal ? min(p.Tk, pr + 1) : p.Tk;
  } else {
    return static_cast<int>(ld_nc_u32(p.ntiles + item));
  }
}

// List entry of key block kb (0/1) of tile t: block index | kept-by-first-half << 30 |
// kept-by-second-half << 31.
template <bool kDense>
__device__ __forceinline__ uint32_t item_entry(const uint32_t* ul, int t, int kb) {
  if constexpr (kDense) return static_cast<uint32_t>(2 * t + kb) | 0xC0000000u;
  else return ul[2 * t + kb];
}

template <bool kBF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (kBF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}


template <int D, bool kBF16, bool kDense>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap omap,
                   const Params p) {
  using C = Cfg<D, kDense>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = base;
  uint8_t* sK = sQ + C::kQStages * C::kQBytes;
  uint8_t* sV = sK + C::kKStages * C::kKBytes;
  uint8_t* sEnd = sV + C::kVStages * C::kVBytes;
  float* xchg = reinterpret_cast<float*>(sEnd);
  float2* colslots = reinterpret_cast<float2*>(xchg + 512);  // dense: [parity * 2 + kb][quad][lane]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sEnd + C::kXchgBytes);
  {
    uint32_t dyn;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dyn));
    if (sEnd + C::kAuxBytes > smem_raw + dyn) {
      if (threadIdx.x == 0) atomicOr(&g_device_status, CAB_DEVICE_LAYOUT);
      return;  // shared memory base not aligned as expected: nothing was touched
    }
  }
  uint64_t* q_full = bar;                   // [kQStages] by item
  uint64_t* q_empty = bar + C::kQStages;    // [kQStages]
  uint64_t* k_full = bar + 2 * C::kQStages;
  uint64_t* k_empty = k_full + C::kKStages;
  uint64_t* v_full = k_empty + C::kKStages;
  uint64_t* v_empty = v_full + C::kVStages;
  uint64_t* s_full = v_empty + C::kVStages;
  uint64_t* buf_free = s_full + kSBufs;  // S/P buffer reusable: PV of its last tile completed
  uint64_t* p_full = buf_free + kSBufs;
  uint64_t* o_ready = p_full + kSBufs;  // [2]
  uint64_t* o_free = o_ready + 2;
  uint64_t* drain = o_free + 1;     // [0] S issuer, [1] PV issuer
  // The column-sum rendezvous barriers take one arrival per warp: the warp's lanes write
  // shared memory, __syncwarp() orders those writes before lane 0's (release) arrival.
  uint64_t* cs_full = drain + 2;    // dense: [parity * 2 + kb] column sums of quads 1-3 posted (3)
  uint64_t* cs_free = cs_full + 4;  // dense: [parity * 2 + kb] slots read by quad 0 (1)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(cs_free + 4);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  uint32_t* pv_seen = reinterpret_cast<uint32_t*>(abort_flag + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    if (!kDense) prefetch_tensormap(&omap);
    // sparse: a Q buffer is free once the item's S MMAs have completed and each softmax
    // warp's O store has read its staged box out of it
    for (int s = 0; s < C::kQStages; ++s) { mbar_init(&q_full[s], 1); mbar_init(&q_empty[s], kDense ? 1 : 1 + kSoftmaxWarps); }
    for (int s = 0; s < C::kKStages; ++s) { mbar_init(&k_full[s], 1); mbar_init(&k_empty[s], 1); }
    for (int s = 0; s < C::kVStages; ++s) { mbar_init(&v_full[s], 1); mbar_init(&v_empty[s], 1); }
    for (int s = 0; s < kSBufs; ++s) { mbar_init(&s_full[s], 1); mbar_init(&buf_free[s], 1); }
    for (int s = 0; s < kSBufs; ++s) mbar_init(&p_full[s], kSoftmaxWarps);
    mbar_init(&o_ready[0], 1);
    mbar_init(&o_ready[1], 1);
    *pv_seen = 0u;
    mbar_init(o_free, kSoftmaxWarps);
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
    for (int s = 0; s < 4; ++s) {
      mbar_init(&cs_full[s], 3);
      mbar_init(&cs_free[s], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_o = tmem + kTmemO;
  const int G = p.Hq / p.Hkv;

  if (warp < kFirstSoftmaxWarp) {
    // warpgroup 0: TMA producer, S issuer, PV issuer, PV-completion tracker
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegsLow));
    if (warp == 0) {
      // ------------------------------------------------------------ TMA producer (Q, K, V)
      if (lane == 0) {
        uint32_t gi = 0, kt = 0, vt = 0;
        bool ok = true;
        // L2 priorities: K / V tiles are re-read by the other items of their head (kept),
        // Q is read once per item (streamed); O is stored evict-first as well
        const uint64_t pol_keep = l2_evict_last_policy(), pol_stream = l2_evict_first_policy();
        // Tile counts are read one item ahead and list entries one tile ahead, so no list
        // read sits between a free stage and its TMA issue.
        int T_next = static_cast<int64_t>(blockIdx.x) < p.items ? item_tiles<kDense>(p, blockIdx.x) : 0;
        for (int64_t item = blockIdx.x; item < p.items && ok; item += gridDim.x) {
          const int T = T_next;
          if (item + gridDim.x < p.items) T_next = item_tiles<kDense>(p, item + gridDim.x);
          if (T == 0) continue;
          const uint32_t it = static_cast<uint32_t>(item);
          const int bh = static_cast<int>(it / static_cast<uint32_t>(p.P));
          const int pr = static_cast<int>(it - static_cast<uint32_t>(bh) * static_cast<uint32_t>(p.P));
          const int b = bh / p.Hq, h = bh % p.Hq, hk = h / G;
          const uint32_t* ul = p.ulist + item * p.stride;
          uint32_t e0 = 0u, e1 = 0u;
          if constexpr (!kDense) {
            e0 = ld_nc_u32(ul);
            e1 = ld_nc_u32(ul + 1);
          }
          const int qs = static_cast<int>(gi % C::kQStages);
          if (!mbar_wait(&q_empty[qs], ((gi / C::kQStages) & 1) ^ 1, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&q_full[qs], C::kQBytes);
  #pragma unroll
          for (int a = 0; a < C::kAtoms; ++a)
            tma_load_4d_hint(sQ + qs * C::kQBytes + a * 16384, &qmap, &q_full[qs], 64 * a, 128 * pr, h, b, pol_stream);
          ++gi;
          for (int t = 0; t < T; ++t) {
            const int j0 = kDense ? 2 * t : static_cast<int>(e0 & kIdxMask);
            const int j1 = kDense ? 2 * t + 1 : static_cast<int>(e1 & kIdxMask);
            if constexpr (!kDense) {
              if (t + 1 < T) {
                e0 = ld_nc_u32(ul + 2 * t + 2);
                e1 = ld_nc_u32(ul + 2 * t + 3);
              }
            }
            const int ks = kt % C::kKStages;
            if constexpr (Signals<C>::kKOnSFull) {
              // K stage ks is free once S(kt - kKStages), its last reader, has completed
              if (kt >= static_cast<uint32_t>(C::kKStages)) {
                const uint32_t kd = kt - C::kKStages;
                if (!mbar_wait(&s_full[kd % kSBufs], (kd / kSBufs) & 1, abort_flag)) { ok = false; break; }
              }
            } else {
              if (!mbar_wait(&k_empty[ks], ((kt / C::kKStages) & 1) ^ 1, abort_flag)) { ok = false; break; }
            }
            mbar_arrive_expect_tx(&k_full[ks], C::kKBytes);
            uint8_t* dk = sK + ks * C::kKBytes;
  #pragma unroll
            for (int a = 0; a < C::kAtoms; ++a) {
              tma_load_4d_hint(dk + a * 16384, &kmap, &k_full[ks], 64 * a, 64 * j0, hk, b, pol_keep);
              tma_load_4d_hint(dk + a * 16384 + 8192, &kmap, &k_full[ks], 64 * a, 64 * j1, hk, b, pol_keep);
            }
            ++kt;
            const int vs = vt % C::kVStages;
            // V stage vs is free once PV(vt - kVStages) has completed
            uint64_t* v_free = Signals<C>::kPvOneCommit ? &buf_free[vs] : &v_empty[vs];
            if (!mbar_wait(v_free, ((vt / C::kVStages) & 1) ^ 1, abort_flag)) { ok = false; break; }
            mbar_arrive_expect_tx(&v_full[vs], C::kVBytes);
            uint8_t* dv = sV + vs * C::kVBytes;
  #pragma unroll
            for (int a = 0; a < C::kAtoms; ++a) {
              tma_load_4d_hint(dv + a * 16384, &vmap, &v_full[vs], 64 * a, 64 * j0, hk, b, pol_keep);
              tma_load_4d_hint(dv + a * 16384 + 8192, &vmap, &v_full[vs], 64 * a, 64 * j1, hk, b, pol_keep);
            }
            ++vt;
          }
        }
        if (!ok) {
          // bounded drain of the loads this thread may still have in flight
          for (int s = 0; s < C::kKStages; ++s) (void)mbar_wait(&k_full[s], ((kt + s) / C::kKStages) & 1, nullptr);
        }
      }
      __syncwarp();
    } else if (warp == 1) {
      // ------------------------------------------------------------ S = Q K^T issuer
      if (lane == 0) {
        constexpr uint32_t idesc_s = make_idesc_f16(128, 128, kBF16 ? 1 : 0, 0, 0);
        // Descriptors are built once; per stage and K step only the 14-bit start-address
        // field (16-byte units, shared memory < 256 KB so it never carries) is advanced.
        const uint64_t dQ = make_smem_desc(smem_u32(sQ), 16, 1024, 2);
        const uint64_t dK = make_smem_desc(smem_u32(sK), 16, 1024, 2);
        uint32_t gi = 0, kt = 0, gt = 0;
        bool ok = true;
        int T_next = static_cast<int64_t>(blockIdx.x) < p.items ? item_tiles<kDense>(p, blockIdx.x) : 0;
        for (int64_t item = blockIdx.x; item < p.items && ok; item += gridDim.x) {
          const int T = T_next;
          if (item + gridDim.x < p.items) T_next = item_tiles<kDense>(p, item + gridDim.x);
          if (T == 0) continue;
          const int qs = static_cast<int>(gi % C::kQStages);
          if (!mbar_wait(&q_full[qs], (gi / C::kQStages) & 1, abort_flag)) { ok = false; break; }
          tc_fence_after_sync();
          const uint64_t dq = dQ + static_cast<uint64_t>((qs * C::kQBytes) >> 4);
          for (int t = 0; t < T; ++t) {
            // S(g) = Q K(g)^T into buffer g % 3 once PV(g - 3) (which read P(g - 3) there)
            // has completed; Q and K from shared memory (K-major)
            const uint32_t g = gt + t, buf = g % kSBufs;
            const int ks = kt % C::kKStages;
            // K lands well ahead; the buffer's release (PV(g - 3)) is the event waited on last
            if (!mbar_wait(&k_full[ks], (kt / C::kKStages) & 1, abort_flag) ||
                !mbar_wait(&buf_free[buf], ((g / kSBufs) & 1) ^ 1, abort_flag)) { ok = false; break; }
            tc_fence_after_sync();
            const uint64_t dk = dK + static_cast<uint64_t>((ks * C::kKBytes) >> 4);
            const uint32_t d_s = tmem + buf * 128;
  #pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint64_t off = (kk >> 2) * (16384 >> 4) + (kk & 3) * (32 >> 4);
              mma_f16_ss(d_s, dq + off, dk + off, idesc_s, kk > 0 ? 1u : 0u);
            }
            if constexpr (!Signals<C>::kKOnSFull) mma_commit(&k_empty[ks]);
            mma_commit(&s_full[buf]);
            ++kt;
          }
          if (!ok) break;
          mma_commit(&q_empty[qs]);
          gt += T;
          ++gi;
        }
        if (gi > 0) {
          mma_commit(&drain[0]);
          (void)mbar_wait(&drain[0], 0, nullptr);
        }
      }
      __syncwarp();
    } else if (warp == kPvWarp) {
      // ------------------------------------------------------------ O += P V issuer
      if (lane == 0) {
        constexpr uint32_t idesc_o = make_idesc_f16(128, D, kBF16 ? 1 : 0, 0, 1);
        const uint64_t dV = make_smem_desc(smem_u32(sV), 16384, 1024, 2);
        uint32_t gi = 0, vt = 0, gt = 0;
        bool ok = true;
        int T_next = static_cast<int64_t>(blockIdx.x) < p.items ? item_tiles<kDense>(p, blockIdx.x) : 0;
        for (int64_t item = blockIdx.x; item < p.items && ok; item += gridDim.x) {
          const int T = T_next;
          if (item + gridDim.x < p.items) T_next = item_tiles<kDense>(p, item + gridDim.x);
          if (T == 0) continue;
          for (int t = 0; t < T; ++t) {
            // P from TMEM (in its S buffer), V from shared memory (MN-major)
            const uint32_t g = gt + t;
            const int vs = vt % C::kVStages;
            // Everything that is normally ready early is waited on first, so that P(g), the
            // event on the critical path, is the last wait before the issue.
            if (!mbar_wait(&v_full[vs], (vt / C::kVStages) & 1, abort_flag)) { ok = false; break; }
            if (t == 0 && gi > 0 && !mbar_wait(o_free, (gi - 1) & 1, abort_flag)) { ok = false; break; }
            // the tracker must have taken the previous phase of the completion barrier PV(g) will
            // signal: PV(g - 3) on buf_free[g % 3], or PV(g - 2) on o_ready[g & 1]
            if constexpr (Signals<C>::kPvOneCommit) {
              if (g >= 3 && !counter_wait(pv_seen, g - 2, abort_flag)) { ok = false; break; }
            } else {
              if (g >= 2 && !counter_wait(pv_seen, g - 1, abort_flag)) { ok = false; break; }
            }
            if (!mbar_wait(&p_full[g % kSBufs], (g / kSBufs) & 1, abort_flag)) { ok = false; break; }
            tc_fence_after_sync();
            const uint64_t dv = dV + static_cast<uint64_t>((vs * C::kVBytes) >> 4);
            const uint32_t pt = tmem + (g % kSBufs) * 128;
  #pragma unroll
            for (int kk = 0; kk < 8; ++kk)
              mma_f16_ts(tmem_o, pt + (kk >> 2) * 64 + (kk & 3) * 8,
                         dv + static_cast<uint64_t>(kk * (2048 >> 4)), idesc_o, (t > 0 || kk > 0) ? 1u : 0u);
            if constexpr (!Signals<C>::kPvOneCommit) {
              mma_commit(&v_empty[vs]);
              mma_commit(&o_ready[g & 1]);
            }
            mma_commit(&buf_free[g % kSBufs]);
            ++vt;
          }
          if (!ok) break;
          gt += T;
          ++gi;
        }
        if (gi > 0) {
          mma_commit(&drain[1]);
          (void)mbar_wait(&drain[1], 0, nullptr);
        }
      }
      __syncwarp();
    } else if (warp == kTrackWarp) {
      if (lane == 0) {
        uint32_t gt = 0;
        bool ok = true;
        int T_next = static_cast<int64_t>(blockIdx.x) < p.items ? item_tiles<kDense>(p, blockIdx.x) : 0;
        for (int64_t item = blockIdx.x; item < p.items && ok; item += gridDim.x) {
          const int T = T_next;
          if (item + gridDim.x < p.items) T_next = item_tiles<kDense>(p, item + gridDim.x);
          for (int t = 0; t < T; ++t) {
            const uint32_t g = gt + t;
            const bool okt = Signals<C>::kPvOneCommit ? mbar_wait(&buf_free[g % kSBufs], (g / kSBufs) & 1, abort_flag)
                                                       : mbar_wait(&o_ready[g & 1], (g >> 1) & 1, abort_flag);
            if (!okt) { ok = false; break; }
            counter_store(pv_seen, g + 1);
          }
          gt += T;
        }
      }
      __syncwarp();
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegsHigh));
    // ------------------------------------------------------------ softmax + epilogue
    // Warp w (4..11) owns TMEM lane quadrant w & 3 (rows 32*(w&3) .. +31 of the 128-row
    // tile) and key block kb = (w - 4) / 4 of every 128-key tile (columns 64*kb .. +63).
    // The two threads of a row swap partial row maxima through shared memory
    // (double-buffered by exchange parity) under a 64-thread named barrier.
    const int quad = warp & 3;
    const int kb = (warp - kFirstSoftmaxWarp) >> 2;
    const int r = quad * 32 + lane;
    const int half = r >> 6;
    // Row-pair exchanges (tile maxima, final row sums) alternate between two buffers; `xc`
    // counts this thread's exchanges. A buffer is rewritten two exchanges later, after the
    // partner has passed the exchange in between, i.e. after it has read the buffer. The
    // pair meets at named barrier 1 + quad (64 threads). A warp that leaves the loops
    // early (a bounded wait gave up, which also raised the CTA abort flag) arrives at that
    // barrier once on its way out, so a partner blocked there is released, sees the flag
    // and leaves too; the barrier is never waited on without a way out.
    const int pair_bar = 1 + quad;
    uint32_t xc = 0;
    bool alive = true;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    constexpr int kHalfD = D / 2;
    using InT = typename std::conditional<kBF16, __nv_bfloat16, __half>::type;
    uint32_t gt = 0;
    // The tile count and this thread's first list entry of each item are loaded one item
    // ahead, so their global-memory latency is not paid at the item boundary.
    int T_next = 0;
    uint32_t e_first_next = 0u;
    if (static_cast<int64_t>(blockIdx.x) < p.items) {
      T_next = item_tiles<kDense>(p, blockIdx.x);
      e_first_next = kDense ? item_entry<kDense>(nullptr, 0, kb) : ld_nc_u32(p.ulist + static_cast<int64_t>(blockIdx.x) * p.stride + kb);
    }
    int dense_tiles_seen = 0;  // dense + column sums: key tiles touched in this CTA's private buffer
    uint32_t gq = 0;   // items with tiles so far (their Q buffers alternate like the producer's)
    int pend_q = -1;   // sparse: Q buffer holding this warp's O box until its store has read it
    for (int64_t item = blockIdx.x; item < p.items; item += gridDim.x) {
      const int T = T_next;
      const uint32_t e_first = e_first_next;
      {
        const int64_t nitem = item + gridDim.x;
        if (nitem < p.items) {
          T_next = item_tiles<kDense>(p, nitem);
          e_first_next = kDense ? item_entry<kDense>(nullptr, 0, kb) : ld_nc_u32(p.ulist + nitem * p.stride + kb);
        }
      }
      const uint32_t it = static_cast<uint32_t>(item);
      const int bh = static_cast<int>(it / static_cast<uint32_t>(p.P));
      const int pr = static_cast<int>(it - static_cast<uint32_t>(bh) * static_cast<uint32_t>(p.P));
      const int b = bh / p.Hq, h = bh % p.Hq;
      const int row = 128 * pr + r;
      const int64_t ooff = b * p.o_s0 + h * p.o_s1 + static_cast<int64_t>(row) * p.o_s2;
      InT* orow = reinterpret_cast<InT*>(p.out) + ooff + kb * kHalfD;
      if (T == 0) {
        if (row < p.Nq) {
#pragma unroll
          for (int c = 0; c < kHalfD; c += 8) *reinterpret_cast<uint4*>(orow + c) = make_uint4(0, 0, 0, 0);
          if (p.lse && kb == 0) p.lse[static_cast<int64_t>(bh) * p.Nq + row] = -INFINITY;
        }
        continue;
      }
      const uint32_t* ul = kDense ? nullptr : p.ulist + item * p.stride;
      float m_run = -INFINITY, l = 0.f;
      float m_exact = -INFINITY;  // dense column scores: exact running max (log2 units)
      bool ok = true;
      uint32_t e_next = e_first;
      if constexpr (!kDense) {
        // hand the previous item's Q buffer back to the producer once this warp's O store
        // has read its staged box (kept out of the tile loop, whose code it would slow)
        if (pend_q >= 0) {
          if (lane == 0) {
            bulk_wait_read_all();
            mbar_arrive(&q_empty[pend_q]);
          }
          pend_q = -1;
        }
      }
      for (int t = 0; t < T; ++t) {
        const uint32_t g = gt + t, buf = g % kSBufs;
        const uint32_t e = e_next;
        if (t + 1 < T) e_next = item_entry<kDense>(ul, t + 1, kb);
        const int j = static_cast<int>(e & kIdxMask);
        int lim = ((e >> (30 + half)) & 1u) ? min(64, p.Nk - 64 * j) : 0;
        if (p.causal) lim = min(lim, row - 64 * j + 1);
        lim = max(lim, 0);
        const bool any_live = __any_sync(0xffffffffu, lim > 0);
        const bool all_full = __all_sync(0xffffffffu, lim >= 64);
        const uint32_t scol = tmem + lane_addr + buf * 128 + kb * 64;  // S in, P out

        const bool okw = mbar_wait(&s_full[buf], (g / kSBufs) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, okw)) { ok = false; break; }
        tc_fence_after_sync();
        uint32_t s[64];
        if (any_live) {
          tmem_ld32(scol, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
          tmem_ld32(scol + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
          tmem_wait_ld();
        }
        // row max over this thread's 64 keys: eight independent chains, then a tree
        float mx8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mx8[u] = -INFINITY;
        if (all_full) {
#pragma unroll
          for (int c = 0; c < 64; c += 2)
            mx8[(c >> 1) & 7] = fmax3(mx8[(c >> 1) & 7], __uint_as_float(s[c]), __uint_as_float(s[c + 1]));
        } else if (any_live) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c < lim) mx8[c & 7] = fmaxf(mx8[c & 7], __uint_as_float(s[c]));
        }
        const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        float* xs = xchg + (xc & 1u) * 256;
        xs[kb * 128 + r] = mx;
        named_bar_sync(pair_bar, 64);
        ++xc;
        if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(abort_flag) != 0)) { ok = false; break; }
        const float m_tile = fmaxf(mx, xs[(kb ^ 1) * 128 + r]) * p.scale_log2;  // -inf stays -inf
        float alpha = 1.f;
        bool need = false;
        if (m_run == -INFINITY) {
          m_run = m_tile;
        } else if (m_tile > m_run + kRescaleThreshold) {
          alpha = ex2(m_run - m_tile);
          need = true;
          m_run = m_tile;
          l *= alpha;
        }
        // P overwrites this thread's own S columns (already in registers); PV(g) reads
        // it from there, and S(g + 3) waits for that PV before reusing the buffer.
        float ls[4] = {0.f, 0.f, 0.f, 0.f};  // independent partial row sums
        if (all_full) {
          // two keys per instruction for the scale-and-shift and the running sums
          const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
          const float2 nm2 = make_float2(-m_run, -m_run);
          float2 acc2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t w[16];
#pragma unroll
            for (int y = 0; y < 16; ++y) {
              const int c = 32 * hh + 2 * y;
              const float2 x2 = ffma2(make_float2(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), sc2, nm2);
              const float p0 = ex2(x2.x), p1 = ex2(x2.y);
              acc2[y & 1] = fadd2(acc2[y & 1], make_float2(p0, p1));
              w[y] = pack2<kBF16>(p0, p1);
              if constexpr (kDense) {
                s[c] = __float_as_uint(p0);
                s[c + 1] = __float_as_uint(p1);
              }
            }
            tmem_st16(scol + 16 * hh, w);
          }
          ls[0] = acc2[0].x;
          ls[1] = acc2[0].y;
          ls[2] = acc2[1].x;
          ls[3] = acc2[1].y;
        } else if (any_live) {
          const bool live = m_run != -INFINITY;
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t w[16];
#pragma unroll
            for (int y = 0; y < 16; ++y) {
              const int c = 32 * hh + 2 * y;
              const float p0 = (c < lim && live) ? ex2(fmaf(__uint_as_float(s[c]), p.scale_log2, -m_run)) : 0.f;
              const float p1 = (c + 1 < lim && live) ? ex2(fmaf(__uint_as_float(s[c + 1]), p.scale_log2, -m_run)) : 0.f;
              ls[y & 3] += p0 + p1;
              w[y] = pack2<kBF16>(p0, p1);
              if constexpr (kDense) {
                s[c] = __float_as_uint(p0);
                s[c + 1] = __float_as_uint(p1);
              }
            }
            tmem_st16(scol + 16 * hh, w);
          }
        } else {
          uint32_t w[16];
#pragma unroll
          for (int y = 0; y < 16; ++y) w[y] = 0u;
          tmem_st16(scol, w);
          tmem_st16(scol + 16, w);
          if constexpr (kDense) {
#pragma unroll
            for (int c = 0; c < 64; ++c) s[c] = 0u;
          }
        }
        tmem_wait_st();
        l += (ls[0] + ls[1]) + (ls[2] + ls[3]);
        // O may only be rescaled once PV(g - 1) has finished accumulating into it. The
        // wait sits at the end of the tile: PV(g - 1) ran while this tile's exps did.
        if (__any_sync(0xffffffffu, need)) {
          const bool okp = counter_wait(pv_seen, g, abort_flag);
          if (!__all_sync(0xffffffffu, okp)) { ok = false; break; }
          tc_fence_after_sync();
#pragma unroll
          for (int c = kb * kHalfD; c < (kb + 1) * kHalfD; c += 16) {
            uint32_t o[16];
            tmem_ld16(tmem_o + lane_addr + c, o);
            tmem_wait_ld();
#pragma unroll
            for (int x = 0; x < 16; ++x) o[x] = __float_as_uint(__uint_as_float(o[x]) * alpha);
            tmem_st16(tmem_o + lane_addr + c, o);
          }
          tmem_wait_st();
        }
        tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[buf]);
        if constexpr (kDense) {
          if (p.colsum != nullptr) {
            // Column scores as the reference accumulates them (after P is released, so the PV
            // and the next S MMAs do not wait for this work): exp(s - m) summed over the
            // rows, with m the exact running row max after this tile. P above is relative to
            // the lazily updated m_run, so each row's terms are scaled by 2^(m_run - m_exact);
            // rows past the query end add nothing.
            m_exact = fmaxf(m_exact, m_tile);
            const float cq = (row < p.Nq && m_exact != -INFINITY) ? ex2(m_run - m_exact) : 0.f;
            float v[64];
#pragma unroll
            for (int c = 0; c < 64; ++c) v[c] = __uint_as_float(s[c]) * cq;
            // sum over the warp's 32 rows: five halving exchange steps leave lane l with
            // the sums of columns 2l and 2l + 1
#pragma unroll
            for (int stp = 0; stp < 5; ++stp) {
              const int hw = 32 >> stp, off = 16 >> stp;
              const bool up = (lane & off) != 0;
#pragma unroll
              for (int i = 0; i < hw; ++i) {
                const float send = up ? v[i] : v[i + hw];
                const float keep = up ? v[i + hw] : v[i];
                v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
              }
            }
            // the four row quadrants of this key block meet in shared memory; quadrant 0
            // adds their sum to this CTA's private column buffer
            const int sb = static_cast<int>(g & 1u) * 2 + kb;
            float2* slot = colslots + sb * 128;
            if (quad != 0) {
              const bool okf = mbar_wait(&cs_free[sb], ((g >> 1) & 1u) ^ 1u, abort_flag);
              if (!__all_sync(0xffffffffu, okf)) { ok = false; break; }
              slot[quad * 32 + lane] = make_float2(v[0], v[1]);
              __syncwarp();
              if (lane == 0) mbar_arrive(&cs_full[sb]);
            } else {
              const bool okf = mbar_wait(&cs_full[sb], (g >> 1) & 1u, abort_flag);
              if (!__all_sync(0xffffffffu, okf)) { ok = false; break; }
              const float2 a1 = slot[32 + lane], a2 = slot[64 + lane], a3 = slot[96 + lane];
              __syncwarp();
              if (lane == 0) mbar_arrive(&cs_free[sb]);
              float2* pp = reinterpret_cast<float2*>(p.partial + static_cast<int64_t>(blockIdx.x) * p.pstride +
                                                     128 * t + 64 * kb + 2 * lane);
              atomicAdd(pp, make_float2((v[0] + a1.x) + (a2.x + a3.x), (v[1] + a1.y) + (a2.y + a3.y)));
            }
          }
        }

      }
      if (!ok) {
        alive = false;
        break;
      }
      // ---- epilogue: O / l, each thread writes its half of the row's D columns
      const uint32_t glast = gt + T - 1;
      const bool oko = counter_wait(pv_seen, glast + 1, abort_flag);
      if (!__all_sync(0xffffffffu, oko)) {
        alive = false;
        break;
      }
      tc_fence_after_sync();
      float* xs = xchg + (xc & 1u) * 256;
      xs[kb * 128 + r] = l;
      named_bar_sync(pair_bar, 64);
      ++xc;
      if (__any_sync(0xffffffffu, *reinterpret_cast<volatile int*>(abort_flag) != 0)) { alive = false; break; }
      const float l_row = l + xs[(kb ^ 1) * 128 + r];
      const float inv = l_row > 0.f ? 1.f / l_row : 0.f;
      // O is read into registers and released at once (the next item's first PV may then
      // overwrite it) before the conversion and the global stores
      uint32_t o[kHalfD];
#pragma unroll
      for (int c = 0; c < kHalfD; c += 16)
        tmem_ld16(tmem_o + lane_addr + kb * kHalfD + c, *reinterpret_cast<uint32_t(*)[16]>(&o[c]));
      tmem_wait_ld();
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
      if constexpr (kDense) {
        if (row < p.Nq) {
#pragma unroll
          for (int c = 0; c < kHalfD; c += 8) {
            uint32_t wv[4];
#pragma unroll
            for (int y = 0; y < 4; ++y)
              wv[y] = pack2<kBF16>(__uint_as_float(o[c + 2 * y]) * inv, __uint_as_float(o[c + 2 * y + 1]) * inv);
            *reinterpret_cast<uint4*>(orow + c) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
          }
        }
      } else {
        // O / l goes through this item's Q buffer, whose last reader, S of the item's last
        // tile, has completed (this warp waited for it): the warp stages its 32 rows x D/2
        // columns in the output tensor map's swizzled box layout (16-byte chunk c of row x
        // at chunk c ^ (x & 7) for 128-byte rows, c ^ ((x >> 1) & 3) for 64-byte rows) and
        // lane 0 writes the box with one TMA store; rows past the sequence end are clipped
        // by the tensor map. Coalesced, and the warp moves on without waiting for it.
        constexpr int kRowBytes = kHalfD * 2;
        const int qs = static_cast<int>(gq % C::kQStages);
        uint8_t* wbox = sQ + qs * C::kQBytes + (quad + 4 * kb) * C::kWarpOBytes;
        const int swz = kRowBytes == 128 ? (lane & 7) : ((lane >> 1) & 3);
#pragma unroll
        for (int c = 0; c < kHalfD / 8; ++c) {
          uint32_t wv[4];
#pragma unroll
          for (int y = 0; y < 4; ++y)
            wv[y] = pack2<kBF16>(__uint_as_float(o[8 * c + 2 * y]) * inv, __uint_as_float(o[8 * c + 2 * y + 1]) * inv);
          *reinterpret_cast<uint4*>(wbox + lane * kRowBytes + 16 * (c ^ swz)) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        const int row0 = 128 * pr + 32 * quad;
        if (lane == 0 && row0 < p.Nq) {
          tma_store_4d_hint(&omap, wbox, kb * kHalfD, row0, h, b, l2_evict_first_policy());
          bulk_commit_group();
        }
        pend_q = qs;
      }
      ++gq;
      if (row < p.Nq && p.lse && kb == 0)
        p.lse[static_cast<int64_t>(bh) * p.Nq + row] = l_row > 0.f ? (m_run + __log2f(l_row)) * kLn2 : -INFINITY;
      if constexpr (kDense) {
        // Flush this CTA's private column sums into the caller's scores when the next item
        // belongs to another (b, h) (or there is none), and clear them.
        if (p.colsum != nullptr && quad == 0) {
          dense_tiles_seen = max(dense_tiles_seen, T);
          const int64_t nitem = item + gridDim.x;
          if (nitem >= p.items || nitem / p.P != item / p.P) {
            float* part = p.partial + static_cast<int64_t>(blockIdx.x) * p.pstride;
            float* dst = p.colsum + b * p.cs_s0 + h * p.cs_s1;
            for (int t2 = 0; t2 < dense_tiles_seen; ++t2) {
              const int key = 128 * t2 + 64 * kb + 2 * lane;
              float2* pp = reinterpret_cast<float2*>(part + key);
              const float2 val = *pp;
              if (key < p.Nk) atomicAdd(dst + key, val.x);
              if (key + 1 < p.Nk) atomicAdd(dst + key + 1, val.y);
              *pp = make_float2(0.f, 0.f);
            }
            dense_tiles_seen = 0;
          }
        }
      }
      gt += T;
    }
    if (!alive) named_bar_arrive(pair_bar, 64);  // release a partner blocked at the pair barrier
    if (!kDense && lane == 0) bulk_wait_all();  // the staged boxes stay valid until stored
  }
  tc_fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ CUDA-core kernel
struct SimtParams {
  const void* q;
  const void* k;
  const void* v;
  const int32_t* kv_idx;
  const int32_t* kv_num;
  void* out;
  float* lse;
  int32_t Hq, Hkv, N, M, bs, D, kmax;
  int64_t qs[3], ks[3], vs[3], os[3];
  float scale;
  int32_t causal;
};

template <typename T>
__device__ __forceinline__ float ld_elem(const void* p, int64_t i) {
  if constexpr (std::is_same<T, float>::value) return static_cast<const float*>(p)[i];
  else if constexpr (std::is_same<T, __half>::value) return __half2float(static_cast<const __half*>(p)[i]);
  else return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
}

template <typename T>
__device__ __forceinline__ void st_elem(void* p, int64_t i, float v) {
  if constexpr (std::is_same<T, float>::value) static_cast<float*>(p)[i] = v;
  else if constexpr (std::is_same<T, __half>::value) static_cast<__half*>(p)[i] = __float2half_rn(v);
  else static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
}

// grid (M, Hq, B), block 128 threads; thread t owns query row i*bs + t (t < bs).
template <typename T>
__global__ void __launch_bounds__(128) attn_simt_kernel(const SimtParams p) {
  extern __shared__ float sm[];
  const int D = p.D, bs = p.bs;
  float* sk = sm;                  // [bs][D+1]
  float* sv = sk + bs * (D + 1);   // [bs][D]
  float* sq = sv + bs * D;         // [bs][D+1]
  const int i = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (p.Hq / p.Hkv);
  const int t = threadIdx.x;
  const int row = i * bs + t;
  for (int e = t; e < bs * D; e += blockDim.x) {
    const int rr = e / D, d = e % D;
    const int n = i * bs + rr;
    sq[rr * (D + 1) + d] = n < p.N ? ld_elem<T>(p.q, b * p.qs[0] + h * p.qs[1] + n * p.qs[2] + d) : 0.f;
  }
  float o[128];
#pragma unroll
  for (int d = 0; d < 128; ++d) o[d] = 0.f;
  float m = -INFINITY, l = 0.f;
  const int64_t lrow = (static_cast<int64_t>(b) * p.Hq + h) * p.M + i;
  const int nb = min(max(p.kv_num[lrow], 0), p.kmax);
  for (int x = 0; x < nb; ++x) {
    const int j = p.kv_idx[lrow * p.kmax + x];
    __syncthreads();
    if (j < 0 || j >= p.M) continue;
    for (int e = t; e < bs * D; e += blockDim.x) {
      const int rr = e / D, d = e % D;
      const int n = j * bs + rr;
      const bool in = n < p.N;
      sk[rr * (D + 1) + d] = in ? ld_elem<T>(p.k, b * p.ks[0] + hk * p.ks[1] + n * p.ks[2] + d) : 0.f;
      sv[rr * D + d] = in ? ld_elem<T>(p.v, b * p.vs[0] + hk * p.vs[1] + n * p.vs[2] + d) : 0.f;
    }
    __syncthreads();
    if (t < bs && row < p.N) {
      for (int kk = 0; kk < bs; ++kk) {
        const int kp = j * bs + kk;
        if (kp >= p.N || (p.causal && kp > row)) continue;
        float s = 0.f;
        for (int d = 0; d < D; ++d) s = fmaf(sq[t * (D + 1) + d], sk[kk * (D + 1) + d], s);
        s *= p.scale;
        const float mn = fmaxf(m, s);
        const float corr = expf(m - mn);
        const float pe = expf(s - mn);
        l = l * corr + pe;
#pragma unroll
        for (int d = 0; d < 128; ++d)
          if (d < D) o[d] = o[d] * corr + pe * sv[kk * D + d];
        m = mn;
      }
    }
  }
  if (t < bs && row < p.N) {
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int d = 0; d < 128; ++d)
      if (d < D) st_elem<T>(p.out, b * p.os[0] + h * p.os[1] + static_cast<int64_t>(row) * p.os[2] + d, o[d] * inv);
    if (p.lse) p.lse[(static_cast<int64_t>(b) * p.Hq + h) * p.N + row] = l > 0.f ? m + logf(l) : -INFINITY;
  }
}

struct WsLayout {
  size_t ulist_off, ntiles_off, total;
  int32_t stride;
  int64_t items;
};

static WsLayout ws_layout(int64_t B, int64_t Hq, int64_t N, int64_t bs, int64_t kmax) {
  WsLayout L{};
  const int64_t M = (N + bs - 1) / bs;
  const int64_t P = (M + 1) / 2;
  L.items = B * Hq * P;
  L.stride = static_cast<int32_t>(2 * kmax + 2);
  L.ulist_off = 0;
  const size_t ubytes = static_cast<size_t>(L.items) * L.stride * 4;
  L.ntiles_off = (ubytes + 255) / 256 * 256;
  L.total = L.ntiles_off + (static_cast<size_t>(L.items) * 4 + 255) / 256 * 256;
  return L;
}

static bool use_tensor_cores(int dtype, int64_t D, int64_t bs) {
  return (dtype == CAB_DTYPE_BF16 || dtype == CAB_DTYPE_F16) && bs == 64 && (D == 64 || D == 128);
}

template <int D, bool kBF16, bool kDense>
static int launch_tc(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const CUtensorMap& om,
                     const Params& p, int grid, cudaStream_t st) {
  auto kern = attn_tc_kernel<D, kBF16, kDense>;
  {
    // The softmax warpgroups raise their register limit with setmaxnreg from the pool the
    // CTA was launched with; a build that gave the kernel fewer registers would make that
    // wait forever, so it is refused here.
    static const int regs = [&] {
      cudaFuncAttributes fa{};
      return cudaFuncGetAttributes(&fa, kern) == cudaSuccess ? fa.numRegs : -1;
    }();
    if (regs < kRegsNeeded)
      return fail(CAB_ERR_LAUNCH, "attn_tc_kernel built with %d registers per thread, needs %d", regs, kRegsNeeded);
  }
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<D, kDense>::kSmem);
  kern<<<grid, kAttnThreads, Cfg<D, kDense>::kSmem, st>>>(qm, km, vm, om, p);
  return check_launch("attn_tc_kernel");
}

// Q / K / V / O tensor map over [B, H, rows, D] with {b, h, n} strides in elements; the
// box is box_cols x box_rows (64 columns = one 128-byte swizzle atom for Q, K and V).
static int attn_tensor_map(CUtensorMap* m, const void* ptr, int64_t B, int64_t H, int64_t rows, int64_t D,
                           const int64_t* s, size_t es, int dtype, uint32_t box_rows, uint32_t box_cols = 64,
                           CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  uint64_t dims[4] = {static_cast<uint64_t>(D), static_cast<uint64_t>(rows), static_cast<uint64_t>(H),
                      static_cast<uint64_t>(B)};
  uint64_t str[3] = {static_cast<uint64_t>(s[2]) * es, static_cast<uint64_t>(s[1]) * es,
                     static_cast<uint64_t>(s[0]) * es};
  uint32_t box[4] = {box_cols, box_rows, 1, 1};
  return make_tensor_map(m, tma_type(dtype), 4, ptr, dims, str, box, swz);
}

// Dense (flash) forward: CTAs in the launch and the private column-buffer stride.
struct FlashLayout {
  int grid;
  int64_t items, Tk, pstride;
  size_t partial_bytes;
};

static FlashLayout flash_layout(int64_t B, int64_t Hq, int64_t Nq, int64_t Nk) {
  FlashLayout L{};
  L.items = B * Hq * ((Nq + 127) / 128);
  L.Tk = (Nk + 127) / 128;
  L.pstride = L.Tk * 128;
  L.grid = static_cast<int>(std::min<int64_t>(L.items, current_sm_count()));
  L.partial_bytes = static_cast<size_t>(L.grid) * L.pstride * sizeof(float);
  return L;
}

}  // namespace attn
}  // namespace cab

using namespace cab;

extern "C" int cab_sparse_attn_workspace_size(int64_t B, int64_t Hq, int64_t N, int64_t D, int64_t block_size,
                                              int64_t kmax, int dtype, size_t* bytes) {
  if (!bytes) return fail(CAB_ERR_INVALID_ARG, "attn_workspace_size: NULL output");
  if (B <= 0 || Hq <= 0 || N <= 0 || block_size <= 0 || kmax <= 0)
    return fail(CAB_ERR_INVALID_ARG, "attn_workspace_size: non-positive size");
  *bytes = attn::use_tensor_cores(dtype, D, block_size) ? attn::ws_layout(B, Hq, N, block_size, kmax).total : 0;
  return CAB_OK;
}

extern "C" int cab_sparse_attn_fwd(const void* q, const void* k, const void* v, const int32_t* kv_idx,
                                   const int32_t* kv_num, void* out, float* lse, int64_t B, int64_t Hq,
                                   int64_t Hkv, int64_t N, int64_t D, int64_t block_size, int64_t kmax,
                                   const int64_t* q_strides, const int64_t* k_strides,
                                   const int64_t* v_strides, const int64_t* o_strides, float softmax_scale,
                                   int causal, int dtype, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  using namespace attn;
  if (!q || !k || !v || !kv_idx || !kv_num || !out) return fail(CAB_ERR_INVALID_ARG, "attn: NULL pointer");
  if (!q_strides || !k_strides || !v_strides || !o_strides) return fail(CAB_ERR_INVALID_ARG, "attn: NULL strides");
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || N <= 0 || D <= 0 || block_size <= 0 || kmax <= 0)
    return fail(CAB_ERR_INVALID_ARG, "attn: non-positive size");
  if (Hq % Hkv != 0) return fail(CAB_ERR_INVALID_ARG, "attn: Hq %% Hkv != 0");
  if (!(softmax_scale > 0.f)) return fail(CAB_ERR_INVALID_ARG, "attn: softmax_scale must be > 0");
  const size_t es = dtype_size(dtype);
  if (!es) return fail(CAB_ERR_UNSUPPORTED, "attn: unknown dtype %d", dtype);
  if (N >= (int64_t)1 << 31 || B * Hq >= (int64_t)1 << 31) return fail(CAB_ERR_UNSUPPORTED, "attn: sizes exceed int32");
  const int64_t M = (N + block_size - 1) / block_size;
  if (M >= (int64_t)1 << 30) return fail(CAB_ERR_UNSUPPORTED, "attn: too many blocks");
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  if (use_tensor_cores(dtype, D, block_size)) {
    const WsLayout L = ws_layout(B, Hq, N, block_size, kmax);
    if (L.items >= (int64_t)1 << 31) return fail(CAB_ERR_UNSUPPORTED, "attn: more than 2^31 query-block pairs");
    if (!workspace || workspace_bytes < L.total)
      return fail(CAB_ERR_WORKSPACE, "attn: workspace of %zu bytes needed, %zu given", L.total, workspace_bytes);
    if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || !aligned16(workspace))
      return fail(CAB_ERR_INVALID_ARG, "attn: pointers must be 16-byte aligned");
    const int64_t* ss[4] = {q_strides, k_strides, v_strides, o_strides};
    for (int x = 0; x < 4; ++x)
      for (int i = 0; i < 3; ++i)
        if (ss[x][i] <= 0 || (ss[x][i] * static_cast<int64_t>(es)) % 16 != 0)
          return fail(CAB_ERR_INVALID_ARG, "attn: strides must be positive multiples of 16 bytes");
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    UnionParams up{};
    up.kv_idx = kv_idx;
    up.kv_num = kv_num;
    up.ulist = reinterpret_cast<uint32_t*>(ws + L.ulist_off);
    up.ntiles = reinterpret_cast<int32_t*>(ws + L.ntiles_off);
    up.items = L.items;
    up.M = static_cast<int32_t>(M);
    up.P = static_cast<int32_t>((M + 1) / 2);
    up.kmax = static_cast<int32_t>(kmax);
    up.stride = L.stride;
    up.words = static_cast<int32_t>((M + 31) / 32);
    const size_t usmem = static_cast<size_t>(4) * 2 * up.words * 4;
    if (usmem > 200 * 1024) return fail(CAB_ERR_UNSUPPORTED, "attn: M too large for the union kernel");
    cudaFuncSetAttribute(pair_union_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)usmem);
    const int ugrid = static_cast<int>(std::min<int64_t>((L.items + 3) / 4, (int64_t)current_sm_count() * 16));
    pair_union_kernel<<<ugrid, 128, usmem, st>>>(up);
    if (int rc = check_launch("pair_union_kernel")) return rc;

    CUtensorMap qm{}, km{}, vm{}, om{};
    if (int rc = attn_tensor_map(&qm, q, B, Hq, N, D, q_strides, es, dtype, 128)) return rc;
    if (int rc = attn_tensor_map(&km, k, B, Hkv, N, D, k_strides, es, dtype, 64)) return rc;
    if (int rc = attn_tensor_map(&vm, v, B, Hkv, N, D, v_strides, es, dtype, 64)) return rc;
    // output: one 32-row x D/2 box per softmax warp (128-byte rows for D=128, 64-byte for 64)
    if (int rc = attn_tensor_map(&om, out, B, Hq, N, D, o_strides, es, dtype, 32, static_cast<uint32_t>(D / 2),
                                 D == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B))
      return rc;
    Params p{};
    p.B = static_cast<int32_t>(B);
    p.Hq = static_cast<int32_t>(Hq);
    p.Hkv = static_cast<int32_t>(Hkv);
    p.Nq = static_cast<int32_t>(N);
    p.Nk = static_cast<int32_t>(N);
    p.M = static_cast<int32_t>(M);
    p.P = up.P;
    p.items = L.items;
    p.q = q;
    p.q_s0 = q_strides[0];
    p.q_s1 = q_strides[1];
    p.q_s2 = q_strides[2];
    p.o_s0 = o_strides[0];
    p.o_s1 = o_strides[1];
    p.o_s2 = o_strides[2];
    p.out = out;
    p.lse = lse;
    p.ulist = up.ulist;
    p.ntiles = up.ntiles;
    p.stride = L.stride;
    p.scale_log2 = softmax_scale * kLog2e;
    p.causal = causal != 0;
    const bool bf = dtype == CAB_DTYPE_BF16;
    const int grid = static_cast<int>(std::min<int64_t>(p.items, current_sm_count()));
    if (D == 128)
      return bf ? launch_tc<128, true, false>(qm, km, vm, om, p, grid, st) : launch_tc<128, false, false>(qm, km, vm, om, p, grid, st);
    return bf ? launch_tc<64, true, false>(qm, km, vm, om, p, grid, st) : launch_tc<64, false, false>(qm, km, vm, om, p, grid, st);
  }

  if (block_size > 128 || D > 128)
    return fail(CAB_ERR_UNSUPPORTED, "attn: CUDA-core path needs block_size <= 128 and D <= 128");
  SimtParams sp{};
  sp.q = q; sp.k = k; sp.v = v; sp.kv_idx = kv_idx; sp.kv_num = kv_num; sp.out = out; sp.lse = lse;
  sp.Hq = static_cast<int32_t>(Hq); sp.Hkv = static_cast<int32_t>(Hkv); sp.N = static_cast<int32_t>(N);
  sp.M = static_cast<int32_t>(M); sp.bs = static_cast<int32_t>(block_size); sp.D = static_cast<int32_t>(D);
  sp.kmax = static_cast<int32_t>(kmax);
  for (int i = 0; i < 3; ++i) {
    sp.qs[i] = q_strides[i]; sp.ks[i] = k_strides[i]; sp.vs[i] = v_strides[i]; sp.os[i] = o_strides[i];
  }
  sp.scale = softmax_scale;
  sp.causal = causal != 0;
  const size_t smem = static_cast<size_t>(block_size) * (3 * D + 2) * sizeof(float);
  dim3 grid(static_cast<unsigned>(M), static_cast<unsigned>(Hq), static_cast<unsigned>(B));
  switch (dtype) {
    case CAB_DTYPE_F32:
      cudaFuncSetAttribute(attn_simt_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attn_simt_kernel<float><<<grid, 128, smem, st>>>(sp);
      break;
    case CAB_DTYPE_F16:
      cudaFuncSetAttribute(attn_simt_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attn_simt_kernel<__half><<<grid, 128, smem, st>>>(sp);
      break;
    default:
      cudaFuncSetAttribute(attn_simt_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      attn_simt_kernel<__nv_bfloat16><<<grid, 128, smem, st>>>(sp);
      break;
  }
  return check_launch("attn_simt_kernel");
}

extern "C" int cab_flash_attn_workspace_size(int64_t B, int64_t Hq, int64_t Nq, int64_t Nk, int64_t D, int dtype,
                                             int with_scores, size_t* bytes) {
  (void)D;
  (void)dtype;
  if (!bytes) return fail(CAB_ERR_INVALID_ARG, "flash_workspace_size: NULL output");
  if (B <= 0 || Hq <= 0 || Nq <= 0 || Nk <= 0) return fail(CAB_ERR_INVALID_ARG, "flash_workspace_size: non-positive size");
  *bytes = with_scores ? attn::flash_layout(B, Hq, Nq, Nk).partial_bytes : 0;
  return CAB_OK;
}

extern "C" int cab_flash_attn_fwd(const void* q, const void* k, const void* v, void* out, float* scores,
                                  float* lse, int64_t B, int64_t Hq, int64_t Hkv, int64_t Nq, int64_t Nk,
                                  int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                                  const int64_t* v_strides, const int64_t* o_strides, float softmax_scale,
                                  int causal, int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  using namespace attn;
  if (!q || !k || !v || !out) return fail(CAB_ERR_INVALID_ARG, "flash: NULL pointer");
  if (!q_strides || !k_strides || !v_strides || !o_strides) return fail(CAB_ERR_INVALID_ARG, "flash: NULL strides");
  if (B <= 0 || Hq <= 0 || Hkv <= 0 || Nq <= 0 || Nk <= 0 || D <= 0)
    return fail(CAB_ERR_INVALID_ARG, "flash: non-positive size");
  if (Hq % Hkv != 0) return fail(CAB_ERR_INVALID_ARG, "flash: Hq %% Hkv != 0");
  if (!(softmax_scale > 0.f)) return fail(CAB_ERR_INVALID_ARG, "flash: softmax_scale must be > 0");
  if (causal && Nq != Nk) return fail(CAB_ERR_INVALID_ARG, "flash: causal needs Nq == Nk");
  if (dtype != CAB_DTYPE_BF16 && dtype != CAB_DTYPE_F16)
    return fail(CAB_ERR_UNSUPPORTED, "flash: dtype %d (bf16 / f16 only)", dtype);
  if (D != 64 && D != 128) return fail(CAB_ERR_UNSUPPORTED, "flash: D=%lld (64 or 128 only)", (long long)D);
  if (Nq >= (int64_t)1 << 30 || Nk >= (int64_t)1 << 30 || B * Hq >= (int64_t)1 << 31)
    return fail(CAB_ERR_UNSUPPORTED, "flash: sizes exceed int32");
  const size_t es = dtype_size(dtype);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out) || (scores && !aligned16(scores)))
    return fail(CAB_ERR_INVALID_ARG, "flash: pointers must be 16-byte aligned");
  const int64_t* ss[4] = {q_strides, k_strides, v_strides, o_strides};
  for (int x = 0; x < 4; ++x)
    for (int i = 0; i < 3; ++i)
      if (ss[x][i] <= 0 || (ss[x][i] * static_cast<int64_t>(es)) % 16 != 0)
        return fail(CAB_ERR_INVALID_ARG, "flash: strides must be positive multiples of 16 bytes");
  const FlashLayout L = flash_layout(B, Hq, Nq, Nk);
  if (L.items >= (int64_t)1 << 31) return fail(CAB_ERR_UNSUPPORTED, "flash: more than 2^31 query tiles");
  if (scores) {
    if (!workspace || workspace_bytes < L.partial_bytes)
      return fail(CAB_ERR_WORKSPACE, "flash: workspace of %zu bytes needed, %zu given", L.partial_bytes, workspace_bytes);
    if (!aligned16(workspace)) return fail(CAB_ERR_INVALID_ARG, "flash: workspace must be 16-byte aligned");
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap qm{}, km{}, vm{};
  if (int rc = attn_tensor_map(&qm, q, B, Hq, Nq, D, q_strides, es, dtype, 128)) return rc;
  if (int rc = attn_tensor_map(&km, k, B, Hkv, Nk, D, k_strides, es, dtype, 64)) return rc;
  if (int rc = attn_tensor_map(&vm, v, B, Hkv, Nk, D, v_strides, es, dtype, 64)) return rc;
  if (scores && cudaMemsetAsync(workspace, 0, L.partial_bytes, st) != cudaSuccess) {
    cudaGetLastError();
    return fail(CAB_ERR_LAUNCH, "flash: clearing the workspace failed");
  }
  Params p{};
  p.B = static_cast<int32_t>(B);
  p.Hq = static_cast<int32_t>(Hq);
  p.Hkv = static_cast<int32_t>(Hkv);
  p.Nq = static_cast<int32_t>(Nq);
  p.Nk = static_cast<int32_t>(Nk);
  p.M = static_cast<int32_t>((Nk + 63) / 64);
  p.P = static_cast<int32_t>((Nq + 127) / 128);
  p.Tk = static_cast<int32_t>(L.Tk);
  p.items = L.items;
  p.q = q;
  p.q_s0 = q_strides[0];
  p.q_s1 = q_strides[1];
  p.q_s2 = q_strides[2];
  p.o_s0 = o_strides[0];
  p.o_s1 = o_strides[1];
  p.o_s2 = o_strides[2];
  p.out = out;
  p.lse = lse;
  p.scale_log2 = softmax_scale * kLog2e;
  p.causal = causal != 0;
  p.colsum = scores;
  p.cs_s0 = Hq * Nk;
  p.cs_s1 = Nk;
  p.partial = scores ? static_cast<float*>(workspace) : nullptr;
  p.pstride = L.pstride;
  const bool bf = dtype == CAB_DTYPE_BF16;
  if (D == 128)
    return bf ? launch_tc<128, true, true>(qm, km, vm, qm, p, L.grid, st) : launch_tc<128, false, true>(qm, km, vm, qm, p, L.grid, st);
  return bf ? launch_tc<64, true, true>(qm, km, vm, qm, p, L.grid, st) : launch_tc<64, false, true>(qm, km, vm, qm, p, L.grid, st);
}
