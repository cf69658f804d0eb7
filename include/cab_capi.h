/*
 * cab_capi.h -- C ABI of libcab_b200.so, the sm_100a kernels of CAB-Attention's prefill
 * path (Max-L2 coarsening -> coarse Forman-Ricci score -> per-row top-k block mask ->
 * block-sparse attention).
 *
 * Conventions shared by every entry point:
 *  - Plain device pointers and sizes; no framework types. Outputs and scratch memory are
 *    allocated by the caller. Entry points that need scratch memory have a
 *    `*_workspace_size` query.
 *  - Every call is ordered on the caller's `stream` (a cudaStream_t passed as void*),
 *    does not synchronise with the host and keeps no state between calls.
 *  - Return value: CAB_OK or a CAB_ERR_* code; cab_last_error_string() (per host thread)
 *    describes the last failure. Nothing falls back to another implementation.
 *  - Tensors are row-major. "[B,H,N,D] with strides" means element (b,h,n,d) lives at
 *    ptr[b*s[0] + h*s[1] + n*s[2] + d] (strides in elements, innermost dimension dense).
 *  - dtype: CAB_DTYPE_BF16 / CAB_DTYPE_F16 run on the tensor cores (tcgen05); CAB_DTYPE_F32
 *    runs on CUDA cores in fp32 / fp64.
 *
 * The reference (Js-Hwang1/Bridge-Aware-KV-Cache-Eviction-for-Efficient-Long-Context-
 * Transformers) implements this path in Python modules listed in README.md:189-196
 * (cab_attention/kernels/coarsening.py, cab_attention/kernels/frc_kernel.py,
 * cab_attention/coarse_predictor.py, cab_attention/cab_attention.py); the snapshot keeps
 * their callers, cited per entry point below.
 */
#ifndef CAB_CAPI_H_
#define CAB_CAPI_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CAB_API_VERSION 1

#if defined(__GNUC__)
#define CAB_API __attribute__((visibility("default")))
#else
#define CAB_API
#endif

/* status codes */
#define CAB_OK 0
#define CAB_ERR_INVALID_ARG 1 /* null pointer, bad size, misaligned pointer or stride */
#define CAB_ERR_UNSUPPORTED 2 /* dtype / shape / device not handled by the kernels     */
#define CAB_ERR_LAUNCH 3      /* CUDA launch or driver error                           */
#define CAB_ERR_TIMEOUT 4     /* a device-side wait gave up (see cab_device_status)     */
#define CAB_ERR_WORKSPACE 5   /* workspace missing or smaller than *_workspace_size     */

/* element types */
#define CAB_DTYPE_F32 0
#define CAB_DTYPE_F16 1
#define CAB_DTYPE_BF16 2

/* Direct-connection normalisation of the affinity (compute_block_frc `normalization`) */
#define CAB_NORM_ABS 0    /* |A|                                      */
#define CAB_NORM_MINMAX 1 /* (A - min) / (max - min + 1e-8) per (b,h) */
#define CAB_NORM_RAW 2    /* A                                        */

/* FRC formula (compute_block_frc `formula`) */
#define CAB_FORMULA_ADDITIVE 0       /* F = Direct - lambda * T                        */
#define CAB_FORMULA_MULTIPLICATIVE 1 /* F = Direct / (1 + lambda * T / (Direct + 1e-8)) */

/* redundancy scaling */
#define CAB_RED_SCALE_NONE 0  /* T = Direct @ Direct       */
#define CAB_RED_SCALE_INV_M 1 /* T = (Direct @ Direct) / M */

/* Library version (CAB_API_VERSION). */
CAB_API int cab_get_version(void);

/* Text of the last error raised on this host thread ("" if none). */
CAB_API const char* cab_last_error_string(void);

/* 1 if `device` is an sm_100 part these kernels were built for, else 0. */
CAB_API int cab_device_supported(int device);

/* Synchronises `stream`, then reads and clears the device-side status word of the
 * current device in one atomic exchange (a bit set meanwhile by a kernel on another stream
 * is kept for the next call, never lost) and stores: 0 = fine, CAB_ERR_TIMEOUT if a kernel's
 * bounded wait gave up, CAB_ERR_LAUNCH if a kernel found its shared-memory layout did not
 * fit and did nothing. */
CAB_API int cab_device_status(void* stream, int* status);

/* Failure-detection self-test (no reference counterpart): launches a kernel whose one
 * bounded wait can never be satisfied; after `limit_us` microseconds it gives up exactly
 * as the library's kernels do on a timeout (device status word := timeout, *gave_up_device
 * := 1 in device memory) and returns. Nothing faults, traps or hangs; the next
 * cab_device_status on `stream` reports CAB_ERR_TIMEOUT and the context stays usable. */
CAB_API int cab_selftest_wait_timeout(int64_t limit_us, int* gave_up_device, void* stream);

/*
 * Max-L2 coarsening: for every `block_size`-token block of q [B,Hq,N,D] and
 * k [B,Hkv,N,D], pick the token with the largest L2 norm (norm^2 accumulated in fp64;
 * the lowest index wins ties; a partial last block uses its valid tokens) and copy it to
 * q_coarse [B,Hq,M,D] / k_coarse [B,Hkv,M,D] (dense), M = ceil(N / block_size).
 * q_idx / k_idx ([B,Hq,M] / [B,Hkv,M] int32, absolute token index) may be NULL.
 * Either side may be skipped by passing NULL for its input and outputs.
 * Strides: q_strides/k_strides = {b, h, n} in elements; base pointers and n-strides must be
 * 16-byte aligned. D * sizeof(dtype) must be a multiple of 16 and <= 1024 bytes.
 * Replaces coarsen_qk_max_l2 / coarsen_qk_max_l2_pytorch (cab_attention/kernels/
 * coarsening.py; callers benchmarks/kernel_benchmark.py:82-85,
 * benchmarks/quick_kernel_test.py:54-57, experiments/longbench_qa/methods.py:303,327).
 */
CAB_API int cab_coarsen_maxl2(const void* q, const void* k, void* q_coarse, void* k_coarse,
                      int32_t* q_idx, int32_t* k_idx, int64_t B, int64_t Hq, int64_t Hkv,
                      int64_t N, int64_t D, int64_t block_size, const int64_t* q_strides,
                      const int64_t* k_strides, int dtype, void* stream);

/* Scratch bytes cab_frc needs for these sizes. */
CAB_API int cab_frc_workspace_size(int64_t B, int64_t Hq, int64_t M, int64_t D, int dtype,
                           int normalization, size_t* bytes);

/*
 * Coarse Forman-Ricci score per (b, query head):
 *   A = q_coarse @ k_coarse^T / sqrt(D) / temperature      (query head h uses KV head
 *                                                             h / (Hq / Hkv))
 *   Direct = normalisation(A); T = Direct @ Direct (optionally / M)
 *   F = formula(Direct, T, lambda_redundancy)
 * q_coarse [B,Hq,M,D], k_coarse [B,Hkv,M,D] dense. Outputs [B,Hq,M,M] fp32 dense:
 * frc (required), affinity (= Direct, may be NULL), redundancy (= T, may be NULL).
 * bf16/f16: both products on tcgen05 tensor cores; T takes f16 operands (Direct rounded
 * to f16, |Direct| must stay below 65504) with f32 accumulation. f32: A in fp32 on CUDA
 * cores, T from an f16 hi/lo split (three tensor-core products).
 * Replaces compute_block_frc (cab_attention/kernels/frc_kernel.py; callers
 * experiments/longbench_qa/methods.py:330-336,384-389,452-458,
 * benchmarks/kernel_benchmark.py:149,253, benchmarks/quick_kernel_test.py:67).
 */
CAB_API int cab_frc(const void* q_coarse, const void* k_coarse, float* frc, float* affinity,
            float* redundancy, int64_t B, int64_t Hq, int64_t Hkv, int64_t M, int64_t D,
            int dtype, float temperature, float lambda_redundancy, int normalization,
            int formula, int redundancy_scale, void* workspace, size_t workspace_bytes,
            void* stream);

/*
 * Per-row top-k block selection over scores [BH,M,M] fp32 (dense).
 * Row i keeps k_i = min(k, #candidates) blocks: candidates are all j (or j <= i when
 * `causal`); with `keep_diagonal` block i is always kept and the rest come from j != i.
 * Preference: larger score if select_high else smaller; NaN least preferred; -0 == +0;
 * ties go to the lower block index. Outputs: kv_idx [BH,M,k] int32 ascending, -1 padded;
 * kv_num [BH,M] int32 (= k_i); dense_mask [BH,M,M] uint8 0/1 (may be NULL).
 * Requires 1 <= k <= M <= 49152.
 * Replaces generate_block_mask (cab_attention/kernels/frc_kernel.py; callers
 * experiments/longbench_qa/methods.py:339-345,392-398, benchmarks/kernel_benchmark.py:197).
 */
CAB_API int cab_topk_blocks(const float* scores, int32_t* kv_idx, int32_t* kv_num, uint8_t* dense_mask,
                    int64_t BH, int64_t M, int64_t k, int select_high, int keep_diagonal,
                    int causal, void* stream);

/*
 * Hybrid (CAB V4) block selection: cab_topk_blocks with a second score matrix. Per row,
 * after the forced diagonal, floor(r * magnitude_ratio) of the remaining budget r = k_i - 1
 * (k_i with keep_diagonal off) go to the candidates with the largest `magnitude` score
 * ([BH,M,M] fp32, larger preferred, NaN least); the rest go to the best `scores` (direction
 * select_high) among the candidates not yet taken. Ties go to the lower block index; the
 * causal rule applies to both parts. Outputs as cab_topk_blocks (the union, ascending).
 * The reference's generate_block_mask(magnitude_scores=, magnitude_ratio=) is called by
 * experiments/longbench_qa/methods.py:465-473 and benchmarks/kernel_benchmark.py:201-205
 * but its implementation is absent from the snapshot; this split is the documented rule of
 * methods.py:407-418 ("reserve X% of budget for top-magnitude blocks").
 */
CAB_API int cab_topk_blocks_hybrid(const float* scores, const float* magnitude, int32_t* kv_idx,
                                   int32_t* kv_num, uint8_t* dense_mask, int64_t BH, int64_t M,
                                   int64_t k, double magnitude_ratio, int select_high,
                                   int keep_diagonal, int causal, void* stream);

/*
 * Block max-pool of a dense attention matrix: out[bh,I,J] = max over the
 * block_size x block_size tile (I,J) of attn[bh] ([BH,N,N] dense, f32/f16/bf16), with the
 * zero padding of a partial last block included (fp32 out [BH,M,M], M = ceil(N/block_size)).
 * block_size: a power of two in [8, 1024].
 * Replaces CABV4Attention._coarsen_attention (experiments/longbench_qa/methods.py:535-553).
 */
CAB_API int cab_block_maxpool(const void* attn, float* out, int64_t BH, int64_t N, int64_t block_size,
                              int dtype, void* stream);

/* Scratch bytes cab_sparse_attn_fwd needs for these sizes. */
CAB_API int cab_sparse_attn_workspace_size(int64_t B, int64_t Hq, int64_t N, int64_t D,
                                   int64_t block_size, int64_t kmax, int dtype, size_t* bytes);

/*
 * Block-sparse attention forward: for each query block i of (b, h) attend to the key
 * blocks kv_idx[b,h,i,0:kv_num[b,h,i]] of KV head h / (Hq / Hkv):
 *   out = softmax(q k^T * softmax_scale + mask) v, mask = -inf outside the kept blocks,
 *   beyond N, and (if `causal`) where key position > query position.
 * A row that sees no key gets out = 0 and lse = -inf.
 * q/out [B,Hq,N,D], k/v [B,Hkv,N,D] with {b,h,n} strides (elements, 16-byte aligned);
 * kv_idx [B,Hq,M,kmax] int32 (ascending, entries < M), kv_num [B,Hq,M] int32;
 * lse [B,Hq,N] fp32 natural-log sum-exp (may be NULL).
 * bf16/f16 with block_size 64 and D in {64,128}: TMA-fed tcgen05 kernel, fp32 softmax
 * and accumulation. Other cases (and f32): CUDA-core kernel, fp32 arithmetic.
 * Replaces the FlexAttention / manual sparse-attention step of CABAttention.forward
 * (cab_attention/cab_attention.py; README.md:44-46; manual path
 * experiments/longbench_qa/methods.py:103-119,348-356).
 */
CAB_API int cab_sparse_attn_fwd(const void* q, const void* k, const void* v, const int32_t* kv_idx,
                        const int32_t* kv_num, void* out, float* lse, int64_t B, int64_t Hq,
                        int64_t Hkv, int64_t N, int64_t D, int64_t block_size, int64_t kmax,
                        const int64_t* q_strides, const int64_t* k_strides,
                        const int64_t* v_strides, const int64_t* o_strides,
                        float softmax_scale, int causal, int dtype, void* workspace,
                        size_t workspace_bytes, void* stream);

/*
 * cab_sparse_attn_fwd for callers that cannot allocate device memory: the same inputs,
 * outputs and semantics, without the workspace arguments. No counterpart in the
 * reference (an addition of this library).
 * Who needs it: hosts whose device memory belongs to another allocator (a framework's
 * caching allocator, a serving engine's pre-reserved pool) or bindings that link no CUDA
 * allocator, so they cannot cudaMalloc the workspace cab_sparse_attn_fwd asks for.
 * Scratch: a static 16 MiB device buffer inside the library, held on every GPU that loads
 * it until the process exits. Sizes whose cab_sparse_attn_workspace_size exceeds 16 MiB
 * return CAB_ERR_UNSUPPORTED. The first call in each CUDA context looks up the buffer's
 * address (cudaGetSymbolAddress, with that context current) and caches it against the
 * context's unique ID, so a new context on the device (after cudaDeviceReset, or a
 * driver-API context made current) looks it up again; make that first call before any
 * stream capture. All calls share the buffer, so calls that overlap on the GPU race.
 * The call itself allocates nothing.
 */
CAB_API int cab_sparse_attn_fwd_noalloc(const void* q, const void* k, const void* v,
                                        const int32_t* kv_idx, const int32_t* kv_num, void* out,
                                        float* lse, int64_t B, int64_t Hq, int64_t Hkv, int64_t N,
                                        int64_t D, int64_t block_size, int64_t kmax,
                                        const int64_t* q_strides, const int64_t* k_strides,
                                        const int64_t* v_strides, const int64_t* o_strides,
                                        float softmax_scale, int causal, int dtype, void* stream);

/* Scratch bytes cab_flash_attn_fwd needs (0 when with_scores is 0). Depends on the
 * current device's SM count. */
CAB_API int cab_flash_attn_workspace_size(int64_t B, int64_t Hq, int64_t Nq, int64_t Nk, int64_t D,
                                          int dtype, int with_scores, size_t* bytes);

/*
 * Dense attention forward with cumulative column scores:
 *   out = softmax(q k^T * softmax_scale) v          (each q head h reads KV head h / (Hq/Hkv))
 *   scores[b,h,j] += sum over queries i of exp(s_ij - m_i(j))
 * with s_ij = q_i . k_j * softmax_scale and m_i(j) the running row maximum over the keys
 * of the 128-key blocks 0 .. j/128 (the blocks are visited in order, as the reference's
 * flash kernel accumulates them; the scores are not normalised by the row sums).
 * q/out [B,Hq,Nq,D], k/v [B,Hkv,Nk,D] with {b,h,n} strides (elements, 16-byte aligned);
 * scores [B,Hq,Nk] fp32 dense, accumulated into (may be NULL: no scores, no workspace);
 * lse [B,Hq,Nq] fp32 natural-log sum-exp (may be NULL). Nq may differ from Nk (a decode
 * step against a KV cache); causal (an addition: the reference is non-causal) needs
 * Nq == Nk. bf16/f16 with D in {64, 128}, on tcgen05.
 * Replaces flash_attention_with_cumulative_scores (cab_attention/kernels/
 * flash_attention_accumulate.py:169-261, kernel :23-166; callers
 * experiments/longbench_qa/runner.py:291, experiments/generation_benchmark/driver.py:144
 * through replace_attention_with_flash).
 */
CAB_API int cab_flash_attn_fwd(const void* q, const void* k, const void* v, void* out, float* scores,
                               float* lse, int64_t B, int64_t Hq, int64_t Hkv, int64_t Nq, int64_t Nk,
                               int64_t D, const int64_t* q_strides, const int64_t* k_strides,
                               const int64_t* v_strides, const int64_t* o_strides, float softmax_scale,
                               int causal, int dtype, void* workspace, size_t workspace_bytes,
                               void* stream);

/*
 * Node-level Forman-Ricci curvature of attention graphs attention [batch,N,N] (dense,
 * f32/f16/bf16): strengths S_i = sum_j A_ij, triangles T_i = sum_j sum_k A_ij A_jk
 * (= sum_j A_ij S_j), frc F_i = 4 S_i - 2 S_i + 3 T_i; outputs fp32 [batch,N]
 * (strengths required, triangles may be NULL).
 * Replaces compute_frc_triton / compute_frc_pytorch / compute_frc
 * (cab_attention/kernels/frc_triton.py:167-313, exported by cab_attention/kernels/__init__.py:5).
 */
CAB_API int cab_node_frc(const void* attention, float* frc, float* strengths, float* triangles,
                         int64_t batch, int64_t N, int dtype, void* stream);

/* Scratch bytes cab_evict_select needs. */
CAB_API int cab_evict_workspace_size(int64_t batch, int64_t L, int with_attention, size_t* bytes);

/*
 * Three-component KV-cache eviction selection, one independent selection per sequence:
 * budgets local = int(K*local_ratio), bridge = int(K*bridge_ratio), importance = K - both
 * (each clipped to L); keep [L-local, L), then the `importance` largest scores among the
 * rest (importance [batch,imp_len] fp32, zero-padded / truncated to L; NULL: the range just
 * before the local window), then the bridges: with attention [batch,L,L] fp32 and at least
 * one important position the largest from*to connectivity with the important set, else the
 * smallest |score - lower median of the unselected scores|, else the positions from one
 * third into the unselected ones. Ties go to the lower position. Outputs: keep_indices
 * [batch,K] int64 ascending (-1 padded), counts [batch,4] = kept, local, importance, bridge.
 * L <= 524288. No host synchronisation.
 * Replaces ThreeComponentEvictionPolicy.select_indices (cab_attention/eviction/policy.py:40-210).
 */
CAB_API int cab_evict_select(const float* importance, int64_t imp_len, const float* attention,
                             int64_t batch, int64_t L, int64_t keep_size, double local_ratio,
                             double bridge_ratio, int64_t* keep_indices, int32_t* counts,
                             void* workspace, size_t workspace_bytes, void* stream);

/* Scratch bytes cab_prefill_host needs for these sizes (two device slots of one
 * (batch, KV head) unit each). `keep` = blocks kept per query-block row. */
CAB_API int cab_prefill_host_workspace_size(int64_t B, int64_t Hq, int64_t Hkv, int64_t N,
                                            int64_t D, int64_t block_size, int64_t keep,
                                            int dtype, int normalization, size_t* bytes);

/*
 * The whole prefill path for inputs and outputs in HOST memory: per (b, query head)
 * cab_coarsen_maxl2 -> cab_frc -> cab_topk_blocks (k = keep) -> cab_sparse_attn_fwd, with
 * the same arguments and results as calling those four entry points on device copies of
 * the tensors (bit-identical outputs).
 * q/out [B,Hq,N,D] and k/v [B,Hkv,N,D] are dense host tensors; kv_idx [B,Hq,M,keep] and
 * kv_num [B,Hq,M] (int32, may be NULL) receive the block lists. All host buffers must be
 * page-locked (cudaHostAlloc / cudaHostRegister); anything else is CAB_ERR_INVALID_ARG.
 * The work is streamed one (b, KV head) unit at a time through two device slots of the
 * workspace: the host->device copy of the next unit and the device->host copy of the
 * previous one (on two library-owned copy streams of the current device) overlap the
 * compute of this one (on `stream`). Asynchronous like every entry point: it starts after
 * the work already queued on `stream`, later work on `stream` starts after all of its
 * copies, and the host buffers must stay valid (and `out` unread) until then.
 * No counterpart in the reference (an addition of this library): its callers move whole
 * tensors between host and device around the layer.
 */
CAB_API int cab_prefill_host(const void* q, const void* k, const void* v, void* out,
                             int32_t* kv_idx, int32_t* kv_num, int64_t B, int64_t Hq,
                             int64_t Hkv, int64_t N, int64_t D, int64_t block_size, int64_t keep,
                             float temperature, float lambda_redundancy, int normalization,
                             int formula, int redundancy_scale, int select_high,
                             int keep_diagonal, int causal, float softmax_scale, int dtype,
                             void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CAB_CAPI_H_ */
