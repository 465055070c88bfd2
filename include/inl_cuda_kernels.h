/*
 * libinl_cuda kernel-level entry points and measurement hooks.
 *
 * These take DEVICE pointers (plus a cudaStream_t passed as void*, NULL =
 * legacy default stream) and run one kernel each. They exist so that each
 * kernel can be checked on its own against a CPU restatement of the candle op
 * it replaces, and so that a benchmark can time the dominant kernel on the
 * stream it is launched on.
 */
#ifndef INL_CUDA_KERNELS_H_
#define INL_CUDA_KERNELS_H_

#include <stddef.h>
#include <stdint.h>

#include "inl_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Epilogues of the GEMM entry points. */
#define INL_GEMM_EPI_BF16 0       /* out = bf16(acc) */
#define INL_GEMM_EPI_RESID 1      /* out = bf16(bf16(acc) + resid), out may alias resid */
#define INL_GEMM_EPI_GATED 2      /* out[:, n/2] = act(gate) * up, gate/up interleaved in gate_block rows */
#define INL_GEMM_EPI_F32 3        /* out = acc (f32) */

#define INL_ACT_SILU_ 0
#define INL_ACT_GELU_ERF_ 1
#define INL_ACT_GELU_TANH_ 2

/* Y[M, N] = X[M, K] . W[N, K]^T on the tcgen05 tensor cores, bf16 operands,
 * f32 accumulation, fused epilogue. Replaces candle's Linear::forward (a cuBLAS
 * GEMM through cudarc) at every projection call site of the tower, e.g.
 * crates/inl-text/src/qwen3/mod.rs:236-253 and :110-116. `force_bn` picks the
 * tile width (0 = automatic, 128 or 256); `status` (device int, may be NULL)
 * receives a non-zero code if a device wait ran past its limit. */
INL_API int inl_cuda_gemm_bf16(const void* A, int64_t lda, const void* W, int64_t ldw, int M, int N, int K, int epi, int act,
                       int gate_block, void* out, int64_t ldo, const void* resid, int64_t ldr, int force_bn,
                       int* status, void* stream);

/* f32 SIMT version (epilogues INL_GEMM_EPI_F32, _RESID (f32 residual), _GATED
 * with gate_block 64). Replaces the f32 cuBLAS sgemm of the same call sites. */
INL_API int inl_cuda_gemm_f32(const float* A, int64_t lda, const float* W, int64_t ldw, int M, int N, int K, int epi, int act,
                      float* out, int64_t ldo, const float* resid, int64_t ldr, void* stream);

/* Packed variable-length attention softmax(scale q k^T + mask) v with causal
 * and/or |q - k| > window masks, GQA by head index. cu_seqlens is HOST memory.
 * Replaces attend / repeat_kv / additive_mask
 * (crates/inl-core/src/attention.rs:170-278). window < 0 disables it. */
INL_API int inl_cuda_attention(const void* q, const void* k, const void* v, int64_t ldq, int64_t ldk, int64_t ldv, void* out,
                       int64_t ldo, int dtype, int hq, int hkv, int d, float scale, int causal, int window,
                       const int32_t* cu_seqlens_host, int n_texts, void* stream);

/* Measurement hooks: with profiling on, every GEMM launch of the model is
 * bracketed by CUDA events on the model's stream. kind: 0 qkv, 1 o, 2 gate/up,
 * 3 down, 4 Dense head, -1 all. The reference has no counterpart (its
 * profiling was external, nsys). */
INL_API int inl_cuda_model_set_profiling(inl_model* m, int enable);
INL_API int inl_cuda_model_profile(inl_model* m, int kind, int* launches, double* total_ms, double* flops);

/* Kernel launches issued by the model since the last reset. */
INL_API long long inl_cuda_model_launch_count(inl_model* m, int reset);

/* The model's CUDA stream (cudaStream_t as void*). */
INL_API void* inl_cuda_model_stream(inl_model* m);

#ifdef __cplusplus
}
#endif

#endif /* INL_CUDA_KERNELS_H_ */
