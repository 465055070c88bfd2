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
#define INL_GEMM_EPI_RESID 1      /* out = bf16(acc + resid), out may alias resid */
#define INL_GEMM_EPI_GATED 2      /* out[:, n/2] = act(gate) * up, gate/up interleaved in gate_block rows */
#define INL_GEMM_EPI_F32 3        /* out = acc (f32) */
#define INL_GEMM_EPI_RESID_F32 6  /* out = acc + resid, f32 rows 16-byte aligned; out may alias resid */
#define INL_GEMM_EPI_GATED_F32 7  /* as INL_GEMM_EPI_GATED with an f32 output */

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

/* Every field of the fused GEMM epilogues (see INL_GEMM_EPI_*):
 *  ss_in/ss_in_parts/ss_dim/ss_eps: folded RMSNorm of the A rows; the
 *    accumulator is scaled by rsqrt(sum(ss_in[row, :]) / ss_dim + ss_eps);
 *  ss_out: [M, ceil(N / 64)] sums of squares of the stored bf16 rows (RESID);
 *  qn, kn, pos, cos, hq, hkv, d, max_pos, qk_eps: the QKV epilogue (per-head
 *    RMSNorm of q/k heads, half-split RoPE at pos[row]); cos is the RoPE table
 *    packed by frequency pairs, [d/4, max_pos, 4] f32 holding (cos f, cos f+1,
 *    sin f, sin f+1) for f = 2i, 16-byte aligned; sin is unused (NULL); qn / kn
 *    16-byte aligned. */
typedef struct inl_gemm_ex {
  const void* A;
  int64_t lda;
  const void* W;
  int64_t ldw;
  int M, N, K;
  int epi, act, gate_block;
  void* out;
  int64_t ldo;
  const void* resid;
  int64_t ldr;
  const float* ss_in;
  int ss_in_parts, ss_dim;
  float ss_eps;
  float* ss_out;
  const float* qn;
  const float* kn;
  const int32_t* pos;
  const float* cos;
  const float* sin;
  int hq, hkv, d, max_pos;
  float qk_eps;
  int force_bn;
  int* status;
} inl_gemm_ex;

#define INL_GEMM_EPI_QKV 4

/* The fused-epilogue GEMM of one encoder layer: replaces the candle sequence
 * RMSNorm -> Linear (-> q/k RMSNorm -> rope) (-> residual add) of
 * crates/inl-text/src/qwen3/mod.rs:227-297 with one launch. */
INL_API int inl_cuda_gemm_bf16_ex(const inl_gemm_ex* args, void* stream);

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

/* inl_cuda_attention for callers that must not allocate device memory (a host
 * whose pool allocator owns the GPU's memory, or code where a cudaMalloc or
 * cudaFree would synchronise the device or be refused). No counterpart in the
 * reference, which always allocates through candle. Same arguments, meaning
 * and results as inl_cuda_attention; it calls no cudaMalloc, cudaFree or other
 * allocating routine. Its state (cu_seqlens copy, work list, status word)
 * lives in one file-scope device array of 288.5 KiB that every GPU loading the
 * library holds until exit, so a call takes at most 8192 texts and 32768
 * query blocks (a block is 128 query rows for bf16 head_dim 64/128, 64 for
 * bf16 head_dim 256, 32 for f32); larger calls return INL_ERR_INVALID_INPUT.
 * The work list is built on the device, heaviest first like the allocating
 * entry point's. The first call on each device looks up the array's device
 * address with that device current; make that first call before any stream
 * capture. All calls share the array and would race if they overlapped on
 * the GPU, so each call holds a process-wide lock and waits for its stream to
 * drain before it returns; for that reason a stream that is capturing is
 * refused with INL_ERR_CONFIG before any work is queued. Argument errors are
 * found before any work is queued. A bounded device wait that runs out
 * returns INL_ERR_TIMEOUT. */
INL_API int inl_cuda_attention_noalloc(const void* q, const void* k, const void* v, int64_t ldq, int64_t ldk,
                                       int64_t ldv, void* out, int64_t ldo, int dtype, int hq, int hkv, int d,
                                       float scale, int causal, int window, const int32_t* cu_seqlens_host,
                                       int n_texts, void* stream);

/* Row gather table[ids[t]] * scale -> out [T, H]; dtypes INL_DTYPE_*. An id
 * >= vocab writes zeros and sets *status. Replaces candle's Embedding::forward
 * (index_select) at crates/inl-text/src/qwen3/mod.rs:352. */
INL_API int inl_cuda_embed_gather(const uint32_t* ids, int T, const void* table, int table_dtype, int vocab, int H,
                                  float scale, void* out, int out_dtype, int* status, void* stream);

/* Row RMSNorm (layer_norm = 0): x / sqrt(mean x^2 + eps) * w, or LayerNorm
 * (layer_norm = 1): (x - mean) / sqrt(var + eps) * w (+ b). w, b f32, may be
 * NULL. Replaces candle_nn::ops::rms_norm (crates/inl-text/src/qwen3/mod.rs:86-90)
 * and the reference LayerNorm (crates/inl-sparse/src/modernbert.rs:176-209). */
INL_API int inl_cuda_norm(const void* x, int x_dtype, int64_t ldx, const float* w, const float* b, float eps,
                          int layer_norm, int rows, int H, void* out, int out_dtype, int64_t ldo, void* stream);

/* In place on packed q|k|v rows [T, ld]: per-head RMSNorm of q heads (qw) and
 * k heads (kw) (NULL weight = no norm), weightless RMSNorm of v heads when
 * v_norm, then half-split RoPE of q and k at position pos[t] (device int32)
 * from tables cos/sin [max_pos, d/2] (device f32). Replaces q_norm/k_norm +
 * candle_nn::rotary_emb::rope (crates/inl-text/src/qwen3/mod.rs:236-249). */
INL_API int inl_cuda_qk_norm_rope(void* qkv, int dtype, int64_t ld, int T, int hq, int hkv, int d, const float* qw,
                                  const float* kw, int v_norm, float eps, const int32_t* pos, const float* cos,
                                  const float* sin, int max_pos, int* status, void* stream);

/* pos[t] = t - cu[i] for the text i holding packed token t (cu device int32 [n+1]). */
INL_API int inl_cuda_token_positions(const int32_t* cu, int n, int T, int32_t* pos, void* stream);

/* Last-token head: out[i] = L2(RMSNorm(h[cu[i+1]-1]) * w) in f32 (cu device).
 * Replaces forward_last's narrow + norm and the f32 L2 of
 * crates/inl-text/src/qwen3/mod.rs:339-358,467-469. */
INL_API int inl_cuda_last_token_norm_l2(const void* h, int h_dtype, int64_t ldh, const int32_t* cu, int n,
                                        const float* w, float eps, int H, float* out, void* stream);

/* Gated DeltaNet (Qwen3.5 "linear_attention" layers), f32, packed texts;
 * cu_seqlens is HOST memory. No model path calls these yet: they are the
 * kernel hooks of the next hot-path row, checked against oracle/qwen3_5.py.
 *
 * Depthwise causal convolution then SiLU over each text's tokens, zero before
 * its first token: out[t, c] = silu(sum_j w[c, j] x[t - K + 1 + j, c]),
 * w [C, K]. Replaces GatedDeltaNet::causal_conv
 * (crates/inl-late/src/qwen3_5.rs:463-479). */
INL_API int inl_cuda_causal_conv_silu(const float* x, int64_t ldx, int C, const float* w, int K,
                                      const int32_t* cu_seqlens_host, int n_texts, float* out, int64_t ldo,
                                      void* stream);

/* The gated delta rule per (text, value head) with the per-head gated
 * RMSNorm and silu(z) gate: mixed [T, ld_mixed] = q (nk dk) | k (nk dk) |
 * v (nv dv); b_in / a_in [T, ld_ab] column vh; z [T, ld_z]; out [T, ldo]
 * nv dv columns. dk in {8, 16, 32, 64, 128}, dv <= 128, nv a multiple of nk.
 * Replaces chunk_gated_delta_rule and the gated norm of GatedDeltaNet::forward
 * (crates/inl-late/src/qwen3_5.rs:481-545,612-739). */
INL_API int inl_cuda_gated_delta_rule(const float* mixed, int64_t ld_mixed, const float* b_in, const float* a_in,
                                      int64_t ld_ab, const float* z, int64_t ld_z, const float* dt_bias,
                                      const float* a_log, const float* norm_w, float eps, int nk, int nv, int dk,
                                      int dv, const int32_t* cu_seqlens_host, int n_texts, float* out, int64_t ldo,
                                      void* stream);

/* Measurement hooks: with profiling on, every GEMM and attention launch of
 * the model is bracketed by CUDA events on the model's stream. kind: 0 qkv,
 * 1 o, 2 gate/up, 3 down, 4 Dense head, 5 SPLADE head dense, 6 SPLADE
 * decoder, 7 per-layer-embedding GEMMs, -1 all GEMMs; 100 attention (flops
 * reported as 0). The reference has no counterpart (its profiling was
 * external, nsys). */
INL_API int inl_cuda_model_set_profiling(inl_model* m, int enable);
INL_API int inl_cuda_model_profile(inl_model* m, int kind, int* launches, double* total_ms, double* flops);

/* f32 models' contractions: mode 1 (default) runs each as one bf16 tcgen05
 * GEMM over K' = 3K on split operands, [hi | hi | lo] . [hi | lo | hi] with
 * hi = bf16(x), lo = bf16(x - hi), accumulated in f32 (3xBF16: relative error
 * ~5e-6 per product sum); mode 0 runs them on the SIMT FFMA kernels, the
 * default for the Qwen3.5 late tower (its gated delta rule carries a state
 * from token to token, which grows that error past the reference's 1e-4
 * per component for this tower). The
 * reference runs f32 on cuBLAS SGEMM and found single-pass TF32 too coarse
 * for its sparse golden (docs/DEVICES.md:371-379). */
INL_API int inl_cuda_model_set_f32_gemm(inl_model* m, int mode);

/* Causal last-token pooling (Qwen3 dense, bf16): by default the last layer
 * runs attention on the query tile holding each text's last row and the o /
 * MLP projections on the n last rows only, as the pooled vector needs
 * nothing else. enable = 0 runs that layer on every row (the embeddings are
 * the same function; tests compare the two). The reference computes every
 * row (crates/inl-text/src/qwen3/mod.rs:339-358 narrows after the stack). */
INL_API int inl_cuda_model_set_prune_last(inl_model* m, int enable);

/* Kernel launches issued by the model since the last reset. */
INL_API long long inl_cuda_model_launch_count(inl_model* m, int reset);

/* The model's CUDA stream (cudaStream_t as void*). */
INL_API void* inl_cuda_model_stream(inl_model* m);

#ifdef __cplusplus
}
#endif

#endif /* INL_CUDA_KERNELS_H_ */
