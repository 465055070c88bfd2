/*
 * libinl_cuda: B200 (sm_100a) encoder forward for im-not-llm's embedding
 * engines, behind a plain C ABI (no C++ or torch types in any signature).
 *
 * The library replaces the candle model forward that the reference's engine
 * facades call once per planned batch:
 *   - dense:  Qwen3Embedder::embed            crates/inl-text/src/qwen3/mod.rs:438-470
 *             Gemma2Embedder::embed           crates/inl-text/src/gemma2.rs:770-799
 *   - sparse: ModernBertMlm::splade           crates/inl-sparse/src/modernbert.rs:671-691
 *   - late:   encode_batch (tower+Dense+norm) crates/inl-late/src/native.rs:631-683
 * Inputs are packed variable-length token ids with cumulative offsets
 * (cu_seqlens[0] = 0, cu_seqlens[i+1] - cu_seqlens[i] = tokens of text i)
 * instead of the reference's padded [batch, seq] id matrix: attention never
 * crosses texts and no padding is computed.
 *
 * Ownership: the caller owns ids, cu_seqlens and output buffers; the model
 * owns weights, workspaces and its stream. Threading: a model handle runs one
 * forward at a time (the reference admits one forward per model through a
 * gate, crates/inl-text/src/native.rs:668); calls on one handle must not
 * overlap. Every forward call returns after its results are written.
 *
 * Errors: every function returns an INL_* status; inl_cuda_last_error() gives
 * the message of the last failure on the calling thread.
 */
#ifndef INL_CUDA_H_
#define INL_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define INL_API __attribute__((visibility("default")))
#else
#define INL_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. They map one-to-one onto the reference's InlError classes
 * (crates/inl-core/src/error.rs:5-46, code() :36-46). */
#define INL_OK 0
#define INL_ERR_CONFIG 1        /* InlError::Config: bad or unsupported setting */
#define INL_ERR_INFERENCE 2     /* InlError::Inference: load or forward failed */
#define INL_ERR_TIMEOUT 3       /* InlError::Timeout: a device wait ran past its limit */
#define INL_ERR_INVALID_INPUT 4 /* InlError::InvalidInput: ids / offsets rejected */

/* Compute dtype of a model (the reference's DtypeSpec,
 * crates/inl-core/src/device.rs:13-298). */
#define INL_DTYPE_F32 0
#define INL_DTYPE_BF16 1

/* Where a caller buffer lives. */
#define INL_MEM_HOST 0
#define INL_MEM_DEVICE 1

typedef struct inl_model inl_model;

typedef struct inl_model_info {
  int arch;              /* 0 = qwen3, 1 = modernbert, 2 = gemma-style, 3 = qwen3.5 (late) */
  int dtype;             /* INL_DTYPE_* */
  int device;            /* CUDA ordinal */
  int hidden_size;
  int num_layers;
  int vocab_size;
  int dense_dim;         /* length of one forward_dense output row */
  int multivector_dim;   /* 0 until a Dense head is attached */
  int sparse_dim;        /* vocabulary of forward_sparse rows (0 if none) */
  int max_text_tokens;   /* longest text a forward accepts */
  int is_causal;
} inl_model_info;

/* Load a model from an HF-style config.json text and a safetensors file
 * (f32 or bf16 tensors, checkpoint tensor names), or the
 * model.safetensors.index.json of a sharded checkpoint: its weight_map's
 * files, sorted and each once, are read from the index's directory
 * (safetensors_weight_files, crates/inl-core/src/hub.rs:324-353). Replaces the candle load in
 * Qwen3Embedder::from_hf (crates/inl-text/src/qwen3/mod.rs:378-411),
 * ModernBertMlm::load (crates/inl-sparse/src/modernbert.rs:469-520) and
 * Gemma2Embedder::from_hf (crates/inl-text/src/gemma2.rs:671-700). */
INL_API int inl_cuda_model_create(const char* config_json, const char* safetensors_path, int device, int dtype,
                          inl_model** out);

/* Same, from named host f32 tensors (numels[i] values at data[i]). Replaces
 * VarBuilder::from_tensors as the reference's tests use it
 * (crates/inl-text/src/qwen3/mod.rs:590-594). */
INL_API int inl_cuda_model_create_from_tensors(const char* config_json, int n_tensors, const char* const* names,
                                       const float* const* data, const int64_t* numels, int device, int dtype,
                                       inl_model** out);

/* Parse and validate a config.json text for `dtype` without a device or
 * weights: the checks inl_cuda_model_create makes before loading (the
 * reference's Config::parse / validate of each tower, the SPLADE pooling
 * block, the shapes the CUDA towers take in that dtype). On success `out`
 * describes the model as inl_cuda_model_info would, with device -1 and
 * multivector_dim 0. */
INL_API int inl_cuda_config_check(const char* config_json, int dtype, inl_model_info* out);

/* Attach the Sentence-Transformers Dense projection of a late-interaction
 * model: weight [out_features, in_features] f32 (linear.weight), optional
 * bias [out_features]. in_features is hidden_size; out_features is any
 * positive width in f32, a multiple of 8 in bf16. Replaces the Dense load of
 * crates/inl-late/src/native.rs:546-567. */
INL_API int inl_cuda_model_set_dense_head(inl_model* m, const float* weight, int out_features, int in_features,
                                  const float* bias);

/* Whether forward_multivector L2-normalises each token vector after the Dense
 * projection and bias, x / max(||x||, 1e-12) (1, the default), or returns the
 * projection as it is (0): the late model's Normalize module is optional
 * (crates/inl-late/src/native.rs:472-483, 650-656). */
INL_API int inl_cuda_model_set_dense_normalize(inl_model* m, int normalize);

/* Dense embeddings [n_texts, info.dense_dim] f32, unit length.
 * Qwen3: final RMSNorm of each text's last token, x / sqrt(sum x^2 + 1e-12)
 * (Qwen3Embedder::embed, crates/inl-text/src/qwen3/mod.rs:438-470).
 * Gemma-style: mean pool, dense projections, L2, then Matryoshka truncation to
 * out_dim when out_dim > 0 (crates/inl-text/src/gemma2.rs:622-662;
 * truncate_and_normalize, crates/inl-text/src/native.rs:822-830).
 * out_dim = 0 keeps the full dimension. */
INL_API int inl_cuda_forward_dense(inl_model* m, const uint32_t* ids, int ids_mem, const int32_t* cu_seqlens, int n_texts,
                           int out_dim, float* out, int out_mem);

/* Late-interaction vectors [total_tokens, info.multivector_dim] f32, one per
 * token in packed order: final norm, Dense projection, x / max(|x|, 1e-12)
 * (encode_batch, crates/inl-late/src/native.rs:631-683; no skiplist). */
INL_API int inl_cuda_forward_multivector(inl_model* m, const uint32_t* ids, int ids_mem, const int32_t* cu_seqlens,
                                 int n_texts, float* out, int out_mem);

/* SPLADE term weights [n_texts, info.sparse_dim] f32, dense rows:
 * w_v = log(1 + relu(max_t logit[t, v] + bias_v - shift)) over the text's
 * tokens (SpladePooling::pool_states + finish,
 * crates/inl-sparse/src/modernbert.rs:806-885). Zero entries are absent terms. */
INL_API int inl_cuda_forward_sparse(inl_model* m, const uint32_t* ids, int ids_mem, const int32_t* cu_seqlens, int n_texts,
                            float* out, int out_mem);

/* SPLADE term weights as sparse vectors, compacted on the device: text i's
 * active terms (weight > 0) are indices[offsets[i] .. offsets[i + 1]) in
 * ascending term order with their weights in values[...], the pairs of the
 * reference's SparseVector (crates/inl-sparse/src/lib.rs:51-62), which its
 * encoder builds from the dense rows (crates/inl-sparse/src/native.rs:516-545).
 * offsets (n_texts + 1 entries, host memory) are always written; when
 * offsets[n_texts] exceeds capacity nothing else is written and the call
 * returns INL_ERR_INVALID_INPUT (call again with a capacity of at least
 * offsets[n_texts]). A non-finite weight is INL_ERR_INFERENCE, as the
 * reference's encoder refuses one (native.rs:536-540). indices and values are
 * host or device memory (out_mem); only the active terms cross to the host. */
INL_API int inl_cuda_forward_sparse_compact(inl_model* m, const uint32_t* ids, int ids_mem, const int32_t* cu_seqlens,
                                    int n_texts, int64_t* offsets, int32_t* indices, float* values,
                                    int64_t capacity, int out_mem);

/* Final hidden states [total_tokens, hidden] f32 before any pooling head
 * (after the tower's final norm when normalize_final != 0). For tests and
 * custom heads; the reference exposes the same tensor inside forward_last /
 * hidden_states (crates/inl-text/src/qwen3/mod.rs:339-358,
 * crates/inl-sparse/src/modernbert.rs:621-654). */
INL_API int inl_cuda_forward_hidden(inl_model* m, const uint32_t* ids, int ids_mem, const int32_t* cu_seqlens, int n_texts,
                            int normalize_final, float* out, int out_mem);

INL_API int inl_cuda_model_info(const inl_model* m, inl_model_info* out);

/* Release every device allocation of the model (LoadSlot::unload,
 * crates/inl-core/src/device.rs:303-348). NULL is ignored. */
INL_API void inl_cuda_model_destroy(inl_model* m);

/* Message of the last failure on this thread; returns its full length. */
INL_API int inl_cuda_last_error(char* buf, size_t len);

/* Number of visible CUDA devices (0 without a driver / GPU). */
INL_API int inl_cuda_device_count(void);

/* Library version string. */
INL_API const char* inl_cuda_version(void);

#ifdef __cplusplus
}
#endif

#endif /* INL_CUDA_H_ */
