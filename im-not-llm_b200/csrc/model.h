// Model state of libinl_cuda: configuration, device weights, workspaces and
// the per-forward launch plan. Internal to the library.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <map>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/inl_cuda.h"
#include "json.h"
#include "kernels.h"

namespace inl {

enum Arch : int { ARCH_QWEN3 = 0, ARCH_MODERNBERT = 1, ARCH_GEMMA = 2, ARCH_QWEN35 = 3 };

struct ModelConfig {
  Arch arch = ARCH_QWEN3;
  int H = 0, I = 0, hq = 0, hkv = 0, d = 0, layers = 0, V = 0;
  float eps = 1e-6f;
  double theta = 10000.0;        // rope theta (global / full layers)
  double theta_local = 10000.0;  // rope theta of local / sliding layers
  bool causal = true;
  int max_pos = 32768;           // rope table rows = longest text accepted
  // ModernBERT: a layer is global iff idx % global_every == 0; local layers
  // mask |q - k| > local_half_window.
  int global_every = 3;
  int local_half_window = 64;
  float norm_eps = 1e-5f;
  int pad_token_id = 0;
  // SPLADE head (ModernBERT MLM): logit shift before relu.
  float logit_shift = 0.f;
  // Gemma-style tower: sliding radius, full layer every `full_every` (idx % full_every == full_every-1),
  // attention scale, embedding scale, dense head dims.
  int sliding_window = 512;
  int full_every = 6;
  float attn_scale = 0.f;  // 0 = head_dim^-1/2
  float embed_scale = 1.f;
  std::vector<int> dense_dims;  // Gemma-style projection chain after pooling
  std::vector<char> layer_global;  // per layer: global / full attention (1) or local / sliding (0)
  // SPLADE pooling (ModernBERT MLM head)
  bool decoder_bias = true;
  std::vector<int> prefix_ids, masked_vocab_ids, canonical_ids;
  // Qwen3.5 text tower (crates/inl-late/src/qwen3_5.rs:56-168): per layer
  // Gated DeltaNet (1) or gated full attention (0); DeltaNet head shapes,
  // causal-convolution taps; rotary features per head (partial RoPE).
  std::vector<char> layer_linear;
  int lin_nk = 0, lin_nv = 0, lin_dk = 0, lin_dv = 0, conv_k = 0;
  int rot = 0;
  // EmbeddingGemma 2 (crates/inl-text/src/gemma2.rs:78-211): head_dim and KV
  // heads of every layer after the per_layer_config overrides (empty = d and
  // hkv on every layer), and the per-layer embedding width
  // (hidden_size_per_layer_input; 0 = no per-layer embeddings).
  std::vector<int> layer_d, layer_kv;
  int ple = 0;
  int dl(int l) const { return layer_d.empty() ? d : layer_d[l]; }
  int kvl(int l) const { return layer_kv.empty() ? hkv : layer_kv[l]; }
};

struct TensorSrc {
  const void* data = nullptr;
  int64_t numel = 0;
  std::vector<int64_t> shape;  // may be empty (numel only)
  int bf16 = 0;                // 0 = f32, 1 = bf16
};

using TensorMap = std::map<std::string, TensorSrc>;

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  // Grow-only, geometric (x2, at least 1 MiB) so that a stream of batches of
  // varying size reallocates O(log) times, never inside steady-state runs.
  cudaError_t ensure(size_t n) {
    if (n <= bytes) return cudaSuccess;
    size_t want = n;
    if (want < 2 * bytes) want = 2 * bytes;
    if (want < (size_t(1) << 20)) want = size_t(1) << 20;
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
    cudaError_t e = cudaMalloc(&p, want);
    if (e != cudaSuccess) {
      e = cudaMalloc(&p, n);  // no headroom available: exact size
      if (e != cudaSuccess) return e;
      want = n;
    }
    bytes = want;
    return e;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  template <typename T>
  T* as() const { return static_cast<T*>(p); }
};

struct LayerWeights {
  void* wqkv = nullptr;  // [(hq + 2 hkv) d, H]
  void* wo = nullptr;    // [H, hq d]
  void* wgu = nullptr;   // [2 I, H] gate/up interleaved in gate_block rows
  void* wd = nullptr;    // [H, I]
  float* ln1 = nullptr;  // attention input norm
  float* ln2 = nullptr;  // MLP input norm
  float* ln1_post = nullptr;  // Gemma post-attention norm
  float* ln2_post = nullptr;  // Gemma post-feedforward norm
  float* qn = nullptr;
  float* kn = nullptr;
  // Qwen3.5 Gated DeltaNet layer: [in_proj_qkv; in_proj_z; in_proj_b; in_proj_a] stacked
  // ([conv_dim + nv dv + 2 nv, H]), out_proj [H, nv dv], depthwise kernel [conv_dim, K],
  // per value head dt_bias and A_log, gated-norm weight [dv] (all f32 but the projections).
  void* w_lin_in = nullptr;
  void* w_lin_out = nullptr;
  float* conv_w = nullptr;
  float* dt_bias = nullptr;
  float* a_log = nullptr;
  float* lin_norm = nullptr;
  // EmbeddingGemma 2 per-layer embedding block (PleBlock, crates/inl-text/src/gemma2.rs:256-283):
  // input gate [ple, H], projection [H, ple] in the model dtype; post norm [H] and the layer
  // scalar [1] in f32.
  void* ple_gate = nullptr;
  void* ple_proj = nullptr;
  float* ple_norm = nullptr;
  float* scalar = nullptr;
};

struct ProfileRec {
  cudaEvent_t start, stop;
  double flops;
  int kind;
};

}  // namespace inl

struct inl_model {
  inl::ModelConfig c;
  int dtype = INL_DTYPE_BF16;
  int device = 0;
  cudaStream_t stream = nullptr;
  int* d_status = nullptr;
  int* h_status = nullptr;  // pinned
  int gate_block = 128;
  std::vector<void*> allocs;
  void* embed = nullptr;
  float* final_norm = nullptr;
  float* final_norm_b = nullptr;
  float* emb_norm = nullptr;  // ModernBERT embedding LayerNorm
  std::vector<inl::LayerWeights> layers;
  // rope tables [max_pos, d/2] f32: global and local
  float* cos0 = nullptr;
  float* sin0 = nullptr;
  float* cos1 = nullptr;
  float* sin1 = nullptr;
  float* rope_pairs = nullptr;  // QKV epilogue table [d/4, max_pos] x (cos f, cos f+1, sin f, sin f+1)
  // late Dense head
  void* proj = nullptr;
  float* proj_bias = nullptr;
  int proj_out = 0;
  bool proj_normalize = true;  // L2 after the projection (the Normalize module)
  // SPLADE / MLM head (ModernBERT)
  void* head_dense = nullptr;
  float* head_norm = nullptr;
  float* decoder_bias = nullptr;
  // Gemma-style dense chain (f32 weights) after pooling: dense_chain[j] is [dense_dims[j], in]
  std::vector<float*> dense_chain;
  // SPLADE device tables
  float* open_mask = nullptr;  // [V] 1 / 0
  int* canon = nullptr;        // [V] canonical term or null
  int sparse_dim = 0;
  // EmbeddingGemma 2 per-layer embeddings: projection of the scaled token
  // embeddings [layers * ple, H] (model dtype) and the norm of each layer's slice [ple]
  void* ple_model_proj = nullptr;
  float* ple_model_norm = nullptr;
  // workspaces
  inl::DevBuf h, xn, qkv, attn, ids, cu, pos, work, out, pooled, tmp;
  inl::DevBuf ple_in;  // [T, layers * ple] per-layer inputs of the batch
  // Pruned last layer of causal last-token pooling: the last rows' buffers,
  // the work list of the query tiles holding them, then 0..n.
  inl::DevBuf compact_meta, compact_off, compact_idx, compact_val;  // sparse compaction
  // f32 models: GEMMs as one bf16 tensor-core GEMM over K' = 3K (3xBF16) when
  // on; the split [hi | lo | hi] copy of each f32 weight is made on first use.
  bool f32_split3 = true;
  // Qwen3.5 tower requested in bf16: f32 activations and recurrence, the
  // GEMMs on bf16-rounded operands (one segment of the split path)
  bool f32_bf16_operands = false;
  int api_dtype = 0;  // the dtype the model was created with, as reported
  std::unordered_map<uintptr_t, void*> split_w;
  inl::DevBuf split_a, split_c;
  inl::DevBuf seg_scratch;  // mean pooling's per-chunk partial sums
  inl::DevBuf splitk_ws;    // split-K partial products of the f32 GEMMs
  inl::DevBuf lastbuf, work_last;
  int n_work_last = 0;
  bool prune_last = true;  // off: every layer runs on every row (tests compare the two)
  // Attention work list for layers whose head_dim takes another query block
  // than c.d's (per-layer head shapes); n_work_alt = 0 when every layer shares one.
  inl::DevBuf work_alt;
  int qb_alt = 0;
  int n_work_alt = 0;
  inl::DevBuf ss_a, ss_b;  // per-64-column sums of squares of h (folded RMSNorm)
  inl::DevBuf speak_idx, speak_seg, pooled_i, head_buf;  // SPLADE head scratch
  bool fused = false;      // bf16 fused layer (folded norms, QKV epilogue)
  bool gated_split = false;  // gate/up stored [gate; up] (intermediate not a multiple of gate_block)
  int* h_stage = nullptr;  // pinned staging for cu + work list
  size_t h_stage_bytes = 0;
  // profiling / launch accounting
  bool profiling = false;
  std::vector<inl::ProfileRec> prof;
  std::vector<cudaEvent_t> event_pool;
  long long launches = 0;
};
