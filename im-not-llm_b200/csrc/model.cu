// libinl_cuda runtime: model load (config JSON + safetensors or named host
// tensors), device weight layout, workspaces, and the forward launch plan of
// the packed variable-length encoder, exported through the C ABI of
// include/inl_cuda.h.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/inl_cuda.h"
#include "../../include/inl_cuda_kernels.h"
#include "checkpoint.h"
#include "common.cuh"
#include "model.h"

using inl::DevBuf;
using inl::ProfileRec;
using inl::ModelConfig;
using inl::TensorMap;
using inl::TensorSrc;

namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

#define INL_CUDA_TRY(expr, what)                                                              \
  do {                                                                                        \
    cudaError_t _e = (expr);                                                                  \
    if (_e != cudaSuccess)                                                                    \
      return fail(INL_ERR_INFERENCE, std::string(what) + ": " + cudaGetErrorString(_e));      \
  } while (0)

#define INL_K_TRY(expr, what)                                                                 \
  do {                                                                                        \
    int _r = (expr);                                                                          \
    if (_r != 0) {                                                                            \
      cudaError_t _e = cudaGetLastError();                                                    \
      return fail(INL_ERR_INFERENCE, std::string(what) + " failed (" + std::to_string(_r) + \
                                         "): " + cudaGetErrorString(_e));                     \
    }                                                                                         \
  } while (0)

// ------------------------------------------------------------ config parsing
double num_or(const inl::json::Value& v, const char* key, double def) {
  const inl::json::Value* x = v.get(key);
  return (x && x->is_num()) ? x->num : def;
}
bool bool_or(const inl::json::Value& v, const char* key, bool def) {
  const inl::json::Value* x = v.get(key);
  return (x && x->kind == inl::json::Value::Bool) ? x->b : def;
}
std::string str_or(const inl::json::Value& v, const char* key, const std::string& def) {
  const inl::json::Value* x = v.get(key);
  return (x && x->kind == inl::json::Value::String) ? x->str : def;
}

std::vector<int> int_list(const inl::json::Value* v) {
  std::vector<int> out;
  if (v && v->kind == inl::json::Value::Array)
    for (const auto& x : v->arr) out.push_back(static_cast<int>(x.num));
  return out;
}

// rope_parameters.{full_attention|sliding_attention}.rope_theta, when present.
bool nested_theta(const inl::json::Value& root, const char* kind, double* out) {
  const inl::json::Value* rp = root.get("rope_parameters");
  if (!rp) return false;
  const inl::json::Value* k = rp->get(kind);
  if (!k) return false;
  const inl::json::Value* t = k->get("rope_theta");
  if (!t || !t->is_num()) return false;
  *out = t->num;
  return true;
}

int parse_config(const std::string& text, ModelConfig& c) {
  inl::json::Value root;
  try {
    root = inl::json::parse(text);
  } catch (const std::exception& e) {
    return fail(INL_ERR_CONFIG, std::string("config: ") + e.what());
  }
  if (root.kind != inl::json::Value::Object) return fail(INL_ERR_CONFIG, "config: not a JSON object");
  std::string mt = str_or(root, "model_type", "qwen3");
  // Nested text configs: Qwen3-VL (crates/inl-text/src/qwen3/mod.rs:55-69) and
  // EmbeddingGemma 2 (crates/inl-text/src/gemma2.rs:108-112).
  if (const inl::json::Value* tc = root.get("text_config"); tc && tc->kind == inl::json::Value::Object) {
    inl::json::Value inner = *tc;
    if (!inner.get("model_type")) {
      inl::json::Value name;
      name.kind = inl::json::Value::String;
      name.str = mt;
      inner.obj.emplace_back("model_type", name);
    }
    root = inner;
    mt = str_or(root, "model_type", mt);
  }
  if (mt == "qwen3") c.arch = inl::ARCH_QWEN3;
  else if (mt == "modernbert") c.arch = inl::ARCH_MODERNBERT;
  else if (mt == "gemma_style" || mt == "gemma3_text" || mt == "embedding_gemma2" || mt == "embeddinggemma")
    c.arch = inl::ARCH_GEMMA;
  else if (mt == "qwen3_5" || mt == "qwen3_5_text")
    c.arch = inl::ARCH_QWEN35;
  else
    return fail(INL_ERR_CONFIG, "config: unsupported model_type '" + mt + "'");
  c.H = static_cast<int>(num_or(root, "hidden_size", 0));
  c.I = static_cast<int>(num_or(root, "intermediate_size", 0));
  c.hq = static_cast<int>(num_or(root, "num_attention_heads", 0));
  c.hkv = static_cast<int>(num_or(root, "num_key_value_heads", c.hq));
  c.layers = static_cast<int>(num_or(root, "num_hidden_layers", 0));
  c.V = static_cast<int>(num_or(root, "vocab_size", 0));
  c.d = static_cast<int>(num_or(root, "head_dim", c.hq > 0 ? c.H / c.hq : 0));
  if (c.H <= 0 || c.I <= 0 || c.hq <= 0 || c.hkv <= 0 || c.layers <= 0 || c.V <= 0 || c.d <= 0)
    return fail(INL_ERR_CONFIG, "config: missing or invalid model dimensions");
  if (c.hq % c.hkv != 0)
    return fail(INL_ERR_CONFIG, "config: num_attention_heads must be a multiple of num_key_value_heads");
  if (bool_or(root, "attention_bias", false))
    return fail(INL_ERR_CONFIG, "config: attention_bias = true is not supported");
  c.eps = static_cast<float>(num_or(root, "rms_norm_eps", 1e-6));
  c.theta = num_or(root, "rope_theta", 10000.0);
  c.max_pos = static_cast<int>(std::min(32768.0, num_or(root, "max_position_embeddings", 32768.0)));
  c.pad_token_id = static_cast<int>(num_or(root, "pad_token_id", 0));
  c.layer_global.assign(c.layers, 1);
  if (c.arch == inl::ARCH_QWEN3) {
    c.causal = bool_or(root, "is_causal", true);
    c.theta_local = c.theta;
  } else if (c.arch == inl::ARCH_MODERNBERT) {
    // crates/inl-sparse/src/modernbert.rs:28-166
    c.causal = false;
    c.norm_eps = static_cast<float>(num_or(root, "norm_eps", num_or(root, "layer_norm_eps", 1e-5)));
    double g = num_or(root, "global_rope_theta", 160000.0), l = num_or(root, "local_rope_theta", 10000.0);
    nested_theta(root, "full_attention", &g);
    nested_theta(root, "sliding_attention", &l);
    c.theta = g;
    c.theta_local = l;
    c.global_every = static_cast<int>(num_or(root, "global_attn_every_n_layers", 3));
    c.local_half_window = static_cast<int>(num_or(root, "local_attention", 128)) / 2;
    if (c.global_every <= 0) return fail(INL_ERR_CONFIG, "config: global_attn_every_n_layers must be positive");
    for (int i = 0; i < c.layers; ++i) c.layer_global[i] = (i % c.global_every) == 0;
    if (bool_or(root, "mlp_bias", false) || bool_or(root, "norm_bias", false) ||
        bool_or(root, "classifier_bias", false))
      return fail(INL_ERR_CONFIG, "config: biased ModernBERT mlp/norm/classifier weights are not supported");
    c.decoder_bias = bool_or(root, "decoder_bias", true);
    if (c.H % c.hq != 0) return fail(INL_ERR_CONFIG, "config: hidden_size must be a multiple of num_attention_heads");
    // SPLADE pooling (ShiftedTopKSpladePooling module config), nested under "splade"
    if (const inl::json::Value* sp = root.get("splade"); sp && sp->kind == inl::json::Value::Object) {
      c.logit_shift = static_cast<float>(num_or(*sp, "logit_shift", 0.0));
      c.prefix_ids = int_list(sp->get("prefix_token_ids"));
      c.masked_vocab_ids = int_list(sp->get("masked_vocab_ids"));
      c.canonical_ids = int_list(sp->get("canonical_ids"));
      if (!c.canonical_ids.empty() && static_cast<int>(c.canonical_ids.size()) != c.V)
        return fail(INL_ERR_CONFIG, "config: splade.canonical_ids must have vocab_size entries");
      for (int id : c.prefix_ids)
        if (id < 0 || id >= c.V) return fail(INL_ERR_CONFIG, "config: a prefix token id is outside the vocabulary");
      for (int id : c.masked_vocab_ids)
        if (id < 0 || id >= c.V) return fail(INL_ERR_CONFIG, "config: a masked vocab id is outside the vocabulary");
      for (int id : c.canonical_ids)
        if (id < 0) return fail(INL_ERR_CONFIG, "config: negative canonical id");
      const std::string strategy = str_or(*sp, "pooling_strategy", "max");
      const std::string act = str_or(*sp, "activation_function", "relu");
      if (strategy != "max" || act != "relu")
        return fail(INL_ERR_CONFIG, "config: only max pooling with relu activation is supported");
      if (num_or(*sp, "top_k", 0) > 0) return fail(INL_ERR_CONFIG, "config: SPLADE top_k is not supported");
    }
  } else if (c.arch == inl::ARCH_QWEN35) {
    // Qwen3.5 text tower of the late-interaction engine (crates/inl-late/src/qwen3_5.rs:56-168):
    // the same validation as Config::validate.
    c.causal = bool_or(root, "is_causal", true);
    if (!bool_or(root, "attn_output_gate", true))
      return fail(INL_ERR_CONFIG, "config: only gated Qwen3.5 attention is supported");
    if (str_or(root, "hidden_act", "silu") != "silu") return fail(INL_ERR_CONFIG, "config: hidden_act must be silu");
    c.lin_nk = static_cast<int>(num_or(root, "linear_num_key_heads", 0));
    c.lin_nv = static_cast<int>(num_or(root, "linear_num_value_heads", 0));
    c.lin_dk = static_cast<int>(num_or(root, "linear_key_head_dim", 0));
    c.lin_dv = static_cast<int>(num_or(root, "linear_value_head_dim", 0));
    c.conv_k = static_cast<int>(num_or(root, "linear_conv_kernel_dim", 4));
    if (c.lin_nk <= 0 || c.lin_nv <= 0 || c.lin_dk <= 0 || c.lin_dv <= 0 || c.conv_k <= 0 ||
        c.lin_nv % c.lin_nk != 0)
      return fail(INL_ERR_CONFIG, "config: invalid linear-attention head shapes");
    double theta = 10000.0, factor = 1.0;
    std::string rope_type = "default";
    if (const inl::json::Value* rp = root.get("rope_parameters"); rp && rp->kind == inl::json::Value::Object) {
      theta = num_or(*rp, "rope_theta", theta);
      factor = num_or(*rp, "partial_rotary_factor", factor);
      rope_type = str_or(*rp, "rope_type", rope_type);
    }
    if (rope_type != "default") return fail(INL_ERR_CONFIG, "config: unsupported rope_type " + rope_type);
    c.theta = theta;
    c.rot = static_cast<int>(c.d * factor);
    if (c.rot <= 0 || c.rot % 2 != 0 || c.rot > c.d)
      return fail(INL_ERR_CONFIG, "config: the rotary dimension must be even and at most head_dim");
    const inl::json::Value* kinds = root.get("layer_types");
    if (!kinds || kinds->kind != inl::json::Value::Array || static_cast<int>(kinds->arr.size()) != c.layers)
      return fail(INL_ERR_CONFIG, "config: layer_types must list every layer");
    c.layer_linear.assign(c.layers, 0);
    for (int i = 0; i < c.layers; ++i) {
      const std::string& k = kinds->arr[i].str;
      if (k != "linear_attention" && k != "full_attention")
        return fail(INL_ERR_CONFIG, "config: unsupported layer type " + k);
      c.layer_linear[i] = k == "linear_attention";
    }
  } else {
    // EmbeddingGemma-style tower (crates/inl-text/src/gemma2.rs:78-211)
    c.causal = false;
    c.sliding_window = static_cast<int>(num_or(root, "sliding_window", 512));
    double full = num_or(root, "rope_theta", 1000000.0), slide = num_or(root, "rope_local_base_freq", 10000.0);
    nested_theta(root, "full_attention", &full);
    nested_theta(root, "sliding_attention", &slide);
    if (const inl::json::Value* rp = root.get("rope_parameters"))  // Config::validate (gemma2.rs:157-164)
      for (const char* kind : {"full_attention", "sliding_attention"})
        if (const inl::json::Value* k = rp->get(kind))
          if (std::string t = str_or(*k, "rope_type", "default"); t != "default")
            return fail(INL_ERR_CONFIG, "config: rope_type \"" + t + "\" for " + kind);
    c.theta = full;
    c.theta_local = slide;
    c.attn_scale = 1.0f;  // unscaled scores: q and k are RMS-normalised per head
    const inl::json::Value* kinds = root.get("layer_types");
    if (kinds && kinds->kind == inl::json::Value::Array) {
      if (static_cast<int>(kinds->arr.size()) != c.layers)
        return fail(INL_ERR_CONFIG, "config: layer_types length differs from num_hidden_layers");
      for (int i = 0; i < c.layers; ++i) {
        const std::string& k = kinds->arr[i].str;
        if (k != "full_attention" && k != "sliding_attention")
          return fail(INL_ERR_CONFIG, "config: unknown layer type '" + k + "'");
        c.layer_global[i] = k == "full_attention";
      }
    } else {
      c.full_every = static_cast<int>(num_or(root, "full_attention_every_n_layers", 6));
      if (c.full_every <= 0) return fail(INL_ERR_CONFIG, "config: full_attention_every_n_layers must be positive");
      for (int i = 0; i < c.layers; ++i) c.layer_global[i] = (i % c.full_every) == c.full_every - 1;
    }
    // Per-layer head shapes (Config::layer / validate, crates/inl-text/src/gemma2.rs:150-204):
    // per_layer_config is keyed by the layer index ("05"); each entry may set
    // head_dim and num_key_value_heads. A key that is not a layer index is an error.
    c.layer_d.assign(c.layers, c.d);
    c.layer_kv.assign(c.layers, c.hkv);
    if (const inl::json::Value* plc = root.get("per_layer_config"); plc && plc->kind == inl::json::Value::Object) {
      for (const auto& [key, over] : plc->obj) {
        const size_t digits = key.find_first_not_of("0123456789");
        const bool numeric = !key.empty() && digits == std::string::npos && key.size() <= 9;
        const int index = numeric ? std::stoi(key) : -1;
        if (index < 0 || index >= c.layers)
          return fail(INL_ERR_CONFIG, "config: per_layer_config key \"" + key + "\" is not a layer index");
        if (const inl::json::Value* hd = over.get("head_dim"); hd && hd->is_num())
          c.layer_d[index] = static_cast<int>(hd->num);
        if (const inl::json::Value* kv = over.get("num_key_value_heads"); kv && kv->is_num())
          c.layer_kv[index] = static_cast<int>(kv->num);
      }
    }
    for (int l = 0; l < c.layers; ++l) {
      if (c.layer_d[l] <= 0 || (c.layer_d[l] & 1))
        return fail(INL_ERR_CONFIG, "config: head_dim " + std::to_string(c.layer_d[l]) + " of layer " +
                                        std::to_string(l));
      if (c.layer_kv[l] <= 0 || c.hq % c.layer_kv[l] != 0)
        return fail(INL_ERR_CONFIG, "config: " + std::to_string(c.hq) + " attention heads over " +
                                        std::to_string(c.layer_kv[l]) + " KV heads in layer " + std::to_string(l));
    }
    // One rotary table per layer kind, built for the head_dim of that kind's
    // first layer (gemma2.rs:566-572): every layer of a kind shares it.
    for (int l = 0; l < c.layers; ++l)
      for (int k = 0; k < l; ++k)
        if (c.layer_global[k] == c.layer_global[l] && c.layer_d[k] != c.layer_d[l])
          return fail(INL_ERR_CONFIG, "config: layers " + std::to_string(k) + " and " + std::to_string(l) +
                                          " are of one attention kind with different head_dim");
    c.ple = static_cast<int>(num_or(root, "hidden_size_per_layer_input", 0));
    if (c.ple < 0) return fail(INL_ERR_CONFIG, "config: hidden_size_per_layer_input must not be negative");
    const std::string act = str_or(root, "hidden_activation", "gelu_pytorch_tanh");
    if (act != "gelu_pytorch_tanh") return fail(INL_ERR_CONFIG, "config: hidden_activation must be gelu_pytorch_tanh");
    c.dense_dims = int_list(root.get("dense_dims"));
    if (c.dense_dims.empty() && num_or(root, "embedding_dim", 0) > 0)
      c.dense_dims.push_back(static_cast<int>(num_or(root, "embedding_dim", 0)));
  }
  return INL_OK;
}

// ------------------------------------------------------------ safetensors
struct MappedFile {
  void* base = nullptr;
  size_t size = 0;
  ~MappedFile() {
    if (base) munmap(base, size);
  }
};

int read_safetensors(const char* path, MappedFile& mf, TensorMap& out) {
  int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(INL_ERR_INFERENCE, std::string("cannot open ") + path);
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 8) {
    close(fd);
    return fail(INL_ERR_INFERENCE, std::string("bad safetensors file ") + path);
  }
  mf.size = static_cast<size_t>(st.st_size);
  mf.base = mmap(nullptr, mf.size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (mf.base == MAP_FAILED) {
    mf.base = nullptr;
    return fail(INL_ERR_INFERENCE, std::string("mmap failed for ") + path);
  }
  uint64_t hlen = 0;
  std::memcpy(&hlen, mf.base, 8);
  if (hlen + 8 > mf.size) return fail(INL_ERR_INFERENCE, "safetensors header overruns the file");
  std::string header(static_cast<const char*>(mf.base) + 8, hlen);
  inl::json::Value h;
  try {
    h = inl::json::parse(header);
  } catch (const std::exception& e) {
    return fail(INL_ERR_INFERENCE, std::string("safetensors header: ") + e.what());
  }
  const char* data = static_cast<const char*>(mf.base) + 8 + hlen;
  const size_t data_size = mf.size - 8 - hlen;
  for (const auto& kv : h.obj) {
    if (kv.first == "__metadata__") continue;
    const inl::json::Value& t = kv.second;
    const inl::json::Value* dt = t.get("dtype");
    const inl::json::Value* sh = t.get("shape");
    const inl::json::Value* off = t.get("data_offsets");
    if (!dt || !sh || !off || off->arr.size() != 2) return fail(INL_ERR_INFERENCE, "bad tensor entry " + kv.first);
    TensorSrc src;
    if (dt->str == "F32") src.bf16 = 0;
    else if (dt->str == "BF16") src.bf16 = 1;
    else continue;  // other dtypes are not model weights this library reads
    int64_t numel = 1;
    for (const auto& d : sh->arr) {
      src.shape.push_back(static_cast<int64_t>(d.num));
      numel *= static_cast<int64_t>(d.num);
    }
    const size_t b = static_cast<size_t>(off->arr[0].num), e = static_cast<size_t>(off->arr[1].num);
    if (e > data_size || b > e || (e - b) != static_cast<size_t>(numel) * (src.bf16 ? 2 : 4))
      return fail(INL_ERR_INFERENCE, "tensor " + kv.first + " has inconsistent offsets");
    src.data = data + b;
    src.numel = numel;
    out[kv.first] = src;
  }
  return INL_OK;
}

// ------------------------------------------------------------ weight upload
struct Loader {
  inl_model* m;
  const TensorMap& t;
  std::string prefix;  // tried as "<prefix>name" first, then "name"
  DevBuf staging;

  ~Loader() { staging.release(); }

  const TensorSrc* find(const std::string& name) const {
    if (!prefix.empty()) {
      auto it = t.find(prefix + name);
      if (it != t.end()) return &it->second;
    }
    auto it = t.find(name);
    return it == t.end() ? nullptr : &it->second;
  }

  void* alloc(size_t bytes) {
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) return nullptr;
    m->allocs.push_back(p);
    return p;
  }

  // Upload `name` ([rows, cols]) into dst rows remapped as (r / blk) * blk_stride + off + r % blk.
  int upload(const std::string& name, int rows, int cols, void* dst, int dst_bf16, long long ld_dst, int blk,
             long long blk_stride, long long off, const float* col_scale = nullptr) {
    return upload_part(name, rows, cols, 0, rows, dst, dst_bf16, ld_dst, blk, blk_stride, off, col_scale);
  }

  // Rows [row0, row0 + rows) of `name` ([total_rows, cols]) only.
  int upload_part(const std::string& name, int total_rows, int cols, int row0, int rows, void* dst, int dst_bf16,
                  long long ld_dst, int blk, long long blk_stride, long long off, const float* col_scale = nullptr) {
    const TensorSrc* s = find(name);
    if (!s) return fail(INL_ERR_INFERENCE, "missing weight " + prefix + name);
    if (s->numel != static_cast<int64_t>(total_rows) * cols)
      return fail(INL_ERR_INFERENCE, "weight " + name + " has " + std::to_string(s->numel) + " values, expected " +
                                         std::to_string(static_cast<long long>(total_rows) * cols));
    const size_t es_src = s->bf16 ? 2 : 4;
    const size_t bytes = static_cast<size_t>(rows) * cols * es_src;
    const char* src = static_cast<const char*>(s->data) + static_cast<size_t>(row0) * cols * es_src;
    INL_CUDA_TRY(staging.ensure(bytes), "staging allocation");
    // Stream-ordered copy: a pageable cudaMemcpy may return before its DMA lands,
    // and the model's non-blocking stream does not wait for the legacy stream.
    INL_CUDA_TRY(cudaMemcpyAsync(staging.p, src, bytes, cudaMemcpyHostToDevice, m->stream), "weight upload");
    int r = s->bf16 ? inl::convert_bf16_rows(staging.as<__nv_bfloat16>(), rows, cols, dst, dst_bf16, ld_dst, blk,
                                             blk_stride, off, m->stream, col_scale)
                    : inl::convert_rows(staging.as<float>(), rows, cols, dst, dst_bf16, ld_dst, blk, blk_stride, off,
                                        m->stream, col_scale);
    if (r != 0) return fail(INL_ERR_INFERENCE, "weight conversion launch failed");
    INL_CUDA_TRY(cudaStreamSynchronize(m->stream), "weight conversion");
    return INL_OK;
  }

  bool has(const std::string& name) const { return find(name) != nullptr; }

  int matrix_into(const std::string& name, int rows, int cols, void* dst, int as_bf16) {
    return upload(name, rows, cols, dst, as_bf16, cols, rows, 0, 0);
  }

  int matrix(const std::string& name, int rows, int cols, void** out, int as_bf16) {
    *out = alloc(static_cast<size_t>(rows) * cols * (as_bf16 ? 2 : 4));
    if (!*out) return fail(INL_ERR_INFERENCE, "out of device memory for " + name);
    return upload(name, rows, cols, *out, as_bf16, cols, rows, 0, 0);
  }

  int vec(const std::string& name, int n, float** out, bool optional = false, float fill = 1.f) {
    *out = static_cast<float*>(alloc(static_cast<size_t>(n) * 4));
    if (!*out) return fail(INL_ERR_INFERENCE, "out of device memory for " + name);
    if (!find(name)) {
      if (!optional) return fail(INL_ERR_INFERENCE, "missing weight " + prefix + name);
      std::vector<float> v(n, fill);
      INL_CUDA_TRY(cudaMemcpyAsync(*out, v.data(), static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, m->stream),
                   "fill");
      INL_CUDA_TRY(cudaStreamSynchronize(m->stream), "fill");
      return INL_OK;
    }
    return upload(name, 1, n, *out, 0, n, 1, 0, 0);
  }
};

int build_rope(inl_model* m, double theta, float** cos_out, float** sin_out, float** pairs_out = nullptr,
               int head_dim = 0) {
  const int d = head_dim > 0 ? head_dim : m->c.d;
  const int half = d / 2;
  const int P = m->c.max_pos;
  std::vector<float> c(static_cast<size_t>(P) * half), s(static_cast<size_t>(P) * half);
  // RotaryTable::new (crates/inl-text/src/qwen3/mod.rs:129-153): f64 angles, stored f32.
  std::vector<double> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = 1.0 / std::pow(theta, static_cast<double>(2 * i) / d);
  for (int p = 0; p < P; ++p)
    for (int i = 0; i < half; ++i) {
      const double a = static_cast<double>(p) * inv[i];
      c[static_cast<size_t>(p) * half + i] = static_cast<float>(std::cos(a));
      s[static_cast<size_t>(p) * half + i] = static_cast<float>(std::sin(a));
    }
  const size_t bytes = c.size() * 4;
  void *dc = nullptr, *ds = nullptr;
  INL_CUDA_TRY(cudaMalloc(&dc, bytes), "rope table");
  m->allocs.push_back(dc);
  INL_CUDA_TRY(cudaMalloc(&ds, bytes), "rope table");
  m->allocs.push_back(ds);
  INL_CUDA_TRY(cudaMemcpyAsync(dc, c.data(), bytes, cudaMemcpyHostToDevice, m->stream), "rope upload");
  INL_CUDA_TRY(cudaMemcpyAsync(ds, s.data(), bytes, cudaMemcpyHostToDevice, m->stream), "rope upload");
  INL_CUDA_TRY(cudaStreamSynchronize(m->stream), "rope upload");
  *cos_out = static_cast<float*>(dc);
  *sin_out = static_cast<float*>(ds);
  if (pairs_out) {
    // For the GEMM epilogue: [half / 2, P] float4 = (cos f, cos f+1, sin f, sin f+1), f = 2i.
    std::vector<float> pk(static_cast<size_t>(half) * P * 2);
    for (int i = 0; i < half / 2; ++i)
      for (int p = 0; p < P; ++p) {
        float* o = pk.data() + (static_cast<size_t>(i) * P + p) * 4;
        o[0] = c[static_cast<size_t>(p) * half + 2 * i];
        o[1] = c[static_cast<size_t>(p) * half + 2 * i + 1];
        o[2] = s[static_cast<size_t>(p) * half + 2 * i];
        o[3] = s[static_cast<size_t>(p) * half + 2 * i + 1];
      }
    void* dp = nullptr;
    INL_CUDA_TRY(cudaMalloc(&dp, pk.size() * 4), "rope table");
    m->allocs.push_back(dp);
    INL_CUDA_TRY(cudaMemcpyAsync(dp, pk.data(), pk.size() * 4, cudaMemcpyHostToDevice, m->stream), "rope upload");
    INL_CUDA_TRY(cudaStreamSynchronize(m->stream), "rope upload");
    *pairs_out = static_cast<float*>(dp);
  }
  return INL_OK;
}

// Shapes and dtypes the CUDA towers take, checked before any weight is read:
// the head_dim the RoPE and attention kernels of the dtype support, and the
// Qwen3.5 tower's f32.
bool head_dim_supported(int d, int bf16) {
  return bf16 ? (d == 64 || d == 128 || d == 256) : (d == 8 || d == 16 || d == 32 || d == 64 || d == 128 || d == 256);
}

int shape_support(const ModelConfig& c, int dtype) {
  const int bf = dtype == INL_DTYPE_BF16;
  if (c.arch == inl::ARCH_MODERNBERT && !head_dim_supported(c.d, bf))
    return fail(INL_ERR_CONFIG, "head_dim " + std::to_string(c.d) + " is not supported by the CUDA tower in " +
                                    (bf ? "bf16" : "f32"));
  if (c.arch == inl::ARCH_GEMMA)
    for (int l = 0; l < c.layers; ++l)
      if (!head_dim_supported(c.dl(l), bf))
        return fail(INL_ERR_CONFIG, "head_dim " + std::to_string(c.dl(l)) + " of layer " + std::to_string(l) +
                                        " is not supported by the CUDA tower in " + (bf ? "bf16" : "f32"));
  return INL_OK;
}

// Qwen3 weights (crates/inl-text/src/qwen3/mod.rs:180-330 tensor names).
int load_qwen3(inl_model* m, Loader& L) {
  const ModelConfig& c = m->c;
  const int bf = m->dtype == INL_DTYPE_BF16;
  const int q_out = c.hq * c.d, kv_out = c.hkv * c.d, qkv = q_out + 2 * kv_out;
  // gate/up interleaved in gate_block rows for the gated epilogue, else stored
  // [gate; up] and combined by a separate kernel.
  m->gated_split = (c.I % m->gate_block) != 0;
  const int gb = m->gated_split ? c.I : m->gate_block;
  const long long gstride = m->gated_split ? 0 : 2LL * gb;
  const long long up_off = m->gated_split ? c.I : gb;
  // Fused bf16 layer: folded input norms, q/k norm + RoPE in the QKV epilogue.
  m->fused = bf && !m->gated_split && (c.d == 64 || c.d == 128) && c.H % INL_SS_COLS == 0 && qkv % 256 == 0;
  int r;
  if ((r = L.matrix("embed_tokens.weight", c.V, c.H, &m->embed, bf))) return r;
  m->layers.resize(c.layers);
  for (int l = 0; l < c.layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    inl::LayerWeights& w = m->layers[l];
    const size_t es = bf ? 2 : 4;
    w.wqkv = L.alloc(static_cast<size_t>(qkv) * c.H * es);
    w.wo = L.alloc(static_cast<size_t>(c.H) * q_out * es);
    w.wgu = L.alloc(static_cast<size_t>(2) * c.I * c.H * es);
    w.wd = L.alloc(static_cast<size_t>(c.H) * c.I * es);
    if (!w.wqkv || !w.wo || !w.wgu || !w.wd) return fail(INL_ERR_INFERENCE, "out of device memory for weights");
    if ((r = L.vec(p + "self_attn.q_norm.weight", c.d, &w.qn))) return r;
    if ((r = L.vec(p + "self_attn.k_norm.weight", c.d, &w.kn))) return r;
    if ((r = L.vec(p + "input_layernorm.weight", c.H, &w.ln1))) return r;
    if ((r = L.vec(p + "post_attention_layernorm.weight", c.H, &w.ln2))) return r;
    // bf16: the input norms are folded into the projections that read them
    // (RMSNorm(x) W^T = rsqrt(mean x^2 + eps) * x (W diag(w))^T); the row scale
    // is applied in the GEMM epilogue from sums of squares the producer wrote.
    const float* f1 = m->fused ? w.ln1 : nullptr;
    const float* f2 = m->fused ? w.ln2 : nullptr;
    if ((r = L.upload(p + "self_attn.q_proj.weight", q_out, c.H, w.wqkv, bf, c.H, q_out, 0, 0, f1))) return r;
    if ((r = L.upload(p + "self_attn.k_proj.weight", kv_out, c.H, w.wqkv, bf, c.H, kv_out, 0, q_out, f1))) return r;
    if ((r = L.upload(p + "self_attn.v_proj.weight", kv_out, c.H, w.wqkv, bf, c.H, kv_out, 0, q_out + kv_out, f1)))
      return r;
    if ((r = L.upload(p + "self_attn.o_proj.weight", c.H, q_out, w.wo, bf, q_out, c.H, 0, 0))) return r;
    if ((r = L.upload(p + "mlp.gate_proj.weight", c.I, c.H, w.wgu, bf, c.H, gb, gstride, 0, f2))) return r;
    if ((r = L.upload(p + "mlp.up_proj.weight", c.I, c.H, w.wgu, bf, c.H, gb, gstride, up_off, f2))) return r;
    if ((r = L.upload(p + "mlp.down_proj.weight", c.H, c.I, w.wd, bf, c.I, c.H, 0, 0))) return r;
  }
  if ((r = L.vec("norm.weight", c.H, &m->final_norm))) return r;
  if ((r = build_rope(m, c.theta, &m->cos0, &m->sin0, &m->rope_pairs))) return r;
  return INL_OK;
}

// A zero-centred norm weight uploaded as its scale 1 + w (RmsNorm::load,
// crates/inl-late/src/qwen3_5.rs:194-201).
int vec_plus_one(inl_model* m, Loader& L, const std::string& name, int n, float** out) {
  const TensorSrc* t = L.find(name);
  if (!t) return fail(INL_ERR_INFERENCE, "missing weight " + L.prefix + name);
  if (t->numel != n) return fail(INL_ERR_INFERENCE, "weight " + name + " has the wrong size");
  std::vector<float> v(n);
  if (t->bf16) {
    const uint16_t* b = static_cast<const uint16_t*>(t->data);
    for (int i = 0; i < n; ++i) {
      const uint32_t bits = static_cast<uint32_t>(b[i]) << 16;
      std::memcpy(&v[i], &bits, 4);
    }
  } else {
    std::memcpy(v.data(), t->data, static_cast<size_t>(n) * 4);
  }
  for (float& x : v) x += 1.0f;
  *out = static_cast<float*>(L.alloc(static_cast<size_t>(n) * 4));
  if (!*out) return fail(INL_ERR_INFERENCE, "out of device memory for " + name);
  INL_CUDA_TRY(cudaMemcpyAsync(*out, v.data(), static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice, m->stream),
               "norm upload");
  INL_CUDA_TRY(cudaStreamSynchronize(m->stream), "norm upload");
  return INL_OK;
}

// cos / sin [max_pos, rot / 2] of position * inv_freq computed in f32, as
// rotary_tables does (crates/inl-late/src/qwen3_5.rs:940-958).
int build_rope_f32(inl_model* m, double theta, int rot) {
  const int half = rot / 2, P = m->c.max_pos;
  std::vector<float> c(static_cast<size_t>(P) * half), s(static_cast<size_t>(P) * half);
  const float th = static_cast<float>(theta);
  for (int i = 0; i < half; ++i) {
    const float inv = 1.0f / std::pow(th, static_cast<float>(2 * i) / static_cast<float>(rot));
    for (int p = 0; p < P; ++p) {
      const float ang = static_cast<float>(p) * inv;
      c[static_cast<size_t>(p) * half + i] = static_cast<float>(std::cos(static_cast<double>(ang)));
      s[static_cast<size_t>(p) * half + i] = static_cast<float>(std::sin(static_cast<double>(ang)));
    }
  }
  const size_t bytes = c.size() * 4;
  float *dc = nullptr, *ds = nullptr;
  INL_CUDA_TRY(cudaMalloc(&dc, bytes), "rope table");
  m->allocs.push_back(dc);
  INL_CUDA_TRY(cudaMalloc(&ds, bytes), "rope table");
  m->allocs.push_back(ds);
  INL_CUDA_TRY(cudaMemcpy(dc, c.data(), bytes, cudaMemcpyHostToDevice), "rope table");
  INL_CUDA_TRY(cudaMemcpy(ds, s.data(), bytes, cudaMemcpyHostToDevice), "rope table");
  m->cos0 = dc;
  m->sin0 = ds;
  return INL_OK;
}

// Qwen3.5 text tower (crates/inl-late/src/qwen3_5.rs:816-891 tensor names), f32.
int load_qwen35(inl_model* m, Loader& L) {
  const ModelConfig& c = m->c;
  if (int e = shape_support(c, m->dtype)) return e;
  const int nk = c.lin_nk, nv = c.lin_nv, dk = c.lin_dk, dv = c.lin_dv;
  const int conv_dim = 2 * nk * dk + nv * dv;
  const int lin_rows = conv_dim + nv * dv + 2 * nv;
  const int q_rows = c.hq * 2 * c.d, kv_rows = c.hkv * c.d;
  m->gated_split = (c.I % m->gate_block) != 0;
  const int gb = m->gated_split ? c.I : m->gate_block;
  const long long gstride = m->gated_split ? 0 : 2LL * gb;
  const long long up_off = m->gated_split ? c.I : gb;
  int r;
  if ((r = L.matrix("embed_tokens.weight", c.V, c.H, &m->embed, 0))) return r;
  m->layers.resize(c.layers);
  for (int l = 0; l < c.layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    inl::LayerWeights& w = m->layers[l];
    if ((r = vec_plus_one(m, L, p + "input_layernorm.weight", c.H, &w.ln1))) return r;
    if ((r = vec_plus_one(m, L, p + "post_attention_layernorm.weight", c.H, &w.ln2))) return r;
    if (c.layer_linear[l]) {
      const std::string a = p + "linear_attn.";
      w.w_lin_in = L.alloc(static_cast<size_t>(lin_rows) * c.H * 4);
      w.w_lin_out = L.alloc(static_cast<size_t>(c.H) * nv * dv * 4);
      w.conv_w = static_cast<float*>(L.alloc(static_cast<size_t>(conv_dim) * c.conv_k * 4));
      if (!w.w_lin_in || !w.w_lin_out || !w.conv_w) return fail(INL_ERR_INFERENCE, "out of device memory for weights");
      if ((r = L.upload(a + "in_proj_qkv.weight", conv_dim, c.H, w.w_lin_in, 0, c.H, conv_dim, 0, 0))) return r;
      if ((r = L.upload(a + "in_proj_z.weight", nv * dv, c.H, w.w_lin_in, 0, c.H, nv * dv, 0, conv_dim))) return r;
      if ((r = L.upload(a + "in_proj_b.weight", nv, c.H, w.w_lin_in, 0, c.H, nv, 0, conv_dim + nv * dv))) return r;
      if ((r = L.upload(a + "in_proj_a.weight", nv, c.H, w.w_lin_in, 0, c.H, nv, 0, conv_dim + nv * dv + nv)))
        return r;
      if ((r = L.upload(a + "out_proj.weight", c.H, nv * dv, w.w_lin_out, 0, nv * dv, c.H, 0, 0))) return r;
      if ((r = L.upload(a + "conv1d.weight", conv_dim, c.conv_k, w.conv_w, 0, c.conv_k, conv_dim, 0, 0))) return r;
      if ((r = L.vec(a + "dt_bias", nv, &w.dt_bias))) return r;
      if ((r = L.vec(a + "A_log", nv, &w.a_log))) return r;
      if ((r = L.vec(a + "norm.weight", dv, &w.lin_norm))) return r;
    } else {
      const std::string a = p + "self_attn.";
      w.wqkv = L.alloc(static_cast<size_t>(q_rows + 2 * kv_rows) * c.H * 4);
      w.wo = L.alloc(static_cast<size_t>(c.H) * c.hq * c.d * 4);
      if (!w.wqkv || !w.wo) return fail(INL_ERR_INFERENCE, "out of device memory for weights");
      if ((r = L.upload(a + "q_proj.weight", q_rows, c.H, w.wqkv, 0, c.H, q_rows, 0, 0))) return r;
      if ((r = L.upload(a + "k_proj.weight", kv_rows, c.H, w.wqkv, 0, c.H, kv_rows, 0, q_rows))) return r;
      if ((r = L.upload(a + "v_proj.weight", kv_rows, c.H, w.wqkv, 0, c.H, kv_rows, 0, q_rows + kv_rows))) return r;
      if ((r = L.upload(a + "o_proj.weight", c.H, c.hq * c.d, w.wo, 0, c.hq * c.d, c.H, 0, 0))) return r;
      if ((r = vec_plus_one(m, L, a + "q_norm.weight", c.d, &w.qn))) return r;
      if ((r = vec_plus_one(m, L, a + "k_norm.weight", c.d, &w.kn))) return r;
    }
    w.wgu = L.alloc(static_cast<size_t>(2) * c.I * c.H * 4);
    w.wd = L.alloc(static_cast<size_t>(c.H) * c.I * 4);
    if (!w.wgu || !w.wd) return fail(INL_ERR_INFERENCE, "out of device memory for weights");
    if ((r = L.upload(p + "mlp.gate_proj.weight", c.I, c.H, w.wgu, 0, c.H, gb, gstride, 0))) return r;
    if ((r = L.upload(p + "mlp.up_proj.weight", c.I, c.H, w.wgu, 0, c.H, gb, gstride, up_off))) return r;
    if ((r = L.upload(p + "mlp.down_proj.weight", c.H, c.I, w.wd, 0, c.I, c.H, 0, 0))) return r;
  }
  if ((r = vec_plus_one(m, L, "norm.weight", c.H, &m->final_norm))) return r;
  return build_rope_f32(m, c.theta, c.rot);
}

int upload_host(inl_model* m, void** dst, const void* src, size_t bytes) {
  void* p = nullptr;
  INL_CUDA_TRY(cudaMalloc(&p, std::max<size_t>(bytes, 4)), "device table");
  m->allocs.push_back(p);
  if (bytes) {
    INL_CUDA_TRY(cudaMemcpyAsync(p, src, bytes, cudaMemcpyHostToDevice, m->stream), "table upload");
    INL_CUDA_TRY(cudaStreamSynchronize(m->stream), "table upload");
  }
  *dst = p;
  return INL_OK;
}

// ModernBERT MLM (crates/inl-sparse/src/modernbert.rs:469-520 tensor names);
// the decoder is tied to the token embeddings.
int load_modernbert(inl_model* m, Loader& L) {
  const ModelConfig& c = m->c;
  const int bf = m->dtype == INL_DTYPE_BF16;
  m->gated_split = (c.I % m->gate_block) != 0;
  const int gb = m->gated_split ? c.I : m->gate_block;
  const long long gstride = m->gated_split ? 0 : 2LL * gb;
  const long long up_off = m->gated_split ? c.I : gb;
  int r;
  if ((r = shape_support(c, m->dtype))) return r;
  const size_t es = bf ? 2 : 4;
  if ((r = L.matrix("model.embeddings.tok_embeddings.weight", c.V, c.H, &m->embed, bf))) return r;
  if ((r = L.vec("model.embeddings.norm.weight", c.H, &m->emb_norm))) return r;
  m->layers.resize(c.layers);
  for (int l = 0; l < c.layers; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    inl::LayerWeights& w = m->layers[l];
    w.wqkv = L.alloc(static_cast<size_t>(3) * c.H * c.H * es);
    w.wo = L.alloc(static_cast<size_t>(c.H) * c.H * es);
    w.wgu = L.alloc(static_cast<size_t>(2) * c.I * c.H * es);
    w.wd = L.alloc(static_cast<size_t>(c.H) * c.I * es);
    if (!w.wqkv || !w.wo || !w.wgu || !w.wd) return fail(INL_ERR_INFERENCE, "out of device memory for weights");
    if (l > 0 && (r = L.vec(p + "attn_norm.weight", c.H, &w.ln1))) return r;  // layer 0: identity
    if ((r = L.vec(p + "mlp_norm.weight", c.H, &w.ln2))) return r;
    if ((r = L.matrix_into(p + "attn.Wqkv.weight", 3 * c.H, c.H, w.wqkv, bf))) return r;
    if ((r = L.matrix_into(p + "attn.Wo.weight", c.H, c.H, w.wo, bf))) return r;
    // Wi = [input (activated) ; gate] -> the gated epilogue's layout
    if ((r = L.upload_part(p + "mlp.Wi.weight", 2 * c.I, c.H, 0, c.I, w.wgu, bf, c.H, gb, gstride, 0))) return r;
    if ((r = L.upload_part(p + "mlp.Wi.weight", 2 * c.I, c.H, c.I, c.I, w.wgu, bf, c.H, gb, gstride, up_off)))
      return r;
    if ((r = L.matrix_into(p + "mlp.Wo.weight", c.H, c.I, w.wd, bf))) return r;
  }
  if ((r = L.vec("model.final_norm.weight", c.H, &m->final_norm))) return r;
  if ((r = L.matrix("head.dense.weight", c.H, c.H, &m->head_dense, bf))) return r;
  if ((r = L.vec("head.norm.weight", c.H, &m->head_norm))) return r;
  m->decoder_bias = nullptr;
  if (c.decoder_bias && L.has("decoder.bias") && (r = L.vec("decoder.bias", c.V, &m->decoder_bias))) return r;
  if ((r = build_rope(m, c.theta, &m->cos0, &m->sin0))) return r;
  if ((r = build_rope(m, c.theta_local, &m->cos1, &m->sin1))) return r;
  // SPLADE tables
  std::vector<float> open(c.V, 1.f);
  for (int id : c.masked_vocab_ids) open[id] = 0.f;
  void* p = nullptr;
  if ((r = upload_host(m, &p, open.data(), open.size() * 4))) return r;
  m->open_mask = static_cast<float*>(p);
  m->sparse_dim = c.V;
  if (!c.canonical_ids.empty()) {
    if ((r = upload_host(m, &p, c.canonical_ids.data(), c.canonical_ids.size() * 4))) return r;
    m->canon = static_cast<int*>(p);
    m->sparse_dim = *std::max_element(c.canonical_ids.begin(), c.canonical_ids.end()) + 1;
  }
  return INL_OK;
}

// EmbeddingGemma-style tower (crates/inl-text/src/gemma2.rs:233-494 tensor names):
// per-layer head shapes, the optional per-layer embeddings (PLE) and layer
// scalars; dense head chain kept in f32.
int load_gemma(inl_model* m, Loader& L) {
  const ModelConfig& c = m->c;
  const int bf = m->dtype == INL_DTYPE_BF16;
  m->gated_split = (c.I % m->gate_block) != 0;
  const int gb = m->gated_split ? c.I : m->gate_block;
  const long long gstride = m->gated_split ? 0 : 2LL * gb;
  const long long up_off = m->gated_split ? c.I : gb;
  int r;
  if ((r = shape_support(c, m->dtype))) return r;
  const bool ple = c.ple > 0;
  if (!ple && L.has("ple.per_layer_model_projection.weight"))
    return fail(INL_ERR_CONFIG, "checkpoint has per-layer embeddings but hidden_size_per_layer_input is 0");
  const size_t es = bf ? 2 : 4;
  if ((r = L.matrix("embed_tokens.weight", c.V, c.H, &m->embed, bf))) return r;
  if (ple) {  // PleBlock inputs (gemma2.rs:549-560, 626-630)
    if ((r = L.matrix("ple.per_layer_model_projection.weight", c.layers * c.ple, c.H, &m->ple_model_proj, bf))) return r;
    if ((r = L.vec("ple.per_layer_projection_norm.weight", c.ple, &m->ple_model_norm))) return r;
  }
  m->layers.resize(c.layers);
  for (int l = 0; l < c.layers; ++l) {
    const std::string p = "layers." + std::to_string(l) + ".";
    const int d = c.dl(l), q_out = c.hq * d, kv_out = c.kvl(l) * d, qkv = q_out + 2 * kv_out;
    inl::LayerWeights& w = m->layers[l];
    w.wqkv = L.alloc(static_cast<size_t>(qkv) * c.H * es);
    w.wo = L.alloc(static_cast<size_t>(c.H) * q_out * es);
    w.wgu = L.alloc(static_cast<size_t>(2) * c.I * c.H * es);
    w.wd = L.alloc(static_cast<size_t>(c.H) * c.I * es);
    if (!w.wqkv || !w.wo || !w.wgu || !w.wd) return fail(INL_ERR_INFERENCE, "out of device memory for weights");
    if ((r = L.upload(p + "self_attn.q_proj.weight", q_out, c.H, w.wqkv, bf, c.H, q_out, 0, 0))) return r;
    if ((r = L.upload(p + "self_attn.k_proj.weight", kv_out, c.H, w.wqkv, bf, c.H, kv_out, 0, q_out))) return r;
    if ((r = L.upload(p + "self_attn.v_proj.weight", kv_out, c.H, w.wqkv, bf, c.H, kv_out, 0, q_out + kv_out)))
      return r;
    if ((r = L.upload(p + "self_attn.o_proj.weight", c.H, q_out, w.wo, bf, q_out, c.H, 0, 0))) return r;
    if ((r = L.upload(p + "mlp.gate_proj.weight", c.I, c.H, w.wgu, bf, c.H, gb, gstride, 0))) return r;
    if ((r = L.upload(p + "mlp.up_proj.weight", c.I, c.H, w.wgu, bf, c.H, gb, gstride, up_off))) return r;
    if ((r = L.upload(p + "mlp.down_proj.weight", c.H, c.I, w.wd, bf, c.I, c.H, 0, 0))) return r;
    if ((r = L.vec(p + "self_attn.q_norm.weight", d, &w.qn))) return r;
    if ((r = L.vec(p + "self_attn.k_norm.weight", d, &w.kn))) return r;
    if ((r = L.vec(p + "input_layernorm.weight", c.H, &w.ln1))) return r;
    if ((r = L.vec(p + "post_attention_layernorm.weight", c.H, &w.ln1_post))) return r;
    if ((r = L.vec(p + "pre_feedforward_layernorm.weight", c.H, &w.ln2))) return r;
    if ((r = L.vec(p + "post_feedforward_layernorm.weight", c.H, &w.ln2_post))) return r;
    if (ple) {  // PleBlock and the layer scalar (gemma2.rs:264-272, 467-469)
      if ((r = L.matrix(p + "ple_block.per_layer_input_gate.weight", c.ple, c.H, &w.ple_gate, bf))) return r;
      if ((r = L.matrix(p + "ple_block.per_layer_projection.weight", c.H, c.ple, &w.ple_proj, bf))) return r;
      if ((r = L.vec(p + "ple_block.post_per_layer_input_norm.weight", c.H, &w.ple_norm))) return r;
      if ((r = L.vec(p + "layer_scalar", 1, &w.scalar))) return r;
    }
  }
  if ((r = L.vec("norm.weight", c.H, &m->final_norm))) return r;
  // Dense head: "dense_head.<j>.weight" chain, else the checkpoint's embedding_projection.
  int in = c.H;
  for (size_t j = 0; j < c.dense_dims.size(); ++j) {
    const std::string name =
        L.has("dense_head." + std::to_string(j) + ".weight") ? "dense_head." + std::to_string(j) + ".weight"
                                                             : "embedding_projection.weight";
    void* w = nullptr;
    if ((r = L.matrix(name, c.dense_dims[j], in, &w, 0))) return r;
    m->dense_chain.push_back(static_cast<float*>(w));
    in = c.dense_dims[j];
  }
  m->c.embed_scale = static_cast<float>(std::sqrt(static_cast<double>(c.H)));
  if (bf) {  // the reference multiplies by the scale cast to bf16 (crates/inl-text/src/gemma2.rs:575-587)
    m->c.embed_scale = __bfloat162float(__float2bfloat16_rn(m->c.embed_scale));
  }
  // One table per layer kind, for the head_dim of its first layer (gemma2.rs:566-572).
  int d_full = c.d, d_slide = c.d;
  for (int l = c.layers - 1; l >= 0; --l) (c.layer_global[l] ? d_full : d_slide) = c.dl(l);
  if ((r = build_rope(m, c.theta, &m->cos0, &m->sin0, nullptr, d_full))) return r;          // full layers
  if ((r = build_rope(m, c.theta_local, &m->cos1, &m->sin1, nullptr, d_slide))) return r;  // sliding layers
  return INL_OK;
}

int create_common(const char* config_json, int device, int dtype, inl_model** out, inl_model** mm) {
  if (!out) return fail(INL_ERR_CONFIG, "out is NULL");
  *out = nullptr;
  if (!config_json) return fail(INL_ERR_CONFIG, "config_json is NULL");
  if (dtype != INL_DTYPE_F32 && dtype != INL_DTYPE_BF16) return fail(INL_ERR_CONFIG, "unknown dtype");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0)
    return fail(INL_ERR_CONFIG, "no CUDA device is available");
  if (device < 0 || device >= ndev) return fail(INL_ERR_CONFIG, "device ordinal out of range");
  cudaDeviceProp prop;
  INL_CUDA_TRY(cudaGetDeviceProperties(&prop, device), "device query");
  if (prop.major != 10)
    return fail(INL_ERR_CONFIG, std::string("libinl_cuda is built for sm_100a (B200); device is ") + prop.name);
  INL_CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
  inl_model* m = new inl_model();
  m->dtype = dtype;
  m->api_dtype = dtype;
  m->device = device;
  m->gate_block = dtype == INL_DTYPE_BF16 ? 128 : 64;
  int r = parse_config(config_json, m->c);
  if (r) {
    delete m;
    return r;
  }
  if (m->c.arch == inl::ARCH_QWEN35 && dtype == INL_DTYPE_BF16) {
    // bf16 Qwen3.5 (accepted by the reference, crates/inl-late/src/native.rs:232):
    // the tower keeps f32 activations, norms and the gated delta rule, and runs
    // its GEMMs on bf16-rounded operands with f32 accumulation.
    m->dtype = INL_DTYPE_F32;
    m->gate_block = 64;
    m->f32_bf16_operands = true;
  }
  // f32 GEMMs on the tensor cores (3xBF16, relative error ~5e-6) except for
  // the Qwen3.5 late tower: its gated delta rule carries a state from token to
  // token, and the projections' error grows past the 1e-4 per component that
  // the reference holds its f32 tower to (crates/inl-late/tests/tiny_golden.rs),
  // so it keeps the SIMT FFMA GEMMs.
  m->f32_split3 = m->c.arch != inl::ARCH_QWEN35;
  // f32 towers on the 3xBF16 path interleave gate / up in 128-row blocks, the
  // block of the 256-wide CTA-pair tiles (64 would keep them on 128-wide
  // single-CTA tiles).
  if (m->dtype == INL_DTYPE_F32 && m->f32_split3) m->gate_block = 128;
  if (m->c.H % 8 != 0) {
    delete m;
    return fail(INL_ERR_CONFIG, "hidden_size must be a multiple of 8");
  }
  if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&m->d_status, sizeof(int)) != cudaSuccess ||
      cudaMallocHost(&m->h_status, sizeof(int)) != cudaSuccess ||
      cudaMemset(m->d_status, 0, sizeof(int)) != cudaSuccess) {
    inl_cuda_model_destroy(m);
    return fail(INL_ERR_INFERENCE, "stream / status allocation failed");
  }
  *mm = m;
  return INL_OK;
}

int load_weights(inl_model* m, const TensorMap& t) {
  Loader L{m, t, "", {}};
  // Qwen3-VL checkpoints nest the tower (crates/inl-text/src/qwen3/mod.rs:397-404).
  if (m->c.arch != inl::ARCH_MODERNBERT && !t.count("embed_tokens.weight")) {
    for (const char* p : {"model.language_model.", "model.", "language_model."})
      if (t.count(std::string(p) + "embed_tokens.weight")) {
        L.prefix = p;
        break;
      }
  }
  int r = INL_OK;
  switch (m->c.arch) {
    case inl::ARCH_QWEN3: r = load_qwen3(m, L); break;
    case inl::ARCH_MODERNBERT: r = load_modernbert(m, L); break;
    case inl::ARCH_GEMMA: r = load_gemma(m, L); break;
    case inl::ARCH_QWEN35: r = load_qwen35(m, L); break;
    default: r = fail(INL_ERR_CONFIG, "unknown architecture"); break;
  }
  return r;
}

// ------------------------------------------------------------ forward plan
struct Batch {
  int n = 0;
  int T = 0;
  int max_len = 0;
  int min_len = 0;
  const int32_t* cu_host = nullptr;
  // Causal last-token pooling reads only each text's last row: the last
  // layer then runs attention on the query tile holding that row and the o /
  // MLP projections on the n last rows alone (the row's value does not depend
  // on the other rows' outputs of that layer).
  bool last_only = false;
};

int check_inputs(inl_model* m, const uint32_t* ids, int ids_mem, const int32_t* cu, int n, Batch& b) {
  if (n < 0) return fail(INL_ERR_INVALID_INPUT, "n_texts is negative");
  if (n > 0 && (!cu || !ids)) return fail(INL_ERR_INVALID_INPUT, "ids / cu_seqlens is NULL");
  if (ids_mem != INL_MEM_HOST && ids_mem != INL_MEM_DEVICE) return fail(INL_ERR_INVALID_INPUT, "bad ids_mem");
  b.n = n;
  b.cu_host = cu;
  if (n == 0) return INL_OK;
  if (cu[0] != 0) return fail(INL_ERR_INVALID_INPUT, "cu_seqlens[0] must be 0");
  b.min_len = cu[1] - cu[0];
  for (int i = 0; i < n; ++i) {
    const int len = cu[i + 1] - cu[i];
    if (len < 0) return fail(INL_ERR_INVALID_INPUT, "cu_seqlens must be non-decreasing");
    b.min_len = std::min(b.min_len, len);
    if (len > m->c.max_pos)
      return fail(INL_ERR_INVALID_INPUT, "text " + std::to_string(i) + " has " + std::to_string(len) +
                                             " tokens; the model accepts at most " + std::to_string(m->c.max_pos));
    b.max_len = std::max(b.max_len, len);
  }
  b.T = cu[n];
  if (ids_mem == INL_MEM_HOST) {
    for (int t = 0; t < b.T; ++t)
      if (ids[t] >= static_cast<uint32_t>(m->c.V))
        return fail(INL_ERR_INVALID_INPUT, "token id " + std::to_string(ids[t]) + " at position " +
                                               std::to_string(t) + " is outside the vocabulary");
  }
  return INL_OK;
}

size_t es(const inl_model* m) { return m->dtype == INL_DTYPE_BF16 ? 2 : 4; }

// Token- and text-sized buffers are allocated in granules of 16384 tokens and
// 1024 texts. Batches planned under one token budget then share one allocation,
// and a batch slightly larger than the first one does not reallocate (cudaFree
// synchronises the device) in the middle of a stream of batches.
constexpr size_t kTokenGranule = 16384;
constexpr size_t kTextGranule = 1024;
size_t token_cap(int T) {
  return (static_cast<size_t>(std::max(T, 1)) + kTokenGranule - 1) / kTokenGranule * kTokenGranule;
}
size_t text_cap(int n) {
  return (static_cast<size_t>(std::max(n, 1)) + kTextGranule - 1) / kTextGranule * kTextGranule;
}

int ensure_workspace(inl_model* m, const Batch& b, int n_work) {
  const ModelConfig& c = m->c;
  const size_t T = token_cap(b.T);
  const size_t e = es(m);
  size_t qkv_cols = static_cast<size_t>(c.hq + 2 * c.hkv) * c.d;
  const size_t act_cols = static_cast<size_t>(c.I);
  size_t attn_cols = static_cast<size_t>(c.hq) * c.d;
  size_t tmp_cols = m->gated_split ? 2 * static_cast<size_t>(c.I) : 0;
  if (c.arch == inl::ARCH_QWEN35) {
    // q | gate rows or the stacked DeltaNet input projection; DeltaNet output;
    // the convolution output or the de-interleaved q heads.
    const size_t conv_dim = 2 * static_cast<size_t>(c.lin_nk) * c.lin_dk + static_cast<size_t>(c.lin_nv) * c.lin_dv;
    const size_t lin_cols = conv_dim + static_cast<size_t>(c.lin_nv) * c.lin_dv + 2 * static_cast<size_t>(c.lin_nv);
    qkv_cols = std::max(static_cast<size_t>(2 * c.hq + 2 * c.hkv) * c.d, lin_cols);
    attn_cols = std::max(attn_cols, static_cast<size_t>(c.lin_nv) * c.lin_dv);
    tmp_cols = std::max({tmp_cols, conv_dim, static_cast<size_t>(c.hq) * c.d});
  }
  if (c.arch == inl::ARCH_GEMMA) {
    // the widest layer's q | k | v and attention output; the PLE gate [T, ple]
    for (int l = 0; l < c.layers; ++l) {
      qkv_cols = std::max(qkv_cols, static_cast<size_t>(c.hq + 2 * c.kvl(l)) * c.dl(l));
      attn_cols = std::max(attn_cols, static_cast<size_t>(c.hq) * c.dl(l));
    }
    tmp_cols = std::max(tmp_cols, static_cast<size_t>(c.ple));
    if (c.ple > 0) INL_CUDA_TRY(m->ple_in.ensure(T * c.layers * c.ple * e), "workspace");
  }
  INL_CUDA_TRY(m->h.ensure(T * c.H * e), "workspace");
  INL_CUDA_TRY(m->xn.ensure(T * c.H * e), "workspace");
  INL_CUDA_TRY(m->qkv.ensure(T * std::max(qkv_cols, act_cols) * e), "workspace");
  INL_CUDA_TRY(m->attn.ensure(T * attn_cols * e), "workspace");
  if (tmp_cols) INL_CUDA_TRY(m->tmp.ensure(T * tmp_cols * e), "workspace");
  INL_CUDA_TRY(m->ids.ensure(T * 4), "workspace");
  const size_t parts = static_cast<size_t>((c.H + INL_SS_COLS - 1) / INL_SS_COLS);
  INL_CUDA_TRY(m->ss_a.ensure(T * parts * 4), "workspace");
  INL_CUDA_TRY(m->ss_b.ensure(T * parts * 4), "workspace");
  INL_CUDA_TRY(m->pos.ensure(T * 4), "workspace");
  INL_CUDA_TRY(m->cu.ensure((text_cap(b.n) + 1) * 4), "workspace");
  INL_CUDA_TRY(m->work.ensure(static_cast<size_t>(std::max(n_work, 1)) * 8), "workspace");
  if (m->qb_alt) INL_CUDA_TRY(m->work_alt.ensure(static_cast<size_t>(std::max(m->n_work_alt, 1)) * 8), "workspace");
  if (b.last_only) {
    // last-row buffers: h [n, H], attention rows [n, hq d], MLP rows [n, I] (bf16),
    // sums of squares [n, H / 64] (f32); the work list of last tiles and 0..n
    const size_t n = text_cap(b.n);
    const size_t parts_l = static_cast<size_t>((c.H + INL_SS_COLS - 1) / INL_SS_COLS);
    INL_CUDA_TRY(m->lastbuf.ensure(n * (c.H + static_cast<size_t>(c.hq) * c.d + c.I) * 2 + n * parts_l * 4 + 1024),
                 "workspace");
    INL_CUDA_TRY(m->work_last.ensure(n * 8 + (n + 1) * 4), "workspace");
  }
  const size_t stage = static_cast<size_t>(b.n + 1) * 4 + static_cast<size_t>(n_work + m->n_work_alt) * 8 +
                       (b.last_only ? static_cast<size_t>(b.n) * 8 + static_cast<size_t>(b.n + 1) * 4 : 0) + 64;
  if (stage > m->h_stage_bytes) {
    const size_t want = std::max({stage * 2, m->h_stage_bytes * 2, size_t(1) << 20});
    if (m->h_stage) {
      cudaStreamSynchronize(m->stream);  // the previous forward's copies may still read it
      cudaFreeHost(m->h_stage);
    }
    m->h_stage = nullptr;
    m->h_stage_bytes = 0;
    INL_CUDA_TRY(cudaMallocHost(&m->h_stage, want), "pinned staging");
    m->h_stage_bytes = want;
  }
  return INL_OK;
}

// Attention work items (text, query block of qb rows), heaviest first (key
// blocks a causal query block attends to, or the text's block count) so the
// long tails start early and the short items fill the gaps.
std::vector<std::pair<int, int2>> attention_work(const int* cu_host, int n, int qb, bool causal) {
  std::vector<std::pair<int, int2>> items;
  for (int i = 0; i < n; ++i) {
    const int L = cu_host[i + 1] - cu_host[i];
    const int nb = (L + qb - 1) / qb;
    for (int q = 0; q < nb; ++q) items.push_back({causal ? (q + 1) : nb, make_int2(i, q)});
  }
  std::stable_sort(items.begin(), items.end(), [](const auto& a, const auto& c) { return a.first > c.first; });
  return items;
}

int plan_and_upload(inl_model* m, const uint32_t* ids, int ids_mem, const Batch& b, int* n_work_out) {
  const int bf = m->dtype == INL_DTYPE_BF16;
  const int qb = inl::attention_q_block(bf, m->c.d);
  const std::vector<std::pair<int, int2>> items = attention_work(b.cu_host, b.n, qb, m->c.causal != 0);
  const int n_work = static_cast<int>(items.size());
  // A second list for layers whose head_dim takes another query block.
  m->qb_alt = 0;
  for (int l = 0; l < m->c.layers && !m->c.layer_d.empty(); ++l) {
    const int q = inl::attention_q_block(bf, m->c.dl(l));
    if (q != qb) m->qb_alt = q;
  }
  std::vector<std::pair<int, int2>> alt;
  if (m->qb_alt) alt = attention_work(b.cu_host, b.n, m->qb_alt, m->c.causal != 0);
  m->n_work_alt = static_cast<int>(alt.size());
  // Pruned last layer: the query tile holding each text's last row, heaviest
  // (most key blocks) first.
  std::vector<std::pair<int, int2>> last;
  if (b.last_only) {
    for (int i = 0; i < b.n; ++i) {
      const int q = (b.cu_host[i + 1] - b.cu_host[i] - 1) / qb;
      last.push_back({q, make_int2(i, q)});
    }
    std::stable_sort(last.begin(), last.end(), [](const auto& a, const auto& c) { return a.first > c.first; });
  }
  m->n_work_last = static_cast<int>(last.size());
  int r = ensure_workspace(m, b, n_work);
  if (r) return r;
  int* cu_stage = m->h_stage;
  std::memcpy(cu_stage, b.cu_host, static_cast<size_t>(b.n + 1) * 4);
  int2* work_stage = reinterpret_cast<int2*>(cu_stage + ((b.n + 1 + 3) & ~3));
  for (int i = 0; i < n_work; ++i) work_stage[i] = items[i].second;
  for (int i = 0; i < m->n_work_alt; ++i) work_stage[n_work + i] = alt[i].second;
  if (m->n_work_last > 0) {
    int2* last_stage = work_stage + n_work + m->n_work_alt;
    for (int i = 0; i < m->n_work_last; ++i) last_stage[i] = last[i].second;
    int* iota_stage = reinterpret_cast<int*>(last_stage + m->n_work_last);
    for (int i = 0; i <= b.n; ++i) iota_stage[i] = i;
    INL_CUDA_TRY(cudaMemcpyAsync(m->work_last.p, last_stage, static_cast<size_t>(m->n_work_last) * 8 +
                                                                 static_cast<size_t>(b.n + 1) * 4,
                                 cudaMemcpyHostToDevice, m->stream),
                 "work list upload");
  }
  if (m->n_work_alt > 0)
    INL_CUDA_TRY(cudaMemcpyAsync(m->work_alt.p, work_stage + n_work, static_cast<size_t>(m->n_work_alt) * 8,
                                 cudaMemcpyHostToDevice, m->stream),
                 "work list upload");
  INL_CUDA_TRY(cudaMemcpyAsync(m->cu.p, cu_stage, static_cast<size_t>(b.n + 1) * 4, cudaMemcpyHostToDevice,
                               m->stream),
               "cu_seqlens upload");
  if (n_work > 0)
    INL_CUDA_TRY(cudaMemcpyAsync(m->work.p, work_stage, static_cast<size_t>(n_work) * 8, cudaMemcpyHostToDevice,
                                 m->stream),
                 "work list upload");
  if (b.T > 0) {
    if (ids_mem == INL_MEM_HOST)
      INL_CUDA_TRY(cudaMemcpyAsync(m->ids.p, ids, static_cast<size_t>(b.T) * 4, cudaMemcpyHostToDevice, m->stream),
                   "ids upload");
    INL_K_TRY(inl::token_positions(m->cu.as<int>(), b.n, b.T, m->pos.as<int>(), m->stream), "positions");
    m->launches++;
  }
  *n_work_out = n_work;
  return INL_OK;
}

cudaEvent_t take_event(inl_model* m) {
  if (!m->event_pool.empty()) {
    cudaEvent_t e = m->event_pool.back();
    m->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e;
  cudaEventCreate(&e);
  return e;
}

// y = x . W^T with the model dtype's GEMM and a fused epilogue.
// The bf16 [rows, 3K] split of an f32 matrix (mode 1 [hi | lo | hi] for the
// weight side of a product, mode 0 [hi | hi | lo] for the activation side),
// made once on the model's stream and kept with the weights.
const void* split_weight(inl_model* m, const void* w, int rows, int K, int mode) {
  const uintptr_t key = reinterpret_cast<uintptr_t>(w) | static_cast<uintptr_t>(mode & 3);
  auto it = m->split_w.find(key);
  if (it != m->split_w.end()) return it->second;
  const int segs = mode == 2 ? 1 : 3;
  void* p = nullptr;
  if (cudaMalloc(&p, static_cast<size_t>(rows) * segs * K * 2) != cudaSuccess) return nullptr;
  m->allocs.push_back(p);
  if (inl::split3_bf16(static_cast<const float*>(w), K, rows, K, mode, p, static_cast<long long>(segs) * K,
                       m->stream) != 0)
    return nullptr;
  m->launches++;
  m->split_w[key] = p;
  return p;
}

// An f32 GEMM on the tensor cores: the activations are split into bf16
// [hi | hi | lo], the weight into [hi | lo | hi], and one bf16 GEMM over
// K' = 3K accumulates hi.hi + hi.lo + lo.hi in f32 (relative error ~5e-6,
// against ~2e-3 for a single bf16 product). The residual and gated epilogues
// then run as f32 passes. Returns -1 where a shape does not fit (the SIMT
// path runs instead).
int linear_split3(inl_model* m, const void* A, long long lda, const void* W, int M, int N, int K, int epi, int act,
                  void* out, long long ldo, const void* resid, long long ldr) {
  if ((K % 8) || (lda & 1) || (reinterpret_cast<uintptr_t>(A) & 7)) return -1;
  // one segment (a bf16 product) for a Qwen3.5 tower requested in bf16
  const bool one = m->f32_bf16_operands;
  const void* w3 = split_weight(m, W, N, K, one ? 2 : 1);
  if (!w3) return -3;
  const long long K3 = (one ? 1LL : 3LL) * K;
  if (m->split_a.ensure(token_cap(M) * K3 * 2) != cudaSuccess) return -3;
  if (inl::split3_bf16(static_cast<const float*>(A), lda, M, K, one ? 2 : 0, m->split_a.p, K3, m->stream)) return -3;
  m->launches++;
  const bool plain = epi == INL_EPI_F32 || epi == INL_EPI_BF16;
  // The residual add and the gated activation run in the GEMM's epilogue when
  // the f32 rows are 16-byte aligned (and, gated, the gate blocks match a tile
  // width); otherwise the product goes through scratch and a second kernel.
  const bool out_al = !(reinterpret_cast<uintptr_t>(out) & 15) && (ldo % 8) == 0;
  const bool fuse_resid = epi == INL_EPI_RESID_BF16 && out_al && resid &&
                          !(reinterpret_cast<uintptr_t>(resid) & 15) && (ldr % 4) == 0;
  const bool fuse_gated = epi == INL_EPI_GATED_BF16 && out_al && (m->gate_block == 64 || m->gate_block == 128) &&
                          (N % (2 * m->gate_block)) == 0;
  // Split-K when M is small: with fewer 256 x 256 tiles than half the SMs'
  // CTA pairs (config 1's 1,024 rows: 16 tiles for o and down), each tile's
  // K' is cut into up to 4 slices of at least 8 K blocks, written as f32
  // partial planes and summed in slice order with the residual by a second
  // kernel (deterministic).
  int splits = 1;
  if ((plain || epi == INL_EPI_RESID_BF16) && (N % 256) == 0 && N > 128 && out_al &&
      (epi != INL_EPI_RESID_BF16 || (resid && !(reinterpret_cast<uintptr_t>(resid) & 15) && (ldr % 4) == 0))) {
    const long long pairs = inl::num_sms_cached() / 2;
    const long long tiles = ((M + 255) / 256) * static_cast<long long>(N / 256);
    const int kb = static_cast<int>((K3 + 63) / 64);
    if (tiles * 2 <= pairs) {
      splits = static_cast<int>(std::min<long long>(4, pairs / tiles));
      while (splits > 1 && kb / splits < 8) --splits;
    }
  }
  if (splits > 1) {
    const size_t plane = static_cast<size_t>(M) * N;
    if (m->splitk_ws.ensure(plane * splits * 4) != cudaSuccess) return -3;
    inl::GemmArgs g;
    g.A = m->split_a.as<__nv_bfloat16>();
    g.lda = K3;
    g.W = static_cast<const __nv_bfloat16*>(w3);
    g.ldw = K3;
    g.M = M;
    g.N = N;
    g.K = static_cast<int>(K3);
    g.epi = INL_EPI_F32;
    g.out = m->splitk_ws.p;
    g.ldo = N;
    g.splits = splits;
    g.status = m->d_status;
    int r = inl::gemm_bf16_tn(g, m->stream);  // counted by linear()
    if (r) return r == -1 ? -1 : -3;
    r = inl::splits_reduce_f32(m->splitk_ws.as<float>(), static_cast<long long>(plane), N, splits, M, N,
                               epi == INL_EPI_RESID_BF16 ? static_cast<const float*>(resid) : nullptr, ldr,
                               static_cast<float*>(out), ldo, m->stream);
    if (r) return -3;
    m->launches++;
    return 0;
  }
  if (fuse_resid || fuse_gated) {
    inl::GemmArgs g;
    g.A = m->split_a.as<__nv_bfloat16>();
    g.lda = K3;
    g.W = static_cast<const __nv_bfloat16*>(w3);
    g.ldw = K3;
    g.M = M;
    g.N = N;
    g.K = static_cast<int>(K3);
    g.epi = fuse_resid ? INL_EPI_RESID_F32 : INL_EPI_GATED_F32;
    g.act = act;
    g.gate_block = m->gate_block;
    g.out = out;
    g.ldo = ldo;
    g.resid = static_cast<const __nv_bfloat16*>(resid);  // read as f32 by this epilogue
    g.ldr = ldr;
    g.status = m->d_status;
    const int r = inl::gemm_bf16_tn(g, m->stream);  // counted by linear()
    return r == 0 ? 0 : (r == -1 ? -1 : -3);
  }
  float* dst = static_cast<float*>(out);
  long long ldd = ldo;
  if (!plain || (reinterpret_cast<uintptr_t>(out) & 15) || (ldo % 8)) {
    if (m->split_c.ensure(token_cap(M) * static_cast<size_t>(N) * 4) != cudaSuccess) return -3;
    dst = m->split_c.as<float>();
    ldd = N;
  }
  inl::GemmArgs g;
  g.A = m->split_a.as<__nv_bfloat16>();
  g.lda = K3;
  g.W = static_cast<const __nv_bfloat16*>(w3);
  g.ldw = K3;
  g.M = M;
  g.N = N;
  g.K = static_cast<int>(K3);
  g.epi = INL_EPI_F32;
  g.out = dst;
  g.ldo = ldd;
  g.status = m->d_status;
  int r = inl::gemm_bf16_tn(g, m->stream);  // counted by linear()
  if (r) return r == -1 ? -1 : -3;
  if (epi == INL_EPI_RESID_BF16) {
    r = inl::add_rows_f32(static_cast<float*>(out), ldo, static_cast<const float*>(resid), ldr, dst, ldd, M, N,
                          m->stream);
  } else if (epi == INL_EPI_GATED_BF16) {
    r = inl::act_mul_blocks_f32(dst, ldd, M, N / 2, m->gate_block, act, static_cast<float*>(out), ldo, m->stream);
  } else if (dst != out) {
    r = cudaMemcpy2DAsync(out, ldo * 4, dst, ldd * 4, static_cast<size_t>(N) * 4, M, cudaMemcpyDeviceToDevice,
                          m->stream) == cudaSuccess ? 0 : -3;
  }
  if (!plain || dst != out) m->launches++;
  return r;
}

int linear(inl_model* m, const void* A, long long lda, const void* W, int M, int N, int K, int epi, int act,
           void* out, long long ldo, const void* resid, long long ldr, int kind) {
  ProfileRec rec{};
  if (m->profiling) {
    rec.start = take_event(m);
    rec.stop = take_event(m);
    rec.flops = 2.0 * M * N * K;
    rec.kind = kind;
    cudaEventRecord(rec.start, m->stream);
  }
  int r;
  if (m->dtype == INL_DTYPE_BF16) {
    inl::GemmArgs g;
    g.A = static_cast<const __nv_bfloat16*>(A);
    g.lda = lda;
    g.W = static_cast<const __nv_bfloat16*>(W);
    g.ldw = K;
    g.M = M;
    g.N = N;
    g.K = K;
    g.epi = epi;
    g.act = act;
    g.gate_block = m->gate_block;
    g.out = out;
    g.ldo = ldo;
    g.resid = static_cast<const __nv_bfloat16*>(resid);
    g.ldr = ldr;
    g.status = m->d_status;
    r = inl::gemm_bf16_tn(g, m->stream);
  } else {
    r = (m->f32_split3 || m->f32_bf16_operands) ? linear_split3(m, A, lda, W, M, N, K, epi, act, out, ldo, resid, ldr)
                                                : -1;
  }
  if (r == -1 && m->dtype != INL_DTYPE_BF16 && epi == INL_EPI_GATED_BF16 && m->gate_block != 64) {
    // The SIMT GEMM fuses the gated activation for 64-row gate blocks only:
    // other blocks take the f32 product into scratch, then the activation.
    if (m->split_c.ensure(token_cap(M) * static_cast<size_t>(N) * 4) != cudaSuccess) return -3;
    inl::GemmF32Args g;
    g.A = static_cast<const float*>(A);
    g.lda = lda;
    g.W = static_cast<const float*>(W);
    g.ldw = K;
    g.M = M;
    g.N = N;
    g.K = K;
    g.epi = INL_EPI_F32;
    g.out = m->split_c.as<float>();
    g.ldo = N;
    r = inl::gemm_f32_tn(g, m->stream);
    if (r == 0) {
      m->launches++;
      r = inl::act_mul_blocks_f32(m->split_c.as<float>(), N, M, N / 2, m->gate_block, act, static_cast<float*>(out),
                                  ldo, m->stream);
    }
  } else if (r == -1 && m->dtype != INL_DTYPE_BF16) {
    inl::GemmF32Args g;
    g.A = static_cast<const float*>(A);
    g.lda = lda;
    g.W = static_cast<const float*>(W);
    g.ldw = K;
    g.M = M;
    g.N = N;
    g.K = K;
    g.epi = epi == INL_EPI_BF16 ? INL_EPI_F32 : epi;
    g.act = act;
    g.gate_block = m->gate_block;
    g.out = static_cast<float*>(out);
    g.ldo = ldo;
    g.resid = static_cast<const float*>(resid);
    g.ldr = ldr;
    r = inl::gemm_f32_tn(g, m->stream);
  }
  m->launches++;
  if (m->profiling) {
    cudaEventRecord(rec.stop, m->stream);
    m->prof.push_back(rec);
  }
  return r;
}

// Profiling kind of attention launches (GEMM kinds are 0..99).
constexpr int kProfAttention = 100;

// Attention launch, bracketed by profiling events when profiling is on.
int run_attention(inl_model* m, const inl::AttnArgs& a, cudaStream_t s) {
  ProfileRec rec{};
  if (m->profiling) {
    rec.start = take_event(m);
    rec.stop = take_event(m);
    rec.kind = kProfAttention;
    cudaEventRecord(rec.start, s);
  }
  const int r = inl::attention(a, s);
  if (m->profiling) {
    cudaEventRecord(rec.stop, s);
    m->prof.push_back(rec);
  }
  return r;
}

// bf16 tcgen05 GEMM with every epilogue field (folded norm, QKV, residual sums).
int gemm(inl_model* m, inl::GemmArgs g, int kind) {
  ProfileRec rec{};
  if (m->profiling) {
    rec.start = take_event(m);
    rec.stop = take_event(m);
    rec.flops = 2.0 * g.M * g.N * g.K;
    rec.kind = kind;
    cudaEventRecord(rec.start, m->stream);
  }
  g.status = m->d_status;
  g.gate_block = m->gate_block;
  if (g.ldw == 0) g.ldw = g.K;
  const int r = inl::gemm_bf16_tn(g, m->stream);
  m->launches++;
  if (m->profiling) {
    cudaEventRecord(rec.stop, m->stream);
    m->prof.push_back(rec);
  }
  return r;
}

// The pruned last layer after its attention: the n last rows of the
// attention output and of h are gathered, then the o projection (residual,
// sums of squares for the folded norm), gate/up and down run on those rows
// alone. The result is h's last rows, [n, H] at the start of lastbuf.
int qwen3_last_rows(inl_model* m, const Batch& b, const inl::LayerWeights& w) {
  const ModelConfig& c = m->c;
  const size_t ncap = text_cap(b.n);
  const int q_out = c.hq * c.d;
  const int parts = (c.H + INL_SS_COLS - 1) / INL_SS_COLS;
  cudaStream_t s = m->stream;
  auto* base = static_cast<uint8_t*>(m->lastbuf.p);
  auto* h_last = reinterpret_cast<__nv_bfloat16*>(base);
  auto* a_last = reinterpret_cast<__nv_bfloat16*>(base + ncap * c.H * 2);
  auto* inter = reinterpret_cast<__nv_bfloat16*>(base + ncap * (c.H + q_out) * 2);
  auto* ss_last = reinterpret_cast<float*>(base + ncap * (c.H + q_out + c.I) * 2);
  INL_K_TRY(inl::gather_last_rows_bf16(m->attn.p, q_out, m->cu.as<int>(), b.n, q_out, a_last, q_out, s),
            "gather attention rows");
  INL_K_TRY(inl::gather_last_rows_bf16(m->h.p, c.H, m->cu.as<int>(), b.n, c.H, h_last, c.H, s), "gather rows");
  m->launches += 2;

  inl::GemmArgs o;
  o.A = a_last;
  o.lda = q_out;
  o.W = static_cast<const __nv_bfloat16*>(w.wo);
  o.M = b.n;
  o.N = c.H;
  o.K = q_out;
  o.epi = INL_EPI_RESID_BF16;
  o.out = h_last;
  o.ldo = c.H;
  o.resid = h_last;
  o.ldr = c.H;
  o.ss_out = ss_last;
  INL_K_TRY(gemm(m, o, 1), "o projection");

  inl::GemmArgs gu;
  gu.A = h_last;
  gu.lda = c.H;
  gu.W = static_cast<const __nv_bfloat16*>(w.wgu);
  gu.M = b.n;
  gu.N = 2 * c.I;
  gu.K = c.H;
  gu.epi = INL_EPI_GATED_BF16;
  gu.act = INL_ACT_SILU;
  gu.out = inter;
  gu.ldo = c.I;
  gu.ss_in = ss_last;
  gu.ss_in_parts = parts;
  gu.ss_dim = c.H;
  gu.ss_eps = c.eps;
  INL_K_TRY(gemm(m, gu, 2), "gate/up projection");

  inl::GemmArgs dn;
  dn.A = inter;
  dn.lda = c.I;
  dn.W = static_cast<const __nv_bfloat16*>(w.wd);
  dn.M = b.n;
  dn.N = c.H;
  dn.K = c.I;
  dn.epi = INL_EPI_RESID_BF16;
  dn.out = h_last;
  dn.ldo = c.H;
  dn.resid = h_last;
  dn.ldr = c.H;
  dn.ss_out = ss_last;
  INL_K_TRY(gemm(m, dn, 3), "down projection");
  return INL_OK;
}

// Fused bf16 layer stack: 4 GEMMs + attention per layer. The input RMSNorms
// are folded (weights scaled by the norm weight at load, row scale from the
// sums of squares the previous residual epilogue wrote); q/k RMSNorm + RoPE
// run in the QKV epilogue.
int qwen3_tower_fused(inl_model* m, const Batch& b, int n_work) {
  const ModelConfig& c = m->c;
  const int T = b.T;
  const int q_out = c.hq * c.d, kv_out = c.hkv * c.d, qkv_cols = q_out + 2 * kv_out;
  const int parts = (c.H + INL_SS_COLS - 1) / INL_SS_COLS;
  cudaStream_t s = m->stream;
  INL_K_TRY(inl::embed_gather(m->ids.as<uint32_t>(), T, m->embed, 1, c.V, c.H, 1.0f, m->h.p, 1, m->d_status, s,
                              m->ss_a.as<float>()),
            "embedding");
  m->launches++;
  const __nv_bfloat16* h = m->h.as<__nv_bfloat16>();
  for (int l = 0; l < c.layers; ++l) {
    const inl::LayerWeights& w = m->layers[l];
    const bool pruned = b.last_only && l == c.layers - 1;
    inl::GemmArgs g;
    g.A = h;
    g.lda = c.H;
    g.W = static_cast<const __nv_bfloat16*>(w.wqkv);
    g.M = T;
    g.N = qkv_cols;
    g.K = c.H;
    g.epi = INL_EPI_QKV;
    g.out = m->qkv.p;
    g.ldo = qkv_cols;
    g.ss_in = m->ss_a.as<float>();
    g.ss_in_parts = parts;
    g.ss_dim = c.H;
    g.ss_eps = c.eps;
    g.qn = w.qn;
    g.kn = w.kn;
    g.pos = m->pos.as<int>();
    g.cos = m->rope_pairs;
    g.sin = nullptr;
    g.hq = c.hq;
    g.hkv = c.hkv;
    g.d = c.d;
    g.max_pos = c.max_pos;
    g.qk_eps = c.eps;
    INL_K_TRY(gemm(m, g, 0), "qkv projection");

    inl::AttnArgs aa;
    aa.q = m->qkv.p;
    aa.k = m->qkv.as<__nv_bfloat16>() + q_out;
    aa.v = m->qkv.as<__nv_bfloat16>() + q_out + kv_out;
    aa.ldq = aa.ldk = aa.ldv = qkv_cols;
    aa.out = m->attn.p;
    aa.ldo = q_out;
    aa.bf16 = 1;
    aa.hq = c.hq;
    aa.hkv = c.hkv;
    aa.d = c.d;
    aa.scale = 1.0f / std::sqrt(static_cast<float>(c.d));
    aa.causal = c.causal ? 1 : 0;
    aa.window = -1;
    aa.cu = m->cu.as<int>();
    aa.n = b.n;
    aa.work = pruned ? m->work_last.as<int2>() : m->work.as<int2>();
    aa.n_work = pruned ? m->n_work_last : n_work;
    aa.q_block = inl::attention_q_block(1, c.d);
    aa.total_rows = T;
    aa.status = m->d_status;
    INL_K_TRY(run_attention(m, aa, s), "attention");
    m->launches++;
    if (pruned) {
      INL_K_TRY(qwen3_last_rows(m, b, w), "last-row projections");
      break;
    }

    inl::GemmArgs o;
    o.A = m->attn.as<__nv_bfloat16>();
    o.lda = q_out;
    o.W = static_cast<const __nv_bfloat16*>(w.wo);
    o.M = T;
    o.N = c.H;
    o.K = q_out;
    o.epi = INL_EPI_RESID_BF16;
    o.out = m->h.p;
    o.ldo = c.H;
    o.resid = h;
    o.ldr = c.H;
    o.ss_out = m->ss_b.as<float>();
    INL_K_TRY(gemm(m, o, 1), "o projection");

    inl::GemmArgs gu;
    gu.A = h;
    gu.lda = c.H;
    gu.W = static_cast<const __nv_bfloat16*>(w.wgu);
    gu.M = T;
    gu.N = 2 * c.I;
    gu.K = c.H;
    gu.epi = INL_EPI_GATED_BF16;
    gu.act = INL_ACT_SILU;
    gu.out = m->qkv.p;
    gu.ldo = c.I;
    gu.ss_in = m->ss_b.as<float>();
    gu.ss_in_parts = parts;
    gu.ss_dim = c.H;
    gu.ss_eps = c.eps;
    INL_K_TRY(gemm(m, gu, 2), "gate/up projection");

    inl::GemmArgs dn;
    dn.A = m->qkv.as<__nv_bfloat16>();
    dn.lda = c.I;
    dn.W = static_cast<const __nv_bfloat16*>(w.wd);
    dn.M = T;
    dn.N = c.H;
    dn.K = c.I;
    dn.epi = INL_EPI_RESID_BF16;
    dn.out = m->h.p;
    dn.ldo = c.H;
    dn.resid = h;
    dn.ldr = c.H;
    dn.ss_out = m->ss_a.as<float>();
    INL_K_TRY(gemm(m, dn, 3), "down projection");
  }
  return INL_OK;
}

// act(gate(x)) * up(x) -> out [T, I]: one GEMM with the gated epilogue, or a
// plain [T, 2I] GEMM plus act_mul when gate / up are stored split.
int mlp_gated(inl_model* m, const void* x, int T, const void* wgu, int act, void* out) {
  const ModelConfig& c = m->c;
  const int bf = m->dtype == INL_DTYPE_BF16;
  if (!m->gated_split)
    return linear(m, x, c.H, wgu, T, 2 * c.I, c.H, INL_EPI_GATED_BF16, act, out, c.I, nullptr, 0, 2);
  int r = linear(m, x, c.H, wgu, T, 2 * c.I, c.H, bf ? INL_EPI_BF16 : INL_EPI_F32, 0, m->tmp.p, 2 * c.I, nullptr, 0, 2);
  if (r) return r;
  m->launches++;
  return inl::act_mul(m->tmp.p, bf, T, c.I, act, out, m->stream);
}

// Embedding + every layer; leaves the last hidden state in m->h.
int qwen3_tower(inl_model* m, const Batch& b, int n_work) {
  const ModelConfig& c = m->c;
  const int bf = m->dtype == INL_DTYPE_BF16;
  const int T = b.T;
  const int q_out = c.hq * c.d, kv_out = c.hkv * c.d, qkv_cols = q_out + 2 * kv_out;
  cudaStream_t s = m->stream;
  INL_K_TRY(inl::embed_gather(m->ids.as<uint32_t>(), T, m->embed, bf, c.V, c.H, 1.0f, m->h.p, bf, m->d_status, s),
            "embedding");
  m->launches++;
  for (int l = 0; l < c.layers; ++l) {
    const inl::LayerWeights& w = m->layers[l];
    INL_K_TRY(inl::rms_norm(m->h.p, bf, c.H, w.ln1, c.eps, T, c.H, m->xn.p, bf, c.H, s), "input norm");
    m->launches++;
    INL_K_TRY(linear(m, m->xn.p, c.H, w.wqkv, T, qkv_cols, c.H, INL_EPI_BF16, 0, m->qkv.p, qkv_cols, nullptr, 0, 0),
              "qkv projection");
    inl::QkRopeArgs qa;
    qa.qkv = m->qkv.p;
    qa.bf16 = bf;
    qa.ld = qkv_cols;
    qa.T = T;
    qa.hq = c.hq;
    qa.hkv = c.hkv;
    qa.d = c.d;
    qa.qw = w.qn;
    qa.kw = w.kn;
    qa.eps = c.eps;
    qa.pos = m->pos.as<int>();
    qa.cos = m->cos0;
    qa.sin = m->sin0;
    qa.max_pos = c.max_pos;
    qa.status = m->d_status;
    INL_K_TRY(inl::qk_norm_rope(qa, s), "q/k norm + rope");
    m->launches++;
    inl::AttnArgs aa;
    const size_t e = es(m);
    aa.q = m->qkv.p;
    aa.k = static_cast<const char*>(m->qkv.p) + static_cast<size_t>(q_out) * e;
    aa.v = static_cast<const char*>(m->qkv.p) + static_cast<size_t>(q_out + kv_out) * e;
    aa.ldq = aa.ldk = aa.ldv = qkv_cols;
    aa.out = m->attn.p;
    aa.ldo = q_out;
    aa.bf16 = bf;
    aa.hq = c.hq;
    aa.hkv = c.hkv;
    aa.d = c.d;
    aa.scale = 1.0f / std::sqrt(static_cast<float>(c.d));
    aa.causal = c.causal ? 1 : 0;
    aa.window = -1;
    aa.cu = m->cu.as<int>();
    aa.n = b.n;
    aa.work = m->work.as<int2>();
    aa.n_work = n_work;
    aa.q_block = inl::attention_q_block(bf, c.d);
    aa.total_rows = T;
    aa.status = m->d_status;
    INL_K_TRY(run_attention(m, aa, s), "attention");
    m->launches++;
    INL_K_TRY(linear(m, m->attn.p, q_out, w.wo, T, c.H, q_out, INL_EPI_RESID_BF16, 0, m->h.p, c.H, m->h.p, c.H, 1),
              "o projection");
    INL_K_TRY(inl::rms_norm(m->h.p, bf, c.H, w.ln2, c.eps, T, c.H, m->xn.p, bf, c.H, s), "post-attention norm");
    m->launches++;
    INL_K_TRY(mlp_gated(m, m->xn.p, T, w.wgu, INL_ACT_SILU, m->qkv.p), "gate/up projection");
    INL_K_TRY(linear(m, m->qkv.p, c.I, w.wd, T, c.H, c.I, INL_EPI_RESID_BF16, 0, m->h.p, c.H, m->h.p, c.H, 3),
              "down projection");
  }
  return INL_OK;
}

inl::AttnArgs attn_args(inl_model* m, const Batch& b, int n_work, int qkv_cols, int q_out, int kv_out) {
  const ModelConfig& c = m->c;
  const size_t e = es(m);
  inl::AttnArgs aa;
  aa.q = m->qkv.p;
  aa.k = static_cast<const char*>(m->qkv.p) + static_cast<size_t>(q_out) * e;
  aa.v = static_cast<const char*>(m->qkv.p) + static_cast<size_t>(q_out + kv_out) * e;
  aa.ldq = aa.ldk = aa.ldv = qkv_cols;
  aa.out = m->attn.p;
  aa.ldo = q_out;
  aa.bf16 = m->dtype == INL_DTYPE_BF16;
  aa.hq = c.hq;
  aa.hkv = c.hkv;
  aa.d = c.d;
  aa.scale = 1.0f / std::sqrt(static_cast<float>(c.d));
  aa.causal = 0;
  aa.window = -1;
  aa.cu = m->cu.as<int>();
  aa.n = b.n;
  aa.work = m->work.as<int2>();
  aa.n_work = n_work;
  aa.q_block = inl::attention_q_block(aa.bf16, c.d);
  aa.total_rows = b.T;
  aa.status = m->d_status;
  return aa;
}

inl::QkRopeArgs rope_args(inl_model* m, int T, int qkv_cols, bool global) {
  const ModelConfig& c = m->c;
  inl::QkRopeArgs qa;
  qa.qkv = m->qkv.p;
  qa.bf16 = m->dtype == INL_DTYPE_BF16;
  qa.ld = qkv_cols;
  qa.T = T;
  qa.hq = c.hq;
  qa.hkv = c.hkv;
  qa.d = c.d;
  qa.eps = c.eps;
  qa.pos = m->pos.as<int>();
  qa.cos = global ? m->cos0 : m->cos1;
  qa.sin = global ? m->sin0 : m->sin1;
  qa.max_pos = c.max_pos;
  qa.status = m->d_status;
  return qa;
}

// ModernBERT tower (crates/inl-sparse/src/modernbert.rs:621-654); leaves the
// final-normed hidden state in m->h.
int modernbert_tower(inl_model* m, const Batch& b, int n_work) {
  const ModelConfig& c = m->c;
  const int bf = m->dtype == INL_DTYPE_BF16;
  const int T = b.T, H = c.H;
  const int qkv_cols = 3 * H;
  cudaStream_t s = m->stream;
  INL_K_TRY(inl::embed_gather(m->ids.as<uint32_t>(), T, m->embed, bf, c.V, H, 1.0f, m->h.p, bf, m->d_status, s),
            "embedding");
  INL_K_TRY(inl::layer_norm(m->h.p, bf, H, m->emb_norm, nullptr, c.norm_eps, T, H, m->h.p, bf, H, s),
            "embedding norm");
  m->launches += 2;
  for (int l = 0; l < c.layers; ++l) {
    const inl::LayerWeights& w = m->layers[l];
    const bool global = c.layer_global[l] != 0;
    const void* x = m->h.p;
    if (w.ln1) {  // layer 0 has no attention norm
      INL_K_TRY(inl::layer_norm(m->h.p, bf, H, w.ln1, nullptr, c.norm_eps, T, H, m->xn.p, bf, H, s), "attn norm");
      m->launches++;
      x = m->xn.p;
    }
    INL_K_TRY(linear(m, x, H, w.wqkv, T, qkv_cols, H, bf ? INL_EPI_BF16 : INL_EPI_F32, 0, m->qkv.p, qkv_cols, nullptr,
                     0, 0),
              "Wqkv");
    inl::QkRopeArgs qa = rope_args(m, T, qkv_cols, global);
    INL_K_TRY(inl::qk_norm_rope(qa, s), "rope");
    inl::AttnArgs aa = attn_args(m, b, n_work, qkv_cols, H, H);
    aa.window = global ? -1 : c.local_half_window;
    INL_K_TRY(run_attention(m, aa, s), "attention");
    m->launches += 2;
    INL_K_TRY(linear(m, m->attn.p, H, w.wo, T, H, H, INL_EPI_RESID_BF16, 0, m->h.p, H, m->h.p, H, 1), "Wo");
    INL_K_TRY(inl::layer_norm(m->h.p, bf, H, w.ln2, nullptr, c.norm_eps, T, H, m->xn.p, bf, H, s), "mlp norm");
    m->launches++;
    INL_K_TRY(mlp_gated(m, m->xn.p, T, w.wgu, INL_ACT_GELU_ERF, m->qkv.p), "Wi");
    INL_K_TRY(linear(m, m->qkv.p, c.I, w.wd, T, H, c.I, INL_EPI_RESID_BF16, 0, m->h.p, H, m->h.p, H, 3), "mlp Wo");
  }
  INL_K_TRY(inl::layer_norm(m->h.p, bf, H, m->final_norm, nullptr, c.norm_eps, T, H, m->h.p, bf, H, s),
            "final norm");
  m->launches++;
  return INL_OK;
}

// Attention arguments of one layer's head shape (per-layer head_dim and KV
// heads); the query block and work list follow the head_dim.
void layer_heads(inl_model* m, inl::AttnArgs& aa, int d, int kv) {
  aa.d = d;
  aa.hkv = kv;
  const int qb = inl::attention_q_block(aa.bf16, d);
  if (qb != aa.q_block && qb == m->qb_alt) {
    aa.q_block = qb;
    aa.work = m->work_alt.as<int2>();
    aa.n_work = m->n_work_alt;
  }
}

// EmbeddingGemma-style tower (crates/inl-text/src/gemma2.rs:473-494, 622-647);
// leaves the last hidden state (before the final norm) in m->h. Per layer:
// h += postN(Attn(inN(h))); h += postFF(MLP(preFF(h))); then, with per-layer
// embeddings, h = (h + postPLE(proj(gelu_tanh(gate(h)) * ple_l))) * scalar,
// where ple = RMSNorm(reshape(h0 W_ple^T * H^-1/2, [T, layers, ple])) of the
// scaled token embeddings h0.
int gemma_tower(inl_model* m, const Batch& b, int n_work) {
  const ModelConfig& c = m->c;
  const int bf = m->dtype == INL_DTYPE_BF16;
  const int T = b.T, H = c.H, P = c.ple;
  cudaStream_t s = m->stream;
  const int plain = bf ? INL_EPI_BF16 : INL_EPI_F32;
  const size_t e = es(m);
  INL_K_TRY(inl::embed_gather(m->ids.as<uint32_t>(), T, m->embed, bf, c.V, H, c.embed_scale, m->h.p, bf,
                              m->d_status, s),
            "embedding");
  m->launches++;
  if (P > 0) {  // per-layer inputs, once per forward (gemma2.rs:626-630)
    INL_K_TRY(linear(m, m->h.p, H, m->ple_model_proj, T, c.layers * P, H, plain, 0, m->ple_in.p, c.layers * P,
                     nullptr, 0, 7),
              "per-layer embedding projection");
    INL_K_TRY(inl::scaled_rms_norm(m->ple_in.p, bf, static_cast<long long>(T) * c.layers, P,
                                   static_cast<float>(std::pow(static_cast<double>(H), -0.5)), m->ple_model_norm,
                                   c.eps, s),
              "per-layer embedding norm");
    m->launches++;
  }
  for (int l = 0; l < c.layers; ++l) {
    const inl::LayerWeights& w = m->layers[l];
    const bool full = c.layer_global[l] != 0;
    const int d = c.dl(l), kv = c.kvl(l);
    const int q_out = c.hq * d, kv_out = kv * d, qkv_cols = q_out + 2 * kv_out;
    INL_K_TRY(inl::rms_norm(m->h.p, bf, H, w.ln1, c.eps, T, H, m->xn.p, bf, H, s), "input norm");
    INL_K_TRY(linear(m, m->xn.p, H, w.wqkv, T, qkv_cols, H, plain, 0, m->qkv.p, qkv_cols, nullptr, 0, 0), "qkv");
    inl::QkRopeArgs qa = rope_args(m, T, qkv_cols, full);
    qa.d = d;
    qa.hkv = kv;
    qa.qw = w.qn;
    qa.kw = w.kn;
    qa.v_norm = 1;
    INL_K_TRY(inl::qk_norm_rope(qa, s), "q/k/v norm + rope");
    inl::AttnArgs aa = attn_args(m, b, n_work, qkv_cols, q_out, kv_out);
    layer_heads(m, aa, d, kv);
    aa.scale = c.attn_scale;
    aa.window = full ? -1 : c.sliding_window;
    INL_K_TRY(run_attention(m, aa, s), "attention");
    m->launches += 3;
    INL_K_TRY(linear(m, m->attn.p, q_out, w.wo, T, H, q_out, plain, 0, m->xn.p, H, nullptr, 0, 1), "o projection");
    INL_K_TRY(inl::add_rms_norm(m->h.p, m->xn.p, bf, w.ln1_post, c.eps, T, H, s), "post-attention norm");
    INL_K_TRY(inl::rms_norm(m->h.p, bf, H, w.ln2, c.eps, T, H, m->xn.p, bf, H, s), "pre-feedforward norm");
    m->launches += 2;
    INL_K_TRY(mlp_gated(m, m->xn.p, T, w.wgu, INL_ACT_GELU_TANH, m->qkv.p), "gate/up projection");
    INL_K_TRY(linear(m, m->qkv.p, c.I, w.wd, T, H, c.I, plain, 0, m->xn.p, H, nullptr, 0, 3), "down projection");
    INL_K_TRY(inl::add_rms_norm(m->h.p, m->xn.p, bf, w.ln2_post, c.eps, T, H, s), "post-feedforward norm");
    m->launches++;
    if (P > 0) {  // PleBlock::forward and the layer scalar (gemma2.rs:279-283, 490-493)
      INL_K_TRY(linear(m, m->h.p, H, w.ple_gate, T, P, H, plain, 0, m->tmp.p, P, nullptr, 0, 7),
                "per-layer input gate");
      INL_K_TRY(inl::act_mul_rows(m->tmp.p, P, static_cast<const char*>(m->ple_in.p) + static_cast<size_t>(l) * P * e,
                                  static_cast<long long>(c.layers) * P, bf, T, P, INL_ACT_GELU_TANH, m->tmp.p, P, s),
                "per-layer gate");
      m->launches++;
      INL_K_TRY(linear(m, m->tmp.p, P, w.ple_proj, T, H, P, plain, 0, m->xn.p, H, nullptr, 0, 7),
                "per-layer projection");
      INL_K_TRY(inl::add_rms_norm(m->h.p, m->xn.p, bf, w.ple_norm, c.eps, T, H, s, w.scalar),
                "per-layer norm and scalar");
      m->launches++;
    }
  }
  return INL_OK;
}

// Qwen3.5 text tower of the late-interaction engine (Qwen35Text::forward,
// crates/inl-late/src/qwen3_5.rs:780-915), f32; leaves the last hidden state
// (before the final norm) in m->h. Per layer h += mixer(norm(h)), then
// h += MLP(norm(h)); the mixer is a Gated DeltaNet (one stacked input GEMM,
// causal convolution, recurrent delta rule with the gated norm fused, output
// GEMM) or gated full attention (q | gate, k, v GEMM; q / k norm and partial
// RoPE; attention; sigmoid gate; output GEMM).
int qwen35_tower(inl_model* m, const Batch& b, int n_work) {
  const ModelConfig& c = m->c;
  const int T = b.T;
  cudaStream_t s = m->stream;
  const int nk = c.lin_nk, nv = c.lin_nv, dk = c.lin_dk, dv = c.lin_dv;
  const int conv_dim = 2 * nk * dk + nv * dv;
  const int lin_cols = conv_dim + nv * dv + 2 * nv;
  const int q_rows = c.hq * 2 * c.d, kv = c.hkv * c.d, att_cols = q_rows + 2 * kv, q_out = c.hq * c.d;
  float* qkv = m->qkv.as<float>();
  INL_K_TRY(inl::embed_gather(m->ids.as<uint32_t>(), T, m->embed, 0, c.V, c.H, 1.0f, m->h.p, 0, m->d_status, s),
            "embedding");
  m->launches++;
  for (int l = 0; l < c.layers; ++l) {
    const inl::LayerWeights& w = m->layers[l];
    INL_K_TRY(inl::rms_norm(m->h.p, 0, c.H, w.ln1, c.eps, T, c.H, m->xn.p, 0, c.H, s), "input norm");
    m->launches++;
    if (c.layer_linear[l]) {
      INL_K_TRY(linear(m, m->xn.p, c.H, w.w_lin_in, T, lin_cols, c.H, INL_EPI_BF16, 0, qkv, lin_cols, nullptr, 0, 0),
                "linear-attention input projections");
      INL_K_TRY(inl::causal_conv_silu(qkv, lin_cols, T, conv_dim, w.conv_w, c.conv_k, m->pos.as<int>(),
                                      m->tmp.as<float>(), conv_dim, s),
                "causal convolution");
      m->launches++;
      inl::DeltaArgs da;
      da.mixed = m->tmp.as<float>();
      da.ld_mixed = conv_dim;
      da.z = qkv + conv_dim;
      da.ld_z = lin_cols;
      da.b_in = qkv + conv_dim + nv * dv;
      da.a_in = da.b_in + nv;
      da.ld_ab = lin_cols;
      da.dt_bias = w.dt_bias;
      da.a_log = w.a_log;
      da.norm_w = w.lin_norm;
      da.eps = c.eps;
      da.nk = nk;
      da.nv = nv;
      da.dk = dk;
      da.dv = dv;
      da.cu = m->cu.as<int>();
      da.n = b.n;
      da.out = m->attn.as<float>();
      da.ldo = nv * dv;
      INL_K_TRY(inl::gated_delta_rule(da, s), "gated delta rule");
      m->launches++;
      INL_K_TRY(linear(m, m->attn.p, nv * dv, w.w_lin_out, T, c.H, nv * dv, INL_EPI_RESID_BF16, 0, m->h.p, c.H, m->h.p,
                       c.H, 1),
                "linear-attention output projection");
    } else {
      INL_K_TRY(linear(m, m->xn.p, c.H, w.wqkv, T, att_cols, c.H, INL_EPI_BF16, 0, qkv, att_cols, nullptr, 0, 0),
                "q | gate, k, v projections");
      inl::Qwen35QkArgs qa;
      qa.qkv = qkv;
      qa.ld = att_cols;
      qa.q_out = m->tmp.as<float>();
      qa.ldq = q_out;
      qa.T = T;
      qa.hq = c.hq;
      qa.hkv = c.hkv;
      qa.d = c.d;
      qa.rot = c.rot;
      qa.qw = w.qn;
      qa.kw = w.kn;
      qa.eps = c.eps;
      qa.pos = m->pos.as<int>();
      qa.cos = m->cos0;
      qa.sin = m->sin0;
      qa.max_pos = c.max_pos;
      qa.status = m->d_status;
      INL_K_TRY(inl::qk_prep_gated(qa, s), "q / k norm and rope");
      m->launches++;
      inl::AttnArgs aa;
      aa.q = m->tmp.p;
      aa.ldq = q_out;
      aa.k = qkv + q_rows;
      aa.v = qkv + q_rows + kv;
      aa.ldk = aa.ldv = att_cols;
      aa.out = m->attn.p;
      aa.ldo = q_out;
      aa.bf16 = 0;
      aa.hq = c.hq;
      aa.hkv = c.hkv;
      aa.d = c.d;
      aa.scale = 1.0f / std::sqrt(static_cast<float>(c.d));
      aa.causal = c.causal ? 1 : 0;
      aa.window = -1;
      aa.cu = m->cu.as<int>();
      aa.n = b.n;
      aa.work = m->work.as<int2>();
      aa.n_work = n_work;
      aa.q_block = inl::attention_q_block(0, c.d);
      aa.total_rows = T;
      aa.status = m->d_status;
      INL_K_TRY(run_attention(m, aa, s), "attention");
      m->launches++;
      INL_K_TRY(inl::gate_sigmoid_mul(m->attn.as<float>(), q_out, qkv, att_cols, T, c.hq, c.d, s), "output gate");
      m->launches++;
      INL_K_TRY(linear(m, m->attn.p, q_out, w.wo, T, c.H, q_out, INL_EPI_RESID_BF16, 0, m->h.p, c.H, m->h.p, c.H, 1),
                "o projection");
    }
    INL_K_TRY(inl::rms_norm(m->h.p, 0, c.H, w.ln2, c.eps, T, c.H, m->xn.p, 0, c.H, s), "post-attention norm");
    m->launches++;
    INL_K_TRY(mlp_gated(m, m->xn.p, T, w.wgu, INL_ACT_SILU, qkv), "gate/up projection");
    INL_K_TRY(linear(m, qkv, c.I, w.wd, T, c.H, c.I, INL_EPI_RESID_BF16, 0, m->h.p, c.H, m->h.p, c.H, 3),
              "down projection");
  }
  return INL_OK;
}

int run_tower(inl_model* m, const uint32_t* ids, int ids_mem, const int32_t* cu, int n, Batch& b,
              bool last_token_pooling = false) {
  int r = check_inputs(m, ids, ids_mem, cu, n, b);
  if (r) return r;
  b.last_only = last_token_pooling && m->prune_last && m->fused && m->c.arch == inl::ARCH_QWEN3 && m->c.causal &&
                b.n > 0 && b.min_len > 0;
  INL_CUDA_TRY(cudaSetDevice(m->device), "cudaSetDevice");
  int n_work = 0;
  if ((r = plan_and_upload(m, ids, ids_mem, b, &n_work))) return r;
  if (b.T == 0) return INL_OK;
  if (ids_mem == INL_MEM_DEVICE)
    INL_CUDA_TRY(cudaMemcpyAsync(m->ids.p, ids, static_cast<size_t>(b.T) * 4, cudaMemcpyDeviceToDevice, m->stream),
                 "ids copy");
  switch (m->c.arch) {
    case inl::ARCH_QWEN3: return m->fused ? qwen3_tower_fused(m, b, n_work) : qwen3_tower(m, b, n_work);
    case inl::ARCH_MODERNBERT: return modernbert_tower(m, b, n_work);
    case inl::ARCH_GEMMA: return gemma_tower(m, b, n_work);
    case inl::ARCH_QWEN35: return qwen35_tower(m, b, n_work);
    default: return fail(INL_ERR_CONFIG, "model_type not built");
  }
}

// Check the device status word, then copy `bytes` of device results to the caller.
int finish(inl_model* m, const void* dev_src, size_t bytes, void* out, int out_mem) {
  INL_CUDA_TRY(cudaMemcpyAsync(m->h_status, m->d_status, sizeof(int), cudaMemcpyDeviceToHost, m->stream),
               "status read");
  if (bytes > 0 && out != dev_src) {
    const cudaMemcpyKind kind = out_mem == INL_MEM_DEVICE ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost;
    INL_CUDA_TRY(cudaMemcpyAsync(out, dev_src, bytes, kind, m->stream), "result copy");
  }
  INL_CUDA_TRY(cudaStreamSynchronize(m->stream), "forward");
  const int st = *m->h_status;
  if (st != 0) {
    cudaMemsetAsync(m->d_status, 0, sizeof(int), m->stream);
    cudaStreamSynchronize(m->stream);
    switch (st) {
      case INL_DEV_BAD_INDEX:
        return fail(INL_ERR_INVALID_INPUT, "a token id or position was outside the model's tables");
      default:
        return fail(INL_ERR_TIMEOUT, "a device wait ran past its limit (status " + std::to_string(st) + ")");
    }
  }
  return INL_OK;
}

}  // namespace

// ====================================================================== C ABI
extern "C" {

int inl_cuda_model_create_from_tensors(const char* config_json, int n_tensors, const char* const* names,
                                       const float* const* data, const int64_t* numels, int device, int dtype,
                                       inl_model** out) {
  inl_model* m = nullptr;
  int r = create_common(config_json, device, dtype, out, &m);
  if (r) return r;
  TensorMap t;
  for (int i = 0; i < n_tensors; ++i) {
    if (!names || !names[i] || !data || !data[i] || !numels) {
      inl_cuda_model_destroy(m);
      return fail(INL_ERR_CONFIG, "NULL tensor name or data");
    }
    TensorSrc s;
    s.data = data[i];
    s.numel = numels[i];
    t[names[i]] = s;
  }
  r = load_weights(m, t);
  if (r) {
    inl_cuda_model_destroy(m);
    return r;
  }
  *out = m;
  return INL_OK;
}

int inl_cuda_model_create(const char* config_json, const char* safetensors_path, int device, int dtype,
                          inl_model** out) {
  inl_model* m = nullptr;
  int r = create_common(config_json, device, dtype, out, &m);
  if (r) return r;
  if (!safetensors_path) {
    inl_cuda_model_destroy(m);
    return fail(INL_ERR_CONFIG, "safetensors_path is NULL");
  }
  // One file, or every shard of a model.safetensors.index.json; a tensor
  // named in two shards takes the later file's copy.
  std::vector<std::string> files;
  std::string error;
  if (!inl::checkpoint_files(safetensors_path, &files, &error)) {
    inl_cuda_model_destroy(m);
    return fail(INL_ERR_INFERENCE, error);
  }
  std::vector<std::unique_ptr<MappedFile>> maps;
  TensorMap t;
  for (const std::string& f : files) {
    maps.push_back(std::make_unique<MappedFile>());
    if ((r = read_safetensors(f.c_str(), *maps.back(), t))) break;
  }
  if (!r) r = load_weights(m, t);
  if (r) {
    inl_cuda_model_destroy(m);
    return r;
  }
  *out = m;
  return INL_OK;
}

int inl_cuda_model_set_dense_head(inl_model* m, const float* weight, int out_features, int in_features,
                                  const float* bias) {
  if (!m || !weight) return fail(INL_ERR_CONFIG, "NULL model or weight");
  if (in_features != m->c.H)
    return fail(INL_ERR_CONFIG, "Dense in_features must equal hidden_size (" + std::to_string(m->c.H) + ")");
  if (out_features <= 0) return fail(INL_ERR_CONFIG, "Dense out_features must be positive");
  if (m->dtype == INL_DTYPE_BF16 && out_features % 8 != 0)  // the bf16 GEMM's output rows are 16-byte aligned
    return fail(INL_ERR_CONFIG, "Dense out_features must be a multiple of 8 in bf16");
  INL_CUDA_TRY(cudaSetDevice(m->device), "cudaSetDevice");
  TensorMap t;
  TensorSrc w;
  w.data = weight;
  w.numel = static_cast<int64_t>(out_features) * in_features;
  t["linear.weight"] = w;
  if (bias) {
    TensorSrc b;
    b.data = bias;
    b.numel = out_features;
    t["linear.bias"] = b;
  }
  Loader L{m, t, "", {}};
  int r = L.matrix("linear.weight", out_features, in_features, &m->proj, m->dtype == INL_DTYPE_BF16);
  if (r) return r;
  m->proj_bias = nullptr;
  if (bias && (r = L.vec("linear.bias", out_features, &m->proj_bias))) return r;
  m->proj_out = out_features;
  return INL_OK;
}

int inl_cuda_model_set_dense_normalize(inl_model* m, int normalize) {
  if (!m) return fail(INL_ERR_CONFIG, "NULL model");
  m->proj_normalize = normalize != 0;
  return INL_OK;
}

int inl_cuda_forward_hidden(inl_model* m, const uint32_t* ids, int ids_mem, const int32_t* cu_seqlens, int n_texts,
                            int normalize_final, float* out, int out_mem) {
  if (!m) return fail(INL_ERR_CONFIG, "NULL model");
  Batch b;
  int r = run_tower(m, ids, ids_mem, cu_seqlens, n_texts, b);
  if (r) return r;
  if (b.T == 0) return INL_OK;
  const ModelConfig& c = m->c;
  const size_t bytes = static_cast<size_t>(b.T) * c.H * 4;
  INL_CUDA_TRY(m->out.ensure(token_cap(b.T) * c.H * 4), "output buffer");
  const int bf = m->dtype == INL_DTYPE_BF16;
  // (the ModernBERT tower already ends with its final LayerNorm)
  if (normalize_final && c.arch != inl::ARCH_MODERNBERT) {
    INL_K_TRY(inl::rms_norm(m->h.p, bf, c.H, m->final_norm, c.eps, b.T, c.H, m->out.p, 0, c.H, m->stream),
              "final norm");
  } else {
    if (bf) {
      INL_K_TRY(inl::convert_bf16_rows(m->h.as<__nv_bfloat16>(), b.T, c.H, m->out.p, 0, c.H, b.T, 0, 0, m->stream),
                "cast");
    } else {
      INL_CUDA_TRY(cudaMemcpyAsync(m->out.p, m->h.p, bytes, cudaMemcpyDeviceToDevice, m->stream), "copy");
    }
  }
  m->launches++;
  return finish(m, m->out.p, bytes, out, out_mem);
}

int inl_cuda_forward_dense(inl_model* m, const uint32_t* ids, int ids_mem, const int32_t* cu_seqlens, int n_texts,
                           int out_dim, float* out, int out_mem) {
  if (!m) return fail(INL_ERR_CONFIG, "NULL model");
  if (out_mem != INL_MEM_HOST && out_mem != INL_MEM_DEVICE) return fail(INL_ERR_INVALID_INPUT, "bad out_mem");
  const ModelConfig& c = m->c;
  if (out_dim != 0 && c.arch != inl::ARCH_GEMMA)
    return fail(INL_ERR_CONFIG, "output_dim is only supported for EmbeddingGemma-style models");
  if (c.arch == inl::ARCH_QWEN35)
    return fail(INL_ERR_CONFIG, "a Qwen3.5 late tower has no pooled dense head (use forward_multivector)");
  Batch b;
  int r = run_tower(m, ids, ids_mem, cu_seqlens, n_texts, b, c.arch == inl::ARCH_QWEN3);
  if (r) return r;
  if (b.n == 0) return INL_OK;
  if (!out) return fail(INL_ERR_INVALID_INPUT, "out is NULL");
  const int bf = m->dtype == INL_DTYPE_BF16;
  if (c.arch == inl::ARCH_MODERNBERT) return fail(INL_ERR_CONFIG, "a ModernBERT MLM model has no dense head");
  if (c.arch == inl::ARCH_GEMMA) {
    // final norm -> mean over each text's tokens -> dense chain -> L2 (x / sqrt(sum x^2 + 1e-12))
    // -> Matryoshka truncation (crates/inl-text/src/gemma2.rs:645-661, native.rs:822-830)
    const int D = c.dense_dims.empty() ? c.H : c.dense_dims.back();
    if (out_dim < 0 || out_dim > D) return fail(INL_ERR_CONFIG, "output_dim exceeds the model's embeddings");
    int widest = c.H;
    for (int d : c.dense_dims) widest = std::max(widest, d);
    INL_CUDA_TRY(m->pooled.ensure(text_cap(b.n) * widest * 4), "pooling buffer");
    INL_CUDA_TRY(m->head_buf.ensure(text_cap(b.n) * widest * 4), "pooling buffer");
    INL_K_TRY(inl::rms_norm(m->h.p, bf, c.H, m->final_norm, c.eps, b.T, c.H, m->xn.p, bf, c.H, m->stream),
              "final norm");
    INL_CUDA_TRY(m->seg_scratch.ensure(inl::segment_mean_scratch_bytes(b.n, c.H, b.max_len)), "pooling buffer");
    INL_K_TRY(inl::segment_mean(m->xn.p, bf, c.H, m->cu.as<int>(), b.n, c.H, b.max_len, m->seg_scratch.as<float>(),
                                m->pooled.as<float>(), m->stream),
              "mean pooling");
    m->launches += 3;
    float* cur = m->pooled.as<float>();
    float* nxt = m->head_buf.as<float>();
    int in = c.H;
    for (size_t j = 0; j < m->dense_chain.size(); ++j) {
      // f32 pooled rows through the f32 dense chain: 3xBF16 on the tensor
      // cores where it applies, the SIMT f32 GEMM otherwise
      int dr = m->f32_split3 ? linear_split3(m, cur, in, m->dense_chain[j], b.n, c.dense_dims[j], in, INL_EPI_F32, 0,
                                             nxt, c.dense_dims[j], nullptr, 0)
                             : -1;
      if (dr == -1) {
        inl::GemmF32Args g;
        g.A = cur;
        g.lda = in;
        g.W = m->dense_chain[j];
        g.ldw = in;
        g.M = b.n;
        g.N = c.dense_dims[j];
        g.K = in;
        g.epi = INL_EPI_F32;
        g.out = nxt;
        g.ldo = c.dense_dims[j];
        dr = inl::gemm_f32_tn(g, m->stream);
        m->launches++;
      }
      INL_K_TRY(dr, "dense head");
      std::swap(cur, nxt);
      in = c.dense_dims[j];
    }
    INL_K_TRY(inl::rows_l2_f32(cur, D, b.n, D, -1e-12f, cur, D, m->stream), "normalize");
    m->launches++;
    const int od = out_dim > 0 ? out_dim : D;
    const size_t obytes = static_cast<size_t>(b.n) * od * 4;
    INL_CUDA_TRY(m->out.ensure(text_cap(b.n) * od * 4), "output buffer");
    if (out_dim > 0) {
      INL_K_TRY(inl::truncate_normalize(cur, b.n, D, out_dim, m->out.as<float>(), m->stream), "matryoshka");
      m->launches++;
    } else {
      INL_CUDA_TRY(cudaMemcpyAsync(m->out.p, cur, obytes, cudaMemcpyDeviceToDevice, m->stream), "copy");
    }
    return finish(m, m->out.p, obytes, out, out_mem);
  }
  const size_t bytes = static_cast<size_t>(b.n) * c.H * 4;
  INL_CUDA_TRY(m->out.ensure(text_cap(b.n) * c.H * 4), "output buffer");
  if (b.last_only) {
    // the pruned last layer left each text's last row at row i of lastbuf
    const int* iota = reinterpret_cast<const int*>(m->work_last.as<int2>() + m->n_work_last);
    INL_K_TRY(inl::last_token_norm_l2(m->lastbuf.p, bf, c.H, iota, b.n, m->final_norm, c.eps, c.H,
                                      m->out.as<float>(), m->stream),
              "last-token pooling");
  } else {
    INL_K_TRY(inl::last_token_norm_l2(m->h.p, bf, c.H, m->cu.as<int>(), b.n, m->final_norm, c.eps, c.H,
                                      m->out.as<float>(), m->stream),
              "last-token pooling");
  }
  m->launches++;
  return finish(m, m->out.p, bytes, out, out_mem);
}

int inl_cuda_forward_multivector(inl_model* m, const uint32_t* ids, int ids_mem, const int32_t* cu_seqlens,
                                 int n_texts, float* out, int out_mem) {
  if (!m) return fail(INL_ERR_CONFIG, "NULL model");
  if (!m->proj) return fail(INL_ERR_CONFIG, "no Dense head attached (inl_cuda_model_set_dense_head)");
  const ModelConfig& c = m->c;
  Batch b;
  int r = run_tower(m, ids, ids_mem, cu_seqlens, n_texts, b);
  if (r) return r;
  if (b.T == 0) return INL_OK;
  if (!out) return fail(INL_ERR_INVALID_INPUT, "out is NULL");
  const int bf = m->dtype == INL_DTYPE_BF16;
  const size_t bytes = static_cast<size_t>(b.T) * m->proj_out * 4;
  INL_CUDA_TRY(m->out.ensure(token_cap(b.T) * m->proj_out * 4), "output buffer");
  // final norm on every token -> Dense projection (f32 out) -> F.normalize.
  INL_K_TRY(inl::rms_norm(m->h.p, bf, c.H, m->final_norm, c.eps, b.T, c.H, m->xn.p, bf, c.H, m->stream),
            "final norm");
  m->launches++;
  INL_K_TRY(linear(m, m->xn.p, c.H, m->proj, b.T, m->proj_out, c.H, INL_EPI_F32, 0, m->out.p, m->proj_out, nullptr,
                   0, 4),
            "dense projection");
  if (m->proj_bias || !m->proj_normalize) {
    // + bias, then F.normalize when the model has a Normalize module (native.rs:650-656)
    INL_K_TRY(inl::bias_rows_l2_f32(m->out.as<float>(), m->proj_out, b.T, m->proj_out, m->proj_bias,
                                    m->proj_normalize ? 1 : 0, 1e-12f, m->stream),
              "bias / normalize");
    m->launches++;
  } else {
    INL_K_TRY(inl::rows_l2_f32(m->out.as<float>(), m->proj_out, b.T, m->proj_out, 1e-12f, m->out.as<float>(),
                               m->proj_out, m->stream),
              "normalize");
    m->launches++;
  }
  return finish(m, m->out.p, bytes, out, out_mem);
}

}  // extern "C"

namespace {

// The SPLADE forward up to the dense term-weight rows [n, sparse_dim] f32 in
// m->out (device); b describes the batch.
int sparse_rows(inl_model* m, const uint32_t* ids, int ids_mem, const int32_t* cu_seqlens, int n_texts, Batch& b) {
  const ModelConfig& c = m->c;
  if (c.arch != inl::ARCH_MODERNBERT) return fail(INL_ERR_CONFIG, "this model has no SPLADE head");
  int r = run_tower(m, ids, ids_mem, cu_seqlens, n_texts, b);
  if (r) return r;
  if (b.n == 0) return INL_OK;
  const int bf = m->dtype == INL_DTYPE_BF16;
  const int H = c.H, V = c.V, n = b.n;
  cudaStream_t s = m->stream;
  // Speaking positions: every token whose id is not a prefix id
  // (Speakers::new, crates/inl-sparse/src/modernbert.rs:703-716), packed with
  // the index of their text.
  std::vector<int> idx, seg;
  idx.reserve(b.T);
  seg.reserve(b.T);
  std::vector<uint32_t> host_ids;
  const uint32_t* hid = ids;
  if (!c.prefix_ids.empty() && ids_mem == INL_MEM_DEVICE && b.T > 0) {
    host_ids.resize(b.T);
    INL_CUDA_TRY(cudaMemcpyAsync(host_ids.data(), m->ids.p, static_cast<size_t>(b.T) * 4, cudaMemcpyDeviceToHost, s),
                 "ids read-back");
    INL_CUDA_TRY(cudaStreamSynchronize(s), "ids read-back");
    hid = host_ids.data();
  }
  for (int i = 0; i < n; ++i)
    for (int t = b.cu_host[i]; t < b.cu_host[i + 1]; ++t) {
      if (!c.prefix_ids.empty() &&
          std::find(c.prefix_ids.begin(), c.prefix_ids.end(), static_cast<int>(hid[t])) != c.prefix_ids.end())
        continue;
      idx.push_back(t);
      seg.push_back(i);
    }
  const int Ts = static_cast<int>(idx.size());
  INL_CUDA_TRY(m->pooled_i.ensure(text_cap(n) * V * 4), "pooling buffer");
  INL_K_TRY(inl::fill_i32(m->pooled_i.as<int>(), static_cast<long long>(n) * V, inl::kOrderedNegInf, s), "fill");
  m->launches++;
  if (Ts > 0) {
    INL_CUDA_TRY(m->speak_idx.ensure(token_cap(Ts) * 4), "speaker index");
    INL_CUDA_TRY(m->speak_seg.ensure(token_cap(Ts) * 4), "speaker index");
    INL_CUDA_TRY(m->head_buf.ensure(token_cap(Ts) * H * es(m)), "head buffer");
    INL_CUDA_TRY(cudaMemcpyAsync(m->speak_idx.p, idx.data(), static_cast<size_t>(Ts) * 4, cudaMemcpyHostToDevice, s),
                 "speaker upload");
    INL_CUDA_TRY(cudaMemcpyAsync(m->speak_seg.p, seg.data(), static_cast<size_t>(Ts) * 4, cudaMemcpyHostToDevice, s),
                 "speaker upload");
    // MLM head on the speaking rows: LN(gelu_erf(dense(h))) (project, :657-662)
    INL_K_TRY(inl::gather_rows(m->h.p, bf, H, m->speak_idx.as<int>(), Ts, H, m->head_buf.p, s), "gather");
    m->launches++;
    INL_K_TRY(linear(m, m->head_buf.p, H, m->head_dense, Ts, H, H, bf ? INL_EPI_BF16 : INL_EPI_F32, 0, m->xn.p, H,
                     nullptr, 0, 5),
              "head dense");
    INL_K_TRY(inl::norm_act(m->xn.p, bf, H, m->head_norm, nullptr, c.norm_eps, Ts, H, m->xn.p, bf, H, s),
              "head norm");
    m->launches++;
    // Tied decoder reduced straight into per-text maxima: the [Ts, V] logits never reach memory.
    if (bf) {
      inl::GemmArgs g;
      g.A = static_cast<const __nv_bfloat16*>(m->embed);  // rows = vocabulary
      g.lda = H;
      g.W = m->xn.as<__nv_bfloat16>();  // columns = speaking tokens
      g.ldw = H;
      g.M = V;
      g.N = Ts;
      g.K = H;
      g.epi = INL_EPI_SEGMAX;
      g.seg = m->speak_seg.as<int>();
      g.pooled = m->pooled_i.as<int>();
      g.ldp = V;
      INL_K_TRY(gemm(m, g, 6), "decoder");
    } else {
      // f32: the tied table split as the activation side [hi | hi | lo] (rows =
      // vocabulary), the speaking rows as the weight side [hi | lo | hi], one
      // bf16 SEGMAX GEMM over K' = 3H; or the SIMT f32 SEGMAX GEMM.
      const void* t3 = m->f32_split3 && (H % 8) == 0 ? split_weight(m, m->embed, V, H, 0) : nullptr;
      if (t3) {
        INL_CUDA_TRY(m->split_a.ensure(token_cap(Ts) * 3 * static_cast<size_t>(H) * 2), "split buffer");
        INL_K_TRY(inl::split3_bf16(m->xn.as<float>(), H, Ts, H, 1, m->split_a.p, 3LL * H, s), "split");
        m->launches++;
        inl::GemmArgs g;
        g.A = static_cast<const __nv_bfloat16*>(t3);
        g.lda = 3LL * H;
        g.W = m->split_a.as<__nv_bfloat16>();
        g.ldw = 3LL * H;
        g.M = V;
        g.N = Ts;
        g.K = 3 * H;
        g.epi = INL_EPI_SEGMAX;
        g.seg = m->speak_seg.as<int>();
        g.pooled = m->pooled_i.as<int>();
        g.ldp = V;
        INL_K_TRY(gemm(m, g, 6), "decoder");
      } else {
        INL_K_TRY(inl::gemm_f32_segmax(m->xn.as<float>(), H, static_cast<const float*>(m->embed), H, Ts, V, H,
                                       m->speak_seg.as<int>(), m->pooled_i.as<int>(), V, s),
                  "decoder");
        m->launches++;
      }
    }
  }
  INL_CUDA_TRY(m->out.ensure(text_cap(n) * m->sparse_dim * 4), "output buffer");
  INL_K_TRY(inl::splade_finish(m->pooled_i.as<int>(), n, V, m->decoder_bias, c.logit_shift, m->open_mask, m->canon,
                               m->sparse_dim, m->out.as<float>(), s),
            "splade finish");
  m->launches++;
  return INL_OK;
}

}  // namespace

extern "C" {

int inl_cuda_forward_sparse(inl_model* m, const uint32_t* ids, int ids_mem, const int32_t* cu_seqlens, int n_texts,
                            float* out, int out_mem) {
  if (!m) return fail(INL_ERR_CONFIG, "NULL model");
  Batch b;
  int r = sparse_rows(m, ids, ids_mem, cu_seqlens, n_texts, b);
  if (r) return r;
  if (b.n == 0) return INL_OK;
  if (!out) return fail(INL_ERR_INVALID_INPUT, "out is NULL");
  return finish(m, m->out.p, static_cast<size_t>(b.n) * m->sparse_dim * 4, out, out_mem);
}

int inl_cuda_forward_sparse_compact(inl_model* m, const uint32_t* ids, int ids_mem, const int32_t* cu_seqlens,
                                    int n_texts, int64_t* offsets, int32_t* indices, float* values, int64_t capacity,
                                    int out_mem) {
  if (!m) return fail(INL_ERR_CONFIG, "NULL model");
  if (out_mem != INL_MEM_HOST && out_mem != INL_MEM_DEVICE) return fail(INL_ERR_INVALID_INPUT, "bad out_mem");
  if (n_texts > 0 && !offsets) return fail(INL_ERR_INVALID_INPUT, "offsets is NULL");
  Batch b;
  int r = sparse_rows(m, ids, ids_mem, cu_seqlens, n_texts, b);
  if (r) return r;
  if (b.n == 0) {
    if (offsets) offsets[0] = 0;
    return INL_OK;
  }
  const int n = b.n, D = m->sparse_dim;
  cudaStream_t s = m->stream;
  // pass 1: active terms per row (and a flag for non-finite weights)
  INL_CUDA_TRY(m->compact_meta.ensure((text_cap(n) + 1) * 8 + 64), "compaction buffer");
  int* d_counts = m->compact_meta.as<int>();
  int* d_bad = d_counts + n;  // read back with the counts
  INL_CUDA_TRY(cudaMemsetAsync(d_bad, 0, sizeof(int), s), "compaction");
  INL_K_TRY(inl::sparse_count(m->out.as<float>(), n, D, d_counts, d_bad, s), "sparse count");
  m->launches++;
  std::vector<int> counts(n + 1);
  INL_CUDA_TRY(cudaMemcpyAsync(counts.data(), d_counts, static_cast<size_t>(n + 1) * 4, cudaMemcpyDeviceToHost, s),
               "count read");
  r = finish(m, nullptr, 0, nullptr, INL_MEM_HOST);  // drains the stream, checks the device status word
  if (r) return r;
  if (counts[n] != 0)  // crates/inl-sparse/src/native.rs:536-540
    return fail(INL_ERR_INFERENCE, "non-finite SPLADE term weight");
  offsets[0] = 0;
  for (int i = 0; i < n; ++i) offsets[i + 1] = offsets[i] + counts[i];
  const int64_t total = offsets[n];
  if (total > capacity)
    return fail(INL_ERR_INVALID_INPUT, "the batch has " + std::to_string(total) + " active terms; capacity is " +
                                           std::to_string(capacity) + " (offsets[n_texts] holds the size needed)");
  if (total == 0) return INL_OK;
  if (!indices || !values) return fail(INL_ERR_INVALID_INPUT, "indices / values is NULL");
  // pass 2: every row's active terms in ascending term order at its offset
  INL_CUDA_TRY(m->compact_off.ensure((text_cap(n) + 1) * 8), "compaction buffer");
  INL_CUDA_TRY(cudaMemcpyAsync(m->compact_off.p, offsets, static_cast<size_t>(n + 1) * 8, cudaMemcpyHostToDevice, s),
               "offsets upload");
  int32_t* d_idx = indices;
  float* d_val = values;
  if (out_mem == INL_MEM_HOST) {
    INL_CUDA_TRY(m->compact_idx.ensure(static_cast<size_t>(total) * 4), "compaction buffer");
    INL_CUDA_TRY(m->compact_val.ensure(static_cast<size_t>(total) * 4), "compaction buffer");
    d_idx = m->compact_idx.as<int32_t>();
    d_val = m->compact_val.as<float>();
  }
  INL_K_TRY(inl::sparse_compact(m->out.as<float>(), n, D, m->compact_off.as<long long>(), d_idx, d_val, s),
            "sparse compaction");
  m->launches++;
  if (out_mem == INL_MEM_HOST) {
    INL_CUDA_TRY(cudaMemcpyAsync(indices, d_idx, static_cast<size_t>(total) * 4, cudaMemcpyDeviceToHost, s),
                 "result copy");
    INL_CUDA_TRY(cudaMemcpyAsync(values, d_val, static_cast<size_t>(total) * 4, cudaMemcpyDeviceToHost, s),
                 "result copy");
  }
  return finish(m, nullptr, 0, nullptr, INL_MEM_HOST);
}

int inl_cuda_model_info(const inl_model* m, inl_model_info* out) {
  if (!m || !out) return fail(INL_ERR_CONFIG, "NULL argument");
  out->arch = m->c.arch;
  out->dtype = m->api_dtype;
  out->device = m->device;
  out->hidden_size = m->c.H;
  out->num_layers = m->c.layers;
  out->vocab_size = m->c.V;
  out->dense_dim = (m->c.arch == inl::ARCH_GEMMA && !m->c.dense_dims.empty()) ? m->c.dense_dims.back() : m->c.H;
  out->multivector_dim = m->proj_out;
  out->sparse_dim = m->sparse_dim;
  out->max_text_tokens = m->c.max_pos;
  out->is_causal = m->c.causal ? 1 : 0;
  return INL_OK;
}

int inl_cuda_config_check(const char* config_json, int dtype, inl_model_info* out) {
  if (!config_json || !out) return fail(INL_ERR_CONFIG, "NULL argument");
  if (dtype != INL_DTYPE_F32 && dtype != INL_DTYPE_BF16) return fail(INL_ERR_CONFIG, "unknown dtype");
  ModelConfig c;
  int r = parse_config(config_json, c);
  if (r) return r;
  if (c.H % 8 != 0) return fail(INL_ERR_CONFIG, "hidden_size must be a multiple of 8");
  if ((r = shape_support(c, dtype))) return r;
  *out = inl_model_info{};
  out->arch = c.arch;
  out->dtype = dtype;
  out->device = -1;
  out->hidden_size = c.H;
  out->num_layers = c.layers;
  out->vocab_size = c.V;
  out->dense_dim = (c.arch == inl::ARCH_GEMMA && !c.dense_dims.empty()) ? c.dense_dims.back() : c.H;
  out->multivector_dim = 0;
  out->sparse_dim = c.arch != inl::ARCH_MODERNBERT ? 0
                    : c.canonical_ids.empty() ? c.V
                                              : *std::max_element(c.canonical_ids.begin(), c.canonical_ids.end()) + 1;
  out->max_text_tokens = c.max_pos;
  out->is_causal = c.causal ? 1 : 0;
  return INL_OK;
}

void inl_cuda_model_destroy(inl_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  if (m->stream) cudaStreamSynchronize(m->stream);
  for (void* p : m->allocs) cudaFree(p);
  for (DevBuf* d : {&m->h, &m->xn, &m->qkv, &m->attn, &m->ids, &m->cu, &m->pos, &m->work, &m->out, &m->pooled,
                    &m->tmp, &m->ss_a, &m->ss_b, &m->speak_idx, &m->speak_seg, &m->pooled_i, &m->head_buf,
                    &m->ple_in, &m->work_alt})
    d->release();
  for (auto& r : m->prof) {
    cudaEventDestroy(r.start);
    cudaEventDestroy(r.stop);
  }
  for (cudaEvent_t e : m->event_pool) cudaEventDestroy(e);
  if (m->h_stage) cudaFreeHost(m->h_stage);
  if (m->h_status) cudaFreeHost(m->h_status);
  if (m->d_status) cudaFree(m->d_status);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

int inl_cuda_last_error(char* buf, size_t len) {
  if (buf && len > 0) {
    const size_t n = std::min(len - 1, g_last_error.size());
    std::memcpy(buf, g_last_error.data(), n);
    buf[n] = '\0';
  }
  return static_cast<int>(g_last_error.size());
}

int inl_cuda_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

const char* inl_cuda_version(void) { return "inl_cuda 0.1.0 (sm_100a)"; }

// ---------------------------------------------------------------- profiling
int inl_cuda_model_set_f32_gemm(inl_model* m, int mode) {
  if (!m) return fail(INL_ERR_CONFIG, "NULL model");
  if (mode != 0 && mode != 1) return fail(INL_ERR_CONFIG, "f32 GEMM mode is 0 (SIMT FFMA) or 1 (3xBF16)");
  m->f32_split3 = mode == 1;
  return INL_OK;
}

int inl_cuda_model_set_prune_last(inl_model* m, int enable) {
  if (!m) return fail(INL_ERR_CONFIG, "NULL model");
  m->prune_last = enable != 0;
  return INL_OK;
}

int inl_cuda_model_set_profiling(inl_model* m, int enable) {
  if (!m) return fail(INL_ERR_CONFIG, "NULL model");
  cudaStreamSynchronize(m->stream);
  for (auto& r : m->prof) {
    m->event_pool.push_back(r.start);
    m->event_pool.push_back(r.stop);
  }
  m->prof.clear();
  m->profiling = enable != 0;
  // pre-create events so that timed runs never call cudaEventCreate
  while (m->profiling && m->event_pool.size() < 8192) {
    cudaEvent_t e;
    if (cudaEventCreate(&e) != cudaSuccess) break;
    m->event_pool.push_back(e);
  }
  return INL_OK;
}

int inl_cuda_model_profile(inl_model* m, int kind, int* launches, double* total_ms, double* flops) {
  if (!m) return fail(INL_ERR_CONFIG, "NULL model");
  INL_CUDA_TRY(cudaStreamSynchronize(m->stream), "profile sync");
  int n = 0;
  double ms = 0, fl = 0;
  for (const auto& r : m->prof) {
    if (kind >= 0 ? r.kind != kind : r.kind >= kProfAttention) continue;
    float t = 0;
    cudaEventElapsedTime(&t, r.start, r.stop);
    ms += t;
    fl += r.flops;
    ++n;
  }
  if (launches) *launches = n;
  if (total_ms) *total_ms = ms;
  if (flops) *flops = fl;
  return INL_OK;
}

long long inl_cuda_model_launch_count(inl_model* m, int reset) {
  if (!m) return -1;
  const long long n = m->launches;
  if (reset) m->launches = 0;
  return n;
}

void* inl_cuda_model_stream(inl_model* m) { return m ? static_cast<void*>(m->stream) : nullptr; }

// ------------------------------------------------------------ kernel hooks
int inl_cuda_gemm_bf16(const void* A, int64_t lda, const void* W, int64_t ldw, int M, int N, int K, int epi, int act,
                       int gate_block, void* out, int64_t ldo, const void* resid, int64_t ldr, int force_bn,
                       int* status, void* stream) {
  inl::GemmArgs g;
  g.A = static_cast<const __nv_bfloat16*>(A);
  g.lda = lda;
  g.W = static_cast<const __nv_bfloat16*>(W);
  g.ldw = ldw;
  g.M = M;
  g.N = N;
  g.K = K;
  g.epi = epi;
  g.act = act;
  g.gate_block = gate_block;
  g.out = out;
  g.ldo = ldo;
  g.resid = static_cast<const __nv_bfloat16*>(resid);
  g.ldr = ldr;
  g.status = status;
  g.force_bn = force_bn;
  const int r = inl::gemm_bf16_tn(g, static_cast<cudaStream_t>(stream));
  if (r == -1) return fail(INL_ERR_INVALID_INPUT, "gemm: unsupported shape / alignment / epilogue");
  if (r != 0) return fail(INL_ERR_INFERENCE, std::string("gemm launch failed: ") + cudaGetErrorString(cudaGetLastError()));
  return INL_OK;
}

int inl_cuda_gemm_bf16_ex(const inl_gemm_ex* a, void* stream) {
  if (!a) return fail(INL_ERR_CONFIG, "NULL args");
  inl::GemmArgs g;
  g.A = static_cast<const __nv_bfloat16*>(a->A);
  g.lda = a->lda;
  g.W = static_cast<const __nv_bfloat16*>(a->W);
  g.ldw = a->ldw;
  g.M = a->M;
  g.N = a->N;
  g.K = a->K;
  g.epi = a->epi;
  g.act = a->act;
  g.gate_block = a->gate_block;
  g.out = a->out;
  g.ldo = a->ldo;
  g.resid = static_cast<const __nv_bfloat16*>(a->resid);
  g.ldr = a->ldr;
  g.ss_in = a->ss_in;
  g.ss_in_parts = a->ss_in_parts;
  g.ss_dim = a->ss_dim;
  g.ss_eps = a->ss_eps;
  g.ss_out = a->ss_out;
  g.qn = a->qn;
  g.kn = a->kn;
  g.pos = a->pos;
  g.cos = a->cos;
  g.sin = a->sin;
  g.hq = a->hq;
  g.hkv = a->hkv;
  g.d = a->d;
  g.max_pos = a->max_pos;
  g.qk_eps = a->qk_eps;
  g.force_bn = a->force_bn;
  g.status = a->status;
  const int r = inl::gemm_bf16_tn(g, static_cast<cudaStream_t>(stream));
  if (r == -1) return fail(INL_ERR_INVALID_INPUT, "gemm: unsupported shape / alignment / epilogue");
  if (r != 0) return fail(INL_ERR_INFERENCE, std::string("gemm launch failed: ") + cudaGetErrorString(cudaGetLastError()));
  return INL_OK;
}

int inl_cuda_gemm_f32(const float* A, int64_t lda, const float* W, int64_t ldw, int M, int N, int K, int epi, int act,
                      float* out, int64_t ldo, const float* resid, int64_t ldr, void* stream) {
  inl::GemmF32Args g;
  g.A = A;
  g.lda = lda;
  g.W = W;
  g.ldw = ldw;
  g.M = M;
  g.N = N;
  g.K = K;
  g.epi = epi;
  g.act = act;
  g.out = out;
  g.ldo = ldo;
  g.resid = resid;
  g.ldr = ldr;
  const int r = inl::gemm_f32_tn(g, static_cast<cudaStream_t>(stream));
  if (r == -1) return fail(INL_ERR_INVALID_INPUT, "gemm_f32: unsupported shape / epilogue");
  if (r != 0) return fail(INL_ERR_INFERENCE, "gemm_f32 launch failed");
  return INL_OK;
}

}  // extern "C"

namespace inl {
// Sets the message inl_cuda_last_error returns on this thread; for entry
// points defined in other translation units.
int record_error(int code, const std::string& msg) { return fail(code, msg); }
}  // namespace inl

extern "C" {

static int hook_status(int r, const char* what) {
  if (r == -1) return fail(INL_ERR_INVALID_INPUT, std::string(what) + ": unsupported arguments");
  if (r != 0) return fail(INL_ERR_INFERENCE, std::string(what) + " launch failed");
  return INL_OK;
}

int inl_cuda_embed_gather(const uint32_t* ids, int T, const void* table, int table_dtype, int vocab, int H,
                          float scale, void* out, int out_dtype, int* status, void* stream) {
  return hook_status(inl::embed_gather(ids, T, table, table_dtype == INL_DTYPE_BF16, vocab, H, scale, out,
                                       out_dtype == INL_DTYPE_BF16, status, static_cast<cudaStream_t>(stream)),
                     "embed_gather");
}

int inl_cuda_norm(const void* x, int x_dtype, int64_t ldx, const float* w, const float* b, float eps, int layer_norm,
                  int rows, int H, void* out, int out_dtype, int64_t ldo, void* stream) {
  const int xb = x_dtype == INL_DTYPE_BF16, ob = out_dtype == INL_DTYPE_BF16;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return hook_status(layer_norm ? inl::layer_norm(x, xb, ldx, w, b, eps, rows, H, out, ob, ldo, s)
                                : inl::rms_norm(x, xb, ldx, w, eps, rows, H, out, ob, ldo, s),
                     "norm");
}

int inl_cuda_qk_norm_rope(void* qkv, int dtype, int64_t ld, int T, int hq, int hkv, int d, const float* qw,
                          const float* kw, int v_norm, float eps, const int32_t* pos, const float* cos,
                          const float* sin, int max_pos, int* status, void* stream) {
  inl::QkRopeArgs a;
  a.qkv = qkv;
  a.bf16 = dtype == INL_DTYPE_BF16;
  a.ld = ld;
  a.T = T;
  a.hq = hq;
  a.hkv = hkv;
  a.d = d;
  a.qw = qw;
  a.kw = kw;
  a.v_norm = v_norm;
  a.eps = eps;
  a.pos = pos;
  a.cos = cos;
  a.sin = sin;
  a.max_pos = max_pos;
  a.status = status;
  return hook_status(inl::qk_norm_rope(a, static_cast<cudaStream_t>(stream)), "qk_norm_rope");
}

int inl_cuda_token_positions(const int32_t* cu, int n, int T, int32_t* pos, void* stream) {
  return hook_status(inl::token_positions(cu, n, T, pos, static_cast<cudaStream_t>(stream)), "token_positions");
}

int inl_cuda_last_token_norm_l2(const void* h, int h_dtype, int64_t ldh, const int32_t* cu, int n, const float* w,
                                float eps, int H, float* out, void* stream) {
  return hook_status(inl::last_token_norm_l2(h, h_dtype == INL_DTYPE_BF16, ldh, cu, n, w, eps, H, out,
                                             static_cast<cudaStream_t>(stream)),
                     "last_token_norm_l2");
}

int inl_cuda_attention(const void* q, const void* k, const void* v, int64_t ldq, int64_t ldk, int64_t ldv, void* out,
                       int64_t ldo, int dtype, int hq, int hkv, int d, float scale, int causal, int window,
                       const int32_t* cu_seqlens_host, int n_texts, void* stream) {
  if (n_texts <= 0) return INL_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int qb = inl::attention_q_block(dtype == INL_DTYPE_BF16, d);
  if (!cu_seqlens_host) return fail(INL_ERR_CONFIG, "NULL cu_seqlens");
  if (cu_seqlens_host[0] != 0) return fail(INL_ERR_INVALID_INPUT, "cu_seqlens[0] must be 0");
  for (int i = 0; i < n_texts; ++i)
    if (cu_seqlens_host[i + 1] < cu_seqlens_host[i])
      return fail(INL_ERR_INVALID_INPUT, "cu_seqlens must be non-decreasing");
  std::vector<int2> work;
  for (const auto& it : attention_work(cu_seqlens_host, n_texts, qb, causal != 0)) work.push_back(it.second);
  // Hook scratch (device cu + work list), cached across calls so a timing
  // loop measures the kernel, not allocations; calls are serialised.
  static std::mutex hook_mu;
  static DevBuf hook_cu, hook_work;
  std::lock_guard<std::mutex> lock(hook_mu);
  INL_CUDA_TRY(hook_cu.ensure(static_cast<size_t>(n_texts + 1) * 4), "alloc");
  INL_CUDA_TRY(hook_work.ensure(std::max<size_t>(work.size(), 1) * 8), "alloc");
  int* dcu = hook_cu.as<int>();
  int2* dwork = hook_work.as<int2>();
  cudaMemcpyAsync(dcu, cu_seqlens_host, static_cast<size_t>(n_texts + 1) * 4, cudaMemcpyHostToDevice, s);
  if (!work.empty()) cudaMemcpyAsync(dwork, work.data(), work.size() * 8, cudaMemcpyHostToDevice, s);
  inl::AttnArgs a;
  a.q = q;
  a.k = k;
  a.v = v;
  a.ldq = ldq;
  a.ldk = ldk;
  a.ldv = ldv;
  a.out = out;
  a.ldo = ldo;
  a.bf16 = dtype == INL_DTYPE_BF16;
  a.hq = hq;
  a.hkv = hkv;
  a.d = d;
  a.scale = scale;
  a.causal = causal;
  a.window = window;
  a.cu = dcu;
  a.n = n_texts;
  a.work = dwork;
  a.n_work = static_cast<int>(work.size());
  a.q_block = qb;
  a.total_rows = cu_seqlens_host[n_texts];
  const int r = inl::attention(a, s);
  cudaStreamSynchronize(s);  // the host work list must outlive the copy
  if (r == -1) return fail(INL_ERR_INVALID_INPUT, "attention: unsupported head_dim / heads");
  if (r != 0) return fail(INL_ERR_INFERENCE, "attention launch failed");
  return INL_OK;
}

}  // extern "C"
