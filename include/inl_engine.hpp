// C++ host layer over libinl_cuda: the reference's engine interface for the
// encoder forward, in C++17. It mirrors crates/inl-core (InlError,
// BatchDeadline, the DenseEngine / SparseEngine / LateEngine contracts) and
// the host halves of crates/inl-text, crates/inl-sparse and crates/inl-late
// (planning, one forward at a time, a deadline per batch, results in input
// order, the count and finiteness checks), and calls the model through a
// Backend: the C ABI of include/inl_cuda.h (cuda_backend), or a test double.
//
// Inputs are token-id lists; tokenization stays with the caller (the
// reference tokenizes with the Rust tokenizers crate before these steps).
//
// Sources: im-not-llm_b200/host/engine.cpp (no CUDA) and
// im-not-llm_b200/host/cuda_backend.cpp (links libinl_cuda.so).
#pragma once

#include <cstddef>
#include <cstdint>
#include <functional>
#include <memory>
#include <mutex>
#include <optional>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace inl {

// ------------------------------------------------------------------ errors
// InlError and its variants (crates/inl-core/src/error.rs:5-46): the same
// stable codes and message prefixes.
class InlError : public std::runtime_error {
 public:
  InlError(std::string code, const std::string& prefix, const std::string& msg)
      : std::runtime_error(prefix + msg), code_(std::move(code)), message_(msg) {}
  const std::string& code() const { return code_; }
  const std::string& message() const { return message_; }

 private:
  std::string code_, message_;
};
struct ConfigError : InlError {
  explicit ConfigError(const std::string& m) : InlError("config", "config error: ", m) {}
};
struct InferenceError : InlError {
  explicit InferenceError(const std::string& m) : InlError("inference", "inference failed: ", m) {}
};
struct TimeoutError : InlError {
  explicit TimeoutError(const std::string& m) : InlError("timeout", "inference timeout: ", m) {}
};
struct InvalidInputError : InlError {
  explicit InvalidInputError(const std::string& m) : InlError("invalid_input", "invalid input: ", m) {}
};

// Throws the variant of an INL_* status (INL_OK returns).
void throw_status(int status, const std::string& message);

// ------------------------------------------------------------------ planning
// Input indices by length, longest first; ties keep input order
// (crates/inl-sparse/src/native.rs:548-552, crates/inl-late/src/native.rs:686-690).
std::vector<size_t> longest_first(const std::vector<size_t>& lengths);

// Consecutive ranges [first, second) whose real token sum stays within
// max_batch_tokens and whose size stays within max_texts (0 = unbounded);
// one text always forms a batch. Applied to lengths in longest_first order.
std::vector<std::pair<size_t, size_t>> plan_packed(const std::vector<size_t>& lengths, size_t max_batch_tokens,
                                                   size_t max_texts = 0);

struct Packed {
  std::vector<uint32_t> ids;  // concatenated token ids
  std::vector<int32_t> cu;    // n + 1 offsets, starting at 0
};
Packed pack(const std::vector<std::vector<uint32_t>>& texts, const std::vector<size_t>& members);

// ------------------------------------------------------------------ deadline
// BatchDeadline (crates/inl-core/src/deadline.rs:17-60): runs a task that
// cannot be cancelled on a worker thread and waits at most `budget` seconds.
// After one expiry the deadline is wedged: the stuck thread is left running
// and every later call fails fast with a TimeoutError without running its task.
class BatchDeadline {
 public:
  void ensure_healthy(const std::string& what) const;
  bool wedged() const;
  template <typename T>
  T run(const std::string& what, double budget_seconds, std::function<T()> task);

 private:
  void run_erased(const std::string& what, double budget_seconds, std::function<void()> task);
  std::shared_ptr<std::mutex> mu_ = std::make_shared<std::mutex>();
  std::shared_ptr<bool> wedged_ = std::make_shared<bool>(false);
};

template <typename T>
T BatchDeadline::run(const std::string& what, double budget_seconds, std::function<T()> task) {
  auto result = std::make_shared<std::optional<T>>();
  run_erased(what, budget_seconds, [result, task]() { result->emplace(task()); });
  return std::move(**result);
}

// ------------------------------------------------------------------ model
struct ModelInfo {
  int arch = 0;
  int hidden = 0;
  int dense_dim = 0;
  int sparse_dim = 0;
  int multivector_dim = 0;
  std::string dtype = "bf16";
  int device = 0;
};

struct SparseVector {  // crates/inl-sparse/src/lib.rs:51-62: sorted term ids, positive weights
  std::vector<uint32_t> indices;
  std::vector<float> values;
  static SparseVector from_dense(const float* row, size_t n);
};

// What the engines need from a loaded model. Outputs are row-major f32.
class Backend {
 public:
  virtual ~Backend() = default;
  virtual ModelInfo info() = 0;
  // [n, dense_dim or out_dim] unit vectors
  virtual std::vector<float> dense(const Packed& batch, int out_dim) = 0;
  // one SPLADE vector per text: active terms (weight > 0) in ascending term
  // order; a non-finite weight is an InferenceError
  virtual std::vector<SparseVector> sparse(const Packed& batch) = 0;
  // [total tokens, multivector_dim] per-token vectors in packed order
  virtual std::vector<float> multivector(const Packed& batch) = 0;
};

// Parses and validates a config.json text for dtype "bf16" or "f32" without a
// device (inl_cuda_config_check): the ModelInfo a load would report (device -1,
// multivector_dim 0), or the InlError a load would raise before reading weights.
ModelInfo check_config(const std::string& config_json, const std::string& dtype);

// The model on a GPU through include/inl_cuda.h; dtype "bf16" or "f32";
// safetensors_path is one file or a sharded checkpoint's index.json. For late
// models, dense_head_weight ([out, in] f32, may be empty), its optional bias
// [out] and whether the model has a Normalize module after the Dense.
std::unique_ptr<Backend> cuda_backend(const std::string& config_json, const std::string& safetensors_path, int device,
                                      const std::string& dtype, const std::vector<float>& dense_head_weight = {},
                                      int dense_out = 0, int dense_in = 0,
                                      const std::vector<float>& dense_head_bias = {}, bool dense_normalize = true);

// ------------------------------------------------------------------ engines
struct EngineInfo {  // crates/inl-core/src/engine.rs:10-26
  std::string model_id;
  int dimension = 0;
  std::string dtype;
  std::string device;
  std::string attention = "fused";
  int max_length = 0;
};

struct Options {  // the subset of TextOptions (crates/inl-text/src/native.rs:172-287) the packed path uses
  std::string id = "synthetic";
  size_t batch_size = 4096;
  size_t max_batch_tokens = 65536;
  size_t max_length = 2048;
  double timeout_seconds = 60;
  std::optional<double> per_batch_timeout_seconds;
  std::optional<int> output_dim;
  double batch_timeout() const;  // crates/inl-text/src/native.rs:739-752
};

using Tokens = std::vector<std::vector<uint32_t>>;
using Loader = std::function<std::unique_ptr<Backend>()>;

class EngineBase {
 public:
  EngineBase(Loader loader, Options options);
  virtual ~EngineBase();
  bool is_loaded() const;
  bool unload();
  std::vector<size_t> token_counts(const Tokens& texts) const;
  const Options& options() const { return options_; }
  BatchDeadline& deadline() { return deadline_; }

 protected:
  struct Loaded {
    std::unique_ptr<Backend> backend;
    std::mutex gate;  // one forward at a time (crates/inl-text/src/native.rs:668)
  };
  std::shared_ptr<Loaded> model();
  // Plans longest-first packed batches of `texts`, runs `forward` on each under
  // the deadline and puts the per-text results back in input order.
  template <typename R>
  std::vector<R> run_batches(const std::string& what, const Tokens& texts,
                             std::function<std::vector<R>(Backend&, const Packed&)> forward);

  Options options_;

 private:
  Loader loader_;
  mutable std::mutex load_mu_;
  std::shared_ptr<Loaded> loaded_;
  BatchDeadline deadline_;
};

// The embedding space of a TextEmbedder (crates/inl-text/src/native.rs:156-167).
struct TextIdentity {
  std::string id;
  int dimension = 0;
  std::string dtype;
  std::string device;  // "cuda"
  size_t max_length = 0;
};

// DenseEngine (crates/inl-core/src/engine.rs:66-84) as TextEmbedder implements it.
class TextEmbedder : public EngineBase {
 public:
  using EngineBase::EngineBase;
  EngineInfo load();
  TextIdentity identity();  // loads the model (native.rs:476-488)
  std::vector<std::vector<float>> embed(const Tokens& texts);
};

// SparseEngine (crates/inl-sparse/src/lib.rs:236-252). Construction refuses
// a zero timeout or batch_size with a ConfigError (native.rs:197-210).
class SparseEncoder : public EngineBase {
 public:
  SparseEncoder(Loader loader, Options options);
  EngineInfo load();
  EngineInfo identity() { return load(); }  // crates/inl-sparse/src/native.rs:271-283
  std::vector<SparseVector> encode(const Tokens& texts);
};

// One late task (TaskSetup, crates/inl-late/src/native.rs:122-128): context
// in tokens and the token ids whose vectors are dropped.
struct LateTask {
  size_t length = 2048;
  std::vector<uint32_t> skip;
};

// LateEngine (crates/inl-late/src/lib.rs:38-55): one vector per kept token.
// Construction refuses a zero timeout, batch_size or task length with a
// ConfigError (native.rs:184-202).
class LateEncoder : public EngineBase {
 public:
  LateEncoder(Loader loader, Options options, LateTask query = {}, LateTask document = {});
  EngineInfo load();
  EngineInfo identity() { return load(); }  // crates/inl-late/src/native.rs:256-270
  // task: "query" or "document"
  std::vector<std::vector<std::vector<float>>> encode(const Tokens& texts, const std::string& task = "document");
  // Tokens the model sees per input for `task`, after the task's cut
  // (LateEngine::token_counts, crates/inl-late/src/lib.rs:44-46).
  std::vector<size_t> token_counts(const Tokens& texts, const std::string& task = "document") const;

 private:
  const LateTask& setup(const std::string& task) const;
  LateTask query_, document_;
};

}  // namespace inl
