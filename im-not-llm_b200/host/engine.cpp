// C++ host layer over libinl_cuda (see include/inl_engine.hpp): planning,
// the batch deadline and the three engines. No CUDA here: the model is a
// Backend (cuda_backend.cpp, or a test double).
#include <algorithm>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <exception>
#include <numeric>
#include <thread>

#include "../../include/inl_cuda.h"
#include "../../include/inl_engine.hpp"

namespace inl {

void throw_status(int status, const std::string& message) {
  switch (status) {
    case INL_OK: return;
    case INL_ERR_CONFIG: throw ConfigError(message);
    case INL_ERR_TIMEOUT: throw TimeoutError(message);
    case INL_ERR_INVALID_INPUT: throw InvalidInputError(message);
    default: throw InferenceError(message);
  }
}

// ------------------------------------------------------------------ planning
std::vector<size_t> longest_first(const std::vector<size_t>& lengths) {
  std::vector<size_t> order(lengths.size());
  std::iota(order.begin(), order.end(), size_t{0});
  std::stable_sort(order.begin(), order.end(), [&](size_t a, size_t b) { return lengths[a] > lengths[b]; });
  return order;
}

std::vector<std::pair<size_t, size_t>> plan_packed(const std::vector<size_t>& lengths, size_t max_batch_tokens,
                                                   size_t max_texts) {
  std::vector<std::pair<size_t, size_t>> out;
  size_t start = 0, tokens = 0;
  for (size_t i = 0; i < lengths.size(); ++i) {
    const size_t n = lengths[i], count = i - start + 1;
    if (i > start && (tokens + n > max_batch_tokens || (max_texts && count > max_texts))) {
      out.emplace_back(start, i);
      start = i;
      tokens = n;
    } else {
      tokens += n;
    }
  }
  if (start < lengths.size()) out.emplace_back(start, lengths.size());
  return out;
}

Packed pack(const std::vector<std::vector<uint32_t>>& texts, const std::vector<size_t>& members) {
  Packed p;
  p.cu.reserve(members.size() + 1);
  p.cu.push_back(0);
  for (size_t m : members) {
    p.ids.insert(p.ids.end(), texts[m].begin(), texts[m].end());
    p.cu.push_back(static_cast<int32_t>(p.ids.size()));
  }
  return p;
}

// ------------------------------------------------------------------ deadline
void BatchDeadline::ensure_healthy(const std::string& what) const {
  std::lock_guard<std::mutex> l(*mu_);
  if (*wedged_)
    throw TimeoutError(what + ": an earlier call timed out and its thread is still stuck; restart the process");
}

bool BatchDeadline::wedged() const {
  std::lock_guard<std::mutex> l(*mu_);
  return *wedged_;
}

namespace {
struct TaskState {
  std::mutex mu;
  std::condition_variable cv;
  bool done = false;
  std::exception_ptr error;
};
}  // namespace

void BatchDeadline::run_erased(const std::string& what, double budget_seconds, std::function<void()> task) {
  ensure_healthy(what);
  auto st = std::make_shared<TaskState>();
  // The worker owns its state; a stuck worker outlives this call.
  std::thread([st, task = std::move(task)]() {
    std::exception_ptr err;
    try {
      task();
    } catch (...) {
      err = std::current_exception();
    }
    std::lock_guard<std::mutex> l(st->mu);
    st->error = err;
    st->done = true;
    st->cv.notify_all();
  }).detach();
  std::unique_lock<std::mutex> l(st->mu);
  const auto budget = std::chrono::duration<double>(budget_seconds);
  if (!st->cv.wait_for(l, budget, [&] { return st->done; })) {
    {
      std::lock_guard<std::mutex> w(*mu_);
      *wedged_ = true;
    }
    throw TimeoutError(what + " did not finish within " + std::to_string(budget_seconds) +
                       " s; the process must be restarted");
  }
  if (st->error) {
    try {
      std::rethrow_exception(st->error);
    } catch (const InlError&) {
      throw;  // the engine's own errors keep their variant
    } catch (const std::exception& e) {
      throw InferenceError(what + ": " + e.what());
    }
  }
}

// ------------------------------------------------------------------ engines
double Options::batch_timeout() const {
  const double s = per_batch_timeout_seconds ? *per_batch_timeout_seconds : timeout_seconds;
  if (!(s > 0)) throw ConfigError("timeout_seconds / per_batch_timeout_seconds must be greater than 0");
  return s;
}

SparseVector SparseVector::from_dense(const float* row, size_t n) {
  SparseVector v;
  for (size_t i = 0; i < n; ++i)
    if (row[i] > 0.f) {
      v.indices.push_back(static_cast<uint32_t>(i));
      v.values.push_back(row[i]);
    }
  return v;
}

EngineBase::EngineBase(Loader loader, Options options) : options_(std::move(options)), loader_(std::move(loader)) {}
EngineBase::~EngineBase() = default;

bool EngineBase::is_loaded() const {
  std::lock_guard<std::mutex> l(load_mu_);
  return loaded_ != nullptr;
}

bool EngineBase::unload() {
  std::lock_guard<std::mutex> l(load_mu_);
  if (!loaded_) return false;
  { std::lock_guard<std::mutex> g(loaded_->gate); }  // wait for a forward in progress
  loaded_.reset();
  return true;
}

std::shared_ptr<EngineBase::Loaded> EngineBase::model() {
  std::lock_guard<std::mutex> l(load_mu_);  // concurrent callers share one load; failures are not cached
  if (!loaded_) {
    auto m = std::make_shared<Loaded>();
    m->backend = loader_();
    if (!m->backend) throw InferenceError("model load returned no backend");
    loaded_ = std::move(m);
  }
  return loaded_;
}

std::vector<size_t> EngineBase::token_counts(const Tokens& texts) const {
  std::vector<size_t> out;
  out.reserve(texts.size());
  for (const auto& t : texts) out.push_back(t.size());
  return out;
}

template <typename R>
std::vector<R> EngineBase::run_batches(const std::string& what, const Tokens& texts,
                                       std::function<std::vector<R>(Backend&, const Packed&)> forward) {
  if (texts.empty()) return {};
  if (options_.batch_size == 0)  // crates/inl-text/src/native.rs:552-556
    throw InferenceError("batch_size must be greater than 0");
  deadline_.ensure_healthy(what);
  std::shared_ptr<Loaded> loaded = model();
  const double budget = options_.batch_timeout();
  std::vector<size_t> lengths;
  lengths.reserve(texts.size());
  for (const auto& t : texts) lengths.push_back(t.size());
  const std::vector<size_t> order = longest_first(lengths);
  std::vector<size_t> sorted(order.size());
  for (size_t k = 0; k < order.size(); ++k) sorted[k] = lengths[order[k]];
  std::vector<std::optional<R>> results(texts.size());
  for (const auto& range : plan_packed(sorted, options_.max_batch_tokens, options_.batch_size)) {
    std::vector<size_t> members(order.begin() + range.first, order.begin() + range.second);
    auto batch = std::make_shared<Packed>(pack(texts, members));
    std::lock_guard<std::mutex> gate(loaded->gate);  // queue before the deadline starts
    std::vector<R> out = deadline_.run<std::vector<R>>(
        what + " batch", budget, [loaded, batch, forward]() { return forward(*loaded->backend, *batch); });
    if (out.size() != members.size())
      throw InferenceError(what + " returned " + std::to_string(out.size()) + " results for " +
                           std::to_string(members.size()) + " inputs");
    for (size_t k = 0; k < members.size(); ++k) results[members[k]] = std::move(out[k]);
  }
  std::vector<R> all;
  all.reserve(results.size());
  for (auto& r : results) {
    if (!r) throw InferenceError(what + " lost an input");
    all.push_back(std::move(*r));
  }
  return all;
}

namespace {
Tokens truncate(const Tokens& texts, size_t max_length) {
  Tokens out(texts.size());
  for (size_t i = 0; i < texts.size(); ++i)
    out[i].assign(texts[i].begin(), texts[i].begin() + std::min(texts[i].size(), max_length));
  return out;
}

EngineInfo info_of(const Options& o, int dim, const ModelInfo& mi, size_t max_length) {
  EngineInfo e;
  e.model_id = o.id;
  e.dimension = dim;
  e.dtype = mi.dtype;
  e.device = "cuda:" + std::to_string(mi.device);
  e.max_length = static_cast<int>(max_length);
  return e;
}
}  // namespace

// resolve_output_dim (crates/inl-text/src/native.rs:793-817): Matryoshka
// output only for EmbeddingGemma-style models (arch 2), at their trained
// sizes, never wider than the model's embeddings. 0 = the model's own width.
static int resolve_output_dim(const std::optional<int>& requested, const ModelInfo& mi) {
  if (!requested) return 0;
  const int dim = *requested;
  if (mi.arch != 2) throw ConfigError("output_dim is only supported for EmbeddingGemma 2 models");
  if (dim != 128 && dim != 256 && dim != 512 && dim != 768)
    throw ConfigError("output_dim " + std::to_string(dim) +
                      " is not supported by EmbeddingGemma 2: use one of [128, 256, 512, 768]");
  if (dim > mi.dense_dim)
    throw ConfigError("output_dim " + std::to_string(dim) + " exceeds the model's " + std::to_string(mi.dense_dim) +
                      "-dimensional embeddings");
  return dim;
}

EngineInfo TextEmbedder::load() {
  const ModelInfo mi = model()->backend->info();
  const int out_dim = resolve_output_dim(options_.output_dim, mi);
  return info_of(options_, out_dim ? out_dim : mi.dense_dim, mi, options_.max_length);
}

TextIdentity TextEmbedder::identity() {
  const EngineInfo info = load();
  TextIdentity t;
  t.id = info.model_id;
  t.dimension = info.dimension;
  t.dtype = info.dtype;
  t.device = "cuda";
  t.max_length = options_.max_length;
  return t;
}

std::vector<std::vector<float>> TextEmbedder::embed(const Tokens& texts) {
  const Tokens t = truncate(texts, options_.max_length);
  if (t.empty()) return {};
  const ModelInfo mi = model()->backend->info();
  const int out_dim = resolve_output_dim(options_.output_dim, mi);
  const int dim = out_dim ? out_dim : mi.dense_dim;
  return run_batches<std::vector<float>>(
      "native embedding", t, [out_dim, dim](Backend& b, const Packed& p) {
        const std::vector<float> flat = b.dense(p, out_dim);
        const size_t n = p.cu.size() - 1;
        std::vector<std::vector<float>> rows;
        for (size_t i = 0; i < n && (i + 1) * dim <= flat.size(); ++i)
          rows.emplace_back(flat.begin() + i * dim, flat.begin() + (i + 1) * dim);
        return rows;
      });
}

namespace {
// The sparse and late encoders refuse these options when they are built.
void check_encoder_options(const Options& o) {
  const double s = o.per_batch_timeout_seconds ? *o.per_batch_timeout_seconds : o.timeout_seconds;
  if (!(s > 0))
    throw ConfigError("timeout_seconds / per_batch_timeout_seconds must be greater than 0 for the native encoder");
  if (o.batch_size == 0) throw ConfigError("batch_size must be greater than 0");
}
}  // namespace

SparseEncoder::SparseEncoder(Loader loader, Options options) : EngineBase(std::move(loader), std::move(options)) {
  check_encoder_options(options_);
}

EngineInfo SparseEncoder::load() {
  const ModelInfo mi = model()->backend->info();
  return info_of(options_, mi.sparse_dim, mi, options_.max_length);
}

std::vector<SparseVector> SparseEncoder::encode(const Tokens& texts) {
  const Tokens t = truncate(texts, options_.max_length);
  if (t.empty()) return {};
  // The backend returns the compacted vectors (the library compacts them on
  // the device); a non-finite weight is an inference error there, as in
  // crates/inl-sparse/src/native.rs:536-540.
  return run_batches<SparseVector>("native sparse", t, [](Backend& b, const Packed& p) { return b.sparse(p); });
}

LateEncoder::LateEncoder(Loader loader, Options options, LateTask query, LateTask document)
    : EngineBase(std::move(loader), std::move(options)), query_(std::move(query)), document_(std::move(document)) {
  check_encoder_options(options_);
  if (query_.length == 0 || document_.length == 0) throw ConfigError("max_length must be greater than 0");
}

EngineInfo LateEncoder::load() {
  const ModelInfo mi = model()->backend->info();
  return info_of(options_, mi.multivector_dim, mi, document_.length);
}

const LateTask& LateEncoder::setup(const std::string& task) const {
  if (task == "query") return query_;
  if (task == "document") return document_;
  throw InvalidInputError("unknown late task '" + task + "': use 'query' or 'document'");
}

std::vector<size_t> LateEncoder::token_counts(const Tokens& texts, const std::string& task) const {
  const size_t length = setup(task).length;
  std::vector<size_t> out;
  out.reserve(texts.size());
  for (const auto& t : texts) out.push_back(std::min(t.size(), length));
  return out;
}

std::vector<std::vector<std::vector<float>>> LateEncoder::encode(const Tokens& texts, const std::string& task) {
  const LateTask* setup = &this->setup(task);
  const Tokens t = truncate(texts, setup->length);
  if (t.empty()) return {};
  const size_t D = static_cast<size_t>(model()->backend->info().multivector_dim);
  const std::vector<uint32_t> skip = setup->skip;
  using Matrix = std::vector<std::vector<float>>;
  return run_batches<Matrix>("native late", t, [D, skip](Backend& b, const Packed& p) {
    const std::vector<float> flat = b.multivector(p);
    const size_t n = p.cu.size() - 1;
    std::vector<Matrix> out;
    for (size_t i = 0; i < n; ++i) {
      Matrix kept;  // crates/inl-late/src/native.rs:665-681
      for (int32_t r = p.cu[i]; r < p.cu[i + 1]; ++r) {
        if (std::find(skip.begin(), skip.end(), p.ids[r]) != skip.end()) continue;
        if ((static_cast<size_t>(r) + 1) * D > flat.size()) throw InferenceError("native late encoder returned too few vectors");
        std::vector<float> v(flat.begin() + r * D, flat.begin() + (r + 1) * D);
        for (float x : v)
          if (!std::isfinite(x)) throw InferenceError("native late encoder produced non-finite values");
        kept.push_back(std::move(v));
      }
      out.push_back(std::move(kept));
    }
    return out;
  });
}

}  // namespace inl
