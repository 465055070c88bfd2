// Host-layer tests of include/inl_engine.hpp with a test-double Backend:
// the C++ counterparts of tests/test_planner_engine.py, tests/test_late_tasks.py
// and the reference's own engine tests (crates/inl-core/src/deadline.rs tests,
// crates/inl-text/src/native.rs count checks). Built and run on the CPU by
// tests/test_cpp_host.py; exits non-zero on the first failure.
#include <atomic>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <limits>
#include <thread>

#include "inl_engine.hpp"

#define CHECK(...)                                                                 \
  do {                                                                             \
    if (!(__VA_ARGS__)) {                                                          \
      std::fprintf(stderr, "FAILED %s:%d: %s\n", __FILE__, __LINE__, #__VA_ARGS__); \
      std::exit(1);                                                                \
    }                                                                              \
  } while (0)

template <typename E, typename F>
bool throws(F f) {
  try {
    f();
  } catch (const E&) {
    return true;
  } catch (...) {
    return false;
  }
  return false;
}

using namespace inl;

// dense row i = [len, first id, 0, 0]; sparse row: term (len % V) = 1, term 0 = -1;
// multivector: one vector (token id, position) per token.
struct Fake : Backend {
  std::atomic<int>* calls;
  double delay = 0;
  bool drop = false, nan = false;
  int arch = 0, dense_dim = 4;
  explicit Fake(std::atomic<int>* c) : calls(c) {}
  ModelInfo info() override {
    ModelInfo m;
    m.arch = arch;
    m.dense_dim = dense_dim;
    m.sparse_dim = 5;
    m.multivector_dim = 2;
    return m;
  }
  std::vector<float> dense(const Packed& p, int) override {
    ++*calls;
    if (delay > 0) std::this_thread::sleep_for(std::chrono::duration<double>(delay));
    size_t n = p.cu.size() - 1 - (drop ? 1 : 0);
    std::vector<float> out(n * 4, 0.f);
    for (size_t i = 0; i < n; ++i) {
      out[i * 4] = static_cast<float>(p.cu[i + 1] - p.cu[i]);
      out[i * 4 + 1] = p.cu[i + 1] > p.cu[i] ? static_cast<float>(p.ids[p.cu[i]]) : -1.f;
    }
    return out;
  }
  std::vector<SparseVector> sparse(const Packed& p) override {
    ++*calls;
    const size_t n = p.cu.size() - 1;
    std::vector<float> rows(n * 5, 0.f);
    for (size_t i = 0; i < n; ++i) {
      rows[i * 5] = -1.f;
      rows[i * 5 + (p.cu[i + 1] - p.cu[i]) % 5] += 2.f;
      if (nan) rows[i * 5 + 3] = std::numeric_limits<float>::quiet_NaN();
    }
    // the library's compaction: a non-finite weight is an inference error
    for (float v : rows)
      if (!std::isfinite(v)) throw InferenceError("non-finite SPLADE term weight");
    std::vector<SparseVector> out;
    for (size_t i = 0; i < n; ++i) out.push_back(SparseVector::from_dense(&rows[i * 5], 5));
    return out;
  }
  std::vector<float> multivector(const Packed& p) override {
    ++*calls;
    std::vector<float> out(p.ids.size() * 2);
    for (size_t i = 0; i + 1 < p.cu.size(); ++i)
      for (int32_t r = p.cu[i]; r < p.cu[i + 1]; ++r) {
        out[r * 2] = static_cast<float>(p.ids[r]);
        out[r * 2 + 1] = static_cast<float>(r - p.cu[i]);
      }
    return out;
  }
};

Tokens texts_of(std::vector<size_t> lens) {
  Tokens t;
  uint32_t next = 1;
  for (size_t L : lens) {
    std::vector<uint32_t> x(L);
    for (auto& v : x) v = next++;
    t.push_back(x);
  }
  return t;
}

int main() {
  // ---------------- planning
  CHECK((longest_first({3, 5, 5, 1}) == std::vector<size_t>{1, 2, 0, 3}));
  auto plan = plan_packed({5, 5, 3, 1}, 8);
  CHECK(plan.size() == 3 && plan[0] == std::make_pair<size_t, size_t>(0, 1) &&
        plan[1] == std::make_pair<size_t, size_t>(1, 3) && plan[2] == std::make_pair<size_t, size_t>(3, 4));
  CHECK(plan_packed({9}, 4).size() == 1);          // one text always forms a batch
  CHECK(plan_packed({1, 1, 1}, 100, 2).size() == 2);  // max_texts
  Packed pk = pack(texts_of({2, 0, 3}), {2, 0, 1});
  CHECK((pk.cu == std::vector<int32_t>{0, 3, 5, 5}) && pk.ids.size() == 5 && pk.ids[0] == 3 && pk.ids[3] == 1);

  // ---------------- errors
  CHECK(throws<ConfigError>([] { throw_status(1, "x"); }));
  CHECK(throws<InferenceError>([] { throw_status(2, "x"); }));
  CHECK(throws<TimeoutError>([] { throw_status(3, "x"); }));
  CHECK(throws<InvalidInputError>([] { throw_status(4, "x"); }));
  try {
    throw_status(4, "ids out of range");
  } catch (const InlError& e) {
    CHECK(std::string(e.what()) == "invalid input: ids out of range" && e.code() == "invalid_input");
  }
  Options bad;
  bad.timeout_seconds = 0;
  CHECK(throws<ConfigError>([&] { bad.batch_timeout(); }));

  // ---------------- dense: input order, truncation, batching, count check
  std::atomic<int> calls{0};
  {
    Options o;
    o.max_batch_tokens = 16;
    o.batch_size = 3;
    TextEmbedder e([&] { return std::make_unique<Fake>(&calls); }, o);
    CHECK(!e.is_loaded());
    Tokens t = texts_of({5, 1, 9, 3, 7, 2, 2});
    auto out = e.embed(t);
    CHECK(out.size() == t.size());
    for (size_t i = 0; i < t.size(); ++i) CHECK(out[i][0] == t[i].size() && out[i][1] == t[i][0]);
    CHECK(calls.load() >= 3);  // split by tokens and by batch_size
    CHECK(e.is_loaded() && e.load().dimension == 4 && e.load().attention == "fused");
    CHECK(e.unload() && !e.is_loaded() && !e.unload());
    CHECK(e.embed({}).empty());
    Options o2;
    o2.max_length = 4;
    TextEmbedder e2([&] { return std::make_unique<Fake>(&calls); }, o2);
    CHECK(e2.embed(texts_of({10}))[0][0] == 4.f);
    TextEmbedder e3([&] { auto f = std::make_unique<Fake>(&calls); f->drop = true; return f; }, Options{});
    CHECK(throws<InferenceError>([&] { e3.embed(texts_of({2, 3})); }));
    // output_dim: EmbeddingGemma-style models only, trained sizes, not wider than the model
    Options o4;
    o4.output_dim = 128;
    TextEmbedder e4([&] { return std::make_unique<Fake>(&calls); }, o4);
    CHECK(throws<ConfigError>([&] { e4.load(); }));
    CHECK(throws<ConfigError>([&] { e4.embed(texts_of({2})); }));
    TextEmbedder e5([&] { auto f = std::make_unique<Fake>(&calls); f->arch = 2; f->dense_dim = 768; return f; }, o4);
    CHECK(e5.load().dimension == 128);
    const TextIdentity ident = e5.identity();
    CHECK(ident.dimension == 128 && ident.device == "cuda" && ident.max_length == o4.max_length);
    Options o6;
    o6.output_dim = 300;
    TextEmbedder e6([&] { auto f = std::make_unique<Fake>(&calls); f->arch = 2; f->dense_dim = 768; return f; }, o6);
    CHECK(throws<ConfigError>([&] { e6.load(); }));
    // batch_size 0: an inference error when embedding; sparse / late refuse it when built
    Options z;
    z.batch_size = 0;
    TextEmbedder e7([&] { return std::make_unique<Fake>(&calls); }, z);
    CHECK(e7.embed({}).empty());
    CHECK(throws<InferenceError>([&] { e7.embed(texts_of({2})); }));
    CHECK(throws<ConfigError>([&] { SparseEncoder s([&] { return std::make_unique<Fake>(&calls); }, z); }));
    CHECK(throws<ConfigError>([&] { LateEncoder l([&] { return std::make_unique<Fake>(&calls); }, z); }));
    Options t0;
    t0.timeout_seconds = 0;
    CHECK(throws<ConfigError>([&] { SparseEncoder s([&] { return std::make_unique<Fake>(&calls); }, t0); }));
    LateTask empty_task;
    empty_task.length = 0;
    CHECK(throws<ConfigError>(
        [&] { LateEncoder l([&] { return std::make_unique<Fake>(&calls); }, Options{}, empty_task); }));
  }

  // ---------------- deadline: a stuck forward times out, later calls fail fast
  {
    std::atomic<int> c{0};
    Options o;
    o.per_batch_timeout_seconds = 0.2;
    TextEmbedder e([&] { auto f = std::make_unique<Fake>(&c); f->delay = 1.5; return f; }, o);
    const auto t0 = std::chrono::steady_clock::now();
    CHECK(throws<TimeoutError>([&] { e.embed(texts_of({3})); }));
    CHECK(std::chrono::steady_clock::now() - t0 < std::chrono::seconds(1));
    CHECK(e.deadline().wedged());
    const int before = c.load();
    CHECK(throws<TimeoutError>([&] { e.embed(texts_of({3})); }));
    CHECK(c.load() == before);  // the task did not run
    BatchDeadline d;
    CHECK(d.run<int>("x", 1.0, [] { return 42; }) == 42);
    CHECK(throws<InferenceError>([&] { d.run<int>("x", 1.0, []() -> int { throw std::runtime_error("boom"); }); }));
    CHECK(throws<InvalidInputError>([&] { d.run<int>("x", 1.0, []() -> int { throw InvalidInputError("bad"); }); }));
    CHECK(!d.wedged());
  }

  // ---------------- sparse: sorted positive terms, non-finite is an error
  {
    std::atomic<int> c{0};
    SparseEncoder s([&] { return std::make_unique<Fake>(&c); }, Options{});
    auto v = s.encode(texts_of({3, 5, 6}));
    CHECK(v.size() == 3);
    CHECK((v[0].indices == std::vector<uint32_t>{3}) && v[0].values[0] == 2.f);
    CHECK((v[1].indices == std::vector<uint32_t>{0}) && v[1].values[0] == 1.f);  // term 0: -1 + 2 = 1 > 0
    SparseEncoder sn([&] { auto f = std::make_unique<Fake>(&c); f->nan = true; return f; }, Options{});
    CHECK(throws<InferenceError>([&] { sn.encode(texts_of({2})); }));
    CHECK(s.load().dimension == 5);
  }

  // ---------------- late: task length and skiplist
  {
    std::atomic<int> c{0};
    LateTask q{24, {}}, d{5, {2, 4}};
    LateEncoder l([&] { return std::make_unique<Fake>(&c); }, Options{}, q, d);
    Tokens t = texts_of({7});  // ids 1..7
    auto doc = l.encode(t, "document");
    CHECK(doc.size() == 1 && doc[0].size() == 3);  // cut to 5 (ids 1..5), 2 and 4 dropped
    CHECK(doc[0][0][0] == 1.f && doc[0][1][0] == 3.f && doc[0][2][0] == 5.f && doc[0][2][1] == 4.f);
    auto qry = l.encode(t, "query");
    CHECK(qry[0].size() == 7);
    CHECK(throws<InvalidInputError>([&] { l.encode(t, "passage"); }));
    CHECK(l.load().max_length == 5 && l.load().dimension == 2);
    CHECK((l.token_counts(texts_of({7, 3}), "document") == std::vector<size_t>{5, 3}));
    CHECK((l.token_counts(texts_of({7, 3}), "query") == std::vector<size_t>{7, 3}));
    CHECK(throws<InvalidInputError>([&] { l.token_counts(t, "passage"); }));
  }

  std::printf("all passed\n");
  return 0;
}
