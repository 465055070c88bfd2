// Backend of the C++ host layer over the C ABI of libinl_cuda
// (include/inl_cuda.h): one model handle, host buffers in and out.
#include <algorithm>
#include <string>
#include <vector>

#include "../../include/inl_cuda.h"
#include "../../include/inl_engine.hpp"

namespace inl {
namespace {

std::string last_error() {
  char buf[1024] = {0};
  inl_cuda_last_error(buf, sizeof(buf));
  return buf;
}

void check(int status, const std::string& what) {
  if (status != INL_OK) throw_status(status, what + ": " + last_error());
}

ModelInfo to_info(const inl_model_info& i) {
  ModelInfo o;
  o.arch = i.arch;
  o.hidden = i.hidden_size;
  o.dense_dim = i.dense_dim;
  o.sparse_dim = i.sparse_dim;
  o.multivector_dim = i.multivector_dim;
  o.dtype = i.dtype == INL_DTYPE_BF16 ? "bf16" : "f32";
  o.device = i.device;
  return o;
}

class CudaBackend : public Backend {
 public:
  explicit CudaBackend(inl_model* m) : m_(m) {}
  ~CudaBackend() override { inl_cuda_model_destroy(m_); }
  CudaBackend(const CudaBackend&) = delete;
  CudaBackend& operator=(const CudaBackend&) = delete;

  ModelInfo info() override {
    inl_model_info i{};
    check(inl_cuda_model_info(m_, &i), "model info");
    return to_info(i);
  }

  std::vector<float> dense(const Packed& b, int out_dim) override {
    const int n = static_cast<int>(b.cu.size()) - 1;
    const int dim = out_dim ? out_dim : info().dense_dim;
    std::vector<float> out(static_cast<size_t>(n) * dim);
    check(inl_cuda_forward_dense(m_, b.ids.data(), INL_MEM_HOST, b.cu.data(), n, out_dim, out.data(), INL_MEM_HOST),
          "dense forward");
    return out;
  }

  std::vector<SparseVector> sparse(const Packed& b) override {
    // compacted on the device; only the active terms are copied back
    const int n = static_cast<int>(b.cu.size()) - 1;
    const int64_t cap = std::max<int64_t>(1, static_cast<int64_t>(n) * info().sparse_dim);
    std::vector<int64_t> offsets(static_cast<size_t>(n) + 1);
    std::vector<int32_t> idx(static_cast<size_t>(cap));
    std::vector<float> val(static_cast<size_t>(cap));
    check(inl_cuda_forward_sparse_compact(m_, b.ids.data(), INL_MEM_HOST, b.cu.data(), n, offsets.data(), idx.data(),
                                          val.data(), cap, INL_MEM_HOST),
          "sparse forward");
    std::vector<SparseVector> out(static_cast<size_t>(n));
    for (int i = 0; i < n; ++i) {
      out[i].indices.assign(idx.begin() + offsets[i], idx.begin() + offsets[i + 1]);
      out[i].values.assign(val.begin() + offsets[i], val.begin() + offsets[i + 1]);
    }
    return out;
  }

  std::vector<float> multivector(const Packed& b) override {
    const int n = static_cast<int>(b.cu.size()) - 1;
    std::vector<float> out(b.ids.size() * static_cast<size_t>(info().multivector_dim));
    check(inl_cuda_forward_multivector(m_, b.ids.data(), INL_MEM_HOST, b.cu.data(), n, out.data(), INL_MEM_HOST),
          "multivector forward");
    return out;
  }

 private:
  inl_model* m_;
};

}  // namespace

ModelInfo check_config(const std::string& config_json, const std::string& dtype) {
  if (dtype != "bf16" && dtype != "f32") throw ConfigError("dtype must be bf16 or f32");
  inl_model_info i{};
  check(inl_cuda_config_check(config_json.c_str(), dtype == "bf16" ? INL_DTYPE_BF16 : INL_DTYPE_F32, &i), "config");
  return to_info(i);
}

std::unique_ptr<Backend> cuda_backend(const std::string& config_json, const std::string& safetensors_path, int device,
                                      const std::string& dtype, const std::vector<float>& dense_head_weight,
                                      int dense_out, int dense_in, const std::vector<float>& dense_head_bias,
                                      bool dense_normalize) {
  if (dtype != "bf16" && dtype != "f32") throw ConfigError("dtype must be bf16 or f32");
  inl_model* m = nullptr;
  check(inl_cuda_model_create(config_json.c_str(), safetensors_path.c_str(), device,
                              dtype == "bf16" ? INL_DTYPE_BF16 : INL_DTYPE_F32, &m),
        "model load");
  auto backend = std::make_unique<CudaBackend>(m);
  if (!dense_head_weight.empty()) {
    if (static_cast<size_t>(dense_out) * dense_in != dense_head_weight.size())
      throw ConfigError("Dense head weight has the wrong size");
    if (!dense_head_bias.empty() && dense_head_bias.size() != static_cast<size_t>(dense_out))
      throw ConfigError("Dense head bias has the wrong size");
    check(inl_cuda_model_set_dense_head(m, dense_head_weight.data(), dense_out, dense_in,
                                        dense_head_bias.empty() ? nullptr : dense_head_bias.data()),
          "Dense head");
    check(inl_cuda_model_set_dense_normalize(m, dense_normalize ? 1 : 0), "Dense head");
  }
  return backend;
}

}  // namespace inl
