// Links the C++ host layer's CUDA backend against libinl_cuda.so: checks a
// config without a device (exit 3 / 4 on a wrong answer), then loads a model
// through it and prints the InlError variant a failed load raises (on a host
// without a GPU: "config", no CUDA device).
#include <cstdio>

#include "inl_engine.hpp"

int main(int argc, char** argv) {
  const char* path = argc > 1 ? argv[1] : "/nonexistent/model.safetensors";
  // The config checks run without a device.
  const std::string qwen3 = R"({"model_type": "qwen3", "hidden_size": 64, "intermediate_size": 128,
                                "num_attention_heads": 2, "num_key_value_heads": 1, "num_hidden_layers": 1,
                                "vocab_size": 100, "head_dim": 64})";
  const inl::ModelInfo info = inl::check_config(qwen3, "bf16");
  if (info.arch != 0 || info.hidden != 64 || info.dense_dim != 64 || info.device != -1) return 3;
  try {
    inl::check_config(R"({"model_type": "llama"})", "f32");
    return 4;
  } catch (const inl::ConfigError&) {
  }
  try {
    auto b = inl::cuda_backend(R"({"model_type": "qwen3", "hidden_size": 64, "intermediate_size": 128,
                                   "num_attention_heads": 2, "num_key_value_heads": 1, "num_hidden_layers": 1,
                                   "vocab_size": 100, "head_dim": 64})",
                               path, 0, "bf16");
    std::printf("loaded\n");
    return 2;
  } catch (const inl::InlError& e) {
    std::printf("%s|%s\n", e.code().c_str(), e.what());
    return 0;
  }
}
