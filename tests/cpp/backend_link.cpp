// Links the C++ host layer's CUDA backend against libinl_cuda.so and loads a
// model through it; prints the InlError variant a failed load raises (on a
// host without a GPU: "config", no CUDA device).
#include <cstdio>

#include "inl_engine.hpp"

int main(int argc, char** argv) {
  const char* path = argc > 1 ? argv[1] : "/nonexistent/model.safetensors";
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
