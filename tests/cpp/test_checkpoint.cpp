// Shard resolution of a model load (im-not-llm_b200/csrc/checkpoint.h) on the
// CPU: a .safetensors path is itself; an index names its weight_map's files,
// sorted and each once, next to the index; a broken index is an error.
// Usage: test_checkpoint <scratch dir>
#include <cstdio>
#include <fstream>
#include <string>
#include <vector>

#include "checkpoint.h"

static int failures = 0;
#define CHECK(...)                                                    \
  do {                                                                \
    if (!(__VA_ARGS__)) {                                             \
      std::printf("FAILED line %d: %s\n", __LINE__, #__VA_ARGS__);    \
      ++failures;                                                     \
    }                                                                 \
  } while (0)

static void write(const std::string& path, const std::string& text) { std::ofstream(path) << text; }

int main(int argc, char** argv) {
  if (argc < 2) return 2;
  const std::string dir = argv[1];
  std::vector<std::string> files;
  std::string err;

  CHECK(inl::checkpoint_files(dir + "/model.safetensors", &files, &err));
  CHECK(files == std::vector<std::string>{dir + "/model.safetensors"});

  write(dir + "/model.safetensors.index.json",
        R"({"metadata": {"total_size": 10}, "weight_map": {
             "b.weight": "model-00002-of-00002.safetensors",
             "a.weight": "model-00001-of-00002.safetensors",
             "c.weight": "model-00002-of-00002.safetensors"}})");
  CHECK(inl::checkpoint_files(dir + "/model.safetensors.index.json", &files, &err));
  CHECK(files == std::vector<std::string>{dir + "/model-00001-of-00002.safetensors",
                                          dir + "/model-00002-of-00002.safetensors"});

  write(dir + "/no_map.json", R"({"metadata": {}})");
  CHECK(!inl::checkpoint_files(dir + "/no_map.json", &files, &err));
  CHECK(err.find("has no weight_map") != std::string::npos);

  write(dir + "/bad.json", "{not json");
  CHECK(!inl::checkpoint_files(dir + "/bad.json", &files, &err));
  CHECK(err.find("is invalid") != std::string::npos);

  CHECK(!inl::checkpoint_files(dir + "/missing.index.json", &files, &err));
  CHECK(err.find("cannot be read") != std::string::npos);

  write(dir + "/escape.json", R"({"weight_map": {"a": "../outside.safetensors"}})");
  CHECK(!inl::checkpoint_files(dir + "/escape.json", &files, &err));
  CHECK(err.find("outside its directory") != std::string::npos);

  write(dir + "/dots.json", R"({"weight_map": {"a": "model..v2.safetensors"}})");
  CHECK(inl::checkpoint_files(dir + "/dots.json", &files, &err));
  CHECK(files == std::vector<std::string>{dir + "/model..v2.safetensors"});

  if (failures == 0) std::printf("all passed\n");
  return failures == 0 ? 0 : 1;
}
