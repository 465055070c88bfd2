// Safetensors checkpoint files of a model load: one file, or the shards of a
// sharded checkpoint named by its model.safetensors.index.json. The shard
// list follows safetensors_weight_files (crates/inl-core/src/hub.rs:324-353):
// the file names of the index's weight_map, sorted, each once, found next to
// the index. Header-only (no CUDA), so the host tests build it with g++.
#pragma once

#include <algorithm>
#include <fstream>
#include <sstream>
#include <string>
#include <vector>

#include "json.h"

namespace inl {

inline bool is_index_path(const std::string& path) {
  const std::string suffix = ".json";
  return path.size() >= suffix.size() && path.compare(path.size() - suffix.size(), suffix.size(), suffix) == 0;
}

// Files to read for `path`: {path} for a .safetensors file; the shards for an
// index. Returns false with `error` set when the index cannot be used.
inline bool checkpoint_files(const std::string& path, std::vector<std::string>* files, std::string* error) {
  files->clear();
  if (!is_index_path(path)) {
    files->push_back(path);
    return true;
  }
  std::ifstream in(path, std::ios::binary);
  if (!in) {
    *error = "native model weights index " + path + " cannot be read";
    return false;
  }
  std::stringstream text;
  text << in.rdbuf();
  json::Value index;
  try {
    index = json::parse(text.str());
  } catch (const std::exception& e) {
    *error = "native model " + path + " is invalid: " + e.what();
    return false;
  }
  const json::Value* map = index.get("weight_map");
  if (!map || map->kind != json::Value::Object) {
    *error = "native model " + path + " has no weight_map";
    return false;
  }
  std::vector<std::string> names;
  for (const auto& kv : map->obj)
    if (kv.second.kind == json::Value::String) names.push_back(kv.second.str);
  std::sort(names.begin(), names.end());
  names.erase(std::unique(names.begin(), names.end()), names.end());
  if (names.empty()) {
    *error = "native model " + path + " names no weight files";
    return false;
  }
  const size_t slash = path.find_last_of('/');
  const std::string dir = slash == std::string::npos ? std::string() : path.substr(0, slash + 1);
  for (const std::string& name : names) {
    bool outside = name.empty() || name[0] == '/';
    for (size_t b = 0; !outside && b <= name.size();) {  // no ".." path component
      const size_t e = std::min(name.find('/', b), name.size());
      outside = name.compare(b, e - b, "..") == 0;
      b = e + 1;
    }
    if (outside) {
      *error = "native model " + path + " names a weight file outside its directory: " + name;
      return false;
    }
    files->push_back(dir + name);
  }
  return true;
}

}  // namespace inl
