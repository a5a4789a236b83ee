// Minimal safetensors reader (header JSON + index.json shard map).
//
// Mirrors SafeTensors (src/safetensors.mojo:17-96): a checkpoint directory is
// either one model.safetensors or shards listed in model.safetensors.index.json
// ("weight_map": name -> file).  Each file is [u64 header_len | JSON header |
// data]; header entries are {"dtype", "shape", "data_offsets": [b, e]} relative
// to the data start; "__metadata__" is skipped.
#pragma once
#include <stdint.h>
#include <map>
#include <string>
#include <vector>

namespace q8 {

struct TensorInfo {
  std::string name, dtype, path;
  std::vector<int64_t> shape;
  int64_t begin = 0, end = 0;  // absolute byte range in `path`
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t s : shape) n *= s;
    return n;
  }
};

// Parses all shards of `dir`.  Returns false and fills `err` on failure.
bool safetensors_scan(const std::string& dir, std::map<std::string, TensorInfo>& out, std::string& err);

// Parses one header blob (exposed for tests of the parser).
bool safetensors_parse_header(const std::string& json, const std::string& path, int64_t data_start,
                              std::map<std::string, TensorInfo>& out, std::string& err);

}  // namespace q8
