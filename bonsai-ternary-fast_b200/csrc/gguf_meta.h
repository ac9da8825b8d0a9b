// GGUF metadata as read by csrc/gguf.cpp, for the library's own model binding
// (csrc/qwen35.cpp). Internal: not part of the C ABI.
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace btf {
namespace gguf {

// One metadata value. Scalars fill i and f (integers and bools also as f,
// floats also truncated into i); strings fill s; arrays fill ai/af (numbers)
// or as (strings), with elem_type the element's metadata type.
struct Value {
  uint32_t type = 0, elem_type = 0;
  int64_t i = 0;
  double f = 0;
  std::string s;
  std::vector<int64_t> ai;
  std::vector<double> af;
  std::vector<std::string> as;
};

// Metadata entry `key` of a handle from btf_gguf_open, or nullptr.
const Value* meta(const void* handle, const std::string& key);

}  // namespace gguf
}  // namespace btf
