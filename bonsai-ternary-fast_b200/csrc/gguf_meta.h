// GGUF metadata as read by csrc/gguf.cpp, for the library's own model binding
// (csrc/decoder.cu), and the load path's staging rule. Internal: not part of
// the C ABI.
#pragma once
#include <algorithm>
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

// Rows per chunk of btf_gguf_load_panels_rows for `rows` rows of a PTQ1_0
// matrix of width K (a multiple of 128): whole 8-row groups, so every chunk
// starts a panel row group; at most `chunk_bytes` of source per chunk but at
// least one group; no chunk larger than the rows loaded.
inline int64_t staging_rows(int64_t K, int64_t rows, int64_t chunk_bytes) {
  const int64_t row_bytes = K / 128 * 28;
  return std::min<int64_t>((rows + 7) / 8 * 8, std::max<int64_t>(8, chunk_bytes / row_bytes / 8 * 8));
}

// Bytes of each of the loader's two pinned staging buffers.
inline uint64_t staging_buffer_bytes(int64_t K, int64_t rows, int64_t chunk_bytes) {
  return (uint64_t)(staging_rows(K, rows, chunk_bytes) * (K / 128 * 28));
}

}  // namespace gguf
}  // namespace btf
