// Runs the C++ shim's host repack (btf::cuda::repack_panels_host) without a GPU:
// reads N, K and a PTQ1_0 file, writes the panels to a file, and checks that a
// bad shape throws, for tests/test_host.py to compare with the C ABI.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "btf_b200.hpp"

int main(int argc, char** argv) {
  if (argc < 5) return 2;
  const long long N = std::atoll(argv[1]), K = std::atoll(argv[2]);
  std::FILE* f = std::fopen(argv[3], "rb");
  if (!f) return 2;
  std::vector<uint8_t> src((size_t)(N * (K / 128) * 28));
  const size_t got = std::fread(src.data(), 1, src.size(), f);
  std::fclose(f);
  if (got != src.size()) return 2;
  try {
    const btf::cuda::PanelMatrix m = btf::cuda::repack_panels_host(src.data(), N, K, 2);
    if (m.panels.size() != btf::cuda::panel_bytes(N, K)) return 3;
    std::FILE* o = std::fopen(argv[4], "wb");
    if (!o || std::fwrite(m.panels.data(), 1, m.panels.size(), o) != m.panels.size()) return 2;
    std::fclose(o);
  } catch (const std::exception& e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 1;
  }
  try {
    btf::cuda::repack_panels_host(src.data(), N, 100);
    return 4;  // K % 128 must throw
  } catch (const std::runtime_error&) {
  }
  return 0;
}
