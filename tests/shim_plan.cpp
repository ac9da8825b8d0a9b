// Runs the C++ shim's plan_memory (btf::cuda::MemoryPlan) on a GGUF without a
// GPU: prints device bytes, host bytes, the bytes-per-step figures, then the
// table, for tests/test_plan.py to compare with the C ABI.
#include <cstdio>

#include "btf_b200.hpp"

int main(int argc, char** argv) {
  if (argc < 2) return 2;
  btf::cuda::DecoderOptions o;
  o.n_ctx = 64;
  try {
    const btf::cuda::MemoryPlan p = btf::cuda::plan_memory(argv[1], o);
    std::printf("%llu %llu %llu %llu\n%s", (unsigned long long)p.device_bytes(), (unsigned long long)p.host_bytes(),
                (unsigned long long)p.decode_bytes_fixed, (unsigned long long)p.decode_bytes_per_ctx,
                p.table().c_str());
  } catch (const std::exception& e) {
    std::fprintf(stderr, "%s\n", e.what());
    return 1;
  }
  return 0;
}
