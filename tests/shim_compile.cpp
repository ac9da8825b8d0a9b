// Compile-only check: a reference-style call site (src/cuda/gpu_decoder.cu:396-416
// of bonsai-ternary-fast) written against btf::cuda builds with include/btf_b200.hpp.
#include <string>
#include <vector>

#include "btf_b200.hpp"

void ffn_call_site(const uint8_t* gate, const uint8_t* up, const uint8_t* down, float* G, float* x, int E, int F,
                   int M, btf::cuda::Q8Act act, cudaStream_t st) {
  namespace c = btf::cuda;
  const c::GemvSeg gu[2] = {{gate, nullptr, F, G, F}, {up, nullptr, F, nullptr, 0}};
  c::launch_gemv(gu, 2, E, M, act, c::kSwiglu, st);
  c::launch_prep(G, F, M, F, nullptr, 1e-6f, c::Hx{}, nullptr, 0, act, st);
  const c::GemvSeg d{down, nullptr, E, x, E};
  c::launch_gemv(&d, 1, F, M, act, c::kAdd, st);
}

// The decoder call pattern of the reference's CLI (FastDecoder: prefill, then greedy steps).
int decode_call_site(const std::string& path, const std::vector<int32_t>& prompt, std::vector<float>& logits) {
  btf::cuda::DecoderOptions o;
  o.n_ctx = 64;
  const btf::cuda::MemoryPlan plan = btf::cuda::plan_memory(path, o);
  if (plan.device_bytes() == 0 || plan.table().empty()) return -1;
  btf::cuda::Decoder dec(path, o);
  logits.resize(dec.n_vocab());
  int t = dec.prefill(prompt.data(), (int)prompt.size(), logits.data());
  for (int i = 0; i < 4; ++i) t = dec.step(t, nullptr);
  dec.reset();
  const btf_step_stats st = dec.stats();
  dec.reset_stats();
  return t + dec.pos() + (int)st.steps + (dec.device_bytes() == plan.device_bytes() ? 0 : 1);
}
