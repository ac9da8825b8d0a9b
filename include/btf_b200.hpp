// C++17 mirror of the reference's launcher interface (src/cuda/kernels.cuh:13-56
// of bonsai-ternary-fast), implemented over the btf_b200 C ABI. Call sites
// written against btf::cuda (e.g. src/cuda/gpu_decoder.cu:396-450) compile
// unchanged; errors throw std::runtime_error like the reference's launchers.
//
// Differences a maintainer must know:
//   - GemvSeg::codes points at the PANEL buffer of the matrix (include/btf_b200.h)
//     and GemvSeg::scales must be nullptr: the scales live inside the panels;
//   - launch_repack keeps the reference's T2 output; launch_repack_panels is the
//     loader for the B200 layout and needs N and K;
//   - launch_prep runs the whole prep (RMSNorm, permutation, signs, Hadamard, Q8);
//   - Decoder is the batch-1 decode step over a qwen35 GGUF (btf_decoder_*);
//     plan_memory sizes it before it is opened (btf_plan_memory);
//   - repack_panels_host / PanelMatrix are the host repack (repack / PackedMatrix)
//     for the panel layout.
#pragma once
#include <cuda_runtime_api.h>

#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

#include "btf_b200.h"

namespace btf {
namespace cuda {

inline void throw_if(int status, const char* what) {
  if (status != BTF_OK)
    throw std::runtime_error(std::string(what) + ": " + btf_status_string(status) + ": " + btf_last_error());
}

// kernels.cuh:17
inline void kernels_init(int device) { throw_if(btf_init(device), "kernels_init"); }

// kernels.cuh:20
inline int gemv_max_nb(int K) { return btf_gemv_max_nb(K); }

// kernels.cuh:24 (T2 output, unchanged semantics)
inline void launch_repack(const uint8_t* src, int64_t nblocks, uint8_t* codes, uint16_t* scales, cudaStream_t st) {
  throw_if(btf_repack_t2(src, nblocks, codes, scales, st), "launch_repack");
}

// B200 resident layout: PTQ1_0 rows -> panels (size btf_panel_bytes(N, K)).
inline void launch_repack_panels(const uint8_t* src, int64_t N, int64_t K, uint8_t* panels, cudaStream_t st) {
  throw_if(btf_repack_panels(src, N, K, panels, st), "launch_repack_panels");
}

// kernels.cuh:27-31
struct Q8Act {
  int8_t* q = nullptr;  // [M][K]
  float* d = nullptr;   // [M][K/32]
  int* s = nullptr;     // [M][K/32]
};

// kernels.cuh:34-38
struct Hx {
  int block = 0;
  int perm_hd = 0, perm_nk = 0, perm_rep = 0;
  const float* signs = nullptr;
};

// kernels.cuh:42-43 — RMSNorm -> permutation -> signs -> Hadamard -> Q8_0.
inline void launch_prep(const float* x, int ldx, int M, int n, const float* normw, float eps, const Hx& hx,
                        float* xn_out, int ldxn, const Q8Act& a, cudaStream_t st) {
  const btf_hx h{hx.block, hx.perm_hd, hx.perm_nk, hx.perm_rep, hx.signs};
  throw_if(btf_prep(x, ldx, M, n, normw, eps, h, xn_out, ldxn, btf_q8act{a.q, a.d, a.s}, st), "launch_prep");
}

// kernels.cuh:46-53
struct GemvSeg {
  const uint8_t* codes = nullptr;    // panel buffer
  const uint16_t* scales = nullptr;  // must be nullptr (scales are in the panels)
  int N = 0;
  float* y = nullptr;
  int ldy = 0;
};
enum GemvMode { kStore = BTF_STORE, kAdd = BTF_ADD, kSwiglu = BTF_SWIGLU };

// kernels.cuh:56
inline void launch_gemv(const GemvSeg* segs, int nseg, int K, int M, const Q8Act& a, GemvMode mode, cudaStream_t st) {
  if (nseg < 1 || nseg > 3) throw std::runtime_error("gemv: 1..3 segments");
  btf_gemv_seg s[3];
  for (int i = 0; i < nseg; ++i) {
    if (segs[i].scales) throw std::runtime_error("gemv: GemvSeg::scales must be nullptr with the panel layout");
    s[i] = btf_gemv_seg{segs[i].codes, segs[i].N, segs[i].y, segs[i].ldy};
  }
  throw_if(btf_gemv(s, nseg, K, M, btf_q8act{a.q, a.d, a.s}, (int)mode, st), "launch_gemv");
}

// The batch-1 decode step (btf_decoder_*). Mirrors FastDecoder
// (include/btf/fast.hpp:71-101): step() returns the greedy next token and fills
// the logits when given; prefill() feeds the prompt one token per step.
struct DecoderOptions {  // the FastOptions fields the decoder uses (fast.hpp:13-27)
  int n_ctx = 4096;
  bool round_q_f16 = true;
  int attn_splits = 16;
  bool cuda_graph = true;
  int staging_mb = 64;
  bool drop_page_cache = true;
};

inline btf_decoder_opts to_c(const DecoderOptions& o) {
  return btf_decoder_opts{o.n_ctx,      o.round_q_f16 ? 1 : 0, o.attn_splits,
                          o.cuda_graph ? 1 : 0, o.staging_mb, o.drop_page_cache ? 0 : 1};
}

class Decoder {
 public:
  explicit Decoder(const std::string& gguf_path, const DecoderOptions& o = DecoderOptions()) {
    const btf_decoder_opts c = to_c(o);
    throw_if(btf_decoder_open(gguf_path.c_str(), &c, &h_), "btf_decoder_open");
  }
  Decoder(const Decoder&) = delete;
  Decoder& operator=(const Decoder&) = delete;
  ~Decoder() { btf_decoder_close(h_); }
  int step(int32_t token, float* logits) {
    int32_t next = -1;
    throw_if(btf_decoder_step(h_, token, logits, &next), "btf_decoder_step");
    return next;
  }
  // FastDecoder::prefill (gpu_decoder.cu:154-171): chunks of up to max_batch tokens
  int prefill(const int32_t* tokens, int n, float* logits, int max_batch = 0) {
    int32_t next = -1;
    throw_if(btf_decoder_prefill(h_, tokens, n, max_batch, logits, &next), "btf_decoder_prefill");
    return next;
  }
  void reset() { throw_if(btf_decoder_reset(h_), "btf_decoder_reset"); }
  // FastDecoder::stats / reset_stats / device_bytes (fast.hpp:90-95)
  btf_step_stats stats() const {
    btf_step_stats s{};
    throw_if(btf_decoder_stats(h_, &s), "btf_decoder_stats");
    return s;
  }
  void reset_stats() { throw_if(btf_decoder_reset_stats(h_), "btf_decoder_reset_stats"); }
  uint64_t device_bytes() const { return info().device_bytes; }
  int pos() const { return info().pos; }
  int n_vocab() const { return info().dims.n_vocab; }
  btf_decoder_info info() const {
    btf_decoder_info i{};
    throw_if(btf_decoder_get_info(h_, &i), "btf_decoder_get_info");
    return i;
  }

 private:
  void* h_ = nullptr;
};

// One ternary matrix in the panel layout on the host. Mirrors PackedMatrix /
// repack / packed_codes_bytes (include/btf/fast.hpp:33-46, src/repack.cpp:16-45)
// for the panel layout: one buffer of panel_bytes(N, K) holds the codes and the
// scales. Host only; needs no GPU.
struct PanelMatrix {
  int64_t N = 0, K = 0;
  std::vector<uint8_t> panels;
};
inline uint64_t panel_bytes(int64_t N, int64_t K) { return (uint64_t)btf_panel_bytes(N, K); }
// Repacks a PTQ1_0 tensor of N rows x K columns (src points to row 0) on the
// host with `threads` threads (0 = all, as FastOptions::threads).
inline PanelMatrix repack_panels_host(const uint8_t* src, int64_t N, int64_t K, int threads = 0) {
  if (!src || N <= 0 || K <= 0 || K % 128)
    throw std::runtime_error("repack_panels_host: null source or bad shape (K a positive multiple of 128)");
  PanelMatrix m;
  m.N = N;
  m.K = K;
  m.panels.resize(panel_bytes(N, K));
  throw_if(btf_repack_panels_host(src, N, K, m.panels.data(), threads), "repack_panels_host");
  return m;
}

// The decoder's memory before it is opened. Mirrors PlanItem / MemoryPlan /
// plan_memory (include/btf/fast.hpp:50-69, src/repack.cpp:114-204) for the
// panel layout: items, device_bytes(), host_bytes(), table(), and the
// bytes-per-step figures. Host only; needs no GPU.
struct PlanItem {
  std::string what;
  uint64_t bytes = 0;
  bool host = false;
};
struct MemoryPlan {
  std::vector<PlanItem> items;
  uint64_t decode_bytes_fixed = 0;
  uint64_t decode_bytes_per_ctx = 0;
  uint64_t device_bytes() const {
    uint64_t s = 0;
    for (const auto& i : items) s += i.host ? 0 : i.bytes;
    return s;
  }
  uint64_t host_bytes() const {
    uint64_t s = 0;
    for (const auto& i : items) s += i.host ? i.bytes : 0;
    return s;
  }
  std::string table() const {
    std::string out;
    char buf[256];
    for (const auto& i : items) {
      std::snprintf(buf, sizeof buf, "  %-44s %-6s %14llu B  %9.2f MiB\n", i.what.c_str(), i.host ? "host" : "device",
                    (unsigned long long)i.bytes, i.bytes / 1048576.0);
      out += buf;
    }
    std::snprintf(buf, sizeof buf, "  %-44s %-6s %14llu B  %9.2f MiB (%.3f GB)\n", "total resident", "device",
                  (unsigned long long)device_bytes(), device_bytes() / 1048576.0, device_bytes() / 1e9);
    return out + buf;
  }
};

inline MemoryPlan plan_memory(const std::string& gguf_path, const DecoderOptions& o = DecoderOptions(),
                              int world = 1, int rank = 0) {
  const btf_decoder_opts c = to_c(o);
  btf_memory_plan p{};
  throw_if(btf_plan_memory(gguf_path.c_str(), &c, world, rank, &p), "btf_plan_memory");
  MemoryPlan m;
  m.items = {{"ternary matrices in panels (" + std::to_string(p.n_matrices) + ")", p.panel_bytes, false},
             {"f32 vectors (norms, ssm, conv1d, signs)", p.vector_bytes, false},
             {"KV cache fp16", p.kv_cache_bytes, false},
             {"delta-net + conv state", p.state_bytes, false},
             {"activations, partials, Q8, argmax", p.work_bytes, false},
             {"token in/out", p.pinned_bytes, true},
             {"load staging (peak, freed after load)", p.staging_bytes, true}};
  m.decode_bytes_fixed = p.decode_bytes_fixed;
  m.decode_bytes_per_ctx = p.decode_bytes_per_ctx;
  return m;
}

}  // namespace cuda
}  // namespace btf
