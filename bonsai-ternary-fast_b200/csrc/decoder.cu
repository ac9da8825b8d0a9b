// Batch-1 decode step of the qwen35 hybrid decoder (gated delta net + gated
// full attention) on the library's kernels, as one CUDA graph.
//
// Mirrors GpuDecoder (src/cuda/gpu_decoder.cu of bonsai-ternary-fast:
// forward_chunk :401-450, enqueue_step / capture :461-486) and computes what the
// reference's CPU emulator computes (src/emu_decoder.cpp:167-220, gdn :222-303,
// attn :305-375): per layer a fused prep (RMSNorm -> Hadamard transform -> Q8)
// feeding the ternary GEMVs, the mixer (delta rule or attention), the FFN with
// SwiGLU, then the output norm, lm_head and a greedy argmax. The model binding
// restates bd::Model::bind (ref/bonsai-decoder/src/model.cpp:68-205) over the
// library's own GGUF reader. Weights stay resident; the position and the next
// input token live in device memory, so the captured graph replays for every
// token. Batch 1 only: a prompt is fed one token per step.
#include <cuda_fp16.h>
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <vector>

#include "btf_b200.h"
#include "common.cuh"
#include "decode.h"
#include "gguf_meta.h"

namespace btf {
namespace {

constexpr uint32_t kF32 = 0, kF16 = 1, kBF16 = 30, kPTQ = 143;

struct Mat {
  uint8_t* pan = nullptr;
  int N = 0, K = 0;
  btf_hx hx{0, 0, 0, 0, nullptr};
  int row0 = 0, n = 0;  // this rank's rows [row0, row0 + n) (n = N on one GPU)
};

// Row shard of `rank` among `world`: whole 8-row groups, ceil(groups / world)
// groups per rank, the last ranks clipped (shard.shard_rows in Python).
void shard_rows(int N, int world, int rank, int* r0, int* n) {
  const int groups = (N + kRows - 1) / kRows;
  const int per = (groups + world - 1) / world * kRows;
  *r0 = std::min(N, rank * per);
  *n = std::max(0, std::min(N, *r0 + per) - *r0);
}

struct Layer {
  bool rec = false;
  float *attn_norm = nullptr, *post_norm = nullptr;
  Mat gate, up, down;
  // gated delta net
  Mat qkv, zg, out;
  float *alpha_w = nullptr, *beta_w = nullptr, *ssm_a = nullptr, *ssm_dt = nullptr, *conv_w = nullptr,
        *ssm_norm = nullptr;
  int ab_bf16 = 0;
  float *conv_state = nullptr, *ssm_state = nullptr;
  // attention
  Mat wq, wk, wv, wo;
  float *q_norm = nullptr, *k_norm = nullptr;
  __half *kc = nullptr, *vc = nullptr;
};

struct Decoder {
  int device = 0;
  cudaStream_t st = nullptr;
  btf_decoder_dims d{};
  btf_decoder_opts o{};
  int C = 0, DK = 0, DV = 0, NK = 0, NV = 0, QK = 0, DI = 0, Kmax = 0;
  float theta_scale = 0.f;
  std::vector<Layer> L;
  Mat embd, output;
  float* out_norm = nullptr;
  int inv_block = 0;
  float* inv_signs = nullptr;
  std::vector<void*> allocs;
  // step buffers
  float *x = nullptr, *xn = nullptr, *bA = nullptr, *bB = nullptr, *bC = nullptr, *bO = nullptr,
        *bG = nullptr, *logits = nullptr, *part = nullptr, *amax_v = nullptr;
  int* attn_cnt = nullptr;  // per-head split counters of the attention launch (zero between launches)
  int* amax_i = nullptr;
  int8_t* aq = nullptr;
  float* ad = nullptr;
  int32_t* as = nullptr;
  int32_t *d_tok = nullptr, *d_pos = nullptr, *d_next = nullptr;
  // prompt chunks (btf_decoder_prefill): up to kMaxChunk tokens and their positions
  static constexpr int kMaxChunk = 8;
  int32_t *d_ptok = nullptr, *d_ppos = nullptr;
  int32_t* h_io = nullptr;  // pinned: [0] token in, [1] token out
  int pos = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  uint64_t weight_bytes = 0, state_bytes = 0, kv_bytes_per_token = 0;
  // Memory plan (btf_plan_memory): every device allocation by kind. A dry
  // decoder runs the same binding and buffer set-up, sizes every allocation
  // and touches no device: no allocation, copy, fill or launch.
  enum Kind { kPanels, kVectors, kKv, kState, kWork, kKinds };
  bool dry = false;
  uint64_t dev_bytes[kKinds] = {};
  uint64_t sign_bytes = 0, staging_peak = 0;
  int n_mats = 0;
  // Step accounting (FastDecoder::stats): steps, host wall time inside
  // step/run, device time between CUDA events around them. The events of an
  // asynchronous run are read when the stats are next touched.
  uint64_t n_steps = 0;
  double wall_s = 0, gpu_s = 0;
  cudaEvent_t ev[2] = {nullptr, nullptr};
  bool ev_pending = false;
  static constexpr int kArgmaxParts = 148;
  // tensor parallelism: every matmul N-sharded over `world` ranks, its outputs
  // stored into every rank's arena (btf_gemv_gather, counted completion). The
  // arena holds the activation buffers after a 256-byte control block (arrival
  // counter +0, consumed arrivals +4, CTA completion +8), laid out the same on
  // every rank; peers[r] is rank r's arena as mapped in this process.
  int world = 1, rank = 0;
  uint8_t* arena = nullptr;
  size_t arena_bytes = 0;
  uint8_t* peers[BTF_MAX_RANKS] = {};
  bool connected = false;
  static constexpr size_t kCtl = 256;

  ~Decoder() {
    for (cudaEvent_t e : ev)
      if (e) cudaEventDestroy(e);
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    if (st) cudaStreamSynchronize(st);
    for (void* p : allocs) cudaFree(p);
    if (h_io) cudaFreeHost(h_io);
    if (st) cudaStreamDestroy(st);
  }
  template <class T>
  T* alloc(size_t n, int* rc, Kind kind = kWork) {
    void* p = nullptr;
    if (*rc) return nullptr;
    const size_t bytes = n * sizeof(T) > 0 ? n * sizeof(T) : 16;
    dev_bytes[kind] += bytes;
    if (dry) return nullptr;
    const cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
      *rc = cuda_fail(e, "btf_decoder: cudaMalloc");
      return nullptr;
    }
    allocs.push_back(p);
    return static_cast<T*>(p);
  }
  uint64_t device_total() const {
    uint64_t t = 0;
    for (uint64_t b : dev_bytes) t += b;
    return t;
  }
};

// ---------------------------------------------------------------- buffers
int make_buffers(Decoder& D) {
  int rc = BTF_OK;
  const btf_decoder_dims& d = D.d;
  const int E = d.n_embd, F = d.n_ff, H = d.n_head, HK = d.n_head_kv, HD = d.head_dim;
  int n_gdn = 0, n_attn = 0;
  for (auto& l : D.L) (l.rec ? n_gdn : n_attn)++;
  const int wa = std::max(n_gdn ? D.C : 0, n_attn ? 2 * H * HD : 0);
  const int wb = std::max(n_gdn ? D.DI : 0, n_attn ? HK * HD : 0);
  const int wc = std::max(n_gdn ? D.C : 0, n_attn ? HK * HD : 0);
  const int wo = std::max(n_gdn ? D.DI : 0, n_attn ? H * HD : 0);
  D.Kmax = std::max({E, F, wo});
  // activation buffers in one arena (shared with the other ranks under tensor parallelism)
  // the row buffers hold a prompt chunk of kMaxChunk rows (decode steps use row 0);
  // the logits (the last token's) hold one row
  const int R = Decoder::kMaxChunk;
  const int sizes[8] = {R * E, R * E, R * wa, R * wb, R * wc, R * wo, R * F, d.n_vocab};
  size_t off[8], total = Decoder::kCtl;
  for (int i = 0; i < 8; ++i) {
    off[i] = total;
    total += ((size_t)sizes[i] * 4 + 255) / 256 * 256;
  }
  D.arena = D.alloc<uint8_t>(total, &rc);
  if (rc) return rc;
  D.arena_bytes = total;
  if (!D.dry && cudaMemset(D.arena, 0, total) != cudaSuccess) return fail(BTF_ERR_CUDA, "btf_decoder: arena clear");
  float** dst[8] = {&D.x, &D.xn, &D.bA, &D.bB, &D.bC, &D.bO, &D.bG, &D.logits};
  if (!D.dry)
    for (int i = 0; i < 8; ++i) *dst[i] = reinterpret_cast<float*>(D.arena + off[i]);
  D.peers[D.rank] = D.arena;
  D.part = D.alloc<float>((size_t)std::max(1, H) * D.o.attn_splits * (HD + 2), &rc);
  D.attn_cnt = D.alloc<int>((size_t)std::max(1, H), &rc);
  if (!rc && !D.dry && cudaMemset(D.attn_cnt, 0, sizeof(int) * std::max(1, H)) != cudaSuccess)
    return fail(BTF_ERR_CUDA, "btf_decoder: counter clear");
  D.amax_v = D.alloc<float>(Decoder::kArgmaxParts, &rc);
  D.amax_i = D.alloc<int>(Decoder::kArgmaxParts, &rc);
  D.aq = D.alloc<int8_t>((size_t)R * D.Kmax, &rc);
  D.ad = D.alloc<float>((size_t)R * D.Kmax / 32, &rc);
  D.as = D.alloc<int32_t>((size_t)R * D.Kmax / 32, &rc);
  D.d_tok = D.alloc<int32_t>(4 + 2 * R, &rc);
  if (rc) return rc;
  if (!D.dry) {
    D.d_pos = D.d_tok + 1;
    D.d_next = D.d_tok + 2;
    D.d_ptok = D.d_tok + 4;
    D.d_ppos = D.d_tok + 4 + R;
  }
  for (Layer& l : D.L) {
    if (l.rec) {
      l.conv_state = D.alloc<float>((size_t)d.conv_kernel * D.C, &rc, Decoder::kState);  // ring of K input rows
      l.ssm_state = D.alloc<float>((size_t)D.NV * D.DV * D.DK, &rc, Decoder::kState);
      D.state_bytes += 2 * ((uint64_t)(d.conv_kernel - 1) * D.C + (uint64_t)D.NV * D.DV * D.DK) * 4;
    } else {
      l.kc = D.alloc<__half>((size_t)D.o.n_ctx * HK * HD, &rc, Decoder::kKv);
      l.vc = D.alloc<__half>((size_t)D.o.n_ctx * HK * HD, &rc, Decoder::kKv);
      D.kv_bytes_per_token += 2ull * HK * HD * 2;
    }
  }
  if (rc || D.dry) return rc;
  const cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&D.h_io), 4 * sizeof(int32_t), cudaHostAllocDefault);
  return e == cudaSuccess ? BTF_OK : cuda_fail(e, "btf_decoder: pinned io");
}

int reset_state(Decoder& D) {
  cudaError_t e = cudaSuccess;
  for (Layer& l : D.L) {
    if (l.rec) {
      if (e == cudaSuccess)
        e = cudaMemsetAsync(l.conv_state, 0, (size_t)D.d.conv_kernel * D.C * sizeof(float), D.st);
      if (e == cudaSuccess) e = cudaMemsetAsync(l.ssm_state, 0, (size_t)D.NV * D.DV * D.DK * sizeof(float), D.st);
    }
  }
  if (e == cudaSuccess) e = cudaMemsetAsync(D.d_tok, 0, 4 * sizeof(int32_t), D.st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(D.st);
  D.pos = 0;
  return e == cudaSuccess ? BTF_OK : cuda_fail(e, "btf_decoder_reset");
}

// ---------------------------------------------------------------- one step
// One output of a GEMV launch: matrix m into y (the full output row of the
// local buffer; null for the up half of SwiGLU).
struct Out {
  const Mat* m;
  float* y;
};
int gemv(Decoder& D, std::initializer_list<Out> outs, int K, int mode, int M = 1) {
  const btf_q8act act{D.aq, D.ad, D.as};
  btf_gemv_seg segs[3];
  int ns = 0;
  const bool tp = D.world > 1;
  for (const Out& o : outs)
    segs[ns++] = {o.m->pan, tp ? o.m->n : o.m->N, o.y ? o.y + (tp ? o.m->row0 : 0) : nullptr, o.y ? o.m->N : 0};
  if (!tp) return btf_gemv(segs, ns, K, M, act, mode, D.st);
  btf_gather g{};
  g.world = D.world;
  g.rank = D.rank;
  const int nout = mode == BTF_SWIGLU ? 1 : ns;
  for (int s = 0; s < nout; ++s)
    for (int r = 0; r < D.world; ++r)
      g.peer_y[s][r] = reinterpret_cast<float*>(D.peers[r] + (reinterpret_cast<uint8_t*>(segs[s].y) - D.arena));
  for (int r = 0; r < D.world; ++r) g.flags[r] = reinterpret_cast<unsigned*>(D.peers[r]);
  g.expect = reinterpret_cast<unsigned*>(D.arena + 4);
  g.done = reinterpret_cast<unsigned*>(D.arena + 8);
  return btf_gemv_gather(segs, ns, K, M, act, mode, &g, D.st);
}
// M rows of width n (row stride n) -> the Q8 activation (and xn rows when non-null)
int prep(Decoder& D, const float* x, int n, const float* normw, const btf_hx& hx, float* xn, int M = 1) {
  const btf_q8act act{D.aq, D.ad, D.as};
  return btf_prep(x, n, M, n, normw, D.d.rms_eps, hx, xn, n, act, D.st);
}
#define BTF_TRY(call)                   \
  do {                                  \
    const int rc_ = (call);             \
    if (rc_) return rc_;                \
  } while (0)
#define BTF_TRYC(call)                                                        \
  do {                                                                        \
    const cudaError_t e_ = (call);                                            \
    if (e_ != cudaSuccess) return cuda_fail(e_, "btf_decoder: step kernel"); \
  } while (0)

// Enqueues one decode step for the token at d_tok: logits, the greedy token
// into d_next and d_tok, and pos + 1.
int enqueue_step(Decoder& D) {
  const btf_decoder_dims& d = D.d;
  const int E = d.n_embd, F = d.n_ff, H = d.n_head, HK = d.n_head_kv, HD = d.head_dim;
  BTF_TRYC(launch_embed(D.embd.pan, d.n_vocab, E, D.d_tok, D.inv_block, D.inv_signs, D.x, D.st));
  for (Layer& l : D.L) {
    if (l.rec) {
      BTF_TRY(prep(D, D.x, E, l.attn_norm, l.qkv.hx, D.xn));
      BTF_TRY(gemv(D, {{&l.qkv, D.bA}, {&l.zg, D.bB}}, E, BTF_STORE));
      const GdnArgs ga{D.xn, l.alpha_w, l.beta_w, l.ssm_dt, l.ssm_a, E, l.ab_bf16, D.bA, l.conv_state, l.conv_w,
                       d.conv_kernel, D.C, D.bB, l.ssm_state, l.ssm_norm, D.NK, D.DK, D.DV, D.QK, d.rms_eps, D.d_pos,
                       D.bO, D.NV};
      BTF_TRYC(launch_gdn_mix(ga, D.st));
      BTF_TRY(prep(D, D.bO, D.DI, nullptr, l.out.hx, nullptr));
      BTF_TRY(gemv(D, {{&l.out, D.x}}, D.DI, BTF_ADD));
    } else {
      BTF_TRY(prep(D, D.x, E, l.attn_norm, l.wq.hx, nullptr));
      BTF_TRY(gemv(D, {{&l.wq, D.bA}, {&l.wk, D.bB}, {&l.wv, D.bC}}, E, BTF_STORE));
      BTF_TRYC(launch_attention_fused(D.bA, D.bB, D.bC, l.q_norm, l.k_norm, H, HK, HD, d.n_rot, D.theta_scale,
                                      d.rms_eps, D.d_pos, D.o.round_q_f16, l.kc, l.vc, D.o.n_ctx, D.o.attn_splits,
                                      D.part, D.attn_cnt, D.bO, D.st));
      BTF_TRY(prep(D, D.bO, H * HD, nullptr, l.wo.hx, nullptr));
      BTF_TRY(gemv(D, {{&l.wo, D.x}}, H * HD, BTF_ADD));
    }
    BTF_TRY(prep(D, D.x, E, l.post_norm, l.gate.hx, nullptr));
    BTF_TRY(gemv(D, {{&l.gate, D.bG}, {&l.up, nullptr}}, E, BTF_SWIGLU));
    BTF_TRY(prep(D, D.bG, F, nullptr, l.down.hx, nullptr));
    BTF_TRY(gemv(D, {{&l.down, D.x}}, F, BTF_ADD));
  }
  BTF_TRY(prep(D, D.x, E, D.out_norm, D.output.hx, nullptr));
  BTF_TRY(gemv(D, {{&D.output, D.logits}}, E, BTF_STORE));
  BTF_TRYC(launch_argmax(D.logits, d.n_vocab, D.amax_v, D.amax_i, Decoder::kArgmaxParts, D.d_next, D.d_tok, D.d_pos,
                         D.st));
  return BTF_OK;
}

// Enqueues one prompt chunk of M tokens (d_ptok[0..M), positions d_ppos[0..M)),
// as the reference's forward_chunk (src/cuda/gpu_decoder.cu:401-450): every
// prep and ternary matmul runs once over the M rows (the weights stream once per
// chunk); the recurrent mixer and the attention run token by token in order, at
// each token's own position, so the state and the KV cache advance exactly as in
// M decode steps. The logits, the greedy token (into d_next and d_tok) come
// from the chunk's last token.
int enqueue_chunk(Decoder& D, int M) {
  const btf_decoder_dims& d = D.d;
  const int E = d.n_embd, F = d.n_ff, H = d.n_head, HK = d.n_head_kv, HD = d.head_dim;
  for (int m = 0; m < M; ++m)
    BTF_TRYC(launch_embed(D.embd.pan, d.n_vocab, E, D.d_ptok + m, D.inv_block, D.inv_signs, D.x + (size_t)m * E,
                          D.st));
  for (Layer& l : D.L) {
    if (l.rec) {
      const int C = l.qkv.N, Z = l.zg.N;
      BTF_TRY(prep(D, D.x, E, l.attn_norm, l.qkv.hx, D.xn, M));
      BTF_TRY(gemv(D, {{&l.qkv, D.bA}, {&l.zg, D.bB}}, E, BTF_STORE, M));
      for (int m = 0; m < M; ++m) {
        const GdnArgs ga{D.xn + (size_t)m * E, l.alpha_w, l.beta_w, l.ssm_dt, l.ssm_a, E, l.ab_bf16,
                         D.bA + (size_t)m * C, l.conv_state, l.conv_w, d.conv_kernel, D.C, D.bB + (size_t)m * Z,
                         l.ssm_state, l.ssm_norm, D.NK, D.DK, D.DV, D.QK, d.rms_eps, D.d_ppos + m,
                         D.bO + (size_t)m * D.DI, D.NV};
        BTF_TRYC(launch_gdn_mix(ga, D.st));
      }
      BTF_TRY(prep(D, D.bO, D.DI, nullptr, l.out.hx, nullptr, M));
      BTF_TRY(gemv(D, {{&l.out, D.x}}, D.DI, BTF_ADD, M));
    } else {
      const int NQ = l.wq.N, NK = l.wk.N, NV = l.wv.N, HO = H * HD;
      BTF_TRY(prep(D, D.x, E, l.attn_norm, l.wq.hx, nullptr, M));
      BTF_TRY(gemv(D, {{&l.wq, D.bA}, {&l.wk, D.bB}, {&l.wv, D.bC}}, E, BTF_STORE, M));
      for (int m = 0; m < M; ++m) {
        const float* qf = D.bA + (size_t)m * NQ;
        BTF_TRYC(launch_attention_fused(qf, D.bB + (size_t)m * NK, D.bC + (size_t)m * NV, l.q_norm, l.k_norm, H, HK,
                                        HD, d.n_rot, D.theta_scale, d.rms_eps, D.d_ppos + m, D.o.round_q_f16, l.kc,
                                        l.vc, D.o.n_ctx, D.o.attn_splits, D.part, D.attn_cnt,
                                        D.bO + (size_t)m * HO, D.st));
      }
      BTF_TRY(prep(D, D.bO, HO, nullptr, l.wo.hx, nullptr, M));
      BTF_TRY(gemv(D, {{&l.wo, D.x}}, HO, BTF_ADD, M));
    }
    BTF_TRY(prep(D, D.x, E, l.post_norm, l.gate.hx, nullptr, M));
    BTF_TRY(gemv(D, {{&l.gate, D.bG}, {&l.up, nullptr}}, E, BTF_SWIGLU, M));
    BTF_TRY(prep(D, D.bG, F, nullptr, l.down.hx, nullptr, M));
    BTF_TRY(gemv(D, {{&l.down, D.x}}, F, BTF_ADD, M));
  }
  BTF_TRY(prep(D, D.x + (size_t)(M - 1) * E, E, D.out_norm, D.output.hx, nullptr));
  BTF_TRY(gemv(D, {{&D.output, D.logits}}, E, BTF_STORE));
  BTF_TRYC(launch_argmax(D.logits, d.n_vocab, D.amax_v, D.amax_i, Decoder::kArgmaxParts, D.d_next, D.d_tok, nullptr,
                         D.st));
  return BTF_OK;
}

int capture(Decoder& D) {
  cudaError_t e = cudaStreamBeginCapture(D.st, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return cuda_fail(e, "btf_decoder: begin capture");
  const int rc = enqueue_step(D);
  cudaGraph_t g = nullptr;
  e = cudaStreamEndCapture(D.st, &g);
  if (rc) {
    if (g) cudaGraphDestroy(g);
    return rc;
  }
  if (e != cudaSuccess) return cuda_fail(e, "btf_decoder: end capture");
  D.graph = g;
  e = cudaGraphInstantiate(&D.exec, g, 0);
  return e == cudaSuccess ? BTF_OK : cuda_fail(e, "btf_decoder: graph instantiate");
}

// Runs one step (graph replay or eager) on D.st, no host synchronisation.
int run_step(Decoder& D) {
  if (D.pos >= D.o.n_ctx) return fail(BTF_ERR_ARG, "btf_decoder: context full (n_ctx %d)", D.o.n_ctx);
  if (D.world > 1 && !D.connected) return fail(BTF_ERR_STATE, "btf_decoder: tensor-parallel decoder not connected");
  if (D.o.cuda_graph) {
    if (!D.exec) BTF_TRY(capture(D));
    const cudaError_t e = cudaGraphLaunch(D.exec, D.st);
    if (e != cudaSuccess) return cuda_fail(e, "btf_decoder: graph launch");
  } else {
    BTF_TRY(enqueue_step(D));
  }
  D.pos += 1;
  return BTF_OK;
}

// ---------------------------------------------------------------- weights
int upload_f32(Decoder& D, const void* src, uint32_t type, int64_t n, float** out) {
  if (type != kF32 && type != kBF16 && type != kF16)
    return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: vector tensor of type %u", type);
  int rc = BTF_OK;
  float* p = D.alloc<float>(n, &rc, Decoder::kVectors);
  if (rc || D.dry) return rc;
  std::vector<float> h(n);
  const uint16_t* s16 = static_cast<const uint16_t*>(src);
  if (type == kF32) {
    std::memcpy(h.data(), src, n * 4);
  } else if (type == kBF16) {
    for (int64_t i = 0; i < n; ++i) {
      const uint32_t b = (uint32_t)s16[i] << 16;
      std::memcpy(&h[i], &b, 4);
    }
  } else if (type == kF16) {
    for (int64_t i = 0; i < n; ++i) h[i] = __half2float(__ushort_as_half(s16[i]));
  } else {
    return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: vector tensor of type %u", type);
  }
  const cudaError_t e = cudaMemcpy(p, h.data(), n * 4, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "btf_decoder: upload");
  *out = p;
  return BTF_OK;
}

struct Binder {
  Decoder& D;
  void* g;
  std::set<std::string> folded;
  std::map<int, float*> signs;  // device sign vectors by width
  int block = 0;
  bool explicit_signs = false, v_grouped = false;

  const gguf::Value* kv(const std::string& k) { return gguf::meta(g, k); }
  int64_t geti(const std::string& k, int64_t def, bool* missing = nullptr) {
    const gguf::Value* v = kv(k);
    if (!v || v->type == 8 || v->type == 9) {
      if (missing) *missing = true;
      return def;
    }
    return v->i;
  }
  double getf(const std::string& k, double def) {
    const gguf::Value* v = kv(k);
    return (!v || v->type == 8 || v->type == 9) ? def : v->f;
  }
  std::string gets(const std::string& k) {
    const gguf::Value* v = kv(k);
    return v && v->type == 8 ? v->s : std::string();
  }
  bool tensor(const std::string& name, btf_gguf_tensor_info* t, int64_t* idx = nullptr) {
    const int64_t i = btf_gguf_find(g, name.c_str());
    if (i < 0) return false;
    if (idx) *idx = i;
    return btf_gguf_tensor(g, i, t) == BTF_OK;
  }
  // A PTQ1_0 matrix [out][in] -> panels, with its input transform (model.cpp:29-58).
  // Under tensor parallelism only this rank's rows are loaded (shard = false:
  // the embedding table, which every rank reads whole).
  int mat(const std::string& name, Mat* m, bool shard = true) {
    btf_gguf_tensor_info t;
    int64_t idx = -1;
    if (!tensor(name, &t, &idx)) return fail(BTF_ERR_ARG, "btf_decoder: missing tensor %s", name.c_str());
    if (t.type != kPTQ || t.n_dims != 2) return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: %s is not a 2-D PTQ1_0 matrix", name.c_str());
    m->K = (int)t.ne[0];
    m->N = (int)t.ne[1];
    if (m->K % 128) return fail(BTF_ERR_ARG, "btf_decoder: %s width %d is not a multiple of 128", name.c_str(), m->K);
    m->row0 = 0;
    m->n = m->N;
    if (shard && D.world > 1) {
      shard_rows(m->N, D.world, D.rank, &m->row0, &m->n);
      int lr0 = 0, ln = 0;
      shard_rows(m->N, D.world, D.world - 1, &lr0, &ln);
      if (ln <= 0) return fail(BTF_ERR_ARG, "btf_decoder: %s has too few rows for %d ranks", name.c_str(), D.world);
    }
    int rc = BTF_OK;
    m->pan = D.alloc<uint8_t>(btf_panel_bytes(m->n, m->K), &rc, Decoder::kPanels);
    if (rc) return rc;
    D.n_mats += 1;
    const int64_t chunk = (int64_t)D.o.staging_mb << 20;  // source bytes per chunk of the load
    if (D.dry) {
      // the loader's two pinned staging buffers, freed after each matrix
      D.staging_peak = std::max<uint64_t>(D.staging_peak, 2 * gguf::staging_buffer_bytes(m->K, m->n, chunk));
    } else {
      BTF_TRY(btf_gguf_load_panels_rows(g, idx, m->row0, m->n, m->pan, chunk, D.st));
    }
    D.weight_bytes += btf_panel_bytes(m->n, m->K);
    if (folded.count(name)) {
      if (m->K % block) return fail(BTF_ERR_ARG, "btf_decoder: %s width not a multiple of the hadamard block", name.c_str());
      m->hx.block = block;
      if (explicit_signs) {
        auto it = signs.find(m->K);
        if (it == signs.end()) return fail(BTF_ERR_ARG, "btf_decoder: no sign vector for width %d (%s)", m->K, name.c_str());
        m->hx.signs = it->second;
      }
      if (v_grouped && name.find(".ssm_out.") != std::string::npos) {
        const int nv = D.NV, nk = D.NK;
        if (nk <= 0 || nv <= 0 || nv % nk || m->K % nv) return fail(BTF_ERR_ARG, "btf_decoder: bad GDN head geometry");
        m->hx.perm_hd = m->K / nv;
        m->hx.perm_nk = nk;
        m->hx.perm_rep = nv / nk;
      }
    }
    return BTF_OK;
  }
  int vec(const std::string& name, float** out, int64_t expect, uint32_t* type = nullptr) {
    btf_gguf_tensor_info t;
    if (!tensor(name, &t)) return fail(BTF_ERR_ARG, "btf_decoder: missing tensor %s", name.c_str());
    int64_t n = 1;
    for (int i = 0; i < t.n_dims; ++i) n *= t.ne[i];
    if (expect >= 0 && n != expect) return fail(BTF_ERR_ARG, "btf_decoder: %s has %lld elements, expected %lld", name.c_str(), (long long)n, (long long)expect);
    if (type) *type = t.type;
    D.weight_bytes += n * 4;
    return upload_f32(D, t.data, t.type, n, out);
  }

  int bind() {
    if (gets("general.architecture") != "qwen35")
      return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: architecture '%s' (this decoder implements qwen35)",
                  gets("general.architecture").c_str());
    const std::string p = "qwen35.";
    bool miss = false;
    btf_decoder_dims& d = D.d;
    d.n_layer = (int)geti(p + "block_count", 0, &miss);
    d.n_embd = (int)geti(p + "embedding_length", 0, &miss);
    d.n_ff = (int)geti(p + "feed_forward_length", 0, &miss);
    d.n_head = (int)geti(p + "attention.head_count", 0, &miss);
    d.n_head_kv = (int)geti(p + "attention.head_count_kv", 0, &miss);
    d.head_dim = (int)geti(p + "attention.key_length", d.n_head ? d.n_embd / d.n_head : 0);
    if (geti(p + "attention.value_length", d.head_dim) != d.head_dim)
      return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: key_length != value_length");
    d.n_rot = (int)geti(p + "rope.dimension_count", d.head_dim);
    d.rope_base = (float)getf(p + "rope.freq_base", 10000.0);
    if (getf(p + "rope.scaling.factor", 1.0) != 1.0) return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: rope scaling");
    d.rms_eps = (float)getf(p + "attention.layer_norm_rms_epsilon", 1e-6);
    d.conv_kernel = (int)geti(p + "ssm.conv_kernel", 0, &miss);
    d.d_state = (int)geti(p + "ssm.state_size", 0, &miss);
    d.n_group = (int)geti(p + "ssm.group_count", 0, &miss);
    d.dt_rank = (int)geti(p + "ssm.time_step_rank", 0, &miss);
    const int d_inner = (int)geti(p + "ssm.inner_size", 0, &miss);
    d.d_inner = d_inner;
    const int interval = (int)geti(p + "full_attention_interval", 4);
    d.n_layer -= (int)geti(p + "nextn_predict_layers", 0);
    if (miss) return fail(BTF_ERR_ARG, "btf_decoder: missing qwen35 hyperparameters");
    if (d.n_head_kv <= 0 || d.n_head % d.n_head_kv || d.n_group <= 0 || d.dt_rank % d.n_group || d.n_rot > d.head_dim ||
        d.n_rot % 2 || interval <= 0)
      return fail(BTF_ERR_ARG, "btf_decoder: inconsistent qwen35 hyperparameters");
    D.DK = d.d_state;
    if (d_inner % d.dt_rank) return fail(BTF_ERR_ARG, "btf_decoder: ssm.inner_size %% time_step_rank");
    D.DV = d_inner / d.dt_rank;
    D.NK = d.n_group;
    D.NV = d.dt_rank;
    D.QK = d.d_state * d.n_group;
    D.DI = d_inner;
    D.C = 2 * D.QK + d_inner;
    // prism Hadamard metadata (model.cpp:100-156)
    const int version = (int)geti("prism.hadamard.version", 0);
    const bool tied = geti("prism.hadamard.tied_output", 0) != 0;
    std::set<std::string> inverse;
    if (version) {
      if ((version != 1 && version != 2) || ((version == 2) != tied))
        return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: prism.hadamard.version %d", version);
      block = (int)geti("prism.hadamard.block_size", 0);
      if (block <= 0 || (block & (block - 1)) || block > 1024) return fail(BTF_ERR_ARG, "btf_decoder: bad hadamard block");
      d.hadamard_block = block;
      if (gets("prism.hadamard.transform") != "normalized-sylvester-walsh-hadamard" ||
          gets("prism.hadamard.axis") != "input-last-dimension")
        return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: hadamard transform / axis");
      const std::string mode = gets("prism.hadamard.sign_mode");
      if (mode != "identity" && mode != "explicit") return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: sign mode %s", mode.c_str());
      explicit_signs = mode == "explicit";
      const gguf::Value* wn = kv("prism.hadamard.weight_names");
      if (!wn || wn->as.empty()) return fail(BTF_ERR_ARG, "btf_decoder: prism.hadamard.weight_names missing");
      folded.insert(wn->as.begin(), wn->as.end());
      if (explicit_signs) {
        const gguf::Value* sw = kv("prism.hadamard.sign_widths");
        const gguf::Value* sv = kv("prism.hadamard.sign_values");
        if (!sw || !sv || sw->ai.empty()) return fail(BTF_ERR_ARG, "btf_decoder: explicit sign mode without sign arrays");
        size_t off = 0;
        for (int64_t width : sw->ai) {
          if (width <= 0 || width % block || off + width > sv->ai.size() || signs.count((int)width))
            return fail(BTF_ERR_ARG, "btf_decoder: bad sign width");
          std::vector<float> h(width);
          for (int64_t i = 0; i < width; ++i) {
            const int64_t v = sv->ai[off + i];
            if (v != 1 && v != -1) return fail(BTF_ERR_ARG, "btf_decoder: sign values must be +-1");
            h[i] = (float)v;
          }
          int rc = BTF_OK;
          float* dv = D.alloc<float>(width, &rc, Decoder::kVectors);
          if (rc) return rc;
          D.sign_bytes += (uint64_t)width * 4;
          if (!D.dry && cudaMemcpy(dv, h.data(), width * 4, cudaMemcpyHostToDevice) != cudaSuccess)
            return fail(BTF_ERR_CUDA, "btf_decoder: sign upload");
          signs[(int)width] = dv;
          off += width;
        }
        if (off != sv->ai.size()) return fail(BTF_ERR_ARG, "btf_decoder: sign_values length");
      }
      v_grouped = geti("prism.hadamard.gdn_v_grouped", 0) != 0;
      if (const gguf::Value* inv = kv("prism.hadamard.inverse_weight_names")) {
        for (auto& s : inv->as) {
          if (s != "token_embd.weight") return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: inverse table %s", s.c_str());
          inverse.insert(s);
        }
      }
      if (tied) folded.insert("token_embd.weight");
    }
    // embedding (never transformed on lookup), output norm, lm_head
    const bool embd_folded = folded.count("token_embd.weight") != 0;
    folded.erase("token_embd.weight");
    BTF_TRY(mat("token_embd.weight", &D.embd, false));
    D.weight_bytes -= btf_panel_bytes(D.embd.N, D.embd.K);  // one row per step is read, counted below
    D.weight_bytes += (uint64_t)D.embd.K / 4 + (uint64_t)D.embd.K / 64;
    d.n_vocab = D.embd.N;
    if (D.embd.K != d.n_embd) return fail(BTF_ERR_ARG, "btf_decoder: token_embd width");
    if (inverse.count("token_embd.weight")) {
      D.inv_block = block;
      if (explicit_signs) {
        auto it = signs.find(d.n_embd);
        if (it == signs.end()) return fail(BTF_ERR_ARG, "btf_decoder: no sign vector for the embedding width");
        D.inv_signs = it->second;
      }
    }
    BTF_TRY(vec("output_norm.weight", &D.out_norm, d.n_embd));
    btf_gguf_tensor_info t;
    if (tensor("output.weight", &t)) {
      BTF_TRY(mat("output.weight", &D.output));
    } else {
      if (embd_folded) folded.insert("token_embd.weight");
      BTF_TRY(mat("token_embd.weight", &D.output));
    }
    D.L.resize(d.n_layer);
    for (int il = 0; il < d.n_layer; ++il) {
      const std::string b = "blk." + std::to_string(il) + ".";
      Layer& l = D.L[il];
      l.rec = ((il + 1) % interval) != 0;
      BTF_TRY(vec(b + "attn_norm.weight", &l.attn_norm, d.n_embd));
      BTF_TRY(vec(b + "post_attention_norm.weight", &l.post_norm, d.n_embd));
      BTF_TRY(mat(b + "ffn_gate.weight", &l.gate));
      BTF_TRY(mat(b + "ffn_up.weight", &l.up));
      BTF_TRY(mat(b + "ffn_down.weight", &l.down));
      if (l.rec) {
        BTF_TRY(mat(b + "attn_qkv.weight", &l.qkv));
        BTF_TRY(mat(b + "attn_gate.weight", &l.zg));
        uint32_t at = 0;
        BTF_TRY(vec(b + "ssm_alpha.weight", &l.alpha_w, (int64_t)D.NV * d.n_embd, &at));
        BTF_TRY(vec(b + "ssm_beta.weight", &l.beta_w, (int64_t)D.NV * d.n_embd));
        l.ab_bf16 = at == kBF16;
        BTF_TRY(vec(b + "ssm_a", &l.ssm_a, D.NV));
        BTF_TRY(vec(b + "ssm_dt.bias", &l.ssm_dt, D.NV));
        BTF_TRY(vec(b + "ssm_conv1d.weight", &l.conv_w, (int64_t)d.conv_kernel * D.C));
        BTF_TRY(vec(b + "ssm_norm.weight", &l.ssm_norm, D.DV));
        BTF_TRY(mat(b + "ssm_out.weight", &l.out));
        if (l.qkv.N != D.C || l.zg.N != D.DI || l.out.K != D.DI)
          return fail(BTF_ERR_ARG, "btf_decoder: %sGDN matrix shapes", b.c_str());
      } else {
        BTF_TRY(mat(b + "attn_q.weight", &l.wq));
        BTF_TRY(mat(b + "attn_k.weight", &l.wk));
        BTF_TRY(mat(b + "attn_v.weight", &l.wv));
        BTF_TRY(mat(b + "attn_output.weight", &l.wo));
        BTF_TRY(vec(b + "attn_q_norm.weight", &l.q_norm, d.head_dim));
        BTF_TRY(vec(b + "attn_k_norm.weight", &l.k_norm, d.head_dim));
        if (l.wq.N != 2 * d.head_dim * d.n_head || l.wk.N != d.head_dim * d.n_head_kv ||
            l.wo.K != d.head_dim * d.n_head)
          return fail(BTF_ERR_ARG, "btf_decoder: %sattention matrix shapes", b.c_str());
      }
    }
    return BTF_OK;
  }
};

// Geometry the kernels support.
int check_dims(const Decoder& D) {
  const btf_decoder_dims& d = D.d;
  if (d.n_embd % 128 || d.n_ff % 128 || D.DI % 128 || (d.n_head * d.head_dim) % 128)
    return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: matmul widths must be multiples of 128");
  if (d.head_dim % 32 || d.head_dim > 256) return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: head_dim must be 32..256, a multiple of 32");
  if (D.DK % 16 || D.DK > 128 || D.DV * 4 > 1024 || D.DV % 8)
    return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: GDN head sizes (k <= 128, multiple of 16; v <= 256, multiple of 8)");
  if (d.conv_kernel < 2) return fail(BTF_ERR_UNSUPPORTED, "btf_decoder: conv_kernel < 2");
  if (D.o.n_ctx < 1 || D.o.attn_splits < 1 || D.o.attn_splits > 256)
    return fail(BTF_ERR_ARG, "btf_decoder: n_ctx >= 1 and 1 <= attn_splits <= 256");
  if (D.o.staging_mb < 1 || D.o.staging_mb > 4096) return fail(BTF_ERR_ARG, "btf_decoder: staging_mb 1..4096");
  return BTF_OK;
}

int finish_open(Decoder& D) {
  BTF_TRY(check_dims(D));
  D.theta_scale = std::pow(D.d.rope_base, -2.0f / (float)D.d.n_rot);
  BTF_TRY(make_buffers(D));
  if (D.dry) return BTF_OK;
  for (cudaEvent_t& e : D.ev)
    if (cudaEventCreate(&e) != cudaSuccess) return fail(BTF_ERR_CUDA, "btf_decoder: events");
  return reset_state(D);
}

// Adds the device time of the last bracketed step or run once its end event is reached.
int settle(Decoder& D) {
  if (!D.ev_pending) return BTF_OK;
  D.ev_pending = false;
  float ms = 0.f;
  cudaError_t e = cudaEventSynchronize(D.ev[1]);
  if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, D.ev[0], D.ev[1]);
  if (e != cudaSuccess) return cuda_fail(e, "btf_decoder: step timing");
  D.gpu_s += ms * 1e-3;
  return BTF_OK;
}

double seconds_since(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

btf_decoder_opts defaults(const btf_decoder_opts* o) {
  btf_decoder_opts r{4096, 1, 16, 1, 64, 0};
  if (o) r = *o;
  if (r.staging_mb == 0) r.staging_mb = 64;
  return r;
}

// The decoder's device, library state and stream (nothing for a dry decoder).
int device_setup(Decoder& D, const char* who) {
  if (D.dry) return BTF_OK;
  if (cudaGetDevice(&D.device) != cudaSuccess) return fail(BTF_ERR_CUDA, "%s: no device", who);
  if (int rc = btf_init(D.device)) return rc;
  if (cudaStreamCreateWithFlags(&D.st, cudaStreamNonBlocking) != cudaSuccess) return fail(BTF_ERR_CUDA, "%s: stream", who);
  return BTF_OK;
}

// Binds a qwen35 GGUF: loads this rank's weights and allocates the step buffers
// (a dry decoder only sizes them).
int open_gguf(Decoder& D, const char* path) {
  BTF_TRY(device_setup(D, "btf_decoder_open"));
  void* g = nullptr;
  BTF_TRY(btf_gguf_open(path, &g));
  Binder b{D, g};
  const int rc = b.bind();
  btf_gguf_close(g);
  if (rc) return rc;
  BTF_TRY(finish_open(D));
  if (!D.dry && !D.o.keep_page_cache) {
    // the weights are resident: the file's pages need not stay cached (gpu_decoder.cu:385-391)
    const int fd = ::open(path, O_RDONLY);
    if (fd >= 0) {
      posix_fadvise(fd, 0, 0, POSIX_FADV_DONTNEED);
      ::close(fd);
    }
  }
  return BTF_OK;
}

// Seeded synthetic weights of geometry R.d on this rank (a dry decoder only sizes them).
int build_synthetic(Decoder& R, uint64_t seed);

int check_tp(int world, int rank, const char* who) {
  if (world < 1 || world > BTF_MAX_RANKS || rank < 0 || rank >= world)
    return fail(BTF_ERR_ARG, "%s: need 1 <= world <= %d and 0 <= rank < world", who, BTF_MAX_RANKS);
  return BTF_OK;
}

}  // namespace
}  // namespace btf

using namespace btf;

extern "C" {

int btf_decoder_open_tp(const char* gguf_path, const btf_decoder_opts* opts, int world, int rank, void** handle) {
  if (!gguf_path || !handle) return fail(BTF_ERR_ARG, "btf_decoder_open: null argument");
  BTF_TRY(check_tp(world, rank, "btf_decoder_open"));
  *handle = nullptr;
  auto D = std::make_unique<Decoder>();
  D->o = defaults(opts);
  D->world = world;
  D->rank = rank;
  BTF_TRY(open_gguf(*D, gguf_path));
  D->connected = world == 1;
  *handle = D.release();
  return BTF_OK;
}

int btf_decoder_open(const char* gguf_path, const btf_decoder_opts* opts, void** handle) {
  return btf_decoder_open_tp(gguf_path, opts, 1, 0, handle);
}

int btf_decoder_synthetic_tp(const btf_decoder_dims* dims, uint64_t seed, const btf_decoder_opts* opts, int world,
                             int rank, void** handle) {
  if (!dims || !handle) return fail(BTF_ERR_ARG, "btf_decoder_synthetic: null argument");
  BTF_TRY(check_tp(world, rank, "btf_decoder_synthetic"));
  *handle = nullptr;
  auto D = std::make_unique<Decoder>();
  D->o = defaults(opts);
  D->d = *dims;
  D->world = world;
  D->rank = rank;
  BTF_TRY(build_synthetic(*D, seed));
  D->connected = world == 1;
  *handle = D.release();
  return BTF_OK;
}

}  // extern "C"

namespace btf {
namespace {

int build_synthetic(Decoder& R, uint64_t seed) {
  const int world = R.world, rank = R.rank;
  const btf_decoder_dims& d = R.d;
  if (d.n_layer <= 0 || d.n_head_kv <= 0 || d.n_head % d.n_head_kv || d.n_group <= 0 || d.dt_rank % d.n_group ||
      d.n_rot > d.head_dim || d.n_rot % 2 || d.n_vocab <= 0)
    return fail(BTF_ERR_ARG, "btf_decoder_synthetic: inconsistent dims");
  if (d.hadamard_block < 0 || (d.hadamard_block & (d.hadamard_block - 1)) || d.hadamard_block > 1024)
    return fail(BTF_ERR_ARG, "btf_decoder_synthetic: hadamard_block 0 or a power of two <= 1024");
  BTF_TRY(device_setup(R, "btf_decoder_synthetic"));
  if (R.d.d_inner == 0) R.d.d_inner = d.dt_rank * d.d_state;
  if (d.d_inner % d.dt_rank) return fail(BTF_ERR_ARG, "btf_decoder_synthetic: d_inner %% dt_rank");
  R.DK = d.d_state;
  R.NK = d.n_group;
  R.NV = d.dt_rank;
  R.DV = d.d_inner / d.dt_rank;
  R.DI = d.d_inner;
  R.QK = d.d_state * d.n_group;
  R.C = 2 * R.QK + R.DI;
  BTF_TRY(check_dims(R));
  if (d.hadamard_block && (d.n_embd % d.hadamard_block || d.n_ff % d.hadamard_block || R.DI % d.hadamard_block ||
                           (d.n_head * d.head_dim) % d.hadamard_block))
    return fail(BTF_ERR_ARG, "btf_decoder_synthetic: matmul widths must be multiples of hadamard_block");
  int rc = BTF_OK;
  uint64_t s = seed * 1000003ull;
  const int blk = d.hadamard_block;
  // sharded: this rank's rows of the full matrix (the embedding table is never sharded)
  auto mat = [&](Mat* m, int N, int K, bool ssm_out, bool shard = true) -> int {
    m->N = N;
    m->K = K;
    m->row0 = 0;
    m->n = N;
    if (shard && world > 1) {
      shard_rows(N, world, rank, &m->row0, &m->n);
      int lr0 = 0, ln = 0;
      shard_rows(N, world, world - 1, &lr0, &ln);
      if (ln <= 0)
        return fail(BTF_ERR_ARG, "btf_decoder_synthetic: %d output rows leave a rank of %d without rows", N, world);
    }
    m->pan = R.alloc<uint8_t>(btf_panel_bytes(m->n, K), &rc, Decoder::kPanels);
    if (rc) return rc;
    R.n_mats += 1;
    R.weight_bytes += btf_panel_bytes(m->n, K);
    if (blk) {
      m->hx.block = blk;
      if (ssm_out) {
        m->hx.perm_hd = K / R.NV;
        m->hx.perm_nk = R.NK;
        m->hx.perm_rep = R.NV / R.NK;
      }
    }
    ++s;
    if (R.dry) return BTF_OK;
    const cudaError_t e = launch_fill_panels(m->pan, m->row0, m->n, N, K, s, 1.0f / std::sqrt((float)K), R.st);
    return e == cudaSuccess ? BTF_OK : cuda_fail(e, "btf_decoder_synthetic: fill");
  };
  auto vec = [&](float** p, int64_t n, float base, float spread) -> int {
    *p = R.alloc<float>(n, &rc, Decoder::kVectors);
    if (rc) return rc;
    R.weight_bytes += n * 4;
    ++s;
    if (R.dry) return BTF_OK;
    const cudaError_t e = launch_fill_uniform(*p, n, s, base, spread, R.st);
    return e == cudaSuccess ? BTF_OK : cuda_fail(e, "btf_decoder_synthetic: fill");
  };
  const int E = d.n_embd, F = d.n_ff, H = d.n_head, HK = d.n_head_kv, HD = d.head_dim;
  BTF_TRY(mat(&R.embd, d.n_vocab, E, false, false));
  R.embd.hx = btf_hx{0, 0, 0, 0, nullptr};
  R.weight_bytes -= btf_panel_bytes(d.n_vocab, E);
  R.weight_bytes += (uint64_t)E / 4 + (uint64_t)E / 64;
  R.inv_block = blk;
  BTF_TRY(vec(&R.out_norm, E, 1.0f, 0.3f));
  BTF_TRY(mat(&R.output, d.n_vocab, E, false));
  R.L.resize(d.n_layer);
  for (int il = 0; il < d.n_layer; ++il) {
    Layer& l = R.L[il];
    l.rec = ((il + 1) % 4) != 0;
    BTF_TRY(vec(&l.attn_norm, E, 1.0f, 0.3f));
    BTF_TRY(vec(&l.post_norm, E, 0.8f, 0.3f));
    BTF_TRY(mat(&l.gate, F, E, false));
    BTF_TRY(mat(&l.up, F, E, false));
    BTF_TRY(mat(&l.down, E, F, false));
    if (l.rec) {
      BTF_TRY(mat(&l.qkv, R.C, E, false));
      BTF_TRY(mat(&l.zg, R.DI, E, false));
      BTF_TRY(vec(&l.alpha_w, (int64_t)R.NV * E, 0.f, 1.0f / std::sqrt((float)E)));
      BTF_TRY(vec(&l.beta_w, (int64_t)R.NV * E, 0.f, 1.0f / std::sqrt((float)E)));
      BTF_TRY(vec(&l.ssm_a, R.NV, -0.1f, 0.09f));
      BTF_TRY(vec(&l.ssm_dt, R.NV, 0.f, 4.0f));
      BTF_TRY(vec(&l.conv_w, (int64_t)d.conv_kernel * R.C, 0.f, 0.6f));
      BTF_TRY(vec(&l.ssm_norm, R.DV, 0.85f, 0.3f));
      BTF_TRY(mat(&l.out, E, R.DI, true));
    } else {
      BTF_TRY(mat(&l.wq, 2 * H * HD, E, false));
      BTF_TRY(mat(&l.wk, HK * HD, E, false));
      BTF_TRY(mat(&l.wv, HK * HD, E, false));
      BTF_TRY(mat(&l.wo, E, H * HD, false));
      BTF_TRY(vec(&l.q_norm, HD, 1.2f, 0.3f));
      BTF_TRY(vec(&l.k_norm, HD, 1.2f, 0.3f));
    }
  }
  if (!R.dry && cudaStreamSynchronize(R.st) != cudaSuccess) return fail(BTF_ERR_CUDA, "btf_decoder_synthetic: fill");
  return finish_open(R);
}

}  // namespace
}  // namespace btf

extern "C" {

int btf_decoder_synthetic(const btf_decoder_dims* dims, uint64_t seed, const btf_decoder_opts* opts, void** handle) {
  return btf_decoder_synthetic_tp(dims, seed, opts, 1, 0, handle);
}

int btf_shard_rows(int N, int world, int rank, int* row0, int* rows) {
  if (N <= 0 || world < 1 || rank < 0 || rank >= world || !row0 || !rows)
    return fail(BTF_ERR_ARG, "btf_shard_rows: need N > 0, 0 <= rank < world and output pointers");
  shard_rows(N, world, rank, row0, rows);
  return BTF_OK;
}

int btf_decoder_arena(void* handle, void** base, uint64_t* bytes) {
  if (!handle || !base || !bytes) return fail(BTF_ERR_ARG, "btf_decoder_arena: null argument");
  const Decoder& D = *static_cast<const Decoder*>(handle);
  *base = D.arena;
  *bytes = D.arena_bytes;
  return BTF_OK;
}

int btf_decoder_connect(void* handle, void* const* peer_arenas) {
  if (!handle || !peer_arenas) return fail(BTF_ERR_ARG, "btf_decoder_connect: null argument");
  Decoder& D = *static_cast<Decoder*>(handle);
  if (D.world < 2) return fail(BTF_ERR_STATE, "btf_decoder_connect: not a tensor-parallel decoder");
  if (D.exec) return fail(BTF_ERR_STATE, "btf_decoder_connect: already captured");
  for (int r = 0; r < D.world; ++r) {
    if (r != D.rank && !peer_arenas[r]) return fail(BTF_ERR_ARG, "btf_decoder_connect: arena of rank %d is null", r);
    D.peers[r] = r == D.rank ? D.arena : static_cast<uint8_t*>(peer_arenas[r]);
  }
  D.connected = true;
  return BTF_OK;
}

int btf_decoder_step(void* handle, int32_t token, float* logits, int32_t* next) {
  if (!handle) return fail(BTF_ERR_ARG, "btf_decoder_step: null handle");
  Decoder& D = *static_cast<Decoder*>(handle);
  if (token < 0 || token >= D.d.n_vocab) return fail(BTF_ERR_ARG, "btf_decoder_step: token %d out of range", token);
  const auto t0 = std::chrono::steady_clock::now();
  BTF_TRY(settle(D));
  D.h_io[0] = token;
  cudaError_t e = cudaMemcpyAsync(D.d_tok, D.h_io, sizeof(int32_t), cudaMemcpyHostToDevice, D.st);
  if (e == cudaSuccess) e = cudaEventRecord(D.ev[0], D.st);
  if (e != cudaSuccess) return cuda_fail(e, "btf_decoder_step: token");
  BTF_TRY(run_step(D));
  e = cudaEventRecord(D.ev[1], D.st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(D.h_io + 1, D.d_next, sizeof(int32_t), cudaMemcpyDeviceToHost, D.st);
  if (e == cudaSuccess && logits)
    e = cudaMemcpyAsync(logits, D.logits, (size_t)D.d.n_vocab * sizeof(float), cudaMemcpyDeviceToHost, D.st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(D.st);
  if (e != cudaSuccess) return cuda_fail(e, "btf_decoder_step");
  D.ev_pending = true;
  BTF_TRY(settle(D));
  D.n_steps += 1;
  D.wall_s += seconds_since(t0);
  if (next) *next = D.h_io[1];
  return BTF_OK;
}

int btf_decoder_prefill(void* handle, const int32_t* tokens_host, int n, int max_chunk, float* logits,
                        int32_t* next) {
  if (!handle || !tokens_host || n < 1) return fail(BTF_ERR_ARG, "btf_decoder_prefill: null handle/tokens or n < 1");
  Decoder& D = *static_cast<Decoder*>(handle);
  if (max_chunk == 0) max_chunk = Decoder::kMaxChunk;
  if (max_chunk < 1 || max_chunk > Decoder::kMaxChunk)
    return fail(BTF_ERR_ARG, "btf_decoder_prefill: max_chunk must be 1..%d (got %d)", Decoder::kMaxChunk, max_chunk);
  if (D.world > 1)
    return fail(BTF_ERR_UNSUPPORTED, "btf_decoder_prefill: tensor-parallel decoders take the prompt by btf_decoder_step");
  if (D.pos + n > D.o.n_ctx) return fail(BTF_ERR_ARG, "btf_decoder_prefill: context full (n_ctx %d)", D.o.n_ctx);
  for (int i = 0; i < n; ++i)
    if (tokens_host[i] < 0 || tokens_host[i] >= D.d.n_vocab)
      return fail(BTF_ERR_ARG, "btf_decoder_prefill: token %d out of range", tokens_host[i]);
  BTF_TRY(settle(D));
  for (int i = 0; i < n; i += max_chunk) {
    const int M = std::min(max_chunk, n - i);
    int32_t tp[2 * Decoder::kMaxChunk] = {};
    for (int m = 0; m < M; ++m) {
      tp[m] = tokens_host[i + m];
      tp[Decoder::kMaxChunk + m] = D.pos + m;
    }
    // the previous chunk's kernels are done with the chunk arrays (the stream is idle here)
    cudaError_t e = cudaStreamSynchronize(D.st);
    if (e == cudaSuccess) e = cudaMemcpy(D.d_ptok, tp, 2 * Decoder::kMaxChunk * sizeof(int32_t), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "btf_decoder_prefill: tokens");
    BTF_TRY(enqueue_chunk(D, M));
    D.pos += M;
    const int32_t pos = D.pos;  // the device position the next step reads
    if ((e = cudaStreamSynchronize(D.st)) == cudaSuccess)
      e = cudaMemcpy(D.d_pos, &pos, sizeof(int32_t), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return cuda_fail(e, "btf_decoder_prefill");
  }
  cudaError_t e = cudaMemcpy(D.h_io + 1, D.d_next, sizeof(int32_t), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess && logits)
    e = cudaMemcpy(logits, D.logits, (size_t)D.d.n_vocab * sizeof(float), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "btf_decoder_prefill: results");
  if (next) *next = D.h_io[1];
  return BTF_OK;
}

int btf_decoder_run(void* handle, int steps) {
  if (!handle || steps < 0) return fail(BTF_ERR_ARG, "btf_decoder_run: bad argument");
  Decoder& D = *static_cast<Decoder*>(handle);
  const auto t0 = std::chrono::steady_clock::now();
  BTF_TRY(settle(D));
  cudaError_t e = cudaEventRecord(D.ev[0], D.st);
  if (e != cudaSuccess) return cuda_fail(e, "btf_decoder_run: event");
  int done = 0, rc = BTF_OK;
  for (; done < steps && rc == BTF_OK; ++done) rc = run_step(D);
  if (rc) --done;
  D.n_steps += done;
  if ((e = cudaEventRecord(D.ev[1], D.st)) != cudaSuccess && rc == BTF_OK) rc = cuda_fail(e, "btf_decoder_run: event");
  D.ev_pending = e == cudaSuccess;
  D.wall_s += seconds_since(t0);
  return rc;
}

int btf_decoder_stats(void* handle, btf_step_stats* out) {
  if (!handle || !out) return fail(BTF_ERR_ARG, "btf_decoder_stats: null argument");
  Decoder& D = *static_cast<Decoder*>(handle);
  BTF_TRY(settle(D));
  std::memset(out, 0, sizeof *out);
  out->steps = D.n_steps;
  out->wall_s = D.wall_s;
  out->gpu_s = D.gpu_s;
  // weights and the embedding table are device-resident: a step copies none
  // and reads nothing from mapped host memory
  out->weight_xfer_bytes = 0;
  out->weight_xfer_s = 0;
  out->mapped_read_bytes = 0;
  return BTF_OK;
}

int btf_decoder_reset_stats(void* handle) {
  if (!handle) return fail(BTF_ERR_ARG, "btf_decoder_reset_stats: null handle");
  Decoder& D = *static_cast<Decoder*>(handle);
  BTF_TRY(settle(D));
  D.n_steps = 0;
  D.wall_s = D.gpu_s = 0;
  return BTF_OK;
}

int btf_decoder_reset(void* handle) {
  if (!handle) return fail(BTF_ERR_ARG, "btf_decoder_reset: null handle");
  return reset_state(*static_cast<Decoder*>(handle));
}

int btf_decoder_close(void* handle) {
  delete static_cast<Decoder*>(handle);
  return BTF_OK;
}

int btf_decoder_get_info(void* handle, btf_decoder_info* out) {
  if (!handle || !out) return fail(BTF_ERR_ARG, "btf_decoder_get_info: null argument");
  const Decoder& D = *static_cast<const Decoder*>(handle);
  out->dims = D.d;
  out->pos = D.pos;
  out->stream = D.st;
  out->weight_bytes = D.weight_bytes;
  out->state_bytes = D.state_bytes;
  out->kv_bytes_per_token = D.kv_bytes_per_token;
  out->logits = D.logits;
  out->device_bytes = D.device_total();
  return BTF_OK;
}

}  // extern "C"

namespace btf {
namespace {

void fill_plan(const Decoder& D, btf_memory_plan* p) {
  std::memset(p, 0, sizeof *p);
  p->panel_bytes = D.dev_bytes[Decoder::kPanels];
  p->vector_bytes = D.dev_bytes[Decoder::kVectors];
  p->kv_cache_bytes = D.dev_bytes[Decoder::kKv];
  p->state_bytes = D.dev_bytes[Decoder::kState];
  p->work_bytes = D.dev_bytes[Decoder::kWork];
  p->device_bytes = D.device_total();
  p->pinned_bytes = 4 * sizeof(int32_t);
  p->staging_bytes = D.staging_peak;
  // every resident byte one step reads once (one embedding row, the weights,
  // the sign vectors), the recurrent state read and written, the logits
  // written and read by the argmax; plus the K and V rows per cached token
  p->decode_bytes_fixed = D.weight_bytes + D.sign_bytes + D.state_bytes + 2ull * D.d.n_vocab * 4;
  p->decode_bytes_per_ctx = D.kv_bytes_per_token;
  p->n_matrices = D.n_mats;
  p->dims = D.d;
}

}  // namespace
}  // namespace btf

extern "C" {

int btf_plan_memory(const char* gguf_path, const btf_decoder_opts* opts, int world, int rank, btf_memory_plan* out) {
  if (!gguf_path || !out) return fail(BTF_ERR_ARG, "btf_plan_memory: null argument");
  BTF_TRY(check_tp(world, rank, "btf_plan_memory"));
  Decoder D;
  D.dry = true;
  D.o = defaults(opts);
  D.world = world;
  D.rank = rank;
  BTF_TRY(open_gguf(D, gguf_path));
  fill_plan(D, out);
  return BTF_OK;
}

int btf_plan_memory_synthetic(const btf_decoder_dims* dims, const btf_decoder_opts* opts, int world, int rank,
                              btf_memory_plan* out) {
  if (!dims || !out) return fail(BTF_ERR_ARG, "btf_plan_memory_synthetic: null argument");
  BTF_TRY(check_tp(world, rank, "btf_plan_memory_synthetic"));
  Decoder D;
  D.dry = true;
  D.o = defaults(opts);
  D.d = *dims;
  D.world = world;
  D.rank = rank;
  BTF_TRY(build_synthetic(D, 0));
  fill_plan(D, out);
  return BTF_OK;
}

}  // extern "C"
