// C entry points over the REFERENCE's own compiled sources — TEST INFRASTRUCTURE ONLY.
//
// oracle/Makefile compiles this file together with the reference's sources
// (src/repack.cpp and ref/bonsai-decoder/src/{types,cpu_ops,gguf,model,
// mapped_file}.cpp, read in place from the reference tree) into
// oracle/_ref/libbtf_ref.so. Nothing here re-implements reference math except
// ref_gemv, whose 20-line loop is the body of the private member
// EmuDecoder::gemv (src/emu_decoder.cpp:143-165) restated around the public
// helpers it calls (btf::sub_dot_host, bd::fp16_to_f32, bd::ThreadPool),
// because that member is not reachable from outside its translation unit.
//
// Used by tests/ to pin oracle/oracle.c, and by bench.py's CPU baseline /
// `--impl reference` arm as the reference's own CPU GEMV.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "bd/cpu_ops.hpp"
#include "bd/gguf.hpp"
#include "bd/types.hpp"
#include "btf/fast.hpp"
#include "btf/packed.hpp"
#include <memory>

#define REF_API extern "C" __attribute__((visibility("default")))

REF_API uint16_t ref_f32_to_f16(float f) { return bd::f32_to_fp16(f); }
REF_API float ref_f16_to_f32(uint16_t h) { return bd::fp16_to_f32(h); }

// bd::quant_row(PTQ1_0) — ref/bonsai-decoder/src/types.cpp:289-320
REF_API void ref_ptq_quant_row(const float* x, uint8_t* out, int64_t k) { bd::quant_row(bd::T_PTQ1_0, x, out, k); }

// bd::ptq1_0_trit — ref/bonsai-decoder/include/bd/types.hpp:70-78
REF_API int ref_ptq_trit(const uint8_t* blk, int e) { return bd::ptq1_0_trit(blk, e); }

// btf::repack_rows — src/repack.cpp:16-27
REF_API void ref_repack_rows(const uint8_t* src, int64_t rows, int64_t K, uint8_t* codes, uint16_t* scales) {
  btf::repack_rows(src, rows, K, codes, scales);
}

// btf::packed_code — include/btf/packed.hpp:94-98
REF_API int ref_packed_code(const uint8_t* row_codes, int64_t e) { return btf::packed_code(row_codes, e); }

// btf::q8_block_host — include/btf/packed.hpp:117-134
REF_API int ref_q8_block(const float* x, int8_t* q, float* d) { return btf::q8_block_host(x, q, d); }

// bd::round_q8_0 — ref/bonsai-decoder/src/cpu_ops.cpp:189-197
REF_API void ref_round_q8_0(const float* x, int64_t n, float* out) { bd::round_q8_0(x, n, out); }

// btf::sub_dot_host — include/btf/packed.hpp:108-113
REF_API int ref_sub_dot(uint32_t w0, uint32_t w1, const uint32_t* aw) { return btf::sub_dot_host(w0, w1, aw); }

// bd::ThreadPool — ref/bonsai-decoder/src/cpu_ops.cpp:19-73
REF_API void* ref_pool_create(int threads) { return new bd::ThreadPool(threads); }
REF_API void ref_pool_destroy(void* p) { delete static_cast<bd::ThreadPool*>(p); }
REF_API int ref_pool_size(void* p) { return static_cast<bd::ThreadPool*>(p)->size(); }

// The emulator GEMV, src/emu_decoder.cpp:143-165, on T2 codes/scales.
// add != 0: y += W x, else y = W x. pool may be null (one thread).
REF_API void ref_gemv(void* pool, const uint8_t* codes, const uint16_t* scales, int64_t N, int64_t K,
                      const int8_t* q, const float* d, const int32_t* s, int M, float* y, int64_t ldy, int add) {
  const int64_t nsub = K / 32;
  auto run = [&](int64_t b, int64_t e) {
    for (int64_t r = b; r < e; ++r) {
      const uint8_t* cr = codes + r * (K / 4);
      const uint16_t* sr = scales + r * (K / 128);
      for (int m = 0; m < M; ++m) {
        const uint32_t* aw = reinterpret_cast<const uint32_t*>(q + (size_t)m * K);
        float acc = 0.f;
        for (int64_t sb = 0; sb < nsub; ++sb) {
          uint32_t w0, w1;
          std::memcpy(&w0, cr + sb * 8, 4);
          std::memcpy(&w1, cr + sb * 8 + 4, 4);
          const int idot = btf::sub_dot_host(w0, w1, aw + sb * 8) - s[(size_t)m * nsub + sb];
          acc += bd::fp16_to_f32(sr[sb / 4]) * d[(size_t)m * nsub + sb] * (float)idot;
        }
        float& out = y[(size_t)m * ldy + r];
        out = add ? out + acc : acc;
      }
    }
  };
  if (pool)
    static_cast<bd::ThreadPool*>(pool)->parallel_for(N, run);
  else
    run(0, N);
}

// bd::matvec_raw(ggml_act = true) on a raw PTQ1_0 [N][K] tensor —
// ref/bonsai-decoder/src/cpu_ops.cpp:199-243, the second oracle of
// tests/test_packed.cpp:63-87.
REF_API void ref_matvec_raw(void* pool, const uint8_t* src, int64_t N, int64_t K, const float* x, float* y) {
  bd::GgufTensor t;
  t.name = "w";
  t.ne = {K, N};
  t.type = bd::T_PTQ1_0;
  t.data = src;
  bd::ThreadPool one(1);
  bd::ThreadPool& p = pool ? *static_cast<bd::ThreadPool*>(pool) : one;
  bd::matvec_raw(p, t, x, y, true);
}

// bd::rmsnorm — ref/bonsai-decoder/src/cpu_ops.cpp:121-127
REF_API void ref_rmsnorm(const float* x, const float* w, int64_t n, float eps, float* y) { bd::rmsnorm(x, w, n, eps, y); }

// bd::hadamard_input — ref/bonsai-decoder/src/cpu_ops.cpp:90-111
REF_API void ref_hadamard_input(int block, int perm_hd, int perm_nk, int perm_rep, const float* signs, const float* x,
                                int64_t n, float* out) {
  bd::HadamardXform hx;
  hx.active = block > 0;
  hx.block = block;
  std::vector<float> sg;
  if (signs) {
    sg.assign(signs, signs + n);
    hx.signs = &sg;
  }
  hx.perm_hd = perm_hd;
  hx.perm_nk = perm_nk;
  hx.perm_rep = perm_rep;
  bd::hadamard_input(hx, x, n, out);
}

// bd::GgufWriter — ref/bonsai-decoder/include/bd/gguf.hpp:88-114: writes a GGUF
// file with a few metadata entries of several kinds and the given 2-D tensors
// (ne0 = row length, ne1 = rows). Used to make test fixtures.
REF_API int ref_gguf_write(const char* path, int n, const char** names, const int64_t* ne0, const int64_t* ne1,
                           const uint32_t* types, const uint8_t** data, const uint64_t* bytes, uint32_t alignment) {
  bd::GgufWriter w;
  w.kv_str("general.architecture", "bonsai-test");
  w.kv_u32("test.u32", 7u);
  w.kv_arr_f32("test.floats", {1.5f, -2.0f, 3.25f});
  w.kv_arr_str("test.strings", {"alpha", "beta"});
  w.kv_bool("test.flag", true);
  for (int i = 0; i < n; ++i)
    w.tensor(names[i], {ne0[i], ne1[i]}, types[i], std::vector<uint8_t>(data[i], data[i] + bytes[i]));
  const std::vector<uint8_t> img = w.finish(alignment);
  FILE* f = std::fopen(path, "wb");
  if (!f) return 1;
  const size_t wr = std::fwrite(img.data(), 1, img.size(), f);
  std::fclose(f);
  return wr == img.size() ? 0 : 2;
}

// bd::Gguf::open — the reference's reader, for cross-checking where a tensor's
// data starts in the file.
REF_API int64_t ref_gguf_tensor_offset(const char* path, const char* name) {
  auto g = bd::Gguf::open(path);
  const bd::GgufTensor* t = g->tensor(name);
  return t ? (int64_t)(g->data_offset + t->offset) : -1;  // byte offset of the tensor data in the file
}

// ---------------------------------------------------------------- whole decoder
// bd::make_synth_qwen35 (ref/bonsai-decoder/src/synth.cpp:50-177): writes the
// reference's synthetic qwen35 GGUF (every layer type, prism Hadamard fold,
// PTQ1_0 matrices, BF16 alpha/beta) to `path`. geom (may be null) overrides
// {n_embd, n_ff, n_head, n_head_kv, head_dim, n_rot, d_state, n_group, dt_rank,
// hadamard_block, hadamard, explicit_signs, gdn_v_grouped, small_mat_type}.
#include "bd/synth.hpp"
#include "bd/model.hpp"

REF_API int ref_synth_write(const char* path, int n_layer, uint64_t seed, const int* geom) {
  bd::SynthOptions o;
  o.n_layer = n_layer;
  o.seed = seed;
  if (geom) {
    o.n_embd = geom[0]; o.n_ff = geom[1]; o.n_head = geom[2]; o.n_head_kv = geom[3]; o.head_dim = geom[4];
    o.n_rot = geom[5]; o.d_state = geom[6]; o.n_group = geom[7]; o.dt_rank = geom[8]; o.hadamard_block = geom[9];
    o.hadamard = geom[10] != 0; o.explicit_signs = geom[11] != 0; o.gdn_v_grouped = geom[12] != 0;
    o.small_mat_type = (uint32_t)geom[13];
  }
  const std::vector<uint8_t> img = bd::make_synth_qwen35(o);
  FILE* f = std::fopen(path, "wb");
  if (!f) return 1;
  const size_t wr = std::fwrite(img.data(), 1, img.size(), f);
  std::fclose(f);
  return wr == img.size() ? 0 : 2;
}

// btf::make_emu_decoder (src/emu_decoder.cpp:377-379): the reference's CPU
// emulator of its CUDA decode step, over a model file.
struct RefEmu {
  std::unique_ptr<bd::Model> model;
  std::unique_ptr<btf::FastDecoder> dec;
};
REF_API void* ref_emu_open(const char* path, int n_ctx, int round_q_f16, int threads) {
  try {
    auto* e = new RefEmu;
    e->model = bd::Model::load(path);
    btf::FastOptions o;
    o.n_ctx = n_ctx;
    o.round_q_f16 = round_q_f16 != 0;
    o.threads = threads;
    o.max_batch = 1;
    e->dec = btf::make_emu_decoder(*e->model, o);
    return e;
  } catch (const std::exception& ex) {
    std::fprintf(stderr, "ref_emu_open: %s\n", ex.what());
    return nullptr;
  }
}
// One decode step: returns the greedy next token; logits (n_vocab floats) may be null.
REF_API int ref_emu_step(void* h, int32_t token, float* logits) {
  return static_cast<RefEmu*>(h)->dec->step(token, logits);
}
REF_API void ref_emu_reset(void* h) { static_cast<RefEmu*>(h)->dec->reset(); }
REF_API void ref_emu_close(void* h) { delete static_cast<RefEmu*>(h); }
// {n_layer, n_embd, n_ff, n_vocab, n_head, n_head_kv, head_dim, n_rot, d_state, n_group, dt_rank, d_inner, conv_kernel}
REF_API void ref_emu_hparams(void* h, int* out) {
  const bd::HParams& p = static_cast<RefEmu*>(h)->model->hp;
  const int v[13] = {p.n_layer, p.n_embd, p.n_ff, p.n_vocab, p.n_head, p.n_head_kv, p.head_dim,
                     p.n_rot, p.d_state, p.n_group, p.dt_rank, p.d_inner, p.conv_kernel};
  std::memcpy(out, v, sizeof v);
}
