// Launchers of the non-matmul decode-step kernels (csrc/decode.cu). Internal:
// the decoder (csrc/decoder.cu) calls them; the C ABI exposes the decoder.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

namespace btf {

// x[E] = inverse transform of row *tok of a panel matrix [V][E] (blk = 0: none).
cudaError_t launch_embed(const uint8_t* panels, int V, int E, const int32_t* tok, int blk, const float* signs,
                         float* x, cudaStream_t st);
// The recurrent mixer of NV v-heads (one kernel): alpha/beta gates from xn, the
// causal conv (ring [K][C] indexed by *pos) + SiLU of qkv, the gated delta rule
// on state [NV][DV][DK], RMSNorm(norm_w) * silu(z) -> o[NV * DV].
struct GdnArgs {
  const float *xn, *aw, *bw, *dt, *a;
  int E, bf16_in;
  const float* qkv;
  float* ring;
  const float* conv_w;
  int K, C;
  const float* z;
  float* state;
  const float* norm_w;
  int NK, DK, DV, QK;
  float eps;
  const int32_t* pos;
  float* o;
  int NV;
};
cudaError_t launch_gdn_mix(const GdnArgs& args, cudaStream_t st);
// The attention of one layer at position *pos, one launch: q/k RMSNorm + RoPE
// (q fp16-rounded when round_q), k and v into row *pos of the fp16 caches
// [n_ctx][HK*D], softmax attention of the H q-heads over keys 0..*pos in
// `splits` key ranges (part: [H][splits][D + 2] floats), combined by each
// head's last CTA, times sigmoid(gate) -> o[H*D]. cnt: H ints, zero before the
// first launch (each launch leaves them zero).
cudaError_t launch_attention_fused(const float* qf, const float* k, const float* v, const float* qn, const float* kn,
                                   int H, int HK, int D, int R, float theta_scale, float eps, const int32_t* pos,
                                   int round_q, void* kc, void* vc, int n_ctx, int splits, float* part, int* cnt,
                                   float* o, cudaStream_t st);
// Greedy argmax of x[n] (lowest index on ties) -> *out; also *tok_next = token and
// *pos += 1 when those are non-null. pv/pi: `parts` partials.
cudaError_t launch_argmax(const float* x, int n, float* pv, int* pi, int parts, int32_t* out, int32_t* tok_next,
                          int32_t* pos, cudaStream_t st);
// Seeded synthetic weights: rows [row0, row0 + rows) (row0 a multiple of 8) of
// a panel matrix [N][K] of codes 0..2 with fp16 scales |N(0,1)| * scale_mul
// (each value a function of its position in the full matrix), and uniform
// floats base +- spread.
cudaError_t launch_fill_panels(uint8_t* panels, int row0, int rows, int N, int K, uint64_t seed, float scale_mul,
                               cudaStream_t st);
cudaError_t launch_fill_uniform(float* x, int64_t n, uint64_t seed, float base, float spread, cudaStream_t st);

}  // namespace btf
