// Kernels of the batch-1 decode step other than the matmuls (the ternary
// GEMVs and the fused prep live in gemv.cu and quant.cu).
//
// Each kernel restates one piece of the reference's CPU emulator of its CUDA
// decode step (src/emu_decoder.cpp of bonsai-ternary-fast), which is the
// oracle the decoder is tested against:
//   embed_kernel      packed token_embd row -> inverse transform   (:175-183)
//   gdn_mix_kernel    per v-head: alpha / beta dots, causal conv +
//                     SiLU, gated delta rule, gated RMSNorm         (:235-298)
//   attn_fused_kernel q/k RMSNorm, partial RoPE, fp16 KV write      (:307-338)
//                     and softmax attention over the fp16 KV cache
//                     in key splits, then the sigmoid gate          (:339-372)
//   argmax kernels    greedy token, lowest index on ties            (:214-217)
// The decode position lives in device memory, so one captured graph serves
// every token. Every kernel is launched with programmatic dependent launch:
// it may start while the previous kernel drains and reads that kernel's
// outputs only after griddepcontrol.wait.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cfloat>

#include "common.cuh"
#include "decode.h"

namespace btf {
namespace {

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }
// bd::softplus (cpu_ops.cpp:136): threshold 20
__device__ __forceinline__ float softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
// bd::f32_to_bf16 (types.cpp:64-70) then back: round to nearest even on the bits
__device__ __forceinline__ float round_bf16(float f) {
  uint32_t x = __float_as_uint(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return __uint_as_float(((x >> 16) | 0x40u) << 16);
  x += 0x7fffu + ((x >> 16) & 1u);
  return __uint_as_float((x >> 16) << 16);
}

// Block-wide sum of one double per thread (blockDim.x a multiple of 32, <= 1024).
__device__ double block_sum(double v, double* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  double s = 0.0;
  for (int i = 0; i < nw; ++i) s += red[i];
  return s;
}

// Two block sums at once, in block_sum's order, with one barrier: red must hold
// 2 x 32 doubles and must not be read by an unfinished earlier reduction (the
// caller alternates buffers, or a barrier lies between).
__device__ void block_sum2(double& a, double& b, double* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
  }
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  if ((threadIdx.x & 31) == 0) {
    red[w] = a;
    red[32 + w] = b;
  }
  __syncthreads();
  double sa = 0.0, sb = 0.0;
  for (int i = 0; i < nw; ++i) {
    sa += red[i];
    sb += red[32 + i];
  }
  a = sa;
  b = sb;
}

// bd::rmsnorm (cpu_ops.cpp:116-122): double sum of squares, float mean,
// 1/sqrt(mean + eps) in float.
__device__ __forceinline__ float rms_scale(double sumsq, int n, float eps) {
  const float mean = (float)(sumsq / n);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

// ------------------------------------------------------------------ embed
// One CTA per transform block of `blk` columns (blk threads; blk = 0: no
// transform, 256 columns per CTA). Row r of the panel matrix: group r/8, quad
// (r%8)/4, bit pair 2*(r%4) of byte (c%4) of word (c%16)/4 of the 16-column half.
__global__ void embed_kernel(const uint8_t* __restrict__ pan, int V, int E, int S, const int32_t* __restrict__ tok,
                             int blk, const float* __restrict__ signs, float* __restrict__ x) {
  extern __shared__ float sh[];
  pdl_launch_dependents();
  pdl_wait();  // the token is written by the previous step's argmax
  const int n = blk ? blk : blockDim.x;
  const int e = blockIdx.x * n + threadIdx.x;
  const int r = min(max(*tok, 0), V - 1);  // the host validates tokens; the clamp keeps reads in bounds
  const int g = r >> 3, rr = r & 7, h = rr >> 2, k = rr & 3;
  float v = 0.f;
  if (e < E) {
    const int j = e >> 10, c = e & 1023, bb = c >> 7, sb = (c >> 5) & 3, hv = (c >> 4) & 1;
    const uint8_t* p = pan + ((int64_t)g * S + j) * kPanelBytes;
    const uint8_t byte = p[h * 1024 + hv * 512 + (bb * 4 + sb) * 16 + ((c >> 2) & 3) * 4 + (c & 3)];
    const int code = (byte >> (2 * k)) & 3;
    const uint16_t sc = *reinterpret_cast<const uint16_t*>(p + kCodeBytes + bb * 16 + rr * 2);
    v = __fmul_rn((float)(code - 1), __half2float(__ushort_as_half(sc)));
  }
  if (!blk) {
    if (e < E) x[e] = v;
    return;
  }
  // bd::hadamard_inverse (cpu_ops.cpp:109-114): fwht of the block, * 1/sqrt(blk), then signs
  if (n == 1024) {
    // the same butterflies in the same order with 2 barriers: lengths 1 .. 16 in
    // shuffles (warp c holds columns 32c .. 32c+31), a padded transpose (column
    // 32 l + c to thread (c, l)) for lengths 32 .. 512, and back
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int len = 1; len < 32; len <<= 1) {
      const float q = __shfl_xor_sync(0xffffffffu, v, len);
      v = (lane & len) ? __fsub_rn(q, v) : __fadd_rn(v, q);
    }
    sh[threadIdx.x + w] = v;
    __syncthreads();
    float t = sh[33 * lane + w];
    for (int k2 = 1; k2 < 32; k2 <<= 1) {
      const float q = __shfl_xor_sync(0xffffffffu, t, k2);
      t = (lane & k2) ? __fsub_rn(q, t) : __fadd_rn(t, q);
    }
    sh[33 * lane + w] = t;
    __syncthreads();
    if (e < E) {
      float o = __fmul_rn(sh[threadIdx.x + w], __fdiv_rn(1.0f, __fsqrt_rn((float)n)));
      if (signs) o = __fmul_rn(o, signs[e]);
      x[e] = o;
    }
    return;
  }
  sh[threadIdx.x] = v;
  __syncthreads();
  for (int len = 1; len < n; len <<= 1) {
    const int i = threadIdx.x;
    float a = 0.f, b = 0.f;
    const bool lo = !(i & len);
    if (lo) {
      a = sh[i];
      b = sh[i + len];
    }
    __syncthreads();
    if (lo) {
      sh[i] = __fadd_rn(a, b);
      sh[i + len] = __fsub_rn(a, b);
    }
    __syncthreads();
  }
  if (e < E) {
    float o = __fmul_rn(sh[threadIdx.x], __fdiv_rn(1.0f, __fsqrt_rn((float)n)));
    if (signs) o = __fmul_rn(o, signs[e]);
    x[e] = o;
  }
}

// ------------------------------------------------------------------ delta-net mixer
// One CTA per v-head h (kTpc threads per state column): the whole recurrent
// mixer of one head after the qkv / z GEMV.
//   alpha / beta (emulator :235-249): beta = sigmoid(bw[h] . x),
//     g = softplus(aw[h] . x + dt[h]) * a[h], x = xn rounded to bf16 when the
//     weights are bf16;
//   causal conv + SiLU (:251-264) of the head's channels: q and k rows of
//     k-head kh = h % NK and the head's v row. The conv state is a ring of K
//     input rows indexed by position: tap i reads the input of position
//     pos - (K-1) + i; the step writes only slot pos % K, which no tap of this
//     step reads, so heads sharing a k-head read and write it without a race
//     (they write the same values);
//   gated delta rule (:266-290) on the l2-normalised q, k, then RMSNorm with
//     ssm_norm and * silu(z) (:291-298).
constexpr int kTpc = 4;
struct GdnParams {
  const float *xn, *aw, *bw, *dt, *a;
  int E, bf16_in;
  const float* qkv;   // [C] GEMV output (conv input)
  float* ring;        // [K][C]
  const float* conv_w;  // [C][K]
  int K, C;
  const float* z;     // [DI]
  float* state;       // [NV][DV][DK]
  const float* norm_w;
  int NK, DK, DV, QK;
  float eps;
  const int32_t* pos;
  float* o;           // [DI]
};
__global__ void gdn_mix_kernel(const __grid_constant__ GdnParams p) {
  extern __shared__ float sm[];  // q[DK], k[DK], v[DV], out[DV]
  // reduction buffers, used in turn: each is rewritten only after a barrier
  // that follows every read of its previous use
  __shared__ double red[2][64];
  float* q = sm;
  float* k = sm + p.DK;
  float* vv = sm + 2 * p.DK;
  float* ov = sm + 2 * p.DK + p.DV;
  const int h = blockIdx.x, kh = h % p.NK, tid = threadIdx.x;
  // the head's alpha / beta weight rows (16-byte loads; E % 4 == 0, rows 16-byte
  // aligned) are constants: the first kPre float4 of each per thread are fetched
  // before the wait, while the previous kernel drains
  constexpr int kPre = 4;
  const float4* a4 = reinterpret_cast<const float4*>(p.aw + (int64_t)h * p.E);
  const float4* b4 = reinterpret_cast<const float4*>(p.bw + (int64_t)h * p.E);
  const int n4 = p.E >> 2;
  float4 ap[kPre], bp[kPre];
#pragma unroll
  for (int u = 0; u < kPre; ++u) {
    const int i = tid + u * blockDim.x;
    ap[u] = i < n4 ? a4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    bp[u] = i < n4 ? b4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float nw0 = tid < p.DV ? p.norm_w[tid] : 0.f;  // the output norm weight (a constant)
  pdl_launch_dependents();
  pdl_wait();  // xn, qkv, z and the ring come from earlier kernels
  const float z0 = tid < p.DV ? p.z[(int64_t)h * p.DV + tid] : 0.f;  // read early, used last
  // thread (j, part) holds floats i = 16 t + 4 part + {0..3} of state column j
  // (DK <= 128); its part of the state is loaded now, so that the read is in
  // flight during the dots, the conv and the norms below
  const int j = tid / kTpc, part = tid % kTpc;
  const int nt = p.DK / (4 * kTpc);
  float4* col = reinterpret_cast<float4*>(p.state + ((int64_t)h * p.DV + j) * p.DK) + part;
  float4 st[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) st[t] = t < nt ? col[t * kTpc] : make_float4(0.f, 0.f, 0.f, 0.f);
  // alpha / beta dots
  double sa = 0.0, sb = 0.0;
  {
    const float4* x4 = reinterpret_cast<const float4*>(p.xn);
    auto dot = [&](const float4& av, const float4& bv, float4 xv) {
      if (p.bf16_in) xv = make_float4(round_bf16(xv.x), round_bf16(xv.y), round_bf16(xv.z), round_bf16(xv.w));
      sa += (double)__fmul_rn(av.x, xv.x) + (double)__fmul_rn(av.y, xv.y) + (double)__fmul_rn(av.z, xv.z) +
            (double)__fmul_rn(av.w, xv.w);
      sb += (double)__fmul_rn(bv.x, xv.x) + (double)__fmul_rn(bv.y, xv.y) + (double)__fmul_rn(bv.z, xv.z) +
            (double)__fmul_rn(bv.w, xv.w);
    };
#pragma unroll
    for (int u = 0; u < kPre; ++u) {
      const int i = tid + u * blockDim.x;
      if (i < n4) dot(ap[u], bp[u], x4[i]);
    }
#pragma unroll 4
    for (int i = tid + kPre * blockDim.x; i < n4; i += blockDim.x) dot(a4[i], b4[i], x4[i]);
  }
  block_sum2(sa, sb, red[0]);
  const float bt = sigmoidf_((float)sb);
  const float decay = expf(__fmul_rn(softplus(__fadd_rn((float)sa, p.dt[h])), p.a[h]));
  // conv + silu of the head's channels
  const int pos = *p.pos, nch = 2 * p.DK + p.DV;
  for (int idx = tid; idx < nch; idx += blockDim.x) {
    const int c = idx < p.DK ? kh * p.DK + idx
                             : idx < 2 * p.DK ? p.QK + kh * p.DK + (idx - p.DK) : 2 * p.QK + h * p.DV + (idx - 2 * p.DK);
    float sum = 0.f;
    for (int i = 0; i < p.K - 1; ++i) {
      const int slot = ((pos - (p.K - 1) + i) % p.K + p.K) % p.K;
      sum = __fadd_rn(sum, __fmul_rn(p.ring[(int64_t)slot * p.C + c], p.conv_w[(int64_t)c * p.K + i]));
    }
    const float xin = p.qkv[c];
    sum = __fadd_rn(sum, __fmul_rn(xin, p.conv_w[(int64_t)c * p.K + p.K - 1]));
    p.ring[(int64_t)(pos % p.K) * p.C + c] = xin;
    sm[idx] = silu(sum);  // q | k | v
  }
  __syncthreads();
  // bd::l2norm (cpu_ops.cpp:124-129) of q and k: x / max(sqrt(sum x^2), eps), sum in double
  double sq = 0.0, sk = 0.0;
  for (int i = tid; i < p.DK; i += blockDim.x) {
    sq += (double)q[i] * q[i];
    sk += (double)k[i] * k[i];
  }
  block_sum2(sq, sk, red[1]);
  // the l2-normalised q and k (x * (1 / max(norm, eps)), rounded as the
  // emulator's stored values) are formed where they are read below
  const float iq = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn((float)sq), p.eps));
  const float ik = __fdiv_rn(1.0f, fmaxf(__fsqrt_rn((float)sk), p.eps));
  const float qscale = __fdiv_rn(1.0f, __fsqrt_rn((float)p.DK));
  const float4* k4 = reinterpret_cast<const float4*>(k) + part;
  const float4* q4 = reinterpret_cast<const float4*>(q) + part;
  const float vj = vv[j];
  float kv = 0.f;
  auto nrm = [](float4 x, float s) {
    return make_float4(__fmul_rn(x.x, s), __fmul_rn(x.y, s), __fmul_rn(x.z, s), __fmul_rn(x.w, s));
  };
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    if (t < nt) {
      const float4 c = st[t], kk = nrm(k4[t * kTpc], ik);
      st[t] = make_float4(__fmul_rn(c.x, decay), __fmul_rn(c.y, decay), __fmul_rn(c.z, decay), __fmul_rn(c.w, decay));
      kv = __fadd_rn(kv, __fmul_rn(st[t].x, kk.x));
      kv = __fadd_rn(kv, __fmul_rn(st[t].y, kk.y));
      kv = __fadd_rn(kv, __fmul_rn(st[t].z, kk.z));
      kv = __fadd_rn(kv, __fmul_rn(st[t].w, kk.w));
    }
  }
#pragma unroll
  for (int off = 1; off < kTpc; off <<= 1) kv += __shfl_xor_sync(0xffffffffu, kv, off);
  const float dl = __fmul_rn(__fsub_rn(vj, kv), bt);
  float acc = 0.f;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    if (t < nt) {
      const float4 kk = nrm(k4[t * kTpc], ik), qq = nrm(q4[t * kTpc], iq);
      float4 c = st[t];
      c.x = __fadd_rn(c.x, __fmul_rn(kk.x, dl));
      c.y = __fadd_rn(c.y, __fmul_rn(kk.y, dl));
      c.z = __fadd_rn(c.z, __fmul_rn(kk.z, dl));
      c.w = __fadd_rn(c.w, __fmul_rn(kk.w, dl));
      col[t * kTpc] = c;
      acc = __fadd_rn(acc, __fmul_rn(c.x, qq.x));
      acc = __fadd_rn(acc, __fmul_rn(c.y, qq.y));
      acc = __fadd_rn(acc, __fmul_rn(c.z, qq.z));
      acc = __fadd_rn(acc, __fmul_rn(c.w, qq.w));
    }
  }
#pragma unroll
  for (int off = 1; off < kTpc; off <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (part == 0) ov[j] = __fmul_rn(acc, qscale);
  __syncthreads();
  // bd::rmsnorm over the head's DV outputs with ssm_norm, then * silu(z)
  double ss = 0.0, unused = 0.0;
  for (int i = tid; i < p.DV; i += blockDim.x) ss += (double)ov[i] * ov[i];
  block_sum2(ss, unused, red[0]);
  const float sc = rms_scale(ss, p.DV, p.eps);
  for (int i = tid; i < p.DV; i += blockDim.x) {
    const bool first = i == tid;
    const float y = __fmul_rn(__fmul_rn(ov[i], sc), first ? nw0 : p.norm_w[i]);
    p.o[(int64_t)h * p.DV + i] = __fmul_rn(y, silu(first ? z0 : p.z[(int64_t)h * p.DV + i]));
  }
}

constexpr int kAttnWarps = 4;  // fewest warps of an attention CTA

// ------------------------------------------------------------------ attention, one launch
// The step's attention of one layer in one launch. Grid (H, splits), T
// threads (T >= D, a multiple of 32). CTA (h, sp):
//   - q of head h: RMSNorm with q_norm, then RoPE on the first R dims at
//     position *pos (theta_0 = pos, theta_{i+1} = theta_i * base^(-2/R) in
//     float, as the emulator; pairs (i, i + R/2)), rounded to fp16 when
//     round_q, into shared memory;
//   - the CTA whose key range holds *pos also forms k (the same with k_norm)
//     and v of kv-head g, rounded to fp16, writes them to cache row *pos and
//     takes key *pos from shared memory (the CTAs of the kv-head's other q-heads
//     write the same values; no CTA reads that cache row from global memory);
//   - split sp covers keys [sp * chunk, min((sp + 1) * chunk, pos + 1)); warp w
//     walks every (T/32)-th key: a lane-sliced dot q.k (D/32 dims per lane),
//     then an online softmax with its running max / sum and V accumulator; the
//     warps are merged into part[h][sp] = (max, sum, acc[D]);
//   - the last CTA of head h to finish (a per-head counter; the writers fence
//     before they count) combines the splits,
//     o = (sum_s acc_s e^{m_s - M}) / (sum_s l_s e^{m_s - M}) * sigmoid(gate),
//     and resets the counter for the next launch.
struct AttnParams {
  const float *qf, *kin, *vin, *qn, *kn;
  int H, HK, D, R;
  float theta_scale, eps, scale;
  const int32_t* pos;
  int round_q, chunk;
  __half *kc, *vc;
  float* part;
  int* cnt;
  float* o;
};

// out[i] = rope(rmsnorm(x) * w)[i] for i < D (RoPE on the first R dims at
// position pos, pairs (i, i + R/2)); hv: D floats of scratch. Ends with a barrier.
__device__ void attn_norm_rope(const float* __restrict__ x, const float* __restrict__ w, int D, int R, float eps,
                               float theta_scale, int pos, float* hv, float* out, double* red) {
  const int i = threadIdx.x;
  const float xv = i < D ? x[i] : 0.f;
  const double ss = block_sum(i < D ? (double)xv * xv : 0.0, red);
  const float sc = rms_scale(ss, D, eps);
  if (i < D) hv[i] = __fmul_rn(__fmul_rn(xv, sc), w[i]);
  __syncthreads();
  if (i < D) {
    float outv = hv[i];
    if (i < R) {
      const int ic = i < R / 2 ? i : i - R / 2;
      float theta = (float)pos;
      for (int t = 0; t < ic; ++t) theta = __fmul_rn(theta, theta_scale);
      const float c = cosf(theta), s = sinf(theta);
      const float x0 = hv[ic], x1 = hv[ic + R / 2];
      outv = i < R / 2 ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s)) : __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
    out[i] = outv;
  }
  __syncthreads();
}

__global__ void attn_fused_kernel(const __grid_constant__ AttnParams p) {
  extern __shared__ float sm[];  // q[D], k[D], v[D], scratch[D], per warp: m, l, acc[D]
  __shared__ double red[32];
  __shared__ int is_last;
  pdl_launch_dependents();
  pdl_wait();
  const int D = p.D, h = blockIdx.x, sp = blockIdx.y, tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  const int nw = blockDim.x >> 5;
  const int g = h / (p.H / p.HK), pos = *p.pos, T = pos + 1;
  const int t0 = sp * p.chunk, t1 = min(t0 + p.chunk, T);
  const bool mine = t0 <= pos && pos < t1;  // this split holds the new key (CTA-uniform)
  float* qs = sm;
  float* ks = sm + D;
  float* vs = sm + 2 * D;
  float* hv = sm + 3 * D;
  attn_norm_rope(p.qf + (int64_t)h * 2 * D, p.qn, D, p.R, p.eps, p.theta_scale, pos, hv, qs, red);
  if (p.round_q && tid < D) qs[tid] = __half2float(__float2half_rn(qs[tid]));
  const int64_t kvw = (int64_t)p.HK * D;
  if (mine) {
    attn_norm_rope(p.kin + (int64_t)g * D, p.kn, D, p.R, p.eps, p.theta_scale, pos, hv, ks, red);
    if (tid < D) {
      const __half kh = __float2half_rn(ks[tid]), vh = __float2half_rn(p.vin[(int64_t)g * D + tid]);
      ks[tid] = __half2float(kh);
      vs[tid] = __half2float(vh);
      p.kc[(int64_t)pos * kvw + (int64_t)g * D + tid] = kh;
      p.vc[(int64_t)pos * kvw + (int64_t)g * D + tid] = vh;
    }
  }
  __syncthreads();
  // the key range: online softmax per warp
  float* wm = sm + 4 * D + wp * (D + 2);
  const int per = D / 32;
  float m = -INFINITY, l = 0.f;
  float acc[8];  // D <= 256
#pragma unroll
  for (int r = 0; r < 8; ++r) acc[r] = 0.f;
  for (int t = t0 + wp; t < t1; t += nw) {
    const bool fresh = t == pos;  // the new key, from shared memory
    const __half* kt = p.kc + (int64_t)t * kvw + (int64_t)g * D;
    float dd = 0.f;
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (r < per)
        dd = fmaf(qs[lane * per + r], fresh ? ks[lane * per + r] : __half2float(kt[lane * per + r]), dd);
#pragma unroll
    for (int o = 16; o; o >>= 1) dd += __shfl_xor_sync(0xffffffffu, dd, o);
    const float sc = dd * p.scale;
    const float mn = fmaxf(m, sc);
    const float cf = expf(m - mn), pf = expf(sc - mn);
    l = l * cf + pf;
    const __half* vt = p.vc + (int64_t)t * kvw + (int64_t)g * D;
#pragma unroll
    for (int r = 0; r < 8; ++r)
      if (r < per) acc[r] = fmaf(pf, fresh ? vs[lane * per + r] : __half2float(vt[lane * per + r]), acc[r] * cf);
    m = mn;
  }
  if (lane == 0) {
    wm[0] = m;
    wm[1] = l;
  }
#pragma unroll
  for (int r = 0; r < 8; ++r)
    if (r < per) wm[2 + lane * per + r] = acc[r];
  __syncthreads();
  // merge the warps into this split's partial
  float* out = p.part + ((int64_t)h * gridDim.y + sp) * (D + 2);
  {
    float M = -INFINITY;
    for (int w = 0; w < nw; ++w) M = fmaxf(M, sm[4 * D + w * (D + 2)]);
    for (int i = tid; i < D + 2; i += blockDim.x) {
      float v = 0.f;
      for (int w = 0; w < nw; ++w) {
        const float* ww = sm + 4 * D + w * (D + 2);
        const float f = ww[0] == -INFINITY ? 0.f : expf(ww[0] - M);
        if (i == 1) v += ww[1] * f;
        else if (i >= 2) v += ww[i] * f;
      }
      out[i] = i == 0 ? M : v;
    }
  }
  // the last CTA of head h combines the splits
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = atomicAdd(p.cnt + h, 1) == (int)gridDim.y - 1;
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const int splits = gridDim.y;
  const float* ph = p.part + (int64_t)h * splits * (D + 2);  // other CTAs' writes: read past L1 (__ldcg)
  float M = -INFINITY;
  for (int s2 = 0; s2 < splits; ++s2) M = fmaxf(M, __ldcg(ph + (int64_t)s2 * (D + 2)));
  float L = 0.f;
  for (int s2 = 0; s2 < splits; ++s2) {
    const float ms = __ldcg(ph + (int64_t)s2 * (D + 2));
    if (ms != -INFINITY) L += __ldcg(ph + (int64_t)s2 * (D + 2) + 1) * expf(ms - M);
  }
  for (int i = tid; i < D; i += blockDim.x) {
    float a = 0.f;
    for (int s2 = 0; s2 < splits; ++s2) {
      const float ms = __ldcg(ph + (int64_t)s2 * (D + 2));
      if (ms != -INFINITY) a += __ldcg(ph + (int64_t)s2 * (D + 2) + 2 + i) * expf(ms - M);
    }
    const float gate = p.qf[(int64_t)h * 2 * D + D + i];
    p.o[(int64_t)h * D + i] = a / L * sigmoidf_(gate);
  }
  if (tid == 0) p.cnt[h] = 0;
}

// ------------------------------------------------------------------ argmax
// Stage 1: CTA b takes a contiguous range; (value, index) with the lowest
// index among equal maxima. NaN counts as -inf (the emulator's
// `lg[i] > lg[best]` never picks a NaN), so all-NaN logits give index 0.
__device__ __forceinline__ void better(float& v, int& i, float v2, int i2) {
  if (i2 < 0) return;
  if (v2 != v2) v2 = -INFINITY;
  if (i < 0 || v2 > v || (v2 == v && i2 < i)) {
    v = v2;
    i = i2;
  }
}
__global__ void argmax1_kernel(const float* __restrict__ x, int n, float* __restrict__ pv, int* __restrict__ pi) {
  __shared__ float sv[32];
  __shared__ int si[32];
  pdl_launch_dependents();
  pdl_wait();
  const int per = (n + gridDim.x - 1) / gridDim.x, b0 = blockIdx.x * per, b1 = min(n, b0 + per);
  float v = -INFINITY;
  int idx = -1;
  for (int i = b0 + threadIdx.x; i < b1; i += blockDim.x) better(v, idx, x[i], i);
#pragma unroll
  for (int o = 16; o; o >>= 1) better(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
  if ((threadIdx.x & 31) == 0) {
    sv[threadIdx.x >> 5] = v;
    si[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) better(v, idx, sv[w], si[w]);
    pv[blockIdx.x] = v;
    pi[blockIdx.x] = idx;
  }
}
// Stage 2: one warp; writes the token, and the next step's input token and
// position (pos += 1) when those pointers are given.
__global__ void argmax2_kernel(const float* __restrict__ pv, const int* __restrict__ pi, int parts,
                               int32_t* __restrict__ out, int32_t* __restrict__ tok_next, int32_t* __restrict__ pos) {
  pdl_launch_dependents();
  pdl_wait();
  float v = -INFINITY;
  int idx = -1;
  for (int i = threadIdx.x; i < parts; i += 32) better(v, idx, pv[i], pi[i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) better(v, idx, __shfl_xor_sync(0xffffffffu, v, o), __shfl_xor_sync(0xffffffffu, idx, o));
  if (threadIdx.x == 0) {
    const int t = idx < 0 ? 0 : idx;
    *out = t;
    if (tok_next) *tok_next = t;
    if (pos) *pos += 1;
  }
}

// Fills a panel buffer with seeded valid codes (0..2) and fp16 scales
// |N(0,1)| * scale_mul; padding rows / columns get code 1 and scale 0.
__device__ __forceinline__ uint32_t mix32(uint64_t x) {
  x ^= x >> 33;
  x *= 0xff51afd7ed558ccdull;
  x ^= x >> 33;
  x *= 0xc4ceb9fe1a85ec53ull;
  x ^= x >> 33;
  return (uint32_t)x;
}
// Row groups g0 .. of the full matrix: every value depends on its global
// position only, so a row shard holds exactly the rows of the full matrix.
__global__ void fill_panels_kernel(uint8_t* __restrict__ pan, int64_t npanels, int g0, int N, int K, int S,
                                   uint64_t seed, float scale_mul) {
  const int64_t nb = npanels * kPanelBytes;
  for (int64_t bl = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; bl < nb; bl += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = bl + (int64_t)g0 * S * kPanelBytes;  // global byte index
    const int64_t pidx = b / kPanelBytes;
    const int off = (int)(b % kPanelBytes);
    const int g = (int)(pidx / S), j = (int)(pidx % S);
    if (off < kCodeBytes) {
      // byte: 4 rows (bit pairs) of one column
      const int h = off >> 10, c = j * 1024 + ((off >> 4) & 31) / 4 * 128 + ((off >> 4) & 3) * 32 +
                                   ((off >> 9) & 1) * 16 + ((off >> 2) & 3) * 4 + (off & 3);
      uint32_t rnd = mix32(seed * 0x9e3779b97f4a7c15ull + (uint64_t)b);
      uint8_t byte = 0;
      for (int k = 0; k < 4; ++k) {
        const int row = g * 8 + h * 4 + k;
        int code = 1;
        if (row < N && c < K) {
          code = (int)((rnd & 0xffff) % 3u);
          rnd >>= 8;
          rnd ^= mix32((uint64_t)b * 4 + k + seed);
        }
        byte |= (uint8_t)(code << (2 * k));
      }
      pan[bl] = byte;
    } else {
      const int so = off - kCodeBytes, bb = so >> 4, rr = (so >> 1) & 7;
      const int row = g * 8 + rr, col = j * 1024 + bb * 128;
      if (so & 1) continue;  // the even byte writes both bytes of the fp16
      float v = 0.f;
      if (row < N && col < K) {
        const uint32_t a = mix32(seed ^ (0xabcdef12ull + (uint64_t)b)), c2 = mix32(seed + 77 + (uint64_t)b * 3);
        const float u1 = ((a >> 8) + 1) * (1.0f / 16777217.0f), u2 = (c2 >> 8) * (1.0f / 16777216.0f);
        v = fabsf(sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2)) * scale_mul;
      }
      const uint16_t hb = __half_as_ushort(__float2half_rn(v));
      pan[bl] = (uint8_t)(hb & 0xff);
      pan[bl + 1] = (uint8_t)(hb >> 8);
    }
  }
}

// Seeded floats: base + uniform(-spread, spread).
__global__ void fill_uniform_kernel(float* __restrict__ x, int64_t n, uint64_t seed, float base, float spread) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t a = mix32(seed * 0x9e3779b97f4a7c15ull + (uint64_t)i);
    x[i] = base + spread * (2.0f * ((a >> 8) * (1.0f / 16777216.0f)) - 1.0f);
  }
}

}  // namespace

// ------------------------------------------------------------------ launchers
cudaError_t launch_embed(const uint8_t* pan, int V, int E, const int32_t* tok, int blk, const float* signs, float* x,
                         cudaStream_t st) {
  const int n = blk ? blk : 256;
  return launch_pdl(embed_kernel, dim3((E + n - 1) / n), dim3(n), blk ? (blk + blk / 32) * sizeof(float) : 0, st,
                    pan, V, E,
                    (int)slices_of(E), tok, blk, signs, x);
}
cudaError_t launch_gdn_mix(const GdnArgs& g, cudaStream_t st) {
  const GdnParams p{g.xn, g.aw, g.bw, g.dt, g.a, g.E, g.bf16_in, g.qkv, g.ring, g.conv_w, g.K, g.C, g.z, g.state,
                    g.norm_w, g.NK, g.DK, g.DV, g.QK, g.eps, g.pos, g.o};
  return launch_pdl(gdn_mix_kernel, dim3(g.NV), dim3(g.DV * kTpc), (size_t)(2 * g.DK + 2 * g.DV) * sizeof(float), st,
                    p);
}
cudaError_t launch_attention_fused(const float* qf, const float* k, const float* v, const float* qn, const float* kn,
                                   int H, int HK, int D, int R, float theta_scale, float eps, const int32_t* pos,
                                   int round_q, void* kc, void* vc, int n_ctx, int splits, float* part, int* cnt,
                                   float* o, cudaStream_t st) {
  const int threads = (D + 31) / 32 * 32 > kAttnWarps * 32 ? (D + 31) / 32 * 32 : kAttnWarps * 32;
  AttnParams p{qf, k, v, qn, kn, H, HK, D, R, theta_scale, eps, 1.0f / sqrtf((float)D), pos, round_q,
               (n_ctx + splits - 1) / splits, static_cast<__half*>(kc), static_cast<__half*>(vc), part, cnt, o};
  const size_t smem = (size_t)(4 * D + (threads / 32) * (D + 2)) * sizeof(float);
  return launch_pdl(attn_fused_kernel, dim3(H, splits), dim3(threads), smem, st, p);
}
cudaError_t launch_argmax(const float* x, int n, float* pv, int* pi, int parts, int32_t* out, int32_t* tok_next,
                          int32_t* pos, cudaStream_t st) {
  if (cudaError_t e = launch_pdl(argmax1_kernel, dim3(parts), dim3(256), 0, st, x, n, pv, pi)) return e;
  return launch_pdl(argmax2_kernel, dim3(1), dim3(32), 0, st, static_cast<const float*>(pv),
                    static_cast<const int*>(pi), parts, out, tok_next, pos);
}
cudaError_t launch_fill_panels(uint8_t* pan, int row0, int rows, int N, int K, uint64_t seed, float scale_mul,
                               cudaStream_t st) {
  const int64_t np = groups_of(rows) * slices_of(K);
  fill_panels_kernel<<<1184, 256, 0, st>>>(pan, np, row0 / kRows, N, K, (int)slices_of(K), seed, scale_mul);
  return cudaGetLastError();
}
cudaError_t launch_fill_uniform(float* x, int64_t n, uint64_t seed, float base, float spread, cudaStream_t st) {
  fill_uniform_kernel<<<592, 256, 0, st>>>(x, n, seed, base, spread);
  return cudaGetLastError();
}

}  // namespace btf
