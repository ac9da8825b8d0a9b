// Q8_0 activation quantiser, bit-exact to the reference's host rule
// q8_block_host (include/btf/packed.hpp:117-134): per 32-column block
//   amax = max |x|, d = fp16_rne(amax / 127) kept as fp32,
//   id = amax != 0 ? 127 / amax : 0, q = round_half_even(x * id), s = sum(q).
// IEEE division and multiplication only (no fast-math), as in the quantising
// tail of the reference's prep_kernel (src/cuda/kernels.cu:185-201).
#include <algorithm>

#include "common.cuh"

namespace btf {
namespace {

constexpr int kQThreads = 256;

// One thread per 4 consecutive values, 8 lanes per 32-block (q8_quad).
__global__ void __launch_bounds__(kQThreads)
    quant_q8_kernel(const float* __restrict__ x, int ldx, int K, int8_t* __restrict__ q, float* __restrict__ d,
                    int32_t* __restrict__ s, unsigned long long* stamp) {
  const int nquad = K / 4;
  const int qi = blockIdx.x * kQThreads + threadIdx.x;
  const int m = blockIdx.y;
  pdl_launch_dependents();
  pdl_wait();
  if (blockIdx.x * kQThreads >= nquad) return;  // whole block beyond the row (CTA-uniform)
  const bool vec = ((reinterpret_cast<uintptr_t>(x) | ((uintptr_t)ldx * 4)) & 15) == 0;
  const bool ok = qi < nquad;  // K % 32 == 0: a 32-block is all in or all out
  const float4 v = ok ? load4(x + (size_t)m * ldx + qi * 4, vec) : make_float4(0.f, 0.f, 0.f, 0.f);
  float dq;
  int sum;
  const uint32_t q4 = q8_quad(v, dq, sum);
  if (ok) {
    *reinterpret_cast<uint32_t*>(q + (size_t)m * K + qi * 4) = q4;
    if ((qi & 7) == 0) {
      d[(size_t)m * (K / 32) + (qi >> 3)] = dq;
      s[(size_t)m * (K / 32) + (qi >> 3)] = sum;
    }
  }
  stamp_end(stamp);
}

// ---------------------------------------------------------------- fused prep
// RMSNorm -> permutation -> signs -> blockwise Walsh-Hadamard -> Q8_0, the
// reference's launch_prep (src/cuda/kernels.cu:147-202, :745-774). Host forms:
// bd::rmsnorm / bd::hadamard_input (ref/bonsai-decoder/src/cpu_ops.cpp:90-127)
// and q8_block_host. One CTA per (span of S <= 1024 columns, row); the span is
// the largest power of two <= 1024 dividing n, so Hadamard blocks never cross
// CTAs. Every butterfly computes (a + b, a - b) in the host's stage order, and
// the norm scale and the products are correctly rounded, so only the order of
// the double sum of squares differs from the host.
constexpr int kPrepThreads = 256;      // fewest threads a CTA is launched with
constexpr int kPrepMaxThreads = 1024;  // one thread per column of a 1024-wide span

struct PrepParams {
  const float* x;
  int ldx, n, S;
  const float* normw;
  float eps;
  int block, perm_hd, perm_nk, perm_rep;
  const float* signs;
  float* xn_out;
  int ldxn;
  int8_t* q;
  float* d;
  int32_t* s;
};

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <bool NORM>
__global__ void __launch_bounds__(kPrepMaxThreads, 1) prep_kernel(const __grid_constant__ PrepParams a) {
  extern __shared__ float buf[];  // [S + S / 32]
  __shared__ double red[kPrepMaxThreads / 32];
  const int nthr = blockDim.x, nwarp = nthr >> 5;
  const int m = blockIdx.y, base = blockIdx.x * a.S;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* xr = a.x + (size_t)m * a.ldx;
  // column map of this thread's first span column (the launch gives every
  // column its own thread), and its norm weight and sign: constants, fetched
  // before the wait while the previous kernel drains
  auto src_of = [&](int og) {
    if (a.perm_rep <= 1) return og;
    const int dd = og % a.perm_hd, t = og / a.perm_hd;  // tiled [hd, nk, rep] -> grouped [hd, rep, nk]
    const int r = t % a.perm_rep, k = t / a.perm_rep;
    return dd + a.perm_hd * (k + a.perm_nk * r);
  };
  const int og0 = base + threadIdx.x, src0 = src_of(og0);
  const bool own = threadIdx.x < a.S;
  float w0 = 1.0f, wo0 = 1.0f, sg0 = 1.0f;
  if (own) {
    if constexpr (NORM) {
      w0 = a.normw[src0];
      wo0 = a.normw[og0];
    }
    if (a.signs) sg0 = a.signs[og0];
  }
  pdl_launch_dependents();
  pdl_wait();  // x is written by the previous kernel
  // this thread's first span column (and its own-order column for xn), loaded
  // before the norm pass so that both reads of x are in flight together
  const float x0 = own ? xr[src0] : 0.f;
  const float xo0 = own && a.xn_out ? xr[og0] : 0.f;
  float scale = 1.0f;
  if constexpr (NORM) {
    double acc = 0.0;
    if ((reinterpret_cast<uintptr_t>(xr) & 15) == 0 && (a.n & 3) == 0) {
      // 16-byte loads, several in flight per thread (the row is read with one latency, not n/256)
      const float4* x4 = reinterpret_cast<const float4*>(xr);
#pragma unroll 4
      for (int i = threadIdx.x; i < (a.n >> 2); i += nthr) {
        const float4 v = x4[i];
        acc += (double)v.x * (double)v.x + (double)v.y * (double)v.y + (double)v.z * (double)v.z +
               (double)v.w * (double)v.w;
      }
    } else {
#pragma unroll 4
      for (int i = threadIdx.x; i < a.n; i += nthr) acc += (double)xr[i] * (double)xr[i];
    }
    acc = warp_sum_d(acc);
    if (lane == 0) red[warp] = acc;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < nwarp; ++w) tot += red[w];
    const float mean = (float)(tot / (double)a.n);
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.eps)));
  }
  if (a.S == 1024 && nthr == 1024) {
    // One column per thread (column e = threadIdx.x of the span, warp c holds
    // 32c .. 32c+31): the butterflies of length 1 .. 16 run on registers
    // (shuffles), then one padded transpose through shared memory gives thread
    // (c, l) column 32 l + c, so the lengths 32 .. 512 are shuffles too; the
    // transpose back leaves each warp its own 32-column Q8 block. Same stage
    // order and (a + b, a - b) pairs as below, 2 barriers instead of 7.
    float v = x0;
    if constexpr (NORM) v = __fmul_rn(__fmul_rn(v, scale), w0);
    if (a.signs) v = __fmul_rn(v, sg0);
    const int og = base + (int)threadIdx.x;
    if (a.xn_out) {
      float u = xo0;
      if constexpr (NORM) u = __fmul_rn(__fmul_rn(u, scale), wo0);
      a.xn_out[(size_t)m * a.ldxn + og] = u;
    }
    if (a.block > 1) {
      const int lim = min(a.block, 32);
      for (int len = 1; len < lim; len <<= 1) {
        const float p = __shfl_xor_sync(0xffffffffu, v, len);
        v = (lane & len) ? __fsub_rn(p, v) : __fadd_rn(v, p);
      }
      if (a.block > 32) {
        buf[threadIdx.x + warp] = v;  // column e at e + e / 32: conflict-free both ways
        __syncthreads();
        float t = buf[33 * lane + warp];  // column 32 lane + warp
        for (int k = 1; 32 * k < a.block; k <<= 1) {  // length 32 k
          const float p = __shfl_xor_sync(0xffffffffu, t, k);
          t = (lane & k) ? __fsub_rn(p, t) : __fadd_rn(t, p);
        }
        buf[33 * lane + warp] = t;
        __syncthreads();
        v = buf[threadIdx.x + warp];
      }
      v = __fmul_rn(v, __fdiv_rn(1.0f, __fsqrt_rn((float)a.block)));
    }
    float dq;
    int sum;
    const int qv = q8_warp(v, dq, sum);
    a.q[(size_t)m * a.n + og] = (int8_t)qv;
    if (lane == 0) {
      const size_t bi = (size_t)m * (a.n / 32) + (base / 32 + warp);
      a.d[bi] = dq;
      a.s[bi] = sum;
    }
    return;
  }
  for (int o = threadIdx.x; o < a.S; o += nthr) {
    const bool first = o == (int)threadIdx.x;  // the prefetched column
    const int og = base + o, src = first ? src0 : src_of(og);
    float v = first ? x0 : xr[src];
    if constexpr (NORM) v = __fmul_rn(__fmul_rn(v, scale), first ? w0 : a.normw[src]);
    if (a.signs) v = __fmul_rn(v, first ? sg0 : a.signs[og]);
    buf[o] = v;
    if (a.xn_out) {
      float u = first ? xo0 : xr[og];
      if constexpr (NORM) u = __fmul_rn(__fmul_rn(u, scale), first ? wo0 : a.normw[og]);
      a.xn_out[(size_t)m * a.ldxn + og] = u;
    }
  }
  __syncthreads();
  float hs = 1.0f;
  if (a.block > 1) {
    // stages len = 1 .. 16 inside each warp's 32 consecutive values (shuffles)
    const int lim = min(a.block, 32);
    for (int c = warp; c < a.S / 32; c += nwarp) {
      float v = buf[c * 32 + lane];
      for (int len = 1; len < lim; len <<= 1) {
        const float p = __shfl_xor_sync(0xffffffffu, v, len);
        v = (lane & len) ? __fsub_rn(p, v) : __fadd_rn(v, p);
      }
      buf[c * 32 + lane] = v;
    }
    __syncthreads();
    // stages len = 32 .. block/2 in shared memory
    for (int len = 32; len < a.block; len <<= 1) {
      for (int pidx = threadIdx.x; pidx < (a.S >> 1); pidx += nthr) {
        const int j = (pidx / len) * (len << 1) + (pidx % len);
        const float x0 = buf[j], x1 = buf[j + len];
        buf[j] = __fadd_rn(x0, x1);
        buf[j + len] = __fsub_rn(x0, x1);
      }
      __syncthreads();
    }
    hs = __fdiv_rn(1.0f, __fsqrt_rn((float)a.block));
  }
  for (int g = warp; g < a.S / 32; g += nwarp) {
    float v = buf[g * 32 + lane];
    if (a.block > 1) v = __fmul_rn(v, hs);
    float dq;
    int sum;
    const int qv = q8_warp(v, dq, sum);
    const size_t col = (size_t)base + g * 32 + lane;
    a.q[(size_t)m * a.n + col] = (int8_t)qv;
    if (lane == 0) {
      const size_t bi = (size_t)m * (a.n / 32) + (base / 32 + g);
      a.d[bi] = dq;
      a.s[bi] = sum;
    }
  }
}

int span_of(int n) {
  int s = 1;
  while (s < 1024 && n % (s * 2) == 0) s *= 2;
  return s;
}

}  // namespace
}  // namespace btf

using namespace btf;

extern "C" int btf_prep(const float* x, int ldx, int M, int n, const float* normw, float eps, btf_hx hx,
                        float* xn_out, int ldxn, btf_q8act act, void* stream) {
  if (M <= 0) return BTF_OK;
  if (n <= 0 || n % 32 || ldx < n) return fail(BTF_ERR_ARG, "btf_prep: need n a positive multiple of 32 and ldx >= n");
  if (!x || !act.q || !act.d || !act.s) return fail(BTF_ERR_ARG, "btf_prep: null pointer");
  if (xn_out && ldxn < n) return fail(BTF_ERR_ARG, "btf_prep: ldxn < n");
  if (M > 65535) return fail(BTF_ERR_ARG, "btf_prep: M=%d exceeds 65535", M);
  const int S = span_of(n);
  if (hx.block < 0 || (hx.block > 0 && ((hx.block & (hx.block - 1)) || S % hx.block)))
    return fail(BTF_ERR_ARG, "btf_prep: hadamard block %d must be a power of two dividing the span %d", hx.block, S);
  if (hx.perm_rep > 1 && (hx.perm_hd <= 0 || hx.perm_nk <= 0 || (int64_t)hx.perm_hd * hx.perm_nk * hx.perm_rep != n))
    return fail(BTF_ERR_ARG, "btf_prep: permutation geometry hd*nk*rep must equal n");
  if (!current_device()) return BTF_ERR_STATE;
  PrepParams p{x, ldx, n, S, normw, eps, hx.block, hx.perm_hd, hx.perm_nk, hx.perm_rep, hx.signs, xn_out, ldxn,
               act.q, act.d, act.s};
  const dim3 grid(n / S, M);
  const size_t smem = (size_t)(S + S / 32) * sizeof(float);  // padded for the one-column-per-thread transpose
  const int threads = std::max(kPrepThreads, S);  // S <= 1024: one thread per column of the span
  const cudaError_t e = normw ? launch_pdl(prep_kernel<true>, grid, dim3(threads), smem, (cudaStream_t)stream, p)
                              : launch_pdl(prep_kernel<false>, grid, dim3(threads), smem, (cudaStream_t)stream, p);
  return e == cudaSuccess ? launch_status("prep_kernel") : cuda_fail(e, "prep_kernel launch");
}

extern "C" int btf_quant_q8(const float* x, int ldx, int M, int K, btf_q8act act, void* stream) {
  if (M <= 0) return BTF_OK;
  if (K <= 0 || K % 32 || ldx < K)
    return fail(BTF_ERR_ARG, "btf_quant_q8: need K a positive multiple of 32 and ldx >= K (K=%d ldx=%d)", K, ldx);
  if (!x || !act.q || !act.d || !act.s) return fail(BTF_ERR_ARG, "btf_quant_q8: null pointer");
  if (!current_device()) return BTF_ERR_STATE;
  if (((uintptr_t)act.q & 3) != 0) return fail(BTF_ERR_ARG, "btf_quant_q8: q must be 4-byte aligned");
  const dim3 grid((K / 4 + kQThreads - 1) / kQThreads, M);
  if (grid.y > 65535) return fail(BTF_ERR_ARG, "btf_quant_q8: M=%d exceeds 65535", M);
  const cudaError_t e = launch_pdl(quant_q8_kernel, grid, dim3(kQThreads), 0, (cudaStream_t)stream, x, ldx, K,
                                   act.q, act.d, act.s, take_stamp());
  return e == cudaSuccess ? launch_status("quant_q8_kernel") : cuda_fail(e, "quant_q8_kernel launch");
}
