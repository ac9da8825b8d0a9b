// Q8_0 activation quantiser, bit-exact to the reference's host rule
// q8_block_host (include/btf/packed.hpp:117-134): per 32-column block
//   amax = max |x|, d = fp16_rne(amax / 127) kept as fp32,
//   id = amax != 0 ? 127 / amax : 0, q = round_half_even(x * id), s = sum(q).
// IEEE division and multiplication only (no fast-math), as in the quantising
// tail of the reference's prep_kernel (src/cuda/kernels.cu:185-201).
#include "common.cuh"

namespace btf {
namespace {

constexpr int kQThreads = 256;

// One thread per 4 consecutive values, 8 lanes per 32-block (q8_quad).
__global__ void __launch_bounds__(kQThreads)
    quant_q8_kernel(const float* __restrict__ x, int ldx, int K, int8_t* __restrict__ q, float* __restrict__ d,
                    int32_t* __restrict__ s) {
  const int nquad = K / 4;
  const int qi = blockIdx.x * kQThreads + threadIdx.x;
  const int m = blockIdx.y;
  pdl_launch_dependents();
  pdl_wait();
  if (blockIdx.x * kQThreads >= nquad) return;  // whole block beyond the row (warp-uniform)
  const bool vec = ((reinterpret_cast<uintptr_t>(x) | ((uintptr_t)ldx * 4)) & 15) == 0;
  const bool ok = qi < nquad;  // K % 32 == 0: a 32-block is all in or all out
  const float4 v = ok ? load4(x + (size_t)m * ldx + qi * 4, vec) : make_float4(0.f, 0.f, 0.f, 0.f);
  float dq;
  int sum;
  const uint32_t q4 = q8_quad(v, dq, sum);
  if (!ok) return;
  *reinterpret_cast<uint32_t*>(q + (size_t)m * K + qi * 4) = q4;
  if ((qi & 7) == 0) {
    d[(size_t)m * (K / 32) + (qi >> 3)] = dq;
    s[(size_t)m * (K / 32) + (qi >> 3)] = sum;
  }
}

}  // namespace
}  // namespace btf

using namespace btf;

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
                                   act.q, act.d, act.s);
  return e == cudaSuccess ? launch_status("quant_q8_kernel") : cuda_fail(e, "quant_q8_kernel launch");
}
