// Load-time repack kernels: PTQ1_0 -> panel layout (the B200 resident form),
// PTQ1_0 -> T2 (the reference's resident form), and T2 <-> panels.
//
// Replaces repack_kernel / launch_repack (src/cuda/kernels.cu:110-128, :737-743
// of the reference). One thread per 128-column block; a 28-byte source block is
// read as seven 32-bit words (the source may be mapped host memory, as in the
// reference's staged upload, src/cuda/gpu_decoder.cu:284-300).
#include <algorithm>

#include "common.cuh"
#include "layout.h"

namespace btf {
namespace {

constexpr int kThreads = 256;

struct Src7 {
  uint32_t v[7];
  __device__ __forceinline__ uint32_t operator()(int i) const { return (v[i >> 2] >> (8 * (i & 3))) & 0xffu; }
};

__device__ __forceinline__ void load_block(const uint8_t* src, int64_t blk, Src7& s, uint16_t& scale) {
  const uint32_t* p = reinterpret_cast<const uint32_t*>(src + blk * 28);
#pragma unroll
  for (int i = 0; i < 7; ++i) s.v[i] = p[i];
  scale = (uint16_t)(s.v[6] >> 16);
}

// Grid covers the padded domain: G*2 row quads x S*8 blocks, one thread each;
// rows >= N and blocks >= K/128 are written as padding (code 1, scale 0).
__global__ void __launch_bounds__(kThreads)
    repack_panels_kernel(const uint8_t* __restrict__ src, int64_t N, int64_t K, uint8_t* __restrict__ panels) {
  const int64_t nbk = K / 128, S = slices_of(K), bpr = S * kBlocksPerSlice;
  const int64_t total = groups_of(N) * 2 * bpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t qd = i / bpr, b = i - qd * bpr;
    uint32_t tw[4][8];
    uint16_t sc[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t n = qd * 4 + k;
      sc[k] = 0;
      if (n < N && b < nbk) {
        Src7 s;
        load_block(src, n * nbk + b, s, sc[k]);
        ptq_block_to_t2(s, tw[k]);
      } else {
#pragma unroll
        for (int w = 0; w < 8; ++w) tw[k][w] = kPadWord;
      }
    }
    store_quad_block(panels + panel_offset(qd / 2, b / kBlocksPerSlice, S), (int)(qd % 2), (int)(b % kBlocksPerSlice),
                     tw, sc);
  }
}

__global__ void __launch_bounds__(kThreads)
    repack_t2_kernel(const uint8_t* __restrict__ src, int64_t nblocks, uint4* __restrict__ codes,
                     uint16_t* __restrict__ scales) {
  for (int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; b < nblocks; b += (int64_t)gridDim.x * blockDim.x) {
    Src7 s;
    uint16_t scale;
    load_block(src, b, s, scale);
    uint32_t w[8];
    ptq_block_to_t2(s, w);
    codes[2 * b] = make_uint4(w[0], w[1], w[2], w[3]);
    codes[2 * b + 1] = make_uint4(w[4], w[5], w[6], w[7]);
    scales[b] = scale;
  }
}

__global__ void __launch_bounds__(kThreads)
    t2_to_panels_kernel(const uint8_t* __restrict__ codes, const uint16_t* __restrict__ scales, int64_t N, int64_t K,
                        uint8_t* __restrict__ panels) {
  const int64_t nbk = K / 128, S = slices_of(K), bpr = S * kBlocksPerSlice;
  const int64_t total = groups_of(N) * 2 * bpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t qd = i / bpr, b = i - qd * bpr;
    uint32_t tw[4][8];
    uint16_t sc[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t n = qd * 4 + k;
      sc[k] = 0;
      if (n < N && b < nbk) {
        const uint4* sp = reinterpret_cast<const uint4*>(codes + (n * nbk + b) * 32);
        const uint4 c0 = sp[0], c1 = sp[1];
        tw[k][0] = c0.x; tw[k][1] = c0.y; tw[k][2] = c0.z; tw[k][3] = c0.w;
        tw[k][4] = c1.x; tw[k][5] = c1.y; tw[k][6] = c1.z; tw[k][7] = c1.w;
        sc[k] = scales[n * nbk + b];
      } else {
#pragma unroll
        for (int w = 0; w < 8; ++w) tw[k][w] = kPadWord;
      }
    }
    store_quad_block(panels + panel_offset(qd / 2, b / kBlocksPerSlice, S), (int)(qd % 2), (int)(b % kBlocksPerSlice),
                     tw, sc);
  }
}

__global__ void __launch_bounds__(kThreads)
    panels_to_t2_kernel(const uint8_t* __restrict__ panels, int64_t N, int64_t K, uint8_t* __restrict__ codes,
                        uint16_t* __restrict__ scales) {
  const int64_t nbk = K / 128, S = slices_of(K);
  const int64_t nquad = (N + 3) / 4;
  const int64_t total = nquad * nbk;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t qd = i / nbk, b = i - qd * nbk;
    uint32_t tw[4][8];
    uint16_t sc[4];
    load_quad_block(panels + panel_offset(qd / 2, b / kBlocksPerSlice, S), (int)(qd % 2), (int)(b % kBlocksPerSlice),
                    tw, sc);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t n = qd * 4 + k;
      if (n >= N) break;
      uint4* dst = reinterpret_cast<uint4*>(codes + (n * nbk + b) * 32);
      dst[0] = make_uint4(tw[k][0], tw[k][1], tw[k][2], tw[k][3]);
      dst[1] = make_uint4(tw[k][4], tw[k][5], tw[k][6], tw[k][7]);
      scales[n * nbk + b] = sc[k];
    }
  }
}

int grid_for(int64_t work) {
  const DeviceInfo* d = current_device();
  const int64_t cap = d ? (int64_t)d->sm_count * 32 : 4096;
  return (int)std::max<int64_t>(1, std::min<int64_t>((work + kThreads - 1) / kThreads, cap));
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int check_nk(const char* fn, int64_t N, int64_t K) {
  if (N <= 0 || K <= 0 || K % 128) return fail(BTF_ERR_ARG, "%s: need N > 0 and K a positive multiple of 128 (N=%lld K=%lld)", fn, (long long)N, (long long)K);
  return BTF_OK;
}

}  // namespace
}  // namespace btf

using namespace btf;

extern "C" {

int btf_repack_panels(const void* ptq_src, int64_t N, int64_t K, void* panels, void* stream) {
  if (int st = check_nk("btf_repack_panels", N, K)) return st;
  if (!ptq_src || !panels || !aligned(ptq_src, 4) || !aligned(panels, 16))
    return fail(BTF_ERR_ARG, "btf_repack_panels: null or misaligned pointer (src needs 4 B, panels 16 B)");
  if (!current_device()) return BTF_ERR_STATE;
  const int64_t total = groups_of(N) * 2 * slices_of(K) * kBlocksPerSlice;
  repack_panels_kernel<<<grid_for(total), kThreads, 0, (cudaStream_t)stream>>>(
      static_cast<const uint8_t*>(ptq_src), N, K, static_cast<uint8_t*>(panels));
  return launch_status("repack_panels_kernel");
}

int btf_repack_t2(const void* ptq_src, int64_t nblocks, uint8_t* codes, uint16_t* scales, void* stream) {
  if (nblocks <= 0) return BTF_OK;  // like the reference launcher, nothing to do
  if (!ptq_src || !codes || !scales || !aligned(ptq_src, 4) || !aligned(codes, 16) || !aligned(scales, 2))
    return fail(BTF_ERR_ARG, "btf_repack_t2: null or misaligned pointer");
  if (!current_device()) return BTF_ERR_STATE;
  repack_t2_kernel<<<grid_for(nblocks), kThreads, 0, (cudaStream_t)stream>>>(
      static_cast<const uint8_t*>(ptq_src), nblocks, reinterpret_cast<uint4*>(codes), scales);
  return launch_status("repack_t2_kernel");
}

int btf_t2_to_panels(const uint8_t* codes, const uint16_t* scales, int64_t N, int64_t K, void* panels,
                     void* stream) {
  if (int st = check_nk("btf_t2_to_panels", N, K)) return st;
  if (!codes || !scales || !panels || !aligned(codes, 16) || !aligned(scales, 2) || !aligned(panels, 16))
    return fail(BTF_ERR_ARG, "btf_t2_to_panels: null or misaligned pointer");
  if (!current_device()) return BTF_ERR_STATE;
  const int64_t total = groups_of(N) * 2 * slices_of(K) * kBlocksPerSlice;
  t2_to_panels_kernel<<<grid_for(total), kThreads, 0, (cudaStream_t)stream>>>(codes, scales, N, K,
                                                                             static_cast<uint8_t*>(panels));
  return launch_status("t2_to_panels_kernel");
}

int btf_panels_to_t2(const void* panels, int64_t N, int64_t K, uint8_t* codes, uint16_t* scales, void* stream) {
  if (int st = check_nk("btf_panels_to_t2", N, K)) return st;
  if (!codes || !scales || !panels || !aligned(codes, 16) || !aligned(scales, 2) || !aligned(panels, 16))
    return fail(BTF_ERR_ARG, "btf_panels_to_t2: null or misaligned pointer");
  if (!current_device()) return BTF_ERR_STATE;
  panels_to_t2_kernel<<<grid_for((N + 3) / 4 * (K / 128)), kThreads, 0, (cudaStream_t)stream>>>(
      static_cast<const uint8_t*>(panels), N, K, codes, scales);
  return launch_status("panels_to_t2_kernel");
}

}  // extern "C"
