// Shared definitions of the btf_b200 CUDA library: status plumbing, the panel
// layout, and the few PTX instructions the kernels use directly.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#include "btf_b200.h"

namespace btf {

// ------------------------------------------------------------------ status
// Records a message for btf_last_error() and returns `status`.
int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
// Turns a CUDA error into BTF_ERR_CUDA with `what` as context.
int cuda_fail(cudaError_t e, const char* what);
// Status of the most recent launch on this thread.
inline int launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? BTF_OK : cuda_fail(e, what);
}

// Per-device limits captured by btf_init().
struct DeviceInfo {
  bool ready = false;
  int sm_count = 0;
  int optin_smem = 0;   // max dynamic shared memory per block (opt-in)
  int smem_per_sm = 0;
  int l2_bytes = 0;
  int* err_word = nullptr;  // device address of the error word (bounded-wait time-outs)
};
// State of the current device, or nullptr (and a recorded error) if btf_init
// was not called for it.
const DeviceInfo* current_device();

// ------------------------------------------------------------------ layout
constexpr int kRows = BTF_PANEL_ROWS;         // rows per row group
constexpr int kCols = BTF_PANEL_COLS;         // columns per slice
constexpr int kPanelBytes = BTF_PANEL_BYTES;  // 8 * 256 code bytes + 8 * 8 * 2 scale bytes
constexpr int kCodeBytes = 2048;              // code part of a panel
constexpr int kSubPerSlice = 32;              // 32-column sub-blocks per slice
constexpr int kBlocksPerSlice = 8;            // 128-column scale blocks per slice

__host__ __device__ inline int64_t groups_of(int64_t N) { return (N + kRows - 1) / kRows; }
__host__ __device__ inline int64_t slices_of(int64_t K) { return (K + kCols - 1) / kCols; }
__host__ __device__ inline int64_t panel_offset(int64_t g, int64_t j, int64_t S) { return (g * S + j) * kPanelBytes; }
// Byte offset inside a panel of row r's codes for sub-block l, and of row r's scale for block b.
__host__ __device__ inline int code_offset(int r, int l) { return r * 256 + l * 8; }
__host__ __device__ inline int scale_offset(int r, int b) { return kCodeBytes + b * 16 + r * 2; }

// Byte of a 32-bit T2 code word filled with code 1 (trit 0) in every field.
constexpr uint32_t kPadWord = 0x55555555u;

// ------------------------------------------------------------------ PTX
// 8-byte streaming load that bypasses L1 (each weight byte is read once).
__device__ __forceinline__ uint2 ld_stream_v2(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// Read-only load that may stay in L1 (activations, shared by every warp).
__device__ __forceinline__ uint4 ld_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Byte-wise dot product, unsigned bytes of a times signed bytes of b, plus c.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Integer-to-float by exponent bias: for |i| < 2^22, the float with bits
// (0x4B400000 + i) equals 12582912 + i exactly, so subtracting 12582912 gives
// (float)i with one FADD.
constexpr int kMagicInt = 0x4B400000;
constexpr float kMagicFloat = 12582912.0f;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace btf

namespace btf {

// ------------------------------------------------------------------ Q8 (one 32-block per warp)
// Quantises the 32 values of a block held one per lane, bit-exact to the host
// rule q8_block_host (include/btf/packed.hpp:117-134 of the reference):
// amax = max |x| (a block of zeros keeps the last element's sign, as the host's
// sequential (amax > a ? amax : a) update does), d = fp16_rne(amax / 127),
// id = amax != 0 ? 127 / amax : 0, q = round_half_even(x * id), s = sum(q).
// Returns q of this lane; d and s are valid in every lane.
__device__ __forceinline__ int q8_warp(float v, float& dq, int& sum) {
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float last = __shfl_sync(0xffffffffu, v, 31);
  const float amax_signed = amax == 0.0f ? last : amax;
  dq = __half2float(__float2half_rn(__fdiv_rn(amax_signed, 127.0f)));
  const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
  const int qv = __float2int_rn(__fmul_rn(v, id));
  sum = qv;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  return qv;
}

// Same rule with each thread holding 4 consecutive values of a block and a
// block spread over 8 consecutive lanes (lane & 7 = which 4 values). Returns the
// four q of this thread packed as int8x4; d and s valid in all 8 lanes.
__device__ __forceinline__ uint32_t q8_quad(float4 v, float& dq, int& sum) {
  float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float last = __shfl_sync(0xffffffffu, v.w, (threadIdx.x & 31) | 7);  // element 31 of the block
  const float amax_signed = amax == 0.0f ? last : amax;
  dq = __half2float(__float2half_rn(__fdiv_rn(amax_signed, 127.0f)));
  const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
  const int q0 = __float2int_rn(__fmul_rn(v.x, id)), q1 = __float2int_rn(__fmul_rn(v.y, id));
  const int q2 = __float2int_rn(__fmul_rn(v.z, id)), q3 = __float2int_rn(__fmul_rn(v.w, id));
  sum = q0 + q1 + q2 + q3;
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  return (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
         ((uint32_t)(q3 & 0xff) << 24);
}

// Same rule with one thread holding a whole 32-value block (v[k] = values
// 4k..4k+3): the per-block division and fp16 rounding run once per block.
// Returns the 32 q as int8 in qa (values 0..15) and qb (values 16..31).
__device__ __forceinline__ void q8_block32(const float4 (&v)[8], uint4& qa, uint4& qb, float& dq, int& sum) {
  float amax = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k)
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w))));
  const float amax_signed = amax == 0.0f ? v[7].w : amax;  // element 31 of the block
  dq = __half2float(__float2half_rn(__fdiv_rn(amax_signed, 127.0f)));
  const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
  uint32_t w[8];
  int s = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int q0 = __float2int_rn(__fmul_rn(v[k].x, id)), q1 = __float2int_rn(__fmul_rn(v[k].y, id));
    const int q2 = __float2int_rn(__fmul_rn(v[k].z, id)), q3 = __float2int_rn(__fmul_rn(v[k].w, id));
    s += q0 + q1 + q2 + q3;
    w[k] = (uint32_t)(q0 & 0xff) | ((uint32_t)(q1 & 0xff) << 8) | ((uint32_t)(q2 & 0xff) << 16) |
           ((uint32_t)(q3 & 0xff) << 24);
  }
  qa = make_uint4(w[0], w[1], w[2], w[3]);
  qb = make_uint4(w[4], w[5], w[6], w[7]);
  sum = s;
}

// Loads 4 consecutive floats (vector load when 16-byte aligned).
__device__ __forceinline__ float4 load4(const float* p, bool vec) {
  if (vec) return *reinterpret_cast<const float4*>(p);
  return make_float4(p[0], p[1], p[2], p[3]);
}

// ------------------------------------------------------------------ async copies, barriers, PDL
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// 1-D bulk copy global -> shared (TMA unit), completion counted on `bar`.
// dst, src and bytes must be multiples of 16; the copy lands in this CTA only.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// 1-D bulk prefetch global -> L2 (no shared memory, no completion tracking).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

#ifndef BTF_WAIT_HINT_NS
#define BTF_WAIT_HINT_NS 0
#endif
// try_wait with a suspend-time hint: a thread whose phase is not complete sleeps
// until the phase completes or about `hint_ns` pass, instead of spinning.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity) {
#if BTF_WAIT_HINT_NS > 0
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"((uint32_t)BTF_WAIT_HINT_NS)
      : "memory");
  return ok != 0;
#else
  return mbar_try_wait(bar, parity);
#endif
}

// Waits for phase `parity` of `bar` for at most about `limit_ns`; false on
// time-out. The clock is read once per 8 tries so that a waiting warp issues
// few instructions.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 8; ++i)
      if (mbar_try_wait_sleep(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue now / wait until the previous kernel's memory is visible.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Thread-block clusters (distributed shared memory). The barriers are the
// hardware cluster barrier: every thread of every CTA of the cluster executes
// each arrive/wait pair exactly once, unconditionally.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_cluster_b32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared::cluster.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// Device-side error word (time-outs of bounded waits); read by btf_device_error().
constexpr int kErrWaitTimeout = 1;

// Kernel end stamps (btf_stamp_next): the slot requested for the next launch made
// by this host thread, or nullptr; taking it clears the request.
unsigned long long* take_stamp();
// Called by every thread of a CTA at its very end (CTA-uniform `slot`): once
// the CTA's work is done, thread 0 raises *slot to the global timer (ns), so
// after the launch *slot is the end time of its last CTA.
__device__ __forceinline__ void stamp_end(unsigned long long* slot) {
  if (slot == nullptr) return;
  __syncthreads();
  if (threadIdx.x == 0) atomicMax(slot, (unsigned long long)globaltimer_ns());
}

// Launches kern<<<grid, block, smem, st>>> with programmatic stream
// serialisation enabled, so it may overlap the tail of the previous kernel.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// launch_pdl with a thread-block cluster of `cluster` CTAs along x (1 = none).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                               int cluster, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cluster > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace btf
