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
};
// State of the current device, or nullptr (and a recorded error) if btf_init
// was not called for it.
const DeviceInfo* current_device();

// ------------------------------------------------------------------ layout
constexpr int kRows = BTF_PANEL_ROWS;         // rows per row group
constexpr int kCols = BTF_PANEL_COLS;         // columns per slice
constexpr int kPanelBytes = BTF_PANEL_BYTES;  // 16 * 256 code bytes + 16 * 8 * 2 scale bytes
constexpr int kCodeBytes = 4096;              // code part of a panel
constexpr int kSubPerSlice = 32;              // 32-column sub-blocks per slice
constexpr int kBlocksPerSlice = 8;            // 128-column scale blocks per slice

__host__ __device__ inline int64_t groups_of(int64_t N) { return (N + kRows - 1) / kRows; }
__host__ __device__ inline int64_t slices_of(int64_t K) { return (K + kCols - 1) / kCols; }
__host__ __device__ inline int64_t panel_offset(int64_t g, int64_t j, int64_t S) { return (g * S + j) * kPanelBytes; }
// Byte offset inside a panel of row r's codes for sub-block l, and of row r's scale for block b.
__host__ __device__ inline int code_offset(int r, int l) { return r * 256 + l * 8; }
__host__ __device__ inline int scale_offset(int r, int b) { return kCodeBytes + b * 32 + r * 2; }

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
