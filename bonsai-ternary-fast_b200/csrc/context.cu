// Library state: error reporting, per-device initialisation, layout sizes.
#include <cstdarg>
#include <cstring>
#include <mutex>

#include "common.cuh"

namespace btf {

namespace {
thread_local std::string g_last_error;
thread_local unsigned long long* g_stamp_next = nullptr;
constexpr int kMaxDevices = 64;
DeviceInfo g_dev[kMaxDevices];
std::mutex g_dev_mu;
}  // namespace

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(BTF_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

unsigned long long* take_stamp() {
  unsigned long long* s = g_stamp_next;
  g_stamp_next = nullptr;
  return s;
}

const DeviceInfo* current_device() {
  int dev = -1;
  const cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cuda_fail(e, "cudaGetDevice");
    return nullptr;
  }
  if (dev < 0 || dev >= kMaxDevices || !g_dev[dev].ready) {
    fail(BTF_ERR_STATE, "btf_init(%d) has not been called for the current device", dev);
    return nullptr;
  }
  return &g_dev[dev];
}

// Kernel attribute set-up lives beside each kernel; btf_init calls these.
int gemv_setup(DeviceInfo& d);
int gemm_setup(DeviceInfo& d);
int gemm_wm_setup(DeviceInfo& d);
int gemv_mma_setup(DeviceInfo& d);
int chain_setup(DeviceInfo& d);

}  // namespace btf

using namespace btf;

extern "C" {

const char* btf_status_string(int status) {
  switch (status) {
    case BTF_OK: return "ok";
    case BTF_ERR_ARG: return "invalid argument";
    case BTF_ERR_CUDA: return "CUDA error";
    case BTF_ERR_UNSUPPORTED: return "unsupported";
    case BTF_ERR_TIMEOUT: return "device wait timed out";
    case BTF_ERR_STATE: return "not initialised";
    default: return "unknown status";
  }
}

const char* btf_last_error(void) { return g_last_error.c_str(); }

const char* btf_version(void) { return "btf_b200 0.2 (sm_100a)"; }

int btf_stamp_next(unsigned long long* slot) {
  if (slot && (reinterpret_cast<uintptr_t>(slot) & 7))
    return fail(BTF_ERR_ARG, "btf_stamp_next: the slot must be 8-byte aligned");
  g_stamp_next = slot;
  return BTF_OK;
}

int btf_init(int device) {
  if (device < 0 || device >= kMaxDevices) return fail(BTF_ERR_ARG, "btf_init: device %d out of range", device);
  std::lock_guard<std::mutex> lock(g_dev_mu);
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  e = cudaSetDevice(device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  DeviceInfo d;
  int major = 0, minor = 0;
  int st = BTF_OK;
  if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, device)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&d.optin_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&d.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device)) !=
          cudaSuccess ||
      (e = cudaDeviceGetAttribute(&d.l2_bytes, cudaDevAttrL2CacheSize, device)) != cudaSuccess) {
    st = cuda_fail(e, "cudaDeviceGetAttribute");
  } else if (major != 10 || minor != 0) {
    st = fail(BTF_ERR_UNSUPPORTED, "btf_b200 is built for sm_100a (B200); device %d is sm_%d%d", device, major, minor);
  } else if (g_dev[device].ready) {
    st = BTF_OK;  // already initialised
  } else if ((st = gemv_setup(d)) == BTF_OK && (st = gemm_setup(d)) == BTF_OK && (st = gemm_wm_setup(d)) == BTF_OK &&
             (st = gemv_mma_setup(d)) == BTF_OK && (st = chain_setup(d)) == BTF_OK) {
    d.ready = true;
    g_dev[device] = d;
  }
  cudaSetDevice(prev);
  return st;
}

int64_t btf_panel_bytes(int64_t N, int64_t K) {
  if (N < 0 || K < 0) return 0;
  return groups_of(N) * slices_of(K) * (int64_t)kPanelBytes;
}
int64_t btf_t2_codes_bytes(int64_t N, int64_t K) { return N * (K / 4); }
int64_t btf_t2_scales_bytes(int64_t N, int64_t K) { return N * (K / 128) * 2; }

}  // extern "C"

// ---- device buffers shared across processes (CUDA IPC)
extern "C" {

int btf_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes == 0) return fail(BTF_ERR_ARG, "btf_alloc: null out pointer or zero size");
  const cudaError_t e = cudaMalloc(ptr, bytes);
  return e == cudaSuccess ? BTF_OK : cuda_fail(e, "btf_alloc");
}

int btf_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? BTF_OK : cuda_fail(e, "btf_free");
}

int btf_ipc_handle(void* ptr, void* handle64) {
  if (!ptr || !handle64) return fail(BTF_ERR_ARG, "btf_ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return cuda_fail(e, "btf_ipc_handle");
  static_assert(sizeof h == 64, "CUDA IPC handles are 64 bytes");
  memcpy(handle64, &h, sizeof h);
  return BTF_OK;
}

int btf_ipc_open(const void* handle64, void** ptr) {
  if (!handle64 || !ptr) return fail(BTF_ERR_ARG, "btf_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle64, sizeof h);
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? BTF_OK : cuda_fail(e, "btf_ipc_open");
}

int btf_ipc_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? BTF_OK : cuda_fail(e, "btf_ipc_close");
}

}  // extern "C"
