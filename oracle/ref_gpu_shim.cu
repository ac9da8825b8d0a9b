// C entry points over the reference's OWN CUDA launchers (src/cuda/kernels.cu,
// compiled unmodified from the reference tree by oracle/Makefile into
// _ref/libbtf_ref_gpu.so). TEST AND BENCHMARK INFRASTRUCTURE ONLY: bench.py times
// the reference's GPU GEMV through it as the GPU baseline beside the product's
// numbers, on the same shapes; the product never links it.
//
// Each function maps one reference launcher (src/cuda/kernels.cuh:17-56) and
// turns its std::runtime_error into a nonzero status with a message.
#include <cstring>
#include <stdexcept>
#include <string>

#include "kernels.cuh"

namespace {
thread_local std::string g_err;
template <typename F>
int guarded(F&& f) {
  try {
    f();
    g_err.clear();
    return 0;
  } catch (const std::exception& e) {
    g_err = e.what();
    return 1;
  }
}
}  // namespace

extern "C" {

__attribute__((visibility("default"))) const char* ref_gpu_last_error(void) { return g_err.c_str(); }

// btf::cuda::kernels_init (kernels.cuh:17) on `device` (made current).
__attribute__((visibility("default"))) int ref_gpu_init(int device) {
  return guarded([&] {
    if (cudaSetDevice(device) != cudaSuccess) throw std::runtime_error("cudaSetDevice");
    btf::cuda::kernels_init(device);
  });
}

// btf::cuda::gemv_max_nb (kernels.cuh:20).
__attribute__((visibility("default"))) int ref_gpu_max_nb(int K) { return btf::cuda::gemv_max_nb(K); }

// btf::cuda::launch_repack (kernels.cuh:24): PTQ1_0 blocks -> T2 codes + fp16 scales.
__attribute__((visibility("default"))) int ref_gpu_repack(const void* src, long long nblocks, void* codes,
                                                          void* scales, void* stream) {
  return guarded([&] {
    btf::cuda::launch_repack(static_cast<const uint8_t*>(src), nblocks, static_cast<uint8_t*>(codes),
                             static_cast<uint16_t*>(scales), static_cast<cudaStream_t>(stream));
  });
}

// btf::cuda::launch_prep (kernels.cuh:42-43) with no norm and no transform: Q8_0 of x.
__attribute__((visibility("default"))) int ref_gpu_quant(const float* x, int ldx, int M, int n, void* q, void* d,
                                                         void* s, void* stream) {
  return guarded([&] {
    btf::cuda::Q8Act a;
    a.q = static_cast<int8_t*>(q);
    a.d = static_cast<float*>(d);
    a.s = static_cast<int*>(s);
    btf::cuda::Hx hx;
    btf::cuda::launch_prep(x, ldx, M, n, nullptr, 0.0f, hx, nullptr, 0, a, static_cast<cudaStream_t>(stream));
  });
}

// btf::cuda::launch_gemv (kernels.cuh:56) over nseg T2 segments.
__attribute__((visibility("default"))) int ref_gpu_gemv(const void* const* codes, const void* const* scales,
                                                        const int* N, float* const* y, const int* ldy, int nseg,
                                                        int K, int M, const void* q, const void* d, const void* s,
                                                        int mode, void* stream) {
  return guarded([&] {
    btf::cuda::GemvSeg segs[3];
    for (int i = 0; i < nseg && i < 3; ++i) {
      segs[i].codes = static_cast<const uint8_t*>(codes[i]);
      segs[i].scales = static_cast<const uint16_t*>(scales[i]);
      segs[i].N = N[i];
      segs[i].y = y[i];
      segs[i].ldy = ldy[i];
    }
    btf::cuda::Q8Act a;
    a.q = const_cast<int8_t*>(static_cast<const int8_t*>(q));
    a.d = const_cast<float*>(static_cast<const float*>(d));
    a.s = const_cast<int*>(static_cast<const int*>(s));
    btf::cuda::launch_gemv(segs, nseg, K, M, a, static_cast<btf::cuda::GemvMode>(mode),
                           static_cast<cudaStream_t>(stream));
  });
}

}  // extern "C"
