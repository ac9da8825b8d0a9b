// btf_gemm_f32_noalloc: the prefill GEMM from fp32 activations, for callers
// that cannot allocate device memory.
//
// The ordinary route from fp32 activations to a prefill GEMM is two calls,
// btf_quant_q8 into a caller-owned Q8 activation and btf_gemm from it, so the
// caller has to find M*K + 2*(M*K/32)*4 bytes of device memory for that
// intermediate. Some hosts cannot: an engine whose memory manager reserves the
// whole device at start-up and hands a plugin only its operand tensors, or a
// latency-bound serving loop where a cudaMalloc (which may synchronise the
// device) is not allowed between steps. This entry point keeps the Q8
// intermediate in the file-scope device array below instead and runs the same
// two kernels (quant_q8_kernel, then gemm_kernel) on it, through the same entry
// points, so its results are those of the two-call route.
//
// The array belongs to the module: every GPU that loads the library holds its
// own copy of it until the process exits. Its size fixes the largest call,
// M*K <= BTF_GEMM_NOALLOC_MAX_MK.
#include "common.cuh"

namespace btf {
namespace {

constexpr int64_t kMaxMK = BTF_GEMM_NOALLOC_MAX_MK;
constexpr int64_t kQBytes = kMaxMK;                 // int8 q [M][K]
constexpr int64_t kDBytes = kMaxMK / 32 * 4;        // fp32 d [M][K/32]
constexpr int64_t kSBytes = kMaxMK / 32 * 4;        // int32 s [M][K/32]
static_assert(kMaxMK % (32 * 64) == 0, "every region starts on a 256-byte boundary");
static_assert(kQBytes % 256 == 0 && kDBytes % 256 == 0, "q, d and s start 256-byte aligned");

}  // namespace

// The Q8 activation of the most recent call on this device: q, then d, then s.
// Its name in host code is only a host-side handle for the runtime; the
// device address comes from cudaGetSymbolAddress (scratch_base below).
static __device__ __align__(256) uint8_t g_q8_scratch[kQBytes + kDBytes + kSBytes];

namespace {

// Device address of g_q8_scratch on the current device, looked up on every
// call (a cheap host-side lookup once the module is loaded on the device). No
// address is cached, so a cudaDeviceReset followed by btf_init, which loads the
// module again and may place the array elsewhere, is handled.
int scratch_base(uint8_t** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_q8_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "btf_gemm_f32_noalloc: cudaGetSymbolAddress");
  *out = static_cast<uint8_t*>(p);
  return BTF_OK;
}

}  // namespace
}  // namespace btf

using namespace btf;

extern "C" int btf_gemm_f32_noalloc(const btf_gemv_seg* segs, int nseg, int K, int M, const float* x, int ldx,
                                    int mode, void* stream) {
  if (M <= 0) return BTF_OK;
  if (K <= 0 || K % 128) return fail(BTF_ERR_ARG, "btf_gemm_f32_noalloc: K must be a positive multiple of 128 (K=%d)", K);
  if ((int64_t)M * K > kMaxMK)
    return fail(BTF_ERR_ARG,
                "btf_gemm_f32_noalloc: M*K = %lld exceeds the static scratch of %lld elements "
                "(BTF_GEMM_NOALLOC_MAX_MK); use btf_quant_q8 + btf_gemm with a caller buffer",
                (long long)M * K, (long long)kMaxMK);
  if (!x || ldx < K) return fail(BTF_ERR_ARG, "btf_gemm_f32_noalloc: null x or ldx < K (ldx=%d K=%d)", ldx, K);
  if (!segs || nseg < 1 || nseg > 3) return fail(BTF_ERR_ARG, "btf_gemm_f32_noalloc: 1..3 segments (got %d)", nseg);
  if (mode != BTF_STORE && mode != BTF_ADD)
    return fail(BTF_ERR_ARG, "btf_gemm_f32_noalloc: mode must be BTF_STORE or BTF_ADD");
  for (int i = 0; i < nseg; ++i)  // btf_gemm's segment rules, checked before anything is launched
    if (!segs[i].panels || (reinterpret_cast<uintptr_t>(segs[i].panels) & 15) || segs[i].N <= 0 || !segs[i].y ||
        segs[i].ldy < segs[i].N)
      return fail(BTF_ERR_ARG, "btf_gemm_f32_noalloc: segment %d has a bad panel buffer, N, y or ldy", i);
  if (!current_device()) return BTF_ERR_STATE;
  uint8_t* base = nullptr;
  if (int rc = scratch_base(&base)) return rc;
  // Nothing is cleared: the quantiser writes every q, d and s of the M x K
  // activation, and the GEMM reads only those (its tensor maps end at row M).
  btf_q8act act;
  act.q = reinterpret_cast<int8_t*>(base);
  act.d = reinterpret_cast<float*>(base + kQBytes);
  act.s = reinterpret_cast<int32_t*>(base + kQBytes + kDBytes);
  if (int rc = btf_quant_q8(x, ldx, M, K, act, stream)) return rc;
  return btf_gemm(segs, nseg, K, M, act, mode, stream);
}
