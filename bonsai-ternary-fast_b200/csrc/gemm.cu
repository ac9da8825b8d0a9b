// Ternary GEMM for prefill batches (M >= 64) on the tcgen05 int8 tensor cores.
//
// Same result as the GEMV (src/cuda/kernels.cu:238-334 of the reference, which
// serves M > 8 as repeated 8-row GEMV launches, :805-821): for every output
// (m, n),
//   y[m][n] {=, +=} sum_kb  d[m][kb] * scale[n][kb/4] * idot[m][n][kb],
//   idot = sum over the 32 columns of block kb of q[m][k] * trit[n][k].
// The activation scale changes every 32 columns, so each 32-deep MMA result is
// an exact int32 idot that the epilogue must scale on its own: one
// tcgen05.mma.kind::i8 (M=128, N=64, K=32) per 32-column step, each into its
// own TMEM region, and the CUDA-core epilogue does the fp32 work.
//
// One CTA computes a 128 x 64 output tile; warp roles:
//   warp 0      producer: TMA (tensor map, 128B swizzle) of the int8
//               activation tile [128 rows][128 cols] per 128-column chunk, and
//               1-D bulk copies of the weight panels (8 rows x 1024 cols each);
//   warp 1      MMA issuer (one thread) + TMEM owner (alloc / dealloc);
//   warps 2-5   expand the 2-bit codes of the chunk into int8 trits in the
//               canonical K-major SW128 layout the MMA reads, and stage the
//               chunk's activation scales d and fp32 weight scales;
//   warps 6-21  epilogue: TMEM -> registers (tcgen05.ld 32x32b, 16 columns),
//               per step T += d * idot, per 128-column block acc += scale * T;
//               MMA completion and TMEM release are signalled once per chunk
//               (4 steps), with 2 chunks in flight in TMEM.
// Every wait is bounded; on a time-out the kernel records an error word, stops
// issuing work, waits (bounded) for its MMAs, frees TMEM and returns.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace btf {
namespace {

constexpr int kTileM = 128;
constexpr int kTileN = 64;
constexpr int kChunk = 128;          // K columns per pipeline chunk (one scale block)
constexpr int kStepsPerChunk = 4;    // 32-column MMA steps per chunk
#ifndef BTF_GEMM_STAGES
#define BTF_GEMM_STAGES 8
#endif
#ifndef BTF_GEMM_RASTER_M
#define BTF_GEMM_RASTER_M 1
#endif
constexpr int kStagesA = BTF_GEMM_STAGES;  // A / B stages (chunks): freed by the MMA alone
constexpr int kStagesS = 8;          // weight-scale stages (freed by the epilogue)
constexpr int kPrefetch = 4;         // chunks of weight codes the expanders hold in registers
constexpr int kDRegions = 8;         // TMEM accumulator regions (one per in-flight step)
constexpr int kChunkSlots = kDRegions / kStepsPerChunk;  // chunks in flight in TMEM (2): one barrier pair each
constexpr int kTmemCols = kDRegions * kTileN;  // 512: all of TMEM
constexpr int kEpiWarps = 16;        // 4 per SMSP: TMEM-load latency of one hides behind the others' math
constexpr int kEpiCols = kTileN * 4 / kEpiWarps;  // columns per epilogue thread (16)
constexpr int kThreads = (6 + kEpiWarps) * 32;
constexpr int kExpWarp0 = 2, kEpiWarp0 = 6;
constexpr uint64_t kGemmWaitNs = 1000000000ull;

constexpr int kABytes = kTileM * kChunk;                  // 16 KB
constexpr int kBBytes = kTileN * kChunk;                  // 8 KB
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kStagesA * kABytes;
constexpr int kOffS = kOffB + kStagesA * kBBytes;          // s: [stage][64] fp32 weight scales
constexpr int kOffBar = kOffS + kStagesS * kTileN * 4;
constexpr int kNumBars = 3 * kStagesA + 2 * kStagesS + 2 * kChunkSlots + 4;
constexpr int kOffTmemSlot = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffTmemSlot + 16 + 1024;      // + slack for 1024-B alignment
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");

struct GemmParams {
  const uint8_t* pan;  // weight panels of an [N][K] matrix
  int N, M, K, S;
  float* y;
  int ldy;
  const float* d;      // activation block scales [M][K/32]
  int mode;            // BTF_STORE / BTF_ADD
  int* err;
};

// ---- tcgen05 / descriptor helpers (PTX ISA, sm_100a)
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
  // K-major, 128-byte swizzle: start >> 4, LBO = 16 B (unused when swizzled),
  // SBO = 1024 B between 8-row groups, descriptor version 1, layout type 2.
  return (uint64_t)((addr >> 4) & 0x3fffu) | ((uint64_t)1u << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}
// kind::i8 instruction descriptor: D s32, A s8, B s8, both K-major, M = 128, N = 64.
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTileN >> 3) << 17) |
                            ((uint32_t)(kTileM >> 4) << 24);

__device__ __forceinline__ void mma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate), "r"(0u)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// 32 lanes x 16 columns of 32-bit TMEM -> 16 registers per thread, without the
// wait: the registers are valid only after tmem_wait16 on the same array.
__device__ __forceinline__ void tmem_ld16_async(uint32_t addr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(addr)
      : "memory");
}
// The wait names the destination registers as read-write operands, so the
// compiler orders every use of them after it.
__device__ __forceinline__ void tmem_wait16(uint32_t (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
                 "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// 4 codes (bytes 0..2 in the low 2 bits of each byte) -> 4 int8 trits (code - 1)
__device__ __forceinline__ uint32_t codes_to_trits(uint32_t c) {
  return ((c | 0x80808080u) - 0x01010101u) ^ 0x80808080u;
}

__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmA, const GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base (SW128 atoms and TMA destinations)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#if BTF_GEMM_RASTER_M
  // the M tiles of one N tile run side by side: they share its weight codes in L2
  const int n0 = blockIdx.y * kTileN, m0 = blockIdx.x * kTileM;
#else
  const int n0 = blockIdx.x * kTileN, m0 = blockIdx.y * kTileM;
#endif
  const int nchunks = p.K / kChunk;

  const uint32_t bar0 = sbase + kOffBar;
  auto a_full = [&](int s) { return bar0 + (0 * kStagesA + s) * 8; };
  auto ab_empty = [&](int s) { return bar0 + (1 * kStagesA + s) * 8; };
  auto b_full = [&](int s) { return bar0 + (2 * kStagesA + s) * 8; };
  auto s_full = [&](int s) { return bar0 + (3 * kStagesA + s) * 8; };
  auto s_empty = [&](int s) { return bar0 + (3 * kStagesA + kStagesS + s) * 8; };
  // per chunk slot cs (TMEM regions 4cs .. 4cs+3): MMAs done / read out by the epilogue
  auto mma_done = [&](int cs) { return bar0 + (3 * kStagesA + 2 * kStagesS + cs) * 8; };
  auto d_free = [&](int cs) { return bar0 + (3 * kStagesA + 2 * kStagesS + kChunkSlots + cs) * 8; };
  const uint32_t final_bar = bar0 + (3 * kStagesA + 2 * kStagesS + 2 * kChunkSlots) * 8;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffTmemSlot + 8);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffTmemSlot);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesA; ++s) {
      mbar_init(a_full(s), 1);
      mbar_init(ab_empty(s), 1);
      mbar_init(b_full(s), 4);
    }
    for (int s = 0; s < kStagesS; ++s) {
      mbar_init(s_full(s), 4);
      mbar_init(s_empty(s), kEpiWarps);
    }
    for (int r = 0; r < kChunkSlots; ++r) {
      mbar_init(mma_done(r), 1);
      mbar_init(d_free(r), kEpiWarps);
    }
    mbar_init(final_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {  // TMEM: all 512 columns (8 regions x 64) for this CTA
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
    if (*abort_flag) return false;
    if (mbar_wait_bounded(bar, parity, kGemmWaitNs)) return true;
    atomicCAS(p.err, 0, kErrWaitTimeout);
    *abort_flag = 1;
    return false;
  };

  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int issued = 0;
      pdl_wait();  // the activation tile is written by the previous kernel
      for (int c = 0; c < nchunks; ++c) {
        const int s = c % kStagesA;
        if (c >= kStagesA && !wait(ab_empty(s), (uint32_t)((c / kStagesA - 1) & 1))) break;
        mbar_expect_tx(a_full(s), kABytes);
        tma_load_2d(sbase + kOffA + s * kABytes, &tmA, c * kChunk, m0, a_full(s));
        issued = c + 1;
      }
      if (*abort_flag)  // leave no copy in flight into this CTA's shared memory (bounded)
        for (int c = max(0, issued - kStagesA); c < issued; ++c)
          mbar_wait_bounded(a_full(c % kStagesA), (uint32_t)((c / kStagesA) & 1), kGemmWaitNs / 10);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      for (int c = 0; c < nchunks; ++c) {
        const int s = c % kStagesA;
        const uint32_t ph = (uint32_t)((c / kStagesA) & 1);
        if (!wait(a_full(s), ph) || !wait(b_full(s), ph)) break;
        const int cs = c % kChunkSlots;
        if (c >= kChunkSlots && !wait(d_free(cs), (uint32_t)((c / kChunkSlots - 1) & 1))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < kStepsPerChunk; ++ks) {
          const uint64_t ad = smem_desc_sw128(sbase + kOffA + s * kABytes + ks * 32);
          const uint64_t bd = smem_desc_sw128(sbase + kOffB + s * kBBytes + ks * 32);
          mma_i8(tmem_base + (cs * kStepsPerChunk + ks) * kTileN, ad, bd, 0u);
        }
        mma_commit(mma_done(cs));  // the chunk's 4 steps (commits track all prior MMAs)
        mma_commit(ab_empty(s));   // A and B of this chunk are free once its MMAs finish
      }
      mma_commit(final_bar);  // completes when every MMA issued above has finished
      mbar_wait_bounded(final_bar, 0, kGemmWaitNs);
    }
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------------------------ code expanders
    // Thread e owns one row quad (4 rows) x 16 columns of every chunk: the
    // 16-byte quad word at panel offset h*1024 + v*512 + (4b + t/2)*16 (b = chunk
    // within its 1024-column slice). The words are read from global memory
    // kPrefetch chunks ahead into registers; threads e < 64 also fetch the fp16
    // block scale of tile row e.
    const int e = threadIdx.x - kExpWarp0 * 32;  // 0..127
    const int G = (int)groups_of(p.N);
    const int g0 = n0 / kRows;
    const int qd = e >> 3, t = e & 7;
    const int gi = qd >> 1, h = qd & 1, v = t & 1;
    const bool have_codes = g0 + gi < G;
    const uint8_t* cbase = p.pan + (int64_t)(g0 + min(gi, G - 1 - g0)) * p.S * kPanelBytes + h * 1024 + v * 512 +
                           (t >> 1) * 16;
    const int sg = e >> 3, sr = e & 7;  // scale: row group and row of tile row e (e < 64)
    const bool have_scale = e < kTileN && g0 + sg < G;
    const uint8_t* sbase_g = p.pan + (int64_t)(g0 + min(sg, G - 1 - g0)) * p.S * kPanelBytes + kCodeBytes + sr * 2;
    auto code_addr = [&](int c) { return cbase + (int64_t)(c >> 3) * kPanelBytes + (c & 7) * 64; };
    auto scale_addr = [&](int c) { return sbase_g + (int64_t)(c >> 3) * kPanelBytes + (c & 7) * 16; };
    uint4 wq[kPrefetch];
    uint16_t sq[kPrefetch];
#pragma unroll
    for (int u = 0; u < kPrefetch; ++u) {
      wq[u] = (have_codes && u < nchunks) ? ld_nc_v4(code_addr(u)) : make_uint4(0, 0, 0, 0);
      sq[u] = (have_scale && u < nchunks) ? __ldg(reinterpret_cast<const unsigned short*>(scale_addr(u))) : 0;
    }
    bool ok = true;
    for (int c0 = 0; c0 < nchunks && ok; c0 += kPrefetch) {
#pragma unroll
      for (int u = 0; u < kPrefetch; ++u) {
        const int c = c0 + u;
        if (c >= nchunks) break;
        const int s = c % kStagesA, ss = c % kStagesS;
        if (c >= kStagesA && !wait(ab_empty(s), (uint32_t)((c / kStagesA - 1) & 1))) {
          ok = false;
          break;
        }
        if (c >= kStagesS && !wait(s_empty(ss), (uint32_t)((c / kStagesS - 1) & 1))) {
          ok = false;
          break;
        }
        const uint4 w = wq[u];
        const uint16_t hb = sq[u];
        if (c + kPrefetch < nchunks) {
          if (have_codes) wq[u] = ld_nc_v4(code_addr(c + kPrefetch));
          if (have_scale) sq[u] = __ldg(reinterpret_cast<const unsigned short*>(scale_addr(c + kPrefetch)));
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int n = gi * 8 + h * 4 + k;  // row of the tile
          uint4 o;
          o.x = codes_to_trits((w.x >> (2 * k)) & 0x03030303u);
          o.y = codes_to_trits((w.y >> (2 * k)) & 0x03030303u);
          o.z = codes_to_trits((w.z >> (2 * k)) & 0x03030303u);
          o.w = codes_to_trits((w.w >> (2 * k)) & 0x03030303u);
          const int off = (n >> 3) * 1024 + (n & 7) * 128 + ((t ^ (n & 7)) << 4);
          *reinterpret_cast<uint4*>(smem + kOffB + s * kBBytes + off) = o;
        }
        if (e < kTileN)
          reinterpret_cast<float*>(smem + kOffS)[ss * kTileN + e] = __half2float(__ushort_as_half(hb));
        fence_proxy_async_smem();  // generic writes of B -> visible to the tensor core (async proxy)
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(b_full(s));
          mbar_arrive(s_full(ss));
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                    // TMEM lane quarter this warp may access
    const int cg = (warp - kEpiWarp0) >> 2;    // column group of the tile
    const int m = q * 32 + lane;               // tile row of this thread
    constexpr int H = kEpiCols / 2;
    float2 acc[H], tsum[H];
#pragma unroll
    for (int i = 0; i < H; ++i) acc[i] = tsum[i] = make_float2(0.f, 0.f);
    const float2 nmagic = make_float2(-kMagicFloat, -kMagicFloat);
    // activation scales of this row, [K/32] fp32, read from global memory one
    // chunk ahead (rows beyond M read row M-1: their sums are never stored)
    pdl_wait();  // d is written by the previous kernel; y is read (BTF_ADD) and written below
    const float4* drow = reinterpret_cast<const float4*>(p.d + (int64_t)min(m0 + m, p.M - 1) * (p.K / 32));
    float4 dnext = __ldg(drow);
    auto step_math = [&](const uint32_t (&dr)[16], float dk) {
      const float2 d2 = make_float2(dk, dk);
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const float2 f = __fadd2_rn(
            make_float2(__int_as_float((int)dr[2 * i] + kMagicInt), __int_as_float((int)dr[2 * i + 1] + kMagicInt)),
            nmagic);
        tsum[i] = __ffma2_rn(d2, f, tsum[i]);
      }
    };
    bool ok = true;
    for (int c = 0; c < nchunks && ok; ++c) {
      const int ss = c % kStagesS;
      const float4 dv = dnext;
      if (c + 1 < nchunks) dnext = __ldg(drow + c + 1);
      const float dk[4] = {dv.x, dv.y, dv.z, dv.w};
      uint32_t dr[2][kEpiCols];
      // one wait per chunk; step ks + 1 is loaded while step ks's math runs
      const int cs = c % kChunkSlots;
      if (!wait(mma_done(cs), (uint32_t)((c / kChunkSlots) & 1))) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + cs * kStepsPerChunk * kTileN + cg * kEpiCols;
      tmem_ld16_async(taddr, dr[0]);
#pragma unroll
      for (int ks = 0; ks < kStepsPerChunk; ++ks) {
        tmem_wait16(dr[ks & 1]);
        if (ks + 1 < kStepsPerChunk) tmem_ld16_async(taddr + (ks + 1) * kTileN, dr[(ks + 1) & 1]);
        step_math(dr[ks & 1], dk[ks]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(d_free(cs));
      if (!wait(s_full(ss), (uint32_t)((c / kStagesS) & 1))) break;
      const float* sc = reinterpret_cast<const float*>(smem + kOffS) + ss * kTileN + cg * kEpiCols;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const float2 s2 = make_float2(sc[2 * i], sc[2 * i + 1]);
        acc[i] = __ffma2_rn(s2, tsum[i], acc[i]);
        tsum[i] = make_float2(0.f, 0.f);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty(ss));
    }
    if (ok && !*abort_flag && m0 + m < p.M) {
      float* yr = p.y + (int64_t)(m0 + m) * p.ldy + n0 + cg * kEpiCols;
#pragma unroll
      for (int i = 0; i < H; ++i) {
        const int n = n0 + cg * kEpiCols + 2 * i;
        if (n < p.N) {
          if (p.mode == BTF_ADD) yr[2 * i] += acc[i].x;
          else yr[2 * i] = acc[i].x;
        }
        if (n + 1 < p.N) {
          if (p.mode == BTF_ADD) yr[2 * i + 1] += acc[i].y;
          else yr[2 * i + 1] = acc[i].y;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"((uint32_t)kTmemCols)
                 : "memory");
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(f);
  });
  return fn;
}

}  // namespace

int gemm_setup(DeviceInfo& d) {
  if (d.optin_smem < kSmemBytes) return fail(BTF_ERR_UNSUPPORTED, "btf_gemm needs %d B of shared memory", kSmemBytes);
  const cudaError_t e = cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  return e == cudaSuccess ? BTF_OK : cuda_fail(e, "cudaFuncSetAttribute(gemm_kernel)");
}

// One matrix: y[M][ldy] (=|+=) W q. Called by btf_gemm / btf_gemv (M >= 64).
int run_gemm(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act, int mode, cudaStream_t st) {
  const DeviceInfo* dev = current_device();
  if (!dev) return BTF_ERR_STATE;
  const EncodeFn enc = encode_fn();
  if (!enc) return fail(BTF_ERR_CUDA, "btf_gemm: cuTensorMapEncodeTiled unavailable");
  // activation tile map: int8 [M][K], box 128 columns x 128 rows, 128B swizzle,
  // rows beyond M read as zero
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)K};
  const cuuint32_t box[2] = {(cuuint32_t)kChunk, (cuuint32_t)kTileM};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t*>(act.q), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(BTF_ERR_ARG, "btf_gemm: tensor map encoding failed (%d)", (int)r);
  GemmParams p{};
  p.pan = static_cast<const uint8_t*>(seg.panels);
  p.N = seg.N;
  p.M = M;
  p.K = K;
  p.S = (int)slices_of(K);
  p.y = seg.y;
  p.ldy = seg.ldy;
  p.d = act.d;
  p.mode = mode;
  p.err = dev->err_word;
#if BTF_GEMM_RASTER_M
  const dim3 grid((M + kTileM - 1) / kTileM, (seg.N + kTileN - 1) / kTileN);
#else
  const dim3 grid((seg.N + kTileN - 1) / kTileN, (M + kTileM - 1) / kTileM);
#endif
  const cudaError_t e = launch_pdl(gemm_kernel, grid, dim3(kThreads), (size_t)kSmemBytes, st, map, p);
  return e == cudaSuccess ? launch_status("gemm_kernel") : cuda_fail(e, "gemm_kernel launch");
}

}  // namespace btf

using namespace btf;

extern "C" int btf_gemm(const btf_gemv_seg* segs, int nseg, int K, int M, btf_q8act act, int mode, void* stream) {
  if (M <= 0) return BTF_OK;
  if (!segs || nseg < 1 || nseg > 3) return fail(BTF_ERR_ARG, "btf_gemm: 1..3 segments (got %d)", nseg);
  if (mode != BTF_STORE && mode != BTF_ADD) return fail(BTF_ERR_ARG, "btf_gemm: mode must be BTF_STORE or BTF_ADD");
  if (K <= 0 || K % 128) return fail(BTF_ERR_ARG, "btf_gemm: K must be a positive multiple of 128 (K=%d)", K);
  if (!act.q || !act.d || (reinterpret_cast<uintptr_t>(act.q) & 15) || (reinterpret_cast<uintptr_t>(act.d) & 15))
    return fail(BTF_ERR_ARG, "btf_gemm: q and d must be 16-byte aligned");
  for (int i = 0; i < nseg; ++i) {
    if (!segs[i].panels || (reinterpret_cast<uintptr_t>(segs[i].panels) & 15) || segs[i].N <= 0 || !segs[i].y ||
        segs[i].ldy < segs[i].N)
      return fail(BTF_ERR_ARG, "btf_gemm: segment %d has a bad panel buffer, N, y or ldy", i);
  }
  for (int i = 0; i < nseg; ++i)
    if (int rc = run_gemm(segs[i], K, M, act, mode, (cudaStream_t)stream)) return rc;
  return BTF_OK;
}
