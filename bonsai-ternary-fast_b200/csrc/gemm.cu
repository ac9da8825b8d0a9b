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
// Epilogue arithmetic: one packed FMA and one packed add per element per step.
// A bias MMA of two constant tiles (2 x 64 over 32 columns, N = 256: a chunk's
// 4 regions at once) sets the regions to 4096 before the data MMAs accumulate,
// so each region ends as P = idot + 4096 in [0, 8192]. P's bits read as an
// fp32 value are the denormal P * 2^-149, and
//   fma(d * 2^110, P * 2^-149, -d * 2^-27) = RN(d * idot) * 2^-39
// exactly: the FMA's product is exact, d * 2^110 and d * 2^-27 are exact powers
// of two times d, and the one rounding of a normal result commutes with the
// 2^-39. The 2^39 returns in the weight scale (scale * 2^39, exact), so no
// integer-to-float conversion runs. Q8 scales are fp16 values (0 or 2^-24 ..
// 65504, or inf), so every finite d takes this path; |d| >= 2^18, inf and NaN
// take a conversion path instead.
//
// One CTA computes a 128 x 64 output tile, one 128-column chunk of K at a time:
//   warp 0      producer (one thread): per chunk, TMA of the int8 activation
//               tile (128B swizzle), the tile's raw 2-bit codes and fp16
//               scales (one box each) into input stage s, and of the
//               activation scales d into scale stage ss;
//   warp 1      MMA issuer (one thread) + TMEM owner: per chunk one bias MMA
//               and 4 data MMAs into one of 2 TMEM chunk slots (4 x 64 columns);
//   warps 2-3   expanders: raw codes -> int8 trits in the canonical K-major
//               SW128 layout the MMA reads; fp16 scales -> fp32 (x 2^39);
//   warps 4-19  epilogue: tcgen05.ld (32x32b, 16 columns) of step k+1 in
//               flight during the math of step k, per step T += RN(d * idot),
//               per chunk acc += scale * T; a chunk slot is released as soon as
//               its last step is in registers. The output tile leaves through
//               shared memory as whole rows.
// Per chunk the epilogue makes 2 waits (scales, MMA results) and 2 arrivals.
// Every wait is bounded; on a time-out the kernel records an error word, stops
// issuing work, waits (bounded) for its copies and MMAs, frees TMEM and returns.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "tcgen05.cuh"

namespace btf {
namespace {

using namespace tc;

constexpr int kTileM = 128;
constexpr int kTileN = 64;
constexpr int kChunk = 128;          // K columns per pipeline chunk (one scale block)
constexpr int kStepsPerChunk = 4;    // 32-column MMA steps per chunk
#ifndef BTF_GEMM_STAGES
#define BTF_GEMM_STAGES 7
#endif
#ifndef BTF_GEMM_RASTER_M
#define BTF_GEMM_RASTER_M 1
#endif
constexpr int kStagesA = BTF_GEMM_STAGES;  // input stages: A, codes, raw scales (TMA) and B (expanders)
constexpr int kStagesS = 8;          // scale stages: d (TMA) and fp32 weight scales (expanders)
constexpr int kChunkSlots = 2;       // chunks in flight in TMEM
constexpr int kTmemCols = kChunkSlots * kStepsPerChunk * kTileN;  // 512: all of TMEM
constexpr int kEpiWarps = 16;        // 4 per SMSP
constexpr int kEpiCols = kTileN * 4 / kEpiWarps;  // columns per epilogue thread (16)
constexpr int kExpWarps = 2;         // code expanders (64 threads: 2 row quads x 16 columns each)
constexpr int kExpWarp0 = 2, kEpiWarp0 = kExpWarp0 + kExpWarps;
constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;  // 20 warps: 5 per SMSP leaves 96 registers a thread
// bias MMA: every region starts at sum over 32 columns of kBiasA * kBiasB
constexpr int kBiasA = 2, kBiasB = 64, kBias = 32 * kBiasA * kBiasB;  // 4096 >= 32 * 128
static_assert(kBias == 4096, "the bias is a power of two");
constexpr uint64_t kGemmWaitNs = 1000000000ull;

// Input stage s (chunk c, c % kStagesA == s):
//   A  [128 rows][128 cols] int8 activations (128B swizzle)
//   B  [64 rows][128 cols] int8 trits (128B swizzle), written by the expanders
//   C  raw 2-bit codes of the tile's 8 row groups: [group][quad h][half v][64 B]
//   R  raw fp16 weight scales: [group][row] (16 B per group)
// Scale stage ss (c % kStagesS == ss):
//   D  activation block scales d: [128 rows][4] fp32
//   W  fp32 weight scales x 2^39: [64]
constexpr int kABytes = kTileM * kChunk;                  // 16 KB
constexpr int kBBytes = kTileN * kChunk;                  // 8 KB
constexpr int kCBytes = kTileN * kChunk / 4;              // 2 KB
constexpr int kRBytes = kTileN * 2;                       // 128 B
constexpr int kDBytes = kTileM * kStepsPerChunk * 4;      // 2 KB
constexpr int kWBytes = kTileN * 4;                       // 256 B
constexpr int kStageTxA = kABytes + kCBytes + kRBytes;
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kStagesA * kABytes;
constexpr int kOffC = kOffB + kStagesA * kBBytes;
constexpr int kOffR = kOffC + kStagesA * kCBytes;
constexpr int kOffD = kOffR + kStagesA * kRBytes;
constexpr int kOffW = kOffD + kStagesS * kDBytes;
// bias operands: K-major, no swizzle, 8-row x 16-byte core matrices (LBO 128 B
// along K, SBO 256 B along M/N); every byte equal, so any core-matrix order
// reads the same values
constexpr int kBiasN = kStepsPerChunk * kTileN;            // 256: one bias MMA covers a chunk's 4 regions
constexpr int kBiasABytes = kTileM * 32, kBiasBBytes = kBiasN * 32;  // 4 KB, 8 KB
constexpr int kOffBiasA = (kOffW + kStagesS * kWBytes + 1023) / 1024 * 1024;
constexpr int kOffBiasB = kOffBiasA + kBiasABytes;
constexpr int kOffBar = kOffBiasB + kBiasBBytes;
constexpr int kNumBars = 3 * kStagesA + 3 * kStagesS + 2 * kChunkSlots + 1;
constexpr int kOffFlags = kOffBar + kNumBars * 8;         // TMEM base (4 B), abort flag (4 B)
constexpr int kSmemBytes = kOffFlags + 16 + 1024;         // + slack for 1024-B alignment
static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
static_assert(kOffC % 128 == 0 && kOffR % 128 == 0 && kOffD % 128 == 0 && kOffW % 128 == 0, "TMA destinations");
constexpr int kStgLd = kTileN + 4;  // output staging row (floats): conflict-free float4 writes
static_assert(kTileM * kStgLd * 4 <= kStagesA * kABytes, "output staging fits the A ring");

struct GemmParams {
  int N, M, K;
  float* y;
  int ldy;
  int mode;            // BTF_STORE / BTF_ADD
  int* err;
  int32_t* idot;       // DUMP kernel: [M][N][K/32] integer accumulators (no y is stored)
};

// kind::i8 instruction descriptors of this kernel (M = 128 activation rows)
constexpr uint32_t kIdesc = tc::idesc_i8(kTileM, kTileN);
constexpr uint32_t kIdescBias = tc::idesc_i8(kTileM, kBiasN);
static_assert(kBiasN <= 256 && kBiasN % 16 == 0, "M=128 MMA: N a multiple of 16 up to 256");

// Tensor maps: tmA the int8 activation [M][K]; tmC the panel codes as a 5-D
// tensor {512 B of a quad half, half v, quad h, slice, group}; tmR the panel
// scales {16 B of a block, slice, group}; tmD the activation scales [M][K/32].
// DUMP (parity/debug): the same kernel writes every 32-column region's integer
// accumulator P - kBias (= idot) to p.idot instead of storing y.
template <bool DUMP>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmC,
                const __grid_constant__ CUtensorMap tmR, const __grid_constant__ CUtensorMap tmD, const GemmParams p) {
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
  auto a_full = [&](int s) { return bar0 + (0 * kStagesA + s) * 8; };    // TMA: A, C, R of stage s
  auto ab_empty = [&](int s) { return bar0 + (1 * kStagesA + s) * 8; };  // MMA commit: stage s read
  auto b_full = [&](int s) { return bar0 + (2 * kStagesA + s) * 8; };    // expanders: B[s] written
  auto d_full = [&](int s) { return bar0 + (3 * kStagesA + s) * 8; };    // TMA: D of scale stage s
  auto s_full = [&](int s) { return bar0 + (3 * kStagesA + kStagesS + s) * 8; };      // expanders: W (and D) ready
  auto s_empty = [&](int s) { return bar0 + (3 * kStagesA + 2 * kStagesS + s) * 8; };  // epilogue: stage read
  auto mma_done = [&](int cs) { return bar0 + (3 * kStagesA + 3 * kStagesS + cs) * 8; };
  auto d_free = [&](int cs) { return bar0 + (3 * kStagesA + 3 * kStagesS + kChunkSlots + cs) * 8; };
  const uint32_t final_bar = bar0 + (3 * kStagesA + 3 * kStagesS + 2 * kChunkSlots) * 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffFlags);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffFlags + 8);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesA; ++s) {
      mbar_init(a_full(s), 1);
      mbar_init(ab_empty(s), 1);
      mbar_init(b_full(s), kExpWarps);
    }
    for (int s = 0; s < kStagesS; ++s) {
      mbar_init(d_full(s), 1);
      mbar_init(s_full(s), kExpWarps);
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
  {  // the bias MMA's constant operand tiles
    const uint32_t va = 0x01010101u * kBiasA, vb = 0x01010101u * kBiasB;
    for (int i = threadIdx.x; i < (kBiasABytes + kBiasBBytes) / 16; i += kThreads) {
      const uint32_t v = i < kBiasABytes / 16 ? va : vb;
      reinterpret_cast<uint4*>(smem + kOffBiasA)[i] = make_uint4(v, v, v, v);
    }
    fence_proxy_async_smem();  // generic writes -> visible to the tensor core (async proxy)
  }
  if (warp == 1) {  // TMEM: all 512 columns (2 chunk slots x 4 regions x 64) for this CTA
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"((uint32_t)kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // bounded wait; false (and the abort flag set) on a time-out or after another role's time-out
  auto wait = [&](uint32_t bar, uint32_t parity) -> bool {
    if (mbar_try_wait(bar, parity)) return true;
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
      const int g0 = n0 / kRows;
      pdl_wait();  // the activation and its scales are written by the previous kernel
      // stage indices and fill parities as counters (kStagesA need not be a power of 2)
      int s = 0, ss = 0;
      uint32_t ph = 0, phs = 0;
      for (int c = 0; c < nchunks; ++c) {
        if (c >= kStagesA && !wait(ab_empty(s), ph ^ 1u)) break;
        mbar_expect_tx(a_full(s), kStageTxA);
        tma_load_2d(sbase + kOffA + s * kABytes, &tmA, c * kChunk, m0, a_full(s));
        tma_load_5d(sbase + kOffC + s * kCBytes, &tmC, (c & 7) * 64, 0, 0, c >> 3, g0, a_full(s));
        tma_load_3d(sbase + kOffR + s * kRBytes, &tmR, (c & 7) * 16, c >> 3, g0, a_full(s));
        if (c >= kStagesS && !wait(s_empty(ss), phs ^ 1u)) {
          issued = -(c + 1);  // stage s of chunk c is in flight, its scale stage is not
          break;
        }
        mbar_expect_tx(d_full(ss), kDBytes);
        tma_load_2d(sbase + kOffD + ss * kDBytes, &tmD, c * kStepsPerChunk, m0, d_full(ss));
        issued = c + 1;
        if (++s == kStagesA) s = 0, ph ^= 1u;
        if (++ss == kStagesS) ss = 0, phs ^= 1u;
      }
      if (*abort_flag) {  // leave no copy in flight into this CTA's shared memory (bounded)
        const int na = issued < 0 ? -issued : issued, nd = issued < 0 ? -issued - 1 : issued;
        for (int c = max(0, na - kStagesA); c < na; ++c)
          mbar_wait_bounded(a_full(c % kStagesA), (uint32_t)((c / kStagesA) & 1), kGemmWaitNs / 10);
        for (int c = max(0, nd - kStagesS); c < nd; ++c)
          mbar_wait_bounded(d_full(c % kStagesS), (uint32_t)((c / kStagesS) & 1), kGemmWaitNs / 10);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // descriptors: the start-address field (address >> 4, 14 bits) takes the
      // byte offsets >> 4 by plain addition (shared memory < 256 KB)
      const uint64_t bias_ad = smem_desc_noswz(sbase + kOffBiasA), bias_bd = smem_desc_noswz(sbase + kOffBiasB);
      const uint64_t a_desc0 = smem_desc_sw128(sbase + kOffA), b_desc0 = smem_desc_sw128(sbase + kOffB);
      int s = 0;
      uint32_t ph = 0;
      for (int c = 0; c < nchunks; ++c) {
        if (!wait(a_full(s), ph) || !wait(b_full(s), ph)) break;
        const int cs = c & (kChunkSlots - 1);
        if (c >= kChunkSlots && !wait(d_free(cs), (uint32_t)(((c / kChunkSlots) - 1) & 1))) break;
        tc_fence_after();
        const uint32_t dt = tmem_base + cs * kStepsPerChunk * kTileN;
        mma_i8<kIdescBias>(dt, bias_ad, bias_bd, 0u);  // the chunk's 4 regions = kBias
        const uint64_t ad = a_desc0 + (uint64_t)((s * kABytes) >> 4), bd = b_desc0 + (uint64_t)((s * kBBytes) >> 4);
#pragma unroll
        for (int ks = 0; ks < kStepsPerChunk; ++ks)
          mma_i8<kIdesc>(dt + ks * kTileN, ad + (ks * 32 >> 4), bd + (ks * 32 >> 4), 1u);  // += idot
        mma_commit(mma_done(cs));  // the chunk's MMAs (commits track all prior MMAs)
        mma_commit(ab_empty(s));   // A and B of this chunk are free once its MMAs finish
        if (++s == kStagesA) s = 0, ph ^= 1u;
      }
      mma_commit(final_bar);  // completes when every MMA issued above has finished
      mbar_wait_bounded(final_bar, 0, kGemmWaitNs);
    }
  } else if (warp < kEpiWarp0) {
    // ------------------------------------------------------------ code expanders
    // Thread e expands two row quads (quad h of row groups gi and gi + 4) x 16
    // columns (sub-block t/2, half t&1) of every chunk: the 16-byte quad words
    // at C[s] + group*256 + h*128 + (t&1)*64 + (t/2)*16, into int8 trits of the
    // K-major SW128 B tile. It also converts the fp16 scale of tile row e.
    const int e = threadIdx.x - kExpWarp0 * 32;  // 0..63
    const int t = e & 7, h = (e >> 3) & 1, gi = e >> 4;
    const int coff = gi * 256 + h * 128 + (t & 1) * 64 + (t >> 1) * 16;
    int s = 0, ss = 0;
    uint32_t ph = 0, phs = 0;
    for (int c = 0; c < nchunks; ++c) {
      // a_full(s) for chunk c implies the MMAs of chunk c - kStagesA (which read B[s]) are done
      if (!wait(a_full(s), ph)) break;
      const uint8_t* cs = smem + kOffC + s * kCBytes;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint4 w = *reinterpret_cast<const uint4*>(cs + coff + r * 4 * 256);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int n = (gi + 4 * r) * 8 + h * 4 + k;  // row of the tile
          uint4 o;
          o.x = codes_to_trits((w.x >> (2 * k)) & 0x03030303u);
          o.y = codes_to_trits((w.y >> (2 * k)) & 0x03030303u);
          o.z = codes_to_trits((w.z >> (2 * k)) & 0x03030303u);
          o.w = codes_to_trits((w.w >> (2 * k)) & 0x03030303u);
          const int off = (n >> 3) * 1024 + (n & 7) * 128 + ((t ^ (n & 7)) << 4);
          *reinterpret_cast<uint4*>(smem + kOffB + s * kBBytes + off) = o;
        }
      }
      fence_proxy_async_smem();  // generic writes of B -> visible to the tensor core (async proxy)
      const uint16_t hb = *reinterpret_cast<const uint16_t*>(smem + kOffR + s * kRBytes + e * 2);
      __syncwarp();
      if (lane == 0) mbar_arrive(b_full(s));
      // scale stage: W after the epilogue has released the stage, forwarded once D has landed
      if (c >= kStagesS && !wait(s_empty(ss), phs ^ 1u)) break;
      reinterpret_cast<float*>(smem + kOffW + ss * kWBytes)[e] = __half2float(__ushort_as_half(hb)) * 0x1p39f;
      if (!wait(d_full(ss), phs)) break;
      __syncwarp();
      if (lane == 0) mbar_arrive(s_full(ss));
      if (++s == kStagesA) s = 0, ph ^= 1u;
      if (++ss == kStagesS) ss = 0, phs ^= 1u;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;                    // TMEM lane quarter this warp may access
    const int cg = (warp - kEpiWarp0) >> 2;    // column group of the tile
    const int m = q * 32 + lane;               // tile row of this thread
    // a warp whose 32 rows all lie beyond M keeps the barrier protocol but skips the loads and math
    const bool rows_live = m0 + q * 32 < p.M;
    constexpr int H = kEpiCols / 2;
    float2 acc[H], tsum[H];
#pragma unroll
    for (int i = 0; i < H; ++i) acc[i] = tsum[i] = make_float2(0.f, 0.f);
    pdl_wait();  // y is read (BTF_ADD) and written below
    // T (= tsum) gets RN(d * idot) * 2^-39 for one 32-column step; `first` starts a new 128-column block
    auto step_math = [&](const uint32_t (&dr)[16], float dk, bool first) {
      if (fabsf(dk) < 0x1p18f) {
        const float2 a2 = make_float2(dk * 0x1p110f, dk * 0x1p110f);
        const float2 c2 = make_float2(dk * -0x1p-27f, dk * -0x1p-27f);  // -kBias * 2^-149 * d * 2^110
#pragma unroll
        for (int i = 0; i < H; ++i) {
          const float2 r = __ffma2_rn(a2, make_float2(__uint_as_float(dr[2 * i]), __uint_as_float(dr[2 * i + 1])), c2);
          tsum[i] = first ? r : __fadd2_rn(tsum[i], r);
        }
      } else {  // |d| >= 2^18, inf or NaN: d * 2^110 would overflow; convert the integers instead
        const float ds = dk * 0x1p-39f;
#pragma unroll
        for (int i = 0; i < H; ++i) {
          const float2 r = make_float2(ds * (float)((int)dr[2 * i] - kBias), ds * (float)((int)dr[2 * i + 1] - kBias));
          tsum[i] = first ? r : __fadd2_rn(tsum[i], r);
        }
      }
    };
    bool ok = true;
    if (!rows_live) {
      // every row of this warp lies beyond M: only the barrier protocol. Each
      // arrival follows the wait on the same use of the barrier's stage or
      // slot, which keeps it in that use's phase.
      int ss = 0;
      uint32_t phs = 0;
      for (int c = 0; c < nchunks && ok; ++c) {
        const int cs = c & (kChunkSlots - 1);
        ok = wait(s_full(ss), phs) && wait(mma_done(cs), (uint32_t)((c / kChunkSlots) & 1));
        __syncwarp();
        if (ok && lane == 0) {
          mbar_arrive(d_free(cs));
          mbar_arrive(s_empty(ss));
        }
        if (++ss == kStagesS) ss = 0, phs ^= 1u;
      }
    } else if (nchunks > 0) {
      const uint32_t tlane = tmem_base + ((uint32_t)(q * 32) << 16) + cg * kEpiCols;
      uint32_t buf[2][kEpiCols];
      int ss = 0;
      uint32_t phs = 0;
      // prologue: chunk 0's scales and the load of its first step
      ok = wait(s_full(0), 0) && wait(mma_done(0), 0);
      float4 dv = ok ? *reinterpret_cast<const float4*>(smem + kOffD + m * 16) : make_float4(0.f, 0.f, 0.f, 0.f);
      if (ok) {
        tc_fence_after();
        tmem_ld16_async(tlane, buf[0]);
      }
      for (int c = 0; c < nchunks && ok; ++c) {
        const int cs = c & (kChunkSlots - 1);
        const float dk[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
        for (int ks = 0; ks < kStepsPerChunk; ++ks) {
          tmem_wait16(buf[ks & 1]);  // step ks of chunk c
          if (ks + 1 < kStepsPerChunk) {
            tmem_ld16_async(tlane + (cs * kStepsPerChunk + ks + 1) * kTileN, buf[(ks + 1) & 1]);
          } else {
            // the chunk is in registers: release its slot, start the next chunk's first load
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(d_free(cs));
            if (c + 1 < nchunks) {
              const int cn = c + 1, csn = cn & (kChunkSlots - 1);
              if (!wait(mma_done(csn), (uint32_t)((cn / kChunkSlots) & 1))) ok = false;
              if (ok) {
                tc_fence_after();
                tmem_ld16_async(tlane + csn * kStepsPerChunk * kTileN, buf[0]);
              }
            }
          }
          if constexpr (DUMP) {
            if (m0 + m < p.M) {
              const int nsub = p.K >> 5, nb = n0 + cg * kEpiCols;
              int32_t* out = p.idot + ((int64_t)(m0 + m) * p.N + nb) * nsub + c * kStepsPerChunk + ks;
#pragma unroll
              for (int i = 0; i < kEpiCols; ++i)
                if (nb + i < p.N) out[(int64_t)i * nsub] = (int)buf[ks & 1][i] - kBias;
            }
          }
          step_math(buf[ks & 1], dk[ks], ks == 0);
        }
        // weight scales of the chunk's 128-column block; then the stage is free
        const float* sc = reinterpret_cast<const float*>(smem + kOffW + ss * kWBytes) + cg * kEpiCols;
#pragma unroll
        for (int i = 0; i < H; ++i) {
          const float2 s2 = make_float2(sc[2 * i], sc[2 * i + 1]);
          acc[i] = __ffma2_rn(s2, tsum[i], acc[i]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(s_empty(ss));
        if (++ss == kStagesS) ss = 0, phs ^= 1u;
        if (ok && c + 1 < nchunks) {
          if (!wait(s_full(ss), phs)) ok = false;
          else dv = *reinterpret_cast<const float4*>(smem + kOffD + ss * kDBytes + m * 16);
        }
      }
      if (!ok) tmem_wait16(buf[0]);  // no load left in flight
    }
    // The tile goes out through shared memory as whole rows. The A ring is idle
    // here: this warp has seen every chunk's MMAs complete, and they consumed
    // every chunk's TMA.
    float* stg = reinterpret_cast<float*>(smem + kOffA);  // [128][kStgLd]
    if (rows_live) {
      float4* dst = reinterpret_cast<float4*>(stg + m * kStgLd + cg * kEpiCols);
#pragma unroll
      for (int i = 0; i < H / 2; ++i) dst[i] = make_float4(acc[2 * i].x, acc[2 * i].y, acc[2 * i + 1].x, acc[2 * i + 1].y);
    }
    // every epilogue warp reaches this barrier once (its chunk loop always ends)
    asm volatile("bar.sync 1, %0;" ::"r"(kEpiWarps * 32) : "memory");
    if (!DUMP && !*abort_flag) {
      const int we = warp - kEpiWarp0;
#pragma unroll 1
      for (int rr = 0; rr < kTileM / kEpiWarps; ++rr) {
        const int r = we * (kTileM / kEpiWarps) + rr;
        if (m0 + r >= p.M) break;
        float* yr = p.y + (int64_t)(m0 + r) * p.ldy + n0;
#pragma unroll
        for (int h2 = 0; h2 < kTileN / 32; ++h2) {
          const int col = h2 * 32 + lane;
          if (n0 + col < p.N) {
            const float v = stg[r * kStgLd + col];
            if (p.mode == BTF_ADD) yr[col] += v;
            else yr[col] = v;
          }
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

}  // namespace

int gemm_setup(DeviceInfo& d) {
  if (d.optin_smem < kSmemBytes) return fail(BTF_ERR_UNSUPPORTED, "btf_gemm needs %d B of shared memory", kSmemBytes);
  cudaError_t e = cudaFuncSetAttribute(gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  return e == cudaSuccess ? BTF_OK : cuda_fail(e, "cudaFuncSetAttribute(gemm_kernel)");
}

// One matrix: y[M][ldy] (=|+=) W q. Called by btf_gemm, which btf_gemv calls
// for M >= 64 in store / add mode.
bool wm_serves(const btf_gemv_seg& seg, int M, const btf_q8act& act);
bool mma_serves(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act);
bool mma_two_pass_serves(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act);
int run_gemv_mma_rows(const btf_gemv_seg* segs, int nseg, int K, int m0, int M, const btf_q8act& act, int mode,
                      cudaStream_t st);
int run_gemv_mma(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act, int mode, cudaStream_t st,
                 int32_t* idot, const btf_gather* g, int gseg);
int run_gemm_wm(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act, int mode, cudaStream_t st,
                int32_t* idot, const btf_gather* g, int gseg);

int run_gemm(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act, int mode, cudaStream_t st,
             int32_t* idot = nullptr) {
  const DeviceInfo* dev = current_device();
  if (!dev) return BTF_ERR_STATE;
  const EncodeFn enc = encode_fn();
  if (!enc) return fail(BTF_ERR_CUDA, "btf_gemm: cuTensorMapEncodeTiled unavailable");
  auto encode = [&](CUtensorMap* map, CUtensorMapDataType type, int rank, const void* base, const cuuint64_t* dims,
                    const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle swz,
                    const char* what) -> int {
    const cuuint32_t estr[5] = {1, 1, 1, 1, 1};
    const CUresult r = enc(map, type, (cuuint32_t)rank, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? BTF_OK : fail(BTF_ERR_ARG, "btf_gemm: %s tensor map encoding failed (%d)", what, (int)r);
  };
  const int64_t S = slices_of(K), G = groups_of(seg.N);
  const uint8_t* pan = static_cast<const uint8_t*>(seg.panels);
  CUtensorMap mA, mC, mR, mD;
  {  // activation: int8 [M][K], box 128 columns x 128 rows, 128B swizzle; rows beyond M read as zero
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {(cuuint32_t)kChunk, (cuuint32_t)kTileM};
    if (int rc = encode(&mA, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, act.q, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B, "activation"))
      return rc;
  }
  {  // panel codes {x: 512 B of a quad half (8 blocks x 64 B), half v (stride 512), quad h (1024), slice, group};
     // box: one block (64 B) x 2 halves x 2 quads x 1 slice x 8 groups; groups beyond G read as zero
    const cuuint64_t dims[5] = {512, 2, 2, (cuuint64_t)S, (cuuint64_t)G};
    const cuuint64_t strides[4] = {512, 1024, (cuuint64_t)kPanelBytes,
                                   (cuuint64_t)(S * kPanelBytes)};
    const cuuint32_t box[5] = {64, 2, 2, 1, (cuuint32_t)(kTileN / kRows)};
    if (int rc = encode(&mC, CU_TENSOR_MAP_DATA_TYPE_UINT8, 5, pan, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE,
                        "panel code"))
      return rc;
  }
  {  // panel scales {x: 128 B (8 blocks x 8 rows fp16), slice, group}; box: one block (16 B) x 1 x 8 groups
    const cuuint64_t dims[3] = {128, (cuuint64_t)S, (cuuint64_t)G};
    const cuuint64_t strides[2] = {(cuuint64_t)kPanelBytes, (cuuint64_t)(S * kPanelBytes)};
    const cuuint32_t box[3] = {16, 1, (cuuint32_t)(kTileN / kRows)};
    if (int rc = encode(&mR, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, pan + kCodeBytes, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE, "panel scale"))
      return rc;
  }
  {  // activation block scales: fp32 [M][K/32], box 4 blocks (one chunk) x 128 rows
    const cuuint64_t dims[2] = {(cuuint64_t)(K / 32), (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)(K / 32) * 4};
    const cuuint32_t box[2] = {(cuuint32_t)kStepsPerChunk, (cuuint32_t)kTileM};
    if (int rc = encode(&mD, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, act.d, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_NONE, "activation scale"))
      return rc;
  }
  GemmParams p{};
  p.N = seg.N;
  p.M = M;
  p.K = K;
  p.y = seg.y;
  p.ldy = seg.ldy;
  p.mode = mode;
  p.err = dev->err_word;
  p.idot = idot;
#if BTF_GEMM_RASTER_M
  const dim3 grid((M + kTileM - 1) / kTileM, (seg.N + kTileN - 1) / kTileN);
#else
  const dim3 grid((seg.N + kTileN - 1) / kTileN, (M + kTileM - 1) / kTileM);
#endif
  const cudaError_t e = idot ? launch_pdl(gemm_kernel<true>, grid, dim3(kThreads), (size_t)kSmemBytes, st, mA, mC,
                                          mR, mD, p)
                             : launch_pdl(gemm_kernel<false>, grid, dim3(kThreads), (size_t)kSmemBytes, st, mA, mC,
                                          mR, mD, p);
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
  // per segment: a small batch over a very large matrix goes to the warp-MMA
  // kernel, over many weight tiles to the weight-major kernel
  for (int i = 0; i < nseg; ++i) {
    if (mma_two_pass_serves(segs[i], K, M, act)) {  // two warp-MMA passes of 16 rows
      if (int rc = run_gemv_mma_rows(segs + i, 1, K, 0, 16, act, mode, (cudaStream_t)stream)) return rc;
      if (int rc = run_gemv_mma_rows(segs + i, 1, K, 16, M - 16, act, mode, (cudaStream_t)stream)) return rc;
      continue;
    }
    const int rc = mma_serves(segs[i], K, M, act)
                       ? run_gemv_mma(segs[i], K, M, act, mode, (cudaStream_t)stream, nullptr, nullptr, 0)
                   : wm_serves(segs[i], M, act)
                       ? run_gemm_wm(segs[i], K, M, act, mode, (cudaStream_t)stream, nullptr, nullptr, 0)
                       : run_gemm(segs[i], K, M, act, mode, (cudaStream_t)stream);
    if (rc) return rc;
  }
  return BTF_OK;
}

extern "C" int btf_gemm_idot(const void* panels, int N, int K, int M, btf_q8act act, int32_t* idot, void* stream) {
  if (M <= 0) return BTF_OK;
  if (!panels || (reinterpret_cast<uintptr_t>(panels) & 15) || N <= 0 || K <= 0 || K % 128 || !idot || !act.q ||
      !act.d || (reinterpret_cast<uintptr_t>(act.q) & 15) || (reinterpret_cast<uintptr_t>(act.d) & 15))
    return fail(BTF_ERR_ARG, "btf_gemm_idot: bad arguments (K % 128, q and d 16-byte aligned)");
  const btf_gemv_seg seg{panels, N, nullptr, N};
  return run_gemm(seg, K, M, act, BTF_STORE, (cudaStream_t)stream, idot);
}
