// Weight-major ternary GEMM on the tcgen05 tensor cores, for small batches
// (1 <= M <= 64 rows per tile): the 128-row MMA operand is the WEIGHTS and the
// activation rows are the MMA's N side.
//
// Same contract as gemm_kernel (gemm.cu), which replaces the reference's
// repeated small-batch passes of launch_gemv (src/cuda/kernels.cu:805-821)
// with the math of src/emu_decoder.cpp:143-165: per (activation row m, weight
// row n, 32-column step) one exact int32 idot, scaled by fp16 scale[n] * d[m]
// and summed in fp32. gemm_kernel puts 128 activation rows on the MMA's M side,
// so a batch of 16 fills an eighth of every instruction; here a CTA covers 128
// weight rows x up to 64 activation rows, and every weight byte is read once
// for the whole batch.
//
// The kernel is persistent: CTA b takes the 128-row weight tiles b, b + grid,
// ... and its pipelines run on across tile boundaries, so the epilogue writes
// one tile's rows while the next tile's copies and MMAs are in flight. NA (16,
// 32 or 64) is the activation rows padded to the MMA's N; a TMEM slot of 256
// columns holds 256 / (4 NA) whole 128-column blocks (4 steps of NA columns).
//   workers     kBlockWorkers blocks in flight, each owned by a pair of warps
//               (a single warp at NA = 64). Per 1024-column slice, the tile's 16
//               whole panels and the slice's d and s (activation block scales
//               and sums) are copied into a slice stage (the worker that
//               finishes a slice's last block reloads it). Per block, the pair
//               turns the 2-bit codes into int8 codes (trit + 1: 0, 1, 2) of the
//               K-major SW128 A tile and the fp16 weight scales into fp32
//               (x 2^39); the helper warp writes each activation row's d per
//               step and the code-sum correction below, and loads the pair's
//               next activation tile; the leader's lane 0 issues the block's
//               MMAs (a bias MMA over the block's 4 regions, 4 data MMAs: A =
//               weight codes, B = activations) and their commits. Blocks own
//               disjoint TMEM regions: 2 slots of 256 columns in flight;
//   epilogue    TMEM lane = weight row; each warp reads 16 activation rows x
//               the 4 steps of its blocks of every slot. Warp 0 owns TMEM.
// Arithmetic: the codes are trit + 1, so a step's MMA result is sum (t+1) q =
// idot + s, with s = sum q of the step (the Q8 block sum); a bias MMA of two
// constant tiles first sets every region to 8192, so P = idot + s + 8192 lies
// in [64, 16320]. P's bits read as fp32 are the denormal P * 2^-149, and
//   x = fma(P * 2^-149, 2^110, -2^-26) = (idot + s) * 2^-39
// exactly (an exact product, and an integer below 2^14 times 2^-39 for the
// sum). Per step T = fma(d, x, T); per block T -= sum_steps d * s * 2^-39 (the
// expanders' correction) and acc += scale * 2^39 * T. No integer-to-float
// conversion runs, and every finite d takes the same path. The warps of one
// column group that read different blocks of a slot add their sums in a fixed
// order at the end of the tile, and rows go to y with coalesced stores (lanes
// are consecutive weight rows).
// Every wait is bounded; on a time-out the kernel records the error word, stops
// issuing work, waits (bounded) for its copies and MMAs, frees TMEM and returns.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "tcgen05.cuh"

namespace btf {
namespace {

using namespace tc;

constexpr int kTileW = 128;         // weight rows per tile (MMA M)
constexpr int kNAMax = 64;          // activation rows per tile at most (MMA N)
constexpr int kWmMaxM = kNAMax;     // btf_gemm_wm takes 1 <= M <= this
constexpr int kWmMinM = 9;          // btf_gemv / btf_gemm route 9 <= M <= 64 here (wm_serves)
constexpr int kChunk = 128;         // K columns per block (one weight-scale block)
constexpr int kSteps = 4;           // 32-column MMA steps per block
constexpr int kBlocksPerSliceW = kCols / kChunk;  // 8 blocks per 1024-column panel slice
constexpr int kGroups = kTileW / kRows;  // 16 panel row groups per tile
constexpr int kSlots = 2;           // TMEM slots in flight
constexpr int kSlotCols = 256;      // TMEM columns per slot
constexpr int kTmemCols = kSlots * kSlotCols;  // 512: all of TMEM
constexpr int kBiasA = 4, kBiasB = 64, kBias = 32 * kBiasA * kBiasB;  // every region starts at 8192
static_assert(kBias == 8192, "the bias is a power of two above 32 * 2 * 127");
constexpr uint64_t kWaitNs = 1000000000ull;

// Shared memory, per padded batch width NA:
//   code ring   (2 stages) one 1024-column slice of the tile: the 16 row
//               groups' whole panels (16 x 2176 B, 1-D bulk copies: codes and
//               fp16 scales), the activation scales d of the slice [NA][32]
//               fp32 and the activation block sums s [NA][32] int32 (128B
//               swizzled tiled copies of NA rows each);
//   A ring      (kAStages) [128][128] int8 codes (trit + 1) of one block
//               (SW128), block i in stage i % kAStages;
//   B ring      (kBStages) [NA][128] int8 activations of one block (SW128,
//               TMA), block i in stage i % kBStages, loaded by the helper of
//               block i - kBlockWorkers;
//   scale ring  (kScaleStages) per block: W fp32 weight scales x 2^39 [128],
//               d [4 steps][NA] fp32, the code-sum correction
//               -sum_steps d * s * 2^-39 [NA] fp32, and (dump form) s [4][NA];
//   Stg         [16 activation rows][128 weight rows] fp32, the end-of-tile
//               combine (NA < 64).
// Whole panels keep the number of copy requests per block low (a tiled copy of
// a block's codes alone is 64 rows of 64 bytes).
constexpr int kABytes = kTileW * kChunk;          // 16 KB
constexpr int kPanelsBytes = kGroups * kPanelBytes;  // 34816 B
constexpr int kCodeStages = 2;
constexpr int kStgBytes = 16 * kTileW * 4;        // 8 KB
// bias operands: K-major, no swizzle, 8-row x 16-byte core matrices; every
// byte equal, so any core-matrix order reads the same values
constexpr int kBiasABytes = kTileW * 32, kBiasBBytes = kSlotCols * 32;
constexpr int align1k(int x) { return (x + 1023) / 1024 * 1024; }

template <int NA>
struct Shape {
  static_assert(NA == 16 || NA == 32 || NA == 64, "NA is 16, 32 or 64");
  static constexpr int kNcg = NA / 16;             // 16-row column groups per step
  static constexpr int kBlkPerSlot = 4 / kNcg;     // blocks per TMEM slot
  // epilogue warps: 4 lane quarters x 4 at NA = 64; x 2 below, each warp then
  // reading 2 blocks (NA = 16) or both column groups' blocks (NA = 32) of a slot
  static constexpr int kEpiWarps = NA == 64 ? 16 : 8;
  // warps per block: a pair below NA = 64; one at NA = 64, whose 16 epilogue
  // warps leave no register room for more
  static constexpr int kP = NA == 64 ? 1 : 2;
  // blocks in flight (one pair, or warp, each): 5 at NA = 16, whose 6 A stages
  // keep a pair's next block out of its own previous block's stage (6 pairs,
  // 20 warps at 96 registers, measured slower); 4 otherwise
  static constexpr int kBlockWorkers = NA == 16 ? 5 : 4;
  static constexpr int kWorkers = kBlockWorkers * kP;
  static constexpr int kEpiWarp0 = kWorkers;
  static constexpr int kThreads = (kWorkers + kEpiWarps) * 32;  // 576 (NA 16), 512 (32), 640 (64)
  static constexpr uint32_t kIdesc = idesc_i8(kTileW, NA);
  static constexpr uint32_t kIdescBias = idesc_i8(kTileW, kSteps * NA);  // a block's 4 regions
  static_assert(kBlkPerSlot * kSteps * NA == kSlotCols, "a slot is whole blocks");
  // ring depths: what fits 227 KB for this width
  static constexpr int kAStages = NA == 16 ? 6 : NA == 32 ? 4 : 3;
  static constexpr int kBStages = NA == 64 ? 6 : 8;
  static constexpr int kScaleStages = NA == 64 ? 4 : 8;  // a power of two
  static constexpr int kBBytes = NA * kChunk;
  static constexpr int kDSliceBytes = NA * 32 * 4;  // d (and s) of one slice: [NA][32]
  static constexpr int kCodeStageBytes = kPanelsBytes + 2 * kDSliceBytes;
  // scale stage
  static constexpr int kSOffD = kTileW * 4, kSOffCorr = kSOffD + kSteps * NA * 4, kSOffS = kSOffCorr + NA * 4;
  static constexpr int kScaleStageBytes = kSOffS + kSteps * NA * 4;
  static constexpr int kOffCode = 0;
  static constexpr int kOffA = align1k(kOffCode + kCodeStages * kCodeStageBytes);
  static constexpr int kOffB = kOffA + kAStages * kABytes;
  static constexpr int kOffS = kOffB + kBStages * kBBytes;
  static constexpr int kOffStg = kOffS + kScaleStages * kScaleStageBytes;
  static constexpr int kOffBiasA = align1k(kOffStg + (NA < 64 ? kStgBytes : 0));
  static constexpr int kOffBiasB = kOffBiasA + kBiasABytes;
  static constexpr int kOffBar = kOffBiasB + kBiasBBytes;
  // c_full; a_empty; b_full, b_empty; s_full, s_empty; mma_done, d_free; final; pair
  static constexpr int kNumBars =
      kCodeStages + kAStages + 2 * kBStages + 2 * kScaleStages + 2 * kSlots + 1 + kBlockWorkers;
  // the activation of block j + kBlockWorkers goes into the stage of an older block than j
  static_assert(kBStages > kBlockWorkers, "activation ring deeper than the blocks in flight");
  // TMEM base (4 B), abort flag (4 B), slice counters (4 B each)
  static constexpr int kOffFlags = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffFlags + 16 + 4 * (kCodeStages + 1) + 1024;  // + slack for 1024-B alignment
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  static_assert(kCodeStageBytes % 1024 == 0 && kBBytes % 1024 == 0 && kOffB % 1024 == 0, "SW128 / copy alignment");
  static_assert(kOffS % 16 == 0 && kOffStg % 16 == 0 && kScaleStageBytes % 16 == 0, "vector accesses aligned");
};

struct WmParams {
  int N, M, K;
  int ntiles;           // ceil(N / 128)
  int nslices;          // panel slices per row group: ceil(K / 1024)
  int ngroups;          // row groups of the matrix: ceil(N / 8)
  const uint8_t* panels;
  float* y;
  int ldy;
  int mode;             // BTF_STORE / BTF_ADD
  int* err;
  int32_t* idot;        // DUMP kernel: [M][N][K/32] integer accumulators (no y is stored)
  // GATHER kernel (tagged N-sharded store): every output goes to all `world`
  // ranks' full-width buffers as one 64-bit word (value bits | tag << 32), at
  // the same index as y; tag = *epoch * 1024 + site
  int world;
  unsigned long long* peer[BTF_MAX_RANKS];
  const unsigned* epoch;
  int site;
  unsigned long long* stamp;  // end stamp slot (btf_stamp_next) or null
};

// Tensor maps: tmB the int8 activation [M][K] (box 128 x NA, SW128); tmD the
// activation scales [M][K/32] and tmS the activation block sums [M][K/32]
// (box 32 x NA: one slice). The panels arrive by 1-D bulk copies from p.panels.
// DUMP (parity/debug): the kernel writes every step's integer accumulator
// P - kBias (= idot) to p.idot and stores no y. GATHER: the tagged N-sharded
// store of btf_gemv_gather (store mode).
template <int NA, bool DUMP, bool GATHER = false>
__global__ void __launch_bounds__(Shape<NA>::kThreads, 1)
    gemm_wm_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmD,
                   const __grid_constant__ CUtensorMap tmS, const WmParams p) {
  using S = Shape<NA>;
  constexpr int CS = kCodeStages, AS = S::kAStages, BS = S::kBStages, SS = S::kScaleStages;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base (SW128 atoms and TMA destinations)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = p.K / kChunk;                                     // blocks per tile
  const int nsl = (nb + kBlocksPerSliceW - 1) / kBlocksPerSliceW;  // slices per tile
  const int nslots = (nb + S::kBlkPerSlot - 1) / S::kBlkPerSlot;   // TMEM slot uses per tile
  // this CTA's tiles: blockIdx.x, blockIdx.x + gridDim.x, ... (the grid is at most ntiles)
  const int my_tiles = ((int)blockIdx.x < p.ntiles) ? (p.ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

  const uint32_t bar0 = sbase + S::kOffBar;
  auto c_full = [&](int q) { return bar0 + q * 8; };                          // copies: slice stage q landed
  auto a_empty = [&](int s) { return bar0 + (CS + s) * 8; };                  // MMA commit: A[s] read
  auto b_full = [&](int s) { return bar0 + (CS + AS + s) * 8; };              // TMA: B[s] landed
  auto b_empty = [&](int s) { return bar0 + (CS + AS + BS + s) * 8; };        // MMA commit: B[s] read
  constexpr int kB1 = CS + AS + 2 * BS;
  auto s_full = [&](int s) { return bar0 + (kB1 + s) * 8; };                  // worker: scale stage ready
  auto s_empty = [&](int s) { return bar0 + (kB1 + SS + s) * 8; };            // epilogue: stage read
  auto mma_done = [&](int cs) { return bar0 + (kB1 + 2 * SS + cs) * 8; };     // MMA commits: slot written
  auto d_free = [&](int cs) { return bar0 + (kB1 + 2 * SS + kSlots + cs) * 8; };  // epilogue: slot read
  const uint32_t final_bar = bar0 + (kB1 + 2 * SS + 2 * kSlots) * 8;
  // both warps of a block's pair have written their halves of the A tile (a
  // two-arrival barrier both wait on, so neither can run a phase ahead)
  auto pair_done = [&](int pw) { return bar0 + (kB1 + 2 * SS + 2 * kSlots + 1 + pw) * 8; };
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + S::kOffFlags);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::kOffFlags + 8);
  int* slice_cnt = reinterpret_cast<int*>(smem + S::kOffFlags + 16);  // blocks of slice stage q expanded
  // scale stage ss: W, d [step][row], correction, s [step][row]
  auto sstage = [&](int ss) { return smem + S::kOffS + ss * S::kScaleStageBytes; };

  if (threadIdx.x == 0) {
    for (int q = 0; q < CS; ++q) {
      mbar_init(c_full(q), 1);
      slice_cnt[q] = 0;
    }
    slice_cnt[CS] = 0;  // slices issued
    for (int s = 0; s < AS; ++s) mbar_init(a_empty(s), 1);
    for (int s = 0; s < BS; ++s) {
      mbar_init(b_full(s), 1);
      mbar_init(b_empty(s), 1);
    }
    for (int s = 0; s < SS; ++s) {
      mbar_init(s_full(s), S::kP);  // each warp of the block's pair
      mbar_init(s_empty(s), 4 * S::kNcg);  // the warps that read one block: 4 lane quarters x column groups
    }
    for (int r = 0; r < kSlots; ++r) {
      mbar_init(mma_done(r), S::kBlkPerSlot);  // one commit per block of the slot
      mbar_init(d_free(r), S::kEpiWarps);
    }
    mbar_init(final_bar, S::kWorkers);
    for (int i = 0; i < S::kBlockWorkers; ++i) mbar_init(pair_done(i), 2);
    *abort_flag = 0;
    fence_mbar_init();
  }
  {  // the bias MMA's constant operand tiles
    const uint32_t va = 0x01010101u * kBiasA, vb = 0x01010101u * kBiasB;
    for (int i = threadIdx.x; i < (kBiasABytes + kBiasBBytes) / 16; i += S::kThreads) {
      const uint32_t v = i < kBiasABytes / 16 ? va : vb;
      reinterpret_cast<uint4*>(smem + S::kOffBiasA)[i] = make_uint4(v, v, v, v);
    }
    fence_proxy_async_smem();  // generic writes -> visible to the tensor core (async proxy)
  }
  if (warp == 0) {  // TMEM: all 512 columns (2 slots x 256) for this CTA
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
    if (mbar_wait_bounded(bar, parity, kWaitNs)) return true;
    atomicCAS(p.err, 0, kErrWaitTimeout);
    *abort_flag = 1;
    return false;
  };
  // the same wait made warp-uniform: every lane waits, the warp goes on only if all of them saw the phase
  auto wwait = [&](uint32_t bar, uint32_t parity) -> bool { return __all_sync(0xffffffffu, wait(bar, parity)); };
  // a warp-uniform wait that sleeps between tries (about 100 ns), for the
  // epilogue's long waits: a spinning warp would take issue slots from the
  // worker warp on its SM sub-partition
  auto wwait_sleep = [&](uint32_t bar, uint32_t parity) -> bool {
    bool done = mbar_try_wait(bar, parity);
    if (!__all_sync(0xffffffffu, done)) {
      const uint64_t t0 = globaltimer_ns();
      for (;;) {
        __nanosleep(100);
        done = mbar_try_wait(bar, parity);
        if (__all_sync(0xffffffffu, done)) break;
        if (*abort_flag || globaltimer_ns() - t0 > kWaitNs) {
          atomicCAS(p.err, 0, kErrWaitTimeout);
          *abort_flag = 1;
          return false;
        }
      }
    }
    return true;
  };

  pdl_launch_dependents();

  if (warp < S::kWorkers) {
    // ------------------------------------------------------------ workers
    // Worker pair (or single warp at NA = 64) w takes the CTA's blocks w, w + B,
    // ... (B = kBlockWorkers; over all its tiles). For each, half `half` of the
    // pair: the 2-bit codes of its 8 (or 16) row groups become int8 codes (trit + 1) of the
    // K-major SW128 A tile (lane: quad h of row groups gi, gi + 2, ... x 16
    // columns, sub-block t/2, half t&1 of the panel), and the scale stage gets
    // its rows' fp32 weight scales. The leader's lane 0, once its partner's
    // half is written, issues the block's MMAs: a bias MMA over its 4 regions,
    // then 4 steps. The other warp (the single warp at NA = 64) writes d per
    // step and the code-sum correction, and its lane 0 loads the activation
    // tile of the pair's next block (once the stage's previous block, kBStages
    // back, has been read by its MMAs). The warp that expands the last of a
    // slice's blocks reloads its stage with the slice kCodeStages ahead.
    constexpr int P = S::kP;
    const int w = warp / P, half = warp % P;
    const bool leader = half == 0;
    const bool helper = P == 1 || !leader;  // d, s, the correction and the activation loads
    const int t = lane & 7, h = (lane >> 3) & 1, gi = lane >> 4;
    const int coff = h * 1024 + (t & 1) * 512 + (t >> 1) * 16;
    const int total_sl = my_tiles * nsl, total_blk = my_tiles * nb;
    int* slices_issued = slice_cnt + CS;  // slices whose copies were issued (for the abort drain)
    // one slice into stage gsl % CS: the tile's whole panels of the slice and its d and s
    auto issue_slice = [&](int gsl) {
      const int ti = gsl / nsl, sl = gsl % nsl, q = gsl % CS;
      const int g0 = ((int)blockIdx.x + ti * (int)gridDim.x) * kGroups;
      const int ng = min(kGroups, p.ngroups - g0);  // row groups of a partial last tile are left unloaded
      uint8_t* dst = smem + S::kOffCode + q * S::kCodeStageBytes;
      mbar_expect_tx(c_full(q), (uint32_t)(ng * kPanelBytes + 2 * S::kDSliceBytes));
      for (int g = 0; g < ng; ++g)
        bulk_g2s(smem_u32(dst + g * kPanelBytes), p.panels + ((int64_t)(g0 + g) * p.nslices + sl) * kPanelBytes,
                 kPanelBytes, c_full(q));
      tma_load_2d(smem_u32(dst + kPanelsBytes), &tmD, sl * 32, 0, c_full(q));
      tma_load_2d(smem_u32(dst + kPanelsBytes + S::kDSliceBytes), &tmS, sl * 32, 0, c_full(q));
      *slices_issued = gsl + 1;
    };
    // the activation tile of CTA block j into B stage j % BS
    auto issue_b = [&](int j) {
      const int bs = j % BS;
      mbar_expect_tx(b_full(bs), S::kBBytes);
      tma_load_2d(sbase + S::kOffB + bs * S::kBBytes, &tmB, (j % nb) * kChunk, 0, b_full(bs));
    };
    const int my_blocks = total_blk > w ? (total_blk - 1 - w) / S::kBlockWorkers + 1 : 0;
    int b_issued = 0;  // this warp's blocks whose activation copy was issued (lane 0)
    if (lane == 0) {
      pdl_wait();  // the activation, its scales and sums are written by the previous kernel
      if (warp == 0)
        for (int g = 0; g < min(CS, total_sl); ++g) issue_slice(g);
      if (helper && my_blocks > 0) issue_b(w), b_issued = 1;
    }
    int last_gsl = -1;
    bool ok = true;
    for (int k = 0; k < my_blocks && ok; ++k) {
      const int j = w + k * S::kBlockWorkers, ti = j / nb, kb = j % nb;
      const int gsl = ti * nsl + (kb >> 3), q = gsl % CS, b = kb & (kBlocksPerSliceW - 1);
      if (gsl != last_gsl) {
        if (!wwait(c_full(q), (uint32_t)((gsl / CS) & 1))) break;
        last_gsl = gsl;
      }
      const int sa = j % AS;
      if (j >= AS && !wwait(a_empty(sa), (uint32_t)(((j / AS) - 1) & 1))) break;
      const uint8_t* cst = smem + S::kOffCode + q * S::kCodeStageBytes;
      uint8_t* as = smem + S::kOffA + sa * kABytes;
#pragma unroll
      for (int r = 0; r < kGroups / 2 / P; ++r) {
        const int g = half * (kGroups / P) + gi + 2 * r;
        const uint4 c4 = *reinterpret_cast<const uint4*>(cst + g * kPanelBytes + coff + b * 64);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int n = g * 8 + h * 4 + kk;  // row of the tile
          const uint4 o = make_uint4((c4.x >> (2 * kk)) & 0x03030303u, (c4.y >> (2 * kk)) & 0x03030303u,
                                     (c4.z >> (2 * kk)) & 0x03030303u, (c4.w >> (2 * kk)) & 0x03030303u);
          *reinterpret_cast<uint4*>(as + (n >> 3) * 1024 + (n & 7) * 128 + ((t ^ (n & 7)) << 4)) = o;
        }
      }
      fence_proxy_async_smem();  // generic writes of A -> visible to the tensor core (async proxy)
      // scale stage of block j: after the epilogue has released block j - SS's
      const int ss = j & (SS - 1);
      if (j >= SS && !wwait(s_empty(ss), (uint32_t)(((j / SS) - 1) & 1))) break;
      uint8_t* sst = sstage(ss);
#pragma unroll
      for (int r = 0; r < kTileW / 32 / P; ++r) {
        // fp16 scale of tile row `row` for this block: [block][row in group]
        const int row = half * (kTileW / P) + lane + 32 * r;
        const uint16_t hb =
            *reinterpret_cast<const uint16_t*>(cst + (row >> 3) * kPanelBytes + kCodeBytes + b * 16 + (row & 7) * 2);
        reinterpret_cast<float*>(sst)[row] = __half2float(__ushort_as_half(hb)) * 0x1p39f;
      }
#pragma unroll
      for (int m = lane; helper && m < NA; m += 32) {
        // row m's d and s of this block: 16-byte chunk b of its 128-byte slice
        // row, which the 128B-swizzled copy placed at chunk b ^ (m & 7)
        const int off = m * 128 + ((b ^ (m & 7)) << 4);
        const float4 d4 = *reinterpret_cast<const float4*>(cst + kPanelsBytes + off);
        const int4 s4 = *reinterpret_cast<const int4*>(cst + kPanelsBytes + S::kDSliceBytes + off);
        float* dT = reinterpret_cast<float*>(sst + S::kSOffD);  // [step][row]
        dT[0 * NA + m] = d4.x;
        dT[1 * NA + m] = d4.y;
        dT[2 * NA + m] = d4.z;
        dT[3 * NA + m] = d4.w;
        // the codes are trit + 1, so each step's MMA adds s = sum q of the
        // step: correction -sum_steps d * s * 2^-39 for the epilogue's block sum
        float c = fmaf(d4.x * -0x1p-39f, (float)s4.x, 0.f);
        c = fmaf(d4.y * -0x1p-39f, (float)s4.y, c);
        c = fmaf(d4.z * -0x1p-39f, (float)s4.z, c);
        c = fmaf(d4.w * -0x1p-39f, (float)s4.w, c);
        reinterpret_cast<float*>(sst + S::kSOffCorr)[m] = c;
        if constexpr (DUMP) {
          int* sT = reinterpret_cast<int*>(sst + S::kSOffS);
          sT[0 * NA + m] = s4.x;
          sT[1 * NA + m] = s4.y;
          sT[2 * NA + m] = s4.z;
          sT[3 * NA + m] = s4.w;
        }
      }
      __syncwarp();
      int lok = 1;
      if (lane == 0) {
        mbar_arrive(s_full(ss));
        // this warp is done with the slice stage for block j; the last of the
        // slice's blocks reloads the stage
        const int in_slice = P * min(kBlocksPerSliceW, nb - (kb & ~(kBlocksPerSliceW - 1)));
        __threadfence_block();  // this warp's reads of the stage come before its count
        if (atomicAdd(&slice_cnt[q], 1) + 1 == in_slice) {
          slice_cnt[q] = 0;
          if (gsl + CS < total_sl) {
            fence_proxy_async_smem();  // the generic reads of the stage before the copies that overwrite it
            issue_slice(gsl + CS);
          }
        }
      }
      if (helper && lane == 0) {
        // the activation of this pair's next block j + B: its stage's previous
        // block j + B - BS was issued well before this block's MMAs
        if (b_issued == k + 1 && b_issued < my_blocks) {
          const int jn = j + S::kBlockWorkers;
          if (jn < BS || wait(b_empty(jn % BS), (uint32_t)((jn / BS - 1) & 1))) {
            issue_b(jn);
            ++b_issued;
          }
        }
      }
      if (leader && lane == 0) {
        // the block's MMAs, once its activation has landed and its slot is free
        const int bs = j % BS;
        const int pos = kb % S::kBlkPerSlot, u = ti * nslots + kb / S::kBlkPerSlot, cs = u & 1;
        if (P > 1) mbar_arrive(pair_done(w));  // after this warp's A writes and proxy fences
        lok = wait(b_full(bs), (uint32_t)((j / BS) & 1));
        if (lok && P > 1) lok = wait(pair_done(w), (uint32_t)(k & 1));  // the partner's half of A
        if (lok && u >= kSlots) lok = wait(d_free(cs), (uint32_t)(((u >> 1) - 1) & 1));
        if (lok) {
          tc_fence_after();
          const uint32_t dt = tmem_base + cs * kSlotCols + pos * kSteps * NA;
          // the block's 4 regions = kBias
          mma_i8<S::kIdescBias>(dt, smem_desc_noswz(sbase + S::kOffBiasA), smem_desc_noswz(sbase + S::kOffBiasB), 0u);
          const uint64_t ad = smem_desc_sw128(sbase + S::kOffA + sa * kABytes);
          const uint64_t bd = smem_desc_sw128(sbase + S::kOffB + bs * S::kBBytes);
#pragma unroll
          for (int ks = 0; ks < kSteps; ++ks)
            mma_i8<S::kIdesc>(dt + ks * NA, ad + (ks * 32 >> 4), bd + (ks * 32 >> 4), 1u);
          mma_commit(a_empty(sa));  // A and B of this block are free once its MMAs finish
          mma_commit(b_empty(bs));
          // one commit per block of the slot; the last block of a partial slot also commits for the missing ones
          const int reps = kb == nb - 1 ? S::kBlkPerSlot - pos : 1;
          for (int r = 0; r < reps; ++r) mma_commit(mma_done(cs));
        }
      }
      if (!leader && lane == 0) {  // after this warp's A writes and proxy fences; then the leader's
        mbar_arrive(pair_done(w));
        lok = wait(pair_done(w), (uint32_t)(k & 1));
      }
      ok = __shfl_sync(0xffffffffu, lok, 0) != 0;
    }
    if (lane == 0) {
      mma_commit(final_bar);  // completes (with the other workers') when every MMA issued above has finished
      mbar_wait_bounded(final_bar, 0, kWaitNs);
      if (*abort_flag) {  // leave no copy in flight into this CTA's shared memory (bounded)
        for (int c = max(0, b_issued - 2); helper && c < b_issued; ++c) {
          const int jc = w + c * S::kBlockWorkers;
          mbar_wait_bounded(b_full(jc % BS), (uint32_t)((jc / BS) & 1), kWaitNs / 10);
        }
        if (warp == 0)
          for (int c = max(0, *slices_issued - CS); c < *slices_issued; ++c)
            mbar_wait_bounded(c_full(c % CS), (uint32_t)((c / CS) & 1), kWaitNs / 10);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Warp (q, j): TMEM lanes q*32.. (weight rows), column group cg of every
    // step (16 activation rows), blocks blk0, blk0 + kBlkStep, ... of every
    // slot (their sums collect in the same accumulators).
    constexpr int kBlkStep = (S::kEpiWarps / 4) / S::kNcg;  // warps of one (quarter, column group)
    const int we = warp - S::kEpiWarp0;
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int cg = (we >> 2) % S::kNcg, blk0 = (we >> 2) / S::kNcg;
    const int n = q * 32 + lane;      // weight row of the tile
    const bool live = cg * 16 < p.M;  // some of this warp's activation rows exist
    float* stg = reinterpret_cast<float*>(smem + S::kOffStg);
    // x = fma(P * 2^-149, 2^110, -2^-26) = (P - 8192) * 2^-39 exactly: P's bits
    // read as fp32 are the denormal P * 2^-149, the product is exact and so is
    // the sum, an integer below 2^14 times 2^-39
    const float2 k110 = make_float2(0x1p110f, 0x1p110f), nbias = make_float2(-0x1p-26f, -0x1p-26f);
    pdl_wait();  // y is read (BTF_ADD) and written below
    int u = 0, git = 0;  // TMEM slot uses; this tile's first block in the CTA's block sequence
    bool ok = true;
    for (int ti = 0; ti < my_tiles; ++ti, git += nb) {
      const int n0 = ((int)blockIdx.x + ti * (int)gridDim.x) * kTileW;
      float2 acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = make_float2(0.f, 0.f);
      for (int su = 0; su < nslots; ++su, ++u) {
        const int cs = u & 1;
        if (ok) ok = wwait_sleep(mma_done(cs), (uint32_t)(u >> 1) & 1u);
        tc_fence_after();
#pragma unroll 1
        for (int blk = blk0; blk < S::kBlkPerSlot && ok; blk += kBlkStep) {
          const int kb = su * S::kBlkPerSlot + blk;
          if (kb >= nb) break;  // the last slot of a tile may hold fewer blocks
          const int gb = git + kb, ss = gb & (SS - 1);
          if (!wwait(s_full(ss), (uint32_t)(gb / SS) & 1u)) {
            ok = false;
            break;
          }
          if (live) {
            const uint32_t tl = tmem_base + ((uint32_t)(q * 32) << 16) + cs * kSlotCols + blk * kSteps * NA + cg * 16;
            const float4* dp = reinterpret_cast<const float4*>(sstage(ss) + S::kSOffD) + cg * 4;  // d [step][row]
            uint32_t buf[2][16];
            float2 tsum[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) tsum[i] = make_float2(0.f, 0.f);
            tmem_ld16_async(tl, buf[0]);
#pragma unroll
            for (int ks = 0; ks < kSteps; ++ks) {
              tmem_wait16(buf[ks & 1]);
              if (ks + 1 < kSteps) tmem_ld16_async(tl + (ks + 1) * NA, buf[(ks + 1) & 1]);  // in flight during the math
              const uint32_t* P = buf[ks & 1];
              if constexpr (DUMP) {  // integer accumulators only: idot = P - kBias - s, no y
                if (n0 + n < p.N) {
                  const int* sT = reinterpret_cast<const int*>(sstage(ss) + S::kSOffS) + ks * NA + cg * 16;
                  const int64_t mstride = (int64_t)p.N * (p.K >> 5);
                  int32_t* out = p.idot + (int64_t)(n0 + n) * (p.K >> 5) + kb * kSteps + ks + cg * 16 * mstride;
#pragma unroll
                  for (int i = 0; i < 16; ++i, out += mstride)
                    if (cg * 16 + i < p.M) *out = (int)P[i] - kBias - sT[i];
                }
              } else {
#pragma unroll
                for (int v = 0; v < 4; ++v) {  // activation rows 4v .. 4v+3 of the column group
                  const float4 d4 = dp[ks * (NA / 4) + v];
                  const float2 x0 = __ffma2_rn(
                      make_float2(__uint_as_float(P[4 * v]), __uint_as_float(P[4 * v + 1])), k110, nbias);
                  const float2 x1 = __ffma2_rn(
                      make_float2(__uint_as_float(P[4 * v + 2]), __uint_as_float(P[4 * v + 3])), k110, nbias);
                  tsum[2 * v] = __ffma2_rn(make_float2(d4.x, d4.y), x0, tsum[2 * v]);
                  tsum[2 * v + 1] = __ffma2_rn(make_float2(d4.z, d4.w), x1, tsum[2 * v + 1]);
                }
              }
            }
            if constexpr (!DUMP) {
              // the block sum less the code-sum correction, times the weight scale
              const float4* cp = reinterpret_cast<const float4*>(sstage(ss) + S::kSOffCorr) + cg * 4;
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                const float4 c4 = cp[v];
                tsum[2 * v] = __fadd2_rn(tsum[2 * v], make_float2(c4.x, c4.y));
                tsum[2 * v + 1] = __fadd2_rn(tsum[2 * v + 1], make_float2(c4.z, c4.w));
              }
              const float w = reinterpret_cast<const float*>(sstage(ss))[n];
#pragma unroll
              for (int i = 0; i < 8; ++i) acc[i] = __ffma2_rn(make_float2(w, w), tsum[i], acc[i]);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(s_empty(ss));
        }
        if (!ok) continue;
        // this warp's reads of the slot are done
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(d_free(cs));
      }
      // End of tile: the per-warp sums of a column group are added in blk0
      // order through shared memory; every epilogue warp reaches each barrier.
#pragma unroll 1
      for (int r = 1; r < kBlkStep; ++r) {
#pragma unroll 1
        for (int c = 0; c < S::kNcg; ++c) {
          if (blk0 == r && cg == c) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              stg[(2 * i) * kTileW + n] = acc[i].x;
              stg[(2 * i + 1) * kTileW + n] = acc[i].y;
            }
          }
          asm volatile("bar.sync 1, %0;" ::"r"(S::kEpiWarps * 32) : "memory");
          if (blk0 == 0 && cg == c) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              acc[i].x += stg[(2 * i) * kTileW + n];
              acc[i].y += stg[(2 * i + 1) * kTileW + n];
            }
          }
          asm volatile("bar.sync 1, %0;" ::"r"(S::kEpiWarps * 32) : "memory");
        }
      }
      if (GATHER && blk0 == 0 && live && ok && !*abort_flag && n0 + n < p.N) {
        // every rank's copy: one single-copy-atomic 64-bit word per output
        const unsigned long long tag = (unsigned long long)(*p.epoch * 1024u + (unsigned)p.site) << 32;
        const int64_t idx0 = (int64_t)(cg * 16) * p.ldy + n0 + n;
        const int mrows = min(16, p.M - cg * 16);
#pragma unroll 1
        for (int r = 0; r < p.world; ++r) {
          unsigned long long* dst = p.peer[r] + idx0;
#pragma unroll
          for (int i = 0; i < 16; ++i, dst += p.ldy) {
            const float v = (i & 1) ? acc[i >> 1].y : acc[i >> 1].x;
            if (i < mrows) *dst = (unsigned long long)__float_as_uint(v) | tag;
          }
        }
      } else if (!DUMP && !GATHER && blk0 == 0 && live && ok && !*abort_flag && n0 + n < p.N) {
        // a warp's 32 lanes store 32 consecutive floats of one row
        float* dst = p.y + (int64_t)(cg * 16) * p.ldy + n0 + n;
        const int mrows = min(16, p.M - cg * 16);
        const bool add = p.mode == BTF_ADD;
#pragma unroll
        for (int i = 0; i < 16; ++i, dst += p.ldy) {
          const float v = (i & 1) ? acc[i >> 1].y : acc[i >> 1].x;
          if (i < mrows) *dst = add ? *dst + v : v;
          if ((i & 3) == 3) asm volatile("" ::: "memory");  // at most 4 reads of y in flight: the register budget
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"((uint32_t)kTmemCols)
                 : "memory");
  }
  stamp_end(p.stamp);
}

template <int NA>
cudaError_t launch_wm(dim3 grid, cudaStream_t st, const CUtensorMap& mB, const CUtensorMap& mD,
                      const CUtensorMap& mS, const WmParams& p) {
  constexpr size_t smem = (size_t)Shape<NA>::kSmemBytes;
  constexpr int threads = Shape<NA>::kThreads;
  if (p.world > 0) return launch_pdl(gemm_wm_kernel<NA, false, true>, grid, dim3(threads), smem, st, mB, mD, mS, p);
  return p.idot ? launch_pdl(gemm_wm_kernel<NA, true>, grid, dim3(threads), smem, st, mB, mD, mS, p)
                : launch_pdl(gemm_wm_kernel<NA, false>, grid, dim3(threads), smem, st, mB, mD, mS, p);
}

template <int NA>
cudaError_t set_smem() {
  cudaError_t e = cudaFuncSetAttribute(gemm_wm_kernel<NA, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       Shape<NA>::kSmemBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_wm_kernel<NA, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Shape<NA>::kSmemBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_wm_kernel<NA, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Shape<NA>::kSmemBytes);
  return e;
}

}  // namespace

int gemm_wm_setup(DeviceInfo& d) {
  constexpr int need = std::max(Shape<16>::kSmemBytes, std::max(Shape<32>::kSmemBytes, Shape<64>::kSmemBytes));
  if (d.optin_smem < need) return fail(BTF_ERR_UNSUPPORTED, "btf_gemm_wm needs %d B of shared memory", need);
  cudaError_t e = set_smem<16>();
  if (e == cudaSuccess) e = set_smem<32>();
  if (e == cudaSuccess) e = set_smem<64>();
  return e == cudaSuccess ? BTF_OK : cuda_fail(e, "cudaFuncSetAttribute(gemm_wm_kernel)");
}

// Dispatch rule of btf_gemv / btf_gemm: the weight-major kernel serves
// 9 <= M <= 64 (below that the GEMV passes read the weights once or twice and
// are faster) when a segment has enough 128-row tiles to fill most SMs; it also
// needs the block sums s 16-byte aligned (tensor-map base).
bool wm_serves(const btf_gemv_seg& seg, int M, const btf_q8act& act) {
  const DeviceInfo* dev = current_device();
  return dev && M >= kWmMinM && M <= kWmMaxM && act.s && (reinterpret_cast<uintptr_t>(act.s) & 15) == 0 &&
         (seg.N + kTileW - 1) / kTileW >= dev->sm_count * 2 / 3;
}

// One matrix, 1 <= M <= kWmMaxM: y[M][ldy] (=|+=) W q with the weight rows on
// the MMA's 128-row side. idot != nullptr runs the dump form instead; g != null
// (tagged, store mode) stores segment `gseg` into every rank's buffer.
int run_gemm_wm(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act, int mode, cudaStream_t st,
                int32_t* idot, const btf_gather* g, int gseg) {
  const DeviceInfo* dev = current_device();
  if (!dev) return BTF_ERR_STATE;
  const EncodeFn enc = encode_fn();
  if (!enc) return fail(BTF_ERR_CUDA, "btf_gemm_wm: cuTensorMapEncodeTiled unavailable");
  auto encode = [&](CUtensorMap* map, CUtensorMapDataType type, const void* base, const cuuint64_t* dims,
                    const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle swz,
                    const char* what) -> int {
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = enc(map, type, 2u, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? BTF_OK : fail(BTF_ERR_ARG, "btf_gemm_wm: %s tensor map encoding failed (%d)", what, (int)r);
  };
  const int NA = M <= 16 ? 16 : M <= 32 ? 32 : 64;
  CUtensorMap mB, mD, mS;
  {  // activation: int8 [M][K], box 128 columns x NA rows, 128B swizzle; rows beyond M read as zero
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)K};
    const cuuint32_t box[2] = {(cuuint32_t)kChunk, (cuuint32_t)NA};
    if (int rc = encode(&mB, CU_TENSOR_MAP_DATA_TYPE_UINT8, act.q, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                        "activation"))
      return rc;
  }
  {  // activation block scales d (fp32) and sums s (int32), [M][K/32] each: box 32 blocks (one slice) x NA
     // rows, 128B swizzle (a block's 4 values are one 16-byte chunk, spread over the banks by the row);
     // columns past K and rows past M read as zero
    const cuuint64_t dims[2] = {(cuuint64_t)(K / 32), (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)(K / 32) * 4};
    const cuuint32_t box[2] = {32u, (cuuint32_t)NA};
    if (int rc = encode(&mD, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, act.d, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                        "activation scale"))
      return rc;
    if (int rc = encode(&mS, CU_TENSOR_MAP_DATA_TYPE_INT32, act.s, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B,
                        "activation sum"))
      return rc;
  }
  WmParams p{};
  p.N = seg.N;
  p.M = M;
  p.K = K;
  p.ntiles = (seg.N + kTileW - 1) / kTileW;
  p.nslices = (int)slices_of(K);
  p.ngroups = (int)groups_of(seg.N);
  p.panels = static_cast<const uint8_t*>(seg.panels);
  p.y = seg.y;
  p.ldy = seg.ldy;
  p.mode = mode;
  p.err = dev->err_word;
  p.idot = idot;
  p.stamp = take_stamp();
  if (g) {
    p.world = g->world;
    for (int r = 0; r < g->world; ++r) p.peer[r] = reinterpret_cast<unsigned long long*>(g->peer_y[gseg][r]);
    p.epoch = g->epoch;
    p.site = g->site;
  }
  const dim3 grid(std::min(p.ntiles, dev->sm_count));
  const cudaError_t e = NA == 16   ? launch_wm<16>(grid, st, mB, mD, mS, p)
                        : NA == 32 ? launch_wm<32>(grid, st, mB, mD, mS, p)
                                   : launch_wm<64>(grid, st, mB, mD, mS, p);
  return e == cudaSuccess ? launch_status("gemm_wm_kernel") : cuda_fail(e, "gemm_wm_kernel launch");
}

}  // namespace btf

using namespace btf;

extern "C" int btf_gemm_wm(const btf_gemv_seg* segs, int nseg, int K, int M, btf_q8act act, int mode, void* stream) {
  if (M <= 0) return BTF_OK;
  if (M > kWmMaxM) return fail(BTF_ERR_ARG, "btf_gemm_wm: M must be at most %d (M=%d); use btf_gemm", kWmMaxM, M);
  if (!segs || nseg < 1 || nseg > 3) return fail(BTF_ERR_ARG, "btf_gemm_wm: 1..3 segments (got %d)", nseg);
  if (mode != BTF_STORE && mode != BTF_ADD) return fail(BTF_ERR_ARG, "btf_gemm_wm: mode must be BTF_STORE or BTF_ADD");
  if (K <= 0 || K % 128) return fail(BTF_ERR_ARG, "btf_gemm_wm: K must be a positive multiple of 128 (K=%d)", K);
  if (!act.q || !act.d || !act.s || (reinterpret_cast<uintptr_t>(act.q) & 15) ||
      (reinterpret_cast<uintptr_t>(act.d) & 15) || (reinterpret_cast<uintptr_t>(act.s) & 15))
    return fail(BTF_ERR_ARG, "btf_gemm_wm: q, d and s must be 16-byte aligned");
  for (int i = 0; i < nseg; ++i) {
    if (!segs[i].panels || (reinterpret_cast<uintptr_t>(segs[i].panels) & 15) || segs[i].N <= 0 || !segs[i].y ||
        segs[i].ldy < segs[i].N)
      return fail(BTF_ERR_ARG, "btf_gemm_wm: segment %d has a bad panel buffer, N, y or ldy", i);
  }
  for (int i = 0; i < nseg; ++i)
    if (int rc = run_gemm_wm(segs[i], K, M, act, mode, (cudaStream_t)stream, nullptr, nullptr, 0)) return rc;
  return BTF_OK;
}

extern "C" int btf_gemm_wm_idot(const void* panels, int N, int K, int M, btf_q8act act, int32_t* idot,
                                void* stream) {
  if (M <= 0) return BTF_OK;
  if (M > kWmMaxM || !panels || (reinterpret_cast<uintptr_t>(panels) & 15) || N <= 0 || K <= 0 || K % 128 || !idot ||
      !act.q || !act.d || !act.s || (reinterpret_cast<uintptr_t>(act.q) & 15) ||
      (reinterpret_cast<uintptr_t>(act.d) & 15) || (reinterpret_cast<uintptr_t>(act.s) & 15))
    return fail(BTF_ERR_ARG, "btf_gemm_wm_idot: bad arguments (M <= %d, K %% 128, q, d, s 16-byte aligned)", kWmMaxM);
  const btf_gemv_seg seg{panels, N, nullptr, N};
  return run_gemm_wm(seg, K, M, act, BTF_STORE, (cudaStream_t)stream, idot, nullptr, 0);
}
