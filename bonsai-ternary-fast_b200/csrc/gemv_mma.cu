// Small-batch ternary GEMM on warp-level int8 MMA (mma.sync m16n8k32), for
// 1 <= M <= 16 activation rows and K <= 8192 against the resident panels.
//
// Same contract as the GEMV and the weight-major GEMM (one segment per launch):
//   y[m][r] {=, +=} sum_b  scale[r][b/4] * d[m][b] * idot[m][r][b],
// idot the exact int32 dot of the trits of row r and the Q8 values q[m] over
// 32-column block b (the reference's launch_gemv for NB rows,
// src/cuda/kernels.cu:211-334, :776-822; exact integer per block as in its
// emulator, src/emu_decoder.cpp:143-165).
//
// Why a warp MMA here: at M <= 16 the per-block work after the integer dot (one
// fp32 scale per (row, activation row, 32-column block)) is as large as the
// MMA itself, and the tcgen05 weight-major kernel pays for a shared-memory code
// expansion and a TMEM read-back per block with one serial chain per worker.
// The warp MMA takes its A operand from registers, so the 2-bit codes go from
// the staged panel bytes into the fragment with one AND each, and the integer
// result lands in registers for the epilogue.
//
// Data flow:
//   - the CTA's prologue copies the M activation rows (zero rows up to 16) into
//     shared memory with a 32-byte row pad, and builds two small tables: d
//     transposed to [block][row], and per 128 columns the code-sum correction
//     -sum d * s * 2^-39 of each row;
//   - a unit is 32 weight rows (four 8-row panels) x all K; each of the 8 warps
//     streams its own units in stages of 512 columns: its lanes copy the stage's
//     16 code half-regions (256 bytes; row quad h, 16-column half v of each
//     panel) and 4 scale blocks into the warp's ring with 16-byte cp.async
//     copies, one commit group per stage, the first stages before
//     griddepcontrol.wait (the weights do not depend on the previous kernel).
//     The half-regions land 272 bytes apart and the scale blocks 80, so the
//     fragment loads below hit distinct banks. (One TMA bulk copy per
//     half-region streamed at only ~3 TB/s: the copy engine's per-copy cost
//     bounds copies this small.);
//   - the MMA's 16 A rows of a thread are two rows of one row quad (quad g =
//     lane / 4 holds weight rows 4g .. 4g+3): m-tile 0 takes rows 4g (fragment
//     row g) and 4g+1 (row g+8), m-tile 1 rows 4g+2 and 4g+3. Inside a
//     32-column block the K positions are permuted, identically for A and B:
//     positions 4t .. 4t+3 and 16+4t .. 16+4t+3 of thread t = lane % 4 are
//     columns 8t .. 8t+7, so one 8-byte shared load gives a thread its codes for
//     all four rows and another its activation bytes of one row;
//   - the codes of row k sit at bits 2k of each byte, so code word AND
//     (0x03030303 << 2k) is 4^k c (c = trit + 1 in {0, 1, 2}; at most 128, an
//     unsigned A byte). With the accumulator input 2^20 the MMA returns
//     P = 4^k (idot + s) + 2^20 in (2^19, 2^21) (s = the block's sum of q);
//   - epilogue per value: x = fma(P * 2^-149, 2^110, -2^-19)
//     = 4^k (idot + s) * 2^-39 exactly (P's bits read as fp32 are the denormal
//     P * 2^-149; the product is exact, and so is the sum, an integer below
//     2^21 times 2^-39); per block T = fma(d, x, T); per 128 columns
//     acc = fma(scale 2^39 4^-k, T, acc) and acc = fma(scale 2^39, corr, acc)
//     (the powers of two are exact). Packed f32x2 FMAs, two activation rows per
//     instruction.
#include <algorithm>

#include "common.cuh"

namespace btf {
namespace {

#ifndef BTF_MMA_WARPS
#define BTF_MMA_WARPS 8
#endif
constexpr int kMmWarps = BTF_MMA_WARPS;
constexpr int kMmThreads = kMmWarps * 32;
constexpr int kMmPanels = 4;                                       // panels (8 rows each) of a unit
constexpr int kMmRegion = 272;                                     // pitch of a 256-byte code half-region
constexpr int kMmScalePitch = 80;                                  // pitch of a 64-byte scale block
constexpr int kMmScaleOff = 16 * kMmRegion;                        // 4352
constexpr int kMmStage = kMmScaleOff + kMmPanels * kMmScalePitch;  // 4672: 32 rows x 512 columns
constexpr int kMmMaxDepth = 4;
constexpr int kMmBarBytes = 512;  // the activation copy's barrier (last 8 bytes)
constexpr int kMmRowPad = 32;     // activation row pitch K + 32 bytes
constexpr int kMmMaxM = 16;
constexpr int kMmMinM = 3;  // btf_gemv / btf_gemm route calls of 3 <= M <= 16 here (mma_serves)
constexpr int kMmMaxK = 8192;
constexpr uint64_t kMmWaitNs = 1000000000ull;
constexpr int kMmBias = 1 << 20;
static_assert(kMmRegion % 16 == 0 && kMmScalePitch % 16 == 0 && kMmStage % 16 == 0, "bulk copy alignment");

// shared memory of a launch: ring, barriers, activation rows, d table, correction table
__host__ __device__ constexpr int mm_ring_bytes(int depth) { return kMmWarps * depth * kMmStage; }
__host__ __device__ constexpr int mm_act_off(int depth) { return mm_ring_bytes(depth) + kMmBarBytes; }
__host__ __device__ constexpr int mm_dt_off(int depth, int K) { return mm_act_off(depth) + 16 * (K + kMmRowPad); }
__host__ __device__ constexpr int mm_ct_off(int depth, int K) { return mm_dt_off(depth, K) + 16 * 4 * (K / 32); }
__host__ __device__ constexpr int mm_smem(int depth, int K) { return mm_ct_off(depth, K) + 16 * 4 * (K / 128); }

struct MmParams {
  const uint8_t* panels;
  float* y;
  int ldy, N, K, M, mode, depth;
  int ngroups, nhalves, nunits;  // 8-row groups, 512-column stages per unit, 32-row units
  const int8_t* q;
  const float* d;
  const int32_t* s;
  int32_t* idot;  // dump form: idot[m][n][K/32], no y
  int* err;
  unsigned long long* stamp;
  // GATHER form (tagged N-sharded store): every output goes to all `world`
  // ranks' buffers as a 64-bit word (fp32 bits | tag << 32) at the same index
  // as y; tag = *epoch * 1024 + site
  int world;
  unsigned long long* peer[BTF_MAX_RANKS];
  const unsigned* epoch;
  int site;
};

// D = A (16 x 32, u8, row) * B (32 x 8, s8, col) + C (every element kMmBias), int32
__device__ __forceinline__ void mma_u8s8(int (&dd)[4], const uint32_t (&a)[4], uint2 b) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %10, %10, %10};"
      : "=r"(dd[0]), "=r"(dd[1]), "=r"(dd[2]), "=r"(dd[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "r"(kMmBias));
}

// 16-byte asynchronous global -> shared copy (L2 only), and its group fences
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// waits until at most n (0 .. kMmMaxDepth - 1) of this thread's groups are pending
__device__ __forceinline__ void cp_async_wait(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
  }
}

__device__ __forceinline__ uint2 ld8(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ float2 ld8f(const float* p) { return *reinterpret_cast<const float2*>(p); }

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 as_f2(int x, int y) { return make_float2(__int_as_float(x), __int_as_float(y)); }
__device__ __forceinline__ float h2f_bits(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

// x = fma(P * 2^-149, 2^110, -2^-19) = 4^k (idot + s) 2^-39 for row k of a
// quad; the 4^k is removed with the weight scale (see the header)
__device__ __forceinline__ float2 mm_x(int p0, int p1) {
  return ffma2(as_f2(p0, p1), make_float2(0x1p110f, 0x1p110f), make_float2(-0x1p-19f, -0x1p-19f));
}

// DUMP writes the exact idot of every (row, activation row, block) instead of
// y; GATHER stores tagged words into every rank's buffer (store mode).
template <bool DUMP, bool GATHER = false>
__global__ void __launch_bounds__(kMmThreads, 1) gemv_mma_kernel(const __grid_constant__ MmParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int depth = p.depth, K = p.K;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t ring = sbase + warp * depth * kMmStage;
  const int H = p.nhalves;
  const int W = gridDim.x * kMmWarps, wg = blockIdx.x * kMmWarps + warp;
  const int my_units = wg < p.nunits ? (p.nunits - wg + W - 1) / W : 0;
  const int items = my_units * H;  // (unit, 512-column stage) items of this warp, unit-major

  // Item `it` (unit wg + (it / H) W, columns 512 (it % H) ..) into `slot`, one
  // commit group per item: 16-byte copies, lane-strided over the stage's 16
  // code half-regions (row quad h, 16-column half v of each panel; 256 bytes)
  // and its 4 scale blocks (64 bytes); panels past the matrix are skipped.
  auto issue = [&](int it, int slot) {
    const int u = wg + (it / H) * W, j = it % H;
    const int np = min(kMmPanels, p.ngroups - kMmPanels * u);
    const uint32_t dst = ring + slot * kMmStage;
    const int64_t S = (p.nhalves + 1) >> 1;
    const uint8_t* pan0 = p.panels + panel_offset((int64_t)kMmPanels * u, j >> 1, S);
    const int64_t pstride = S * kPanelBytes;  // next 8-row group, same slice
    const int half = j & 1;
#pragma unroll
    for (int c = lane; c < 16 * 16 + kMmPanels * 4; c += 32) {
      if (c < 256) {
        const int r = c >> 4, ch = c & 15;
        if ((r >> 2) < np)
          cp_async16(dst + r * kMmRegion + ch * 16, pan0 + (r >> 2) * pstride + (r & 3) * 512 + half * 256 + ch * 16);
      } else {
        const int pi = (c - 256) >> 2, ch = c & 3;
        if (pi < np)
          cp_async16(dst + kMmScaleOff + pi * kMmScalePitch + ch * 16,
                     pan0 + pi * pstride + kCodeBytes + half * 64 + ch * 16);
      }
    }
    cp_async_commit();
  };

  const int pre = min(items, depth);
  for (int it = 0; it < pre; ++it) issue(it, it);  // the panels do not depend on the previous kernel
  pdl_launch_dependents();
  pdl_wait();  // q, d, s (and y in add mode) are written by earlier kernels

  // activation rows (bulk copies; zeros past M), d transposed to [block][row],
  // and the per-128-column correction -sum_steps d s 2^-39 of each row
  const int pitch = K + kMmRowPad, kb = K >> 5;
  uint8_t* qs = smem + mm_act_off(depth);
  float* dt = reinterpret_cast<float*>(smem + mm_dt_off(depth, K));
  float* ct = reinterpret_cast<float*>(smem + mm_ct_off(depth, K));
  const uint32_t act_bar = sbase + mm_ring_bytes(depth) + kMmBarBytes - 8;
  if (warp == 0) {
    if (lane == 0) {
      mbar_init(act_bar, 1);
      fence_mbar_init();
      mbar_expect_tx(act_bar, (uint32_t)(p.M * K));
    }
    __syncwarp();
    if (lane < p.M) bulk_g2s(smem_u32(qs + lane * pitch), p.q + (size_t)lane * K, (uint32_t)K, act_bar);
  }
  for (int i = threadIdx.x; i < (16 - p.M) * (K >> 4); i += kMmThreads) {
    const int m = p.M + i / (K >> 4), c = i % (K >> 4);
    *reinterpret_cast<uint4*>(qs + m * pitch + 16 * c) = make_uint4(0u, 0u, 0u, 0u);
  }
#pragma unroll 2
  for (int i = threadIdx.x; i < 16 * (K >> 7); i += kMmThreads) {  // one row's 4 blocks of 32 columns
    const int m = i / (K >> 7), b4 = i % (K >> 7);
    float4 d4 = make_float4(0.f, 0.f, 0.f, 0.f);
    int4 s4 = make_int4(0, 0, 0, 0);
    if (m < p.M) {
      d4 = reinterpret_cast<const float4*>(p.d + (size_t)m * kb)[b4];
      s4 = reinterpret_cast<const int4*>(p.s + (size_t)m * kb)[b4];
    }
    dt[(4 * b4 + 0) * 16 + m] = d4.x;
    dt[(4 * b4 + 1) * 16 + m] = d4.y;
    dt[(4 * b4 + 2) * 16 + m] = d4.z;
    dt[(4 * b4 + 3) * 16 + m] = d4.w;
    float c = fmaf(d4.x * -0x1p-39f, (float)s4.x, 0.f);
    c = fmaf(d4.y * -0x1p-39f, (float)s4.y, c);
    c = fmaf(d4.z * -0x1p-39f, (float)s4.z, c);
    ct[b4 * 16 + m] = fmaf(d4.w * -0x1p-39f, (float)s4.w, c);
  }
  __syncthreads();  // the barrier's initialisation is visible to every warp
  // CTA-uniform: every warp either runs its items or, after a time-out, none
  const bool failed_act = __syncthreads_or(!mbar_wait_bounded(act_bar, 0u, kMmWaitNs)) != 0;
  if (failed_act && threadIdx.x == 0) atomicCAS(p.err, 0, kErrWaitTimeout);
  // the epoch is advanced in stream order: read after griddepcontrol.wait
  const unsigned long long tag = GATHER ? (unsigned long long)(*p.epoch * 1024u + (unsigned)p.site) << 32 : 0ull;

  const uint32_t M3 = 0x03030303u;
  const bool add = p.mode == BTF_ADD;
  const bool vec = ((reinterpret_cast<uintptr_t>(p.y) & 15) == 0) && (p.ldy & 3) == 0;
  const uint8_t* qrow0 = smem + mm_act_off(depth) + g * pitch + tig * 8;  // + 8 pitch for n-tile 1
  const float* dt0 = dt + 2 * tig;                                          // + 16 b + 8 nt
  const float* ct0 = ct + 2 * tig;                                          // + 16 gb + 8 nt
  const uint8_t* ringp = smem + warp * depth * kMmStage;
  float2 acc[4][2];  // [row 4g + k][n-tile]: (column 2t, column 2t + 1)
#pragma unroll
  for (int k = 0; k < 4; ++k) acc[k][0] = acc[k][1] = make_float2(0.f, 0.f);
  int slot = 0;
#pragma unroll 1
  for (int it = 0; it < (failed_act ? 0 : items); ++it) {
    const int j = it % H;
    const int u = wg + (it / H) * W;
    cp_async_wait(min(items - 1, it + depth - 1) - it);  // this item's group has landed
    __syncwarp();  // and every lane's copies of it are visible to the warp
    const uint8_t* st = ringp + slot * kMmStage;
    const uint8_t* code = st + (2 * g + (tig >> 1)) * kMmRegion + (tig & 1) * 8;  // + 16 per 32-column step
    const uint8_t* scl = st + kMmScaleOff + (g >> 1) * kMmScalePitch + (g & 1) * 8;  // + 16 per 128 columns
    const int nb = min(4, (K >> 7) - 4 * j);
#pragma unroll 1
    for (int bb = 0; bb < nb; ++bb) {
      const int gb = 4 * j + bb;  // 128-column block of the row
      // the block's 16 MMAs first (independent), then their epilogue
      uint2 cw[4], qv[4][2];
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        cw[ks] = ld8(code + (bb * 4 + ks) * 16);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) qv[ks][nt] = ld8(qrow0 + nt * 8 * pitch + gb * 128 + ks * 32);
      }
      int P[4][2][2][4];  // [step][n-tile][m-tile][fragment]
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        // m-tile 0: rows 4g (fragment row g) and 4g+1 (row g+8); m-tile 1: 4g+2, 4g+3
        const uint32_t a0[4] = {cw[ks].x & M3, cw[ks].x & (M3 << 2), cw[ks].y & M3, cw[ks].y & (M3 << 2)};
        const uint32_t a1[4] = {cw[ks].x & (M3 << 4), cw[ks].x & (M3 << 6), cw[ks].y & (M3 << 4),
                                cw[ks].y & (M3 << 6)};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          mma_u8s8(P[ks][nt][0], a0, qv[ks][nt]);
          mma_u8s8(P[ks][nt][1], a1, qv[ks][nt]);
        }
      }
      float2 T[4][2];
#pragma unroll
      for (int k = 0; k < 4; ++k) T[k][0] = T[k][1] = make_float2(0.f, 0.f);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const int(&d0)[4] = P[ks][nt][0];
          const int(&d1)[4] = P[ks][nt][1];
          if constexpr (DUMP) {
            const int r0 = 32 * u + 4 * g, blk = gb * 4 + ks;
            const int pv[4][2] = {{d0[0], d0[1]}, {d0[2], d0[3]}, {d1[0], d1[1]}, {d1[2], d1[3]}};
#pragma unroll
            for (int k = 0; k < 4; ++k)
#pragma unroll
              for (int c = 0; c < 2; ++c) {
                const int m = nt * 8 + 2 * tig + c;
                if (m < p.M && r0 + k < p.N)
                  p.idot[((int64_t)m * p.N + r0 + k) * kb + blk] =
                      ((pv[k][c] - kMmBias) >> (2 * k)) - p.s[(size_t)m * kb + blk];
              }
          } else {
            const float2 dv = ld8f(dt0 + (gb * 4 + ks) * 16 + nt * 8);
            T[0][nt] = ffma2(dv, mm_x(d0[0], d0[1]), T[0][nt]);
            T[1][nt] = ffma2(dv, mm_x(d0[2], d0[3]), T[1][nt]);
            T[2][nt] = ffma2(dv, mm_x(d1[0], d1[1]), T[2][nt]);
            T[3][nt] = ffma2(dv, mm_x(d1[2], d1[3]), T[3][nt]);
          }
        }
      }
      if constexpr (!DUMP) {
        const uint2 sc = ld8(scl + bb * 16);  // fp16 scales of rows 4g .. 4g+3, this block
        // T of row k holds 4^k times the block sum: acc += scale 2^39 4^-k T + scale 2^39 corr
        const float w[4] = {h2f_bits(sc.x & 0xffffu) * 0x1p39f, h2f_bits(sc.x >> 16) * 0x1p39f,
                            h2f_bits(sc.y & 0xffffu) * 0x1p39f, h2f_bits(sc.y >> 16) * 0x1p39f};
        const float wk[4] = {w[0], w[1] * 0x1p-2f, w[2] * 0x1p-4f, w[3] * 0x1p-6f};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const float2 cv = ld8f(ct0 + gb * 16 + nt * 8);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            acc[k][nt] = ffma2(make_float2(w[k], w[k]), cv,
                               ffma2(make_float2(wk[k], wk[k]), T[k][nt], acc[k][nt]));
        }
      }
    }
    __syncwarp();  // every lane's reads of the slot are done
    if (it + depth < items) issue(it + depth, slot);
    if (++slot == depth) slot = 0;
    if (j == H - 1) {  // the unit's last stage: rows 32u + 4g .. +3
      if constexpr (!DUMP) {
        const int r0 = 32 * u + 4 * g;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int m = nt * 8 + 2 * tig + c;
            if (m >= p.M) continue;
            float v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = c ? acc[k][nt].y : acc[k][nt].x;
            if constexpr (GATHER) {  // one single-copy-atomic 64-bit word per output and rank
              const int64_t idx = (int64_t)m * p.ldy + r0;
              unsigned long long wv[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) wv[k] = (unsigned long long)__float_as_uint(v[k]) | tag;
              for (int r = 0; r < p.world; ++r) {
                unsigned long long* dst = p.peer[r] + idx;
                if ((p.ldy & 3) == 0 && (reinterpret_cast<uintptr_t>(p.peer[r]) & 31) == 0 && r0 + 3 < p.N) {
                  // one 32-byte store of four words (each word single-copy atomic): the 8
                  // lanes of a row quad column write 256 contiguous bytes, whole sectors
                  asm volatile("st.global.v4.u64 [%0], {%1, %2, %3, %4};" ::"l"(dst), "l"(wv[0]), "l"(wv[1]),
                               "l"(wv[2]), "l"(wv[3])
                               : "memory");
                } else if ((p.ldy & 1) == 0 && (reinterpret_cast<uintptr_t>(p.peer[r]) & 15) == 0 && r0 + 3 < p.N) {
                  // two 16-byte stores of two words each (each word single-copy atomic): the 8
                  // lanes of a row quad column write 256 contiguous bytes per activation row
                  asm volatile("st.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(wv[0]), "l"(wv[1]) : "memory");
                  asm volatile("st.global.v2.u64 [%0], {%1, %2};" ::"l"(dst + 2), "l"(wv[2]), "l"(wv[3]) : "memory");
                } else {
#pragma unroll
                  for (int k = 0; k < 4; ++k)
                    if (r0 + k < p.N) dst[k] = wv[k];
                }
              }
              continue;
            }
            float* dst = p.y + (int64_t)m * p.ldy + r0;
            if (vec && r0 + 3 < p.N) {
              float4 o = make_float4(v[0], v[1], v[2], v[3]);
              if (add) {
                const float4 yo = *reinterpret_cast<const float4*>(dst);
                o = make_float4(yo.x + o.x, yo.y + o.y, yo.z + o.z, yo.w + o.w);
              }
              *reinterpret_cast<float4*>(dst) = o;
            } else {
#pragma unroll
              for (int k = 0; k < 4; ++k)
                if (r0 + k < p.N) dst[k] = add ? dst[k] + v[k] : v[k];
            }
          }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[k][0] = acc[k][1] = make_float2(0.f, 0.f);
    }
  }
  // leave no copy in flight into shared memory: this warp's skipped items
  // (after an activation time-out) and, bounded, the activation copy
  asm volatile("cp.async.wait_all;" ::: "memory");
  if (failed_act && threadIdx.x == 0) mbar_wait_bounded(act_bar, 0u, kMmWaitNs / 10);
  stamp_end(p.stamp);
}

}  // namespace

int gemv_mma_setup(DeviceInfo& d) {
  const int need = mm_smem(2, kMmMaxK);
  if (d.optin_smem < need) return fail(BTF_ERR_UNSUPPORTED, "btf_gemv_mma needs %d B of shared memory", need);
  cudaError_t e = cudaFuncSetAttribute(gemv_mma_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, need);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemv_mma_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, need);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemv_mma_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, need);
  return e == cudaSuccess ? BTF_OK : cuda_fail(e, "cudaFuncSetAttribute(gemv_mma_kernel)");
}

// Dispatch rule of btf_gemv / btf_gemm / btf_gemv_gather (K <= 8192; q, d
// and s 16-byte aligned), from B200 timings at K = 5120 against the other
// kernels on the same call:
//   - 9 <= M <= 16: from (SM count) 32-row units on (the weight-major tcgen05
//     kernel was slower at every N measured, 5120 to 248320 rows, e.g. 23
//     against 26 us at 17408; on fewer units the GEMV passes are faster);
//   - 5 <= M <= 8: from 2 x (SM count) 32-row units on (two 4-row GEMV passes
//     are faster on smaller matrices: 17 against 23 us at 6144 rows);
//   - 3 <= M <= 4: from 8 x (SM count) units on (one GEMV pass is faster on
//     smaller matrices). M = 1 and 2 stay on the GEMV.
// A warp's one unit takes ~21 us at K = 5120, which bounds small matrices.
bool mma_serves(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act) {
  const DeviceInfo* dev = current_device();
  if (!dev || M < kMmMinM || M > kMmMaxM || K <= 0 || K % 128 != 0 || K > kMmMaxK || !act.q || !act.d || !act.s ||
      (reinterpret_cast<uintptr_t>(act.q) & 15) || (reinterpret_cast<uintptr_t>(act.d) & 15) ||
      (reinterpret_cast<uintptr_t>(act.s) & 15))
    return false;
  const int64_t units = (groups_of(seg.N) + kMmPanels - 1) / kMmPanels;
  if (M >= 9) return units >= dev->sm_count;
  if (M >= 5) return units >= 2 * dev->sm_count;
  return units >= (int64_t)dev->sm_count * kMmWarps;
}

// Two passes of 16 rows for 17 <= M <= 32 over lm_head-size matrices (at least
// 8 x (SM count) 32-row units per segment): each pass streams the weights once
// more, and the two still beat the weight-major kernel's one pass (lm_head,
// K = 5120, M = 32: 275 against 375 us; 37888 rows: 47 against 60 us).
bool mma_two_pass_serves(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act) {
  const DeviceInfo* dev = current_device();
  return dev && M > kMmMaxM && M <= 2 * kMmMaxM && mma_serves(seg, K, kMmMaxM, act) &&
         (groups_of(seg.N) + kMmPanels - 1) / kMmPanels >= (int64_t)dev->sm_count * kMmWarps;
}

// One segment, 1 <= M <= kMmMaxM, K <= kMmMaxK; idot != nullptr runs the dump
// form; g != null (tagged, store mode) stores segment `gseg` into every rank's buffer.
int run_gemv_mma(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act, int mode, cudaStream_t st,
                 int32_t* idot, const btf_gather* g, int gseg) {
  const DeviceInfo* dev = current_device();
  if (!dev) return BTF_ERR_STATE;
  MmParams p{};
  p.panels = static_cast<const uint8_t*>(seg.panels);
  p.y = seg.y;
  p.ldy = seg.ldy;
  p.N = seg.N;
  p.K = K;
  p.M = M;
  p.mode = mode;
  p.ngroups = (int)groups_of(seg.N);
  p.nhalves = (K + 511) / 512;
  p.nunits = (p.ngroups + kMmPanels - 1) / kMmPanels;
  p.q = act.q;
  p.d = act.d;
  p.s = act.s;
  p.idot = idot;
  p.err = dev->err_word;
  p.stamp = take_stamp();
  if (g) {
    p.world = g->world;
    for (int r = 0; r < g->world; ++r) p.peer[r] = reinterpret_cast<unsigned long long*>(g->peer_y[gseg][r]);
    p.epoch = g->epoch;
    p.site = g->site;
  }
  // the deepest ring that fits beside this K's activation tables
  const int limit = mm_smem(2, kMmMaxK);
  p.depth = 2;
  while (p.depth < kMmMaxDepth && mm_smem(p.depth + 1, K) <= limit) ++p.depth;
  const size_t smem = (size_t)mm_smem(p.depth, K);
  const int grid = std::max(1, std::min(dev->sm_count, (p.nunits + kMmWarps - 1) / kMmWarps));
  const cudaError_t e = idot ? launch_pdl(gemv_mma_kernel<true>, dim3(grid), dim3(kMmThreads), smem, st, p)
                        : g    ? launch_pdl(gemv_mma_kernel<false, true>, dim3(grid), dim3(kMmThreads), smem, st, p)
                               : launch_pdl(gemv_mma_kernel<false>, dim3(grid), dim3(kMmThreads), smem, st, p);
  return e == cudaSuccess ? launch_status("gemv_mma_kernel") : cuda_fail(e, "gemv_mma_kernel launch");
}

// Rows m0 .. m0 + M of the activation through run_gemv_mma (row views of the
// Q8 activation and of each segment's output; K % 128 == 0 keeps them 16-byte aligned).
int run_gemv_mma_rows(const btf_gemv_seg* segs, int nseg, int K, int m0, int M, const btf_q8act& act, int mode,
                      cudaStream_t st) {
  const btf_q8act sub{act.q + (size_t)m0 * K, act.d + (size_t)m0 * (K / 32), act.s + (size_t)m0 * (K / 32)};
  for (int i = 0; i < nseg; ++i) {
    btf_gemv_seg sg = segs[i];
    sg.y = segs[i].y + (size_t)m0 * segs[i].ldy;
    if (int rc = run_gemv_mma(sg, K, M, sub, mode, st, nullptr, nullptr, 0)) return rc;
  }
  return BTF_OK;
}

}  // namespace btf

using namespace btf;

namespace {
bool mma_args_ok(const btf_q8act& act, int K, int M) {
  return M <= kMmMaxM && K > 0 && K % 128 == 0 && K <= kMmMaxK && act.q && act.d && act.s &&
         (reinterpret_cast<uintptr_t>(act.q) & 15) == 0 && (reinterpret_cast<uintptr_t>(act.d) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(act.s) & 15) == 0;
}
}  // namespace

extern "C" int btf_gemv_mma(const btf_gemv_seg* segs, int nseg, int K, int M, btf_q8act act, int mode,
                            void* stream) {
  if (M <= 0) return BTF_OK;
  if (!mma_args_ok(act, K, M))
    return fail(BTF_ERR_ARG,
                "btf_gemv_mma: need M <= %d, K a positive multiple of 128 up to %d, q, d, s 16-byte aligned",
                kMmMaxM, kMmMaxK);
  if (!segs || nseg < 1 || nseg > 3) return fail(BTF_ERR_ARG, "btf_gemv_mma: 1..3 segments (got %d)", nseg);
  if (mode != BTF_STORE && mode != BTF_ADD) return fail(BTF_ERR_ARG, "btf_gemv_mma: mode must be BTF_STORE or BTF_ADD");
  for (int i = 0; i < nseg; ++i)
    if (!segs[i].panels || (reinterpret_cast<uintptr_t>(segs[i].panels) & 15) || segs[i].N <= 0 || !segs[i].y ||
        segs[i].ldy < segs[i].N)
      return fail(BTF_ERR_ARG, "btf_gemv_mma: segment %d has a bad panel buffer, N, y or ldy", i);
  for (int i = 0; i < nseg; ++i)
    if (int rc = run_gemv_mma(segs[i], K, M, act, mode, (cudaStream_t)stream, nullptr, nullptr, 0)) return rc;
  return BTF_OK;
}

extern "C" int btf_gemv_mma_idot(const void* panels, int N, int K, int M, btf_q8act act, int32_t* idot,
                                 void* stream) {
  if (M <= 0) return BTF_OK;
  if (!mma_args_ok(act, K, M) || !panels || (reinterpret_cast<uintptr_t>(panels) & 15) || N <= 0 || !idot)
    return fail(BTF_ERR_ARG, "btf_gemv_mma_idot: bad arguments (M <= %d, K %% 128 up to %d, q, d, s 16-byte aligned)",
                kMmMaxM, kMmMaxK);
  const btf_gemv_seg seg{panels, N, nullptr, N};
  return run_gemv_mma(seg, K, M, act, BTF_STORE, (cudaStream_t)stream, idot, nullptr, 0);
}
