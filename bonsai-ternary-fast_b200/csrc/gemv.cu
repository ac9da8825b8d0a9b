// Ternary GEMV / small-batch GEMM on the panel layout (CUDA cores, dp4a).
//
// Replaces gemv_kernel<NB, MODE> / launch_gemv of the reference
// (src/cuda/kernels.cu:211-334, :776-822). Same math per output row r and
// activation row m:
//   y[m][r] {=, +=} sum_s  (fp16 scale[r][s/4] * d[m][s]) * idot[m][r][s],
//   idot = sum over the 32 columns of sub-block s of trit * q  (exact int32),
// with the swiglu epilogue silu(gate) * up (kernels.cu:318-320).
//
// B200 design (not the reference's):
//   - persistent grid (one or two CTAs per SM); each CTA owns a contiguous,
//     balanced range of "units" (one 8-row group of a segment, all K; for
//     swiglu the gate and up groups of the same rows), so every SM streams
//     the same number of bytes;
//   - each of the 8 warps is its own producer: lane 0 keeps a ring of DEPTH
//     panels (2176 B, 8 rows x 1024 columns + scales; swiglu: gate + up)
//     filled by 1-D TMA bulk copies (cp.async.bulk, this CTA only) on an
//     mbarrier per slot; waits are bounded and report a device error word;
//   - programmatic dependent launch: the weight copies of the first DEPTH
//     panels are issued before griddepcontrol.wait, i.e. while the previous
//     kernel in the stream (quantiser or GEMV) is still finishing; the
//     activation is read only after the wait;
//   - the activation (Q8, or fp32 quantised in the prologue with the same
//     bit-exact rule as btf_quant_q8) sits in shared memory, split so that the
//     lane loads are bank-conflict free; lane l always handles sub-block l of
//     a slice, so its activation is loaded once per panel and reused for all
//     8 (16) rows;
//   - codes are stored row-interleaved (one 32-bit word = 4 rows x 4 columns,
//     row k in bits 2k..2k+1 of each byte): one AND with 0x03030303 << 2k gives
//     4^k x the codes of row k aligned with the int8x4 activation word, so each
//     (row, 4 columns) costs one LOP3 + one unsigned x signed dp4a, and the 4^k
//     is removed once per (row, sub-block) by an exact arithmetic shift;
//     -sum(q) and the int->float conversion are one biased add (kMagicInt);
//     the fp32 epilogue runs on row pairs with packed f32x2 FMA (sm_100).
#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemv_core.cuh"

namespace btf {
namespace {

// Launch shape (tuned on B200 by sweeping these; overridable at build time).
#ifndef BTF_GEMV_WARPS
#define BTF_GEMV_WARPS 8
#endif
#ifndef BTF_GEMV_SMEM_KB
#define BTF_GEMV_SMEM_KB 110
#endif
#ifndef BTF_GEMV_MAX_CTAS
#define BTF_GEMV_MAX_CTAS 2
#endif
#ifndef BTF_GEMV_MINB
#define BTF_GEMV_MINB 1
#endif
#ifndef BTF_GEMV_GRID_CTAS
#define BTF_GEMV_GRID_CTAS BTF_GEMV_MAX_CTAS
#endif
constexpr int kWarps = BTF_GEMV_WARPS;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxSeg = 3;
constexpr int kMaxNb = 4;                                  // activation rows per pass
constexpr int kGemmMinM = 64;                              // btf_gemv hands M >= this to btf_gemm
constexpr uint64_t kWaitLimitNs = 1000000000ull;           // 1 s per bounded wait
constexpr uint64_t kGatherWaitNs = 2000000000ull;          // 2 s for the other ranks' arrivals

constexpr size_t kSmemTarget = BTF_GEMV_SMEM_KB * 1024;    // ring + activation budget per CTA
constexpr int kGridCtasPerSm = BTF_GEMV_GRID_CTAS;         // persistent CTAs per SM launched (<= resident)
#ifndef BTF_GEMV_BALANCED
#define BTF_GEMV_BALANCED 1
#endif
constexpr bool kBalancedGrid = BTF_GEMV_BALANCED;

#ifndef BTF_GEMV_FUSE_CLUSTER
#define BTF_GEMV_FUSE_CLUSTER 4
#endif
// btf_gemv_f32: CTAs per cluster that share the quantisation of the activation
// (each quantises 1/kFuseCluster of it into every CTA's shared memory)
constexpr int kFuseCluster = BTF_GEMV_FUSE_CLUSTER;
#ifndef BTF_GEMV_RING_AFTER_STAGE
#define BTF_GEMV_RING_AFTER_STAGE 0
#endif
// cluster path: start the weight ring only once the activation is quantised
constexpr bool kRingAfterStage = BTF_GEMV_RING_AFTER_STAGE;
static_assert(kFuseCluster == 1 || kFuseCluster == 2 || kFuseCluster == 4 || kFuseCluster == 8, "cluster size");
#ifndef BTF_GEMV_PREWAIT
#define BTF_GEMV_PREWAIT 2
#endif
constexpr int kPrewaitPanels = BTF_GEMV_PREWAIT;           // panels per warp copied before griddepcontrol.wait
// 512-thread builds raised an illegal-address fault in the bench on B200 whose
// cause was not found (a CPU replay of every index stayed in bounds); only
// 128- and 256-thread CTAs are built.
static_assert(kWarps == 4 || kWarps == 8, "gemv_kernel is built with 4 or 8 warps per CTA");

struct GemvParams {
  const uint8_t* pan0;
  const uint8_t* pan1;
  const uint8_t* pan2;
  float* y0;
  float* y1;
  float* y2;
  int n0, n1, n2;
  int ld0, ld1, ld2;
  int u1, u2, utotal;  // cumulative unit (8-row group) counts of the segments
  int K, S, nsub;
  int m0, nb;          // activation rows m0 .. m0 + nb - 1 (nb <= NB)
  const int8_t* q;     // Q8 input (FUSE == false)
  const float* d;
  const int32_t* s;
  const float* x;      // fp32 input (FUSE == true)
  int ldx;
  int slots;           // ring slots of a CTA, shared by the warps that have work
  int* err;
  btf_gather gather;   // world == 0: plain launch; else the epilogue all-gathers over NVLink
  unsigned long long* stamp;  // end stamp slot (btf_stamp_next) or null
  int32_t* idot;              // DUMP kernels: [M][n0][K/32] integer dots of segment 0 (no y is stored)
};

using namespace core;

// Shared-memory layout (bytes), identical on host and device.
struct SmemPlan {
  int stage, ring, bars, act, pieces, total;
  __host__ __device__ SmemPlan(int mode, int nb, int S, int slots) {
    stage = (mode == BTF_SWIGLU ? 2 : 1) * kPanelBytes;
    ring = slots * stage;
    bars = (slots * 8 + 15) / 16 * 16;  // keeps the uint4 activation arrays 16-byte aligned
    act = nb * S * kSubPerSlice * 40;  // qa 16 B + qb 16 B + d 4 B + magic_s 4 B per sub-block
    pieces = kWarps * kMaxNb * 16 * 4;  // per-warp partial row sums when units are split by slices
    total = ring + bars + act + pieces;
  }
};

// End of an N-sharded launch: once every CTA of this launch on this rank has
// made its stores to all ranks visible system-wide, the last one adds 1 to every
// rank's arrival counter and waits (bounded) until its own counter shows this
// launch's arrivals from all ranks. Arrivals of a rank's next launch can only
// come after that rank's wait for this one, so a cumulative count suffices.
__device__ __noinline__ void gather_arrive(const btf_gather& g, int* err) {
  // The CTA barrier orders every thread's output stores before thread 0's
  // acq_rel count below, and the last CTA's release-adds to the other ranks
  // (system scope) are ordered after all counts.
  __syncthreads();
  if (threadIdx.x != 0) return;
  unsigned prev;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(g.done) : "memory");
  if (prev != gridDim.x - 1) return;
  *g.done = 0;  // the next launch's CTAs touch it only after this launch completes
  // release.sys is cumulative: every CTA's stores, ordered before its acq_rel
  // count and so before this thread, are visible to whoever acquires the add
  for (int r = 0; r < g.world; ++r)
    asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(g.flags[r]) : "memory");
  const unsigned target = *g.expect + (unsigned)g.world;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(g.flags[g.rank]) : "memory");
    if ((int)(v - target) >= 0) break;
    if (globaltimer_ns() - t0 > kGatherWaitNs) {
      atomicCAS(err, 0, kErrWaitTimeout);
      break;
    }
  }
  *g.expect = target;
}

// GATHER: 0 = plain launch; 1 = N-sharded, counted completion; 2 = N-sharded,
// tagged (value, tag) words. Compile-time, so plain launches carry none of it.
// DUMP (parity/debug, store mode, one segment): the same kernel writes, for
// every (m, row, sub-block), the fp32 operand its epilogue multiplies
// ((float)idot from the biased integer) as int32 to p.idot, instead of y.
template <int NB, int MODE, bool FUSE, int GATHER, bool DUMP = false>
__global__ void __launch_bounds__(kThreads, BTF_GEMV_MINB) gemv_kernel(const __grid_constant__ GemvParams p) {
  constexpr bool kSwi = MODE == BTF_SWIGLU;
  constexpr bool kCluster = FUSE && kFuseCluster > 1;
  extern __shared__ __align__(128) uint8_t smem[];
  if constexpr (kCluster) cluster_arrive_relaxed();  // matched by the wait before the first remote store
  const int S = p.S;
  const int nsp = S * kSubPerSlice;  // sub-blocks incl. padding to whole slices
  const SmemPlan plan(MODE, NB, S, p.slots);
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + plan.ring);
  uint4* qa_s = reinterpret_cast<uint4*>(smem + plan.ring + plan.bars);
  uint4* qb_s = qa_s + NB * nsp;
  float* d_s = reinterpret_cast<float*>(qb_s + NB * nsp);
  int* ms_s = reinterpret_cast<int*>(d_s + NB * nsp);
  float* pieces = reinterpret_cast<float*>(smem + plan.ring + plan.bars + plan.act);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u_begin = (int)((int64_t)blockIdx.x * p.utotal / gridDim.x);
  const int u_end = (int)((int64_t)(blockIdx.x + 1) * p.utotal / gridDim.x);
  const int cta_units = u_end - u_begin;
  // With fewer units than warps, each unit is cut into G slice ranges handled
  // by G warps (partial sums combined in shared memory at the end); otherwise
  // warp w takes units u_begin + w, u_begin + w + kWarps, ...
  const int G = (cta_units > 0 && cta_units < kWarps) ? min(kWarps / cta_units, S) : 1;
  const int part = warp % G;
  const int first = u_begin + (G > 1 ? warp / G : warp);
  const int stride = G > 1 ? cta_units : kWarps;  // unit step between a warp's units
  const bool has_work = G > 1 ? warp < cta_units * G : first < u_end;
  const int j_lo = G > 1 ? part * S / G : 0, j_hi = G > 1 ? (part + 1) * S / G : S;
  const int n_units = !has_work ? 0 : G > 1 ? 1 : (u_end - first + kWarps - 1) / kWarps;
  const int n_panels = n_units * (j_hi - j_lo);
  // the ring is split among the warps that have work only, so a CTA with few
  // (long) units keeps proportionally more of each warp's panels in flight
  const int active = G > 1 ? cta_units * G : min(kWarps, cta_units);
  const int depth = active > 0 ? p.slots / active : p.slots;
  const uint32_t my_bars = smem_u32(bars + warp * depth);
  const uint32_t my_ring = smem_u32(ring + warp * depth * plan.stage);

  // unit -> (segment, row group)
  auto locate = [&](int u, int& seg, int& g) {
    seg = kSwi ? 0 : (u >= p.u1) + (u >= p.u2);
    g = u - (seg == 0 ? 0 : seg == 1 ? p.u1 : p.u2);
  };
  // Output store: this rank's buffer, or (N-sharded launch) every rank's
  // buffer over NVLink; the value is the same everywhere.
  // Tagged N-sharded launches store (value bits | tag << 32) as one 64-bit word
  // (single-copy atomic), so a reader that sees the tag also sees the value.
  unsigned tag = 0;  // set after griddepcontrol.wait (the epoch is advanced in stream order)
  auto put = [&](int seg, float* y, int64_t idx, float val) {
    if constexpr (DUMP) {
      return;
    } else if constexpr (GATHER == 0) {
      y[idx] = val;
    } else if constexpr (GATHER == 2) {
      const unsigned long long w = (unsigned long long)__float_as_uint(val) | ((unsigned long long)tag << 32);
      for (int r = 0; r < p.gather.world; ++r) reinterpret_cast<unsigned long long*>(p.gather.peer_y[seg][r])[idx] = w;
    } else {
      for (int r = 0; r < p.gather.world; ++r) p.gather.peer_y[seg][r][idx] = val;
    }
  };
  auto get = [&](const float* y, int64_t idx) -> float {  // current output (BTF_ADD)
    if constexpr (GATHER == 2) return __uint_as_float(reinterpret_cast<const unsigned*>(y)[2 * idx]);
    else return y[idx];
  };
  // Copy issue state (used by lane 0): next panel's unit, slice, slot and
  // source pointers. A unit's S panels are contiguous, so moving to the next
  // slice is a pointer bump; only a new unit needs locate().
  int is_ui = 0, is_j = j_lo, is_slot = 0, is_count = 0;
  const uint8_t* is_a = nullptr;
  const uint8_t* is_b = nullptr;
  auto unit_src = [&](int ui) {
    int seg, g;
    locate(first + ui * stride, seg, g);
    const int64_t off = ((int64_t)g * S + j_lo) * kPanelBytes;
    is_a = (seg == 0 ? p.pan0 : seg == 1 ? p.pan1 : p.pan2) + off;
    is_b = kSwi ? p.pan1 + off : nullptr;
  };
  auto issue_next = [&]() {  // lane 0: start the copies of the next panel, advance
    const uint32_t bar = my_bars + is_slot * 8, dst = my_ring + is_slot * plan.stage;
    mbar_expect_tx(bar, plan.stage);
    bulk_g2s(dst, is_a, kPanelBytes, bar);
    if (kSwi) bulk_g2s(dst + kPanelBytes, is_b, kPanelBytes, bar);
    ++is_count;
    if (++is_slot == depth) is_slot = 0;
    if (++is_j == j_hi) {
      is_j = j_lo;
      if (++is_ui < n_units) unit_src(is_ui);
    } else {
      is_a += kPanelBytes;
      if (kSwi) is_b += kPanelBytes;
    }
  };

  if (lane == 0 && n_panels > 0) {
    for (int i = 0; i < depth; ++i) mbar_init(my_bars + i * 8, 1);
    fence_mbar_init();
  }
  __syncwarp();
  pdl_launch_dependents();
  // Weights never depend on the previous kernel: before waiting for it, start
  // the copy of this warp's FIRST panel only. Every warp's first panel is thus
  // ahead of everyone's later panels in the memory queues, so all warps can
  // start computing early instead of some waiting behind a whole-ring burst.
  if (lane == 0 && n_panels > 0) {
    unit_src(0);
    issue_next();
    while (is_count < kPrewaitPanels && is_count < depth && is_count < n_panels) issue_next();
  }
  pdl_wait();
  if constexpr (GATHER == 2) tag = *p.gather.epoch * 1024u + (unsigned)p.gather.site;
  // Add mode: the current y of the rows a lane will write is loaded when their
  // unit starts, so the read-modify-write at the unit's end does not wait on
  // it (only the unit's owner writes those rows). G = 1: lanes 4r hold row r of
  // the warp's current unit (the reduce_rows8 map); G > 1: the combining lane
  // (row lane & 7, activation row lane >> 3) of the warp's unit.
  constexpr bool kPreY = MODE == BTF_ADD && !DUMP;
  float ypre[NB];
#pragma unroll
  for (int m = 0; m < NB; ++m) ypre[m] = 0.0f;
  auto prefetch_y = [&](int uix) {  // G = 1: unit first + uix * stride
    if (uix >= n_units || (lane & 3) != 0) return;
    int seg, g;
    locate(first + uix * stride, seg, g);
    const int n = seg == 0 ? p.n0 : seg == 1 ? p.n1 : p.n2;
    const int ldy = seg == 0 ? p.ld0 : seg == 1 ? p.ld1 : p.ld2;
    const float* y = seg == 0 ? p.y0 : seg == 1 ? p.y1 : p.y2;
    const int row = g * kRows + (lane >> 2);
#pragma unroll
    for (int m = 0; m < NB; ++m)
      if (row < n && m < p.nb) ypre[m] = get(y, (int64_t)(p.m0 + m) * ldy + row);
  };
  if constexpr (kPreY) {
    if (G == 1) {
      prefetch_y(0);
    } else if (has_work && part == 0) {
      int seg, g;
      locate(first, seg, g);
      const int n = seg == 0 ? p.n0 : seg == 1 ? p.n1 : p.n2;
      const int ldy = seg == 0 ? p.ld0 : seg == 1 ? p.ld1 : p.ld2;
      const float* y = seg == 0 ? p.y0 : seg == 1 ? p.y1 : p.y2;
      const int r = lane & 7, m = lane >> 3, row = g * kRows + r;
      if (m < NB && row < n && m < p.nb) ypre[0] = get(y, (int64_t)(p.m0 + m) * ldy + row);
    }
  }
  // The activation is read next (few KB, L2-resident); the rest of the ring is
  // started once those loads are in flight.
  auto start_ring = [&]() {
    if (lane == 0)
      while (is_count < depth && is_count < n_panels) issue_next();
  };

  // ---- activation -> shared memory (padded to whole slices with q = 0)
  if constexpr (FUSE) {
    // one thread per (row, 32-column block): the per-block division and fp16
    // rounding run once per block; the next round's loads are in flight while
    // this round is quantised, and the weight ring starts behind the first loads
    const bool vec = ((reinterpret_cast<uintptr_t>(p.x) | ((uintptr_t)p.ldx * 4)) & 15) == 0;
    const int total = NB * nsp;  // (row, block) items incl. padding
    auto load_blk = [&](int i, float4 (&v)[8]) {
      const int m = i / nsp, b = i - m * nsp;
      const bool ok = i < total && m < p.nb && b < p.nsub;
      const float* src = p.x + (int64_t)(p.m0 + (ok ? m : 0)) * p.ldx + (ok ? b : 0) * 32;
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] = ok ? load4(src + 4 * k, vec) : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    float4 cur[8], nxt[8];
    if constexpr (kCluster) {
      // this CTA's share of the (row, block) items, written into the shared
      // memory of every CTA of the cluster (same offsets: same launch, same plan)
      const uint32_t rank = cluster_ctarank();
      const int lo = (int)((int64_t)rank * total / kFuseCluster);
      const int hi = (int)((int64_t)(rank + 1) * total / kFuseCluster);
      const int i0 = lo + (int)threadIdx.x;
      load_blk(i0 < hi ? i0 : total, cur);
      if (!kRingAfterStage) start_ring();
      __syncwarp();
      cluster_wait_acquire();  // every CTA of the cluster is running: remote stores are safe
      for (int i = i0; i < hi; i += kThreads) {
        load_blk(i + kThreads < hi ? i + kThreads : total, nxt);
        uint4 qa, qb;
        float dq;
        int sum;
        q8_block32(cur, qa, qb, dq, sum);
        const uint32_t aqa = smem_u32(qa_s + i), aqb = smem_u32(qb_s + i);
        const uint32_t ad = smem_u32(d_s + i), ams = smem_u32(ms_s + i);
#pragma unroll
        for (int c = 0; c < kFuseCluster; ++c) {
          st_cluster_v4(mapa_shared(aqa, c), qa);
          st_cluster_v4(mapa_shared(aqb, c), qb);
          st_cluster_b32(mapa_shared(ad, c), __float_as_uint(dq));
          st_cluster_b32(mapa_shared(ams, c), (uint32_t)(kMagicInt - sum));
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) cur[k] = nxt[k];
      }
      __syncwarp();
      cluster_arrive_release();  // publish this CTA's stores ...
      if (kRingAfterStage) start_ring();
      __syncwarp();
      cluster_wait_acquire();    // ... and see everyone else's
    } else {
      load_blk(threadIdx.x, cur);
      start_ring();
      for (int i = threadIdx.x; i < total; i += kThreads) {
        load_blk(i + kThreads, nxt);
        uint4 qa, qb;
        float dq;
        int sum;
        q8_block32(cur, qa, qb, dq, sum);
        qa_s[i] = qa;
        qb_s[i] = qb;
        d_s[i] = dq;
        ms_s[i] = kMagicInt - sum;
#pragma unroll
        for (int k = 0; k < 8; ++k) cur[k] = nxt[k];
      }
    }
  } else {
    // chunks of kStageIters items per thread (one chunk covers K <= 17408 for NB = 1)
    constexpr int kStageIters = (NB * 544 + kThreads - 1) / kThreads;
    for (int base = 0; base < NB * nsp; base += kStageIters * kThreads) {
      uint4 ra[kStageIters], rb[kStageIters];
      float rd[kStageIters];
      int rs[kStageIters];
#pragma unroll
      for (int it = 0; it < kStageIters; ++it) {
        const int i = base + (int)threadIdx.x + it * kThreads;
        ra[it] = rb[it] = make_uint4(0, 0, 0, 0);
        rd[it] = 0.0f;
        rs[it] = 0;
        if (i < NB * nsp) {
          const int m = i / nsp, sb = i - m * nsp;
          if (m < p.nb && sb < p.nsub) {
            const int64_t row = p.m0 + m;
            const uint4* src = reinterpret_cast<const uint4*>(p.q + row * p.K + (int64_t)sb * 32);
            ra[it] = src[0];
            rb[it] = src[1];
            rd[it] = p.d[row * p.nsub + sb];
            rs[it] = p.s[row * p.nsub + sb];
          }
        }
      }
      if (base == 0) start_ring();
#pragma unroll
      for (int it = 0; it < kStageIters; ++it) {
        const int i = base + (int)threadIdx.x + it * kThreads;
        if (i < NB * nsp) {
          qa_s[i] = ra[it];
          qb_s[i] = rb[it];
          d_s[i] = rd[it];
          ms_s[i] = kMagicInt - rs[it];
        }
      }
    }
  }
  __syncthreads();

  // acc[panel][quad][row pair][m]: rows (4h + 2e, 4h + 2e + 1) of the panel
  float2 acc[kSwi ? 2 : 1][2][2][NB];
#pragma unroll
  for (int pp = 0; pp < (kSwi ? 2 : 1); ++pp)
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int e = 0; e < 2; ++e)
#pragma unroll
        for (int m = 0; m < NB; ++m) acc[pp][h][e][m] = make_float2(0.0f, 0.0f);

  int slot = 0, j = j_lo, ui = 0;
  uint32_t phase = 0;
  bool aborted = false;
  for (int k = 0; k < n_panels; ++k) {
    const uint32_t bar = my_bars + slot * 8;
    const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar, phase, kWaitLimitNs));
    if (!ok) {
      // report, let copies already in flight land (bounded), and leave
      if (lane == 0) {
        atomicCAS(p.err, 0, kErrWaitTimeout);
        int s2 = slot;
        uint32_t ph2 = phase;
        for (int kk = k + 1; kk < is_count; ++kk) {
          if (++s2 == depth) {
            s2 = 0;
            ph2 ^= 1u;
          }
          mbar_wait_bounded(my_bars + s2 * 8, ph2, kWaitLimitNs / 10);
        }
      }
      __syncwarp();
      aborted = true;  // leave the loop but still reach the CTA barrier below
      break;
    }
    const uint8_t* stage = ring + (warp * depth + slot) * plan.stage;
    constexpr int kPan = kSwi ? 2 : 1;  // panels per stage (gate, up)
    uint4 cw[kPan][2][2];               // [panel][quad][half]
    float sc[kPan][kRows];
#pragma unroll
    for (int pp = 0; pp < kPan; ++pp) {
      const uint8_t* pan = stage + pp * kPanelBytes;
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int v = 0; v < 2; ++v)
          cw[pp][h][v] = *reinterpret_cast<const uint4*>(pan + h * 1024 + v * 512 + lane * 16);
      const uint4 s4 = *reinterpret_cast<const uint4*>(pan + kCodeBytes + (lane >> 2) * 16);
      sc[pp][0] = half_lo(s4.x); sc[pp][1] = half_hi(s4.x);
      sc[pp][2] = half_lo(s4.y); sc[pp][3] = half_hi(s4.y);
      sc[pp][4] = half_lo(s4.z); sc[pp][5] = half_hi(s4.z);
      sc[pp][6] = half_lo(s4.w); sc[pp][7] = half_hi(s4.w);
    }
#pragma unroll
    for (int m = 0; m < NB; ++m) {
      const int ai = m * nsp + j * kSubPerSlice + lane;
      const uint4 qa = qa_s[ai], qb = qb_s[ai];
      const float dm = d_s[ai];
      const int ms = ms_s[ai];
      const float2 d2 = make_float2(dm, dm);
      const float2 nmagic = make_float2(-kMagicFloat, -kMagicFloat);
#pragma unroll
      for (int pp = 0; pp < kPan; ++pp)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          int c[4] = {0, 0, 0, 0};
          quad_dots(cw[pp][h][0], cw[pp][h][1], qa, qb, c);
          const float2 f01 = __fadd2_rn(make_float2(__int_as_float(biased_idot<0>(c[0], ms)),
                                                    __int_as_float(biased_idot<1>(c[1], ms))), nmagic);
          const float2 f23 = __fadd2_rn(make_float2(__int_as_float(biased_idot<2>(c[2], ms)),
                                                    __int_as_float(biased_idot<3>(c[3], ms))), nmagic);
          const int r = 4 * h;
          if constexpr (DUMP) {
            int seg_d, g_d;
            locate(first + ui * stride, seg_d, g_d);
            const int sb = j * kSubPerSlice + lane;
            if (m < p.nb && sb < p.nsub) {
              const float fv[4] = {f01.x, f01.y, f23.x, f23.y};
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int row = g_d * kRows + r + k;
                if (row < p.n0) p.idot[((int64_t)(p.m0 + m) * p.n0 + row) * p.nsub + sb] = __float2int_rz(fv[k]);
              }
            }
          }
          const float2 s01 = __fmul2_rn(make_float2(sc[pp][r], sc[pp][r + 1]), d2);
          const float2 s23 = __fmul2_rn(make_float2(sc[pp][r + 2], sc[pp][r + 3]), d2);
          acc[pp][h][0][m] = __ffma2_rn(s01, f01, acc[pp][h][0][m]);
          acc[pp][h][1][m] = __ffma2_rn(s23, f23, acc[pp][h][1][m]);
        }
    }
    __syncwarp();
    if (lane == 0 && is_count < n_panels) {
      fence_proxy_async_smem();  // our generic-proxy reads of the slot precede the next async write
      issue_next();
    }
    if (++slot == depth) {
      slot = 0;
      phase ^= 1u;
    }
    if (++j == j_hi) {  // this warp's part of the unit is done: reduce over lanes
      j = j_lo;
      int seg, g;
      locate(first + ui * stride, seg, g);
      ++ui;
      const int n = seg == 0 ? p.n0 : seg == 1 ? p.n1 : p.n2;
      const int ldy = seg == 0 ? p.ld0 : seg == 1 ? p.ld1 : p.ld2;
      float* y = seg == 0 ? p.y0 : seg == 1 ? p.y1 : p.y2;
#pragma unroll
      for (int m = 0; m < NB; ++m) {
        float v[kRows], u[kRows];
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            v[4 * h + 2 * e] = acc[0][h][e][m].x;
            v[4 * h + 2 * e + 1] = acc[0][h][e][m].y;
            acc[0][h][e][m] = make_float2(0.0f, 0.0f);
            if constexpr (kSwi) {
              u[4 * h + 2 * e] = acc[kSwi ? 1 : 0][h][e][m].x;
              u[4 * h + 2 * e + 1] = acc[kSwi ? 1 : 0][h][e][m].y;
              acc[kSwi ? 1 : 0][h][e][m] = make_float2(0.0f, 0.0f);
            }
          }
        const int row_l = reduce_rows8(v, lane);
        float up = 0.0f;
        if constexpr (kSwi) {
          reduce_rows8(u, lane);  // same lane -> row map as v
          up = u[0];
        }
        if ((lane & 3) == 0) {
          if (G > 1) {  // partial over slices [j_lo, j_hi): combined below
            pieces[(warp * kMaxNb + m) * 16 + row_l] = v[0];
            if constexpr (kSwi) pieces[(warp * kMaxNb + m) * 16 + kRows + row_l] = up;
          } else {
            const int row = g * kRows + row_l;
            if (row < n && m < p.nb) {
              const int64_t idx = (int64_t)(p.m0 + m) * ldy + row;
              if constexpr (MODE == BTF_STORE) put(seg, y, idx, v[0]);
              else if constexpr (MODE == BTF_ADD) put(seg, y, idx, (kPreY ? ypre[m] : get(y, idx)) + v[0]);
              else put(seg, y, idx, silu(v[0]) * up);
            }
          }
        }
      }
      if constexpr (kPreY) {
        if (G == 1) prefetch_y(ui);  // the next unit's rows
      }
    }
  }

  if (G > 1) {  // CTA-uniform: the G parts of each unit are summed in part order
    __syncthreads();
    if (has_work && part == 0 && !aborted) {
      int seg, g;
      locate(first, seg, g);
      const int n = seg == 0 ? p.n0 : seg == 1 ? p.n1 : p.n2;
      const int ldy = seg == 0 ? p.ld0 : seg == 1 ? p.ld1 : p.ld2;
      float* y = seg == 0 ? p.y0 : seg == 1 ? p.y1 : p.y2;
      const int r = lane & 7, m = lane >> 3;
      if (m < NB) {
        float sg = 0.0f, su = 0.0f;
        for (int w = warp; w < warp + G; ++w) {
          sg += pieces[(w * kMaxNb + m) * 16 + r];
          if constexpr (kSwi) su += pieces[(w * kMaxNb + m) * 16 + kRows + r];
        }
        const int row = g * kRows + r;
        if (row < n && m < p.nb) {
          const int64_t idx = (int64_t)(p.m0 + m) * ldy + row;
          if constexpr (MODE == BTF_STORE) put(seg, y, idx, sg);
          else if constexpr (MODE == BTF_ADD) put(seg, y, idx, (kPreY ? ypre[0] : get(y, idx)) + sg);
          else put(seg, y, idx, silu(sg) * su);
        }
      }
    }
  }
  if constexpr (GATHER == 1) gather_arrive(p.gather, p.err);
  stamp_end(p.stamp);
}

// Cross-rank barrier (one thread): the release-adds / bounded acquire wait of
// gather_arrive, on its own.
__global__ void gather_barrier_kernel(const __grid_constant__ btf_gather g, int* err) {
  for (int r = 0; r < g.world; ++r)
    asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(g.flags[r]) : "memory");
  const unsigned target = *g.expect + (unsigned)g.world;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(g.flags[g.rank]) : "memory");
    if ((int)(v - target) >= 0) break;
    if (globaltimer_ns() - t0 > kGatherWaitNs) {
      atomicCAS(err, 0, kErrWaitTimeout);
      break;
    }
  }
  *g.expect = target;
}

// Tagged gather: a new epoch (one thread, in stream order).
__global__ void gather_epoch_kernel(unsigned* epoch) { *epoch += 1u; }

struct TaggedBufs {
  btf_tagged_buf b[8];
  int n;
};
// Tagged gather: every thread checks word i of every buffer (bounded spin on
// the tag half with system-scope relaxed loads, so no stale L1 copy is read).
__global__ void __launch_bounds__(1024) gather_wait_kernel(const __grid_constant__ TaggedBufs t, const unsigned* epoch,
                                                           int* err) {
  pdl_launch_dependents();
  pdl_wait();  // this rank's own stores come from the previous kernel
  const unsigned e = *epoch * 1024u;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint64_t t0 = globaltimer_ns();
  for (int bi = 0; bi < t.n; ++bi) {
    if (i >= t.b[bi].words) continue;
    const unsigned want = e + (unsigned)t.b[bi].site;
    const unsigned* hi = reinterpret_cast<const unsigned*>(t.b[bi].p + i) + 1;
    for (;;) {
      unsigned v;
      asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(hi) : "memory");
      if (v == want) break;
      if (globaltimer_ns() - t0 > kGatherWaitNs) {
        atomicCAS(err, 0, kErrWaitTimeout);
        return;
      }
    }
  }
}

using KernelFn = void (*)(const GemvParams);

template <int MODE, bool FUSE, int GATHER>
KernelFn pick(int NB) {
  switch (NB) {
    case 1: return gemv_kernel<1, MODE, FUSE, GATHER>;
    case 2: return gemv_kernel<2, MODE, FUSE, GATHER>;
    default: return gemv_kernel<4, MODE, FUSE, GATHER>;
  }
}
template <bool FUSE, int GATHER>
KernelFn pick_mode(int NB, int mode) {
  return mode == BTF_STORE ? pick<BTF_STORE, FUSE, GATHER>(NB)
         : mode == BTF_ADD ? pick<BTF_ADD, FUSE, GATHER>(NB)
                           : pick<BTF_SWIGLU, FUSE, GATHER>(NB);
}
// the integer-dump form of the store kernel (btf_gemv_idot)
KernelFn pick_dump(int NB) {
  switch (NB) {
    case 1: return gemv_kernel<1, BTF_STORE, false, 0, true>;
    case 2: return gemv_kernel<2, BTF_STORE, false, 0, true>;
    default: return gemv_kernel<4, BTF_STORE, false, 0, true>;
  }
}
// fused-quantise launches are never N-sharded
KernelFn pick(int NB, int mode, bool fuse, int gather) {
  if (fuse) return pick_mode<true, 0>(NB, mode);
  return gather == 0 ? pick_mode<false, 0>(NB, mode) : gather == 1 ? pick_mode<false, 1>(NB, mode)
                                                                   : pick_mode<false, 2>(NB, mode);
}

bool aligned(const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; }

int check_segs(const char* fn, const btf_gemv_seg* segs, int nseg, int K, int mode) {
  if (!segs || nseg < 1 || nseg > kMaxSeg) return fail(BTF_ERR_ARG, "%s: 1..3 segments (got %d)", fn, nseg);
  if (mode != BTF_STORE && mode != BTF_ADD && mode != BTF_SWIGLU) return fail(BTF_ERR_ARG, "%s: bad mode %d", fn, mode);
  if (mode == BTF_SWIGLU && (nseg != 2 || segs[0].N != segs[1].N))
    return fail(BTF_ERR_ARG, "%s: swiglu needs gate+up segments with the same N", fn);
  if (K <= 0 || K % 128) return fail(BTF_ERR_ARG, "%s: K must be a positive multiple of 128 (K=%d)", fn, K);
  for (int i = 0; i < nseg; ++i) {
    if (!segs[i].panels || !aligned(segs[i].panels, 16) || segs[i].N <= 0)
      return fail(BTF_ERR_ARG, "%s: segment %d has a null/misaligned panel buffer or N <= 0", fn, i);
    const bool needs_y = !(mode == BTF_SWIGLU && i == 1);
    if (needs_y && (!segs[i].y || segs[i].ldy < segs[i].N))
      return fail(BTF_ERR_ARG, "%s: segment %d needs y and ldy >= N", fn, i);
  }
  return BTF_OK;
}

// CTAs of `fn` that fit on one SM with `smem` bytes of dynamic shared memory
// (registers and shared memory), cached: the grid is persistent, so it must
// not exceed what is co-resident.
int resident_ctas(KernelFn fn, int smem) {
  struct Entry { KernelFn fn; int smem; int n; };
  static Entry cache[64];
  static int used = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].fn == fn && cache[i].smem == smem) return cache[i].n;
  int n = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, fn, kThreads, smem) != cudaSuccess || n < 1) n = 1;
  n = std::min(n, kGridCtasPerSm);
  if (used < 64) cache[used++] = Entry{fn, smem, n};
  return n;
}

// CTAs of `fn` resident at once when launched in clusters of `cluster` CTAs
// (whole clusters only; capped at kGridCtasPerSm per SM), cached per (kernel, smem).
int resident_cluster_ctas(KernelFn fn, int smem, int cluster, cudaStream_t st) {
  struct Entry { KernelFn fn; int smem; int n; };
  static Entry cache[64];
  static int used = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].fn == fn && cache[i].smem == smem) return cache[i].n;
  const DeviceInfo* dev = current_device();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster * 64);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) != cudaSuccess) clusters = 0;
  int n = std::min(clusters * cluster, dev ? dev->sm_count * kGridCtasPerSm : clusters * cluster);
  if (used < 64) cache[used++] = Entry{fn, smem, n};
  return n;
}

// Launches the GEMV over M rows in passes of at most kMaxNb activation rows.
int run_gemv(const btf_gemv_seg* segs, int nseg, int K, int M, const btf_q8act* act, const float* x, int ldx,
             int mode, cudaStream_t st, const btf_gather* gather = nullptr, int32_t* idot = nullptr) {
  const DeviceInfo* dev = current_device();
  if (!dev) return BTF_ERR_STATE;
  GemvParams p{};
  const uint8_t* pans[kMaxSeg] = {nullptr, nullptr, nullptr};
  float* ys[kMaxSeg] = {nullptr, nullptr, nullptr};
  int ns[kMaxSeg] = {0, 0, 0}, lds[kMaxSeg] = {0, 0, 0}, units[kMaxSeg] = {0, 0, 0};
  for (int i = 0; i < nseg; ++i) {
    pans[i] = static_cast<const uint8_t*>(segs[i].panels);
    ys[i] = segs[i].y;
    ns[i] = segs[i].N;
    lds[i] = segs[i].ldy;
    units[i] = (int)groups_of(segs[i].N);
  }
  if (mode == BTF_SWIGLU) units[1] = 0;  // a swiglu unit covers the gate and up groups together
  p.pan0 = pans[0]; p.pan1 = pans[1]; p.pan2 = pans[2];
  p.y0 = ys[0]; p.y1 = ys[1]; p.y2 = ys[2];
  p.n0 = ns[0]; p.n1 = ns[1]; p.n2 = ns[2];
  p.ld0 = lds[0]; p.ld1 = lds[1]; p.ld2 = lds[2];
  p.u1 = units[0];
  p.u2 = units[0] + units[1];
  p.utotal = units[0] + units[1] + units[2];
  p.K = K;
  p.S = (int)slices_of(K);
  p.nsub = K / 32;
  if (act) {
    p.q = act->q;
    p.d = act->d;
    p.s = act->s;
  }
  p.x = x;
  p.ldx = ldx;
  p.err = dev->err_word;
  if (gather) p.gather = *gather;
  p.stamp = take_stamp();  // every pass raises it: the slot ends as the last pass's end
  p.idot = idot;
  for (int m0 = 0; m0 < M; m0 += kMaxNb) {
    const int nb = std::min(kMaxNb, M - m0);
    const int NB = nb <= 1 ? 1 : nb <= 2 ? 2 : 4;
    // ring slots: fill ~kSmemTarget, at least 2 per warp
    const SmemPlan base(mode, NB, p.S, 0);
    const size_t room = kSmemTarget > (size_t)base.act ? kSmemTarget - (size_t)base.act : 0;
    const int slots = std::max(2 * kWarps, std::min((int)(room / (base.stage + 8)), 64));
    const SmemPlan plan(mode, NB, p.S, slots);
    if (plan.total > dev->optin_smem - 1024)
      return fail(BTF_ERR_UNSUPPORTED, "btf_gemv: K=%d with %d activation rows needs %d B of shared memory (max %d)",
                  K, NB, plan.total, dev->optin_smem - 1024);
    p.slots = slots;
    p.m0 = m0;
    p.nb = nb;
    const KernelFn fn = idot ? pick_dump(NB) : pick(NB, mode, x != nullptr, !gather ? 0 : gather->tagged ? 2 : 1);
    const int cluster = x != nullptr ? kFuseCluster : 1;
    const int resident = cluster > 1 ? resident_cluster_ctas(fn, plan.total, cluster, st)
                                     : dev->sm_count * resident_ctas(fn, plan.total);
    if (resident < cluster) return fail(BTF_ERR_UNSUPPORTED, "btf_gemv_f32: no cluster of %d CTAs fits", cluster);
    // every CTA gets ceil(utotal / resident CTAs) units, or fewer; whole clusters
    const int cap = std::max(1, std::min(p.utotal, resident));
    const int upc = (p.utotal + cap - 1) / cap;
    int grid = kBalancedGrid ? (p.utotal + upc - 1) / upc : cap;
    grid = std::min((grid + cluster - 1) / cluster * cluster, resident / cluster * cluster);
    const cudaError_t e = launch_pdl_cluster(fn, dim3(grid), dim3(kThreads), (size_t)plan.total, st, cluster, p);
    if (e != cudaSuccess) return cuda_fail(e, "gemv_kernel launch");
    if (int rc = launch_status("gemv_kernel")) return rc;
  }
  return BTF_OK;
}

template <int MODE, bool FUSE, int GATHER>
cudaError_t set_attrs(int smem) {
  cudaError_t e;
  if ((e = cudaFuncSetAttribute(gemv_kernel<1, MODE, FUSE, GATHER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                smem)))
    return e;
  if ((e = cudaFuncSetAttribute(gemv_kernel<2, MODE, FUSE, GATHER>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                smem)))
    return e;
  return cudaFuncSetAttribute(gemv_kernel<4, MODE, FUSE, GATHER>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
}
template <bool FUSE, int GATHER>
cudaError_t set_attrs_all(int smem) {
  cudaError_t e;
  if ((e = set_attrs<BTF_STORE, FUSE, GATHER>(smem)) || (e = set_attrs<BTF_ADD, FUSE, GATHER>(smem))) return e;
  return set_attrs<BTF_SWIGLU, FUSE, GATHER>(smem);
}

}  // namespace

// One error word per device (module-scope device variable, no allocation).
__device__ int g_device_error;

int gemv_setup(DeviceInfo& d) {
  cudaError_t e;
  void* ew = nullptr;
  if ((e = cudaGetSymbolAddress(&ew, g_device_error)) != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress");
  d.err_word = static_cast<int*>(ew);
  // leave room for static shared memory (per-block limit = dynamic + static)
  const int dyn = d.optin_smem - 1024;
  if ((e = set_attrs_all<false, 0>(dyn)) || (e = set_attrs_all<false, 1>(dyn)) || (e = set_attrs_all<false, 2>(dyn)) ||
      (e = set_attrs_all<true, 0>(dyn)))
    return cuda_fail(e, "cudaFuncSetAttribute(gemv_kernel)");
  for (int nb : {1, 2, 4})
    if ((e = cudaFuncSetAttribute(pick_dump(nb), cudaFuncAttributeMaxDynamicSharedMemorySize, dyn)))
      return cuda_fail(e, "cudaFuncSetAttribute(gemv_kernel, dump)");
  return BTF_OK;
}

// the weight-major GEMM's dispatch rule and launch (gemm_wm.cu), and the
// warp-MMA small-batch GEMM's rule (gemv_mma.cu)
bool wm_serves(const btf_gemv_seg& seg, int M, const btf_q8act& act);
bool mma_serves(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act);
bool mma_two_pass_serves(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act);
int run_gemv_mma_rows(const btf_gemv_seg* segs, int nseg, int K, int m0, int M, const btf_q8act& act, int mode,
                      cudaStream_t st);
int run_gemv_mma(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act, int mode, cudaStream_t st,
                 int32_t* idot, const btf_gather* g, int gseg);
int run_gemm_wm(const btf_gemv_seg& seg, int K, int M, const btf_q8act& act, int mode, cudaStream_t st,
                int32_t* idot, const btf_gather* g, int gseg);

}  // namespace btf

using namespace btf;

extern "C" {

int btf_gemv_max_nb(int K) { return (K > 0 && K % 128 == 0) ? kMaxNb : 0; }

int btf_gemv(const btf_gemv_seg* segs, int nseg, int K, int M, btf_q8act act, int mode, void* stream) {
  if (M <= 0) return BTF_OK;
  if (int rc = check_segs("btf_gemv", segs, nseg, K, mode)) return rc;
  if (!act.q || !act.d || !act.s || !aligned(act.q, 16) || !aligned(act.d, 4) || !aligned(act.s, 4))
    return fail(BTF_ERR_ARG, "btf_gemv: activation pointers null or misaligned (q needs 16 B)");
  // A batch of rows is a dense contraction: instead of the reference's repeated
  // small-batch passes over the weights (kernels.cu:805-821), store / add calls
  // go to the MMA kernels (d 16-byte aligned): 3..16 rows over very large
  // matrices (an lm_head) to the warp-MMA kernel, 9..64 rows over large
  // matrices to the tcgen05 weight-major kernel (one weight pass each), 64
  // rows and more to the 128-row tcgen05 GEMM.
  if (mode != BTF_SWIGLU && aligned(act.d, 16)) {
    bool mma = true, mma2 = true, wm = true;
    for (int i = 0; i < nseg; ++i) mma = mma && mma_serves(segs[i], K, M, act);
    if (mma) return btf_gemv_mma(segs, nseg, K, M, act, mode, stream);
    for (int i = 0; i < nseg; ++i) mma2 = mma2 && mma_two_pass_serves(segs[i], K, M, act);
    if (mma2) {  // 17..32 rows over lm_head-size matrices: two warp-MMA passes of 16 rows
      take_stamp();  // a stamp request would land on the first pass only: drop it
      if (int rc = run_gemv_mma_rows(segs, nseg, K, 0, 16, act, mode, (cudaStream_t)stream)) return rc;
      return run_gemv_mma_rows(segs, nseg, K, 16, M - 16, act, mode, (cudaStream_t)stream);
    }
    for (int i = 0; i < nseg; ++i) wm = wm && wm_serves(segs[i], M, act);
    if (wm) return btf_gemm_wm(segs, nseg, K, M, act, mode, stream);
    if (M >= kGemmMinM) {
      take_stamp();  // the 128-row GEMM writes no end stamp: drop a pending request
      return btf_gemm(segs, nseg, K, M, act, mode, stream);
    }
  }
  return run_gemv(segs, nseg, K, M, &act, nullptr, 0, mode, (cudaStream_t)stream);
}

int btf_gemv_gather(const btf_gemv_seg* segs, int nseg, int K, int M, btf_q8act act, int mode, const btf_gather* g,
                    void* stream) {
  if (M <= 0) return BTF_OK;
  if (int rc = check_segs("btf_gemv_gather", segs, nseg, K, mode)) return rc;
  if (!act.q || !act.d || !act.s || !aligned(act.q, 16) || !aligned(act.d, 4) || !aligned(act.s, 4))
    return fail(BTF_ERR_ARG, "btf_gemv_gather: activation pointers null or misaligned (q needs 16 B)");
  if (!g || g->world < 2 || g->world > BTF_MAX_RANKS || g->rank < 0 || g->rank >= g->world)
    return fail(BTF_ERR_ARG, "btf_gemv_gather: need 2 <= world <= %d and 0 <= rank < world", BTF_MAX_RANKS);
  if (g->tagged) {
    if (!g->epoch || g->site < 0 || g->site >= 1024)
      return fail(BTF_ERR_ARG, "btf_gemv_gather: tagged launch needs an epoch counter and 0 <= site < 1024");
  } else if (!g->expect || !g->done) {
    return fail(BTF_ERR_ARG, "btf_gemv_gather: expect/done counters are null");
  }
  const int nout = mode == BTF_SWIGLU ? 1 : nseg;  // segments with an output
  for (int r = 0; r < g->world; ++r) {
    if (!g->tagged && !g->flags[r]) return fail(BTF_ERR_ARG, "btf_gemv_gather: arrival counter of rank %d is null", r);
    for (int s = 0; s < nout; ++s)
      if (!g->peer_y[s][r]) return fail(BTF_ERR_ARG, "btf_gemv_gather: peer_y[%d][%d] is null", s, r);
  }
  for (int s = 0; s < nout; ++s)
    if (g->peer_y[s][g->rank] != segs[s].y)
      return fail(BTF_ERR_ARG, "btf_gemv_gather: peer_y[%d][rank] must be segs[%d].y", s, s);
  // tagged store calls over large shards: the warp-MMA GEMM (3..16 rows over
  // lm_head-size shards) or the weight-major tcgen05 GEMM, one weight pass
  if (g->tagged && mode == BTF_STORE && aligned(act.d, 16)) {
    bool mma = true, wm = true;
    for (int i = 0; i < nseg; ++i) mma = mma && mma_serves(segs[i], K, M, act);
    if (mma) {
      for (int i = 0; i < nseg; ++i)
        if (int rc = run_gemv_mma(segs[i], K, M, act, mode, (cudaStream_t)stream, nullptr, g, i)) return rc;
      return BTF_OK;
    }
    for (int i = 0; i < nseg; ++i) wm = wm && wm_serves(segs[i], M, act);
    if (wm) {
      for (int i = 0; i < nseg; ++i)
        if (int rc = run_gemm_wm(segs[i], K, M, act, mode, (cudaStream_t)stream, nullptr, g, i)) return rc;
      return BTF_OK;
    }
  }
  if (!g->tagged && M > kMaxNb)  // counted completion: one arrival per launch, so one pass
    return fail(BTF_ERR_UNSUPPORTED, "btf_gemv_gather: counted completion needs M <= %d (one pass)", kMaxNb);
  return run_gemv(segs, nseg, K, M, &act, nullptr, 0, mode, (cudaStream_t)stream, g);
}

int btf_gather_epoch_advance(unsigned int* epoch, void* stream) {
  if (!epoch) return fail(BTF_ERR_ARG, "btf_gather_epoch_advance: null epoch");
  if (!current_device()) return BTF_ERR_STATE;
  gather_epoch_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(epoch);
  return launch_status("gather_epoch_kernel");
}

int btf_gather_barrier(const btf_gather* g, void* stream) {
  if (!g || g->world < 2 || g->world > BTF_MAX_RANKS || g->rank < 0 || g->rank >= g->world || !g->expect)
    return fail(BTF_ERR_ARG, "btf_gather_barrier: need 2 <= world <= %d, a rank and an expect counter", BTF_MAX_RANKS);
  for (int r = 0; r < g->world; ++r)
    if (!g->flags[r]) return fail(BTF_ERR_ARG, "btf_gather_barrier: arrival counter of rank %d is null", r);
  const DeviceInfo* dev = current_device();
  if (!dev) return BTF_ERR_STATE;
  gather_barrier_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(*g, dev->err_word);
  return launch_status("gather_barrier_kernel");
}

int btf_gather_wait(const btf_tagged_buf* bufs, int n, const unsigned int* epoch, void* stream) {
  if (!bufs || n < 1 || n > 8 || !epoch) return fail(BTF_ERR_ARG, "btf_gather_wait: 1..8 buffers and an epoch");
  TaggedBufs t{};
  int64_t most = 0;
  for (int i = 0; i < n; ++i) {
    if (!bufs[i].p || bufs[i].words < 0 || bufs[i].site < 0 || bufs[i].site >= 1024 || !aligned(bufs[i].p, 8))
      return fail(BTF_ERR_ARG, "btf_gather_wait: buffer %d is null, misaligned or has a bad site", i);
    t.b[i] = bufs[i];
    most = std::max(most, bufs[i].words);
  }
  t.n = n;
  const DeviceInfo* dev = current_device();
  if (!dev) return BTF_ERR_STATE;
  const int grid = (int)std::max<int64_t>(1, (most + 1023) / 1024);
  const cudaError_t e = launch_pdl(gather_wait_kernel, dim3(grid), dim3(1024), 0, (cudaStream_t)stream, t, epoch,
                                   dev->err_word);
  return e == cudaSuccess ? launch_status("gather_wait_kernel") : cuda_fail(e, "gather_wait_kernel launch");
}

int btf_gemv_f32(const btf_gemv_seg* segs, int nseg, int K, int M, const float* x, int ldx, int mode, void* stream) {
  if (M <= 0) return BTF_OK;
  if (int rc = check_segs("btf_gemv_f32", segs, nseg, K, mode)) return rc;
  if (!x || ldx < K || !aligned(x, 4)) return fail(BTF_ERR_ARG, "btf_gemv_f32: x null/misaligned or ldx < K");
  return run_gemv(segs, nseg, K, M, nullptr, x, ldx, mode, (cudaStream_t)stream);
}

int btf_device_error(int clear) {
  const DeviceInfo* dev = current_device();
  if (!dev) return -1;
  int v = 0;
  cudaError_t e = cudaMemcpy(&v, dev->err_word, sizeof v, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "btf_device_error"), -1;
  if (clear && v) {
    const int z = 0;
    if ((e = cudaMemcpy(dev->err_word, &z, sizeof z, cudaMemcpyHostToDevice)) != cudaSuccess)
      return cuda_fail(e, "btf_device_error"), -1;
  }
  return v;
}

int btf_gemv_idot(const void* panels, int N, int K, int M, btf_q8act act, int32_t* idot, void* stream) {
  if (M <= 0) return BTF_OK;
  if (!panels || !idot || !act.q || !act.d || !act.s || N <= 0 || K <= 0 || K % 128 || !aligned(act.q, 16) ||
      !aligned(panels, 16) || !aligned(act.d, 4) || !aligned(act.s, 4))
    return fail(BTF_ERR_ARG, "btf_gemv_idot: bad arguments");
  btf_gemv_seg seg{panels, N, nullptr, N};
  return run_gemv(&seg, 1, K, M, &act, nullptr, 0, BTF_STORE, (cudaStream_t)stream, nullptr, idot);
}

}  // extern "C"
