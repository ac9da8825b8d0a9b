// Persistent GEMV chain: a decoder's sequence of ternary matmul call sites in
// ONE launch.
//
// Replaces the per-matmul launch_prep + launch_gemv pairs that the reference
// decoder issues into its captured stream for one token
// (GpuDecoder::forward_chunk / gdn_layer / attn_layer, src/cuda/gpu_decoder.cu:
// 401-450; launchers src/cuda/kernels.cu:745-822) when each matmul's input is
// produced by the matmul before it. Every op is the GEMV of btf_gemv (the same
// per-row math as gemv_kernel<NB, MODE>, src/cuda/kernels.cu:238-334: store /
// add / swiglu over 1..3 segments) with its activation prepared in the op's own
// prologue: optional RMSNorm (bd::rmsnorm's double sum of squares,
// ref/bonsai-decoder/src/cpu_ops.cpp:113-127, in a fixed parallel order) then
// Q8_0 with the btf_quant_q8 rule (q8_block_host, include/btf/packed.hpp:117-134).
//
// B200 design:
//   - one persistent, co-resident grid (two CTAs per SM) runs every op. Op i+1
//     reads its input only when every CTA has finished op i: a monotonic
//     completion counter in the program buffer (release add per CTA, acquire
//     polling with a bounded wait), the same ordering as back-to-back launches;
//   - the weight stream does not stop at op boundaries: each warp's ring of
//     panel slots (1-D bulk copies on mbarriers) is refilled from the warp's
//     panel sequence over the WHOLE program, so while a CTA waits for the last
//     rows of op i and quantises op i+1's input, the panels of op i+1 (and of
//     the ops after it) are already landing in shared memory;
//   - per op the unit split is that of gemv_kernel: a balanced, contiguous
//     range of 8-row groups per CTA, and units cut into slice ranges across
//     warps when a CTA has fewer units than warps;
//   - every wait is bounded (globaltimer); on time-out the device error word is
//     set, the CTA stops computing, waits (bounded) for its own copies in
//     flight, keeps counting so that no other CTA waits longer, and returns.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "gemv_core.cuh"

namespace btf {
namespace {

using namespace core;

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxNb = 2;  // activation rows of a chain (one pass per op)
constexpr int kCluster = 4;  // CTAs that share the quantisation of each op's input (DSMEM)
constexpr uint64_t kWaitNs = 1000000000ull;
#ifndef BTF_CHAIN_SMEM_KB
#define BTF_CHAIN_SMEM_KB 110
#endif
constexpr int kSmemTarget = BTF_CHAIN_SMEM_KB * 1024;  // two CTAs per SM
// Programmatic dependent launch of the chain itself stays off: with it, a run
// launched while the previous one drained was observed on B200 with one of its
// 4-CTA clusters left unscheduled while the other CTAs waited for it (the grid
// waits on itself, so every CTA must be resident). A plain launch starts on an
// idle device. The chain still lets a PDL kernel after it start early.
#ifndef BTF_CHAIN_PDL
#define BTF_CHAIN_PDL 0
#endif
#ifndef BTF_CHAIN_PREWAIT
#define BTF_CHAIN_PREWAIT 2
#endif
constexpr int kPrewait = BTF_CHAIN_PREWAIT;  // panels per warp copied before griddepcontrol.wait

// One op as the device reads it (128 bytes). y pointers and n/ld per segment;
// u1/u2/utotal: cumulative 8-row-group counts of the segments (a swiglu unit
// covers the gate and up groups of the same rows).
struct __align__(16) ChainOp {
  const uint8_t* pan[3];
  float* y[3];
  const float* x;      // fp32 input [M][ldx]
  const float* normw;  // RMSNorm weight [K] or null
  int n[3];
  int ld[3];
  int u1, u2, utotal;
  int K, S, nsub;
  int mode, ldx;
  float eps;
  int pad;
};
static_assert(sizeof(ChainOp) == 128, "ChainOp is 128 bytes");

// Program buffer: this header, then the ops.
struct ChainHeader {
  unsigned ctr;   // CTA-op completions (monotonic across launches)
  unsigned base;  // ctr at the start of the current launch
  // first wait that gave up: [0] = 1 + kind (1: counter, 2: weight slot), then
  // block, warp, op, target or slot, value seen or phase, panels issued, consumed
  unsigned gaveup[8];
  unsigned pad0[22];
  unsigned exit_ctr;  // CTAs that finished the current launch
  unsigned pad1[31];
};
static_assert(sizeof(ChainHeader) == 256, "ChainHeader is 256 bytes");

struct ChainParams {
  const ChainOp* ops;
  ChainHeader* hdr;
  int n_ops;
  int nb;       // activation rows (<= NB)
  int depth;    // ring slots per warp
  int max_nsp;  // largest S * 32 over the ops (activation area)
  int* err;
};

// Small shared-memory items after the pieces (byte offsets): a window of op
// descriptors (op o in slot o % kWin; during op i it holds ops i .. i + kWin - 1,
// so that the weight producers never read the op table in global memory, whose
// latency under the weight stream is microseconds), double red[kWarps][kMaxNb],
// double cred[kCluster][kMaxNb], float scale[kMaxNb], the abort flag, the
// producers' plans.
constexpr int kWin = 8;  // op descriptors held in shared memory: the current op and the 7 after it
constexpr int kMiscWin = 0, kMiscRed = kWin * 128, kMiscCred = kMiscRed + 128, kMiscScale = kMiscCred + 64,
              kMiscAbort = kMiscScale + 16, kMiscPlan = kMiscAbort + 16, kMiscBytes = kMiscPlan + kWarps * 32;

// The producer's plan for its current op (per warp, shared memory; read only at
// unit boundaries, so it need not occupy registers through the compute loop).
struct ProdPlan {
  int first, stride, units, j_lo, j_hi, swi;
};

// Shared-memory layout (bytes), identical on host and device.
struct ChainSmem {
  int ring, bars, act, pieces, misc, total;
  __host__ __device__ ChainSmem(int nb, int max_nsp, int depth) {
    ring = kWarps * depth * kPanelBytes;
    bars = (kWarps * depth * 8 + 15) / 16 * 16;
    act = nb * max_nsp * 40;  // qa 16 B + qb 16 B + d 4 B + magic_s 4 B per sub-block
    pieces = kWarps * kMaxNb * 16 * 4;
    misc = kMiscBytes;
    total = ring + bars + act + pieces + misc;
  }
};

// The part of op work a warp of this CTA does (the unit split of gemv_kernel).
struct WarpPlan {
  int first, stride, n_units, j_lo, j_hi, G, part, cta_units;
  bool has_work;
};
__device__ __forceinline__ WarpPlan warp_plan(int utotal, int S, int warp) {
  WarpPlan w;
  const int u_begin = (int)((int64_t)blockIdx.x * utotal / gridDim.x);
  const int u_end = (int)((int64_t)(blockIdx.x + 1) * utotal / gridDim.x);
  w.cta_units = u_end - u_begin;
  w.G = (w.cta_units > 0 && w.cta_units < kWarps) ? min(kWarps / w.cta_units, S) : 1;
  w.part = warp % w.G;
  w.first = u_begin + (w.G > 1 ? warp / w.G : warp);
  w.stride = w.G > 1 ? w.cta_units : kWarps;
  w.has_work = w.G > 1 ? warp < w.cta_units * w.G : w.first < u_end;
  w.j_lo = w.G > 1 ? w.part * S / w.G : 0;
  w.j_hi = w.G > 1 ? (w.part + 1) * S / w.G : S;
  w.n_units = !w.has_work ? 0 : w.G > 1 ? 1 : (u_end - w.first + kWarps - 1) / kWarps;
  return w;
}

// unit -> (segment, row group)
__device__ __forceinline__ void locate(int u, bool swi, int u1, int u2, int& seg, int& g) {
  seg = swi ? 0 : (u >= u1) + (u >= u2);
  g = u - (seg == 0 ? 0 : seg == 1 ? u1 : u2);
}

__device__ __forceinline__ float4 load4_cg(const float* p, bool vec) {
  if (vec) return __ldcg(reinterpret_cast<const float4*>(p));
  return make_float4(__ldcg(p), __ldcg(p + 1), __ldcg(p + 2), __ldcg(p + 3));
}

// Thread 0: waits, bounded, until the completion counter reaches `target`.
// false on time-out (error word set), or when a wait has lasted 100 us and the
// error word shows that another CTA already gave up (a CTA that gave up stops
// computing, so its rows never arrive).
__device__ bool wait_count(const unsigned* ctr, unsigned target, int* err, unsigned& seen) {
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    seen = v;
    if ((int)(v - target) >= 0) break;
    const uint64_t dt = globaltimer_ns() - t0;
    if (dt > 100000) {
      int e;
      asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(e) : "l"(err) : "memory");
      if (e != 0) return false;
    }
    if (dt > kWaitNs) {
      atomicCAS(err, 0, kErrWaitTimeout);
      return false;
    }
  }
  __threadfence();
  return true;
}

// Records the first wait of a launch that gave up (diagnostics for the host).
__device__ void record_gaveup(ChainHeader* h, unsigned kind, unsigned warp, unsigned op, unsigned a, unsigned b,
                              unsigned c, unsigned d) {
  if (atomicCAS(&h->gaveup[0], 0u, 1u + kind) != 0u) return;
  h->gaveup[1] = blockIdx.x;
  h->gaveup[2] = warp;
  h->gaveup[3] = op;
  h->gaveup[4] = a;
  h->gaveup[5] = b;
  h->gaveup[6] = c;
  h->gaveup[7] = d;
}

__device__ __forceinline__ void st_cluster_f64(uint32_t addr, double v) {
  asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(addr), "d"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
  cluster_arrive_release();
  cluster_wait_acquire();
}

// Activation of one op -> shared memory of every CTA of the cluster: per
// (row, 32-column block) item, optional RMSNorm then Q8_0 (btf_quant_q8's
// rule); padding blocks up to whole slices get q = 0, d = 0. CTA r of the
// cluster handles items [r * total / 4, (r + 1) * total / 4) and stores their
// Q8 words into all four CTAs (DSMEM). Sum of squares order (fixed, in double):
// thread t of CTA r sums its items lo_r + t, lo_r + t + 256, ... in turn, each
// item's 32 squares in column order; a butterfly over the 32 lanes (xor 16, 8,
// 4, 2, 1); the 8 warps' totals in warp order; the 4 CTAs' totals in rank order.
// Every thread of every CTA of the cluster calls it (it holds cluster
// barriers); `skip` (the CTA gave up) leaves out the work, not the barriers.
// Precondition: no CTA of the cluster still reads its activation area.
template <int NB>
__device__ __forceinline__ void stage_act(const ChainOp& op, int nb, uint8_t* act, double* red, double* cred,
                                          float* scale_s, bool skip) {
  const int nsp = op.S * kSubPerSlice, nsub = op.nsub, total = NB * nsp;
  const uint32_t rank = cluster_ctarank();
  const int lo = (int)((int64_t)rank * total / kCluster), hi = (int)((int64_t)(rank + 1) * total / kCluster);
  uint4* qa_s = reinterpret_cast<uint4*>(act);
  uint4* qb_s = qa_s + NB * nsp;
  float* d_s = reinterpret_cast<float*>(qb_s + NB * nsp);
  int* ms_s = reinterpret_cast<int*>(d_s + NB * nsp);
  const float* x = op.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(x) | ((uintptr_t)op.ldx * 4)) & 15) == 0;
  auto load_blk = [&](int i, float4 (&v)[8]) {
    const int m = i / nsp, b = i - m * nsp;
    const bool ok = !skip && i < hi && m < nb && b < nsub;
    const float* src = x + (int64_t)(ok ? m : 0) * op.ldx + (ok ? b : 0) * 32;
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = ok ? load4_cg(src + 4 * k, vec) : make_float4(0.f, 0.f, 0.f, 0.f);
  };
  const int i0 = lo + (int)threadIdx.x;
  float4 cur[8];
  load_blk(i0, cur);  // the first round stays in registers for the quantisation
  const bool norm = op.normw != nullptr;
  if (norm) {
    double part[NB];
#pragma unroll
    for (int m = 0; m < NB; ++m) part[m] = 0.0;
    auto accumulate = [&](int i, const float4 (&v)[8]) {
      double bs = 0.0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        bs += (double)v[k].x * (double)v[k].x;
        bs += (double)v[k].y * (double)v[k].y;
        bs += (double)v[k].z * (double)v[k].z;
        bs += (double)v[k].w * (double)v[k].w;
      }
      const int m = i / nsp;
#pragma unroll
      for (int mm = 0; mm < NB; ++mm)
        if (mm == m) part[mm] += bs;
    };
    if (i0 < hi) accumulate(i0, cur);
    for (int i = i0 + kThreads; i < hi; i += kThreads) {
      float4 v[8];
      load_blk(i, v);
      accumulate(i, v);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int mm = 0; mm < NB; ++mm) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) part[mm] += __shfl_xor_sync(0xffffffffu, part[mm], o);
      if (lane == 0) red[warp * kMaxNb + mm] = part[mm];
    }
    __syncthreads();
    if (threadIdx.x < NB && !skip) {  // this CTA's total -> slot `rank` of every CTA of the cluster
      double t = 0.0;
      for (int w = 0; w < kWarps; ++w) t += red[w * kMaxNb + threadIdx.x];
      const uint32_t a = smem_u32(cred + rank * kMaxNb + threadIdx.x);
#pragma unroll
      for (int c = 0; c < kCluster; ++c) st_cluster_f64(mapa_shared(a, c), t);
    }
    cluster_sync_all();
    if (threadIdx.x < NB) {
      double tot = 0.0;
#pragma unroll
      for (int c = 0; c < kCluster; ++c) tot += cred[c * kMaxNb + threadIdx.x];
      const float mean = (float)(tot / (double)op.K);
      scale_s[threadIdx.x] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, op.eps)));
    }
    __syncthreads();
  }
  const bool wvec = (reinterpret_cast<uintptr_t>(op.normw) & 15) == 0;
  for (int i = i0; i < hi && !skip; i += kThreads) {
    if (i != i0) load_blk(i, cur);
    const int m = i / nsp, b = i - m * nsp;
    if (norm && !skip && m < nb && b < nsub) {
      const float sc = scale_s[m];
      const float* wp = op.normw + b * 32;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float4 w4 = load4(wp + 4 * k, wvec);
        cur[k].x = __fmul_rn(__fmul_rn(cur[k].x, sc), w4.x);
        cur[k].y = __fmul_rn(__fmul_rn(cur[k].y, sc), w4.y);
        cur[k].z = __fmul_rn(__fmul_rn(cur[k].z, sc), w4.z);
        cur[k].w = __fmul_rn(__fmul_rn(cur[k].w, sc), w4.w);
      }
    }
    uint4 qa, qb;
    float dq;
    int sum;
    q8_block32(cur, qa, qb, dq, sum);
    const uint32_t aqa = smem_u32(qa_s + i), aqb = smem_u32(qb_s + i);
    const uint32_t ad = smem_u32(d_s + i), ams = smem_u32(ms_s + i);
#pragma unroll
    for (int c = 0; c < kCluster; ++c) {
      st_cluster_v4(mapa_shared(aqa, c), qa);
      st_cluster_v4(mapa_shared(aqb, c), qb);
      st_cluster_b32(mapa_shared(ad, c), __float_as_uint(dq));
      st_cluster_b32(mapa_shared(ams, c), (uint32_t)(kMagicInt - sum));
    }
  }
  cluster_sync_all();  // every CTA's quarter is in every CTA's shared memory
}

template <int NB>
__global__ void __launch_bounds__(kThreads, 2) chain_kernel(const __grid_constant__ ChainParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  cluster_arrive_relaxed();  // matched by the wait before the first remote (DSMEM) store
  const ChainSmem L(NB, p.max_nsp, p.depth);
  uint8_t* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.ring);
  uint8_t* act = smem + L.ring + L.bars;
  float* pieces = reinterpret_cast<float*>(act + L.act);
  uint8_t* misc = reinterpret_cast<uint8_t*>(pieces) + L.pieces;
  ChainOp* win = reinterpret_cast<ChainOp*>(misc + kMiscWin);
  double* red = reinterpret_cast<double*>(misc + kMiscRed);
  double* cred = reinterpret_cast<double*>(misc + kMiscCred);
  float* scale_s = reinterpret_cast<float*>(misc + kMiscScale);
  volatile int* abort_s = reinterpret_cast<int*>(misc + kMiscAbort);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int depth = p.depth;
  const uint32_t my_bars = smem_u32(bars + warp * depth);
  const uint32_t my_ring = smem_u32(ring + (size_t)warp * depth * kPanelBytes);

  // ---- producer (lane 0 of each warp): the warp's panel sequence over the
  // whole program, op by op, unit by unit, slice by slice (gate, then up). It
  // reads op descriptors from the window only: an op beyond the window waits
  // (pr_ready false) until the window has moved far enough.
  int pr_op = 0, pr_ui = 0, pr_j = 0, pr_jhi = 0, pr_slot = 0, pr_issued = 0;
  bool pr_half = false, pr_ready = false;
  const uint8_t* pr_a = nullptr;
  const uint8_t* pr_b = nullptr;
  ProdPlan& pp_s = reinterpret_cast<ProdPlan*>(misc + kMiscPlan)[warp];
  auto unit_src = [&](const ChainOp& o) {
    int seg, g;
    locate(pp_s.first + pr_ui * pp_s.stride, pp_s.swi, o.u1, o.u2, seg, g);
    const int64_t off = ((int64_t)g * o.S + pp_s.j_lo) * kPanelBytes;
    pr_a = o.pan[seg] + off;
    pr_b = o.pan[1] + off;  // read only for swiglu
  };
  auto seek = [&](int from, int limit) {  // first op >= from in which this warp has work
    for (pr_op = from; pr_op < p.n_ops && pr_op < limit; ++pr_op) {
      const ChainOp& o = win[pr_op % kWin];
      const WarpPlan w = warp_plan(o.utotal, o.S, warp);
      if (w.n_units > 0) {
        pp_s.first = w.first;
        pp_s.stride = w.stride;
        pp_s.units = w.n_units;
        pp_s.j_lo = w.j_lo;
        pp_s.j_hi = w.j_hi;
        pp_s.swi = o.mode == BTF_SWIGLU;
        pr_jhi = w.j_hi;
        pr_ui = 0;
        pr_j = w.j_lo;
        pr_half = false;
        unit_src(o);
        pr_ready = true;
        return;
      }
    }
    pr_ready = false;  // pr_op: where to resume (n_ops: the sequence is done)
  };
  auto issue = [&](int limit) {
    const uint32_t bar = my_bars + pr_slot * 8, dst = my_ring + pr_slot * kPanelBytes;
    mbar_expect_tx(bar, kPanelBytes);
    bulk_g2s(dst, pr_half ? pr_b : pr_a, kPanelBytes, bar);
    ++pr_issued;
    if (++pr_slot == depth) pr_slot = 0;
    if (!pr_half && pp_s.swi) {
      pr_half = true;
      return;
    }
    pr_half = false;
    if (++pr_j == pr_jhi) {
      pr_j = pp_s.j_lo;
      if (++pr_ui < pp_s.units) unit_src(win[pr_op % kWin]);
      else seek(pr_op + 1, limit);
    } else {
      pr_a += kPanelBytes;
      pr_b += kPanelBytes;
    }
  };
  // lane 0: keep up to `room` panels in flight beyond those consumed
  auto refill = [&](int room, int limit) {
    if (!pr_ready && pr_op < p.n_ops) seek(pr_op, limit);
    while (pr_ready && pr_issued < room) issue(limit);
  };

  // the first kWin op descriptors (the op table is written before the launch)
  if (threadIdx.x < kWin * 8) {
    const int o = threadIdx.x >> 3;
    if (o < p.n_ops)
      reinterpret_cast<uint4*>(win + o)[threadIdx.x & 7] = reinterpret_cast<const uint4*>(p.ops + o)[threadIdx.x & 7];
  }
  if (threadIdx.x == 0) *abort_s = 0;
  __syncthreads();
  if (lane == 0) {
    for (int i = 0; i < depth; ++i) mbar_init(my_bars + i * 8, 1);
    fence_mbar_init();
    // weights never depend on the previous kernel: start the first panels now
    refill(min(kPrewait, depth), kWin);
  }
  pdl_wait();  // inputs of op 0 and the counters are final once the previous kernel is complete
  if (lane == 0) refill(depth, kWin);
  const unsigned base = __ldcg(&p.hdr->base);  // L2: an L1 line of a previous launch may be stale
  __syncthreads();

  // ---- consumer
  int c_slot = 0, c_count = 0;
  uint32_t c_phase = 0;
  for (int oi = 0; oi < p.n_ops; ++oi) {
    // slide the window: op oi + kWin - 1 replaces op oi - 1, whose slot no warp
    // reads any more (every warp of this CTA has finished op oi - 1); loaded by
    // warp 1 while thread 0 waits for the counter
    if (oi > 0 && threadIdx.x >= 32 && threadIdx.x < 40) {
      const int o = oi + kWin - 1;
      if (o < p.n_ops)
        reinterpret_cast<uint4*>(win + o % kWin)[threadIdx.x - 32] =
            reinterpret_cast<const uint4*>(p.ops + o)[threadIdx.x - 32];
    }
    if (threadIdx.x == 0 && oi > 0 && !*abort_s) {
      unsigned seen = 0;
      const unsigned target = base + (unsigned)oi * gridDim.x;
      if (!wait_count(&p.hdr->ctr, target, p.err, seen)) {
        *abort_s = 1;
        record_gaveup(p.hdr, 1, 0, oi, target, seen, base, 0);
      }
    }
    if (oi == p.n_ops - 1) pdl_launch_dependents();
    __syncthreads();
    const int limit = oi + kWin;
    if (lane == 0) refill(c_count + depth, limit);  // ops that were beyond the window
    const ChainOp& op = win[oi % kWin];
    const WarpPlan w = warp_plan(op.utotal, op.S, warp);
    bool aborted = *abort_s != 0;
    // every CTA of the cluster is running (op 0) or has finished reading its
    // activation area (later ops: every CTA counted the previous op)
    if (oi == 0) cluster_wait_acquire();
    stage_act<NB>(op, p.nb, act, red, cred, scale_s, aborted);

    auto consume = [&](auto mode_tag) {
      constexpr int MODE = decltype(mode_tag)::value;
      constexpr bool kSwi = MODE == BTF_SWIGLU;
      constexpr int kPan = kSwi ? 2 : 1;
      const int nsp = op.S * kSubPerSlice;
      const uint4* qa_s = reinterpret_cast<const uint4*>(act);
      const uint4* qb_s = qa_s + NB * nsp;
      const float* d_s = reinterpret_cast<const float*>(qb_s + NB * nsp);
      const int* ms_s = reinterpret_cast<const int*>(d_s + NB * nsp);
      auto store = [&](int seg, int row, int m, float v, float u) {
        const int n = op.n[seg];
        if (row >= n || m >= p.nb) return;
        float* y = op.y[seg];
        const int64_t idx = (int64_t)m * op.ld[seg] + row;
        if constexpr (MODE == BTF_STORE) y[idx] = v;
        else if constexpr (MODE == BTF_ADD) y[idx] = __ldcg(y + idx) + v;
        else y[idx] = silu(v) * u;
      };
      if (w.n_units > 0 && !aborted) {
        float2 acc[kPan][NB][2][2];
#pragma unroll
        for (int pp = 0; pp < kPan; ++pp)
#pragma unroll
          for (int m = 0; m < NB; ++m)
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int e = 0; e < 2; ++e) acc[pp][m][h][e] = make_float2(0.0f, 0.0f);
        int j = w.j_lo, ui = 0;
        const int n_steps = w.n_units * (w.j_hi - w.j_lo);
        for (int k = 0; k < n_steps; ++k) {
          int s[kPan];
          uint32_t ph[kPan];
          s[0] = c_slot;
          ph[0] = c_phase;
          if constexpr (kPan == 2) {
            s[1] = c_slot + 1;
            ph[1] = c_phase;
            if (s[1] == depth) {
              s[1] = 0;
              ph[1] ^= 1u;
            }
          }
          bool ok = true;
#pragma unroll
          for (int pp = 0; pp < kPan; ++pp)
            ok = ok && __all_sync(0xffffffffu, mbar_wait_bounded(my_bars + s[pp] * 8, ph[pp], kWaitNs));
          if (!ok) {
            if (lane == 0) {
              atomicCAS(p.err, 0, kErrWaitTimeout);
              record_gaveup(p.hdr, 2, warp, oi, s[0], ph[0], pr_issued, c_count);
            }
            *abort_s = 1;
            aborted = true;
            break;
          }
          uint4 cw[kPan][2][2];
          float sc[kPan][8];
#pragma unroll
          for (int pp = 0; pp < kPan; ++pp)
            load_panel(ring + ((size_t)warp * depth + s[pp]) * kPanelBytes, lane, cw[pp], sc[pp]);
#pragma unroll
          for (int m = 0; m < NB; ++m) {
            const int ai = m * nsp + j * kSubPerSlice + lane;
            const uint4 qa = qa_s[ai], qb = qb_s[ai];
            const float dm = d_s[ai];
            const int ms = ms_s[ai];
#pragma unroll
            for (int pp = 0; pp < kPan; ++pp) panel_fma(cw[pp], sc[pp], qa, qb, dm, ms, acc[pp][m]);
          }
          __syncwarp();
          // release the slots and refill them from the program's panel sequence
          c_count += kPan;
          c_slot += kPan;
          if (c_slot >= depth) {
            c_slot -= depth;
            c_phase ^= 1u;
          }
          if (lane == 0) {
            fence_proxy_async_smem();  // our generic-proxy reads of the slots precede the next async writes
            refill(c_count + depth, limit);
          }
          if (++j == w.j_hi) {  // this warp's part of the unit is done: reduce over lanes
            j = w.j_lo;
            int seg, g;
            locate(w.first + ui * w.stride, kSwi, op.u1, op.u2, seg, g);
            ++ui;
#pragma unroll
            for (int m = 0; m < NB; ++m) {
              float v[kRows], u[kRows];
#pragma unroll
              for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                  v[4 * h + 2 * e] = acc[0][m][h][e].x;
                  v[4 * h + 2 * e + 1] = acc[0][m][h][e].y;
                  acc[0][m][h][e] = make_float2(0.0f, 0.0f);
                  if constexpr (kSwi) {
                    u[4 * h + 2 * e] = acc[kPan - 1][m][h][e].x;
                    u[4 * h + 2 * e + 1] = acc[kPan - 1][m][h][e].y;
                    acc[kPan - 1][m][h][e] = make_float2(0.0f, 0.0f);
                  }
                }
              const int row_l = reduce_rows8(v, lane);
              float up = 0.0f;
              if constexpr (kSwi) {
                reduce_rows8(u, lane);  // same lane -> row map as v
                up = u[0];
              }
              if ((lane & 3) == 0) {
                if (w.G > 1) {  // partial over slices [j_lo, j_hi): combined below
                  pieces[(warp * kMaxNb + m) * 16 + row_l] = v[0];
                  if constexpr (kSwi) pieces[(warp * kMaxNb + m) * 16 + kRows + row_l] = up;
                } else {
                  store(seg, g * kRows + row_l, m, v[0], up);
                }
              }
            }
          }
        }
      }
      if (w.G > 1) {  // CTA-uniform: the G parts of each unit are summed in part order
        __syncthreads();
        if (w.has_work && w.part == 0 && !*abort_s) {
          int seg, g;
          locate(w.first, kSwi, op.u1, op.u2, seg, g);
          const int r = lane & 7, m = lane >> 3;
          if (m < NB) {
            float sg = 0.0f, su = 0.0f;
            for (int ww = warp; ww < warp + w.G; ++ww) {
              sg += pieces[(ww * kMaxNb + m) * 16 + r];
              if constexpr (kSwi) su += pieces[(ww * kMaxNb + m) * 16 + kRows + r];
            }
            store(seg, g * kRows + r, m, sg, su);
          }
        }
      }
    };
    if (op.mode == BTF_STORE) consume(std::integral_constant<int, BTF_STORE>{});
    else if (op.mode == BTF_ADD) consume(std::integral_constant<int, BTF_ADD>{});
    else consume(std::integral_constant<int, BTF_SWIGLU>{});

    // every output of this CTA for op oi is stored: count it (release)
    __syncthreads();
    if (threadIdx.x == 0) {
      __threadfence();
      atomicAdd(&p.hdr->ctr, 1u);
    }
  }

  // after a time-out: let this warp's copies in flight land (bounded) before the
  // shared memory they target is released
  if (*abort_s && lane == 0) {
    int s2 = c_slot;
    uint32_t ph2 = c_phase;
    for (int kk = c_count; kk < pr_issued; ++kk) {
      mbar_wait_bounded(my_bars + s2 * 8, ph2, kWaitNs / 10);
      if (++s2 == depth) {
        s2 = 0;
        ph2 ^= 1u;
      }
    }
  }
  // the last CTA out moves the base to the next launch's start
  if (threadIdx.x == 0) {
    const unsigned prev = atomicAdd(&p.hdr->exit_ctr, 1u);
    if (prev == gridDim.x - 1) {
      p.hdr->base = base + (unsigned)p.n_ops * gridDim.x;
      p.hdr->exit_ctr = 0;
      __threadfence();
    }
  }
}

using ChainFn = void (*)(const ChainParams);
ChainFn chain_fn(int NB) { return NB == 1 ? chain_kernel<1> : chain_kernel<2>; }
int nb_of(int M) { return M <= 1 ? 1 : 2; }

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// CTAs of chain_kernel<NB> co-resident on the device with `smem` bytes each,
// launched in clusters of kCluster (whole clusters; at most two CTAs per SM),
// cached per (kernel, smem).
int resident_ctas(ChainFn fn, int smem, const DeviceInfo& dev) {
  struct Entry { ChainFn fn; int smem; int n; };
  static Entry cache[32];
  static int used = 0;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (cache[i].fn == fn && cache[i].smem == smem) return cache[i].n;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kCluster * 64);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)kCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) != cudaSuccess) clusters = 0;
  cudaGetLastError();
  const int n = std::min(clusters * kCluster, dev.sm_count * 2 / kCluster * kCluster);
  if (used < 32) cache[used++] = Entry{fn, smem, n};
  return n;
}

}  // namespace

int chain_setup(DeviceInfo& d) {
  const int dyn = d.optin_smem - 1024;
  for (int NB : {1, 2}) {
    const cudaError_t e = cudaFuncSetAttribute(chain_fn(NB), cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(chain_kernel)");
  }
  return BTF_OK;
}

}  // namespace btf

using namespace btf;

extern "C" {

int64_t btf_chain_program_bytes(int n_ops) {
  if (n_ops < 1) return 0;
  return (int64_t)sizeof(ChainHeader) + (int64_t)n_ops * (int64_t)sizeof(ChainOp);
}

int btf_chain_encode(const btf_chain_op* ops, int n_ops, int M, void* program, btf_chain* chain) {
  if (!ops || n_ops < 1 || !program || !chain)
    return fail(BTF_ERR_ARG, "btf_chain_encode: need ops, n_ops >= 1, a program buffer and a chain");
  if (!aligned(program, 256)) return fail(BTF_ERR_ARG, "btf_chain_encode: the program buffer must be 256-byte aligned");
  if (M < 1 || M > kMaxNb) return fail(BTF_ERR_ARG, "btf_chain_encode: 1 <= M <= %d (got %d)", kMaxNb, M);
  const DeviceInfo* dev = current_device();
  if (!dev) return BTF_ERR_STATE;
  std::vector<uint8_t> buf((size_t)btf_chain_program_bytes(n_ops), 0);
  ChainOp* enc = reinterpret_cast<ChainOp*>(buf.data() + sizeof(ChainHeader));
  int max_nsp = 0;
  for (int i = 0; i < n_ops; ++i) {
    const btf_chain_op& o = ops[i];
    const int nseg = o.nseg, K = o.K, mode = o.mode;
    if (nseg < 1 || nseg > 3) return fail(BTF_ERR_ARG, "btf_chain_encode: op %d: 1..3 segments (got %d)", i, nseg);
    if (mode != BTF_STORE && mode != BTF_ADD && mode != BTF_SWIGLU)
      return fail(BTF_ERR_ARG, "btf_chain_encode: op %d: bad mode %d", i, mode);
    if (mode == BTF_SWIGLU && (nseg != 2 || o.segs[0].N != o.segs[1].N))
      return fail(BTF_ERR_ARG, "btf_chain_encode: op %d: swiglu needs gate+up segments with the same N", i);
    if (K <= 0 || K % 128) return fail(BTF_ERR_ARG, "btf_chain_encode: op %d: K must be a positive multiple of 128", i);
    if (!o.x || !aligned(o.x, 4) || o.ldx < K)
      return fail(BTF_ERR_ARG, "btf_chain_encode: op %d: x null/misaligned or ldx < K", i);
    if (o.normw && !aligned(o.normw, 4)) return fail(BTF_ERR_ARG, "btf_chain_encode: op %d: normw misaligned", i);
    ChainOp& e = enc[i];
    int units[3] = {0, 0, 0};
    for (int s = 0; s < nseg; ++s) {
      const btf_gemv_seg& g = o.segs[s];
      if (!g.panels || !aligned(g.panels, 16) || g.N <= 0)
        return fail(BTF_ERR_ARG, "btf_chain_encode: op %d segment %d: null/misaligned panels or N <= 0", i, s);
      const bool needs_y = !(mode == BTF_SWIGLU && s == 1);
      if (needs_y && (!g.y || !aligned(g.y, 4) || g.ldy < g.N))
        return fail(BTF_ERR_ARG, "btf_chain_encode: op %d segment %d needs y and ldy >= N", i, s);
      e.pan[s] = static_cast<const uint8_t*>(g.panels);
      e.y[s] = g.y;
      e.n[s] = g.N;
      e.ld[s] = g.ldy;
      units[s] = (int)groups_of(g.N);
    }
    if (mode == BTF_SWIGLU) units[1] = 0;
    e.u1 = units[0];
    e.u2 = units[0] + units[1];
    e.utotal = units[0] + units[1] + units[2];
    e.K = K;
    e.S = (int)slices_of(K);
    e.nsub = K / 32;
    e.mode = mode;
    e.x = o.x;
    e.ldx = o.ldx;
    e.normw = o.normw;
    e.eps = o.eps;
    max_nsp = std::max(max_nsp, e.S * kSubPerSlice);
  }
  const int NB = nb_of(M);
  // ring slots per warp: fill the two-CTA budget; one CTA per SM with the whole
  // opt-in budget when the activation leaves fewer than 3 slots a warp
  int depth = 0, smem = 0;
  for (int budget : {kSmemTarget, dev->optin_smem - 1024}) {
    const ChainSmem base(NB, max_nsp, 0);
    const int room = budget - base.total;
    depth = room > 0 ? std::min(room / (kWarps * (kPanelBytes + 8)), 64) : 0;
    smem = ChainSmem(NB, max_nsp, depth).total;
    if (depth >= 3) break;
  }
  if (depth < 2)
    return fail(BTF_ERR_UNSUPPORTED, "btf_chain_encode: K=%d with M=%d leaves no room for the weight ring",
                max_nsp * 32, M);
  const int grid = resident_ctas(chain_fn(NB), smem, *dev);
  if (grid < kCluster) return fail(BTF_ERR_UNSUPPORTED, "btf_chain_encode: no cluster of chain_kernel CTAs fits");
  const cudaError_t e = cudaMemcpy(program, buf.data(), buf.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(e, "btf_chain_encode: upload");
  chain->program = program;
  chain->n_ops = n_ops;
  chain->M = M;
  chain->max_K = max_nsp * 32;
  chain->grid = grid;
  chain->depth = depth;
  chain->smem = smem;
  return BTF_OK;
}

int btf_chain_run(const btf_chain* chain, void* stream) {
  if (!chain || !chain->program || chain->n_ops < 1 || chain->M < 1 || chain->M > kMaxNb ||
      chain->grid < kCluster || chain->grid % kCluster ||
      chain->depth < 2)
    return fail(BTF_ERR_ARG, "btf_chain_run: chain not encoded");
  const DeviceInfo* dev = current_device();
  if (!dev) return BTF_ERR_STATE;
  ChainParams p{};
  p.hdr = static_cast<ChainHeader*>(chain->program);
  p.ops = reinterpret_cast<const ChainOp*>(static_cast<const uint8_t*>(chain->program) + sizeof(ChainHeader));
  p.n_ops = chain->n_ops;
  p.nb = chain->M;
  p.depth = chain->depth;
  p.max_nsp = chain->max_K / 32;
  p.err = dev->err_word;
  const int NB = nb_of(chain->M);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(chain->grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = (size_t)chain->smem;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)kCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = BTF_CHAIN_PDL ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, chain_fn(NB), p);
  return e == cudaSuccess ? launch_status("chain_kernel") : cuda_fail(e, "chain_kernel launch");
}

}  // extern "C"
