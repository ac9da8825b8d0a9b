// Ternary GEMV / small-batch GEMM on the panel layout (CUDA cores, dp4a).
//
// Replaces gemv_kernel<NB, MODE> / launch_gemv of the reference
// (src/cuda/kernels.cu:211-334, :776-822). Same math per output row r and
// activation row m:
//   y[m][r] {=, +=} sum_s  (fp16 scale[r][s/4] * d[m][s]) * idot[m][r][s],
//   idot = sum over the 32 columns of sub-block s of trit * q  (exact int32),
// with the swiglu epilogue silu(gate) * up.
//
// Work decomposition (B200 design, not the reference's):
//   - one warp owns a tile of RW output rows (inside one 16-row group) and
//     walks every 1024-column slice of those rows; lane l always handles
//     sub-block l of the slice, so its activation words for the slice are
//     loaded once and reused for all RW rows;
//   - the codes of the RW rows are 8-byte streaming loads (L1 bypass), the
//     RW fp16 scales of a lane one vector load (they sit contiguous in the
//     panel), and the next slice's codes/scales are loaded before the current
//     slice is computed, so two slices per warp are in flight;
//   - per (row, sub-block) the code dot uses four unshifted code masks
//     (code * 4^k per byte) with unsigned x signed dp4a, one accumulator per
//     k, recombined by exact arithmetic shifts; the -sum(q) correction and the
//     int->float conversion are folded into one biased add (see kMagicInt).
#include <algorithm>

#include "common.cuh"

namespace btf {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxSeg = 3;

struct GemvParams {
  const uint8_t* pan[kMaxSeg];
  float* y[kMaxSeg];
  int n[kMaxSeg];
  int ldy[kMaxSeg];
  int t1, t2, ttotal;  // cumulative warp-tile counts of the segments
  int K, S, nsub;
  int m0, nb;  // activation rows m0 .. m0 + nb - 1 (nb <= NB)
  const int8_t* q;
  const float* d;
  const int32_t* s;
};

// Biased trit dot of one (row, sub-block): returns kMagicInt + idot, where
// magic_s = kMagicInt - sum(q). w0/w1: the two T2 words; qa/qb: the eight
// int8x4 activation words (columns 0..15 and 16..31 of the sub-block).
__device__ __forceinline__ int sub_dot_biased(uint32_t w0, uint32_t w1, const uint4& qa, const uint4& qb,
                                              int magic_s) {
  int c0 = dp4a_us(w0 & 0x03030303u, qa.x, magic_s);
  int c1 = dp4a_us(w0 & 0x0c0c0c0cu, qa.y, 0);
  int c2 = dp4a_us(w0 & 0x30303030u, qa.z, 0);
  int c3 = dp4a_us(w0 & 0xc0c0c0c0u, qa.w, 0);
  c0 = dp4a_us(w1 & 0x03030303u, qb.x, c0);
  c1 = dp4a_us(w1 & 0x0c0c0c0cu, qb.y, c1);
  c2 = dp4a_us(w1 & 0x30303030u, qb.z, c2);
  c3 = dp4a_us(w1 & 0xc0c0c0c0u, qb.w, c3);
  // c_k = 4^k * (code dot of slot k): the shifts are exact.
  return c0 + (c1 >> 2) + (c2 >> 4) + (c3 >> 6);
}

// RWO fp16 scales (RWO consecutive rows, one block) as RWO/2 half2 words.
template <int RWO>
__device__ __forceinline__ void load_scales(const uint8_t* p, uint32_t (&h)[(RWO + 1) / 2]) {
  if constexpr (RWO == 16) {
    const uint4 a = ld_stream_v4(p), b = ld_stream_v4(p + 16);
    h[0] = a.x; h[1] = a.y; h[2] = a.z; h[3] = a.w;
    h[4] = b.x; h[5] = b.y; h[6] = b.z; h[7] = b.w;
  } else if constexpr (RWO == 8) {
    const uint4 a = ld_stream_v4(p);
    h[0] = a.x; h[1] = a.y; h[2] = a.z; h[3] = a.w;
  } else if constexpr (RWO == 4) {
    const uint2 a = ld_stream_v2(p);
    h[0] = a.x; h[1] = a.y;
  } else {
    static_assert(RWO == 2, "RWO must be 2, 4, 8 or 16");
    h[0] = *reinterpret_cast<const uint32_t*>(p);
  }
}

__device__ __forceinline__ float half_lo(uint32_t h2) { return __half2float(__ushort_as_half((unsigned short)(h2 & 0xffffu))); }
__device__ __forceinline__ float half_hi(uint32_t h2) { return __half2float(__ushort_as_half((unsigned short)(h2 >> 16))); }

template <int RWO>
__device__ __forceinline__ float scale_of(const uint32_t (&h)[(RWO + 1) / 2], int i) {
  return (i & 1) ? half_hi(h[i >> 1]) : half_lo(h[i >> 1]);
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// NB: activation rows per pass; RW: rows loaded per warp tile; MODE: BTF_STORE / BTF_ADD / BTF_SWIGLU.
// For swiglu a tile is RW/2 gate rows plus the same RW/2 rows of up.
template <int NB, int RW, int MODE>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const GemvParams p) {
  constexpr bool kSwi = MODE == BTF_SWIGLU;
  constexpr int RWO = kSwi ? RW / 2 : RW;  // output rows per tile
  static_assert(kRows % RWO == 0, "a tile must sit inside one row group");
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (t >= p.ttotal) return;
  const int seg = kSwi ? 0 : (t >= p.t1) + (t >= p.t2);
  const int lt = t - (seg == 0 ? 0 : seg == 1 ? p.t1 : p.t2);
  const int row0 = lt * RWO;
  const int g = row0 / kRows, r_in = row0 % kRows;
  // select by value: indexing the kernel-parameter arrays with a run-time
  // index would copy them to local memory
  const uint8_t* base_a = seg == 0 ? p.pan[0] : seg == 1 ? p.pan[1] : p.pan[2];
  const uint8_t* base_b = kSwi ? p.pan[1] : base_a;
  const int n_seg = seg == 0 ? p.n[0] : seg == 1 ? p.n[1] : p.n[2];
  const int ldy_seg = seg == 0 ? p.ldy[0] : seg == 1 ? p.ldy[1] : p.ldy[2];
  float* y_seg = seg == 0 ? p.y[0] : seg == 1 ? p.y[1] : p.y[2];
  const int64_t S = p.S;
  const int64_t gbase = (int64_t)g * S * kPanelBytes;

  float acc[RW][NB];
#pragma unroll
  for (int i = 0; i < RW; ++i)
#pragma unroll
    for (int m = 0; m < NB; ++m) acc[i][m] = 0.0f;

  // prefetch registers: codes of the RW rows and the scales, for one slice
  uint2 cur[RW];
  uint32_t sca[(RWO + 1) / 2], scb[(RWO + 1) / 2];
  auto load_slice = [&](int64_t j, uint2 (&c)[RW], uint32_t (&sa)[(RWO + 1) / 2], uint32_t (&sb)[(RWO + 1) / 2]) {
    const uint8_t* pa = base_a + gbase + j * kPanelBytes;
    const uint8_t* pb = base_b + gbase + j * kPanelBytes;
#pragma unroll
    for (int i = 0; i < RW; ++i) {
      const uint8_t* pp = (kSwi && i >= RWO) ? pb : pa;
      const int r = r_in + (kSwi ? (i % RWO) : i);
      c[i] = ld_stream_v2(pp + code_offset(r, lane));
    }
    load_scales<RWO>(pa + scale_offset(r_in, lane >> 2), sa);
    if constexpr (kSwi) load_scales<RWO>(pb + scale_offset(r_in, lane >> 2), sb);
  };
  load_slice(0, cur, sca, scb);

  for (int64_t j = 0; j < S; ++j) {
    uint2 nxt[RW];
    uint32_t nsa[(RWO + 1) / 2], nsb[(RWO + 1) / 2];
    if (j + 1 < S) load_slice(j + 1, nxt, nsa, nsb);

    const int sbk = (int)j * kSubPerSlice + lane;
    const bool valid = sbk < p.nsub;
#pragma unroll
    for (int m = 0; m < NB; ++m) {
      uint4 qa = make_uint4(0, 0, 0, 0), qb = qa;
      float dm = 0.0f;
      int magic_s = kMagicInt;
      if (valid && m < p.nb) {
        const int64_t row = p.m0 + m;
        const int8_t* qp = p.q + row * p.K + (int64_t)sbk * 32;
        qa = ld_nc_v4(qp);
        qb = ld_nc_v4(qp + 16);
        dm = p.d[row * p.nsub + sbk];
        magic_s = kMagicInt - p.s[row * p.nsub + sbk];
      }
#pragma unroll
      for (int i = 0; i < RW; ++i) {
        const float sc = (kSwi && i >= RWO) ? scale_of<RWO>(scb, i - RWO) : scale_of<RWO>(sca, i);
        const int biased = sub_dot_biased(cur[i].x, cur[i].y, qa, qb, magic_s);
        const float fi = __int_as_float(biased) - kMagicFloat;
        acc[i][m] = fmaf(sc * dm, fi, acc[i][m]);
      }
    }
    if (j + 1 < S) {
#pragma unroll
      for (int i = 0; i < RW; ++i) cur[i] = nxt[i];
#pragma unroll
      for (int i = 0; i < (RWO + 1) / 2; ++i) {
        sca[i] = nsa[i];
        scb[i] = nsb[i];
      }
    }
  }

  // reduce over the 32 lanes; lane i then owns output row row0 + i
#pragma unroll
  for (int m = 0; m < NB; ++m) {
    float mine = 0.0f, mine_up = 0.0f;
#pragma unroll
    for (int i = 0; i < RW; ++i) {
      const float v = warp_sum(acc[i][m]);
      if (kSwi && i >= RWO) {
        if (lane == i - RWO) mine_up = v;
      } else if (lane == i) {
        mine = v;
      }
    }
    const int row = row0 + lane;
    if (lane < RWO && row < n_seg && m < p.nb) {
      float* yp = y_seg + (int64_t)(p.m0 + m) * ldy_seg + row;
      if constexpr (MODE == BTF_STORE) *yp = mine;
      else if constexpr (MODE == BTF_ADD) *yp += mine;
      else *yp = silu(mine) * mine_up;
    }
  }
}

// Exact idot dump (parity/debug): one thread per (m, row, sub-block).
__global__ void __launch_bounds__(256)
    idot_kernel(const uint8_t* __restrict__ pan, int N, int K, int M, const int8_t* __restrict__ q,
                const int32_t* __restrict__ s, int32_t* __restrict__ idot) {
  const int nsub = K / 32;
  const int64_t S = slices_of(K);
  const int64_t total = (int64_t)M * N * nsub;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int sbk = (int)(i % nsub);
    const int64_t mr = i / nsub;
    const int r = (int)(mr % N), m = (int)(mr / N);
    const uint8_t* pp = pan + panel_offset(r / kRows, sbk / kSubPerSlice, S) + code_offset(r % kRows, sbk % kSubPerSlice);
    const uint2 w = *reinterpret_cast<const uint2*>(pp);
    const int8_t* qp = q + (int64_t)m * K + (int64_t)sbk * 32;
    const uint4 qa = *reinterpret_cast<const uint4*>(qp), qb = *reinterpret_cast<const uint4*>(qp + 16);
    const int magic_s = kMagicInt - s[(int64_t)m * nsub + sbk];
    idot[i] = sub_dot_biased(w.x, w.y, qa, qb, magic_s) - kMagicInt;
  }
}

using KernelFn = void (*)(const GemvParams);

template <int MODE>
KernelFn pick(int NB) {
  switch (NB) {
    case 1: return gemv_kernel<1, 8, MODE>;
    case 2: return gemv_kernel<2, 8, MODE>;
    case 4: return gemv_kernel<4, 4, MODE>;
    default: return gemv_kernel<8, 4, MODE>;
  }
}
// Output rows per warp tile for a given (NB, mode); must match pick().
int rows_per_tile(int NB, int mode) {
  const int rw = NB <= 2 ? 8 : 4;
  return mode == BTF_SWIGLU ? rw / 2 : rw;
}

bool aligned(const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; }

}  // namespace

int gemv_setup(const DeviceInfo&) { return BTF_OK; }

}  // namespace btf

using namespace btf;

extern "C" {

int btf_gemv_max_nb(int K) { return (K > 0 && K % 128 == 0) ? 8 : 0; }

int btf_gemv(const btf_gemv_seg* segs, int nseg, int K, int M, btf_q8act act, int mode, void* stream) {
  if (M <= 0) return BTF_OK;
  if (!segs || nseg < 1 || nseg > kMaxSeg) return fail(BTF_ERR_ARG, "btf_gemv: 1..3 segments (got %d)", nseg);
  if (mode != BTF_STORE && mode != BTF_ADD && mode != BTF_SWIGLU) return fail(BTF_ERR_ARG, "btf_gemv: bad mode %d", mode);
  if (mode == BTF_SWIGLU && (nseg != 2 || segs[0].N != segs[1].N))
    return fail(BTF_ERR_ARG, "btf_gemv: swiglu needs gate+up segments with the same N");
  if (K <= 0 || K % 128) return fail(BTF_ERR_ARG, "btf_gemv: K must be a positive multiple of 128 (K=%d)", K);
  if (!act.q || !act.d || !act.s || !aligned(act.q, 16) || !aligned(act.d, 4) || !aligned(act.s, 4))
    return fail(BTF_ERR_ARG, "btf_gemv: activation pointers null or misaligned (q needs 16 B)");
  for (int i = 0; i < nseg; ++i) {
    if (!segs[i].panels || !aligned(segs[i].panels, 16) || segs[i].N <= 0)
      return fail(BTF_ERR_ARG, "btf_gemv: segment %d has a null/misaligned panel buffer or N <= 0", i);
    const bool needs_y = !(mode == BTF_SWIGLU && i == 1);
    if (needs_y && (!segs[i].y || segs[i].ldy < segs[i].N))
      return fail(BTF_ERR_ARG, "btf_gemv: segment %d needs y and ldy >= N", i);
  }
  const DeviceInfo* dev = current_device();
  if (!dev) return BTF_ERR_STATE;

  GemvParams p{};
  for (int i = 0; i < nseg; ++i) {
    p.pan[i] = static_cast<const uint8_t*>(segs[i].panels);
    p.y[i] = segs[i].y;
    p.n[i] = segs[i].N;
    p.ldy[i] = segs[i].ldy;
  }
  p.K = K;
  p.S = (int)slices_of(K);
  p.nsub = K / 32;
  p.q = act.q;
  p.d = act.d;
  p.s = act.s;
  const cudaStream_t st = (cudaStream_t)stream;
  constexpr int kMaxNb = 8;
  for (int m0 = 0; m0 < M; m0 += kMaxNb) {
    const int nb = std::min(kMaxNb, M - m0);
    const int NB = nb <= 1 ? 1 : nb <= 2 ? 2 : nb <= 4 ? 4 : 8;
    const int rwo = rows_per_tile(NB, mode);
    int tiles[kMaxSeg] = {0, 0, 0};
    const int used = mode == BTF_SWIGLU ? 1 : nseg;
    for (int i = 0; i < used; ++i) tiles[i] = (segs[i].N + rwo - 1) / rwo;
    p.t1 = tiles[0];
    p.t2 = tiles[0] + tiles[1];
    p.ttotal = tiles[0] + tiles[1] + tiles[2];
    p.m0 = m0;
    p.nb = nb;
    const KernelFn fn = mode == BTF_STORE ? pick<BTF_STORE>(NB) : mode == BTF_ADD ? pick<BTF_ADD>(NB) : pick<BTF_SWIGLU>(NB);
    const int grid = (p.ttotal + kWarps - 1) / kWarps;
    fn<<<grid, kThreads, 0, st>>>(p);
    if (int rc = launch_status("gemv_kernel")) return rc;
  }
  return BTF_OK;
}

int btf_gemv_idot(const void* panels, int N, int K, int M, btf_q8act act, int32_t* idot, void* stream) {
  if (M <= 0) return BTF_OK;
  if (!panels || !idot || !act.q || !act.s || N <= 0 || K <= 0 || K % 128 || !aligned(act.q, 16) ||
      !aligned(panels, 16))
    return fail(BTF_ERR_ARG, "btf_gemv_idot: bad arguments");
  const DeviceInfo* dev = current_device();
  if (!dev) return BTF_ERR_STATE;
  const int64_t total = (int64_t)M * N * (K / 32);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((total + 255) / 256, (int64_t)dev->sm_count * 32));
  idot_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(static_cast<const uint8_t*>(panels), N, K, M, act.q, act.s, idot);
  return launch_status("idot_kernel");
}

}  // extern "C"
