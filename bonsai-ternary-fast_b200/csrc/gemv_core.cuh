// Inner arithmetic of the ternary GEMV on the panel layout, shared by the
// single-launch GEMV (gemv.cu) and the persistent GEMV chain (chain.cu).
//
// Per output row r, activation row m and 32-column sub-block s the reference
// computes (src/cuda/kernels.cu:227-334, src/emu_decoder.cpp:143-165)
//   idot = sum over the 32 columns of trit * q   (exact int32)
//   y[m][r] += (fp16 scale[r][s/4] * d[m][s]) * (float)idot.
// Here the codes are quad-interleaved (one 32-bit word = 4 rows x 4 columns,
// row k at bits 2k..2k+1 of each byte), so one AND with 0x03030303 << 2k gives
// 4^k x the codes of row k aligned with the int8x4 activation word: each
// (row, 4 columns) is one LOP3 + one unsigned x signed dp4a, and the 4^k is
// removed once per (row, sub-block) by an exact arithmetic shift. The
// subtraction of sum(q) (code = trit + 1) and the int -> float conversion are
// one biased integer add (kMagicInt).
#pragma once
#include "common.cuh"

namespace btf {
namespace core {

// Per-row code dots of one row quad over one 32-column sub-block. cw0/cw1:
// the quad words of columns 0..15 / 16..31; qa/qb: the activation words of the
// same columns. c[k] = 4^k * code_dot(row k) accumulated onto c[k].
__device__ __forceinline__ void quad_dots(const uint4& cw0, const uint4& cw1, const uint4& qa, const uint4& qb,
                                          int c[4]) {
  const uint32_t w[8] = {cw0.x, cw0.y, cw0.z, cw0.w, cw1.x, cw1.y, cw1.z, cw1.w};
  const uint32_t a[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    c[0] = dp4a_us(w[i] & 0x03030303u, a[i], c[0]);
    c[1] = dp4a_us(w[i] & 0x0c0c0c0cu, a[i], c[1]);
    c[2] = dp4a_us(w[i] & 0x30303030u, a[i], c[2]);
    c[3] = dp4a_us(w[i] & 0xc0c0c0c0u, a[i], c[3]);
  }
}

// kMagicInt + idot of row k from its quad accumulator (exact shift) and
// magic_s = kMagicInt - sum(q). Read as float bits it is 12582912 + idot.
template <int k>
__device__ __forceinline__ int biased_idot(int c, int magic_s) { return (c >> (2 * k)) + magic_s; }

__device__ __forceinline__ float half_lo(uint32_t h2) { return __half2float(__ushort_as_half((unsigned short)(h2 & 0xffffu))); }
__device__ __forceinline__ float half_hi(uint32_t h2) { return __half2float(__ushort_as_half((unsigned short)(h2 >> 16))); }
// silu(g) = g / (1 + e^-g), the reference's swiglu epilogue (kernels.cu:318-320)
__device__ __forceinline__ float silu(float x) { return x / (1.0f + expf(-x)); }

// Sums v[0..7] over the 32 lanes by recursive halving: after 9 shuffles lane l
// holds in v[0] the total of row r(l) = 4*bit4(l) + 2*bit3(l) + bit2(l) (the 4
// lanes of a group of four hold the same row). Returns r(l).
__device__ __forceinline__ int reduce_rows8(float (&v)[8], int lane) {
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // keep rows 0..3 (b4 = 0) or 4..7 (b4 = 1)
    const float send = b4 ? v[i] : v[i + 4];
    const float keep = b4 ? v[i + 4] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b3 ? v[i] : v[i + 2];
    const float keep = b3 ? v[i + 2] : v[i];
    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  {
    const float send = b2 ? v[0] : v[1];
    const float keep = b2 ? v[1] : v[0];
    v[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 2);
  v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
  return 4 * (int)b4 + 2 * (int)b3 + (int)b2;
}

// Codes (quad h, half v) and fp16 scales (as fp32, row order) of one panel in
// shared memory for lane `lane` (sub-block `lane` of the slice).
__device__ __forceinline__ void load_panel(const uint8_t* pan, int lane, uint4 (&cw)[2][2], float (&sc)[8]) {
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int v = 0; v < 2; ++v) cw[h][v] = *reinterpret_cast<const uint4*>(pan + h * 1024 + v * 512 + lane * 16);
  const uint4 s4 = *reinterpret_cast<const uint4*>(pan + 2048 + (lane >> 2) * 16);
  sc[0] = half_lo(s4.x); sc[1] = half_hi(s4.x);
  sc[2] = half_lo(s4.y); sc[3] = half_hi(s4.y);
  sc[4] = half_lo(s4.z); sc[5] = half_hi(s4.z);
  sc[6] = half_lo(s4.w); sc[7] = half_hi(s4.w);
}

// One panel against the staged activation of one row: acc[h][e] accumulates
// rows (4h + 2e, 4h + 2e + 1) with packed f32x2 FMA, per sub-block
// (scale * d) * (float)idot. qa/qb: the lane's activation words; dm: d of the
// block; ms: kMagicInt - sum(q).
__device__ __forceinline__ void panel_fma(const uint4 (&cw)[2][2], const float (&sc)[8], const uint4& qa,
                                          const uint4& qb, float dm, int ms, float2 (&acc)[2][2]) {
  const float2 d2 = make_float2(dm, dm);
  const float2 nmagic = make_float2(-kMagicFloat, -kMagicFloat);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    int c[4] = {0, 0, 0, 0};
    quad_dots(cw[h][0], cw[h][1], qa, qb, c);
    const float2 f01 = __fadd2_rn(make_float2(__int_as_float(biased_idot<0>(c[0], ms)),
                                              __int_as_float(biased_idot<1>(c[1], ms))), nmagic);
    const float2 f23 = __fadd2_rn(make_float2(__int_as_float(biased_idot<2>(c[2], ms)),
                                              __int_as_float(biased_idot<3>(c[3], ms))), nmagic);
    const int r = 4 * h;
    const float2 s01 = __fmul2_rn(make_float2(sc[r], sc[r + 1]), d2);
    const float2 s23 = __fmul2_rn(make_float2(sc[r + 2], sc[r + 3]), d2);
    acc[h][0] = __ffma2_rn(s01, f01, acc[h][0]);
    acc[h][1] = __ffma2_rn(s23, f23, acc[h][1]);
  }
}

}  // namespace core
}  // namespace btf
