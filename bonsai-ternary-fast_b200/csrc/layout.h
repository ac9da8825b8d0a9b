// PTQ1_0 block decoding shared by the CUDA repack kernels and the host twin.
//
// A PTQ1_0 block (the GGUF source format) holds 128 trits and an fp16 scale in
// 28 bytes: bytes 0..15 carry elements m + 16n (n = 0..4), bytes 16..23 carry
// 80 + m + 8n, bytes 24..25 carry 120 + h + 2n (n = 0..3), five base-3 digits
// per byte with element n = 0 the most significant; digit n of byte b is
// ((uint8)(b * 3^n) * 3) >> 8 = trit + 1; bytes 26..27 hold the scale.
// (Format: ref/bonsai-decoder/include/bd/types.hpp:67-78 and
// docs/packed-layout.md:6-17 of the reference.)
//
// The decoded form is the eight T2 code words of the block
// (include/btf/packed.hpp:6-14 of the reference): column e goes to word e / 16
// at bit 8 * (e % 4) + 2 * ((e / 4) % 4), so (word >> 2k) & 0x03030303 is four
// codes lined up with the int8x4 activation word of columns 16w + 4k .. +3.
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define BTF_HD __host__ __device__ __forceinline__
#define BTF_UNROLL _Pragma("unroll")
#else
#define BTF_HD inline
#define BTF_UNROLL
#endif

namespace btf {

// Shift of column e inside its T2 word.
BTF_HD constexpr int t2_bit(int e) { return 8 * (e & 3) + 2 * ((e >> 2) & 3); }

// trit + 1 (0..2) held as base-3 digit n of byte b.
BTF_HD uint32_t ptq_digit(uint32_t b, uint32_t pow3n) { return (((b * pow3n) & 0xffu) * 3u) >> 8; }

// Decodes one 28-byte block given as its first 26 bytes (byte(i) accessor)
// and returns the eight T2 words.
template <class ByteAt>
BTF_HD void ptq_block_to_t2(const ByteAt& byte, uint32_t w[8]) {
  BTF_UNROLL
  for (int i = 0; i < 8; ++i) w[i] = 0;
  const uint32_t p3[5] = {1u, 3u, 9u, 27u, 81u};
  BTF_UNROLL
  for (int m = 0; m < 16; ++m) {  // elements m + 16n
    const uint32_t b = byte(m);
    BTF_UNROLL
    for (int n = 0; n < 5; ++n) {
      const int e = m + 16 * n;
      w[e >> 4] |= ptq_digit(b, p3[n]) << t2_bit(e);
    }
  }
  BTF_UNROLL
  for (int m = 0; m < 8; ++m) {  // elements 80 + m + 8n
    const uint32_t b = byte(16 + m);
    BTF_UNROLL
    for (int n = 0; n < 5; ++n) {
      const int e = 80 + m + 8 * n;
      w[e >> 4] |= ptq_digit(b, p3[n]) << t2_bit(e);
    }
  }
  BTF_UNROLL
  for (int h = 0; h < 2; ++h) {  // elements 120 + h + 2n
    const uint32_t b = byte(24 + h);
    BTF_UNROLL
    for (int n = 0; n < 4; ++n) {
      const int e = 120 + h + 2 * n;
      w[e >> 4] |= ptq_digit(b, p3[n]) << t2_bit(e);
    }
  }
}

// Row-interleaved ("quad") form used by the panel layout: for 4 rows k = 0..3
// and one 16-column half of a sub-block, word i (columns 4i .. 4i+3) holds the
// code of row k, column 4i + j in byte j at bits 2k .. 2k+1, so
//   word & (0x03030303 << 2k)  ==  4^k * (the four codes of row k)
// lines up with the int8x4 activation word of those columns. The map is a 4x4
// transpose of 2-bit fields and is its own inverse: t2_quad_transpose turns
// the 4 rows' T2 words of a half (t[k]) into the quad words and back.
BTF_HD void t2_quad_transpose(const uint32_t in[4], uint32_t out[4]) {
  BTF_UNROLL
  for (int a = 0; a < 4; ++a) {
    uint32_t w = 0;
    BTF_UNROLL
    for (int b = 0; b < 4; ++b) w |= ((in[b] >> (2 * a)) & 0x03030303u) << (2 * b);
    out[a] = w;
  }
}

// Panel geometry (see include/btf_b200.h).
constexpr int kQuadBytes = 1024;  // one row quad's codes in a panel
constexpr int kHalfBytes = 512;   // one 16-column half of a quad
constexpr int kScaleBase = 2048;

BTF_HD void copy16(uint8_t* dst, const uint32_t w[4]) {
#if defined(__CUDA_ARCH__)
  *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
#else
  for (int i = 0; i < 4; ++i)
    for (int b = 0; b < 4; ++b) dst[4 * i + b] = (uint8_t)(w[i] >> (8 * b));
#endif
}
BTF_HD void load16(const uint8_t* src, uint32_t w[4]) {
#if defined(__CUDA_ARCH__)
  const uint4 v = *reinterpret_cast<const uint4*>(src);
  w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
#else
  for (int i = 0; i < 4; ++i)
    w[i] = (uint32_t)src[4 * i] | ((uint32_t)src[4 * i + 1] << 8) | ((uint32_t)src[4 * i + 2] << 16) |
           ((uint32_t)src[4 * i + 3] << 24);
#endif
}

// Writes one 128-column block (block bb of the panel's slice) of a row quad
// (quad h of the panel) from the 4 rows' T2 words tw[k][0..7] and scales.
BTF_HD void store_quad_block(uint8_t* pan, int h, int bb, const uint32_t tw[4][8], const uint16_t sc[4]) {
  BTF_UNROLL
  for (int sb = 0; sb < 4; ++sb)
    BTF_UNROLL
    for (int v = 0; v < 2; ++v) {
      const uint32_t in[4] = {tw[0][2 * sb + v], tw[1][2 * sb + v], tw[2][2 * sb + v], tw[3][2 * sb + v]};
      uint32_t out[4];
      t2_quad_transpose(in, out);
      copy16(pan + h * kQuadBytes + v * kHalfBytes + (bb * 4 + sb) * 16, out);
    }
  uint8_t* sp = pan + kScaleBase + bb * 16 + h * 8;
  BTF_UNROLL
  for (int k = 0; k < 4; ++k) {
    sp[2 * k] = (uint8_t)(sc[k] & 0xffu);
    sp[2 * k + 1] = (uint8_t)(sc[k] >> 8);
  }
}

// Inverse of store_quad_block: the 4 rows' T2 words and scales of one block.
BTF_HD void load_quad_block(const uint8_t* pan, int h, int bb, uint32_t tw[4][8], uint16_t sc[4]) {
  BTF_UNROLL
  for (int sb = 0; sb < 4; ++sb)
    BTF_UNROLL
    for (int v = 0; v < 2; ++v) {
      uint32_t in[4], out[4];
      load16(pan + h * kQuadBytes + v * kHalfBytes + (bb * 4 + sb) * 16, in);
      t2_quad_transpose(in, out);
      BTF_UNROLL
      for (int k = 0; k < 4; ++k) tw[k][2 * sb + v] = out[k];
    }
  const uint8_t* sp = pan + kScaleBase + bb * 16 + h * 8;
  BTF_UNROLL
  for (int k = 0; k < 4; ++k) sc[k] = (uint16_t)(sp[2 * k] | (sp[2 * k + 1] << 8));
}

}  // namespace btf
