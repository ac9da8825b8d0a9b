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

}  // namespace btf
