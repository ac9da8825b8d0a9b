// Host twin of the panel repack: PTQ1_0 rows -> panel layout on the CPU, the
// same bytes btf_repack_panels writes on the device. Replaces the reference's
// host repack (btf::repack_rows / btf::repack, src/repack.cpp:16-45), which
// fills T2 with a thread pool; here rows are split across std::threads in
// contiguous row-group ranges.
#include <algorithm>
#include <cstring>
#include <thread>
#include <vector>

#include "btf_b200.h"
#include "layout.h"

namespace btf {
int fail(int status, const char* fmt, ...);
namespace {

constexpr int64_t kRowsH = BTF_PANEL_ROWS;
constexpr int64_t kPanelH = BTF_PANEL_BYTES;

// trit + 1 (0..2) held as base-3 digit n of byte b (pow3n = 3^n): the rule of
// ptq_digit in layout.h.
inline uint32_t digit(uint32_t b, uint32_t pow3n) { return (((b * pow3n) & 0xffu) * 3u) >> 8; }

// In a panel, the codes of a row quad for one 16-column half are 16 bytes in
// column order, byte = code(row 0) | code(row 1) << 2 | code(row 2) << 4 |
// code(row 3) << 6 (the bytes store_quad_block in layout.h writes on the
// device). t[k][b] holds the five codes of source byte b for row k of the quad,
// already in place: byte n of the entry is digit n << 2k. So four lookups and
// three ORs give the quad bytes of the five columns one source byte position
// carries. pad is a source byte whose digits are all 1 (trit 0), for padding.
struct QuadLut {
  uint64_t t[4][256];
  uint8_t pad = 0;
  QuadLut() {
    for (int k = 0; k < 4; ++k)
      for (uint32_t b = 0; b < 256; ++b) {
        uint64_t v = 0;
        for (uint32_t n = 0, p = 1; n < 5; ++n, p *= 3) v |= (uint64_t)(digit(b, p) << (2 * k)) << (8 * n);
        t[k][b] = v;
      }
    for (uint32_t b = 0; b < 256; ++b)
      if (digit(b, 1) == 1 && digit(b, 3) == 1 && digit(b, 9) == 1 && digit(b, 27) == 1 && digit(b, 81) == 1) {
        pad = (uint8_t)b;
        break;
      }
  }
};
const QuadLut& quad_lut() {
  static const QuadLut lut;
  return lut;
}

// The 128 quad bytes of one 128-column block of a row quad (blk[k]: row k's
// PTQ1_0 block). Bytes 0..15 of a block hold columns m + 16n, bytes 16..23
// columns 80 + m + 8n, bytes 24..25 columns 120 + h + 2n (4 digits), digit
// n = 0 the most significant.
inline void quad_block(const QuadLut& L, const uint8_t* const blk[4], uint8_t q[128]) {
  auto at = [&](int i) {
    return L.t[0][blk[0][i]] | L.t[1][blk[1][i]] | L.t[2][blk[2][i]] | L.t[3][blk[3][i]];
  };
  for (int m = 0; m < 16; ++m) {
    const uint64_t v = at(m);
    for (int n = 0; n < 5; ++n) q[m + 16 * n] = (uint8_t)(v >> (8 * n));
  }
  for (int m = 0; m < 8; ++m) {
    const uint64_t v = at(16 + m);
    for (int n = 0; n < 5; ++n) q[80 + m + 8 * n] = (uint8_t)(v >> (8 * n));
  }
  for (int h = 0; h < 2; ++h) {
    const uint64_t v = at(24 + h);
    for (int n = 0; n < 4; ++n) q[120 + h + 2 * n] = (uint8_t)(v >> (8 * n));
  }
}

// Panel rows [8 g0, 8 g1).
void repack_groups(const uint8_t* src, int64_t N, int64_t K, uint8_t* panels, int64_t g0, int64_t g1) {
  const QuadLut& L = quad_lut();
  const int64_t nbk = K / 128, S = (K + BTF_PANEL_COLS - 1) / BTF_PANEL_COLS, bpr = S * 8;
  uint8_t pad_blk[28];
  std::memset(pad_blk, L.pad, 26);
  pad_blk[26] = pad_blk[27] = 0;  // scale 0
  alignas(16) uint8_t q[128];
  for (int64_t g = g0; g < g1; ++g)
    for (int h = 0; h < 2; ++h)
      for (int64_t b = 0; b < bpr; ++b) {
        uint8_t* pan = panels + (g * S + b / 8) * kPanelH;
        const int bb = (int)(b % 8);
        const uint8_t* blk[4];
        for (int k = 0; k < 4; ++k) {
          const int64_t n = g * kRowsH + h * 4 + k;
          blk[k] = (n < N && b < nbk) ? src + (n * nbk + b) * 28 : pad_blk;
        }
        quad_block(L, blk, q);
        for (int sb = 0; sb < 4; ++sb)
          for (int v = 0; v < 2; ++v)
            std::memcpy(pan + h * kQuadBytes + v * kHalfBytes + (bb * 4 + sb) * 16, q + 32 * sb + 16 * v, 16);
        uint8_t* sp = pan + kScaleBase + bb * 16 + h * 8;
        for (int k = 0; k < 4; ++k) {
          sp[2 * k] = blk[k][26];
          sp[2 * k + 1] = blk[k][27];
        }
      }
}

}  // namespace
}  // namespace btf

extern "C" int btf_repack_panels_host(const void* ptq_src_host, int64_t N, int64_t K, void* panels_host,
                                      int threads) {
  if (!ptq_src_host || !panels_host || N <= 0 || K <= 0 || K % 128)
    return btf::fail(BTF_ERR_ARG, "btf_repack_panels_host: null pointer or bad shape (N=%lld K=%lld)", (long long)N,
                     (long long)K);
  const int64_t G = (N + btf::kRowsH - 1) / btf::kRowsH;
  int t = threads > 0 ? threads : (int)std::max(1u, std::thread::hardware_concurrency());
  t = (int)std::min<int64_t>(t, G);
  const auto* src = static_cast<const uint8_t*>(ptq_src_host);
  auto* dst = static_cast<uint8_t*>(panels_host);
  if (t <= 1) {
    btf::repack_groups(src, N, K, dst, 0, G);
    return BTF_OK;
  }
  // Threads that cannot be created (std::system_error) or a failed allocation
  // must not unwind across the C ABI: the groups the pool did not start are
  // repacked on this thread instead, after joining the threads that did start.
  std::vector<std::thread> pool;
  int started = 0;
  try {
    pool.reserve((size_t)t);
    for (; started < t; ++started)
      pool.emplace_back(btf::repack_groups, src, N, K, dst, G * started / t, G * (started + 1) / t);
  } catch (...) {
  }
  for (auto& th : pool) th.join();
  if (started < t) btf::repack_groups(src, N, K, dst, G * started / t, G);
  return BTF_OK;
}
