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

struct BytePtr {
  const uint8_t* p;
  uint32_t operator()(int i) const { return p[i]; }
};

void repack_groups(const uint8_t* src, int64_t N, int64_t K, uint8_t* panels, int64_t g0, int64_t g1) {
  const int64_t nbk = K / 128, S = (K + BTF_PANEL_COLS - 1) / BTF_PANEL_COLS, bpr = S * 8;
  for (int64_t g = g0; g < g1; ++g)
    for (int h = 0; h < 2; ++h)
      for (int64_t b = 0; b < bpr; ++b) {
        uint32_t tw[4][8];
        uint16_t sc[4];
        for (int k = 0; k < 4; ++k) {
          const int64_t n = g * kRowsH + h * 4 + k;
          sc[k] = 0;
          if (n < N && b < nbk) {
            const uint8_t* blk = src + (n * nbk + b) * 28;
            ptq_block_to_t2(BytePtr{blk}, tw[k]);
            sc[k] = (uint16_t)(blk[26] | (blk[27] << 8));
          } else {
            for (int w = 0; w < 8; ++w) tw[k][w] = 0x55555555u;
          }
        }
        store_quad_block(panels + (g * S + b / 8) * kPanelH, h, (int)(b % 8), tw, sc);
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
  std::vector<std::thread> pool;
  for (int i = 0; i < t; ++i)
    pool.emplace_back(btf::repack_groups, src, N, K, dst, G * i / t, G * (i + 1) / t);
  for (auto& th : pool) th.join();
  return BTF_OK;
}
