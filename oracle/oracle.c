/*
 * CPU oracle for the ternary GEMV/GEMM hot path — TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the reference algorithm of
 * bonsai-ternary-fast for the path the B200 kernels replace:
 *   PTQ1_0 block encoding/decoding, the T2 repack, the ggml-exact Q8_0
 *   activation quantiser, the per-32-column integer code dot, and the
 *   emulator GEMV loop (store / add / swiglu).
 * Every function names the reference file:line it follows (paths relative to
 * the reference project root).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library, and only as the checker or the timed CPU baseline. The
 * product (the CUDA library) never calls into it.
 *
 * Parity of this restatement is pinned against the reference's own sources,
 * compiled by oracle/Makefile into oracle/_ref/ (see oracle/ref_shim.cpp);
 * tests/test_oracle_pin.py checks the two bit for bit.
 *
 * Build: oracle/Makefile (-O2 -ffp-contract=off, no -ffast-math, no -march:
 * the float operation order below must not be contracted into FMAs, matching
 * the reference's own -O2 build).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ fp16 */

/* fp32 -> fp16 bits, round to nearest even, IEEE semantics incl. subnormals.
 * Follows ref/bonsai-decoder/src/types.cpp:42-62 (bd::f32_to_fp16). */
ORC_API uint16_t orc_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t mag = x & 0x7fffffffu;
  if (mag >= 0x7f800000u) /* inf or nan (nan stays quiet) */
    return (uint16_t)(sign | 0x7c00u | (mag > 0x7f800000u ? 0x0200u : 0u));
  if (mag >= 0x477ff000u) /* >= 65520 rounds past the largest finite half */
    return (uint16_t)(sign | 0x7c00u);
  if (mag < 0x38800000u) { /* below 2^-14: half subnormal or zero */
    if (mag < 0x33000000u) return sign; /* below 2^-25 rounds to zero */
    const uint32_t exp = mag >> 23;
    const uint32_t sig = (mag & 0x007fffffu) | 0x00800000u;
    const uint32_t sh = 126u - exp; /* value = sig * 2^(exp-150) = r * 2^-24 */
    uint32_t r = sig >> sh;
    const uint32_t rem = sig & ((1u << sh) - 1u), half = 1u << (sh - 1u);
    if (rem > half || (rem == half && (r & 1u))) ++r;
    return (uint16_t)(sign | r);
  }
  /* normal: drop 13 mantissa bits and rebias the exponent by 127-15 */
  uint32_t r = (mag >> 13) - (112u << 10);
  const uint32_t rem = mag & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) ++r;
  return (uint16_t)(sign | r);
}

/* fp16 bits -> fp32 (exact). Follows ref/bonsai-decoder/include/bd/types.hpp:37-57. */
ORC_API float orc_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = 113;
      while (!(man & 0x400u)) {
        man <<= 1;
        --e;
      }
      bits = sign | ((uint32_t)e << 23) | ((man & 0x3ffu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* ---------------------------------------------------------------- PTQ1_0 */

/* Element e (0..127) of a 28-byte PTQ1_0 block lives in byte `byte` as base-3
 * digit `digit` (digit 0 = most significant of the five). Mapping from
 * ref/bonsai-decoder/include/bd/types.hpp:70-75. */
static void ptq_slot(int e, int* byte, int* digit) {
  if (e < 80) {
    *byte = e & 15;
    *digit = e >> 4;
  } else if (e < 120) {
    *byte = 16 + ((e - 80) & 7);
    *digit = (e - 80) >> 3;
  } else {
    *byte = 24 + ((e - 120) & 1);
    *digit = (e - 120) >> 1;
  }
}

/* Trit (-1, 0, +1) of element e: digit d of byte b is ((uint8)(b*3^d)*3)>>8 - 1.
 * Follows ref/bonsai-decoder/include/bd/types.hpp:70-78 (bd::ptq1_0_trit). */
ORC_API int orc_ptq_trit(const uint8_t* blk, int e) {
  static const uint32_t pow3[5] = {1u, 3u, 9u, 27u, 81u};
  int b, d;
  ptq_slot(e, &b, &d);
  const uint32_t v = (uint32_t)(uint8_t)(blk[b] * pow3[d]);
  return (int)((v * 3u) >> 8) - 1;
}

/* Encodes nblocks blocks of 128 trits (values -1/0/+1, element order) and one
 * fp16 scale each into 28-byte PTQ1_0 blocks. Byte layout and digit packing
 * follow the PTQ1_0 quantiser, ref/bonsai-decoder/src/types.cpp:289-320:
 * five digits per byte (first element most significant), the 4-digit tail
 * bytes padded with a trailing zero digit, byte = ceil(value * 256 / 243),
 * scale little-endian in bytes 26..27. */
ORC_API void orc_ptq_encode(const int8_t* trits, const uint16_t* scales, int64_t nblocks, uint8_t* out) {
  for (int64_t i = 0; i < nblocks; ++i) {
    const int8_t* t = trits + i * 128;
    uint8_t* y = out + i * 28;
    uint32_t val[26];
    int ndig[26];
    memset(val, 0, sizeof val);
    memset(ndig, 0, sizeof ndig);
    for (int e = 0; e < 128; ++e) {
      int b, d;
      ptq_slot(e, &b, &d);
      (void)d; /* digits arrive in increasing d order for each byte */
      val[b] = val[b] * 3u + (uint32_t)(t[e] + 1);
      ndig[b]++;
    }
    for (int b = 0; b < 26; ++b) {
      uint32_t q = val[b];
      for (int k = ndig[b]; k < 5; ++k) q *= 3u; /* tail bytes: pad to 5 digits */
      q &= 0xffu;                                /* the reference packs in uint8 */
      y[b] = (uint8_t)((q * 256u + 242u) / 243u);
    }
    y[26] = (uint8_t)(scales[i] & 0xffu);
    y[27] = (uint8_t)(scales[i] >> 8);
  }
}

/* Full PTQ1_0 quantiser of one row of k floats (k % 128 == 0): per block
 * d = fp16(amax), trit = lround(x / amax). Follows
 * ref/bonsai-decoder/src/types.cpp:289-320 (bd::quant_row, PTQ1_0 case). */
ORC_API void orc_ptq_quant_row(const float* x, uint8_t* out, int64_t k) {
  for (int64_t i = 0; i < k / 128; ++i) {
    const float* xb = x + i * 128;
    float amax = 0.0f;
    for (int j = 0; j < 128; ++j) amax = fmaxf(amax, fabsf(xb[j]));
    const float id = amax != 0.0f ? 1.0f / amax : 0.0f;
    int8_t t[128];
    for (int j = 0; j < 128; ++j) t[j] = (int8_t)lroundf(xb[j] * id);
    const uint16_t dh = orc_f32_to_f16(amax);
    orc_ptq_encode(t, &dh, 1, out + i * 28);
  }
}

/* ------------------------------------------------------------------ T2 */

/* T2 placement of column e (0..127) inside a block's 32 code bytes.
 * Follows include/btf/packed.hpp:35-38 (code_byte / code_shift). */
static int t2_byte(int e) { return (e >> 5) * 8 + ((e >> 4) & 1) * 4 + (e & 3); }
static int t2_shift(int e) { return ((e >> 2) & 3) * 2; }

/* PTQ1_0 rows -> T2 codes [rows][K/4] + fp16 scales [rows][K/128]. Same result
 * as include/btf/packed.hpp:50-91 (pack_block) driven by src/repack.cpp:16-27
 * (repack_rows): code = trit + 1 at (t2_byte, t2_shift), scale bytes copied. */
ORC_API void orc_repack_t2(const uint8_t* src, int64_t rows, int64_t K, uint8_t* codes, uint16_t* scales) {
  const int64_t nb = K / 128;
  for (int64_t r = 0; r < rows; ++r) {
    for (int64_t b = 0; b < nb; ++b) {
      const uint8_t* blk = src + (r * nb + b) * 28;
      uint8_t* c = codes + (r * nb + b) * 32;
      memset(c, 0, 32);
      for (int e = 0; e < 128; ++e) {
        const int code = orc_ptq_trit(blk, e) + 1;
        c[t2_byte(e)] |= (uint8_t)(code << t2_shift(e));
      }
      scales[r * nb + b] = (uint16_t)(blk[26] | (blk[27] << 8));
    }
  }
}

/* Code (0..2) of column e of one T2 row. Follows include/btf/packed.hpp:94-98. */
ORC_API int orc_t2_code(const uint8_t* row_codes, int64_t e) {
  const uint8_t* blk = row_codes + (e / 128) * 32;
  const int c = (int)(e % 128);
  return (blk[t2_byte(c)] >> t2_shift(c)) & 3;
}

/* ------------------------------------------------------------------- Q8 */

/* ggml Q8_0 of one 32-block: d = fp16(amax/127) held in fp32, q = RNE(x*127/amax),
 * returns sum(q). Follows include/btf/packed.hpp:117-134 (q8_block_host),
 * including its amax update rule. */
ORC_API int orc_q8_block(const float* x, int8_t* q, float* d) {
  float amax = 0.0f;
  for (int i = 0; i < 32; ++i) {
    const float a = x[i] < 0 ? -x[i] : x[i];
    amax = amax > a ? amax : a;
  }
  *d = orc_f16_to_f32(orc_f32_to_f16(amax / 127.0f));
  const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
  int s = 0;
  for (int i = 0; i < 32; ++i) {
    const float r = nearbyintf(x[i] * id); /* default environment: ties to even */
    q[i] = (int8_t)(int)r;
    s += (int)r;
  }
  return s;
}

/* Q8 of M rows of width K (row stride ldx floats) into q[M][K], d/s[M][K/32].
 * The per-row loop of src/emu_decoder.cpp:135-138 without the norm/WHT. */
ORC_API void orc_q8_rows(const float* x, int64_t ldx, int M, int K, int8_t* q, float* d, int32_t* s) {
  for (int m = 0; m < M; ++m)
    for (int b = 0; b < K / 32; ++b) {
      const int64_t o = (int64_t)m * (K / 32) + b;
      s[o] = orc_q8_block(x + m * ldx + b * 32, q + (int64_t)m * K + b * 32, d + o);
    }
}

/* ggml round trip of Q8_0: out = RNE(x*id) * d. Follows
 * ref/bonsai-decoder/src/cpu_ops.cpp:189-197 (bd::round_q8_0). */
ORC_API void orc_round_q8_0(const float* x, int64_t n, float* out) {
  for (int64_t b = 0; b < n; b += 32) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[b + i]));
    const float d = orc_f16_to_f32(orc_f32_to_f16(amax / 127.0f));
    const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
    for (int i = 0; i < 32; ++i) out[b + i] = nearbyintf(x[b + i] * id) * d;
  }
}

/* ------------------------------------------------------------ code dots */

/* Signed byte-wise dot of two int8x4 words plus c (dp4a semantics).
 * Follows include/btf/packed.hpp:101-104 (dp4a_host). */
static int dp4a_ss(uint32_t a, uint32_t b, int c) {
  for (int i = 0; i < 4; ++i) c += (int)(int8_t)(a >> (8 * i)) * (int)(int8_t)(b >> (8 * i));
  return c;
}

/* Code dot of one 32-column sub-block: the two T2 words against the eight
 * activation words. Follows include/btf/packed.hpp:108-113 (sub_dot_host). */
ORC_API int orc_sub_dot(uint32_t w0, uint32_t w1, const uint32_t* aw) {
  int acc = 0;
  for (int k = 0; k < 4; ++k) acc = dp4a_ss((w0 >> (2 * k)) & 0x03030303u, aw[k], acc);
  for (int k = 0; k < 4; ++k) acc = dp4a_ss((w1 >> (2 * k)) & 0x03030303u, aw[4 + k], acc);
  return acc;
}

static uint32_t load_u32(const void* p) {
  uint32_t v;
  memcpy(&v, p, 4);
  return v;
}

/* Integer trit dot of every (m, row, sub-block): idot = code_dot - sum(q), the
 * exact int32 partial the GEMV scales. Out: idot[M][N][K/32].
 * Same integers as src/emu_decoder.cpp:154-157. */
ORC_API void orc_idot(const uint8_t* codes, int64_t N, int64_t K, const int8_t* q, const int32_t* s, int M,
                      int32_t* idot) {
  const int64_t nsub = K / 32;
  for (int m = 0; m < M; ++m) {
    const uint8_t* aq = (const uint8_t*)(q + (int64_t)m * K);
    for (int64_t r = 0; r < N; ++r) {
      const uint8_t* cr = codes + r * (K / 4);
      for (int64_t sb = 0; sb < nsub; ++sb) {
        uint32_t aw[8];
        for (int k = 0; k < 8; ++k) aw[k] = load_u32(aq + sb * 32 + 4 * k);
        idot[((int64_t)m * N + r) * nsub + sb] =
            orc_sub_dot(load_u32(cr + sb * 8), load_u32(cr + sb * 8 + 4), aw) - s[(int64_t)m * nsub + sb];
      }
    }
  }
}

/* ------------------------------------------------------------------ GEMV */

typedef struct {
  const uint8_t* codes;
  const uint16_t* scales;
  int64_t N, K;
  const int8_t* q;
  const float* d;
  const int32_t* s;
  int M;
  float* y;
  int64_t ldy;
  int add;
  int64_t r0, r1;
} gemv_job;

/* Rows [r0, r1) of the emulator GEMV: per row and activation row, ascending
 * sub-block s, acc += fp16(scale[s/4]) * d[s] * (float)idot (left to right,
 * no fused multiply-add); out = add ? out + acc : acc.
 * Follows src/emu_decoder.cpp:143-165 (EmuDecoder::gemv). */
static void gemv_rows(const gemv_job* j) {
  const int64_t nsub = j->K / 32;
  for (int64_t r = j->r0; r < j->r1; ++r) {
    const uint8_t* cr = j->codes + r * (j->K / 4);
    const uint16_t* sr = j->scales + r * (j->K / 128);
    for (int m = 0; m < j->M; ++m) {
      const uint8_t* aq = (const uint8_t*)(j->q + (int64_t)m * j->K);
      float acc = 0.0f;
      for (int64_t sb = 0; sb < nsub; ++sb) {
        uint32_t aw[8];
        for (int k = 0; k < 8; ++k) aw[k] = load_u32(aq + sb * 32 + 4 * k);
        const int idot =
            orc_sub_dot(load_u32(cr + sb * 8), load_u32(cr + sb * 8 + 4), aw) - j->s[(int64_t)m * nsub + sb];
        const float sd = orc_f16_to_f32(sr[sb / 4]) * j->d[(int64_t)m * nsub + sb];
        acc += sd * (float)idot;
      }
      float* out = &j->y[(int64_t)m * j->ldy + r];
      *out = j->add ? *out + acc : acc;
    }
  }
}

static void* gemv_thread(void* p) {
  gemv_rows((const gemv_job*)p);
  return NULL;
}

/* y[M][ldy] (=|+=) W x over N rows, rows split into `threads` contiguous
 * chunks the way ref/bonsai-decoder/src/cpu_ops.cpp:57-73 (ThreadPool) splits
 * them. mode 0 = store, 1 = add. threads <= 1 runs on the calling thread. */
ORC_API void orc_gemv(const uint8_t* codes, const uint16_t* scales, int64_t N, int64_t K, const int8_t* q,
                      const float* d, const int32_t* s, int M, float* y, int64_t ldy, int mode, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if (threads == 1 || N < 2 * threads) {
    gemv_job j = {codes, scales, N, K, q, d, s, M, y, ldy, mode == 1, 0, N};
    gemv_rows(&j);
    return;
  }
  gemv_job jobs[256];
  pthread_t th[256];
  for (int t = 0; t < threads; ++t) {
    gemv_job j = {codes, scales, N, K, q, d, s, M, y, ldy, mode == 1, N * t / threads, N * (t + 1) / threads};
    jobs[t] = j;
  }
  for (int t = 1; t < threads; ++t) pthread_create(&th[t], NULL, gemv_thread, &jobs[t]);
  gemv_rows(&jobs[0]);
  for (int t = 1; t < threads; ++t) pthread_join(th[t], NULL);
}

/* silu(gate) * up over the gate/up pair, both [M][N] emulator GEMVs.
 * The swiglu epilogue of src/cuda/kernels.cu:319-320 with silu as
 * ref/bonsai-decoder/include/bd/cpu_ops.hpp (x / (1 + exp(-x))). */
ORC_API void orc_gemv_swiglu(const uint8_t* gc, const uint16_t* gs, const uint8_t* uc, const uint16_t* us, int64_t N,
                             int64_t K, const int8_t* q, const float* d, const int32_t* s, int M, float* y,
                             int64_t ldy, int threads) {
  float* g = (float*)malloc(sizeof(float) * (size_t)M * (size_t)N);
  float* u = (float*)malloc(sizeof(float) * (size_t)M * (size_t)N);
  orc_gemv(gc, gs, N, K, q, d, s, M, g, N, 0, threads);
  orc_gemv(uc, us, N, K, q, d, s, M, u, N, 0, threads);
  for (int m = 0; m < M; ++m)
    for (int64_t r = 0; r < N; ++r) {
      const float a = g[(int64_t)m * N + r];
      y[(int64_t)m * ldy + r] = a / (1.0f + expf(-a)) * u[(int64_t)m * N + r];
    }
  free(g);
  free(u);
}

/* Double-precision reference GEMV on T2 codes: per sub-block the exact trit
 * dot times (double)fp16(scale) * d. Follows tests/test_gpu_kernels.cpp:177-193
 * (ref_gemv), the tolerance reference of the reference's GPU tests. */
ORC_API void orc_gemv_f64(const uint8_t* codes, const uint16_t* scales, int64_t N, int64_t K, const int8_t* q,
                          const float* d, int M, double* y) {
  const int64_t nsub = K / 32;
  for (int m = 0; m < M; ++m)
    for (int64_t r = 0; r < N; ++r) {
      double acc = 0.0;
      for (int64_t b = 0; b < nsub; ++b) {
        long dot = 0;
        for (int i = 0; i < 32; ++i) {
          const int64_t e = b * 32 + i;
          dot += (long)(orc_t2_code(codes + r * (K / 4), e) - 1) * q[(int64_t)m * K + e];
        }
        acc += (double)orc_f16_to_f32(scales[r * (K / 128) + b / 4]) * d[(int64_t)m * nsub + b] * (double)dot;
      }
      y[(int64_t)m * N + r] = acc;
    }
}

/* ------------------------------------------------------------------ prep (norm, permutation, signs, WHT, Q8) */

/* RMSNorm. Follows ref/bonsai-decoder/src/cpu_ops.cpp:121-127 (bd::rmsnorm):
 * double sum of squares in index order, mean = (float)(sum / n),
 * scale = 1 / sqrtf(mean + eps), y = x * scale * w (w = NULL: 1). */
ORC_API void orc_rmsnorm(const float* x, const float* w, int64_t n, float eps, float* y) {
  double sum = 0.0;
  for (int64_t i = 0; i < n; ++i) sum += (double)x[i] * x[i];
  const float mean = (float)(sum / (double)n);
  const float scale = 1.0f / sqrtf(mean + eps);
  for (int64_t i = 0; i < n; ++i) y[i] = x[i] * scale * (w ? w[i] : 1.0f);
}

/* In-place fast Walsh-Hadamard transform of n (power of two) values with the
 * 1/sqrt(n) scale. Follows ref/bonsai-decoder/src/cpu_ops.cpp:76-88 (bd::fwht):
 * stages len = 1, 2, 4, ...; butterfly (a, b) -> (a + b, a - b). */
static void orc_fwht(float* x, int n) {
  for (int len = 1; len < n; len <<= 1)
    for (int i = 0; i < n; i += len << 1)
      for (int j = i; j < i + len; ++j) {
        const float a = x[j], b = x[j + len];
        x[j] = a + b;
        x[j + len] = a - b;
      }
  const float s = 1.0f / sqrtf((float)n);
  for (int i = 0; i < n; ++i) x[i] *= s;
}

/* Input transform of a folded-Hadamard weight. Follows
 * ref/bonsai-decoder/src/cpu_ops.cpp:90-111 (bd::hadamard_input): optional
 * permutation out[d + hd*(r + rep*k)] = x[d + hd*(k + nk*r)] (perm_rep > 1),
 * optional sign flip, then blockwise FWHT of size `block` (block == 0: copy). */
ORC_API void orc_hadamard_input(int block, int perm_hd, int perm_nk, int perm_rep, const float* signs, const float* x,
                                int64_t n, float* out) {
  if (block <= 0) {
    if (out != x) memcpy(out, x, (size_t)n * sizeof(float));
    return;
  }
  if (perm_rep > 1) {
    for (int k = 0; k < perm_nk; ++k)
      for (int r = 0; r < perm_rep; ++r)
        for (int d = 0; d < perm_hd; ++d)
          out[d + (int64_t)perm_hd * (r + perm_rep * k)] = x[d + (int64_t)perm_hd * (k + perm_nk * r)];
  } else if (out != x) {
    memcpy(out, x, (size_t)n * sizeof(float));
  }
  if (signs)
    for (int64_t i = 0; i < n; ++i) out[i] *= signs[i];
  for (int64_t b = 0; b < n; b += block) orc_fwht(out + b, block);
}

/* The whole prep of M rows (the host form of launch_prep, as the reference's
 * test_prep builds it, tests/test_gpu_kernels.cpp:117-127): RMSNorm (normw
 * non-NULL), the input transform, Q8_0 per 32 (orc_q8_block). xn (optional)
 * receives the normalised, untransformed rows. */
ORC_API void orc_prep_rows(const float* x, int64_t ldx, int M, int n, const float* normw, float eps, int block,
                           int perm_hd, int perm_nk, int perm_rep, const float* signs, float* xn, int8_t* q, float* d,
                           int32_t* s) {
  float* t = (float*)malloc((size_t)n * sizeof(float));
  float* u = (float*)malloc((size_t)n * sizeof(float));
  for (int m = 0; m < M; ++m) {
    const float* xr = x + (int64_t)m * ldx;
    if (normw)
      orc_rmsnorm(xr, normw, n, eps, u);
    else
      memcpy(u, xr, (size_t)n * sizeof(float));
    if (xn) memcpy(xn + (int64_t)m * n, u, (size_t)n * sizeof(float));
    orc_hadamard_input(block, perm_hd, perm_nk, perm_rep, signs, u, n, t);
    for (int b = 0; b < n / 32; ++b)
      s[(int64_t)m * (n / 32) + b] = orc_q8_block(t + b * 32, q + (int64_t)m * n + b * 32, d + (int64_t)m * (n / 32) + b);
  }
  free(t);
  free(u);
}
