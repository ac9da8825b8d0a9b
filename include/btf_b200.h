/*
 * btf_b200 — B200-native (sm_100a) ternary GEMV/GEMM hot path, C ABI.
 *
 * Drop-in boundary for bonsai-ternary-fast's CUDA matmul path. Each entry
 * point names the reference interface it replaces (paths relative to the
 * reference project root). Conventions:
 *   - every pointer is a DEVICE pointer unless its name ends in _host;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream);
 *   - launches are asynchronous, allocate nothing and never synchronise, so
 *     they are legal inside CUDA graph capture (like src/cuda/kernels.cuh:3-7);
 *   - every function returns a status code (BTF_OK = 0) instead of throwing;
 *     btf_last_error() gives a one-line message for the calling thread.
 *
 * Resident weight layout ("panels", replaces T2 of include/btf/packed.hpp:6-14):
 *   a [N][K] ternary matrix is cut into row groups of 8 rows and column slices
 *   of 1024 columns (32 sub-blocks of 32 = 8 PTQ1_0 blocks of 128).
 *   Panel (g, j) is 2176 contiguous bytes at ((g * S) + j) * 2176, S = ceil(K/1024):
 *     bytes [0, 2048):    codes, 2 bits each (code = trit + 1), as 32-bit words:
 *                         quad h (rows 4h..4h+3), half v, sub-block l, word i at
 *                         h*1024 + v*512 + l*16 + i*4 holds columns 32l + 16v + 4i + c
 *                         (c = byte 0..3) of row 4h + k at bits 8c + 2k .. 8c + 2k + 1;
 *     bytes [2048, 2176): fp16 block scales, block b (0..7) of row r at 2048 + b*16 + r*2.
 *   A row group's S panels are contiguous, so one 1-D bulk copy per panel streams
 *   8 rows x 1024 columns with their scales; in a word, (word & (3 << 2k) per byte)
 *   is 4^k times the codes of row 4h + k, ready for a byte-wise dot product with
 *   the int8x4 activation word of the same four columns.
 *   Rows >= N and columns >= K are padding (code 1 = trit 0, scale 0).
 *   Total size: btf_panel_bytes(N, K).
 */
#ifndef BTF_B200_H
#define BTF_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes */
#define BTF_OK 0
#define BTF_ERR_ARG 1         /* bad shape, pointer, alignment or mode */
#define BTF_ERR_CUDA 2        /* a CUDA runtime call failed */
#define BTF_ERR_UNSUPPORTED 3 /* valid request the library does not serve (e.g. K too wide) */
#define BTF_ERR_TIMEOUT 4     /* a bounded device-side wait gave up */
#define BTF_ERR_STATE 5       /* library not initialised for this device */

/* GEMV output modes. Same values as GemvMode in src/cuda/kernels.cuh:53. */
#define BTF_STORE 0  /* y  = W x */
#define BTF_ADD 1    /* y += W x */
#define BTF_SWIGLU 2 /* y  = silu(W_gate x) * (W_up x); segs[0] = gate, segs[1] = up */

/* Layout constants. */
#define BTF_PANEL_ROWS 8
#define BTF_PANEL_COLS 1024
#define BTF_PANEL_BYTES 2176

/* One matrix of a multi-segment GEMV. Mirrors GemvSeg (src/cuda/kernels.cuh:46-52)
 * with the T2 codes/scales pair replaced by one panel buffer. */
typedef struct btf_gemv_seg {
  const void* panels; /* btf_panel_bytes(N, K) bytes, 16-byte aligned */
  int N;              /* output rows */
  float* y;           /* [M][ldy]; unused for segs[1] of BTF_SWIGLU */
  int ldy;
} btf_gemv_seg;

/* Q8_0 activations of M rows of width K. Mirrors Q8Act (src/cuda/kernels.cuh:27-31). */
typedef struct btf_q8act {
  int8_t* q;  /* [M][K], 16-byte aligned */
  float* d;   /* [M][K/32] fp16-valued block scales */
  int32_t* s; /* [M][K/32] sum of q per block */
} btf_q8act;

/* ---- library / device state */
const char* btf_status_string(int status);
/* Last error message of the calling thread ("" if none). */
const char* btf_last_error(void);
/* Library version string. */
const char* btf_version(void);

/* Per-device set-up: shared-memory opt-ins and device limits. Call once per
 * device, outside stream capture, before any launch on that device.
 * Replaces btf::cuda::kernels_init (src/cuda/kernels.cuh:17, kernels.cu:718-729). */
int btf_init(int device);

/* Largest activation batch one GEMV launch keeps per pass for width K; M above
 * it is processed in passes. Replaces gemv_max_nb (src/cuda/kernels.cuh:20). */
int btf_gemv_max_nb(int K);

/* ---- layout sizes */
/* Bytes of the panel layout of an [N][K] matrix (K % 128 == 0). */
int64_t btf_panel_bytes(int64_t N, int64_t K);
/* Reference T2 sizes, include/btf/fast.hpp:45-46. */
int64_t btf_t2_codes_bytes(int64_t N, int64_t K);
int64_t btf_t2_scales_bytes(int64_t N, int64_t K);

/* ---- repack (load time)
 * PTQ1_0 (28-byte blocks, [N][K/128] in row order, 4-byte aligned; the source
 * may be mapped host memory) -> panel layout. Replaces launch_repack
 * (src/cuda/kernels.cuh:24, kernels.cu:737-743) for the B200 layout. */
int btf_repack_panels(const void* ptq_src, int64_t N, int64_t K, void* panels, void* stream);
/* Host twin of btf_repack_panels: same bytes, computed on the CPU.
 * Replaces btf::repack_rows / btf::repack (src/repack.cpp:16-45). */
int btf_repack_panels_host(const void* ptq_src_host, int64_t N, int64_t K, void* panels_host, int threads);
/* PTQ1_0 -> reference T2 codes [nblocks][32 B] + fp16 scales [nblocks], exactly
 * launch_repack's output (src/cuda/kernels.cuh:24), for callers that keep T2. */
int btf_repack_t2(const void* ptq_src, int64_t nblocks, uint8_t* codes, uint16_t* scales, void* stream);
/* Resident T2 (codes [N][K/4], scales [N][K/128]) -> panel layout. */
int btf_t2_to_panels(const uint8_t* codes, const uint16_t* scales, int64_t N, int64_t K, void* panels,
                     void* stream);
/* Panel layout -> T2 (inverse, for tests and for callers that read T2 back). */
int btf_panels_to_t2(const void* panels, int64_t N, int64_t K, uint8_t* codes, uint16_t* scales, void* stream);

/* ---- Q8 activation quantiser
 * x [M][ldx] fp32 -> Q8_0 (bit-exact to q8_block_host, include/btf/packed.hpp:117-134).
 * The quantising part of launch_prep (src/cuda/kernels.cuh:42-43, kernels.cu:185-201)
 * for a raw input (no norm, no Hadamard transform). K % 32 == 0. */
int btf_quant_q8(const float* x, int ldx, int M, int K, btf_q8act act, void* stream);

/* Input transform of a folded-Hadamard weight. Mirrors Hx (src/cuda/kernels.cuh:34-38):
 * block = 0: none; else blockwise Walsh-Hadamard of `block` (a power of two dividing
 * the span, the largest power of two <= 1024 dividing n); perm_rep > 1: tiled
 * [hd, nk, rep] -> grouped [hd, rep, nk] permutation first; signs: per-column +-1. */
typedef struct btf_hx {
  int block;
  int perm_hd, perm_nk, perm_rep;
  const float* signs; /* [n] or NULL */
} btf_hx;

/* ---- fused prep: RMSNorm (normw != NULL) -> permutation -> signs -> Hadamard
 * -> Q8_0, plus the normalised rows in xn_out [M][ldxn] when non-NULL.
 * Replaces launch_prep (src/cuda/kernels.cuh:42-43, kernels.cu:745-774). With
 * normw == NULL and hx.block == 0 it is bit-exact to btf_quant_q8. */
int btf_prep(const float* x, int ldx, int M, int n, const float* normw, float eps, btf_hx hx, float* xn_out,
             int ldxn, btf_q8act act, void* stream);

/* ---- ternary GEMV (batch M, CUDA cores: dp4a on the 2-bit codes)
 * Replaces launch_gemv (src/cuda/kernels.cuh:56, kernels.cu:776-822).
 * 1..3 segments sharing K and the activation; BTF_SWIGLU needs exactly two
 * segments (gate, up) with the same N. K % 128 == 0. Store / add calls with d
 * 16-byte aligned run on the tensor cores: K <= 8192 and, with u the 32-row
 * units of every segment and S the SM count, 9 <= M <= 16 and u >= S,
 * 5 <= M <= 8 and u >= 2 S, or 3 <= M <= 4 and u >= 8 S as btf_gemv_mma (q, d,
 * s 16-byte aligned); 17 <= M <= 32 with u >= 8 S (and K <= 8192) as two
 * btf_gemv_mma passes of 16 rows; else 9 <= M <= 64 as btf_gemm_wm when
 * every segment has at least 2/3 as many 128-row tiles as the device has SMs
 * (and s is 16-byte aligned), M >= 64 otherwise as btf_gemm. Other calls and
 * swiglu run in passes of btf_gemv_max_nb(K) rows. */
int btf_gemv(const btf_gemv_seg* segs, int nseg, int K, int M, btf_q8act act, int mode, void* stream);

/* Fused form: the activation is given as fp32 x [M][ldx] and quantised to Q8_0
 * inside the GEMV (same bit-exact rule as btf_quant_q8), saving the separate
 * quantiser launch of launch_prep + launch_gemv. */
int btf_gemv_f32(const btf_gemv_seg* segs, int nseg, int K, int M, const float* x, int ldx, int mode, void* stream);

/* Device error word of the current device: nonzero after a bounded device-side
 * wait gave up (the kernel then returned early instead of hanging). Synchronous;
 * not for use inside stream capture. clear != 0 resets it. Returns -1 on failure. */
int btf_device_error(int clear);

/* Measurement hook, no counterpart in the reference: the next btf_quant_q8,
 * btf_gemv / btf_gemv_f32 / btf_gemv_gather, btf_gemm_wm or btf_gemv_mma call made by this host
 * thread makes its kernel raise *slot (device memory, 8-byte aligned) to the device's global
 * timer in ns as each CTA finishes, so after the launch *slot holds the end time
 * of its last CTA (atomic max: a slot that starts at 0, or keeps an earlier
 * replay's stamp, ends with this launch's end). The request applies to one call
 * and is then cleared; slot = NULL clears it. Legal during stream capture: a
 * captured launch stamps the same slot at every replay. Exclusive kernel times
 * (end minus the previous kernel's end) then add up to the step time without
 * events between the launches, which would break programmatic dependent launch. */
int btf_stamp_next(unsigned long long* slot);

/* ---- ternary GEMM for prefill batches (M >= 64): tcgen05 int8 tensor cores
 * (kind::i8, one exact 32-deep MMA step per activation block, fp32 epilogue on
 * the CUDA cores). Same result contract as btf_gemv for BTF_STORE / BTF_ADD; it
 * replaces the repeated 8-row passes of launch_gemv (src/cuda/kernels.cu:805-821)
 * for large M. q and d must be 16-byte aligned. A segment that btf_gemv would
 * give to btf_gemv_mma runs there; one with M <= 64 and at least 2/3 as many
 * 128-row tiles as SMs (s 16-byte aligned) runs on the weight-major kernel of
 * btf_gemm_wm instead. */
int btf_gemm(const btf_gemv_seg* segs, int nseg, int K, int M, btf_q8act act, int mode, void* stream);

/* The GEMM for small batches (1 <= M <= 64), weight-major: the weights are the
 * tensor core's 128-row operand and the M activation rows (padded to 16, 32 or
 * 64) its N side, so every weight byte is read once for the whole batch. A
 * persistent kernel: one CTA per SM walks 128-row weight tiles. Same result
 * contract and arguments as btf_gemm (store / add modes, 1..3 segments, K a
 * multiple of 128); q, d and s must be 16-byte aligned; M > 64 returns
 * BTF_ERR_ARG. It replaces the batch-M passes of launch_gemv
 * (src/cuda/kernels.cu:805-821). btf_gemv and btf_gemm route their small-batch
 * calls over large matrices here. */
int btf_gemm_wm(const btf_gemv_seg* segs, int nseg, int K, int M, btf_q8act act, int mode, void* stream);

/* The small-batch GEMM on warp-level int8 MMA (1 <= M <= 16, K <= 8192): 32
 * weight rows per warp, the 2-bit codes moved from the staged panels straight
 * into the MMA operand registers, one exact 32-deep integer dot per activation
 * block and the fp32 block scaling in registers; the activation rows sit in
 * shared memory. Every weight byte is read once for the batch. Same result
 * contract and arguments as btf_gemm_wm (store / add, 1..3 segments, K a
 * multiple of 128, q, d and s 16-byte aligned); M > 16 or K > 8192 returns
 * BTF_ERR_ARG. Replaces the batch-M passes of launch_gemv
 * (src/cuda/kernels.cu:805-821). */
int btf_gemv_mma(const btf_gemv_seg* segs, int nseg, int K, int M, btf_q8act act, int mode, void* stream);

/* The prefill GEMM from fp32 activations x [M][ldx], allocating nothing. No
 * counterpart in the reference: it exists for callers that cannot allocate
 * device memory, such as a plugin whose host engine has reserved the whole
 * device and passes it only operand tensors, or a serving loop that may not
 * call cudaMalloc (which can synchronise the device) between steps. It
 * quantises x exactly as btf_quant_q8 does and runs btf_gemm, with the Q8
 * intermediate in a fixed device array inside the library instead of a caller
 * buffer, so its outputs equal those of btf_quant_q8 + btf_gemm.
 *   - Limit: M * K <= BTF_GEMM_NOALLOC_MAX_MK (512 x 17408); larger calls return
 *     BTF_ERR_ARG. Every GPU that loads the library holds the array
 *     (BTF_GEMM_NOALLOC_MAX_MK * 1.25 bytes, about 11 MB) until the process exits.
 *   - Every call looks up the array's device address (cudaGetSymbolAddress); the
 *     first call on a device may also load the library's module there, so make
 *     that first call outside any stream capture.
 *   - All calls on a device share the one array: calls that can overlap on the
 *     GPU (different streams without ordering between them) race. Calls in one
 *     stream are ordered and safe.
 *   - segs, K, mode and the output contract are btf_gemm's; x needs ldx >= K. */
#define BTF_GEMM_NOALLOC_MAX_MK 8912896
int btf_gemm_f32_noalloc(const btf_gemv_seg* segs, int nseg, int K, int M, const float* x, int ldx, int mode,
                         void* stream);

/* ---- persistent GEMV chain: a decoder's sequence of matmul call sites in ONE launch
 * Replaces the per-matmul launch_prep + launch_gemv pairs that the reference
 * decoder issues into its captured stream for one token (GpuDecoder::forward_chunk /
 * gdn_layer / attn_layer, src/cuda/gpu_decoder.cu:401-450; launchers
 * src/cuda/kernels.cu:745-822) when each matmul's input is written by the matmul
 * before it. Op i is btf_gemv(segs, nseg, K, M, Q8(prep(x)), mode) with prep =
 * RMSNorm with normw (when normw != NULL; bd::rmsnorm's formula,
 * ref/bonsai-decoder/src/cpu_ops.cpp:113-127, its double sum of squares taken in a
 * fixed parallel order) and Q8 = btf_quant_q8's rule. Ops run in order: op i+1
 * reads its x only after every output of ops 0..i is stored, exactly as if each op
 * were its own launch in one stream, so any op may read what earlier ops wrote
 * (including in-place BTF_ADD outputs). One persistent grid runs all ops; the
 * weight panels of later ops stream into shared memory while earlier ops finish. */
typedef struct btf_chain_op {
  btf_gemv_seg segs[3]; /* btf_gemv's segments; nseg used */
  int nseg;
  int K;               /* K % 128 == 0 */
  int mode;            /* BTF_STORE / BTF_ADD / BTF_SWIGLU */
  const float* x;      /* fp32 input [M][ldx], 4-byte aligned */
  int ldx;             /* >= K */
  const float* normw;  /* RMSNorm weight [K] applied before Q8, or NULL */
  float eps;           /* RMSNorm epsilon */
} btf_chain_op;

/* An encoded chain (filled by btf_chain_encode; pass it to btf_chain_run). */
typedef struct btf_chain {
  void* program; /* the caller's device buffer holding the encoded ops and counters */
  int n_ops;
  int M;         /* activation rows, 1..2 */
  int max_K;     /* widest op input, in columns padded to 1024 */
  int grid;      /* CTAs of one run (persistent, all co-resident) */
  int depth;     /* weight-ring slots per warp */
  int smem;      /* dynamic shared memory per CTA */
} btf_chain;

/* Device bytes of the program buffer of an n_ops chain. */
int64_t btf_chain_program_bytes(int n_ops);
/* Validates and encodes ops[0..n_ops) for M activation rows into `program` (a
 * caller-owned, 256-byte-aligned device buffer of btf_chain_program_bytes(n_ops)
 * bytes) on the current device. Set-up call: it copies synchronously, so make it
 * outside stream capture. The pointers in ops are used by every later run. */
int btf_chain_encode(const btf_chain_op* ops, int n_ops, int M, void* program, btf_chain* chain);
/* One run of the whole chain: one launch, asynchronous, allocates nothing, legal
 * inside CUDA graph capture. The grid waits on itself, so do not run other
 * kernels concurrently on this device that could keep its CTAs from being resident
 * (a CTA that waits 1 s gives up: BTF error word set, outputs incomplete). Runs of
 * one program must be ordered (one stream). */
int btf_chain_run(const btf_chain* chain, void* stream);

/* Debug/parity entry point: the exact int32 trit dot of every (m, row,
 * sub-block), idot[M][N][K/32] = code_dot - sum(q) -- the integers the GEMV
 * scales (src/emu_decoder.cpp:154-157). It runs the shipped GEMV kernel itself in
 * its dump form: each value is the fp32 operand that kernel's epilogue multiplies
 * (the biased integer of its dp4a dots converted exactly), written as int32. */
int btf_gemv_idot(const void* panels, int N, int K, int M, btf_q8act act, int32_t* idot, void* stream);
/* The same dump from the tcgen05 GEMM (btf_gemm): each 32-column step's integer
 * accumulator read from tensor memory (P - 4096 of its biased region), the
 * integers the GEMM's epilogue scales; idot[M][N][K/32]. q and d 16-byte aligned. */
int btf_gemm_idot(const void* panels, int N, int K, int M, btf_q8act act, int32_t* idot, void* stream);

/* The same dump from the weight-major GEMM (btf_gemm_wm), 1 <= M <= 64. */
int btf_gemm_wm_idot(const void* panels, int N, int K, int M, btf_q8act act, int32_t* idot, void* stream);

/* The same dump from the warp-MMA small-batch GEMM (btf_gemv_mma), 1 <= M <= 16, K <= 8192. */
int btf_gemv_mma_idot(const void* panels, int N, int K, int M, btf_q8act act, int32_t* idot, void* stream);

/* ---- N-sharded GEMV with the all-gather fused into the epilogue
 * The reference is single-GPU (src/cuda/gpu_decoder.cu); this is the B200
 * build's multi-GPU form of launch_gemv (src/cuda/kernels.cuh:56). Rank r of
 * `world` holds rows [row0_r, row0_r + n_r) of every matrix and runs
 * btf_gemv_gather on them with the SAME activation as every other rank. Every
 * output value is stored into every rank's full output buffer over NVLink
 * (peer pointers from CUDA IPC; plain stores). The last CTA of the launch on
 * each rank then adds 1 to every rank's arrival counter (system scope) and
 * waits, bounded, until its own counter shows all `world` ranks of this
 * launch, so when the launch completes in stream order the gathered outputs
 * are complete on this rank. Every rank must make the same sequence of
 * btf_gemv_gather calls with one arrival counter. A wait that gives up sets the
 * device error word (btf_device_error). */
#define BTF_MAX_RANKS 8
typedef struct btf_gather {
  int world; /* ranks, 2..BTF_MAX_RANKS */
  int rank;  /* this rank */
  /* per segment s: where segs[s].y lies in each rank's output buffer, as mapped
   * in this process; peer_y[s][rank] must equal segs[s].y */
  float* peer_y[3][BTF_MAX_RANKS];
  unsigned int* flags[BTF_MAX_RANKS]; /* each rank's arrival counter, as mapped here */
  unsigned int* expect;               /* this rank's consumed-arrivals counter (device, starts at 0) */
  unsigned int* done;                 /* this rank's CTA completion counter (device, starts at 0) */
  /* Tagged form (tagged != 0): the outputs are 64-bit words (fp32 value bits in
   * the low half, tag in the high half) and no counter is used: every word is
   * stored with one single-copy-atomic 64-bit store, so a reader that sees the
   * expected tag in a word also sees that launch's value. tag = *epoch * 1024 +
   * site (site < 1024, unique per launch within an epoch). Readers check tags
   * with btf_gather_wait; btf_gather_epoch_advance starts a new epoch. */
  int tagged;
  int site;
  const unsigned int* epoch; /* this rank's epoch counter (device) */
} btf_gather;
/* Counted completion serves M <= btf_gemv_max_nb(K) (one pass, one arrival per
 * launch); the tagged form serves any M (every pass stores its rows' words with
 * the launch's tag). Tagged store calls that btf_gemv would give to
 * btf_gemv_mma (the rule above, per shard) run on the warp-MMA GEMM;
 * otherwise those with 9 <= M <= 64 whose every shard has at
 * least 2/3 as many 128-row tiles as SMs run on the weight-major tcgen05 GEMM
 * (btf_gemm_wm); both make one pass over the shard's weights, with the same
 * tagged stores (d and s 16-byte aligned). */
int btf_gemv_gather(const btf_gemv_seg* segs, int nseg, int K, int M, btf_q8act act, int mode, const btf_gather* g,
                    void* stream);

/* Tagged-gather helpers. One tagged output buffer to check: `words` 64-bit
 * words at `p` that the launch with `site` stores. */
typedef struct btf_tagged_buf {
  const uint64_t* p;
  int64_t words;
  int site;
} btf_tagged_buf;
/* *epoch += 1 (one thread, in stream order): a new epoch for the next launches. */
int btf_gather_epoch_advance(unsigned int* epoch, void* stream);
/* Waits (bounded) until every word of bufs[0..n) carries the tag
 * *epoch * 1024 + site of its buffer; on time-out sets the device error word.
 * n <= 8. The launch returns once the outputs are all there. */
int btf_gather_wait(const btf_tagged_buf* bufs, int n, const unsigned int* epoch, void* stream);
/* Cross-rank barrier in stream order (one thread): adds 1 to every rank's
 * arrival counter (g->flags, system scope) and waits, bounded, until this rank's
 * counter shows all g->world ranks (g->expect tracks the count). With tagged
 * launches it separates epochs: no rank starts storing into a buffer for the next
 * epoch before every rank has finished checking the current one. */
int btf_gather_barrier(const btf_gather* g, void* stream);

/* Device buffers shared across processes (one process per GPU) through CUDA IPC.
 * btf_alloc/btf_free: cudaMalloc/cudaFree on the current device (the IPC
 * handle of a cudaMalloc'd buffer maps exactly that buffer).
 * btf_ipc_handle: 64-byte handle of a btf_alloc buffer (cudaIpcGetMemHandle).
 * btf_ipc_open/btf_ipc_close: map / unmap another process's buffer. */
int btf_alloc(size_t bytes, void** ptr);
int btf_free(void* ptr);
int btf_ipc_handle(void* ptr, void* handle64);
int btf_ipc_open(const void* handle64, void** ptr);
int btf_ipc_close(void* ptr);

/* ---- load path: GGUF (v2/v3) -> resident panels
 * Replaces bd::Gguf + GpuDecoder::upload_mat (ref/bonsai-decoder/src/gguf.cpp,
 * src/cuda/gpu_decoder.cu:284-300). The file is mmapped read-only; tensor data
 * is reached without copying. Load-time functions: they may allocate and
 * synchronise (not for use inside stream capture). */
typedef struct btf_gguf_tensor_info {
  const char* name;  /* valid until btf_gguf_close */
  int n_dims;
  int64_t ne[4];     /* ggml order: ne[0] is the contiguous (row) dimension */
  uint32_t type;     /* ggml type id (PTQ1_0 = 143) */
  const void* data;  /* host pointer into the mapping */
  uint64_t bytes;    /* data bytes for f32/f16/bf16/q8_0/PTQ1_0, else 0 */
} btf_gguf_tensor_info;
int btf_gguf_open(const char* path, void** handle);
int btf_gguf_close(void* handle);
int64_t btf_gguf_tensor_count(const void* handle);
int64_t btf_gguf_find(const void* handle, const char* name); /* index, or -1 */
int btf_gguf_tensor(const void* handle, int64_t index, btf_gguf_tensor_info* out);
/* A 2-D PTQ1_0 tensor [ne1 rows][ne0 columns] -> panels (btf_panel_bytes(ne1, ne0)
 * bytes on the device): whole 8-row groups are staged through two pinned
 * buffers of about staging_bytes and repacked on the GPU as they arrive.
 * Returns after the panels are complete. */
int btf_gguf_load_panels(const void* handle, int64_t index, void* panels, int64_t staging_bytes, void* stream);
/* Rows [row0, row0 + rows) of the tensor (row0 a multiple of 8) into panels of a
 * rows x K matrix (btf_panel_bytes(rows, K)): one rank's shard of an N-sharded matrix. */
int btf_gguf_load_panels_rows(const void* handle, int64_t index, int64_t row0, int64_t rows, void* panels,
                              int64_t staging_bytes, void* stream);

/* ---- batch-1 decode step of the qwen35 hybrid decoder (gated delta net + gated
 * full attention) as one CUDA graph: the decode path the ternary GEMV serves.
 * Replaces GpuDecoder / make_gpu_decoder (src/cuda/gpu_decoder.cu:401-486,
 * include/btf/fast.hpp:71-101) for one token per step. The model comes from a
 * qwen35 GGUF (PTQ1_0 matrices, prism Hadamard fold, ref/bonsai-decoder/src/
 * model.cpp:68-205) or from seeded synthetic weights of a given geometry. */
typedef struct btf_decoder_opts {
  int n_ctx;       /* KV cache capacity in tokens (FastOptions::n_ctx) */
  int round_q_f16; /* round q to fp16 before q.k (FastOptions::round_q_f16) */
  int attn_splits; /* key ranges of the attention (FastOptions::attn_splits), 1..256 */
  int cuda_graph;  /* capture one step as a graph and replay it (FastOptions::cuda_graph) */
  int staging_mb;  /* GGUF load: pinned staging per slot in MiB, 2 slots (FastOptions::staging_mb); 0: 64 */
  int keep_page_cache; /* GGUF load: 0 drops the file's pages from the host page cache once the weights
                          are resident (FastOptions::drop_page_cache, on by default there) */
} btf_decoder_opts;  /* NULL options: {4096, 1, 16, 1, 64, 0} */

typedef struct btf_decoder_dims { /* bd::HParams (ref/bonsai-decoder/include/bd/model.hpp:18-35) */
  int n_layer, n_embd, n_ff, n_vocab, n_head, n_head_kv, head_dim, n_rot;
  int d_state, n_group, dt_rank, d_inner, conv_kernel;
  int hadamard_block; /* 0: no transform (synthetic) */
  float rope_base, rms_eps;
} btf_decoder_dims;

typedef struct btf_decoder_info {
  btf_decoder_dims dims;
  int pos;                     /* tokens decoded since the last reset */
  void* stream;                /* the decoder's CUDA stream */
  uint64_t weight_bytes;       /* resident weights one step reads (one embedding row) */
  uint64_t state_bytes;        /* recurrent state read + written per step */
  uint64_t kv_bytes_per_token; /* KV cache bytes read per step per cached token */
  const float* logits;         /* device [n_vocab] of the last step */
  uint64_t device_bytes;       /* every device allocation the decoder holds (btf_plan_memory's device_bytes) */
} btf_decoder_info;

int btf_decoder_open(const char* gguf_path, const btf_decoder_opts* opts, void** handle);
/* d_inner = 0: dt_rank * d_state. Every layer il with (il + 1) % 4 != 0 is recurrent. */
int btf_decoder_synthetic(const btf_decoder_dims* dims, uint64_t seed, const btf_decoder_opts* opts, void** handle);
/* One step for `token`: the greedy next token into *next; logits (host, n_vocab) when non-NULL. Synchronous. */
int btf_decoder_step(void* handle, int32_t token, float* logits, int32_t* next);
/* The prompt in chunks of up to max_chunk tokens (0: 8; 1..8), as GpuDecoder::prefill /
 * forward_chunk (src/cuda/gpu_decoder.cu:154-171, :401-450): each chunk runs every
 * prep and ternary matmul once over its rows, the mixers and the attention token by
 * token at each token's position. After it, pos += n; the greedy token after the last
 * prompt token goes to *next (and to the device token a btf_decoder_run would read);
 * logits (host, n_vocab) of the last prompt token when non-NULL. Synchronous, eager
 * (no graph). One GPU only: a tensor-parallel decoder returns BTF_ERR_UNSUPPORTED. */
int btf_decoder_prefill(void* handle, const int32_t* tokens_host, int n, int max_chunk, float* logits, int32_t* next);
/* `steps` steps, each fed the previous step's greedy token on the device; asynchronous on the decoder's stream. */
int btf_decoder_run(void* handle, int steps);
int btf_decoder_reset(void* handle);
int btf_decoder_close(void* handle);
int btf_decoder_get_info(void* handle, btf_decoder_info* out);

/* Per-step accounting since the last reset_stats (FastDecoder::stats /
 * reset_stats and StepStats, include/btf/fast.hpp:72-96). Kept across
 * btf_decoder_reset. Reading the stats waits for a pending btf_decoder_run. */
typedef struct btf_step_stats {
  uint64_t steps;             /* steps made by btf_decoder_step and btf_decoder_run */
  double wall_s;              /* host wall time inside those calls */
  double gpu_s;               /* device time between CUDA events around each step / run */
  uint64_t weight_xfer_bytes; /* host-to-device weight copies during those steps: 0 (weights are resident) */
  double weight_xfer_s;       /* wall time of those copies: 0 */
  uint64_t mapped_read_bytes; /* bytes read zero-copy from mapped host memory: 0 (the embedding is resident) */
} btf_step_stats;
int btf_decoder_stats(void* handle, btf_step_stats* out);
int btf_decoder_reset_stats(void* handle);

/* Tensor-parallel decode: every ternary matmul of the step is N-sharded
 * over `world` GPUs (one process each; rank r holds rows shard r of every matrix,
 * whole 8-row groups) and its outputs are stored into every rank's activation
 * arena by btf_gemv_gather (counted completion); the rest of the step runs
 * replicated. Set-up: btf_decoder_synthetic_tp on every rank, export the arena
 * of btf_decoder_arena with btf_ipc_handle, open the peers' with btf_ipc_open,
 * then btf_decoder_connect(h, arenas[world]) before the first step. All ranks
 * then make the same sequence of step / run calls. Tear down only after every
 * rank has synchronised (no rank still stores into another's arena). */
int btf_decoder_synthetic_tp(const btf_decoder_dims* dims, uint64_t seed, const btf_decoder_opts* opts, int world,
                             int rank, void** handle);
/* The same from a qwen35 GGUF: rank `rank` loads its rows of every matrix
 * (btf_gguf_load_panels_rows) and the whole embedding table. */
int btf_decoder_open_tp(const char* gguf_path, const btf_decoder_opts* opts, int world, int rank, void** handle);
/* The row shard of `rank` among `world` that the tensor-parallel decoder uses for
 * an N-row matrix: whole 8-row groups, ceil(groups / world) groups per rank, the
 * last ranks clipped (rows may be 0 for small N). Host-only. */
int btf_shard_rows(int N, int world, int rank, int* row0, int* rows);
int btf_decoder_arena(void* handle, void** base, uint64_t* bytes);
int btf_decoder_connect(void* handle, void* const* peer_arenas);

/* Memory plan of a decoder before it is opened: the exact device allocations
 * btf_decoder_open_tp / btf_decoder_synthetic_tp would make for these options
 * on this rank, and the minimum traffic of one decode step. Replaces
 * btf::plan_memory + MemoryPlan (src/repack.cpp:142-204, include/btf/fast.hpp:50-69)
 * for the panel layout. It runs the decoder's own binding and buffer set-up
 * without touching a device, so it needs no GPU and agrees with the opened
 * decoder's btf_decoder_info.device_bytes by construction. */
typedef struct btf_memory_plan {
  uint64_t panel_bytes;          /* ternary matrices in panels: this rank's rows; the whole embedding table */
  uint64_t vector_bytes;         /* f32 vectors: norms, ssm_alpha/beta, ssm_a, dt bias, conv1d, Hadamard signs */
  uint64_t kv_cache_bytes;       /* fp16 K and V of every attention layer, n_ctx tokens */
  uint64_t state_bytes;          /* conv ring + delta-rule state of every recurrent layer */
  uint64_t work_bytes;           /* activation arena, attention partials, Q8 activation, argmax partials, token/pos */
  uint64_t device_bytes;         /* sum of the five above */
  uint64_t pinned_bytes;         /* resident pinned host memory (the step's token in/out) */
  uint64_t staging_bytes;        /* peak pinned staging while loading a GGUF, freed after each matrix */
  uint64_t decode_bytes_fixed;   /* one step reads every weight byte once (one embedding row), reads and writes
                                    the recurrent state, writes and reads the logits (MemoryPlan::decode_bytes_fixed) */
  uint64_t decode_bytes_per_ctx; /* plus this per token already in the KV cache (K and V rows) */
  int n_matrices;                /* ternary matrices resident (lm_head counted, tied or not) */
  btf_decoder_dims dims;         /* the geometry bound */
} btf_memory_plan;

int btf_plan_memory(const char* gguf_path, const btf_decoder_opts* opts, int world, int rank, btf_memory_plan* out);
int btf_plan_memory_synthetic(const btf_decoder_dims* dims, const btf_decoder_opts* opts, int world, int rank,
                              btf_memory_plan* out);

#ifdef __cplusplus
}
#endif

#endif /* BTF_B200_H */
