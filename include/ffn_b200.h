/*
 * ffn_b200.h -- C ABI of the B200 fused feed-forward operator
 *
 *     Y = GELU(X . W1^T) . W2^T      (fp16 or bf16, no bias, inference only)
 *
 * X is [M, K] row-major, W1 is [H, K] (torch Linear layout), W2 is [N, H], Y is [M, N].
 * All pointers are device pointers owned by the caller, and no entry point synchronises the
 * stream it is given.  The one entry point that allocates device memory is
 * ffn_b200_peer_alloc (cudaMalloc of a peer-visible buffer for the multi-GPU path).  The
 * library also holds static device arrays on every GPU that loads it, until the process
 * exits: the 32 MiB scratch of ffn_b200_run_noalloc (FFN_B200_NOALLOC_SCRATCH_BYTES) and
 * 10 KiB for the CTA-pair placement map and its probe (int32[512] + int32[2][1024]).
 *
 * Each entry point replaces one piece of the reference implementation (hxtsg/ffn_optim):
 *
 *   ffn_b200_make_plan  <- ops/host/tiling.py:58-74 (make_plan) together with the
 *                          Selection rules of ops/host/dispatch.py:42-66
 *   ffn_b200_prepare    <- ops/api.py:48-89 (prepare_ffn: device checks, block_num limit,
 *                          compile_kernel of ops/host/dispatch.py:97-116)
 *   ffn_b200_run        <- ops/api.py:37-45 (PreparedFFN.run -> artifact(...) launch, the
 *                          single host->device boundary of the reference)
 *   ffn_b200_launch     <- ops/api.py:92-94 (ffn: prepare + run in one call)
 *
 * Return codes are FFN_B200_OK (0) or one of the ffn_b200_status values below; the Python
 * host layer maps them onto the reference's exception types (ValueError, NotApplicable,
 * DependencyUnavailable, KernelCompilationError, RuntimeError).
 */
#ifndef FFN_B200_H
#define FFN_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FFN_B200_ABI_VERSION 2

#if defined(__GNUC__)
#define FFN_B200_EXPORT __attribute__((visibility("default")))
#else
#define FFN_B200_EXPORT
#endif

typedef enum {
  FFN_B200_OK = 0,
  FFN_B200_ERR_INVALID = 1,        /* bad shape, pointer, pitch or enum (reference: ValueError) */
  FFN_B200_ERR_NOT_APPLICABLE = 2, /* streamk without a tail wave (reference: NotApplicable) */
  FFN_B200_ERR_UNAVAILABLE = 3,    /* full_load_b (reference: DependencyUnavailable) */
  FFN_B200_ERR_DEVICE = 4,         /* not an sm_100 device or block_num > SM count */
  FFN_B200_ERR_CUDA = 5,           /* a CUDA runtime / driver call failed */
  FFN_B200_ERR_ALIGNMENT = 6,      /* base not 16-byte aligned or pitch not a multiple of 8 elements */
  FFN_B200_ERR_TOO_LARGE = 7,      /* tile count does not fit one launch */
  FFN_B200_ERR_SCRATCH = 8         /* needs more scratch than ffn_b200_run_noalloc holds */
} ffn_b200_status;

typedef enum { FFN_B200_F16 = 0, FFN_B200_BF16 = 1 } ffn_b200_dtype;

/* Index into the reference's DOWN_IMPLS tuple (ops/host/dispatch.py:15). */
typedef enum {
  FFN_B200_DOWN_BASIC = 0,
  FFN_B200_DOWN_FULL_LOAD_A = 1,
  FFN_B200_DOWN_FULL_LOAD_B = 2,
  FFN_B200_DOWN_STREAMK = 3
} ffn_b200_down_impl;

/* Activation of the hidden layer (the problem's `gelu` field): the reference kernel's rational
 * GELU (its clipped rational erf, ops/kernel/ffn.py:548-572, validation/reference.py:5-13),
 * the exact-erf GELU (CUDA's erff), SiLU (z * sigmoid(z)), or SwiGLU (SiLU(x.Wg^T) * (x.Wu^T)); the
 * last two are beyond the reference's V1.  For SwiGLU, h is the hidden width and W1 holds
 * ffn_b200_swiglu_rows(h, plan.swap_ab) rows: with swap_ab == 0, blocks of 64 gate rows each
 * followed by the matching 64 up rows (zero rows pad the last block); with swap_ab == 1, gate
 * row i at row 2i and up row i at row 2i + 1.  W1 is then not a Linear weight of shape [h, K]:
 * plan first, pack, then prepare (ffn_optim_b200.prepare_ffn does this). */
typedef enum { FFN_B200_GELU_RATIONAL = 0, FFN_B200_GELU_ERF = 1, FFN_B200_SILU = 2, FFN_B200_SWIGLU = 3 } ffn_b200_gelu;

/* Weight storage: the input dtype, or fp8 e4m3 codes with one fp32 scale per row
 * (W[r, c] = code[r, c] * scale[r]; see ffn_b200_quantize_fp8_rows).  fp8 weights are
 * widened to the input dtype on chip; they apply to decode tiles (M <= 64). */
typedef enum { FFN_B200_WEIGHTS_NATIVE = 0, FFN_B200_WEIGHTS_FP8_ROWS = 1 } ffn_b200_weight_format;

/* Device-side error codes written to status[0] by the kernel (0 = no error). */
typedef enum {
  FFN_B200_KERNEL_OK = 0,
  FFN_B200_KERNEL_PIPE_TIMEOUT = 1, /* an on-chip pipeline wait ran past the wait limit */
  FFN_B200_KERNEL_DEP_TIMEOUT = 2,  /* a down tile waited too long for its hidden rows */
  FFN_B200_KERNEL_SK_TIMEOUT = 3,   /* a Stream-K owner (or a hidden-slice reduction) waited too
                                       long for a partial */
  FFN_B200_KERNEL_PEER_TIMEOUT = 4, /* a band owner waited too long for another GPU's partial */
  FFN_B200_KERNEL_CLAIM_RANGE = 5,  /* a tile claim fell outside this launch's range: the
                                       counters were not reset after an earlier error */
  FFN_B200_KERNEL_FP16_RANGE = 6    /* fp8 weights with bf16 activations: an activation is
                                       beyond +-65504, the fp16 range of that path's MMA */
} ffn_b200_kernel_error;

typedef struct {
  int64_t m, k, h, n;  /* M = prod(leading dims of X) */
  int32_t dtype;       /* ffn_b200_dtype */
  int32_t down_impl;   /* ffn_b200_down_impl */
  int32_t gelu;        /* ffn_b200_gelu */
  int32_t block_num;   /* persistent CTA count; 0 = one per SM */
  int32_t sm_count;    /* SMs of the target device; 0 = query the current device */
  /* Tuning overrides, 0 = automatic (benchmarks and tests use them): */
  int32_t tile_variant; /* 1 + variant id forces one kernel variant (automatic: CTA pairs for long
                           prefill runs -- at least 8 waves of 256x256 tiles --, else 128x256 or
                           128x128 one-CTA tiles; decode tiles for M <= 64)
                           (1: 128x256, 2: 128x128, 3: swap 16, 4: swap 64, 5: CTA pair 256x256,
                            6: swap 16 with 256-wide K stages, 7: swap 64 with 128-wide K stages,
                            8/9/10: hidden-resident row blocks with a 64/128/256-column Y
                            (down_impl full_load_a only), 11/12: swap 16 / swap 64 with fp8
                            weights (weight_format FFN_B200_WEIGHTS_FP8_ROWS only), 13: hidden-
                            slice decode, M <= 16: clusters of 8 CTAs each owning 128 hidden
                            rows, no hidden tensor in global memory, Y reduced over the
                            clusters (automatic for M <= 16 when the clusters share the hidden
                            super-blocks evenly; plan.row_split = 8 is the cluster size)) */
  int32_t raster_group; /* tile rows per raster group (default: balances A and B bytes per wave) */
  int32_t l2_policy;    /* 1: no L2 eviction hints (default); 2: evict-last on the row operand and
                           evict-first on the column operand (measured: far more DRAM traffic);
                           3: explicit evict-normal hint on every operand load;
                           4: evict-last on the row operand only */
  int32_t schedule;     /* data-parallel tile order: 1 static (owner c takes tiles c, c+C, ...),
                           2 dynamic (after its first tile each owner claims the next tile of the
                           raster from a device counter), 3 static with bounded drift (an owner
                           starts its tile of wave i once every owner has started wave i-1);
                           0 = 3 for CTA-pair tiles, static otherwise */
  int32_t weight_format; /* ffn_b200_weight_format of W1 and W2 */
} ffn_b200_problem;

/* One GEMM phase (up: Z = X.W1^T, down: Y = hidden.W2^T) as scheduled on the device.
 * rows/cols are the tile grid of the MMA's A and B operands; k_blocks is the number of
 * tile_k-wide K steps (pipeline stages) per tile.  dp_tiles are computed whole by one CTA; the sk_tiles tail
 * is split along K over the first sk_ctas CTAs (Stream-K), sk_iters (+1 for the first
 * sk_rem CTAs) K steps per CTA. */
typedef struct {
  int32_t tiles_r, tiles_q, tiles, k_blocks;
  int32_t dp_tiles, sk_tiles, sk_iters, sk_rem;
  int32_t group;
  int32_t sk_ctas; /* CTAs sharing the Stream-K tail (the first sk_ctas; each gets >= 16 K steps) */
} ffn_b200_phase_plan;

typedef struct {
  int32_t variant;       /* kernel instantiation id */
  int32_t swap_ab;       /* 1: weights are the MMA's M operand and tokens its N (small M) */
  int32_t cta_pair;      /* 1: a cluster of two CTAs computes each tile (tcgen05 cta_group::2) */
  int32_t tile_m, tile_n, tile_k, stages;
  int32_t block_num;     /* CTAs launched (even for CTA pairs) */
  int32_t tmem_cols;
  int64_t smem_bytes;
  ffn_b200_phase_plan up, down;
  int64_t workspace_floats; /* fp32 Stream-K partials: 2 phases x block_num x tile_m x tile_n */
  int64_t counter_words;    /* u32 words: two u64 tile-claim counters (up, down), the u64
                               launch count (the device-side launch epoch), then the
                               hidden-row-block readiness counters */
  int64_t flag_words;       /* u32 Stream-K partial-ready flags: 2 x block_num */
  int64_t status_words;     /* i32 status words */
  int32_t schedule;         /* resolved schedule: 1 static, 2 dynamic, 3 static with bounded drift */
  int32_t row_split;        /* row-block plans: CTAs (one cluster) sharing each row block's H
                               chunks, 1, 2, 4 or 8; 1 for the other plans */
} ffn_b200_plan;

/* Device buffers.  ld* are row pitches in elements; each must be a multiple of 8 and each
 * base 16-byte aligned (TMA).  hidden is [M, ldh] scratch of the input dtype; y is the
 * [M, ldy] output.  workspace/counters/flags/status are sized by ffn_b200_plan and must be
 * zero-filled before the first run of a handle; counters must be 8-byte aligned. */
typedef struct {
  const void* x;  int64_t ldx;
  const void* w1; int64_t ldw1;
  const void* w2; int64_t ldw2;
  void* hidden;   int64_t ldh;
  void* y;        int64_t ldy;
  float* workspace;
  uint32_t* counters;
  uint32_t* flags;
  int32_t* status;
  const float* w1_scale; /* FFN_B200_WEIGHTS_FP8_ROWS: [H] and [N] fp32 row scales, else NULL */
  const float* w2_scale;
  const void* bias1;     /* optional [H] and [N] biases in the input dtype (16-byte aligned), or
                            NULL: hidden = act(X.W1^T + b1), Y = hidden.W2^T + b2, each bias
                            added to the fp32 sum (beyond the reference's V1) */
  const void* bias2;
} ffn_b200_buffers;

typedef struct ffn_b200_handle ffn_b200_handle;

FFN_B200_EXPORT int ffn_b200_abi_version(void);
FFN_B200_EXPORT const char* ffn_b200_strerror(int code);

/* Number of SMs and compute capability of a device (no kernel launch). */
FFN_B200_EXPORT int ffn_b200_device_info(int device, int* sm_count, int* cc_major, int* cc_minor);

/* Host-only planning: tile shapes, Stream-K split and scratch sizes.  Needs no GPU when
 * problem->sm_count > 0. */
FFN_B200_EXPORT int ffn_b200_make_plan(const ffn_b200_problem* problem, ffn_b200_plan* plan);

/* Validates device and buffers, encodes the TMA tensor maps and returns a handle that
 * launches one fused kernel per ffn_b200_run.  The launch epoch lives on the device (a
 * 64-bit launch count at the start of `counters`), so the readiness counters never need
 * clearing between runs and a run captured in a CUDA graph replays any number of times. */
FFN_B200_EXPORT int ffn_b200_prepare(const ffn_b200_problem* problem, const ffn_b200_buffers* buffers,
                     int device, ffn_b200_handle** handle);

/* One asynchronous launch on `stream` (a cudaStream_t; may be capturing into a CUDA graph).
 * Runs of one handle must be serialised on one stream (graph replays included). */
FFN_B200_EXPORT int ffn_b200_run(ffn_b200_handle* handle, void* stream);

/* Re-points X and Y of a prepared handle (same shapes and pitches) without re-planning. */
FFN_B200_EXPORT int ffn_b200_rebind_io(ffn_b200_handle* handle, const void* x, void* y);

/* Clears counters, flags and status on `stream` and restarts the epoch; call after a run
 * reported a kernel error. */
FFN_B200_EXPORT int ffn_b200_reset(ffn_b200_handle* handle, void* stream);

/* Upper bound, in nanoseconds, of every wait inside the kernel (default 4 s). */
FFN_B200_EXPORT int ffn_b200_set_wait_limit(ffn_b200_handle* handle, uint64_t nanoseconds);

/* Test hook: 1 makes every down tile wait for one readiness signal too many, so the
 * bounded wait runs out and the kernel reports FFN_B200_KERNEL_DEP_TIMEOUT. */
FFN_B200_EXPORT int ffn_b200_set_fault_injection(ffn_b200_handle* handle, int mode);

/* ---- Multi-GPU (tensor parallel over H) with the reduce-scatter fused into the kernel ----
 * Peer-visible device buffers: ffn_b200_peer_alloc allocates `bytes` (zeroed) on the current
 * device and returns a 64-byte CUDA IPC handle; another process opens it with
 * ffn_b200_peer_open (NVLink peer access), closes with ffn_b200_peer_close; the owner frees
 * with ffn_b200_peer_free.  Reference counterpart: none (the reference is single-device;
 * this replaces an NCCL reduce-scatter after the kernel). */
FFN_B200_EXPORT int ffn_b200_peer_alloc(uint64_t bytes, void** dev_ptr, void* ipc_handle);
FFN_B200_EXPORT int ffn_b200_peer_open(const void* ipc_handle, void** dev_ptr);
FFN_B200_EXPORT int ffn_b200_peer_close(void* dev_ptr);
FFN_B200_EXPORT int ffn_b200_peer_free(void* dev_ptr);

/* Element type of the partial Y tiles that the fused reduce-scatter sends between GPUs:
 * fp32 (default: the owner sums unrounded partials, so P GPUs keep the single-GPU error
 * bound), the input dtype (half the NVLink bytes; each partial is rounded once before the
 * sum, which adds up to P-1 roundings to every output), or fp32 rounded to nearest at 24
 * bits (sign, exponent, 15 mantissa bits: 3/4 of the fp32 bytes, sent as a 16-bit and an
 * 8-bit plane; each partial carries a relative error below 2^-16, 128 times finer than a
 * bf16 output ulp). */
typedef enum { FFN_B200_PARTIAL_F32 = 0, FFN_B200_PARTIAL_INPUT = 1, FFN_B200_PARTIAL_F24 = 2 } ffn_b200_partial;

/* Sizes of one rank's staging buffer (partial tiles of type `partial`, two launch
 * parities) and push counts for a `world`-GPU reduce-scatter of this handle's down phase. */
FFN_B200_EXPORT int ffn_b200_reduce_scatter_bytes(const ffn_b200_handle* handle, int world, int32_t partial,
                                                  uint64_t* stage_bytes, uint64_t* flag_bytes);

/* Turns the handle's down phase into a fused reduce-scatter over `world` GPUs: this rank
 * (`rank`) owns Y rows [rank*M/world, (rank+1)*M/world), written to `y_local`
 * ([M/world, ldy_local]); stage_ptrs[r] / flag_ptrs[r] are rank r's staging and count
 * buffers as mapped in this process (own ones included).  Every rank runs its handle once
 * per step; partial tiles of other bands (of type `partial`, the same on every rank) are
 * pushed over NVLink during the epilogue and summed by their owner in ascending rank order.  Needs M divisible by world*128 and a
 * one-CTA prefill tile.  After a kernel error all ranks reset together. */
FFN_B200_EXPORT int ffn_b200_set_reduce_scatter(ffn_b200_handle* handle, int world, int rank, int32_t partial,
                                                void* const* stage_ptrs, void* const* flag_ptrs, void* y_local,
                                                int64_t ldy_local);

/* Overlapped launches (programmatic dependent launch; off by default): with enable = 1,
 * each later run lets its CTAs start, and set up their barriers and tensor memory, while
 * the stream's previous kernel is still finishing; every global memory access of the
 * kernel waits (griddepcontrol.wait) until that kernel has completed and its writes are
 * visible, so results and stream order are those of serial launches.  Saves the launch gap
 * and the setup of back-to-back calls (decode loops, CUDA graphs).  No counterpart in the
 * reference. */
FFN_B200_EXPORT int ffn_b200_set_launch_overlap(ffn_b200_handle* handle, int32_t enable);

/* Tracing: when `device_stamps` (a device uint64[block_num][16], or NULL to switch off) is
 * set, every later run writes per-CTA %globaltimer stamps (ns): 0 setup done, 1 first TMA
 * load, 2 first down tile's hidden rows ready, 3 last load, 4 last MMA commit, 5 last up
 * tile stored, 6 first down accumulator in the epilogue, 7 end; word 8 holds the SM id the
 * CTA ran on (words 9-15 are reserved).  Reference counterpart:
 * the separate profiler pass of performance/collect.py:38-72. */
FFN_B200_EXPORT int ffn_b200_set_trace(ffn_b200_handle* handle, uint64_t* device_stamps);

/* Work-list placement: `device_map` (a device int32[C], C = block_num / CTAs per tile, or
 * NULL for launch order) gives the work-list index of each CTA (CTA pair); it must be a
 * permutation of 0..C-1 and stay valid while set.  Tiles that share operand strips go to
 * neighbouring indices, so the map decides which SMs (GPC, die) share them.  prepare sets
 * one itself for CTA-pair plans that cover every SM: pairs numbered in the GPC-major order
 * of a cooperative launch, measured once per device by two probe launches.  get_owner_map
 * copies up to `capacity` entries of the map in use to host memory and sets `count` to C,
 * or to 0 for launch order.  No reference counterpart (the reference's block-to-tile order
 * is its launch order). */
FFN_B200_EXPORT int ffn_b200_set_owner_map(ffn_b200_handle* handle, const int32_t* device_map);

/* fp8 weights: row r of `src` [rows, cols] (fp16/bf16, pitch ld_src elements) becomes
 * scales[r] = absmax(row) / 448 (1 for a zero row) and codes dst[r, c] =
 * RN-even, saturating e4m3(src[r, c] / scales[r]) with IEEE fp32 division; dst pitch ld_dst
 * bytes (a multiple of 16 for TMA).  Asynchronous on `stream`.  No reference counterpart
 * (the reference has no quantized weights). */
FFN_B200_EXPORT int ffn_b200_quantize_fp8_rows(const void* src, int64_t ld_src, int32_t dtype, int64_t rows,
                                               int64_t cols, void* dst, int64_t ld_dst, float* scales, void* stream);
FFN_B200_EXPORT int ffn_b200_get_owner_map(const ffn_b200_handle* handle, int32_t* host_out, int32_t capacity,
                                           int32_t* count);

FFN_B200_EXPORT int ffn_b200_get_plan(const ffn_b200_handle* handle, ffn_b200_plan* plan);
/* Rows of the packed W1 of a SwiGLU problem with hidden width h (see ffn_b200_gelu). */
FFN_B200_EXPORT int64_t ffn_b200_swiglu_rows(int64_t h, int32_t swap_ab);
FFN_B200_EXPORT int ffn_b200_destroy(ffn_b200_handle* handle);

/* Device scratch held by the library itself for ffn_b200_run_noalloc (hidden activations,
 * Stream-K partials and synchronisation words of one call). */
#define FFN_B200_NOALLOC_SCRATCH_BYTES (32ll << 20)

/* Allocation-free run.  No counterpart in the reference: it exists for callers that must
 * not allocate device memory while they run the FFN -- for example an inference engine that
 * hands its plugins a fixed memory budget and calls them from its execution path, where a
 * cudaMalloc would be refused or would synchronise the whole device, or a serving loop that
 * reserves all memory up front.  The caller passes X, W1, W2 and Y (same layout rules as
 * ffn_b200_buffers); the hidden tensor, Stream-K partials and counters live in a 32 MiB
 * array inside the library (FFN_B200_NOALLOC_SCRATCH_BYTES, held by every GPU that loads
 * this code until the process exits).  Problems whose scratch does not fit return
 * FFN_B200_ERR_SCRATCH.  `status` is an optional device int32[4] that receives the kernel's
 * error words (NULL keeps them inside the scratch).  The first call on a device looks up
 * the array's device address (once per device, with that device current); make that first
 * call before any stream capture.  Every call clears the counters it needs on `stream` and
 * then launches once; all calls share the one array, so calls that overlap on the GPU (two
 * streams, two host threads) race and must be serialised by the caller. */
FFN_B200_EXPORT int ffn_b200_run_noalloc(const ffn_b200_problem* problem, const void* x, int64_t ldx,
                                         const void* w1, int64_t ldw1, const void* w2, int64_t ldw2, void* y,
                                         int64_t ldy, int32_t* status, void* stream);

/* One-shot: prepare, clear the scratch words, run once, release the handle. */
FFN_B200_EXPORT int ffn_b200_launch(const ffn_b200_problem* problem, const ffn_b200_buffers* buffers,
                    void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FFN_B200_H */
