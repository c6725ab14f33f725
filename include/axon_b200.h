/*
 * axon_b200.h -- C ABI of the Axon B200 kernel library (libaxon_b200.so).
 *
 * This library replaces the compile + bench leg of Axon (src/axon/bench_runner.py:
 * `_compile_one_nki_kernel` :226-272 and `_bench_one_neff` :144-223, driven by
 * `run_nki_bench` :576-825): instead of compiling an emitted NKI module to a
 * NEFF and running it on a NeuronCore, the host calls one of the entry points
 * below with device pointers.
 *
 * Conventions shared by every entry point:
 *   - Pointers are CUDA device pointers (or managed/peer pointers reachable from
 *     the current device). The caller owns every allocation; scratch space, where
 *     a kernel needs any, is passed in (see the *_workspace_bytes queries).
 *   - Sizes and leading dimensions are in ELEMENTS, int64.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     No entry point synchronises the host; all work is enqueued on `stream`.
 *   - The return value is AXON_OK (0) or a negative AXON_E_* code; the message
 *     for the last failure on the calling thread is axon_last_error().
 *   - `tune` may be NULL (defaults). Its fields select a kernel variant and its
 *     tile knobs; axon_variants() lists what each op accepts. A knob the op does
 *     not use is ignored; a knob outside its legal set is AXON_E_ARG.
 *   - Row-wise ops require row starts and leading dimensions such that every row
 *     begins on a 16-byte boundary for the vectorised path; otherwise they take a
 *     scalar path (same results).
 */
#ifndef AXON_B200_H
#define AXON_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define AXON_API __attribute__((visibility("default")))
#else
#define AXON_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
#define AXON_OK 0
#define AXON_E_SHAPE (-1)       /* sizes out of range or inconsistent           */
#define AXON_E_ALIGN (-2)       /* pointer / stride alignment the op requires    */
#define AXON_E_LAUNCH (-3)      /* kernel launch failed (cudaGetLastError)       */
#define AXON_E_TIMEOUT (-4)     /* a bounded device-side wait gave up            */
#define AXON_E_UNSUPPORTED (-5) /* dtype / variant / layout not implemented      */
#define AXON_E_ARG (-6)         /* bad argument (NULL pointer, bad tune knob)    */
#define AXON_E_CUDA (-7)        /* other CUDA runtime / driver error             */

/* ---- element types -------------------------------------------------------- */
typedef enum axon_dtype {
  AXON_F32 = 0,
  AXON_BF16 = 1,
  AXON_F16 = 2
} axon_dtype_t;

/* ---- variant / tile selection ------------------------------------------- *
 * The CUDA counterpart of Axon's (hw_variant, TILES_IN_BLOCK_*) key
 * (src/axon/bench_runner.py:364-388, src/axon/candidate_filter.py:18-45).
 * Zero in any field means "the op's default".                               */
typedef struct axon_tune {
  int32_t variant;      /* kernel variant id within the op (0 = default)      */
  int32_t threads;      /* CTA size for row / elementwise kernels             */
  int32_t rows_per_cta; /* rows handled by one CTA (row kernels)              */
  int32_t block_m;      /* GEMM CTA tile rows (128)                           */
  int32_t block_n;      /* GEMM CTA tile cols (64..256, multiple of 16)       */
  int32_t block_k;      /* GEMM k-slab per pipeline stage (64)                */
  int32_t stages;       /* GEMM smem pipeline depth (2..8)                    */
  int32_t split;        /* cumsum: elements per tile (variant 0) or CTAs per
                           row cluster (variant 1)                            */
  int32_t precision;    /* silu_mlp activation storage: 1 = one bf16 value,
                           2 / 3 = split terms, 4 = f16, 5 = f16 with an f16
                           W_down from the caller (see axon_silu_mlp)        */
  int32_t max_ctas;     /* GEMM: cap on the persistent grid (0 = one CTA per
                           SM); leaves SMs free for a concurrent collective   */
} axon_tune_t;

/* ---- library metadata ----------------------------------------------------- */

/* Version string, e.g. "axon_b200 0.1.0 sm_100a". */
AXON_API const char* axon_version(void);

/* Message of the last failed call on this thread ("" if none). */
AXON_API const char* axon_last_error(void);

/* Write a JSON description of `op`'s variants and their tile constraints into
 * buf (NUL-terminated, truncated to len). Returns the full length needed, or a
 * negative AXON_E_* code for an unknown op. Replaces the literal
 * `__axon_tile_constraints__` manifest Axon embeds in each emitted module
 * (src/axon/candidate_filter.py:13, :56-87). */
AXON_API int64_t axon_variants(const char* op, char* buf, int64_t len);

/* ---- row-wise normalisation ------------------------------------------------ */

/* y = x * rsqrt(scale * sum_j x[i,j]^2 + eps) * w[j]       (w may be NULL)
 * scale = 1, eps = 0, w = NULL is Axon's `rmsnorm` spec (x / sqrt(sum x^2),
 * kernels/rmsnorm/refs.py:26-30); scale = 1/n, eps = 1e-6 with a weight is the
 * Llama form. Accumulates in fp32. x, y: [m, n] with leading dims ld_x, ld_y;
 * w: [n] of w_dtype. Replaces the compiled `rmsnorm` NEFF. */
AXON_API int axon_rmsnorm(const void* x, const void* w, void* y, int64_t m, int64_t n,
                 int64_t ld_x, int64_t ld_y, int32_t dtype, int32_t w_dtype,
                 float scale, float eps, const axon_tune_t* tune, void* stream);

/* y = (x - mean) / sqrt(mean((x - mean)^2) + eps) per row, no affine
 * (Axon kernels/layernorm/refs.py:26-32). */
AXON_API int axon_layernorm(const void* x, void* y, int64_t m, int64_t n, int64_t ld_x,
                   int64_t ld_y, int32_t dtype, float eps, const axon_tune_t* tune,
                   void* stream);

/* y = exp(x) / sum(exp(x)) per row (Axon kernels/softmax/refs.py:11-13),
 * evaluated max-shifted. */
AXON_API int axon_softmax(const void* x, void* y, int64_t m, int64_t n, int64_t ld_x,
                 int64_t ld_y, int32_t dtype, const axon_tune_t* tune, void* stream);

/* Row-op variants (tune->variant) for the three calls above: 0 = automatic
 * (with 16-byte aligned rows and at least a row per SM: variant 3 for rows of
 * 16 KB and more, variant 2 below; otherwise rows held in registers, or
 * streaming passes for rows too long for them), 1 = streaming passes (any
 * length or alignment), 2 = one warp per row staged in shared memory by bulk
 * copies (16-byte aligned rows of at most 32 KB; tune->threads = warps per
 * CTA x 32), 3 = one persistent CTA per row staged in shared memory in chunks
 * by bulk copies, each chunk refilled with the CTA's next row once read
 * (16-byte aligned rows of a multiple of 16 bytes up to 204544 bytes;
 * tune->threads 64..1024, tune->block_k = chunk KB, tune->max_ctas caps the
 * grid).
 * Synchronise `stream` and report whether a variant-2 or -3 launch since the
 * last call gave up on a bounded copy wait (AXON_E_TIMEOUT; the flag is cleared).
 * No counterpart in the reference (NKI kernels have no device status). */
AXON_API int axon_row_status(void* stream);

/* ---- rotary embedding ------------------------------------------------------ */

/* Axon's `rope` spec layout (kernels/rope/refs.py:26-30): four [half_d, free]
 * tensors of `dtype`, two outputs:
 *   out_even = x_even*cos - x_odd*sin,  out_odd = x_odd*cos + x_even*sin.
 * Outputs may alias their matching inputs (in-place). */
AXON_API int axon_rope_split(const void* x_even, const void* x_odd, const void* cos_t,
                    const void* sin_t, void* out_even, void* out_odd, int64_t half_d,
                    int64_t free_n, int32_t dtype, const axon_tune_t* tune,
                    void* stream);

/* Rotate-half rope on q [seq, n_q, head_dim] and k [seq, n_kv, head_dim]
 * (contiguous, `dtype`), with fp32 tables cos/sin [seq, head_dim/2]:
 *   out[..., :h] = x1*cos - x2*sin,  out[..., h:] = x2*cos + x1*sin.
 * k / k_out may be NULL when n_kv == 0. Outputs may alias inputs. */
AXON_API int axon_rope_rotate_half(const void* q, const void* k, const float* cos_t,
                          const float* sin_t, void* q_out, void* k_out, int64_t seq,
                          int64_t n_q, int64_t n_kv, int64_t head_dim, int32_t dtype,
                          const axon_tune_t* tune, void* stream);

/* ---- prefix sum -------------------------------------------------------------- */

/* Bytes of scratch axon_cumsum needs for this shape and tune (0 if none). */
AXON_API int64_t axon_cumsum_workspace_bytes(int64_t m, int64_t n, const axon_tune_t* tune);

/* Inclusive scan along the last axis (Axon kernels/cumsum/refs.py:20-22):
 * y[i, j] = sum_{t<=j} x[i, t], accumulated in fp32 with a float64 running
 * carry between tiles. in_dtype / out_dtype: AXON_F32 or AXON_BF16.
 * Variant 0: single-pass decoupled look-back across tiles of a row; needs
 * `workspace` (zeroed by the call itself, on `stream`); every device-side
 * wait is bounded and a wait that gives up records AXON_E_TIMEOUT in the
 * workspace status word (read it with axon_cumsum_status). With no
 * tune->split, variant 0 runs a chunk-streaming variant instead when m >= 128
 * and the input rows are 16-byte aligned: variant 3 (16 KB chunks) for rows
 * of at most 32 KB when a workspace is given, else variant 2 (the workspace
 * then only carries the status word). A workspace used with variant 0 is
 * therefore zero-filled before its first use, as variant 3 requires.
 * Variant 1: one thread-block cluster per row exchanging tile sums through
 * distributed shared memory; needs no workspace.
 * Variant 2: one CTA streams each row through a ring of shared-memory chunks
 * filled by bulk copies (tune->stages, tune->block_k = chunk KB); needs no
 * workspace and 16-byte aligned input rows.
 * Variant 3: rows cut into variant 2's chunks, and every CTA (one
 * 1024-thread CTA per SM, min(SMs, m) CTAs; tune->max_ctas caps it) streams
 * an equal contiguous range of the row-major chunk sequence, so the SMs carry
 * equal bytes whatever m is. A row split between two CTAs takes the float64
 * running sum of its head from the previous CTA through a workspace slot:
 * the workspace (axon_cumsum_workspace_bytes) must be zero-filled before its
 * first use and every completed call leaves it so; after AXON_E_TIMEOUT zero
 * it again. tune->stages (default 4) x tune->block_k (16 or 32 KB, default
 * 32) is the ring per CTA; 16-byte aligned input rows.
 * Variants 1, 2 and 3 record a bulk-copy or carry wait that gave up in a
 * device word: axon_cumsum_status(NULL, ...). */
AXON_API int axon_cumsum(const void* x, void* y, int64_t m, int64_t n, int64_t ld_x,
                int64_t ld_y, int32_t in_dtype, int32_t out_dtype, void* workspace,
                int64_t workspace_bytes, const axon_tune_t* tune, void* stream);

/* Synchronise `stream` and report AXON_E_TIMEOUT if a bounded wait gave up:
 * the status word a cumsum left in `workspace` (may be NULL) or the device
 * word of the bulk-copy variants (read and cleared here). */
AXON_API int axon_cumsum_status(const void* workspace, void* stream);

/* Allocation-free form of axon_cumsum (variant 0 only). No counterpart in the
 * reference: it exists for callers that must not allocate device memory --
 * a plugin whose host framework owns every device allocation, or a
 * latency-critical path where cudaMalloc, which can synchronise the device,
 * is not allowed. Instead of a caller workspace it uses one 1 MiB static
 * device array per device that loads the library (held until the process
 * exits), so a scan may use at most (1 MiB - 32) / 32 = 32767 look-back tiles
 * (m * ceil(n / tile), tile = tune->split elements, default 8192); larger
 * shapes return AXON_E_SHAPE. It calls no cudaMalloc or cudaFree. The first
 * call on a device looks up the array's device address (cudaGetSymbolAddress),
 * so make that first call before any stream capture. Every call clears the
 * array on `stream` and then uses it: calls that overlap on the GPU (other
 * streams, other threads) race on the one array and must be serialised by
 * the caller. A look-back wait that gives up records AXON_E_TIMEOUT in the
 * library's device status word, which axon_cumsum_status(NULL, stream) reads
 * and clears; check it before trusting the output. The address lookup is
 * repeated when the current device's context changes (after a
 * cudaDeviceReset, for example). */
AXON_API int axon_cumsum_noalloc(const void* x, void* y, int64_t m, int64_t n, int64_t ld_x,
                                 int64_t ld_y, int32_t in_dtype, int32_t out_dtype,
                                 const axon_tune_t* tune, void* stream);

/* ---- optimizer ---------------------------------------------------------------- */

typedef struct axon_adam_hparams {
  float beta1;        /* 0.9 in Axon's spec (kernels/fused_adam/kernel.py:20) */
  float beta2;        /* 0.999 in Axon's spec (:21)                           */
  float eps;          /* 1e-8 (:22)                                           */
  float step_size;    /* used when step_size_rows == NULL                    */
  float inv_bc2_sqrt; /* used when inv_bc2_sqrt_rows == NULL                 */
  float wd;           /* used when wd_rows == NULL                           */
} axon_adam_hparams_t;

/* L2-regularised Adam over a [rows, cols] block (Axon kernels/fused_adam/
 * refs.py:38-46):
 *   g' = g + wd*p;  m' = b1*m + (1-b1)*g';  v' = b2*v + (1-b2)*g'^2;
 *   p' = p - m' / (sqrt(v')*inv_bc2_sqrt + eps) * step_size.
 * param / exp_avg / exp_avg_sq and their outputs have `state_dtype`, grad has
 * `grad_dtype`; per-row scalars (length rows, `row_dtype`) may be NULL to use
 * the hparams values. Outputs may alias inputs (in-place update). All tensors
 * are contiguous. */
AXON_API int axon_adam(const void* param, const void* grad, const void* exp_avg,
              const void* exp_avg_sq, void* param_out, void* exp_avg_out,
              void* exp_avg_sq_out, int64_t rows, int64_t cols, int32_t state_dtype,
              int32_t grad_dtype, const void* step_size_rows,
              const void* inv_bc2_sqrt_rows, const void* wd_rows, int32_t row_dtype,
              const axon_adam_hparams_t* hp, const axon_tune_t* tune, void* stream);

/* ---- dense ------------------------------------------------------------------- */

#define AXON_EPI_NONE 0      /* C = A @ B                                        */
#define AXON_EPI_ROWSCALE 1  /* C = row_scale[i] * (A @ B)                       */
#define AXON_EPI_SILU_GATE 2 /* C = silu(A @ B) * (A @ B2)  (B2 = up weight)     */
#define AXON_EPI_EXP 3       /* C = exp(A @ B)  (bare exponential, no shift)      */

/* tcgen05 / TMEM GEMM: A [m, k] row-major (lda), B [k, n] row-major (ldb) --
 * the layout Axon's specs pass (kernels/matmul/refs.py:24-25) -- C [m, n]
 * (ldc). A, B, B2: AXON_BF16 or AXON_F16 (same type); C: AXON_BF16, AXON_F16
 * or AXON_F32. fp32 accumulation in tensor memory. k and n must be multiples
 * of 8, lda/ldb/ldc multiples of 8 elements, bases 16-byte aligned (TMA).
 * row_scale: fp32 [m] for AXON_EPI_ROWSCALE, else NULL. b2: [k, n] for
 * AXON_EPI_SILU_GATE, else NULL.
 * tune->variant: 1 = one CTA per 128 x block_n tile (cta_group::1);
 * 2 = CTA pairs, a cluster of two SMs per 256 x block_n tile
 * (cta_group::2, block_n 128 or 256); 0 (default) = 2 unless m < 256, the
 * 256-row tiling would add a mostly empty tile, or block_n is 64.
 * tune->stages: shared-memory ring depth (0 = deepest that fits);
 * tune->max_ctas caps the persistent grid (CTAs, pairs count as two);
 * tune->split > 0 orders the persistent tiles in bands of that many row tiles
 * (each band column by column) instead of column-major over all of them --
 * same tiles, same bits; on B200 it was within run-to-run noise (about 15%)
 * of the default at 8192^3 and the SwiGLU shapes, so the default stays 0. */
AXON_API int axon_gemm(const void* a, const void* b, const void* b2, void* c,
              const float* row_scale, int64_t m, int64_t n, int64_t k, int64_t lda,
              int64_t ldb, int64_t ldc, int32_t ab_dtype, int32_t c_dtype,
              int32_t epilogue, const axon_tune_t* tune, void* stream);

/* Synchronise `stream` and report whether a GEMM since the last call gave up
 * on a bounded pipeline wait (AXON_E_TIMEOUT; the flag is then cleared). */
AXON_API int axon_gemm_status(void* stream);

/* ---- tensor-parallel SwiGLU over NVLink peer memory ----------------------- */

/* The reference's TP MLP resolves the down projection's Partial(+) output with
 * a terminal all-reduce (src/axon/sharding.py:380-384, :514-522). These calls
 * replace that all-reduce with a reduce-scatter fused into the down-projection
 * GEMM plus an owner-side reduce and all-gather push, all over peer memory
 * shared by CUDA IPC. The reference has no counterpart entry points (its
 * collectives are NKI/Neuron runtime calls); the host sequence is
 * enzyme_b200/tp.py `TPSwiGLU(fused=True)`. */

#define AXON_IPC_HANDLE_BYTES 64

/* IPC handle of the allocation holding dev_ptr, and dev_ptr's byte offset in
 * it (torch allocations are sub-ranges of larger device allocations). */
AXON_API int axon_ipc_handle(const void* dev_ptr, void* handle, int64_t* offset);
/* Map a peer process's allocation; *dev_ptr = its base + offset. A process
 * cannot open its own handle. */
AXON_API int axon_ipc_open(const void* handle, int64_t offset, void** dev_ptr);
AXON_API int axon_ipc_close(void* dev_ptr, int64_t offset);

/* Down projection of one token slab on rank `rank` of `world` (<= 8):
 * partial = act [m, k] @ w [k, n] (bf16 x bf16 or f16 x f16, fp32
 * accumulation in TMEM), rounded to f16, with row r written by the GEMM
 * epilogue straight into owner o = r / rows_per_owner's inbox
 * inboxes[o] (a peer or local buffer laid out [world][rows_per_owner][n] f16)
 * at [rank][r - o * rows_per_owner]. m = world * rows_per_owner. tune as
 * axon_gemm's. */
AXON_API int axon_tp_down_partial(const void* act, const void* w, void* const* inboxes, int32_t world,
                         int32_t rank, int64_t m, int64_t n, int64_t k, int64_t rows_per_owner,
                         int32_t ab_dtype, const axon_tune_t* tune, void* stream);

/* Both GEMMs of one rank's SwiGLU shard in one CTA-pair kernel (the fused
 * kernel axon_silu_mlp runs at precision 4): act = silu(x @ w_gate) *
 * (x @ w_up) as f16 in `workspace`, then act @ w_down_h (f16 [n, p], the
 * caller's f16 copy of W_down) with the down projection's f16 partial rows
 * scattered to the owners' inboxes as axon_tp_down_partial does.
 * x [m, k] bf16, w_gate/w_up [k, n] bf16; m = world * rows_per_owner. */
AXON_API int64_t axon_tp_mlp_workspace_bytes(int64_t m, int64_t n);
AXON_API int axon_tp_mlp_partial(const void* x, const void* w_gate, const void* w_up,
                        const void* w_down_h, void* workspace, int64_t workspace_bytes,
                        void* const* inboxes, int32_t world, int32_t rank, int64_t m, int64_t n,
                        int64_t k, int64_t p, int64_t rows_per_owner, const axon_tune_t* tune,
                        void* stream);

/* One whole tensor-parallel SwiGLU step of rank `rank` in one kernel (world
 * 1, 2, 4 or 8; m a multiple of 256): the two GEMMs as axon_tp_mlp_partial,
 * with output rows owned in 8-row granules dealt to the ranks in turn (row r
 * belongs to rank (r / 8) % world), each phase-B warp writing its f16 partial
 * rows into the owners' inboxes and releasing them into the owners' arrival
 * counts arrive[o][r / 256] (system scope). Two reduction warps in every CTA,
 * beside the GEMM roles, resolve the all-reduce while the tiles go on: for
 * each of this rank's rows (1024-column units, in row-block order), once all
 * ranks' partials of its 256-row block have arrived, the world copies are
 * summed in fp32 in rank order, rounded once to bf16 and stored to every
 * rank's output ys[d] [m, p] bf16; at the end each warp adds its unit count
 * to done[d] on every rank. Counts accumulate: step `epoch` (1, 2, ...) is
 * complete on a rank when its done count reaches
 * epoch * axon_tp_step_done_per_epoch(world, m, p) (axon_tp_wait_count).
 * inbox = this rank's inbox, inboxes[o] = rank o's, each [world][m / world][p]
 * f16; workspace as axon_tp_mlp_partial's. tune->rows_per_cta sets the row
 * blocks per group of the tile order (default 4). */
AXON_API int64_t axon_tp_step_done_per_epoch(int32_t world, int64_t m, int64_t p);
AXON_API int axon_tp_mlp_step(const void* x, const void* w_gate, const void* w_up,
                     const void* w_down_h, void* workspace, int64_t workspace_bytes,
                     const void* inbox, void* const* inboxes, int32_t* const* arrive,
                     int32_t* const* done, void* const* ys, int32_t world, int32_t rank,
                     int32_t epoch, int64_t m, int64_t n, int64_t k, int64_t p,
                     const axon_tune_t* tune, void* stream);

/* The same step with the all-reduce done by the NVLink switch (NVLS): each
 * rank's phase-B warps write its f16 partial of y into its own buffer `part`
 * [m, p] (every rank's `part` bound to one NVLink multicast object whose
 * address is part_mc) and release the rows into every rank's arrival counts
 * arrive[d][r / 256]; the reduction warps read each 16-byte packet of this
 * rank's rows once through part_mc with multimem.ld_reduce (the switch adds
 * the world f16 copies, accumulating in fp32, and returns the f16 sum), round
 * it to bf16 and store it once with multimem.st to y_mc, the multicast
 * address of the [m, p] bf16 outputs, which the switch writes into every
 * rank's output. Each partial crosses NVLink once (to the switch) and each
 * output packet leaves its owner once. Counts and completion as
 * axon_tp_mlp_step (the same done count per epoch). The result may differ
 * from axon_tp_mlp_step's in the last bit (the switch's f16 rounding of the
 * sum before bf16); every rank holds the same bits. */
AXON_API int axon_tp_mlp_step_multicast(const void* x, const void* w_gate, const void* w_up,
                               const void* w_down_h, void* workspace, int64_t workspace_bytes,
                               void* part, const void* part_mc, void* y_mc,
                               int32_t* const* arrive, int32_t* const* done, int32_t world,
                               int32_t rank, int32_t epoch, int64_t m, int64_t n, int64_t k,
                               int64_t p, const axon_tune_t* tune, void* stream);

/* Bounded wait (~2 s) on `stream` until *counter >= target (wrap-safe); a
 * wait that gives up records AXON_E_TIMEOUT for axon_tp_status. A later
 * read of an output written through a multicast address is ordered after
 * the wait. */
AXON_API int axon_tp_wait_count(const int32_t* counter, int32_t target, void* stream);

/* After the work already on `stream`: a system-scope fence, then
 * flags[d][rank] = epoch (release) for every rank d (flags[d] = int32[world]
 * on rank d, peer-mapped). */
AXON_API int axon_tp_signal(int32_t* const* flags, int32_t world, int32_t rank, int32_t epoch,
                   void* stream);

/* Bounded wait (~2 s) on `stream` until flags[s] >= epoch for every s <
 * world; a wait that gives up records AXON_E_TIMEOUT for axon_tp_status. */
AXON_API int axon_tp_wait(const int32_t* flags, int32_t world, int32_t epoch, void* stream);

/* Owner side: wait (bounded) until arrive[s] >= epoch for all s, then
 * y_i = sum_s inbox[s][i] (fp32, in rank order, one rounding to out_dtype)
 * for the rows_per_owner x n rows of this rank, stored to every rank's output:
 * outs[d] + (out_row0 + rank * rows + i) * ld_out. max_ctas caps the grid
 * (0 = 2 x SMs) so it can run beside a GEMM. */
AXON_API int axon_tp_reduce_gather(const void* inbox, void* const* outs, const int32_t* arrive,
                          int32_t world, int32_t rank, int32_t epoch, int64_t rows, int64_t n,
                          int64_t out_row0, int64_t ld_out, int32_t out_dtype, int32_t max_ctas,
                          void* stream);

/* The same reduction with this rank's rows written to its own output only
 * (`out`, laid out as one of axon_tp_reduce_gather's outs) ... */
AXON_API int axon_tp_reduce_local(const void* inbox, void* out, const int32_t* arrive, int32_t world,
                         int32_t rank, int32_t epoch, int64_t rows, int64_t n, int64_t out_row0,
                         int64_t ld_out, int32_t out_dtype, int32_t max_ctas, void* stream);

/* ... and then copied to the other ranks by the copy engines: one
 * cudaMemcpyAsync of `bytes` from src (this rank's rows in its own output) to
 * dsts[d] (the same rows in rank d's output) for every d != rank, on
 * `stream`, in ring order from rank + 1. No SM runs the all-gather. */
AXON_API int axon_tp_push_rows(const void* src, void* const* dsts, int64_t bytes, int32_t world,
                      int32_t rank, void* stream);

/* The same reduction with the rows stored once, through out_mc: a multicast
 * address (an NVLink multicast object bound to every rank's output buffer,
 * e.g. a symmetric-memory allocation's multicast pointer), laid out as one of
 * axon_tp_reduce_gather's outs. The switch writes each 16-byte multimem store
 * into every rank's copy, so the all-gather leaves this GPU once instead of
 * world - 1 times. Each storing thread ends with an alias-proxy and a
 * system-scope fence; axon_tp_signal afterwards publishes the rows, and
 * axon_tp_wait on the reader orders them before its later reads. */
AXON_API int axon_tp_reduce_multicast(const void* inbox, void* out_mc, const int32_t* arrive,
                             int32_t world, int32_t rank, int32_t epoch, int64_t rows,
                             int64_t n, int64_t out_row0, int64_t ld_out, int32_t out_dtype,
                             int32_t max_ctas, void* stream);

/* Synchronise `stream`; AXON_E_TIMEOUT if a tensor-parallel flag wait gave up
 * since the last call (the record is then cleared). */
AXON_API int axon_tp_status(void* stream);

/* dst[i] = src[i] converted from src_dtype to dst_dtype (AXON_F32 / AXON_BF16 /
 * AXON_F16; round to nearest even), n elements, contiguous. No counterpart in
 * Axon's specs: the tensor-parallel SwiGLU step uses it to make the f16 copy
 * of its W_down shard once per step before its per-slab GEMMs. */
AXON_API int axon_cast(const void* src, void* dst, int64_t n, int32_t src_dtype, int32_t dst_dtype,
                       void* stream);

/* Diagnostic with no counterpart in the reference: one thread waits for at
 * most limit_ns (<= 5 s) on an mbarrier nothing arrives on and on the device
 * word *flag (which the caller leaves 0), using the bounded waits of the GEMM,
 * the cluster scan and the look-back scan; status2 (two int32 on the device)
 * receives AXON_E_TIMEOUT for each wait that gave up (AXON_OK if the flag was
 * set). Lets tests check the timeout path on a GPU without a fault or hang. */
AXON_API int axon_selftest_bounded_wait(int64_t limit_ns, void* status2, const void* flag, void* stream);

/* Per-row scale r[i] = rsqrt(scale * sum_j x[i,j]^2 + eps) in fp32: the norm
 * prologue of rmsnorm_matmul (Axon kernels/rmsnorm_matmul/refs.py:16-22) and
 * of the SwiGLU config's optional rmsnorm. */
AXON_API int axon_row_rsqrt(const void* x, float* r, int64_t m, int64_t n, int64_t ld_x,
                   int32_t dtype, float scale, float eps, void* stream);

/* (x / sqrt(sum x^2)) @ w (Axon kernels/rmsnorm_matmul/refs.py:16-22): the
 * row-norm prologue followed by the GEMM with a row-scale epilogue.
 * workspace: >= 4*m bytes (the per-row scales). */
AXON_API int axon_rmsnorm_matmul(const void* x, const void* w, void* y, void* workspace,
                        int64_t m, int64_t n, int64_t k, int32_t ab_dtype,
                        int32_t c_dtype, const axon_tune_t* tune, void* stream);

/* C = exp(A @ B) (AXON_EPI_EXP) and, when row_part is not NULL, the sum of
 * each row's stored values over each column tile of the GEMM:
 * row_part[t * part_ld + i] for row i and tile t < ceil(n / block_n)
 * (part_ld >= m; block_n as tune->block_n, or axon_gemm's default for n).
 * Shapes and alignment as axon_gemm. The softmax denominator of
 * axon_attention comes from these sums. */
AXON_API int axon_gemm_exp(const void* a, const void* b, void* c, float* row_part, int64_t part_ld,
                  int64_t m, int64_t n, int64_t k, int64_t lda, int64_t ldb, int64_t ldc,
                  int32_t ab_dtype, int32_t c_dtype, const axon_tune_t* tune, void* stream);

/* C = rsqrt(sum_k h^2 / k + eps)[i] * (h @ w) with h = x + r1 + r2, in one
 * kernel: the three [m, k] inputs (contiguous, bf16 or f16) are summed in
 * fp32 while the A operand is staged in shared memory, the row sums of h^2
 * accumulate beside it, and the scale is applied in the epilogue; h never
 * reaches global memory. w [k, n] (row-major), C [m, n] contiguous (c_dtype).
 * tune: block_n 128 / 256 / 384 / 512 (default: the narrowest covering n, so
 * a row block's inputs are read once up to n = 512), stages, split = k
 * splits (0: split while the tiles leave SMs idle; splits > 1 write fp32
 * partials to the workspace and a second pass adds them in order and applies
 * the scale), max_ctas. k and n multiples of 8. workspace:
 * axon_gemm_resid3_workspace_bytes(m, n, k, tune) bytes (0 without splits). */
AXON_API int64_t axon_gemm_resid3_workspace_bytes(int64_t m, int64_t n, int64_t k,
                                         const axon_tune_t* tune);
AXON_API int axon_gemm_resid3(const void* x, const void* r1, const void* r2, const void* w, void* c,
                     void* workspace, int64_t workspace_bytes, int64_t m, int64_t n, int64_t k,
                     int32_t ab_dtype, int32_t c_dtype, float eps, const axon_tune_t* tune,
                     void* stream);

/* qkv_cte (Axon kernels/qkv_cte/kernel.py:18-27; refs.py:23-36):
 * h = x + mlp_prev + attention_prev, y = (h / sqrt(mean(h^2) + 1e-6)) @ w.
 * x, mlp_prev, attention_prev [m, k] and w [k, n] contiguous, bf16 or f16;
 * y [m, n] (c_dtype). tune->variant 0 (default): one kernel
 * (axon_gemm_resid3, the other tune fields as there); 1 / 2: a row pass
 * writes h (input dtype) and the per-row scale into the workspace and the
 * GEMM (its variant 1 / 2) applies the scale in its epilogue. k a multiple
 * of 8. workspace: axon_qkv_cte_workspace_bytes(m, n, k, tune) bytes,
 * 16-byte aligned (may be 0 for variant 0). */
AXON_API int64_t axon_qkv_cte_workspace_bytes(int64_t m, int64_t n, int64_t k, const axon_tune_t* tune);
AXON_API int axon_qkv_cte(const void* x, const void* mlp_prev, const void* attention_prev,
                 const void* w, void* y, void* workspace, int64_t workspace_bytes, int64_t m,
                 int64_t n, int64_t k, int32_t ab_dtype, int32_t c_dtype,
                 const axon_tune_t* tune, void* stream);

/* softmax_mm (Axon kernels/softmax_mm/kernel.py:7-11; refs.py:16-19):
 * y = (exp(x) / sum(exp(x))) @ w, a bare exponential as in the spec.
 * x [m, k], w [k, n] contiguous bf16 or f16; one row pass writes exp(x) in
 * the input dtype and 1 / (its row sum, over the stored values); the GEMM
 * applies that in its epilogue. workspace: axon_softmax_mm_workspace_bytes. */
AXON_API int64_t axon_softmax_mm_workspace_bytes(int64_t m, int64_t k);
AXON_API int axon_softmax_mm(const void* x, const void* w, void* y, void* workspace,
                    int64_t workspace_bytes, int64_t m, int64_t n, int64_t k, int32_t ab_dtype,
                    int32_t c_dtype, const axon_tune_t* tune, void* stream);

/* attention in one kernel, head dim d = 64 or 128: per 128 query rows,
 * S = q @ k_t_j per 128-key block into tensor memory, P = exp(S) (bf16, keys
 * past s zero) written by four softmax warps into a swizzled shared-memory
 * slab with the row sums kept in registers, O += P @ v_j in tensor memory,
 * y = O / l; scores never reach global memory. Key blocks are split over
 * CTAs while the query blocks leave SMs idle (tune->split: splits, 0 = auto;
 * max_ctas caps the grid), the fp32 partials added in order by a second
 * pass. workspace: axon_attention_fused_workspace_bytes (0 without splits). */
AXON_API int64_t axon_attention_fused_workspace_bytes(int64_t s, int64_t d, const axon_tune_t* tune);
AXON_API int axon_attention_fused(const void* q, const void* k_t, const void* v, void* y, void* workspace,
                         int64_t workspace_bytes, int64_t s, int64_t d, int32_t ab_dtype,
                         int32_t c_dtype, const axon_tune_t* tune, void* stream);

/* attention_nkilib (Axon kernels/attention_nkilib/kernel.py:14-21; refs.py:36-47):
 * y = softmax(q @ k_t) @ v with a bare exponential, q [s, d], k_t [d, s]
 * (pre-transposed), v [s, d], contiguous bf16 or f16; y [s, d] (c_dtype).
 * tune->variant 0 (default): axon_attention_fused for d = 64 or 128; variant
 * 1 (and other d): the first GEMM stores e = exp(q @ k_t) [s, s] in the
 * input dtype with per-tile row sums (axon_gemm_exp, tune->block_n), a small
 * pass forms 1 / row sum, and the second GEMM applies it: y = r * (e @ v).
 * s and d multiples of 8. workspace: axon_attention_workspace_bytes(s, d, tune). */
AXON_API int64_t axon_attention_workspace_bytes(int64_t s, int64_t d, const axon_tune_t* tune);
AXON_API int axon_attention(const void* q, const void* k_t, const void* v, void* y, void* workspace,
                   int64_t workspace_bytes, int64_t s, int64_t d, int32_t ab_dtype,
                   int32_t c_dtype, const axon_tune_t* tune, void* stream);

/* Bytes of scratch axon_silu_mlp needs: the [m, n] activation in ab_dtype
 * times tune->precision terms, or for precision 4 and 5 an f16 activation,
 * room for an f16 copy of w3 ([n, p]) and the fused kernel's counters. */
AXON_API int64_t axon_silu_mlp_workspace_bytes(int64_t m, int64_t n, int64_t p, int32_t ab_dtype,
                                               const axon_tune_t* tune);

/* (silu(x @ w1) * (x @ w2)) @ w3 (Axon kernels/silu_mlp/refs.py:16-21):
 * x [m, k], w1/w2 [k, n], w3 [n, p], y [m, p] of c_dtype. Two tcgen05 GEMMs:
 * gate and up in one pass with the SiLU-gate epilogue writing the activation
 * into `workspace`, then the down projection. tune->precision selects how the
 * activation a is stored:
 *   1 (default)  one ab_dtype value;
 *   2, 3         T split terms (a ~ t0 + t1 + ..., each rounded to ab_dtype,
 *                8 more mantissa bits per term); the down projection
 *                contracts over K = T*n reading w3 once per term (n % 64 == 0);
 *   4            f16 (ab_dtype bf16 only): the call converts w3 to an f16 copy
 *                in the workspace and runs the down projection f16 x f16
 *                (both MMA operands must share a type); 3 more mantissa bits
 *                than bf16 for ~3% extra traffic, finite only while |a| < 65504;
 *   5            as 4, with w3 passed as an f16 [n, p] matrix: the caller's
 *                f16 copy of W_down, converted once when the weights are
 *                loaded, so no call converts it again.
 * An fp32 reference at 1e-2 needs precision >= 2 (or 4) at the SwiGLU config
 * and 3 for N(0, 1) weights. In the column/row tensor-parallel form each rank
 * passes its shard (n = inter / G) and sums the fp32 partial outputs.
 * tune->variant at precision 4 and 5: 1 / 2 = two launches of the one-CTA / CTA-pair
 * GEMM, 3 = both GEMMs in one CTA-pair kernel (m >= 256), 0 (default) = 3
 * while the gate/up GEMM has fewer than 320 256 x 128 tiles, else 2. Other
 * precisions run two launches (variant as axon_gemm's). */
AXON_API int axon_silu_mlp(const void* x, const void* w1, const void* w2, const void* w3,
                  void* y, void* workspace, int64_t workspace_bytes, int64_t m,
                  int64_t n, int64_t k, int64_t p, int32_t ab_dtype, int32_t c_dtype,
                  const axon_tune_t* tune, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AXON_B200_H */
