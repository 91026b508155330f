/*
 * mli_gemv.h -- C ABI of the B200 (sm_100a) INT8 group-64 linear library
 * (libmli_gemv.so).
 *
 * Every pointer is a caller-owned DEVICE pointer unless stated otherwise, and
 * no compute entry point allocates or frees memory (the setup calls
 * mli_peer_alloc and mli_chain_create do, and say so).  Layouts are the ones the
 * MiniLlama-Infra weight file and forward pass use (scripts/quantize_int8_group.py:67-71,
 * src/main_cuda.cpp:364-393, src/model_cuda_v2_shared.cu:384-412):
 *
 *   w_q  int8  [d][n]       row-major, one output row per row
 *   w_s  fp32  [d][n / gs]  one scale per (row, group of gs columns)
 *   x    fp32  [n]          activation (batch 1)     or [m][n] token-major
 *   y    fp32  [d]          output                   or [m][d] token-major
 *
 * n = in-features (the reference's `n`), d = out-features (`d`), gs = group
 * size (the reference's `group_size`; 64 everywhere in MiniLlama-Infra).
 *
 * Streams: `stream` is a cudaStream_t passed as void*; NULL is the legacy
 * default stream, which the reference's <<<>>> launches use.
 *
 * Errors: every entry point returns MLI_OK (0) or an MLI_ERR_* code; a CUDA
 * launch error is returned as MLI_ERR_CUDA and its cudaError_t is kept for
 * mli_last_cuda_error().  The reference launchers (src/model_cuda_v2_shared.cu)
 * return void and check nothing; the drop-in shim below keeps that signature
 * and records the status for mli_last_status().
 */
#ifndef MLI_GEMV_H
#define MLI_GEMV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum mli_status_code {
  MLI_OK = 0,
  MLI_ERR_INVALID_ARG = 1, /* null pointer, non-positive size, bad count     */
  MLI_ERR_UNSUPPORTED = 2, /* shape outside every kernel's limits            */
  MLI_ERR_CUDA = 3,        /* a CUDA runtime call or launch failed           */
  MLI_ERR_DEVICE = 4       /* a kernel gave up on a bounded wait (see below) */
};

/* Launch-option bits for mli_set_launch_flags(). */
#define MLI_LAUNCH_PDL 1u /* programmatic dependent launch (default on) */
/* Batch-1 GEMV tuning: by default a matrix of at least two ring stages per SM
 * runs two CTAs per SM; with this bit only matrices of 16+ stages per SM do,
 * the others leave the second slot to the next kernel in the stream. */
#define MLI_LAUNCH_ONE_CTA 2u
/* Batched W8A8 (tensor cores): by default the K splits of an output tile run
 * as one thread-block cluster and sum their partials over shared memory; with
 * this bit a split-K launch given a workspace sums them there instead (partial
 * sums in the workspace and a second kernel), and one without a workspace does
 * not split K. */
#define MLI_LAUNCH_NO_CLUSTER 4u
/* Batched W8A8 with more than 64 tokens: by default a problem of enough
 * 128 x 128 output tiles to keep the SMs evenly busy (at least one per SM,
 * the busiest SM at most 1.3 x the ideal share) runs as a persistent kernel,
 * one CTA per SM walking whole tiles (no K split); with this bit it takes the
 * split-K kernels. */
#define MLI_LAUNCH_NO_PERSISTENT 8u

/* ---- library state ------------------------------------------------------ */
const char* mli_status_string(int status);
int mli_last_status(void);            /* status of the last call on this thread */
int mli_last_cuda_error(void);        /* cudaError_t behind the last MLI_ERR_CUDA */
int mli_version(void);                /* MAJOR*10000 + MINOR*100 + PATCH */
unsigned mli_get_launch_flags(void);
void mli_set_launch_flags(unsigned flags);
/* Reads and clears the device error word of the current device: 0 when no
 * kernel gave up on a bounded wait since the last call; otherwise the first
 * code recorded: 1 a weight stage never landed in shared memory, 2 the
 * tensor-core pipeline stalled, 3 a rank's rows of a row-sharded layer never
 * arrived, 4 a chained GEMV's inputs were never completed, 5 the batched
 * tensor-core GEMM met a finite group scale of 2^38 or more (its outputs are
 * not written). */
int mli_device_error(unsigned* code_out);

/* ---- batch-1 linear ops (the reference's matmul launchers) ------------- */

/* y = W x with W = w_q * w_s (dequantised per group), fp32 activations.
 * Replaces matmul_int8 (include/model.h:62; src/model_cuda_v2_shared.cu:36-69).
 * fp32 result within max|y - y_ref| / max|y_ref| <= 1e-5 of the reference. */
int mli_gemv_w8a32(float* y, const float* x, const int8_t* w_q,
                   const float* w_s, int n, int d, int group_size,
                   void* stream);

/* Per-token dynamic activation quantisation, bit-identical to the reference:
 * xs[0] = max(max|x| / 127, 1e-8); xq = clamp(rint(x * (1 / xs[0])), +-127).
 * Replaces quantize_activation (include/model.h:64;
 * src/model_cuda_v2_shared.cu:429-460). */
int mli_quantize_activation(int8_t* xq, float* xs, const float* x, int n,
                            void* stream);

/* W8A8: y[r] = sum_g ((float)I[r][g] * w_s[r][g]) * xs[0], with I the exact
 * int32 dot of group g of row r and xq.  Replaces matmul_dp4a
 * (include/model.h:63; src/model_cuda_v2_shared.cu:462-509). */
int mli_gemv_w8a8(float* y, const int8_t* xq, const float* xs,
                  const int8_t* w_q, const float* w_s, int n, int d,
                  int group_size, void* stream);

/* W8A8 with the activation quantiser fused in as a prologue: every CTA
 * quantises x itself, so one launch replaces the reference's pair
 * quantize_activation + matmul_dp4a (src/model_cuda_v2_shared.cu:529-530).
 * xq_out / xs_out may be NULL; when given they receive the same bytes
 * mli_quantize_activation writes. */
int mli_gemv_w8a8_fused(float* y, int8_t* xq_out, float* xs_out,
                        const float* x, const int8_t* w_q, const float* w_s,
                        int n, int d, int group_size, void* stream);

/* fp32 GEMV y = W x, W fp32 [d][n] row-major.  Replaces the reference's
 * matmul (include/model.h:61; src/model_cuda_v2_shared.cu:10-25), which its
 * forward passes use for the tied-embedding classifier (:418, :564): one warp
 * per row with 512-byte coalesced loads instead of one thread per row.
 * Within max|y - y_ref| / max|y_ref| <= 1e-5 of the reference (a different
 * summation order). */
int mli_gemv_f32(float* y, const float* x, const float* w, int n, int d, void* stream);

/* ---- chained decode step (no reference counterpart) -------------------- */

/* Row epilogues of a chained GEMV.  ADD adds each row into y (the residual add
 * after the reference's down projection, src/model_cuda_v2_shared.cu:215-218,
 * :414).  SWIGLU pairs the op with the NEXT op of the chain (gate = this op,
 * up = the next: same n, d, activation and wait, epilogue STORE, its y unused)
 * and stores (g * (1 / (1 + expf(-g)))) * u into this op's y -- the
 * reference's silu_mul (:220-227, :410) fused in; both ops count as complete
 * together.  A SwiGLU pair streams the gate's and the up's rows of a stage
 * together, so one launch reads both matrices once. */
#define MLI_EPI_STORE 0
#define MLI_EPI_ADD 1
#define MLI_EPI_SWIGLU 2

/* One GEMV of a chain: the arguments of mli_gemv_w8a32 (form 0),
 * mli_gemv_w8a8 (form 1) or mli_gemv_w8a8_fused without xq_out/xs_out
 * (form 2), plus `wait`: ops [0, wait) of the chain are complete before this
 * op reads its activation or writes its output (0 <= wait <= own index).  A
 * decode layer q, k, v, o, gate, up, down at chain index b..b+6 uses waits
 * b, b, b, b+3, b+4, b+4, b+6 (o after the attention of q/k/v, gate/up after
 * o, down after gate/up, the next layer after down).
 *
 * An op whose x is the y of an earlier op of the chain reads that op's rows
 * of this launch (the earlier op must lie in its wait prefix); any other x is
 * read as it is when the launch starts.  An ADD op's y likewise starts from
 * the latest earlier op writing the same y (in its wait prefix), else from
 * y's contents at launch.
 *
 * norm_w (forms 0 and 2, may be NULL): the op's activation is
 * norm_w[i] * (x[i] / sqrt(mean(x^2) + 1e-5)) -- the reference's
 * rmsnorm_cuda (src/model_cuda_v2_shared.cu:74-96), and with an ADD op
 * writing x the fused add + RMSNorm of :99-123 -- computed by every CTA from
 * the whole of x (n <= 8192).  Within fp32 rounding of the reference (its sum
 * of squares runs in another order). */
typedef struct mli_gemv_op {
  int form;       /* 0 W8A32, 1 W8A8 (xq, xs given), 2 W8A8 quantising x */
  int n;          /* in-features: a multiple of 256 */
  int d;          /* out-features */
  int group_size; /* 64 */
  int wait;       /* ops [0, wait) complete first */
  int epilogue;   /* MLI_EPI_*: how the op's rows are stored */
  float* y;
  const float* x;    /* forms 0 and 2 */
  const int8_t* xq;  /* form 1 */
  const float* xs;   /* form 1 */
  const int8_t* w_q;
  const float* w_s;
  const float* norm_w; /* RMSNorm weights [n] of the activation, or NULL */
} mli_gemv_op;

typedef struct mli_chain mli_chain; /* opaque */

/* Plans a chain of `count` GEMVs of one form for the current device: checks
 * every op (MLI_ERR_INVALID_ARG / MLI_ERR_UNSUPPORTED as the single calls
 * would; n % 256 == 0, 16-byte aligned x/xq, w_q, w_s), allocates two small
 * device blocks (the op table, and the mirrors: the rows of every op a later
 * op reads, as 8-byte {value, tag} words) and copies the table with
 * synchronous runtime calls: make it before any stream capture.  The op's
 * pointers are baked in; the buffers they name must outlive the chain. */
int mli_chain_create(const mli_gemv_op* ops, int count, mli_chain** chain);

/* A chain whose GEMVs are row-sharded over `world` ranks (one process per
 * GPU, 1 <= world <= 8; every rank creates the same op list with its own
 * rows): op i computes rows [row_offset[i], row_offset[i] + d) of a GEMV of
 * d_total[i] rows, its y pointing at the first of them.  An op whose x is
 * the whole vector (the buffer at y - row_offset of an earlier op, with
 * n == d_total) reads every rank's rows of it: each rank stores the rows it
 * computes, tagged with the launch, into every rank's mirror over NVLink
 * (plain peer stores), and readers check the tags -- no collective, no fence.
 * Mirrors are kept twice, alternating by launch, so a rank may run one launch
 * ahead of another; every launch must read rows of every rank (an FFN block:
 * down reads all of hb), else a rank two launches ahead would overwrite rows
 * still being read (the reader then times out with device error 4).  Ranks
 * must run their chains the same number of times.  Before the first run:
 * mli_chain_export on every rank, mli_peer_open of the other ranks' handles,
 * mli_chain_set_peers. */
int mli_chain_create_sharded(const mli_gemv_op* ops, const int* row_offset, const int* d_total,
                             int count, int world, mli_chain** chain);
/* The CUDA IPC handle (64 bytes) of the chain's mirror block. */
int mli_chain_export(mli_chain* chain, unsigned char* ipc_handle);
/* Every rank's mirror block in this process (peer_mirrors[r] from
 * mli_peer_open of rank r's handle; the own entry, index `rank`, is ignored). */
int mli_chain_set_peers(mli_chain* chain, void* const* peer_mirrors, int rank);
/* Synchronous: the whole rows (d_total floats) of op `op` from the chain's
 * last run, read from this rank's mirror (every rank's rows of a sharded op);
 * *complete = 1 when every row carries that run's tag.  For ops some later op
 * reads (others have no mirror: MLI_ERR_INVALID_ARG). */
int mli_chain_rows(mli_chain* chain, int op, float* out, int* complete);

/* Runs the whole chain as one cooperative launch (one CTA per SM) on
 * `stream`: every op's y is bit-identical to its single call.  A chain's runs
 * must not overlap on the GPU (they share the mirrors); run it in one stream
 * order.  Must be called with the chain's device current (and, for a sharded
 * chain, after mli_chain_set_peers). */
int mli_chain_run(mli_chain* chain, void* stream);

/* Frees the chain's device block (synchronising like cudaFree). */
int mli_chain_destroy(mli_chain* chain);

/* Test hook: the chain plan on a hypothetical device without touching any
 * GPU.  out[7] = grid, shared bytes per CTA, ring slots, slot bytes, work
 * units (weight stages), activation epochs, phases (runs of ops between
 * growing dependency prefixes). */
int mli_debug_plan_chain(const mli_gemv_op* ops, int count, int sm_count,
                         int smem_optin, int* out);

/* ---- batched decode (m independent tokens, no reference counterpart) -- */

/* Row-wise activation quantisation of m tokens: xs has m entries.  Each row
 * is bit-identical to mli_quantize_activation of that row. */
int mli_quantize_activation_rows(int8_t* xq, float* xs, const float* x, int m,
                                 int n, void* stream);

/* Y[t][r] = xs[t] * sum_g w_s[r][g] * I[t][r][g] for m tokens (Y [m][d]).
 * m >= 16 with n % 128 == 0 runs on the tcgen05 kind::i8 tensor-core path
 * (tiles of 128 weight rows x up to 128 tokens); smaller m, or other shapes,
 * on the CUDA-core path.  Each token's row is within the W8A8 tolerance of
 * mli_gemv_w8a8 on that token.  The tensor-core path splits K over CTAs to
 * fill the GPU.  The splits of a tile run as one thread-block cluster and
 * sum their partials in split order over shared memory, when clusters of
 * that size fit the GPU in one wave.  Otherwise the library takes the faster
 * (by its estimate) of the largest cluster that fits and, if `workspace`
 * (device, may be NULL; mli_gemm_w8a8_workspace_bytes(m, n, d) bytes, any
 * contents) is given, the full split with its partial sums in the workspace,
 * summed in split order by a second launch on the same stream.  Calls that
 * share a workspace must not overlap on the GPU. */
size_t mli_gemm_w8a8_workspace_bytes(int m, int n, int d);
int mli_gemm_w8a8(float* y, const int8_t* xq, const float* xs,
                  const int8_t* w_q, const float* w_s, int m, int n, int d,
                  int group_size, void* workspace, size_t workspace_bytes,
                  void* stream);
/* Allocation-free variant of mli_gemm_w8a8 (no counterpart in the reference,
 * which has no batched path).  For callers that cannot allocate device memory
 * for a workspace -- a plugin whose host framework owns all device memory
 * through its own pool, or a serving loop that must not allocate on the
 * request path -- the split-K scratch lives in a fixed 12 MiB array inside
 * the library, which every GPU that loads the library holds until the process
 * exits.  Same results as mli_gemm_w8a8 with a large enough workspace.
 * Accepts only the tensor-core shapes (m >= 16, n % 128 == 0, group_size 64,
 * 16-byte aligned xq and w_q) and shapes whose workspace
 * (mli_gemm_w8a8_workspace_bytes) fits 12 MiB -- every shape on a 148-SM
 * B200 -- and returns MLI_ERR_UNSUPPORTED otherwise.  The first call on a
 * device looks up the array's device address (make it before any stream
 * capture).  All calls share the array: calls that overlap on the GPU race,
 * so issue them in one stream order. */
int mli_gemm_w8a8_noalloc(float* y, const int8_t* xq, const float* xs,
                          const int8_t* w_q, const float* w_s, int m, int n,
                          int d, int group_size, void* stream);
/* The CUDA-core batched path alone, any m (for comparisons). */
int mli_gemm_w8a8_cuda_core(float* y, const int8_t* xq, const float* xs,
                            const int8_t* w_q, const float* w_s, int m, int n,
                            int d, int group_size, void* stream);
/* Several independent batched W8A8 GEMMs with the same token count m in one
 * launch (no reference counterpart): op i computes y = W_i x_i as
 * mli_gemm_w8a8 would (within the W8A8 tolerance; K is split differently, so
 * not bit for bit), deterministic from call to call.  One launch instead of
 * one per matrix: no launch gaps between the matrices, and the small ones
 * share the GPU with the large ones.  1 <= count <= MLI_GEMM_GROUP_MAX,
 * m >= 16, group_size 64, every n % 128 == 0, xq and w_q 16-byte aligned
 * (MLI_ERR_UNSUPPORTED otherwise); no workspace; outputs must not overlap
 * any op's inputs or another op's output.  `ops` is a HOST array. */
#define MLI_GEMM_GROUP_MAX 8
typedef struct mli_gemm_op {
  float* y;            /* [m][d] */
  const int8_t* xq;    /* [m][n] */
  const float* xs;     /* [m] */
  const int8_t* w_q;   /* [d][n] */
  const float* w_s;    /* [d][n / 64] */
  int n, d;
} mli_gemm_op;
int mli_gemm_w8a8_group(const mli_gemm_op* ops, int count, int m, int group_size, void* stream);
/* Tensor-core plan of mli_gemm_w8a8 on the current device (queries it; no
 * launch).  out[5] = tokens per tile, output tiles, K splits, cluster size
 * (1: none), 1 when the splits sum through the workspace.  Returns
 * MLI_ERR_UNSUPPORTED for shapes outside the tensor-core path. */
int mli_debug_plan_gemm(int m, int n, int d, size_t workspace_bytes, int* out);
/* Persistent plan of mli_gemm_w8a8_group (and, with count 1, of
 * mli_gemm_w8a8) on the current device (no launch).  out[5] = 1 when the
 * persistent kernel runs the call, CTAs, output tiles, the busiest CTA's
 * cost and the total cost (a tile costs its K chunks of 128 plus one).  The
 * pointers of `ops` are looked at, not dereferenced. */
int mli_debug_plan_gemm_group(const mli_gemm_op* ops, int count, int m, int* out);

/* Diagnostic: `ctas` CTAs each issue `iters` x 4 back-to-back tcgen05
 * kind::i8 MMAs (M = 128, N = n in {64, 128, 256}, K = 32; 2 * 128 * n * 32
 * integer ops each) on operands resident in shared memory, from one thread,
 * with no loads and no epilogue: timed by the caller, it gives this GPU's
 * int8 tensor-core roof for the batched path's utilisation.  No reference
 * counterpart. */
int mli_debug_int8_mma_peak(int n, int iters, int ctas, void* stream);

/* ---- row-sharded linear layer across GPUs (one process per GPU) --------- */

/* Peer buffers: device memory this process allocates and exports through a
 * CUDA IPC handle (64 bytes), and opens from the other ranks' handles.  These
 * set-up calls allocate; the step calls below do not.  The buffer is zeroed. */
int mli_peer_alloc(size_t bytes, void** ptr, unsigned char* ipc_handle);
int mli_peer_open(const unsigned char* ipc_handle, void** ptr);
int mli_peer_close(void* ptr);
int mli_peer_free(void* ptr);

/* One rank's share of a row-sharded GEMV fused with the all-gather of its
 * output (no reference counterpart: the reference runs its classifier,
 * src/model_cuda_v2_shared.cu:418 / :564, on one GPU).  Rows
 * [row_offset, row_offset + rows) of the d_total-row layer are computed from
 * this rank's weight shard and stored over NVLink into every rank's logits
 * words peer_logits[p] ([2][d_total]; the half is *step & 1), each row as one
 * 8-byte word {fp32 value, tag of the step}; every CTA also stores its rows'
 * (max, first index) as one tagged partial word into every rank's block.  No
 * fence and no counter: a reader knows a word has arrived by its tag.
 * peer_logits is a HOST array of `world` device pointers (offset 256 of
 * every rank's peer block; this rank's own at index `rank`).  form: 0 W8A32,
 * 2 fused W8A8.  d_total < 2^20. */
int mli_gemv_rowshard(int form, unsigned long long* const* peer_logits, const unsigned* step,
                      const float* x, const int8_t* w_q, const float* w_s, int n, int rows,
                      int row_offset, int d_total, int rank, int world, int group_size,
                      void* stream);

/* mli_gemv_rowshard and mli_rowshard_wait_argmax in one launch: the CTAs
 * store their tagged rows and partial words into every rank's block as
 * above; the launch's last CTA then polls (bounded by timeout_us) every
 * rank's partial words of this step, reduces them to the argmax, writes it to
 * *out and advances the step -- one kernel per step.  own_block is this
 * rank's peer block (its header holds the step and the launch's finished-CTA
 * count); shard_rows is a HOST array of `world` row counts (every rank's
 * `rows`) summing to d_total.  On expiry *out = -1 and the device error word
 * is set. */
int mli_gemv_rowshard_argmax(int form, unsigned long long* const* peer_logits, void* own_block,
                             const float* x, const int8_t* w_q, const float* w_s, int n,
                             int rows, int row_offset, int d_total, int rank, int world,
                             int group_size, const int* shard_rows, long long* out,
                             int timeout_us, void* stream);

/* Bytes of one rank's peer block for a d_total-row layer:
 *   [128, 132) uint32 step counter
 *   [192, 196) uint32 finished-CTA count of a fused step (zero between steps)
 *   [256, ...) logits words uint64 [2][d_total] (low 32 bits the fp32 value,
 *              high 32 bits the step's tag), then (16-byte aligned) the CTAs'
 *              partial words uint64 [2][8][512] (low 32 bits the maximum,
 *              high 32 bits (first index << 12) | tag).
 * The tag of step s is (s mod 4095) + 1; a zeroed block matches no step. */
size_t mli_rowshard_block_bytes(int d_total);

/* Completes a row-sharded step on this rank: polls (bounded by timeout_us;
 * on expiry *out = -1 and the device error word is set) every rank's partial
 * words of step *step in this rank's block until their tags arrive, reduces
 * them to the first maximum of the full logits (the reference's host argmax
 * rule), writes its index to *out and increments *step.  form and n are the
 * GEMV's (they fix each rank's CTA count); logits points at offset 256 of
 * this rank's block; shard_rows is a HOST array of `world` row counts summing
 * to d_total. */
int mli_rowshard_wait_argmax(int form, int n, const unsigned long long* logits, unsigned* step,
                             const int* shard_rows, int world, int d_total, long long* out,
                             int timeout_us, void* stream);

/* Index of the first maximum of x[0..n), on the device (replaces the
 * reference's logits copy to the host and host argmax, src/main_cuda.cpp:96-98,
 * src/model_cuda_v2_shared.cu:571-575).  NaN never wins; -0.0 equals +0.0. */
int mli_argmax(const float* x, int n, long long* out, void* stream);

/* ---- offline weight preparation ---------------------------------------- */

/* Group-wise weight quantisation, bit-identical to
 * scripts/quantize_int8_group.py:55-71: scale = max(amax, 1e-9) / 127 per
 * (row, group), q = clip(round_half_even(w / scale), +-127). */
int mli_quantize_weights(int8_t* w_q, float* w_s, const float* w, int rows,
                         int cols, int group_size, void* stream);

/* ---- diagnostics --------------------------------------------------------- */

/* Exact int32 group dot products I[r][g] (d x n/gs), the values the W8A8
 * kernels scale; for bit-exact parity tests. */
int mli_debug_group_dots(int32_t* out, const int8_t* xq, const int8_t* w_q,
                         int n, int d, int group_size, void* stream);

/* Host-only: the launch plan the batch-1 streaming GEMV would use for this
 * shape on a device with the given properties.  form: 0 W8A32, 1 W8A8,
 * 2 fused W8A8.  out[8] = {grid, dynamic smem bytes, slices per row, warps
 * per slice, rows per stage, stages, ring slots, bytes per stage}.  Returns
 * MLI_ERR_UNSUPPORTED for shapes that take the generic kernels. */
int mli_debug_plan_gemv(int form, int n, int d, int sm_count, int smem_per_sm,
                        int smem_optin, int* out);

#ifdef __cplusplus
} /* extern "C" */

/* ---- drop-in shim (libmli_dropin.so, C++ linkage) --------------------------
 * Exactly the reference's launch signatures (include/model.h:61-64), so the
 * reference's forward_cuda / forward_cuda_dp4a (src/model_cuda_v2_shared.cu:370-421,
 * 514-566) link against this library unchanged once the reference's own
 * definitions of these three functions are removed.  They launch on the legacy
 * default stream like the reference and store their status for
 * mli_last_status(). */
void matmul_int8(float* xout, float* x, int8_t* w_q, float* w_s, int n, int d,
                 int group_size);
void matmul_dp4a(float* xout, const int8_t* x_q, const float* x_s,
                 const int8_t* w_q, const float* w_s, int n, int d,
                 int group_size);
void quantize_activation(int8_t* xq, float* xs, const float* x, int n);
/* The fp32 launcher of include/model.h:61 (the classifier's), optional for a
 * maintainer: remove it from the shim's link to keep the reference's own. */
void matmul(float* xout, float* x, float* w, int n, int d);
#endif /* __cplusplus */

#endif /* MLI_GEMV_H */
