/*
 * nnue_ft.h -- C ABI of the B200 (sm_100a) sparse NNUE feature transformer.
 *
 * Drop-in boundary for the one hot path of rgodha24/stockfish-trainer: the
 * feature transformer behind SparseLinearFunction
 * (src/model/modules/feature_transformer/functions.py:10-72) and its kernel
 * factories (src/model/modules/feature_transformer/kernel.py:301-319).
 *
 * Conventions
 *   - All tensors are dense, row-major, caller-owned DEVICE memory on the
 *     current CUDA device; nothing here allocates device memory.  Scratch for
 *     the backward comes from a caller workspace sized by
 *     nnue_ft_backward_workspace_size().
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Calls only
 *     enqueue work; none synchronises the host, so every call can be captured
 *     in a CUDA graph.
 *   - Feature indices are int32, -1 = empty slot, anywhere in the row.  An
 *     index < -1 or >= num_inputs is skipped (never dereferenced) and raises a
 *     sticky device flag read by nnue_ft_device_errors().
 *   - Return value: NNUE_OK or a negative NNUE_ERR_* code; no exceptions
 *     cross this boundary.  nnue_ft_last_error() describes the last failure
 *     on the calling thread.
 *   - Floating point: fp32 only.  The forward and the weight gradient add in
 *     the reference's order (ascending k per position; ascending position per
 *     feature), so both are bit-identical to the reference kernels.
 *   - Process-wide state (one per process, shared by every caller, thread and
 *     stream):
 *       * tuning (nnue_ft_set_param): a change applies to every later call in
 *         the process; change it only while no call of this library is
 *         running or being enqueued;
 *       * one side stream per device, with one fork/join event pair: the
 *         backward's heavy rows and bias sum run there beside the caller's
 *         stream.  Calls from several streams stay correct but serialise
 *         their side-stream work, and a join may wait for another stream's
 *         side work too;
 *       * the kernel timer and the sticky device error word.
 *     The library keeps device-side objects (streams, events) per device for
 *     the life of the process: do not call it across cudaDeviceReset.
 */
#ifndef NNUE_FT_H
#define NNUE_FT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NNUE_OK 0
#define NNUE_ERR_INVALID_ARGUMENT (-1)   /* null pointer, bad shape, misaligned */
#define NNUE_ERR_UNSUPPORTED (-2)        /* sizes beyond the documented limits */
#define NNUE_ERR_WORKSPACE (-3)          /* workspace null or too small */
#define NNUE_ERR_CUDA (-4)               /* a CUDA launch or runtime call failed */

/* Device error flags (nnue_ft_device_errors). */
#define NNUE_DEVERR_BAD_INDEX 1u         /* index < -1 or >= num_inputs was skipped */
#define NNUE_DEVERR_BAD_QUANT_INDEX 2u   /* quantised forward: index outside the table */
#define NNUE_DEVERR_BAD_SEGMENT 4u       /* backward: corrupt workspace (position out of range) */
#define NNUE_DEVERR_BAD_PSQT_INDEX 8u    /* epilogue: PSQT bucket index outside [0, n_psqt) was skipped */
#define NNUE_DEVERR_BAD_POSITION 16u     /* device encoder: a rejected position got all -1 rows */
#define NNUE_DEVERR_EXCHANGE_TIMEOUT 32u /* exchange: a rank did not reach the barrier in time */

/* ABI version (major * 100 + minor). */
int nnue_ft_version(void);

/* Number of CUDA kernels this library has launched in this process (all
 * devices, all threads); lets a caller count launches inside a region. */
uint64_t nnue_ft_launch_count(void);

/* Per-launch timing of the gather kernels (measurement support; no
 * reference counterpart).  Arms the kernel classes in the bit mask `kernels`
 * (1: forward gather kernel, 2: light-row segment-sum kernel, 4: heavy-row
 * segment-sum kernel) for up to `capacity` timed launches in total on the
 * current device: each launch of an armed class is bracketed by a CUDA event
 * pair recorded on the stream it is launched on, so its duration includes
 * whatever runs concurrently on other streams.  kernels == 0 disarms and
 * frees the events.  Not for use under stream capture. */
int nnue_ft_kernel_timer_arm(uint32_t kernels, int32_t capacity);

/* Waits for the timed launches of class `kernel` (0 forward, 1 light rows,
 * 2 heavy rows) and writes up to `max` durations in milliseconds, in launch
 * order; *count receives the number of timed launches of that class. */
int nnue_ft_kernel_timer_read(int32_t kernel, float *ms, int32_t max, int32_t *count);

/* Message for the last failing call on this thread ("" if none). */
const char *nnue_ft_last_error(void);

/* Reads (and with clear != 0 resets) the sticky device error flags of the
 * current device.  Synchronises the device: a debugging aid, not for the
 * hot loop. */
int nnue_ft_device_errors(uint32_t *flags, int clear);

/* Tuning knobs (names: "fwd_chunk_vec", "fwd_items_per_warp", "fwd_unroll",
 * "fwd_min_blocks", "fwd_exact_chunks", "fwd_block", "fwd_groups",
 * "fwd_queue_blocks", "bwd_chunk_vec", "bwd_unroll", "bwd_min_blocks",
 * "bwd_exact_chunks", "bwd_block", "bwd_queue", "bwd_queue_min_blocks",
 * "bwd_queue_min_entries", "fwd_tail", "bwd_tail",
 * "heavy_threshold", "heavy_cap", "sort_blocks_per_sm", "colsum_parts");
 * their meanings and defaults are beside struct Tuning in
 * stockfish_trainer_b200/csrc/nnue_ft.cu.  Unknown names and out-of-range
 * values are rejected with
 * NNUE_ERR_INVALID_ARGUMENT.  Every setting gives the same results.
 * Process-wide; change them only while no call is in flight and never between
 * a backward_prepare and its backward_apply. */
int nnue_ft_set_param(const char *name, int64_t value);
int64_t nnue_ft_get_param(const char *name);

/* ---- forward ------------------------------------------------------------
 * Replaces the TileLang forward kernel (kernel.py:66-105) as called from
 * SparseLinearFunction.forward (functions.py:12-48) and the factory
 * make_sparse_input_linear_forward_kernel(max_active, output_size)(idx,
 * weight, bias, output) (kernel.py:301-312):
 *   output[b, c] = bias[c] + sum_{k ascending, idx[b,k] != -1} weight[idx[b,k], c]
 * idx: [batch, max_active] int32; weight: [num_inputs, output_size] fp32;
 * bias: [output_size]; output: [batch, output_size] (written). */
int nnue_ft_forward(const int32_t *idx, int64_t batch, int32_t max_active, const float *weight,
                    int64_t num_inputs, int32_t output_size, const float *bias, float *output,
                    void *stream);

/* Both perspectives in one launch (the two calls of
 * ComposedFeatureTransformer.forward, src/model/modules/features/composed.py:49-54). */
int nnue_ft_forward_pair(const int32_t *idx0, const int32_t *idx1, int64_t batch, int32_t max_active,
                         const float *weight, int64_t num_inputs, int32_t output_size, const float *bias,
                         float *out0, float *out1, void *stream);

/* ---- backward -----------------------------------------------------------
 * Replaces _build_sorted_backward_inputs (kernel.py:108-138), the bias
 * column sum (kernel.py:269) and the TileLang backward kernel
 * (kernel.py:141-188), as reached from SparseLinearFunction.backward
 * (functions.py:50-72) or make_sparse_input_linear_backward_kernel
 * (kernel.py:315-319).
 *
 * n_persp = 1 (idx1/grad1 unused) or 2.  For every feature row f:
 *   sum(f) = sum over perspectives q of ( sum_{b ascending, f in idx_q[b]} grad_q[b] )
 *   accumulate == 0: weight_grad[f] = sum(f) for EVERY row (untouched rows
 *                    get 0, so weight_grad may be uninitialised memory);
 *                    bias_grad = column sums.
 *   accumulate != 0: weight_grad[f] += sum(f) for touched rows only, exactly
 *                    the reference kernel's update; bias_grad += column sums.
 * The backward is deterministic: same inputs, same bits. */
size_t nnue_ft_backward_workspace_size(int64_t batch, int32_t max_active, int64_t num_inputs,
                                       int32_t output_size, int32_t n_persp);

int nnue_ft_backward(const int32_t *idx0, const int32_t *idx1, int64_t batch, int32_t max_active,
                     const float *grad0, const float *grad1, int32_t n_persp, int64_t num_inputs,
                     int32_t output_size, float *weight_grad, float *bias_grad, int32_t accumulate,
                     void *workspace, size_t workspace_bytes, void *stream);

/* The two phases of nnue_ft_backward.  prepare depends only on the indices
 * (sorted position lists per feature, in the workspace); apply consumes the
 * gradients.  Same sizes and workspace for both; prepare may run as soon as
 * the indices are known (e.g. right after the forward). */
int nnue_ft_backward_prepare(const int32_t *idx0, const int32_t *idx1, int64_t batch, int32_t max_active,
                             int32_t n_persp, int64_t num_inputs, int32_t output_size, void *workspace,
                             size_t workspace_bytes, void *stream);
int nnue_ft_backward_apply(const float *grad0, const float *grad1, int64_t batch, int32_t max_active,
                           int32_t n_persp, int64_t num_inputs, int32_t output_size, float *weight_grad,
                           float *bias_grad, int32_t accumulate, void *workspace, size_t workspace_bytes,
                           void *stream);

/* nnue_ft_backward_apply restricted to weight-gradient rows [row_begin,
 * row_end); the bias gradient is produced only when with_bias != 0 (bias_grad
 * may then be null otherwise).  Lets a data-parallel caller start reducing
 * finished rows while later rows are still being computed. */
int nnue_ft_backward_apply_rows(const float *grad0, const float *grad1, int64_t batch, int32_t max_active,
                                int32_t n_persp, int64_t num_inputs, int32_t output_size, float *weight_grad,
                                float *bias_grad, int32_t accumulate, int64_t row_begin, int64_t row_end,
                                int32_t with_bias, void *workspace, size_t workspace_bytes, void *stream);

/* Forward of both perspectives (nnue_ft_forward_pair) plus, concurrently on
 * the library's side stream, the index-only backward phase
 * (nnue_ft_backward_prepare with n_persp = 2) into `workspace`.  The caller's
 * stream waits for both before its next operation; the backward then needs
 * only nnue_ft_backward_apply with the same sizes and workspace. */
int nnue_ft_forward_pair_prepare(const int32_t *idx0, const int32_t *idx1, int64_t batch, int32_t max_active,
                                 const float *weight, int64_t num_inputs, int32_t output_size, const float *bias,
                                 float *out0, float *out1, void *workspace, size_t workspace_bytes, void *stream);

/* Backward for callers that cannot allocate device memory: the same result
 * as nnue_ft_backward (same arguments minus the workspace), with its scratch
 * taken from a fixed 16 MiB device array inside this library instead of a
 * caller workspace.  It has no counterpart in the reference.
 *   - Who needs it: code that must not call cudaMalloc or an allocator per
 *     call, e.g. a search / inference loop on a fixed memory budget, or a
 *     host that reaches the GPU only through this C ABI with tensors owned by
 *     someone else and no way to provide a workspace.
 *   - Limit: sizes whose nnue_ft_backward_workspace_size() exceeds
 *     nnue_ft_noalloc_scratch_bytes() are rejected with NNUE_ERR_UNSUPPORTED.
 *     With the default tuning that is about 9K HalfKAv2_hm positions, or
 *     about 1.2K Full_Threats+HalfKAv2_hm positions, at C = 1048; tuning set
 *     through nnue_ft_set_param (heavy_cap, colsum_parts) changes the
 *     workspace size, so check
 *     nnue_ft_backward_workspace_size() <= nnue_ft_noalloc_scratch_bytes()
 *     for your shapes rather than rely on those counts, and do not change
 *     tuning while a call may still be running.
 *   - The array exists on every GPU that loads the library until the process
 *     exits.  Every call looks up its device address on the current device;
 *     the first call on each device also loads the library's kernels there
 *     and, like nnue_ft_backward, creates the library's side stream, so make
 *     that first call before any stream capture.
 *   - All calls share the one array and it keeps the previous call's
 *     contents (everything that must start at zero is cleared by each call).
 *     Calls that overlap on the GPU (different streams, or other threads)
 *     race on it: serialise them. */
int nnue_ft_backward_noalloc(const int32_t *idx0, const int32_t *idx1, int64_t batch, int32_t max_active,
                             const float *grad0, const float *grad1, int32_t n_persp, int64_t num_inputs,
                             int32_t output_size, float *weight_grad, float *bias_grad, int32_t accumulate,
                             void *stream);
/* Size of that fixed scratch array, in bytes. */
size_t nnue_ft_noalloc_scratch_bytes(void);

/* ---- quantised (int16) forward ------------------------------------------
 * The inference forward of a serialised net (the engine's accumulator
 * refresh; the engine is not part of the reference):
 *   acc[b, :]  = bias_q + sum weight_q[row(idx[b,k]), :]   int16, wrapping
 *   psqt[b, :] =          sum psqt_q[row(idx[b,k]), :]     int32, wrapping
 * row(i) = i (export-space indices) or, with map_training != 0, the HalfKA
 * training -> export row map of halfka_v2_hm.py:100-134.
 * weight_q: [table_rows, l1] int16 (l1 % 8 == 0); psqt_q: [table_rows, n_psqt]
 * int32 (n_psqt % 4 == 0); all pointers 16-byte aligned. */
int nnue_ft_quantized_forward_pair(const int32_t *idx0, const int32_t *idx1, int32_t n_persp, int64_t batch,
                                   int32_t max_active, const int16_t *weight_q, const int32_t *psqt_q,
                                   int64_t table_rows, int32_t l1, int32_t n_psqt, const int16_t *bias_q,
                                   int32_t map_training, int16_t *acc0, int16_t *acc1, int32_t *psqt0,
                                   int32_t *psqt1, void *stream);

/* HalfKAv2_hm export + FT quantisation (halfka_v2_hm.py:100-134,
 * quantize.py:83-89): weight [24576, l1 + n_psqt] fp32, virtual [768, same]
 * (nullable) -> weight_q [22528, l1] int16 (x * w_scale, half to even),
 * psqt_q [22528, n_psqt] int32 (x * psqt_scale). */
int nnue_ft_halfka_export_quantize(const float *weight, const float *virtual_weight, int32_t l1, int32_t n_psqt,
                                   float w_scale, float psqt_scale, int16_t *weight_q, int32_t *psqt_q,
                                   void *stream);

/* Elementwise fp32 -> int16 quantisation, round half to even (bias path of
 * quantize.py:83). */
int nnue_ft_quantize_i16(const float *x, int64_t n, float scale, int16_t *q, void *stream);

/* ---- composed feature sets: tables in separate allocations ---------------
 * Replaces ComposedFeatureTransformer.forward's
 *   merged = torch.cat([f.merged_weight() for f in self.features], dim=0)
 * (src/model/modules/features/composed.py:49-54) followed by the two
 * SparseLinearFunction calls, and the backward's split of the merged
 * gradient into the per-feature parameters: global row f of the feature set
 * lives in table t (the first with f < rows[0] + ... + rows[t]) at local row
 * f - (rows[0] + ... + rows[t-1]).  tables / weight_grads are HOST arrays of
 * n_tables (1..4) device pointers, each [rows[t], output_size] fp32.
 * Results equal the merged-table calls bit for bit; no merged copy is made. */
int nnue_ft_forward_pair_tables(const int32_t *idx0, const int32_t *idx1, int64_t batch, int32_t max_active,
                                const float *const *tables, const int64_t *table_rows, int32_t n_tables,
                                int32_t output_size, const float *bias, float *out0, float *out1, void *stream);

/* The same forward with the backward's index phase on the library's side
 * stream (like nnue_ft_forward_pair_prepare; num_inputs = sum of rows). */
int nnue_ft_forward_pair_tables_prepare(const int32_t *idx0, const int32_t *idx1, int64_t batch, int32_t max_active,
                                        const float *const *tables, const int64_t *table_rows, int32_t n_tables,
                                        int32_t output_size, const float *bias, float *out0, float *out1,
                                        void *workspace, size_t workspace_bytes, void *stream);

/* nnue_ft_backward_apply for two perspectives with weight_grads split like
 * the tables: every row of every weight_grads[t] is written (or accumulated
 * into when accumulate != 0, touched rows only). */
int nnue_ft_backward_apply_tables(const float *grad0, const float *grad1, int64_t batch, int32_t max_active,
                                  float *const *weight_grads, const int64_t *table_rows, int32_t n_tables,
                                  int32_t output_size, float *bias_grad, int32_t accumulate, void *workspace,
                                  size_t workspace_bytes, void *stream);

/* HalfKav2Hm.merged_weight (halfka_v2_hm.py:69-70):
 * out[r] = weight[r] + virtual_weight[r % period] for r < rows (rows a
 * multiple of period), one fp32 add per element, without materialising
 * virtual_weight.repeat(rows / period, 1). */
int nnue_ft_merge_virtual(const float *weight, int64_t rows, const float *virtual_weight, int64_t period,
                          int32_t cols, float *out, void *stream);

/* ---- FT epilogue (input transform) ---------------------------------------
 * Replaces the tensor ops of NNUEModel._transform_inputs that follow the FT
 * (src/model/model.py:93-115): split off the PSQT columns, clamp to [0, 1],
 * pairwise product of the two halves, perspective order by `us`, x 127/128,
 * PSQT bucket gather and (w - b) * (us - 0.5).  wp, bp: the FT outputs
 * [batch, l1 + n_psqt] fp32; us: [batch] fp32 (0 or 1; the reference's
 * [batch, 1] tensor); psqt_indices: [batch] int64.  l1 must be even.
 * Forward writes l0 [batch, l1] and psqt [batch]. */
int nnue_ft_epilogue_forward(const float *wp, const float *bp, int64_t batch, int32_t l1, int32_t n_psqt,
                             const float *us, const int64_t *psqt_indices, float *l0, float *psqt, void *stream);

/* Backward of the same graph: the gradients torch autograd produces for it,
 * bit for bit (clamp passes gradient only inside [0, 1], the where / select /
 * gather backward terms are added in autograd's way).  grad_l0 and grad_psqt
 * may be null (zero gradient).  Writes grad_wp and grad_bp [batch, l1 + n_psqt]
 * completely: they are the FT backward's grad_output. */
int nnue_ft_epilogue_backward(const float *wp, const float *bp, int64_t batch, int32_t l1, int32_t n_psqt,
                              const float *us, const int64_t *psqt_indices, const float *grad_l0,
                              const float *grad_psqt, float *grad_wp, float *grad_bp, void *stream);

/* ---- Ranger22 parameter update ------------------------------------------
 * Replaces, for one fp32 parameter, the update of Ranger22.step's fused path
 * (src/ranger22/optimizer.py:48-107 _compiled_full_update_{1d,2d}, eager twin
 * :256-301) and, when lookahead_merge != 0, the lookahead blend of that step
 * (:569-597, torch._foreach_lerp_(p, lookahead, 1 - alpha) then
 * lookahead = p).  One pass: p, variance_ma and gma_cur are updated in place
 * (and lookahead on merge steps); grad and gma_prev are read.
 *   rows x cols: a 2-D parameter takes its norm per row (dim = 1); a 1-D
 *   parameter is passed as rows = 1 (norm over the whole vector).
 *   scalars: 12 host floats in the reference's order (optimizer.py:211-245):
 *   lr, inv_sqrt_bc2, eps, two_nl_factor, noise_norm_recip, pnm_a, pnm_b,
 *   step_size, beta2, 1 - beta2, beta1^2, 1 - beta1^2.
 * All device pointers are contiguous fp32 [rows, cols]; nothing is allocated
 * and nothing synchronises the host. */
int nnue_ft_ranger22_step(float *param, const float *grad, float *variance_ma, float *gma_cur, const float *gma_prev,
                          float *lookahead, int64_t rows, int64_t cols, const float *scalars,
                          int32_t lookahead_merge, float lookahead_alpha, void *stream);

/* Number of Full_Threats inputs implied by the offset table (the reference
 * asserts 60720, feature_extraction.rs:826). */
int nnue_threat_table_total(void);

/* Measurement only (no counterpart in the reference): n_warps warps each sum
 * per_warp random 512-byte rows (32 float4) of `table` ([rows, 128] fp32),
 * 8 row loads in flight per warp, indices idx [n_warps * per_warp] in
 * [0, rows).  The achieved bandwidth versus table size is the ceiling for
 * the FT's gathers.  per_warp % 32 == 0, n_warps % 8 == 0; out: [n_warps, 128]. */
int nnue_ft_gather_probe(const float *table, int64_t rows, const int32_t *idx, int32_t per_warp, int32_t n_warps,
                         float *out, void *stream);

/* ---- host-side synthetic inputs (no GPU needed) --------------------------
 * Seeded random positions: per position an independent splitmix64 stream;
 * kings on distinct uniform squares; U{0..30} other pieces of uniform type
 * (P, N, B, R, Q) and colour on distinct empty squares, pawns on ranks 2-7;
 * uniform side to move.  Positions whose Full_Threats count exceeds 128 in
 * either perspective are redrawn from the same stream.
 * board: [count, 64] piece ids (type * 2 + colour, 12 = empty), stm: [count]. */
int nnue_generate_positions(uint64_t seed, int64_t first, int64_t count, uint8_t *board, uint8_t *stm);

/* Feature indices of the reference's feature functions
 * (src/rust/feature_extraction.rs:213-241, 391-404, 581-739):
 * feature_set 0 = HalfKAv2_hm (K = 32), 1 = Full_Threats (K = 128),
 * 2 = Full_Threats+HalfKAv2_hm (K = 160).  white/black: [count, K] int32,
 * compacted, -1 padded; counts (nullable): [count] each.  Host memory.
 * Returns NNUE_ERR_INVALID_ARGUMENT (the rejected positions' rows all -1)
 * when a position has a side without a king, a pawn on the first or last
 * rank, or more than 128 threat / 32 HalfKA features. */
int nnue_encode_features(const uint8_t *board, int64_t count, int32_t feature_set, int32_t *white,
                         int32_t *black, int32_t *white_count, int32_t *black_count, int32_t nthreads);

/* The same feature indices as nnue_encode_features, computed on the GPU
 * from boards in DEVICE memory (replaces the reference's host-side encoder,
 * src/rust/feature_extraction.rs:213-241 via fill_feature_indices_sparse,
 * for a loader that ships boards -- 64 bytes per position -- instead of
 * index rows of 4 * K bytes per perspective).  board: [count, 64] uint8;
 * white/black: [count, K] int32 (K = 32, 128, 160 for feature_set 0, 1, 2),
 * compacted and -1 padded; counts (nullable): [count] int32.  A position the
 * host encoder rejects (a side without a king, a pawn on the first or last
 * rank, more than 128 threat or 32 HalfKA features) gets all -1 rows and
 * count 0 and raises NNUE_DEVERR_BAD_POSITION.  Async on `stream`, except
 * the first call on a device, which uploads the encoder's lookup tables
 * (13 KB, into a static device array) synchronously. */
int nnue_ft_encode_features(const uint8_t *board, int64_t count, int32_t feature_set, int32_t *white,
                            int32_t *black, int32_t *white_count, int32_t *black_count, void *stream);

/* ---- exchange between the GPUs of one node --------------------------------
 * The multi-GPU plumbing of the column-sharded FT step (no reference
 * counterpart: the reference's DDP allreduces the dense weight gradient,
 * src/train/common.py:186-199; this moves index rows, outputs and output
 * gradients instead).  Each rank allocates one exchange buffer
 * (nnue_ft_exchange_alloc, an exception to "nothing here allocates": a
 * buffer of its own, so its IPC handle maps exactly it), shares the handle
 * with the other ranks of the node (any host channel) and maps theirs
 * (nnue_ft_exchange_open).  The buffer's first NNUE_FT_EXCHANGE_FLAG_BYTES
 * are the rank's flag words (zeroed at allocation); the rest is the
 * caller's. */
#define NNUE_FT_IPC_HANDLE_BYTES 64
#define NNUE_FT_EXCHANGE_FLAG_BYTES 256 /* the flag words at the start of an exchange buffer */

/* cudaMalloc'd + zeroed buffer of `bytes` and its CUDA IPC handle
 * (NNUE_FT_IPC_HANDLE_BYTES bytes).  Synchronous.  Free with
 * nnue_ft_exchange_free. */
int nnue_ft_exchange_alloc(size_t bytes, void **ptr, void *ipc_handle);
int nnue_ft_exchange_free(void *ptr);

/* Maps another process's exchange buffer into this process for the current
 * device (peer access enabled as needed); nnue_ft_exchange_close unmaps. */
int nnue_ft_exchange_open(const void *ipc_handle, void **ptr);
int nnue_ft_exchange_close(void *ptr);

/* One block copy: `rows` rows of `width` 16-byte vectors from src (row stride
 * src_ld vectors) to dst (row stride dst_ld vectors); every float is
 * multiplied by `scale` unless scale == 1 (then the bytes are copied as
 * they are).  src is this GPU's memory; dst this GPU's or a mapped peer's.
 * Both 16-byte aligned. */
typedef struct {
  const void *src;
  void *dst;
  int64_t rows;
  int64_t src_ld, dst_ld;
  int32_t width;
  float scale;
} nnue_ft_copy_desc;

/* Runs up to 32 copies in one launch, then a barrier of the n_ranks (<= 15)
 * ranks on `channel` (0..3; independent barriers, so exchanges on different
 * streams may be in flight together, one channel each): flags[s] = rank s's
 * flag words (its exchange buffer's start, mapped here; flags[rank] = this
 * rank's own).  Every rank calls it on a channel in the same order with the
 * same epoch, which grows by one per call on that channel (the first call
 * after allocation uses 1).  When the launch completes on this rank's
 * stream, every rank's copies of this epoch are done and visible.
 * A rank that does not arrive within timeout_ms raises
 * NNUE_DEVERR_EXCHANGE_TIMEOUT and the launch returns without it (the
 * exchanged data is then incomplete).  Not capturable in a CUDA graph
 * (the epoch is a launch argument).  n_copies == 0: the barrier alone. */
int nnue_ft_exchange(const nnue_ft_copy_desc *copies, int32_t n_copies, uint32_t *const *flags, int32_t n_ranks,
                     int32_t rank, int32_t channel, uint32_t epoch, int32_t timeout_ms, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* NNUE_FT_H */
