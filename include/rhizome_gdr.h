/*
 * rhizome_gdr.h -- C ABI of the B200 (sm_100a) gated delta-rule library.
 *
 * The library is the first optimised backend for RHIZOME's GDR op
 * (crates/ops/src/delta.rs). Each entry below names the reference function
 * it stands in for. Conventions, shared by every entry point:
 *
 *  - Ownership: the caller owns every buffer. All tensor arguments are
 *    DEVICE pointers (the plan arena's model: one base plus 256-byte aligned
 *    offsets, crates/plan/src/arena.rs:71-144). No entry point allocates
 *    device memory; scratch comes in through `workspace` and its size from
 *    rhz_gdr_workspace_bytes().
 *  - Streams: every call is asynchronous and ordered on `stream` (a
 *    cudaStream_t; NULL is the legacy default stream). A returned RHZ_OK
 *    means the work was validated and enqueued.
 *  - Errors: the return value is a status code; rhz_last_error() gives the
 *    message of this host thread's last failure. Shape problems return
 *    RHZ_ERR_SHAPE, the counterpart of rhizome_core::Error::Shape
 *    (crates/core/src/error.rs:27); no entry point aborts on user input
 *    (rule R10). An unsupported (op, dtype, shape) combination is a hard
 *    error, never a silent substitute (rule R4).
 *  - Threads: entry points are reentrant and hold no per-call global state;
 *    calls on different streams from different threads are independent.
 *  - Layouts (row-major, innermost last):
 *      q, k, v, o   [tokens][H][d]      dtype (f32 or bf16); o has q's dtype
 *      alpha, beta  [tokens][H]         f32  (alpha: decay in [0,1], beta: write strength)
 *      states       [n][H][d][d]        f32, S[i][j] with i indexing v and j indexing k
 *                                         (DeltaState, delta.rs:59-66)
 *    "tokens" is B*T for a dense batch ([B][T][H][d]) or the packed total of a
 *    variable-length batch addressed by cu_seqlens.
 *  - Math: per (sequence, head), o_t = S_t q_t with
 *      S_t = alpha_t (S_{t-1} - beta_t (S_{t-1} k_t) k_t^T) + beta_t v_t k_t^T
 *    (delta.rs:93-127). q is used as given (callers pre-scale it), d_k = d_v = d.
 *  - Precision: RHZ_DTYPE_F32 runs an fp32 kernel that applies the recurrence
 *    position by position (matches the f64 reference to rtol 1e-5);
 *    RHZ_DTYPE_BF16 runs the chunked (chunk 64) WY/UT tensor-core kernel with
 *    fp32 state and accumulation (rtol 2e-2, atol 1e-2). Index and packing
 *    entries are bit-exact.
 */
#ifndef RHIZOME_GDR_H
#define RHIZOME_GDR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without pulling in the CUDA headers. */
typedef struct CUstream_st *rhz_stream_t;

/* Status codes. */
enum rhz_status {
    RHZ_OK = 0,
    RHZ_ERR_SHAPE = 1,   /* shape/size mismatch (rhizome_core::Error::Shape) */
    RHZ_ERR_INVALID = 2, /* bad argument value: null or misaligned pointer, bad flag */
    RHZ_ERR_DTYPE = 3,   /* unsupported dtype for this entry point */
    RHZ_ERR_DEVICE = 4,  /* CUDA launch/driver error or a device that is not sm_100 */
    RHZ_ERR_TIMEOUT = 5, /* a bounded device-side wait ran out */
    RHZ_ERR_NCCL = 6     /* collective failure (sharded entry points) */
};

/* Element types of q, k, v and o. alpha, beta and states are always f32. */
enum rhz_dtype { RHZ_DTYPE_F32 = 0, RHZ_DTYPE_BF16 = 1 };

/* Flags for rhz_gdr_varlen_fwd. */
#define RHZ_FLAG_ZERO_INIT 1u /* ignore the slots' contents; start every sequence from S = 0 */
#define RHZ_FLAG_NO_STATE_WRITE 2u /* do not write final states back to the slots */

/* Message of this thread's last failing call ("" if none). Never NULL. */
const char *rhz_last_error(void);

/* ABI version of this header (major * 100 + minor). 1.1 added the
 * host-buffer scan, the device status query and the chunked-form setting;
 * 2.0 gives the bf16 tensor-core path caller-owned scratch: a workspace
 * argument on rhz_gdr_varlen_fwd(_norm), and rhz_gdr_workspace_bytes takes
 * the head count, width and dtype. */
#define RHZ_ABI_VERSION 200
int rhz_abi_version(void);

/*
 * Device-side failure status -- an addition of this library (the reference's
 * ops run on the CPU and have no device waits). The tensor-core kernels and
 * the input producer's TMA form bound every wait on a barrier or a copy; a wait that runs out makes the
 * kernel drain its copies, release its resources and return early, leaving
 * that launch's outputs undefined, and sets a sticky flag on the device.
 * rhz_device_status reads the flags of the current device (synchronising
 * with it) into *timed_out (1 if any wait ran out since the last clear, else
 * 0) and clears them when clear != 0.
 */
int rhz_device_status(int32_t *timed_out, int clear);

/*
 * rhz_gdr_set_wait_test -- test hook of the failure path above, an addition
 * of this library. mode 1: in every later grid-form launch each chain CTA
 * waits for a record flag that no producer sets, with waits on other CTAs'
 * flags bounded at limit_ns (1 us .. 2 s); the wait runs out, the kernel
 * drains, returns early and sets the device flag, exactly as a real timeout
 * would (outputs undefined). mode 0 (the default) turns it off.
 * Process-wide; not for production use.
 */
int rhz_gdr_set_wait_test(int32_t mode, int64_t limit_ns);

/*
 * Which tensor-core form runs the bf16, d == 128 chunked scan
 * (rhz_gdr_scan_chunked, rhz_gdr_varlen_fwd): GRID (the default, AUTO) is
 * one launch over every SM in which chain CTAs carry each (sequence, head)
 * item's state and producer CTAs build the per-chunk records; PAIR (a 2-CTA
 * cluster per item) and SOLO (one CTA per item) are the earlier forms. All
 * give the same results within the bf16 tolerance; GRID and PAIR bitwise.
 * Process-wide; the previous setting goes to *previous unless it is NULL.
 * A variant outside the enum returns RHZ_ERR_INVALID.
 */
enum rhz_chunk_kernel { RHZ_CHUNK_AUTO = 0, RHZ_CHUNK_PAIR = 1, RHZ_CHUNK_SOLO = 2, RHZ_CHUNK_GRID = 3 };
int rhz_gdr_set_chunk_kernel(int32_t variant, int32_t *previous);

/*
 * Which form runs rhz_gdr_scan_chunked_bwd: AUTO (the default) takes the
 * chunked tensor-core form for bf16 inputs with d == 128, no segments and
 * 16-byte aligned q, k, v, d_o, and the fp32 reverse scan otherwise; SCAN
 * forces the fp32 reverse scan everywhere. Process-wide; the previous
 * setting goes to *previous unless it is NULL. Anything else returns
 * RHZ_ERR_INVALID.
 */
enum rhz_bwd_kernel { RHZ_BWD_AUTO = 0, RHZ_BWD_SCAN = 1 };
int rhz_gdr_set_bwd_kernel(int32_t variant, int32_t *previous);

/* --------------------------------------------------------------------- */
/* GDR op family                                                          */
/* --------------------------------------------------------------------- */

/*
 * rhz_gdr_step -- replaces gated_delta_step (crates/ops/src/delta.rs:93-127)
 * batched over n sequences x H heads, one new position each (ragged decode
 * for continuous batching). Sequence i's state for head h is
 * state_pool[slot_idx[i]][h] and is updated in place; slot_idx == NULL means
 * slot i. Like the reference step it honours the state it is given (no
 * reset). q, k, v: [n][H][d]; alpha, beta: [n][H]; o: [n][H][d].
 * A slot index outside [0, num_slots) leaves that pool entry untouched and
 * writes NaN to the sequence's output rows.
 */
int rhz_gdr_step(void *o, float *state_pool, const int32_t *slot_idx, const void *q,
                 const void *k, const void *v, const float *alpha, const float *beta,
                 int64_t n, int64_t num_slots, int32_t H, int32_t d, int32_t dtype,
                 rhz_stream_t stream);

/*
 * rhz_gdr_sequential -- replaces gated_delta_sequential
 * (crates/ops/src/delta.rs:132-154) for B x H heads of T positions. The
 * state resets at t = 0 and wherever segment[b][t] != segment[b][t-1]
 * (segment: [B][T] int64, or NULL for one segment per batch row). As in the
 * reference, the reset at t = 0 means `state_init` never reaches the
 * result: it is accepted (may be NULL) and ignored. state_final: [B][H][d][d]
 * (may be NULL). `workspace`: device memory of
 * rhz_gdr_workspace_bytes(B, T, H, d, dtype, segment != NULL) bytes,
 * 256-byte aligned (NULL/0 when that is 0: the f32 path without segments).
 * Calls that share a workspace must not overlap on the GPU.
 */
int rhz_gdr_sequential(void *o, float *state_final, const void *q, const void *k,
                       const void *v, const float *alpha, const float *beta,
                       const int64_t *segment, const float *state_init, int64_t B, int64_t T,
                       int32_t H, int32_t d, int32_t dtype, void *workspace,
                       size_t workspace_bytes, rhz_stream_t stream);

/*
 * rhz_gdr_scan_chunked -- replaces gated_delta_scan_chunked
 * (crates/ops/src/delta.rs:158-197): same arguments and result as
 * rhz_gdr_sequential plus `chunk`. The reference's result does not depend
 * on `chunk` (chunks only bound its loop); any chunk >= 0 is accepted (0 is
 * treated as 1, as chunk.max(1) does) and the device kernels tile by 64
 * positions, anchored at every segment start.
 */
int rhz_gdr_scan_chunked(void *o, float *state_final, const void *q, const void *k,
                         const void *v, const float *alpha, const float *beta,
                         const int64_t *segment, const float *state_init, int64_t chunk,
                         int64_t B, int64_t T, int32_t H, int32_t d, int32_t dtype,
                         void *workspace, size_t workspace_bytes, rhz_stream_t stream);

/*
 * rhz_gdr_scan_chunked_host -- rhz_gdr_scan_chunked with o, state_final, q,
 * k, v, alpha, beta, segment and state_init in HOST memory (the reference
 * op's own calling convention: slices in, vectors out), for callers whose
 * data is not yet on the GPU. The call copies the inputs in and the outputs
 * out itself, pipelined over slabs of positions (a multiple of 64, about
 * T / 8, at least 256) on two copy streams of its own, so the copies of
 * slab j+1 in, the scan of slab j and the copy of slab j-1 out overlap; the
 * scan runs on `stream`, after the work already queued there. Returns when
 * every output is in host memory. Host buffers should be page-locked
 * (cudaHostAlloc / cudaHostRegister) for the copies to overlap; pageable
 * memory works but serialises them. `workspace`: device memory of
 * rhz_gdr_host_workspace_bytes(B, T, H, d, dtype, segment != NULL) bytes,
 * 256-byte aligned (three slab buffer sets, two state pools, the whole
 * alpha and beta arrays and the slab piece tables). B <= 65535. Results: without segments bitwise those of
 * rhz_gdr_scan_chunked (slabs start on 64-position chunk boundaries and the
 * fp32 state crosses slab boundaries unrounded); with segments a segment
 * that spans a slab boundary is chunked from the boundary as well, which
 * changes the bf16 kernel's rounding order within its tolerance.
 */
int rhz_gdr_scan_chunked_host(void *o, float *state_final, const void *q, const void *k,
                              const void *v, const float *alpha, const float *beta,
                              const int64_t *segment, const float *state_init, int64_t chunk,
                              int64_t B, int64_t T, int32_t H, int32_t d, int32_t dtype,
                              void *workspace, size_t workspace_bytes, rhz_stream_t stream);
size_t rhz_gdr_host_workspace_bytes(int64_t B, int64_t T, int32_t H, int32_t d, int32_t dtype,
                                    int has_segment);

/*
 * rhz_gdr_varlen_fwd -- continuous-batching prefill over one packed stream.
 * Sequence i occupies token rows [cu_seqlens[i], cu_seqlens[i+1]) of
 * q/k/v/alpha/beta/o (cu_seqlens: n_seq + 1 int32, device, non-decreasing,
 * cu_seqlens[0] = 0, cu_seqlens[n_seq] <= total_tokens). Each (sequence, head)
 * starts from state_pool[slot_idx[i]][h] (zeros with RHZ_FLAG_ZERO_INIT) and
 * writes its final state back there (unless RHZ_FLAG_NO_STATE_WRITE). This is
 * gated_delta_step applied over the sequence from the slot's state -- the
 * reference's scan with the segment-start reset replaced by the slot's
 * contents. slot_idx == NULL means slot i. Slots must be distinct.
 * `workspace`: device memory of rhz_gdr_varlen_workspace_bytes(n_seq, H, d,
 * dtype) bytes, 256-byte aligned (NULL/0 when that is 0); calls that share
 * a workspace must not overlap on the GPU.
 */
int rhz_gdr_varlen_fwd(void *o, float *state_pool, const int32_t *slot_idx,
                       const int32_t *cu_seqlens, const void *q, const void *k, const void *v,
                       const float *alpha, const float *beta, int64_t n_seq,
                       int64_t total_tokens, int64_t num_slots, int32_t H, int32_t d,
                       int32_t dtype, uint32_t flags, void *workspace, size_t workspace_bytes,
                       rhz_stream_t stream);
/* Scratch of rhz_gdr_varlen_fwd(_norm) for n_seq sequences (0: none needed). */
size_t rhz_gdr_varlen_workspace_bytes(int64_t n_seq, int32_t H, int32_t d, int32_t dtype);

/*
 * rhz_gdr_varlen_fwd_norm -- rhz_gdr_varlen_fwd followed by the Local
 * block's per-head output norm, groupnorm_heads (crates/ops/src/norm.rs:
 * 48-60): every (token, head) output row of d values becomes
 * o / sqrt(mean(o^2) + norm_eps) * norm_scale[0..d) (the reference applies
 * the first d scale entries to every head). On the bf16 d = 128 path the
 * norm runs in the recurrence kernel's epilogue on the fp32 accumulator;
 * otherwise the standalone rhz_groupnorm_heads follows on the same stream.
 * norm_scale: d f32 (16-byte aligned); d a multiple of 4.
 */
int rhz_gdr_varlen_fwd_norm(void *o, float *state_pool, const int32_t *slot_idx,
                            const int32_t *cu_seqlens, const void *q, const void *k, const void *v,
                            const float *alpha, const float *beta, const float *norm_scale,
                            float norm_eps, int64_t n_seq, int64_t total_tokens, int64_t num_slots,
                            int32_t H, int32_t d, int32_t dtype, uint32_t flags, void *workspace,
                            size_t workspace_bytes, rhz_stream_t stream);

/*
 * rhz_groupnorm_heads -- replaces groupnorm_heads (crates/ops/src/norm.rs:
 * 48-60) over `rows` rows of H heads x d values ([rows][H][d], f32 or
 * bf16): each head is RMS-normalised on its own with scale[0..d) and eps
 * (rmsnorm, norm.rs:8-13). out may equal x (in place). d a multiple of 4,
 * at most 512.
 */
int rhz_groupnorm_heads(void *out, const void *x, const float *scale, int64_t rows, int32_t H,
                        int32_t d, float eps, int32_t dtype, rhz_stream_t stream);

/*
 * rhz_gdr_multistep -- replaces gated_delta_multistep
 * (crates/ops/src/delta.rs:201-230): n sequences x H heads of T positions
 * (q, k, v [n][T][H][d]; alpha, beta [n][T][H]), of which the first
 * Tn = min(T, max_positions) (at most 64) are processed. Writes outs
 * [n][Tn][H][d] and the state after every position, states
 * [n][Tn][H][d][d] f32. With state_pool == NULL it follows the reference:
 * the state starts at zero (the reset at t = 0 discards any initial state)
 * and resets where segment[b][t] != segment[b][t-1] (segment [n][T] int64 or
 * NULL). With a state_pool, sequence i starts from state_pool[slot_idx[i]]
 * (slot i when slot_idx is NULL), segments are ignored and the pool is not
 * modified: speculative decoding scores draft positions and commits the
 * state of the last accepted one afterwards (e.g. with
 * rhz_varlen_scatter_states).
 */
int rhz_gdr_multistep(void *outs, float *states, const float *state_pool,
                      const int32_t *slot_idx, const void *q, const void *k, const void *v,
                      const float *alpha, const float *beta, const int64_t *segment, int64_t n,
                      int64_t T, int64_t max_positions, int64_t num_slots, int32_t H, int32_t d,
                      int32_t dtype, rhz_stream_t stream);

/*
 * rhz_gdr_prep -- the Local block's input producer (SPEC.md:53-54, 61-63),
 * the step in front of the recurrence, built from the reference's pieces:
 * per channel the causal depthwise conv of kernel 4, causal_conv1d_step
 * (crates/ops/src/delta.rs:236-243), carried across each sequence from its
 * slot's 3-sample state; then q = l2norm(conv q) * q_scale,
 * k = l2norm(conv k), v = conv v (l2norm, crates/ops/src/elementwise.rs:
 * 125-129), beta = sigmoid(beta_logit) (:5-12), alpha =
 * exp(-softplus(a_head[h]) * softplus(alpha_logit)) (:36-42).
 * Layouts: xq/xk/xv and q/k/v [tokens][H][d] in `dtype`; beta_logit,
 * alpha_logit, alpha, beta [tokens][H] f32; a_head [H]; conv_w [3][H][d][4]
 * and conv_b [3][H][d] f32 for the q, k, v channels; conv_state
 * [num_slots][3][H][d][3] f32, samples oldest first. Sequence i covers
 * [cu_seqlens[i], cu_seqlens[i+1]) (cu_seqlens NULL: n_seq dense rows of
 * seq_len tokens, total_tokens ignored) and uses conv-state slot
 * slot_idx[i] (slot i when slot_idx is NULL). RHZ_FLAG_ZERO_INIT starts
 * every sequence from a zero conv state (a segment start); its last three
 * samples are written back unless RHZ_FLAG_NO_STATE_WRITE (or conv_state is
 * NULL: zero start, nothing written). A slot index outside [0, num_slots)
 * starts from zeros and writes nothing. d a multiple of 4, at most 512.
 * Decode is the same call with one token per sequence.
 */
int rhz_gdr_prep(void *q, void *k, void *v, float *alpha, float *beta, const void *xq,
                 const void *xk, const void *xv, const float *beta_logit, const float *alpha_logit,
                 const float *a_head, const float *conv_w, const float *conv_b, float *conv_state,
                 const int32_t *slot_idx, const int32_t *cu_seqlens, int64_t n_seq,
                 int64_t seq_len, int64_t total_tokens, int64_t num_slots, int32_t H, int32_t d,
                 float q_scale, int32_t dtype, uint32_t flags, rhz_stream_t stream);

/*
 * rhz_gdr_scan_chunked_bwd -- backward of rhz_gdr_sequential /
 * rhz_gdr_scan_chunked (the adjoint the reference names, "reverse scan of
 * the rank-1 update", docs/kernels.md:16, but does not implement; derived
 * from delta.rs:93-127 and checked against f64 central differences). The
 * state resets at t = 0 and where segment[b][t] != segment[b][t-1] (segment
 * [B][T] int64 or NULL), exactly as in the forward. Given d_o [B][T][H][d]
 * (the gradient of o) and d_state_final [B][H][d][d] (the gradient of the
 * final state, or NULL for zero), writes dq, dk, dv [B][T][H][d] (dtype)
 * and dalpha, dbeta [B][T][H] f32. d a multiple of 4, at most 128. Two
 * forms (rhz_gdr_set_bwd_kernel): bf16 inputs with d == 128 and no segments
 * run the chunked tensor-core form (fp16 products, fp32 accumulation, the
 * upstream gradients scaled by an exact power of two; per-chunk records and
 * the states at chunk boundaries in the workspace); everything else runs an
 * fp32 reverse scan (state checkpoints every 8 positions and per-row-block
 * partial sums). Needs `workspace` of rhz_gdr_bwd_workspace_bytes(B, T, H,
 * d) bytes (the larger of the two forms' needs). Both forms are
 * deterministic.
 */
int rhz_gdr_scan_chunked_bwd(void *dq, void *dk, void *dv, float *dalpha, float *dbeta,
                             const void *q, const void *k, const void *v, const float *alpha,
                             const float *beta, const int64_t *segment, const void *d_o,
                             const float *d_state_final, int64_t B, int64_t T, int32_t H,
                             int32_t d, int32_t dtype, void *workspace, size_t workspace_bytes,
                             rhz_stream_t stream);

/* rhz_gdr_bwd_workspace_bytes -- scratch of rhz_gdr_scan_chunked_bwd (0 for unsupported shapes). */
size_t rhz_gdr_bwd_workspace_bytes(int64_t B, int64_t T, int32_t H, int32_t d);

/*
 * rhz_gdr_workspace_bytes -- scratch needed by rhz_gdr_sequential /
 * rhz_gdr_scan_chunked for B x T positions of H heads of width d in
 * `dtype`, with or without a segment array: the tensor-core kernel's
 * record rings and schedule (bf16, d == 128: about 34 MB) plus, with
 * segments, the segment-boundary tables. 0 when nothing is needed.
 */
size_t rhz_gdr_workspace_bytes(int64_t B, int64_t T, int32_t H, int32_t d, int32_t dtype,
                               int has_segment);

/* --------------------------------------------------------------------- */
/* Variable-length packing (bit-exact index work)                         */
/* --------------------------------------------------------------------- */

/*
 * rhz_varlen_prefix_sum -- cu_seqlens[0] = 0, cu_seqlens[i+1] =
 * cu_seqlens[i] + lengths[i] for i < n (int32, device). The packed layout of
 * continuous batching: it replaces building segment ids position by
 * position (delta.rs:21-28, SPEC.md:21-22).
 */
int rhz_varlen_prefix_sum(int32_t *cu_seqlens, const int32_t *lengths, int64_t n,
                          rhz_stream_t stream);

/*
 * rhz_varlen_segments_to_cu_seqlens -- turns a [B][T] int64 segment-id array
 * (delta.rs:27-28) into segment boundaries over the flattened B*T positions:
 * a boundary at every t where b changes, t = 0 within a row, or the id
 * changes (the reset rule of delta.rs:137-141). Writes n_seg + 1 offsets to
 * cu_seqlens (room for B*T + 1) and n_seg to *n_seg_out (device int32).
 */
int rhz_varlen_segments_to_cu_seqlens(int32_t *cu_seqlens, int32_t *n_seg_out,
                                      const int64_t *segment, int64_t B, int64_t T,
                                      void *workspace, size_t workspace_bytes,
                                      rhz_stream_t stream);

/*
 * rhz_varlen_chunk_map -- the chunk list of a packed batch: chunks of
 * `chunk` positions anchored at each sequence's own start (never crossing a
 * sequence end, delta.rs:171-178). Writes chunk_seq[c] (sequence id) and
 * chunk_start[c] (first token row) in (sequence, position) order and the count
 * to *n_chunks_out; max_chunks bounds the output arrays (the count is still
 * reported if larger).
 */
int rhz_varlen_chunk_map(int32_t *chunk_seq, int32_t *chunk_start, int32_t *n_chunks_out,
                         const int32_t *cu_seqlens, int64_t n_seq, int32_t chunk,
                         int64_t max_chunks, void *workspace, size_t workspace_bytes,
                         rhz_stream_t stream);

/* Scratch for rhz_varlen_chunk_map / rhz_varlen_segments_to_cu_seqlens. */
size_t rhz_varlen_workspace_bytes(int64_t n);

/*
 * rhz_varlen_gather_states / rhz_varlen_scatter_states -- copy the d x d
 * states of n sequences x H heads between a slot pool [num_slots][H][d][d]
 * and a dense [n][H][d][d] buffer (dense[i] = pool[slot_idx[i]] and back).
 */
int rhz_varlen_gather_states(float *dense, const float *pool, const int32_t *slot_idx,
                             int64_t n, int64_t num_slots, int32_t H, int32_t d,
                             rhz_stream_t stream);
int rhz_varlen_scatter_states(float *pool, const float *dense, const int32_t *slot_idx,
                              int64_t n, int64_t num_slots, int32_t H, int32_t d,
                              rhz_stream_t stream);

/*
 * rhz_varlen_pack_tokens / rhz_varlen_unpack_tokens -- move rows of
 * row_bytes bytes between a padded [n][max_len] layout and the packed
 * stream addressed by cu_seqlens (padded rows past a sequence's length are
 * left untouched by unpack). row_bytes must be a multiple of 4.
 */
int rhz_varlen_pack_tokens(void *packed, const void *padded, const int32_t *cu_seqlens,
                           int64_t n, int64_t max_len, int64_t row_bytes, rhz_stream_t stream);
int rhz_varlen_unpack_tokens(void *padded, const void *packed, const int32_t *cu_seqlens,
                             int64_t n, int64_t max_len, int64_t row_bytes, rhz_stream_t stream);

/* --------------------------------------------------------------------- */
/* Head sharding across GPUs (bit-exact moves)                             */
/* --------------------------------------------------------------------- */

/*
 * rhz_heads_unshard / rhz_heads_shard -- the full Local-block layer splits
 * its H heads evenly over G ranks (rank r owns heads [r H/G, (r+1) H/G)); the
 * recurrence never mixes heads (delta.rs:93-127 is per head), so the only
 * exchange is an all-gather of per-head outputs. A collective gathers the
 * ranks' [tokens][H/G][d] outputs rank-major into gathered [G][tokens][H/G][d];
 * unshard reorders that into out [tokens][H][d], shard does the reverse.
 * elem_bytes is 2 (bf16) or 4 (f32).
 */
int rhz_heads_unshard(void *out, const void *gathered, int64_t G, int64_t tokens, int32_t H,
                      int32_t d, int32_t elem_bytes, rhz_stream_t stream);
int rhz_heads_shard(void *gathered, const void *full, int64_t G, int64_t tokens, int32_t H,
                    int32_t d, int32_t elem_bytes, rhz_stream_t stream);

/* --------------------------------------------------------------------- */
/* No-allocation variant                                                  */
/* --------------------------------------------------------------------- */

/* Largest B*T accepted by rhz_varlen_segments_to_cu_seqlens_noalloc. */
#define RHZ_NOALLOC_MAX_POSITIONS (1LL << 26)

/*
 * rhz_varlen_segments_to_cu_seqlens_noalloc -- no counterpart in the
 * reference (an addition of this library). Same arguments and results as
 * rhz_varlen_segments_to_cu_seqlens minus the workspace: the scan's scratch
 * lives in a 64 KiB array inside the library (on every GPU that loads it,
 * until the process exits), so the call allocates no device memory at all.
 * It is for callers that cannot allocate: a plan executor that only owns one
 * buffer, sized and laid out before the step runs, with no room set aside
 * for an op's private scratch, or a serving process that reserved all
 * device memory up front for its state slots, where a cudaMalloc in the
 * middle of a step can fail.
 * Limits and rules:
 *   - B*T must not exceed RHZ_NOALLOC_MAX_POSITIONS (2^26); larger inputs
 *     return RHZ_ERR_SHAPE (use the workspace entry point instead);
 *   - the first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture;
 *   - every call shares the one array: calls whose work overlaps on the GPU
 *     (different streams, or different host threads on one device) race.
 */
int rhz_varlen_segments_to_cu_seqlens_noalloc(int32_t *cu_seqlens, int32_t *n_seg_out,
                                              const int64_t *segment, int64_t B, int64_t T,
                                              rhz_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* RHIZOME_GDR_H */
