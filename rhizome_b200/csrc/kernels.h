// Internal launcher interface between the C ABI (capi.cu) and the kernels.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace rhz {

// One recurrence position for a ragged batch (gdr_simt.cu).
struct StepArgs {
    void *o;
    float *pool;
    const int32_t *slots;
    const void *q, *k, *v;
    const float *alpha, *beta;
    int64_t n, num_slots;
    int H, d, dtype;
    cudaStream_t stream;
};

// Whole sequences, position by position in fp32 (gdr_simt.cu) or chunked on
// tensor cores (gdr_chunk_tc.cu). Sequence i covers token rows
// [cu_seqlens[i], cu_seqlens[i+1]) or, with cu_seqlens == nullptr,
// [i * seq_len, (i + 1) * seq_len). n_seq is the host-side upper bound; when
// n_seq_dev is set the device count is used.
struct SeqArgs {
    void *o;
    const void *q, *k, *v;
    const float *alpha, *beta;
    const int32_t *cu_seqlens;
    const int32_t *n_seq_dev;
    int64_t n_seq;
    int64_t seq_len;
    int64_t total_tokens;
    const float *state_in;      // nullptr => zeros
    const int32_t *in_slots;    // nullptr => sequence i uses slot i
    float *state_out;           // nullptr => not written
    const int32_t *out_slots;   // nullptr => sequence i uses slot i
    int64_t num_slots;
    int H, d, dtype;
    cudaStream_t stream;
    const float *norm_scale;    // non-null: groupnorm_heads on o (scale[0..d), norm_eps)
    float norm_eps;
    void *ws;                   // scratch of the tensor-core grid kernel (chunk_grid_ws_bytes)
    size_t ws_bytes;
};

// Up to Tn positions per sequence, state after each position written out
// (gdr_simt.cu). pool == nullptr: zero start with segment resets.
struct MultistepArgs {
    void *outs;
    float *states;
    const float *pool;
    const int32_t *slots;
    const void *q, *k, *v;
    const float *alpha, *beta;
    const int64_t *segment;
    int64_t n, T;
    int Tn;
    int64_t num_slots;
    int H, d, dtype;
    cudaStream_t stream;
};

// Input producer: conv + norms + gates in front of the recurrence (prep.cu).
struct PrepArgs {
    void *q, *k, *v;
    float *alpha, *beta;
    const void *xq, *xk, *xv;
    const float *beta_logit, *alpha_logit, *a_head;
    const float *conv_w, *conv_b;
    float *conv_state;          // nullptr => zero carried state, nothing written
    const int32_t *slots;       // nullptr => sequence i uses slot i
    const int32_t *cu_seqlens;  // nullptr => dense n_seq x seq_len
    int64_t n_seq, seq_len, total_tokens, num_slots;
    int H, d, dtype;
    float q_scale;
    bool zero_init, write_state;
    cudaStream_t stream;
};

int launch_step(const StepArgs &a);
int launch_prep(const PrepArgs &a);
// Sticky flag of the input producer's bounded TMA wait (1: a wait ran out).
int prep_status(int *flag, bool clear);
int launch_multistep(const MultistepArgs &a);
int launch_seq(const SeqArgs &a);
// Tensor-core chunked kernel (bf16, d == 128). Returns RHZ_ERR_SHAPE for
// shapes it does not tile.
int launch_chunk_tc(const SeqArgs &a);
bool chunk_tc_supports(int d, int dtype);
// The two forms behind launch_chunk_tc: a 2-CTA cluster per (sequence, head)
// item (gdr_chunk_tc.cu) and one CTA per item (gdr_chunk_solo.cu).
int launch_chunk_pair(const SeqArgs &a);
int launch_chunk_solo(const SeqArgs &a);
bool chunk_use_solo(int64_t items, int sms);
// Forces one form (RHZ_CHUNK_*), the previous setting to *prev.
int set_chunk_variant(int v, int *prev);
// Sticky device flags: 1 once a bounded wait of that kernel gave up.
int chunk_pair_status(int *flag, bool clear);
int chunk_solo_status(int *flag, bool clear);
// The grid form (gdr_chunk_grid.cu): one cooperative launch, chain CTAs fed
// by producer CTAs through record rings in the workspace.
int launch_chunk_grid(const SeqArgs &a);
size_t chunk_grid_ws_bytes(int64_t n_items, bool packed);
int chunk_grid_status(int *flag, bool clear);
// Test hook of the grid form's failure path (mode 1: chains wait for a flag
// nothing sets, bounded at limit_ns; mode 0: off).
int set_wait_test(int mode, int64_t limit_ns);

// Variable-length index work (varlen.cu).
int launch_prefix_sum(int32_t *cu, const int32_t *lengths, int64_t n, cudaStream_t s);
size_t varlen_ws_bytes(int64_t n);
int launch_segments_to_cu(int32_t *cu, int32_t *n_seg, const int64_t *segment, int64_t B,
                          int64_t T, void *ws, size_t ws_bytes, cudaStream_t s);
int launch_chunk_map(int32_t *chunk_seq, int32_t *chunk_start, int32_t *n_chunks,
                     const int32_t *cu, int64_t n_seq, int chunk, int64_t max_chunks, void *ws,
                     size_t ws_bytes, cudaStream_t s);
int launch_gather_states(float *dense, const float *pool, const int32_t *slots, int64_t n,
                         int64_t num_slots, int H, int d, bool scatter, cudaStream_t s);
// Backward of the sequential / chunked scan (gdr_bwd.cu): resets at t = 0
// and at segment changes; dense [B][T][H][d] layouts.
struct BwdArgs {
    void *dq, *dk, *dv;
    float *dalpha, *dbeta;
    const void *q, *k, *v, *d_o;
    const float *alpha, *beta;
    const int64_t *segment;       // [B][T] or nullptr
    const float *d_state_final;   // [B][H][d][d] or nullptr
    void *workspace;
    int64_t B, T;
    int H, d, dtype;
    cudaStream_t stream;
};
size_t bwd_ws_bytes(int64_t B, int64_t T, int H, int d);
int launch_bwd(const BwdArgs &a);
// Chunked tensor-core backward (gdr_bwd_tc.cu): bf16, d = 128, no segments,
// 16-byte aligned q/k/v/d_o. set_bwd_form(1) forces the fp32 reverse scan.
bool bwd_tc_supports(const BwdArgs &a);
size_t bwd_tc_ws_bytes(int64_t B, int64_t T, int H, int d);
int launch_bwd_tc(const BwdArgs &a);
int set_bwd_form(int form, int *prev);

// groupnorm_heads over rows x H slices of d values (norm.cu); out may be x.
int launch_groupnorm_heads(void *out, const void *x, const float *scale, int64_t rows, int H, int d,
                           float eps, int dtype, cudaStream_t s);
int launch_heads_unshard(void *dst, const void *src, int64_t G, int64_t tokens, int64_t Hs,
                         int64_t row_bytes, bool shard, cudaStream_t s);
int launch_pack_tokens(void *dst, const void *src, const int32_t *cu, int64_t n, int64_t max_len,
                       int64_t row_bytes, bool unpack, cudaStream_t s);

}  // namespace rhz
