// C ABI of the GDR library: argument validation (the shape rules of
// DeltaInputs::is_consistent, crates/ops/src/delta.rs:46-55, on the batched
// layouts), status codes with a per-thread message, and dispatch to the
// kernels. Nothing here allocates device memory; the host-buffer entry point
// keeps three copy streams and a few events per device.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/rhizome_gdr.h"
#include "common.cuh"
#include "kernels.h"

namespace rhz {

namespace {
thread_local char g_last_error[512] = "";

// Immutable per-device properties, filled on first use (the library's only
// global state).
struct DevInfo {
    std::atomic<int> ready{0};
    int sm_count = 0;
    bool sm100 = false;
};
DevInfo g_dev[64];
}  // namespace

int set_error(int code, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

void clear_error() { g_last_error[0] = '\0'; }

int check_launch(const char *what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(RHZ_ERR_DEVICE, "%s: %s", what, cudaGetErrorString(e));
    return RHZ_OK;
}

int device_info(int *sm_count, bool *is_sm100) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(RHZ_ERR_DEVICE, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return set_error(RHZ_ERR_DEVICE, "device ordinal %d out of range", dev);
    DevInfo &d = g_dev[dev];
    if (!d.ready.load(std::memory_order_acquire)) {
        cudaDeviceProp p;
        e = cudaGetDeviceProperties(&p, dev);
        if (e != cudaSuccess)
            return set_error(RHZ_ERR_DEVICE, "cudaGetDeviceProperties: %s", cudaGetErrorString(e));
        d.sm_count = p.multiProcessorCount;
        d.sm100 = p.major == 10 && p.minor == 0;
        d.ready.store(1, std::memory_order_release);
    }
    *sm_count = d.sm_count;
    *is_sm100 = d.sm100;
    return RHZ_OK;
}

namespace {

int require_sm100() {
    int sms = 0;
    bool ok = false;
    int st = device_info(&sms, &ok);
    if (st != RHZ_OK) return st;
    if (!ok) return set_error(RHZ_ERR_DEVICE, "this library is built for sm_100a (B200) only");
    return RHZ_OK;
}

int check_dtype(int32_t dtype) {
    if (dtype != RHZ_DTYPE_F32 && dtype != RHZ_DTYPE_BF16)
        return set_error(RHZ_ERR_DTYPE, "unsupported dtype %d (expected RHZ_DTYPE_F32 or RHZ_DTYPE_BF16)", dtype);
    return RHZ_OK;
}

int check_heads(int32_t H, int32_t d) {
    if (H < 1) return set_error(RHZ_ERR_SHAPE, "H = %d: need at least one head", H);
    // DeltaInputs::is_consistent requires head_dim > 0 (delta.rs:50).
    if (d < 1) return set_error(RHZ_ERR_SHAPE, "head_dim = %d: must be > 0", d);
    if (d > 256) return set_error(RHZ_ERR_SHAPE, "head_dim = %d: kernels tile head widths up to 256", d);
    return RHZ_OK;
}

int check_ptr(const void *p, const char *name, size_t align, bool needed) {
    if (!needed) return RHZ_OK;
    if (p == nullptr) return set_error(RHZ_ERR_INVALID, "%s is NULL", name);
    if (!aligned(p, align)) return set_error(RHZ_ERR_INVALID, "%s is not %zu-byte aligned", name, align);
    return RHZ_OK;
}

#define RHZ_TRY(x)                  \
    do {                            \
        int _st = (x);              \
        if (_st != RHZ_OK) return _st; \
    } while (0)

// Offsets of the sequential/chunked entry points' workspace.
// The tensor-core kernel's scratch (record rings, schedule) comes first,
// then, with segments, the segment-to-cu_seqlens tables.
struct SegWs {
    size_t grid_bytes, cu_off, nseg_off, slot_off, scan_off, total;
};

SegWs seg_ws(int64_t B, int64_t T, int32_t H, int32_t d, int32_t dtype, bool has_segment) {
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    SegWs w{};
    const size_t N = static_cast<size_t>(B * T);
    w.grid_bytes = chunk_tc_supports(d, dtype)
                       ? up(chunk_grid_ws_bytes((has_segment ? B * T : B) * H, has_segment))
                       : 0;
    w.cu_off = w.grid_bytes;
    if (!has_segment) {
        w.nseg_off = w.slot_off = w.scan_off = w.total = w.grid_bytes;
        return w;
    }
    w.nseg_off = up(w.cu_off + (N + 1) * sizeof(int32_t));
    w.slot_off = up(w.nseg_off + sizeof(int32_t));
    w.scan_off = up(w.slot_off + (N + 1) * sizeof(int32_t));
    w.total = w.scan_off + varlen_ws_bytes(static_cast<int64_t>(N));
    return w;
}

// Segment s writes its final state to batch row b only if it is the last
// segment of row b (it ends where the row ends): the state
// gated_delta_sequential returns (delta.rs:153).
__global__ void final_slot_kernel(const int32_t *cu, const int32_t *n_seg, int64_t T, int32_t *slot) {
    const int64_t n = *n_seg;
    for (int64_t s = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; s < n;
         s += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t end = cu[s + 1];
        slot[s] = (end % T == 0) ? static_cast<int32_t>(end / T - 1) : -1;
    }
}

// The tensor-core kernel applies an output norm in its epilogue; the fp32
// scan is followed by the standalone norm over the same rows.
int run_seq(const SeqArgs &a) {
    if (chunk_tc_supports(a.d, a.dtype)) return launch_chunk_tc(a);
    const int st = launch_seq(a);
    if (st != RHZ_OK || a.norm_scale == nullptr) return st;
    const int64_t rows = a.cu_seqlens ? a.total_tokens : a.n_seq * a.seq_len;
    return launch_groupnorm_heads(a.o, a.o, a.norm_scale, rows, a.H, a.d, a.norm_eps, a.dtype, a.stream);
}

int sequential_impl(void *o, float *state_final, const void *q, const void *k, const void *v,
                    const float *alpha, const float *beta, const int64_t *segment,
                    const float *state_init, int64_t B, int64_t T, int32_t H, int32_t d,
                    int32_t dtype, void *workspace, size_t workspace_bytes,
                    rhz_stream_t stream) {
    RHZ_TRY(check_dtype(dtype));
    RHZ_TRY(check_heads(H, d));
    if (B < 0 || T < 0) return set_error(RHZ_ERR_SHAPE, "B = %lld, T = %lld: must be >= 0", (long long)B, (long long)T);
    if (B * T > INT32_MAX - 1) return set_error(RHZ_ERR_SHAPE, "B*T = %lld positions exceeds int32 indexing", (long long)(B * T));
    const bool any = B * T > 0;
    RHZ_TRY(check_ptr(q, "q", 16, any));
    RHZ_TRY(check_ptr(k, "k", 16, any));
    RHZ_TRY(check_ptr(v, "v", 16, any));
    RHZ_TRY(check_ptr(o, "o", 16, any));
    RHZ_TRY(check_ptr(alpha, "alpha", 4, any));
    RHZ_TRY(check_ptr(beta, "beta", 4, any));
    RHZ_TRY(check_ptr(state_final, "state_final", 16, state_final != nullptr));
    RHZ_TRY(check_ptr(segment, "segment", 8, segment != nullptr));
    const SegWs w = seg_ws(B, T, H, d, dtype, segment != nullptr);
    if (any && w.total > 0) {
        if (workspace == nullptr || workspace_bytes < w.total)
            return set_error(RHZ_ERR_INVALID, "workspace too small: need %zu bytes, got %zu", w.total, workspace_bytes);
        RHZ_TRY(check_ptr(workspace, "workspace", 256, true));
    }
    RHZ_TRY(require_sm100());
    cudaStream_t s = as_cuda(stream);
    const size_t state_bytes = static_cast<size_t>(B) * H * d * d * sizeof(float);
    if (T == 0) {
        // The loop never runs: the reference returns init.clone() (delta.rs:135).
        if (state_final && state_bytes) {
            cudaError_t e = state_init
                                ? cudaMemcpyAsync(state_final, state_init, state_bytes,
                                                  cudaMemcpyDeviceToDevice, s)
                                : cudaMemsetAsync(state_final, 0, state_bytes, s);
            if (e != cudaSuccess) return set_error(RHZ_ERR_DEVICE, "state copy: %s", cudaGetErrorString(e));
        }
        return RHZ_OK;
    }
    if (B == 0) return RHZ_OK;

    char *ws = static_cast<char *>(workspace);
    SeqArgs a{};
    a.o = o; a.q = q; a.k = k; a.v = v; a.alpha = alpha; a.beta = beta;
    a.total_tokens = B * T;
    a.H = H; a.d = d; a.dtype = dtype; a.stream = s;
    a.state_in = nullptr;  // reset at t = 0: the initial state never contributes
    a.ws = w.grid_bytes ? ws : nullptr;
    a.ws_bytes = w.grid_bytes;
    if (segment == nullptr) {
        a.cu_seqlens = nullptr;
        a.n_seq = B;
        a.seq_len = T;
        a.state_out = state_final;
        a.num_slots = B;
        return run_seq(a);
    }
    int32_t *cu = reinterpret_cast<int32_t *>(ws + w.cu_off);
    int32_t *nseg = reinterpret_cast<int32_t *>(ws + w.nseg_off);
    int32_t *slots = reinterpret_cast<int32_t *>(ws + w.slot_off);
    RHZ_TRY(launch_segments_to_cu(cu, nseg, segment, B, T, ws + w.scan_off, w.total - w.scan_off, s));
    if (state_final) {
        final_slot_kernel<<<64, 256, 0, s>>>(cu, nseg, T, slots);
        RHZ_TRY(check_launch("final_slot_kernel"));
    }
    a.cu_seqlens = cu;
    a.n_seq_dev = nseg;
    a.n_seq = B * T;
    a.seq_len = 0;
    a.state_out = state_final;
    a.out_slots = state_final ? slots : nullptr;
    a.num_slots = B;
    return run_seq(a);
}

}  // namespace
}  // namespace rhz

using namespace rhz;

extern "C" {

const char *rhz_last_error(void) { return g_last_error; }

int rhz_abi_version(void) { return RHZ_ABI_VERSION; }

int rhz_device_status(int32_t *timed_out, int clear) {
    clear_error();
    if (!timed_out) return set_error(RHZ_ERR_INVALID, "timed_out must not be NULL");
    int a = 0, b = 0, c = 0, e = 0;
    int st = chunk_pair_status(&a, clear != 0);
    if (st == RHZ_OK) st = chunk_solo_status(&b, clear != 0);
    if (st == RHZ_OK) st = chunk_grid_status(&c, clear != 0);
    if (st == RHZ_OK) st = prep_status(&e, clear != 0);
    if (st != RHZ_OK) return st;
    *timed_out = (a | b | c | e) ? 1 : 0;
    return RHZ_OK;
}

int rhz_gdr_set_wait_test(int32_t mode, int64_t limit_ns) {
    clear_error();
    return set_wait_test(mode, limit_ns);
}

int rhz_gdr_set_chunk_kernel(int32_t variant, int32_t *previous) {
    clear_error();
    int prev = 0;
    const int st = set_chunk_variant(variant, &prev);
    if (st == RHZ_OK && previous) *previous = prev;
    return st;
}

int rhz_gdr_set_bwd_kernel(int32_t variant, int32_t *previous) {
    clear_error();
    int prev = 0;
    const int st = set_bwd_form(variant, &prev);
    if (st == RHZ_OK && previous) *previous = prev;
    return st;
}

int rhz_gdr_step(void *o, float *state_pool, const int32_t *slot_idx, const void *q,
                 const void *k, const void *v, const float *alpha, const float *beta, int64_t n,
                 int64_t num_slots, int32_t H, int32_t d, int32_t dtype, rhz_stream_t stream) {
    clear_error();
    RHZ_TRY(check_dtype(dtype));
    RHZ_TRY(check_heads(H, d));
    if (n < 0 || num_slots < 0) return set_error(RHZ_ERR_SHAPE, "n = %lld, num_slots = %lld: must be >= 0", (long long)n, (long long)num_slots);
    if (slot_idx == nullptr && n > num_slots)
        return set_error(RHZ_ERR_SHAPE, "n = %lld sequences but only %lld slots (slot_idx is NULL)", (long long)n, (long long)num_slots);
    if (n * H > INT32_MAX) return set_error(RHZ_ERR_SHAPE, "n*H = %lld exceeds the grid", (long long)(n * H));
    if (n == 0) return RHZ_OK;
    RHZ_TRY(check_ptr(q, "q", 16, true));
    RHZ_TRY(check_ptr(k, "k", 16, true));
    RHZ_TRY(check_ptr(v, "v", 16, true));
    RHZ_TRY(check_ptr(o, "o", 16, true));
    RHZ_TRY(check_ptr(alpha, "alpha", 4, true));
    RHZ_TRY(check_ptr(beta, "beta", 4, true));
    RHZ_TRY(check_ptr(state_pool, "state_pool", 16, true));
    RHZ_TRY(check_ptr(slot_idx, "slot_idx", 4, slot_idx != nullptr));
    RHZ_TRY(require_sm100());
    StepArgs a{o, state_pool, slot_idx, q, k, v, alpha, beta, n, num_slots, H, d, dtype, as_cuda(stream)};
    return launch_step(a);
}

int rhz_gdr_sequential(void *o, float *state_final, const void *q, const void *k, const void *v,
                       const float *alpha, const float *beta, const int64_t *segment,
                       const float *state_init, int64_t B, int64_t T, int32_t H, int32_t d,
                       int32_t dtype, void *workspace, size_t workspace_bytes,
                       rhz_stream_t stream) {
    clear_error();
    return sequential_impl(o, state_final, q, k, v, alpha, beta, segment, state_init, B, T, H, d,
                           dtype, workspace, workspace_bytes, stream);
}

int rhz_gdr_scan_chunked(void *o, float *state_final, const void *q, const void *k,
                         const void *v, const float *alpha, const float *beta,
                         const int64_t *segment, const float *state_init, int64_t chunk,
                         int64_t B, int64_t T, int32_t H, int32_t d, int32_t dtype,
                         void *workspace, size_t workspace_bytes, rhz_stream_t stream) {
    clear_error();
    if (chunk < 0) return set_error(RHZ_ERR_SHAPE, "chunk = %lld: must be >= 0", (long long)chunk);
    return sequential_impl(o, state_final, q, k, v, alpha, beta, segment, state_init, B, T, H, d,
                           dtype, workspace, workspace_bytes, stream);
}

}  // extern "C"

namespace {
int varlen_impl(void *o, float *state_pool, const int32_t *slot_idx, const int32_t *cu_seqlens,
                const void *q, const void *k, const void *v, const float *alpha, const float *beta,
                const float *norm_scale, float norm_eps, int64_t n_seq, int64_t total_tokens,
                int64_t num_slots, int32_t H, int32_t d, int32_t dtype, uint32_t flags,
                void *workspace, size_t workspace_bytes, rhz_stream_t stream) {
    RHZ_TRY(check_dtype(dtype));
    RHZ_TRY(check_heads(H, d));
    if (flags & ~(RHZ_FLAG_ZERO_INIT | RHZ_FLAG_NO_STATE_WRITE))
        return set_error(RHZ_ERR_INVALID, "unknown flags 0x%x", flags);
    if (n_seq < 0 || total_tokens < 0 || num_slots < 0)
        return set_error(RHZ_ERR_SHAPE, "negative size (n_seq %lld, total_tokens %lld, num_slots %lld)",
                         (long long)n_seq, (long long)total_tokens, (long long)num_slots);
    if (total_tokens > INT32_MAX) return set_error(RHZ_ERR_SHAPE, "total_tokens exceeds int32 offsets");
    if (slot_idx == nullptr && n_seq > num_slots)
        return set_error(RHZ_ERR_SHAPE, "n_seq = %lld but only %lld slots (slot_idx is NULL)", (long long)n_seq, (long long)num_slots);
    if (n_seq == 0) return RHZ_OK;
    const size_t need = chunk_tc_supports(d, dtype) ? chunk_grid_ws_bytes(n_seq * H, true) : 0;
    if (need > 0) {
        if (workspace == nullptr || workspace_bytes < need)
            return set_error(RHZ_ERR_INVALID, "workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
        RHZ_TRY(check_ptr(workspace, "workspace", 256, true));
    }
    const bool any = total_tokens > 0;
    RHZ_TRY(check_ptr(cu_seqlens, "cu_seqlens", 4, true));
    RHZ_TRY(check_ptr(q, "q", 16, any));
    RHZ_TRY(check_ptr(k, "k", 16, any));
    RHZ_TRY(check_ptr(v, "v", 16, any));
    RHZ_TRY(check_ptr(o, "o", 16, any));
    RHZ_TRY(check_ptr(alpha, "alpha", 4, any));
    RHZ_TRY(check_ptr(beta, "beta", 4, any));
    const bool need_pool = !(flags & RHZ_FLAG_ZERO_INIT) || !(flags & RHZ_FLAG_NO_STATE_WRITE);
    RHZ_TRY(check_ptr(state_pool, "state_pool", 16, need_pool));
    RHZ_TRY(check_ptr(slot_idx, "slot_idx", 4, slot_idx != nullptr));
    RHZ_TRY(require_sm100());
    SeqArgs a{};
    a.o = o; a.q = q; a.k = k; a.v = v; a.alpha = alpha; a.beta = beta;
    a.cu_seqlens = cu_seqlens;
    a.n_seq = n_seq;
    a.total_tokens = total_tokens;
    a.state_in = (flags & RHZ_FLAG_ZERO_INIT) ? nullptr : state_pool;
    a.in_slots = slot_idx;
    a.state_out = (flags & RHZ_FLAG_NO_STATE_WRITE) ? nullptr : state_pool;
    a.out_slots = slot_idx;
    a.num_slots = num_slots;
    a.H = H; a.d = d; a.dtype = dtype; a.stream = as_cuda(stream);
    a.norm_scale = norm_scale;
    a.norm_eps = norm_eps;
    a.ws = need ? workspace : nullptr;
    a.ws_bytes = need;
    return run_seq(a);
}
}  // namespace

extern "C" {

int rhz_gdr_varlen_fwd(void *o, float *state_pool, const int32_t *slot_idx,
                       const int32_t *cu_seqlens, const void *q, const void *k, const void *v,
                       const float *alpha, const float *beta, int64_t n_seq,
                       int64_t total_tokens, int64_t num_slots, int32_t H, int32_t d,
                       int32_t dtype, uint32_t flags, void *workspace, size_t workspace_bytes,
                       rhz_stream_t stream) {
    clear_error();
    return varlen_impl(o, state_pool, slot_idx, cu_seqlens, q, k, v, alpha, beta, nullptr, 0.f,
                       n_seq, total_tokens, num_slots, H, d, dtype, flags, workspace,
                       workspace_bytes, stream);
}

size_t rhz_gdr_varlen_workspace_bytes(int64_t n_seq, int32_t H, int32_t d, int32_t dtype) {
    if (n_seq < 0 || H < 1 || d < 1) return 0;
    return chunk_tc_supports(d, dtype) ? chunk_grid_ws_bytes(n_seq * H, true) : 0;
}

int rhz_gdr_varlen_fwd_norm(void *o, float *state_pool, const int32_t *slot_idx,
                            const int32_t *cu_seqlens, const void *q, const void *k, const void *v,
                            const float *alpha, const float *beta, const float *norm_scale,
                            float norm_eps, int64_t n_seq, int64_t total_tokens, int64_t num_slots,
                            int32_t H, int32_t d, int32_t dtype, uint32_t flags, void *workspace,
                            size_t workspace_bytes, rhz_stream_t stream) {
    clear_error();
    if (!(norm_eps >= 0.f)) return set_error(RHZ_ERR_INVALID, "norm_eps must be >= 0");
    RHZ_TRY(check_ptr(norm_scale, "norm_scale", 16, true));
    if (d % 4) return set_error(RHZ_ERR_SHAPE, "the output norm needs d a multiple of 4 (got %d)", d);
    return varlen_impl(o, state_pool, slot_idx, cu_seqlens, q, k, v, alpha, beta, norm_scale,
                       norm_eps, n_seq, total_tokens, num_slots, H, d, dtype, flags, workspace,
                       workspace_bytes, stream);
}

size_t rhz_gdr_bwd_workspace_bytes(int64_t B, int64_t T, int32_t H, int32_t d) {
    if (B < 0 || T < 0 || H < 1 || d < 4 || d > 128 || d % 4) return 0;
    return bwd_ws_bytes(B, T, H, d);
}

int rhz_gdr_scan_chunked_bwd(void *dq, void *dk, void *dv, float *dalpha, float *dbeta,
                             const void *q, const void *k, const void *v, const float *alpha,
                             const float *beta, const int64_t *segment, const void *d_o,
                             const float *d_state_final, int64_t B, int64_t T, int32_t H,
                             int32_t d, int32_t dtype, void *workspace, size_t workspace_bytes,
                             rhz_stream_t stream) {
    clear_error();
    RHZ_TRY(check_dtype(dtype));
    if (B < 0 || T < 0 || H < 1 || d < 4 || d > 128 || d % 4)
        return set_error(RHZ_ERR_SHAPE, "backward needs B, T >= 0, H >= 1, d a multiple of 4 in [4, 128] (got %lld, %lld, %d, %d)",
                         (long long)B, (long long)T, H, d);
    if (B * H * ((d + 15) / 16) > INT32_MAX || B * H * T > INT32_MAX)
        return set_error(RHZ_ERR_SHAPE, "B*H*T exceeds the grid");
    if (B == 0 || T == 0) return RHZ_OK;
    const size_t need = bwd_ws_bytes(B, T, H, d);
    if (workspace == nullptr || workspace_bytes < need)
        return set_error(RHZ_ERR_INVALID, "workspace too small: need %zu bytes, got %zu", need, workspace_bytes);
    const size_t vec = dtype == RHZ_DTYPE_BF16 ? 8 : 16;
    RHZ_TRY(check_ptr(workspace, "workspace", 256, true));
    RHZ_TRY(check_ptr(q, "q", vec, true));
    RHZ_TRY(check_ptr(k, "k", vec, true));
    RHZ_TRY(check_ptr(v, "v", vec, true));
    RHZ_TRY(check_ptr(d_o, "d_o", vec, true));
    RHZ_TRY(check_ptr(dq, "dq", vec, true));
    RHZ_TRY(check_ptr(dk, "dk", vec, true));
    RHZ_TRY(check_ptr(dv, "dv", vec, true));
    RHZ_TRY(check_ptr(alpha, "alpha", 4, true));
    RHZ_TRY(check_ptr(beta, "beta", 4, true));
    RHZ_TRY(check_ptr(dalpha, "dalpha", 4, true));
    RHZ_TRY(check_ptr(dbeta, "dbeta", 4, true));
    RHZ_TRY(check_ptr(segment, "segment", 8, segment != nullptr));
    RHZ_TRY(check_ptr(d_state_final, "d_state_final", 16, d_state_final != nullptr));
    RHZ_TRY(require_sm100());
    BwdArgs a{dq, dk, dv, dalpha, dbeta, q, k, v, d_o, alpha, beta, segment, d_state_final,
              workspace, B, T, H, d, dtype, as_cuda(stream)};
    return launch_bwd(a);
}

int rhz_groupnorm_heads(void *out, const void *x, const float *scale, int64_t rows, int32_t H,
                        int32_t d, float eps, int32_t dtype, rhz_stream_t stream) {
    clear_error();
    RHZ_TRY(check_dtype(dtype));
    if (rows < 0 || H < 1 || d < 4 || d > 512 || d % 4)
        return set_error(RHZ_ERR_SHAPE, "groupnorm_heads needs rows >= 0, H >= 1, d a multiple of 4 in [4, 512] (got %lld, %d, %d)",
                         (long long)rows, H, d);
    if (!(eps >= 0.f)) return set_error(RHZ_ERR_INVALID, "eps must be >= 0");
    if (rows * H > (int64_t)INT32_MAX * 8) return set_error(RHZ_ERR_SHAPE, "rows*H exceeds the grid");
    if (rows == 0) return RHZ_OK;
    const size_t vec = dtype == RHZ_DTYPE_BF16 ? 8 : 16;
    RHZ_TRY(check_ptr(out, "out", vec, true));
    RHZ_TRY(check_ptr(x, "x", vec, true));
    RHZ_TRY(check_ptr(scale, "scale", 16, true));
    RHZ_TRY(require_sm100());
    return launch_groupnorm_heads(out, x, scale, rows, H, d, eps, dtype, as_cuda(stream));
}

size_t rhz_gdr_workspace_bytes(int64_t B, int64_t T, int32_t H, int32_t d, int32_t dtype,
                               int has_segment) {
    if (B < 0 || T < 0 || H < 1 || d < 1) return 0;
    return seg_ws(B, T, H, d, dtype, has_segment != 0).total;
}

int rhz_varlen_prefix_sum(int32_t *cu_seqlens, const int32_t *lengths, int64_t n,
                          rhz_stream_t stream) {
    clear_error();
    if (n < 0) return set_error(RHZ_ERR_SHAPE, "n = %lld: must be >= 0", (long long)n);
    RHZ_TRY(check_ptr(cu_seqlens, "cu_seqlens", 4, true));
    RHZ_TRY(check_ptr(lengths, "lengths", 4, n > 0));
    RHZ_TRY(require_sm100());
    return launch_prefix_sum(cu_seqlens, lengths, n, as_cuda(stream));
}

int rhz_varlen_segments_to_cu_seqlens(int32_t *cu_seqlens, int32_t *n_seg_out,
                                      const int64_t *segment, int64_t B, int64_t T,
                                      void *workspace, size_t workspace_bytes,
                                      rhz_stream_t stream) {
    clear_error();
    if (B < 0 || T < 0) return set_error(RHZ_ERR_SHAPE, "B = %lld, T = %lld: must be >= 0", (long long)B, (long long)T);
    if (B * T > INT32_MAX - 1) return set_error(RHZ_ERR_SHAPE, "B*T exceeds int32 offsets");
    RHZ_TRY(check_ptr(cu_seqlens, "cu_seqlens", 4, true));
    RHZ_TRY(check_ptr(n_seg_out, "n_seg_out", 4, true));
    RHZ_TRY(check_ptr(segment, "segment", 8, B * T > 0));
    RHZ_TRY(require_sm100());
    return launch_segments_to_cu(cu_seqlens, n_seg_out, segment, B, T, workspace, workspace_bytes,
                                 as_cuda(stream));
}

int rhz_varlen_chunk_map(int32_t *chunk_seq, int32_t *chunk_start, int32_t *n_chunks_out,
                         const int32_t *cu_seqlens, int64_t n_seq, int32_t chunk,
                         int64_t max_chunks, void *workspace, size_t workspace_bytes,
                         rhz_stream_t stream) {
    clear_error();
    if (n_seq < 0 || max_chunks < 0) return set_error(RHZ_ERR_SHAPE, "negative size");
    if (chunk < 1) return set_error(RHZ_ERR_SHAPE, "chunk = %d: must be >= 1", chunk);
    RHZ_TRY(check_ptr(n_chunks_out, "n_chunks_out", 4, true));
    RHZ_TRY(check_ptr(cu_seqlens, "cu_seqlens", 4, n_seq > 0));
    RHZ_TRY(check_ptr(chunk_seq, "chunk_seq", 4, max_chunks > 0));
    RHZ_TRY(check_ptr(chunk_start, "chunk_start", 4, max_chunks > 0));
    RHZ_TRY(require_sm100());
    return launch_chunk_map(chunk_seq, chunk_start, n_chunks_out, cu_seqlens, n_seq, chunk,
                            max_chunks, workspace, workspace_bytes, as_cuda(stream));
}

size_t rhz_varlen_workspace_bytes(int64_t n) { return varlen_ws_bytes(n); }

int rhz_varlen_gather_states(float *dense, const float *pool, const int32_t *slot_idx,
                             int64_t n, int64_t num_slots, int32_t H, int32_t d,
                             rhz_stream_t stream) {
    clear_error();
    RHZ_TRY(check_heads(H, d));
    if (n < 0 || num_slots < 0) return set_error(RHZ_ERR_SHAPE, "negative size");
    if (slot_idx == nullptr && n > num_slots) return set_error(RHZ_ERR_SHAPE, "n > num_slots with slot_idx NULL");
    RHZ_TRY(check_ptr(dense, "dense", 4, n > 0));
    RHZ_TRY(check_ptr(pool, "pool", 4, n > 0));
    RHZ_TRY(require_sm100());
    return launch_gather_states(dense, pool, slot_idx, n, num_slots, H, d, false, as_cuda(stream));
}

int rhz_varlen_scatter_states(float *pool, const float *dense, const int32_t *slot_idx,
                              int64_t n, int64_t num_slots, int32_t H, int32_t d,
                              rhz_stream_t stream) {
    clear_error();
    RHZ_TRY(check_heads(H, d));
    if (n < 0 || num_slots < 0) return set_error(RHZ_ERR_SHAPE, "negative size");
    if (slot_idx == nullptr && n > num_slots) return set_error(RHZ_ERR_SHAPE, "n > num_slots with slot_idx NULL");
    RHZ_TRY(check_ptr(dense, "dense", 4, n > 0));
    RHZ_TRY(check_ptr(pool, "pool", 4, n > 0));
    RHZ_TRY(require_sm100());
    return launch_gather_states(const_cast<float *>(dense), pool, slot_idx, n, num_slots, H, d,
                                true, as_cuda(stream));
}

int rhz_varlen_pack_tokens(void *packed, const void *padded, const int32_t *cu_seqlens,
                           int64_t n, int64_t max_len, int64_t row_bytes, rhz_stream_t stream) {
    clear_error();
    if (n < 0 || max_len < 0 || row_bytes < 0) return set_error(RHZ_ERR_SHAPE, "negative size");
    if (row_bytes % 4) return set_error(RHZ_ERR_SHAPE, "row_bytes = %lld: must be a multiple of 4", (long long)row_bytes);
    RHZ_TRY(check_ptr(packed, "packed", 4, n > 0));
    RHZ_TRY(check_ptr(padded, "padded", 4, n > 0));
    RHZ_TRY(check_ptr(cu_seqlens, "cu_seqlens", 4, n > 0));
    RHZ_TRY(require_sm100());
    return launch_pack_tokens(packed, padded, cu_seqlens, n, max_len, row_bytes, false, as_cuda(stream));
}

int rhz_varlen_unpack_tokens(void *padded, const void *packed, const int32_t *cu_seqlens,
                             int64_t n, int64_t max_len, int64_t row_bytes, rhz_stream_t stream) {
    clear_error();
    if (n < 0 || max_len < 0 || row_bytes < 0) return set_error(RHZ_ERR_SHAPE, "negative size");
    if (row_bytes % 4) return set_error(RHZ_ERR_SHAPE, "row_bytes = %lld: must be a multiple of 4", (long long)row_bytes);
    RHZ_TRY(check_ptr(packed, "packed", 4, n > 0));
    RHZ_TRY(check_ptr(padded, "padded", 4, n > 0));
    RHZ_TRY(check_ptr(cu_seqlens, "cu_seqlens", 4, n > 0));
    RHZ_TRY(require_sm100());
    return launch_pack_tokens(padded, packed, cu_seqlens, n, max_len, row_bytes, true, as_cuda(stream));
}

int rhz_gdr_multistep(void *outs, float *states, const float *state_pool,
                      const int32_t *slot_idx, const void *q, const void *k, const void *v,
                      const float *alpha, const float *beta, const int64_t *segment, int64_t n,
                      int64_t T, int64_t max_positions, int64_t num_slots, int32_t H, int32_t d,
                      int32_t dtype, rhz_stream_t stream) {
    clear_error();
    RHZ_TRY(check_dtype(dtype));
    RHZ_TRY(check_heads(H, d));
    if (n < 0 || T < 0 || max_positions < 0 || num_slots < 0)
        return set_error(RHZ_ERR_SHAPE, "negative size (n %lld, T %lld, max_positions %lld, num_slots %lld)",
                         (long long)n, (long long)T, (long long)max_positions, (long long)num_slots);
    const int64_t Tn = T < max_positions ? T : max_positions;
    if (Tn > 64) return set_error(RHZ_ERR_SHAPE, "multistep handles at most 64 positions per call (got %lld)", (long long)Tn);
    if (state_pool && slot_idx == nullptr && n > num_slots)
        return set_error(RHZ_ERR_SHAPE, "n = %lld sequences but only %lld slots (slot_idx is NULL)", (long long)n, (long long)num_slots);
    if (n * H > INT32_MAX) return set_error(RHZ_ERR_SHAPE, "n*H exceeds the grid");
    if (n == 0 || Tn == 0) return RHZ_OK;
    RHZ_TRY(check_ptr(q, "q", 16, true));
    RHZ_TRY(check_ptr(k, "k", 16, true));
    RHZ_TRY(check_ptr(v, "v", 16, true));
    RHZ_TRY(check_ptr(outs, "outs", 16, true));
    RHZ_TRY(check_ptr(states, "states", 16, true));
    RHZ_TRY(check_ptr(alpha, "alpha", 4, true));
    RHZ_TRY(check_ptr(beta, "beta", 4, true));
    RHZ_TRY(check_ptr(state_pool, "state_pool", 16, state_pool != nullptr));
    RHZ_TRY(check_ptr(slot_idx, "slot_idx", 4, slot_idx != nullptr));
    RHZ_TRY(check_ptr(segment, "segment", 8, segment != nullptr));
    RHZ_TRY(require_sm100());
    MultistepArgs a{outs, states, state_pool, slot_idx, q, k, v, alpha, beta, segment, n, T,
                    static_cast<int>(Tn), num_slots, H, d, dtype, as_cuda(stream)};
    return launch_multistep(a);
}

int rhz_gdr_prep(void *q, void *k, void *v, float *alpha, float *beta, const void *xq,
                 const void *xk, const void *xv, const float *beta_logit, const float *alpha_logit,
                 const float *a_head, const float *conv_w, const float *conv_b, float *conv_state,
                 const int32_t *slot_idx, const int32_t *cu_seqlens, int64_t n_seq,
                 int64_t seq_len, int64_t total_tokens, int64_t num_slots, int32_t H, int32_t d,
                 float q_scale, int32_t dtype, uint32_t flags, rhz_stream_t stream) {
    clear_error();
    RHZ_TRY(check_dtype(dtype));
    if (H < 1 || d < 4 || d > 512 || d % 4)
        return set_error(RHZ_ERR_SHAPE, "prep needs H >= 1 and d a multiple of 4 in [4, 512] (got H %d, d %d)", H, d);
    if (n_seq < 0 || seq_len < 0 || total_tokens < 0 || num_slots < 0)
        return set_error(RHZ_ERR_SHAPE, "negative size (n_seq %lld, seq_len %lld, total_tokens %lld, num_slots %lld)",
                         (long long)n_seq, (long long)seq_len, (long long)total_tokens, (long long)num_slots);
    if (flags & ~(RHZ_FLAG_ZERO_INIT | RHZ_FLAG_NO_STATE_WRITE))
        return set_error(RHZ_ERR_INVALID, "unknown flags 0x%x", flags);
    if (cu_seqlens == nullptr) total_tokens = n_seq * seq_len;
    if (conv_state && slot_idx == nullptr && n_seq > num_slots)
        return set_error(RHZ_ERR_SHAPE, "n_seq = %lld sequences but only %lld conv-state slots (slot_idx is NULL)",
                         (long long)n_seq, (long long)num_slots);
    if (total_tokens * H > (int64_t)INT32_MAX * 8) return set_error(RHZ_ERR_SHAPE, "tokens*H exceeds the grid");
    if (n_seq == 0 || total_tokens == 0) {
        if (n_seq == 0 || conv_state == nullptr || (flags & RHZ_FLAG_NO_STATE_WRITE)) return RHZ_OK;
    }
    const size_t vec = dtype == RHZ_DTYPE_BF16 ? 8 : 16;
    const bool rows = total_tokens > 0;
    RHZ_TRY(check_ptr(q, "q", vec, rows));
    RHZ_TRY(check_ptr(k, "k", vec, rows));
    RHZ_TRY(check_ptr(v, "v", vec, rows));
    RHZ_TRY(check_ptr(xq, "xq", vec, rows));
    RHZ_TRY(check_ptr(xk, "xk", vec, rows));
    RHZ_TRY(check_ptr(xv, "xv", vec, rows));
    RHZ_TRY(check_ptr(alpha, "alpha", 4, rows));
    RHZ_TRY(check_ptr(beta, "beta", 4, rows));
    RHZ_TRY(check_ptr(beta_logit, "beta_logit", 4, rows));
    RHZ_TRY(check_ptr(alpha_logit, "alpha_logit", 4, rows));
    RHZ_TRY(check_ptr(a_head, "a_head", 4, rows));
    RHZ_TRY(check_ptr(conv_w, "conv_w", 16, true));
    RHZ_TRY(check_ptr(conv_b, "conv_b", 16, true));
    RHZ_TRY(check_ptr(conv_state, "conv_state", 4, conv_state != nullptr));
    RHZ_TRY(check_ptr(slot_idx, "slot_idx", 4, slot_idx != nullptr));
    RHZ_TRY(check_ptr(cu_seqlens, "cu_seqlens", 4, cu_seqlens != nullptr));
    RHZ_TRY(require_sm100());
    PrepArgs a{q, k, v, alpha, beta, xq, xk, xv, beta_logit, alpha_logit, a_head, conv_w, conv_b,
               conv_state, slot_idx, cu_seqlens, n_seq, seq_len, total_tokens, num_slots, H, d, dtype,
               q_scale, (flags & RHZ_FLAG_ZERO_INIT) != 0, conv_state != nullptr && !(flags & RHZ_FLAG_NO_STATE_WRITE),
               as_cuda(stream)};
    return launch_prep(a);
}

int rhz_heads_unshard(void *out, const void *gathered, int64_t G, int64_t tokens, int32_t H,
                      int32_t d, int32_t elem_bytes, rhz_stream_t stream) {
    clear_error();
    if (G < 1 || tokens < 0 || H < 1 || d < 1) return set_error(RHZ_ERR_SHAPE, "bad sizes (G %lld, tokens %lld, H %d, d %d)", (long long)G, (long long)tokens, H, d);
    if (H % G) return set_error(RHZ_ERR_SHAPE, "H = %d heads do not split evenly over G = %lld ranks", H, (long long)G);
    if (elem_bytes != 2 && elem_bytes != 4) return set_error(RHZ_ERR_DTYPE, "elem_bytes = %d (expected 2 or 4)", elem_bytes);
    const int64_t row_bytes = static_cast<int64_t>(d) * elem_bytes;
    if ((H / G) * row_bytes % 4) return set_error(RHZ_ERR_SHAPE, "a rank's rows (%lld bytes) are not a multiple of 4 bytes", (long long)((H / G) * row_bytes));
    RHZ_TRY(check_ptr(out, "out", 16, tokens > 0));
    RHZ_TRY(check_ptr(gathered, "gathered", 16, tokens > 0));
    RHZ_TRY(require_sm100());
    return launch_heads_unshard(out, gathered, G, tokens, H / G, row_bytes, false, as_cuda(stream));
}

int rhz_heads_shard(void *gathered, const void *full, int64_t G, int64_t tokens, int32_t H,
                    int32_t d, int32_t elem_bytes, rhz_stream_t stream) {
    clear_error();
    if (G < 1 || tokens < 0 || H < 1 || d < 1) return set_error(RHZ_ERR_SHAPE, "bad sizes (G %lld, tokens %lld, H %d, d %d)", (long long)G, (long long)tokens, H, d);
    if (H % G) return set_error(RHZ_ERR_SHAPE, "H = %d heads do not split evenly over G = %lld ranks", H, (long long)G);
    if (elem_bytes != 2 && elem_bytes != 4) return set_error(RHZ_ERR_DTYPE, "elem_bytes = %d (expected 2 or 4)", elem_bytes);
    const int64_t row_bytes = static_cast<int64_t>(d) * elem_bytes;
    if ((H / G) * row_bytes % 4) return set_error(RHZ_ERR_SHAPE, "a rank's rows (%lld bytes) are not a multiple of 4 bytes", (long long)((H / G) * row_bytes));
    RHZ_TRY(check_ptr(full, "full", 16, tokens > 0));
    RHZ_TRY(check_ptr(gathered, "gathered", 16, tokens > 0));
    RHZ_TRY(require_sm100());
    return launch_heads_unshard(gathered, full, G, tokens, H / G, row_bytes, true, as_cuda(stream));
}

}  // extern "C"

// ------------------------------------------------------------------------
// Host-buffer chunked scan: the reference signature with every tensor in
// host memory, pipelined over slabs of positions so that the host->device
// copies of slab j+1, the scan of slab j and the device->host copy of slab
// j-1 overlap.
namespace {

constexpr int kHostSets = 3;  // buffer sets in flight

struct HostPlan {
    int64_t slab;      // positions per slab (multiple of 64)
    int64_t n_slabs;
    int64_t max_pieces;
    size_t tok_bytes, gate_bytes, state_bytes, set_bytes;
    size_t q_off, k_off, v_off, o_off, a_off, b_off;  // within a set
    size_t pools_off, gates_off, gates_bytes, meta_off, grid_off, grid_bytes, total;
};

HostPlan host_plan(int64_t B, int64_t T, int32_t H, int32_t d, int32_t dtype, bool has_segment) {
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    HostPlan p{};
    const int64_t t64 = (T + 63) / 64 * 64;
    const int64_t eighth = ((T + 7) / 8 + 63) / 64 * 64;
    p.slab = std::min<int64_t>(t64, std::max<int64_t>(256, eighth));
    if (p.slab < 64) p.slab = 64;
    p.n_slabs = T > 0 ? (T + p.slab - 1) / p.slab : 0;
    p.max_pieces = B * p.n_slabs + (has_segment ? B * T : 0);
    const size_t esz = dtype == RHZ_DTYPE_BF16 ? 2 : 4;
    const size_t rows = static_cast<size_t>(B) * p.slab * H;
    p.tok_bytes = up(rows * d * esz);
    p.gate_bytes = up(rows * sizeof(float));
    p.q_off = 0;
    p.k_off = p.tok_bytes;
    p.v_off = 2 * p.tok_bytes;
    p.o_off = 3 * p.tok_bytes;
    p.a_off = 4 * p.tok_bytes;
    p.b_off = 4 * p.tok_bytes + p.gate_bytes;
    p.set_bytes = 4 * p.tok_bytes + 2 * p.gate_bytes;
    p.state_bytes = up(static_cast<size_t>(B) * H * d * d * sizeof(float));
    p.pools_off = kHostSets * p.set_bytes;
    p.gates_bytes = up(static_cast<size_t>(B) * T * H * sizeof(float));
    p.gates_off = p.pools_off + 2 * p.state_bytes;
    p.meta_off = p.gates_off + 2 * p.gates_bytes;
    // per slab: row offsets (B + 1), piece offsets (pieces + 1), in slots,
    // out slots
    p.grid_off = p.meta_off + up((3 * static_cast<size_t>(p.max_pieces) +
                                  p.n_slabs * static_cast<size_t>(B + 2)) * sizeof(int32_t));
    // the tensor-core kernel's scratch, shared by the slabs (one scan at a time)
    p.grid_bytes = chunk_tc_supports(d, dtype) ? up(chunk_grid_ws_bytes(p.max_pieces * H, true)) : 0;
    p.total = p.grid_off + p.grid_bytes;
    return p;
}

// One slab's pieces: batch row b's positions [t0, t0 + len) split where the
// segment id changes. A piece continues row b's carried state when it starts
// the slab inside the same segment as the previous slab's last position
// (slot b of the previous pool), else starts from zero (slot -1: the reset
// at t = 0 and at segment changes, delta.rs:139-141); the last piece of a
// row writes slot b of the next pool.
void slab_pieces(const int64_t *seg, int64_t B, int64_t T, int64_t t0, int64_t len,
                 std::vector<int32_t> &cu, std::vector<int32_t> &in, std::vector<int32_t> &out) {
    cu.push_back(0);
    for (int64_t b = 0; b < B; ++b) {
        const int64_t *sr = seg ? seg + b * T : nullptr;
        const int32_t base = static_cast<int32_t>(b * len);
        int64_t start = t0;
        auto emit = [&](int64_t s, int64_t e) {
            cu.push_back(base + static_cast<int32_t>(e - t0));
            const bool carry = s == t0 && t0 > 0 && (sr == nullptr || sr[t0] == sr[t0 - 1]);
            in.push_back(carry ? static_cast<int32_t>(b) : -1);
            out.push_back(e == t0 + len ? static_cast<int32_t>(b) : -1);
        };
        if (sr) {
            for (int64_t t = t0 + 1; t < t0 + len; ++t) {
                if (sr[t] != sr[t - 1]) {
                    emit(start, t);
                    start = t;
                }
            }
        }
        emit(start, t0 + len);
    }
}

// Copy streams and events of the host-buffer entry point, created on a
// device's first call and kept for the process (creating and destroying them
// per call cost ~0.2 ms). Calls on one device take the mutex in turn.
struct HostStreams {
    std::mutex m;
    bool ready = false;
    cudaStream_t up = nullptr, down = nullptr;
    cudaEvent_t start = nullptr, in[kHostSets] = {}, comp[kHostSets] = {}, out[kHostSets] = {};
    cudaError_t create() {
        if (ready) return cudaSuccess;
        cudaError_t e = cudaStreamCreateWithFlags(&up, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&down, cudaStreamNonBlocking);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&start, cudaEventDisableTiming);
        for (int i = 0; i < kHostSets && e == cudaSuccess; ++i) {
            e = cudaEventCreateWithFlags(&in[i], cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&comp[i], cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&out[i], cudaEventDisableTiming);
        }
        ready = e == cudaSuccess;
        return e;
    }
};
HostStreams g_host[64];

// Rows [t0, t0 + len) of every batch row of a [B][T][row_bytes] host array
// into (or out of) a packed [B][len][row_bytes] device buffer.
cudaError_t copy_slab(void *dst, const void *src, int64_t B, int64_t T, int64_t t0, int64_t len,
                      size_t row_bytes, bool to_device, cudaStream_t s) {
    if (to_device)
        return cudaMemcpy2DAsync(dst, len * row_bytes,
                                 static_cast<const char *>(src) + t0 * row_bytes, T * row_bytes,
                                 len * row_bytes, B, cudaMemcpyHostToDevice, s);
    return cudaMemcpy2DAsync(static_cast<char *>(dst) + t0 * row_bytes, T * row_bytes, src,
                             len * row_bytes, len * row_bytes, B, cudaMemcpyDeviceToHost, s);
}

}  // namespace

extern "C" {

size_t rhz_gdr_host_workspace_bytes(int64_t B, int64_t T, int32_t H, int32_t d, int32_t dtype,
                                    int has_segment) {
    if (B < 0 || T < 0 || H < 1 || d < 1 || (dtype != RHZ_DTYPE_F32 && dtype != RHZ_DTYPE_BF16))
        return 0;
    return host_plan(B, T, H, d, dtype, has_segment != 0).total;
}

int rhz_gdr_scan_chunked_host(void *o, float *state_final, const void *q, const void *k,
                              const void *v, const float *alpha, const float *beta,
                              const int64_t *segment, const float *state_init, int64_t chunk,
                              int64_t B, int64_t T, int32_t H, int32_t d, int32_t dtype,
                              void *workspace, size_t workspace_bytes, rhz_stream_t stream) {
    clear_error();
    if (chunk < 0) return set_error(RHZ_ERR_SHAPE, "chunk = %lld: must be >= 0", (long long)chunk);
    RHZ_TRY(check_dtype(dtype));
    RHZ_TRY(check_heads(H, d));
    if (B < 0 || T < 0) return set_error(RHZ_ERR_SHAPE, "B = %lld, T = %lld: must be >= 0", (long long)B, (long long)T);
    if (B * T > INT32_MAX - 1) return set_error(RHZ_ERR_SHAPE, "B*T = %lld positions exceeds int32 indexing", (long long)(B * T));
    const bool any = B * T > 0;
    for (const void *p : {static_cast<const void *>(o), q, k, v, static_cast<const void *>(alpha),
                          static_cast<const void *>(beta)})
        if (any && p == nullptr) return set_error(RHZ_ERR_INVALID, "a host tensor (q, k, v, alpha, beta or o) is NULL");
    const size_t state_elems = static_cast<size_t>(B) * H * d * d;
    if (T == 0) {
        // The loop never runs: the reference returns init.clone() (delta.rs:135).
        if (state_final && state_elems) {
            if (state_init) memcpy(state_final, state_init, state_elems * sizeof(float));
            else memset(state_final, 0, state_elems * sizeof(float));
        }
        return RHZ_OK;
    }
    if (B == 0) return RHZ_OK;
    if (B > 65535) return set_error(RHZ_ERR_SHAPE, "B = %lld: the host-buffer entry point takes at most 65535 batch rows", (long long)B);
    const HostPlan pl = host_plan(B, T, H, d, dtype, segment != nullptr);
    if (workspace == nullptr || workspace_bytes < pl.total)
        return set_error(RHZ_ERR_INVALID, "workspace too small: need %zu bytes, got %zu", pl.total, workspace_bytes);
    RHZ_TRY(check_ptr(workspace, "workspace", 256, true));
    RHZ_TRY(require_sm100());

    // Every slab's pieces, built on the host and sent in one copy.
    std::vector<int32_t> meta;
    std::vector<int64_t> rows_at(pl.n_slabs), cu_at(pl.n_slabs), in_at(pl.n_slabs),
        out_at(pl.n_slabs), pieces(pl.n_slabs);
    {
        std::vector<int32_t> cu, in, out;
        for (int64_t j = 0; j < pl.n_slabs; ++j) {
            const int64_t t0 = j * pl.slab, len = std::min(pl.slab, T - t0);
            rows_at[j] = static_cast<int64_t>(meta.size());
            for (int64_t b = 0; b <= B; ++b) meta.push_back(static_cast<int32_t>(b * len));
            cu.clear(); in.clear(); out.clear();
            slab_pieces(segment, B, T, t0, len, cu, in, out);
            pieces[j] = static_cast<int64_t>(in.size());
            cu_at[j] = static_cast<int64_t>(meta.size());
            meta.insert(meta.end(), cu.begin(), cu.end());
            in_at[j] = static_cast<int64_t>(meta.size());
            meta.insert(meta.end(), in.begin(), in.end());
            out_at[j] = static_cast<int64_t>(meta.size());
            meta.insert(meta.end(), out.begin(), out.end());
        }
    }
    char *ws = static_cast<char *>(workspace);
    int32_t *dmeta = reinterpret_cast<int32_t *>(ws + pl.meta_off);
    float *pool[2] = {reinterpret_cast<float *>(ws + pl.pools_off),
                      reinterpret_cast<float *>(ws + pl.pools_off + pl.state_bytes)};
    float *galpha = reinterpret_cast<float *>(ws + pl.gates_off);
    float *gbeta = reinterpret_cast<float *>(ws + pl.gates_off + pl.gates_bytes);
    const size_t esz = dtype == RHZ_DTYPE_BF16 ? 2 : 4;
    const size_t tok_row = static_cast<size_t>(H) * d * esz, gate_row = static_cast<size_t>(H) * sizeof(float);
    cudaStream_t cs = as_cuda(stream);

    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= 64)
        return set_error(RHZ_ERR_DEVICE, "cudaGetDevice: %s", cudaGetErrorString(e));
    HostStreams &hs = g_host[dev];
    std::lock_guard<std::mutex> lock(hs.m);
    e = hs.create();
    if (e == cudaSuccess) e = cudaEventRecord(hs.start, cs);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(hs.up, hs.start, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(hs.down, hs.start, 0);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(dmeta, meta.data(), meta.size() * sizeof(int32_t), cudaMemcpyHostToDevice, hs.up);
    // The gates are small: both whole arrays go in first, in two copies, and
    // each slab's rows are packed on the device. (Per-slab gate copies either
    // queued their fixed cost into the token stream or, on a copy stream of
    // their own, waited up to a millisecond for the copy engine.)
    const size_t gate_all = static_cast<size_t>(B) * T * H * sizeof(float);
    if (e == cudaSuccess) e = cudaMemcpyAsync(galpha, alpha, gate_all, cudaMemcpyHostToDevice, hs.up);
    if (e == cudaSuccess) e = cudaMemcpyAsync(gbeta, beta, gate_all, cudaMemcpyHostToDevice, hs.up);
    int st = RHZ_OK;
    for (int64_t j = 0; j < pl.n_slabs && e == cudaSuccess && st == RHZ_OK; ++j) {
        const int set = static_cast<int>(j % kHostSets);
        char *buf = ws + set * pl.set_bytes;
        const int64_t t0 = j * pl.slab, len = std::min(pl.slab, T - t0);
        // inputs of slab j (after the scan of slab j - kHostSets released the set)
        if (j >= kHostSets) e = cudaStreamWaitEvent(hs.up, hs.comp[set], 0);
        if (e == cudaSuccess) e = copy_slab(buf + pl.q_off, q, B, T, t0, len, tok_row, true, hs.up);
        if (e == cudaSuccess) e = copy_slab(buf + pl.k_off, k, B, T, t0, len, tok_row, true, hs.up);
        if (e == cudaSuccess) e = copy_slab(buf + pl.v_off, v, B, T, t0, len, tok_row, true, hs.up);
        if (e == cudaSuccess) e = cudaEventRecord(hs.in[set], hs.up);
        // the scan of slab j (after its inputs landed and slab j - kHostSets's
        // output left the set)
        if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, hs.in[set], 0);
        if (e == cudaSuccess && j >= kHostSets) e = cudaStreamWaitEvent(cs, hs.out[set], 0);
        if (e != cudaSuccess) break;
        st = launch_pack_tokens(buf + pl.a_off, galpha + t0 * H, dmeta + rows_at[j], B, T, gate_row,
                                false, cs);
        if (st == RHZ_OK)
            st = launch_pack_tokens(buf + pl.b_off, gbeta + t0 * H, dmeta + rows_at[j], B, T,
                                    gate_row, false, cs);
        if (st != RHZ_OK) break;
        SeqArgs a{};
        a.o = buf + pl.o_off;
        a.q = buf + pl.q_off; a.k = buf + pl.k_off; a.v = buf + pl.v_off;
        a.alpha = reinterpret_cast<const float *>(buf + pl.a_off);
        a.beta = reinterpret_cast<const float *>(buf + pl.b_off);
        a.cu_seqlens = dmeta + cu_at[j];
        a.n_seq = pieces[j];
        a.total_tokens = B * len;
        a.state_in = j > 0 ? pool[(j - 1) & 1] : nullptr;
        a.in_slots = dmeta + in_at[j];
        a.state_out = pool[j & 1];
        a.out_slots = dmeta + out_at[j];
        a.num_slots = B;
        a.H = H; a.d = d; a.dtype = dtype; a.stream = cs;
        a.ws = pl.grid_bytes ? ws + pl.grid_off : nullptr;
        a.ws_bytes = pl.grid_bytes;
        st = run_seq(a);
        if (st != RHZ_OK) break;
        e = cudaEventRecord(hs.comp[set], cs);
        // output of slab j
        if (e == cudaSuccess) e = cudaStreamWaitEvent(hs.down, hs.comp[set], 0);
        if (e == cudaSuccess) e = copy_slab(o, buf + pl.o_off, B, T, t0, len, tok_row, false, hs.down);
        if (e == cudaSuccess) e = cudaEventRecord(hs.out[set], hs.down);
    }
    if (e == cudaSuccess && st == RHZ_OK && state_final)
        e = cudaMemcpyAsync(state_final, pool[(pl.n_slabs - 1) & 1], state_elems * sizeof(float),
                            cudaMemcpyDeviceToHost, hs.down);
    // The call returns with every output in host memory (and with the copy
    // streams idle, also on an error path).
    const cudaError_t e2 = cudaStreamSynchronize(hs.down);
    const cudaError_t e3 = cudaStreamSynchronize(cs);
    cudaStreamSynchronize(hs.up);
    if (st != RHZ_OK) return st;
    if (e == cudaSuccess) e = e2 != cudaSuccess ? e2 : e3;
    if (e != cudaSuccess) return set_error(RHZ_ERR_DEVICE, "host-buffer scan: %s", cudaGetErrorString(e));
    return RHZ_OK;
}

}  // extern "C"
