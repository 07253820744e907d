// Chunked gated delta-rule prefill on the sm_100a tensor cores (bf16 inputs,
// fp32 state and accumulation), d_k = d_v = 128, chunk C = 64.
//
// Math (per sequence and head; S is d_v x d_k, row i = v index): inside a
// chunk of positions t = 0..C-1 that starts from state S0,
//   P[t][s] = prod_{r=s+1..t} alpha_r (s <= t),  gamma_t = prod_{r=0..t} alpha_r
//   A[t][s] = beta_t P[t][s] (k_t . k_s) for s < t, T = (I + A)^-1
//   U = T diag(beta) V,  W = T diag(beta gamma) K,  Delta = U - W S0^T
//   O[t] = gamma_t S0 q_t + sum_{s<=t} P[t][s] (q_t . k_s) Delta_s
//   S_C = gamma_{C-1} S0 + sum_s P[C-1][s] Delta_s k_s^T
// which equals C applications of gated_delta_step (crates/ops/src/delta.rs:
// 93-127): S_t = alpha_t S_{t-1} + Delta_t k_t^T with
// Delta_t = beta_t (v_t - alpha_t S_{t-1} k_t). Decays are products of alphas
// (never exp of a difference of large logs, never division by a decay), so
// alpha = 0 and deep underflow are exact.
//
// All products are M = 128 tcgen05 MMAs with the d dimension on M, so every
// accumulator row maps to one TMEM lane and one thread (thread i <-> lane i):
//   D1   = [K; Q] K^T          (128 x 64, K = d)     -> A (fp32 smem) and masked M
//   D_U  = V^T (T diag b)^T    (128 x 64, K = C)
//   D_W  = K^T (T diag bg)^T   (128 x 64, K = C)     -> -W^T (fp16 smem)
//   D_SQ = S0 Q^T              (128 x 64, K = d)
//   D_U += S0 (-W^T)           (128 x 64, K = d)     -> Delta^T (fp16 smem)
//   D_O2 = Delta^T M^T         (128 x 64, K = C)
//   D_S += (P[C-1] Delta)^T K  (128 x 128, K = C)    (D_S pre-scaled by gamma_{C-1})
// The 64 x 64 unit-lower-triangular inverse is done in fp32 on the SIMT
// cores (blocked 16 x 16). Q, K, V tiles arrive by TMA (128-byte swizzle,
// double-buffered one chunk ahead; no multicast). D1 consumes them as bf16;
// they are then converted to fp16 in place and every later product takes
// fp16 operands (A and B of one MMA always share a type): 3 more mantissa
// bits for T, W, Delta, M and the state copy than bf16 would give. The
// state stays in TMEM in fp32 for the whole sequence; an fp16 copy in shared
// memory feeds the MMAs. fp16 intermediates bound |q.k|, |v|, |S| to
// < 65504 (unit-norm keys, as the reference specifies, keep them far below).
//
// One CTA (128 threads, one warpgroup) per SM, persistent over
// (sequence, head) items. Every wait is bounded; a timeout sets a sticky
// device flag, drains in-flight copies and MMAs (bounded), frees TMEM and
// returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"

namespace rhz {

// Sticky per-device flag: set when a bounded device-side wait ran out.
__device__ int g_tc_status = 0;

namespace {
using namespace sm100;

constexpr int CH = 64;    // chunk length
constexpr int HD = 128;   // head dim (d_k = d_v)
constexpr int NT = 128;   // threads per CTA
constexpr int AST = 65;   // fp32 row stride of the A / T tables (bank spread)

// Shared memory map (offsets from a 1024-byte aligned base).
constexpr uint32_t OFF_KQ = 0;                     // 2 stages x 32 KB: [half][K rows | Q rows]
constexpr uint32_t KQ_STAGE = 32768;
constexpr uint32_t OFF_V = 65536;                  // 2 stages x 16 KB: [half][V rows]
constexpr uint32_t V_STAGE = 16384;
constexpr uint32_t OFF_S = 98304;                  // fp16 state [half][128 rows][64]
constexpr uint32_t OFF_TT = 131072;                // fp16 (T diag beta)        [t][s]
constexpr uint32_t OFF_TH = 139264;                // fp16 (T diag beta gamma)  [t][s]
constexpr uint32_t OFF_M = 147456;                 // fp16 masked decayed Q K^T [t][s]
constexpr uint32_t OFF_R = 155648;                 // 48 KB, phase-aliased region:
constexpr uint32_t OFF_WT = OFF_R;                 //   -W^T  [j][t] fp16 (16 KB)
constexpr uint32_t OFF_DT = OFF_R + 16384;         //   Delta^T [i][s] fp16 (16 KB)
constexpr uint32_t OFF_DTS = OFF_R + 32768;        //   (P[C-1] Delta)^T [i][s] fp16 (16 KB)
constexpr uint32_t OFF_AF = OFF_R;                 //   A fp32 [64][65]   (solve phase)
constexpr uint32_t OFF_TF = OFF_R + 64 * AST * 4;  //   T fp32 [64][65]
constexpr uint32_t OFF_XF = OFF_TF + 64 * AST * 4; //   3 x 16x16 fp32 scratch
constexpr uint32_t OFF_SMALL = OFF_R + 49152;      // alpha, beta, gamma, P[C-1][.] (4 x 64 f32)
constexpr uint32_t OFF_BAR = OFF_SMALL + 1024;     // 3 mbarriers + TMEM base address
constexpr uint32_t SMEM_USED = OFF_BAR + 64;
constexpr size_t SMEM_ALLOC = SMEM_USED + 1024;    // slack for 1024-byte alignment
static_assert(OFF_XF + 3 * 256 * 4 <= OFF_R + 49152, "solve scratch overflows its region");
static_assert(SMEM_ALLOC <= 232448, "exceeds the 227 KB opt-in shared memory");

// TMEM columns (f32 accumulators, 128 lanes each).
constexpr uint32_t TM_D1 = 0, TM_U = 64, TM_W = 128, TM_SQ = 192, TM_O2 = 256, TM_S = 320;
constexpr uint32_t TM_COLS = 512;

// D1 runs on the bf16 tiles as loaded; every later product runs in fp16
// (the tiles are converted in place after D1), 3 more mantissa bits than bf16.
constexpr uint32_t ID_D1 = idesc_bf16(128, 64, false, false);
constexpr uint32_t ID_KK64 = idesc_f16(128, 64, false, false);
constexpr uint32_t ID_MK64 = idesc_f16(128, 64, true, false);
constexpr uint32_t ID_KM64 = idesc_f16(128, 64, false, true);
constexpr uint32_t ID_KM128 = idesc_f16(128, 128, false, true);
constexpr uint32_t LOAD_BYTES = 6 * 8192;  // K, Q, V: two 64 x 64 bf16 boxes each

struct TcParams {
    __nv_bfloat16 *o;
    const float *alpha, *beta;
    const int32_t *cu_seqlens, *n_seq_dev;
    int64_t n_seq, seq_len, total_tokens;
    const float *state_in;
    const int32_t *in_slots;
    float *state_out;
    const int32_t *out_slots;
    int64_t num_slots;
    int H;
};

__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
}

// 64 values as fp16 into row `row` of a 128-byte-swizzled block of
// 128-byte rows (the canonical SWIZZLE_128B operand layout).
__device__ __forceinline__ void st_row64_f16(uint8_t *blk, uint32_t row, const float *v) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint4 w;
        w.x = pack_f16x2(v[8 * c + 0], v[8 * c + 1]);
        w.y = pack_f16x2(v[8 * c + 2], v[8 * c + 3]);
        w.z = pack_f16x2(v[8 * c + 4], v[8 * c + 5]);
        w.w = pack_f16x2(v[8 * c + 6], v[8 * c + 7]);
        *reinterpret_cast<uint4 *>(blk + sw128_offset(row, c)) = w;
    }
}

__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t x) {
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162 *>(&x);
    return pack_f16x2(__low2float(b), __high2float(b));
}

// K, Q (32 KB) and V (16 KB) tiles of one stage, bf16 -> fp16 in place (the
// swizzled layout is elementwise, so it is unchanged). bf16 values inside the
// fp16 normal range convert exactly.
__device__ __forceinline__ void tiles_to_f16(uint8_t *kq, uint8_t *vv, int tid) {
    for (int i = tid; i < 3072; i += NT) {
        uint4 *ptr = reinterpret_cast<uint4 *>(i < 2048 ? kq + i * 16 : vv + (i - 2048) * 16);
        uint4 w = *ptr;
        w.x = bf16x2_to_f16x2(w.x);
        w.y = bf16x2_to_f16x2(w.y);
        w.z = bf16x2_to_f16x2(w.z);
        w.w = bf16x2_to_f16x2(w.w);
        *ptr = w;
    }
}

__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
    tmem_ld32(taddr, *reinterpret_cast<float(*)[32]>(&v[0]));
    tmem_ld32(taddr + 32, *reinterpret_cast<float(*)[32]>(&v[32]));
}

// 64 x 64 unit lower triangular inverse T = (I + A)^-1 of a strictly lower A,
// fp32, blocked 4 x 4 in 16 x 16 tiles. All 128 threads; ends synchronised.
__device__ void solve_unit_lower(const float *Af, float *Tf, float *Xf, int tid) {
    // Diagonal tiles by forward substitution: thread (I, j) solves column j.
    if (tid < 64) {
        const int I = tid >> 4, j = tid & 15;
        const float *A = Af + (16 * I) * AST + 16 * I;
        float x[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            float acc = (r == j) ? 1.f : 0.f;
#pragma unroll
            for (int c = 0; c < r; ++c)
                if (c >= j) acc = fmaf(-A[r * AST + c], x[c], acc);
            x[r] = (r >= j) ? acc : 0.f;
        }
        float *T = Tf + (16 * I) * AST + 16 * I;
#pragma unroll
        for (int r = 0; r < 16; ++r) T[r * AST + j] = x[r];
    }
    // Tiles above the diagonal are zero.
    for (int idx = tid; idx < 6 * 256; idx += NT) {
        const int b = idx >> 8, e = idx & 255;
        const int I = b < 3 ? 0 : (b < 5 ? 1 : 2);
        const int J = b < 3 ? b + 1 : (b < 5 ? b - 1 : 3);
        Tf[(16 * I + (e >> 4)) * AST + 16 * J + (e & 15)] = 0.f;
    }
    __syncthreads();
    // Off-diagonal tiles by distance: T_IJ = -T_II sum_{K=J}^{I-1} A_IK T_KJ.
#pragma unroll 1
    for (int dist = 1; dist < 4; ++dist) {
        const int nb = 4 - dist;
        for (int idx = tid; idx < nb * 256; idx += NT) {
            const int b = idx >> 8, e = idx & 255, r = e >> 4, c = e & 15;
            const int I = b + dist, J = b;
            float acc = 0.f;
            for (int K = J; K < I; ++K) {
                const float *A = Af + (16 * I + r) * AST + 16 * K;
                const float *T = Tf + (16 * K) * AST + 16 * J + c;
#pragma unroll
                for (int kk = 0; kk < 16; ++kk) acc = fmaf(A[kk], T[kk * AST], acc);
            }
            Xf[b * 256 + e] = acc;
        }
        __syncthreads();
        for (int idx = tid; idx < nb * 256; idx += NT) {
            const int b = idx >> 8, e = idx & 255, r = e >> 4, c = e & 15;
            const int I = b + dist, J = b;
            const float *D = Tf + (16 * I + r) * AST + 16 * I;
            float acc = 0.f;
#pragma unroll
            for (int kk = 0; kk < 16; ++kk) acc = fmaf(D[kk], Xf[b * 256 + kk * 16 + c], acc);
            Tf[(16 * I + r) * AST + 16 * J + c] = -acc;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(NT, 1)
    gdr_chunk_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tid = threadIdx.x, warp = tid >> 5;
    float *sa = reinterpret_cast<float *>(smem + OFF_SMALL);
    float *sb = sa + 64, *sg = sa + 128, *spend = sa + 192;
    uint64_t *bar_load = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *bar_mma = bar_load + 2;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar_load + 3);
    float *Af = reinterpret_cast<float *>(smem + OFF_AF);
    float *Tf = reinterpret_cast<float *>(smem + OFF_TF);
    float *Xf = reinterpret_cast<float *>(smem + OFF_XF);
    const uint32_t sbase = smem_u32(smem);

    if (tid == 0) {
        mbar_init(&bar_load[0], 1);
        mbar_init(&bar_load[1], 1);
        mbar_init(bar_mma, 1);
        mbar_fence_init();
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_k);
        prefetch_tmap(&tm_v);
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, TM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);  // this thread's lane

    const int H = p.H;
    int64_t n_seq = p.n_seq;
    if (p.n_seq_dev) {
        const int64_t nd = *p.n_seq_dev;
        n_seq = nd < n_seq ? nd : n_seq;
    }
    const int64_t n_items = n_seq * H;
    const int64_t tok_stride = static_cast<int64_t>(H) * HD;

    uint32_t load_iter = 0;  // chunk tiles requested so far
    uint32_t mma_phase = 0;
    int pending_stage = -1;  // thread 0: a requested tile not yet consumed
    uint32_t pending_parity = 0;
    bool failed = false, mma_pending = false;

    auto issue_loads = [&](uint32_t iter, int64_t tok, int h) {
        const uint32_t st = iter & 1u;
        uint64_t *bar = &bar_load[st];
        uint8_t *kq = smem + OFF_KQ + st * KQ_STAGE;
        uint8_t *vv = smem + OFF_V + st * V_STAGE;
        mbar_arrive_expect_tx(bar, LOAD_BYTES);
        const int t32 = static_cast<int>(tok);
        tma_load_3d(kq, &tm_k, 0, h, t32, bar);
        tma_load_3d(kq + 16384, &tm_k, 64, h, t32, bar);
        tma_load_3d(kq + 8192, &tm_q, 0, h, t32, bar);
        tma_load_3d(kq + 24576, &tm_q, 64, h, t32, bar);
        tma_load_3d(vv, &tm_v, 0, h, t32, bar);
        tma_load_3d(vv + 8192, &tm_v, 64, h, t32, bar);
        pending_stage = static_cast<int>(st);
        pending_parity = (iter >> 1) & 1u;
    };
    // Commit the issued MMAs and wait for them on every thread.
    auto mma_sync = [&]() -> bool {
        if (tid == 0) umma_commit(bar_mma);
        mma_pending = true;
        const bool ok = mbar_wait(bar_mma, mma_phase);
        if (__syncthreads_or(!ok)) return false;
        mma_phase ^= 1u;
        mma_pending = false;
        tc_fence_after();
        return true;
    };
    // Make thread-written smem operands and TMEM stores visible to the MMA issuer.
    auto operands_ready = [&]() {
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    };

    for (int64_t item = blockIdx.x; item < n_items && !failed; item += gridDim.x) {
        const int64_t seq = item / H;
        const int h = static_cast<int>(item - seq * H);
        int64_t t0, t1;
        if (p.cu_seqlens) {
            // Offsets are caller data: clamp them to the packed stream.
            t0 = p.cu_seqlens[seq];
            t1 = p.cu_seqlens[seq + 1];
            t0 = t0 < 0 ? 0 : (t0 > p.total_tokens ? p.total_tokens : t0);
            t1 = t1 < t0 ? t0 : (t1 > p.total_tokens ? p.total_tokens : t1);
        } else {
            t0 = seq * p.seq_len;
            t1 = t0 + p.seq_len;
        }
        const int nch = static_cast<int>((t1 - t0 + CH - 1) / CH);

        // ---- initial state: row tid of S -> TMEM (fp32) and the fp16 copy
        {
            int64_t slot = -1;
            if (p.state_in) slot = p.in_slots ? static_cast<int64_t>(p.in_slots[seq]) : seq;
            const bool have = p.state_in && slot >= 0 && slot < p.num_slots;
            const float *src = have ? p.state_in + ((slot * H + h) * HD + tid) * HD : nullptr;
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
                float v[32];
#pragma unroll
                for (int e = 0; e < 32; e += 4) {
                    float4 f = have ? *reinterpret_cast<const float4 *>(src + 32 * q4 + e)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
                    v[e] = f.x; v[e + 1] = f.y; v[e + 2] = f.z; v[e + 3] = f.w;
                }
                tmem_st32(trow + TM_S + 32 * q4, v);
                // fp16 copy: columns 32*q4 .. +31 -> half q4/2, chunks (q4&1)*4 .. +3
                uint8_t *blk = smem + OFF_S + (q4 >> 1) * 16384;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    uint4 w;
                    w.x = pack_f16x2(v[8 * c + 0], v[8 * c + 1]);
                    w.y = pack_f16x2(v[8 * c + 2], v[8 * c + 3]);
                    w.z = pack_f16x2(v[8 * c + 4], v[8 * c + 5]);
                    w.w = pack_f16x2(v[8 * c + 6], v[8 * c + 7]);
                    *reinterpret_cast<uint4 *>(blk + sw128_offset(tid, (q4 & 1) * 4 + c)) = w;
                }
            }
            tmem_wait_st();
        }
        if (tid == 0 && nch > 0) issue_loads(load_iter, t0, h);
        operands_ready();

        for (int c = 0; c < nch; ++c) {
            const int64_t ts = t0 + static_cast<int64_t>(c) * CH;
            const int L = static_cast<int>((t1 - ts) < CH ? (t1 - ts) : CH);
            const uint32_t st = load_iter & 1u;
            const uint32_t lpar = (load_iter >> 1) & 1u;
            const uint32_t kq = sbase + OFF_KQ + st * KQ_STAGE;
            const uint32_t vb = sbase + OFF_V + st * V_STAGE;

            // Gates (padded rows: alpha = 1, beta = 0 -> they write nothing).
            if (tid < CH) {
                const bool in = tid < L;
                sa[tid] = in ? p.alpha[(ts + tid) * H + h] : 1.f;
                sb[tid] = in ? p.beta[(ts + tid) * H + h] : 0.f;
            }
            const bool ok = mbar_wait(&bar_load[st], lpar);
            if (__syncthreads_or(!ok)) { failed = true; break; }
            if (tid == 0) pending_stage = -1;
            ++load_iter;
            // Prefetch the next chunk into the other stage: its previous
            // contents were last read by MMAs that have completed.
            if (tid == 0 && c + 1 < nch) issue_loads(load_iter, ts + CH, h);

            // ---- D1 = [K; Q] K^T
            if (tid == 0) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                    umma_f16(tmem + TM_D1, sdesc_sw128(kq + off, 16, 1024),
                              sdesc_sw128(kq + off, 16, 1024), ID_D1, kk > 0);
                }
            }
            if (!mma_sync()) { failed = true; break; }
            tiles_to_f16(smem + OFF_KQ + st * KQ_STAGE, smem + OFF_V + st * V_STAGE, tid);
            {
                float x[64];
                tmem_ld64(trow + TM_D1, x);
                tmem_wait_ld();
                const int r = tid & 63;
                const bool qk = tid >= 64;
                const float br = sb[r];
                float run = 1.f;
#pragma unroll
                for (int s = 63; s >= 0; --s) {
                    const bool in = s <= r;
                    const float ps = in ? run : 0.f;
                    if (tid == 63) spend[s] = ps;
                    x[s] = qk ? (in ? ps * x[s] : 0.f) : (s < r ? br * ps * x[s] : 0.f);
                    run = in ? run * sa[s] : run;
                }
                if (!qk) {
                    sg[r] = run;
#pragma unroll
                    for (int s = 0; s < 64; ++s) Af[r * AST + s] = x[s];
                } else {
                    st_row64_f16(smem + OFF_M, r, x);
                }
            }
            __syncthreads();
            solve_unit_lower(Af, Tf, Xf, tid);
            {
                const int t = tid & 63;
                const bool hat = tid >= 64;
                float x[64];
#pragma unroll
                for (int s = 0; s < 64; ++s) {
                    const float sc = hat ? sb[s] * sg[s] : sb[s];
                    x[s] = Tf[t * AST + s] * sc;
                }
                st_row64_f16(smem + (hat ? OFF_TH : OFF_TT), t, x);
            }
            operands_ready();

            // ---- D_U = V^T (T diag b)^T, D_W = K^T (T diag bg)^T, D_SQ = S0 Q^T
            if (tid == 0) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    umma_f16(tmem + TM_U, sdesc_sw128(vb + kk * 2048, 8192, 1024),
                              sdesc_sw128(sbase + OFF_TT + kk * 32, 16, 1024), ID_MK64, kk > 0);
                }
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    umma_f16(tmem + TM_W, sdesc_sw128(kq + kk * 2048, 16384, 1024),
                              sdesc_sw128(sbase + OFF_TH + kk * 32, 16, 1024), ID_MK64, kk > 0);
                }
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                    umma_f16(tmem + TM_SQ, sdesc_sw128(sbase + OFF_S + off, 16, 1024),
                              sdesc_sw128(kq + off + 8192, 16, 1024), ID_KK64, kk > 0);
                }
            }
            if (!mma_sync()) { failed = true; break; }
            {
                float x[64];
                tmem_ld64(trow + TM_W, x);  // W[t][j = tid] for all t
                tmem_wait_ld();
#pragma unroll
                for (int t = 0; t < 64; ++t) x[t] = -x[t];
                st_row64_f16(smem + OFF_WT, tid, x);
            }
            operands_ready();

            // ---- Delta^T = U^T - S0 W^T (accumulated onto D_U)
            if (tid == 0) {
#pragma unroll
                for (int kk = 0; kk < 8; ++kk) {
                    const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                    umma_f16(tmem + TM_U, sdesc_sw128(sbase + OFF_S + off, 16, 1024),
                              sdesc_sw128(sbase + OFF_WT + kk * 2048, 8192, 1024), ID_KM64, 1);
                }
            }
            if (!mma_sync()) { failed = true; break; }
            {
                float x[64];
                tmem_ld64(trow + TM_U, x);  // Delta[s][i = tid] for all s
                tmem_wait_ld();
                st_row64_f16(smem + OFF_DT, tid, x);
#pragma unroll
                for (int s = 0; s < 64; ++s) x[s] *= spend[s];
                st_row64_f16(smem + OFF_DTS, tid, x);
                // D_S <- gamma_{C-1} D_S before the rank-C update accumulates.
                const float gC = sg[63];
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    float v[32];
                    tmem_ld32(trow + TM_S + 32 * q4, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] *= gC;
                    tmem_st32(trow + TM_S + 32 * q4, v);
                }
                tmem_wait_st();
            }
            operands_ready();

            // ---- D_O2 = Delta^T M^T ; D_S += (P[C-1] Delta)^T K
            if (tid == 0) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    umma_f16(tmem + TM_O2, sdesc_sw128(sbase + OFF_DT + kk * 32, 16, 1024),
                              sdesc_sw128(sbase + OFF_M + kk * 32, 16, 1024), ID_KK64, kk > 0);
                }
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    umma_f16(tmem + TM_S, sdesc_sw128(sbase + OFF_DTS + kk * 32, 16, 1024),
                              sdesc_sw128(kq + kk * 2048, 16384, 1024), ID_KM128, 1);
                }
            }
            if (!mma_sync()) { failed = true; break; }

            // ---- epilogue: O = gamma (S0 Q^T) + Delta^T M^T; refresh the fp16 state
            {
                float sq[64], o2[64];
                tmem_ld64(trow + TM_SQ, sq);
                tmem_ld64(trow + TM_O2, o2);
                tmem_wait_ld();
                __nv_bfloat16 *op = p.o + ts * tok_stride + static_cast<int64_t>(h) * HD + tid;
#pragma unroll
                for (int t = 0; t < 64; ++t) {
                    if (t < L) op[t * tok_stride] = __float2bfloat16_rn(fmaf(sg[t], sq[t], o2[t]));
                }
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    float v[32];
                    tmem_ld32(trow + TM_S + 32 * q4, v);
                    tmem_wait_ld();
                    uint8_t *blk = smem + OFF_S + (q4 >> 1) * 16384;
#pragma unroll
                    for (int cc = 0; cc < 4; ++cc) {
                        uint4 w;
                        w.x = pack_f16x2(v[8 * cc + 0], v[8 * cc + 1]);
                        w.y = pack_f16x2(v[8 * cc + 2], v[8 * cc + 3]);
                        w.z = pack_f16x2(v[8 * cc + 4], v[8 * cc + 5]);
                        w.w = pack_f16x2(v[8 * cc + 6], v[8 * cc + 7]);
                        *reinterpret_cast<uint4 *>(blk + sw128_offset(tid, (q4 & 1) * 4 + cc)) = w;
                    }
                }
            }
            operands_ready();
        }
        if (failed) break;

        // ---- final state
        if (p.state_out) {
            const int64_t slot = p.out_slots ? static_cast<int64_t>(p.out_slots[seq]) : seq;
            if (slot >= 0 && slot < p.num_slots) {
                float *dst = p.state_out + ((slot * H + h) * HD + tid) * HD;
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    float v[32];
                    tmem_ld32(trow + TM_S + 32 * q4, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        *reinterpret_cast<float4 *>(dst + 32 * q4 + e) =
                            make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                }
            }
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    }

    if (failed) {
        // Drain what this CTA still has in flight (bounded), then report.
        if (tid == 0) {
            if (pending_stage >= 0) mbar_wait(&bar_load[pending_stage], pending_parity, 200000000ull);
            if (mma_pending) mbar_wait(bar_mma, mma_phase, 200000000ull);
            atomicExch(&g_tc_status, 1);
        }
        __syncthreads();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, TM_COLS);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

int make_tmap(CUtensorMap *m, const void *base, int64_t tokens, int H) {
    auto fn = encode_fn();
    if (!fn) return set_error(RHZ_ERR_DEVICE, "cuTensorMapEncodeTiled is unavailable");
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(HD), static_cast<cuuint64_t>(H),
                          static_cast<cuuint64_t>(tokens)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(HD) * 2,
                             static_cast<cuuint64_t>(H) * HD * 2};
    cuuint32_t box[3] = {64, 1, CH};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims,
                    strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(RHZ_ERR_DEVICE, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return RHZ_OK;
}

}  // namespace

bool chunk_tc_supports(int d, int dtype) { return d == HD && dtype == RHZ_DTYPE_BF16; }

int launch_chunk_tc(const SeqArgs &a) {
    if (!chunk_tc_supports(a.d, a.dtype))
        return set_error(RHZ_ERR_SHAPE, "tensor-core kernel needs bf16 and head_dim 128 (got %d)", a.d);
    const int64_t tokens = a.cu_seqlens ? a.total_tokens : a.n_seq * a.seq_len;
    if (a.n_seq == 0) return RHZ_OK;
    if (tokens <= 0) {
        // Every sequence is empty: final state = initial state.
        SeqArgs b = a;
        return launch_seq(b);
    }
    CUtensorMap tq, tk, tv;
    int st = make_tmap(&tq, a.q, tokens, a.H);
    if (st == RHZ_OK) st = make_tmap(&tk, a.k, tokens, a.H);
    if (st == RHZ_OK) st = make_tmap(&tv, a.v, tokens, a.H);
    if (st != RHZ_OK) return st;
    int sms = 148;
    bool sm100 = true;
    device_info(&sms, &sm100);
    const int64_t items = a.n_seq * a.H;
    const int grid = static_cast<int>(items < sms ? items : sms);
    static std::once_flag attr_once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(attr_once, [] {
        attr_err = cudaFuncSetAttribute(gdr_chunk_tc_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(SMEM_ALLOC));
    });
    if (attr_err != cudaSuccess)
        return set_error(RHZ_ERR_DEVICE, "gdr_chunk_tc_kernel smem attribute: %s", cudaGetErrorString(attr_err));
    TcParams p;
    p.o = static_cast<__nv_bfloat16 *>(a.o);
    p.alpha = a.alpha;
    p.beta = a.beta;
    p.cu_seqlens = a.cu_seqlens;
    p.n_seq_dev = a.n_seq_dev;
    p.n_seq = a.n_seq;
    p.seq_len = a.seq_len;
    p.total_tokens = tokens;
    p.state_in = a.state_in;
    p.in_slots = a.in_slots;
    p.state_out = a.state_out;
    p.out_slots = a.out_slots;
    p.num_slots = a.num_slots;
    p.H = a.H;
    gdr_chunk_tc_kernel<<<grid, NT, SMEM_ALLOC, a.stream>>>(tq, tk, tv, p);
    return check_launch("gdr_chunk_tc_kernel");
}

}  // namespace rhz
