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
// Delta_t = beta_t (v_t - alpha_t S_{t-1} k_t).
//
// Decays: with gl_t the prefix sum of log2(alpha) over the chunk's nonzero
// alphas and z_t the number of zero alphas so far,
//   P[t][s] = (z_t == z_s) ? exp2(gl_t - gl_s) : 0,
// so alpha = 0 (a reset) gives exactly zero and the table costs one exp2 per
// entry with no sequential product chain; only differences t >= s are ever
// exponentiated (never above 1, no overflow).
//
// Work split. Everything that depends only on the chunk's keys and gates --
// the decayed [K; Q] K^T, the unit-lower-triangular inverse T, T diag(beta)
// and W -- is independent across chunks; only the products with S form the
// sequential chain. Each (sequence, head) item therefore runs on a cluster of
// two CTAs:
//   rank 1, the producer: for every chunk, D1 = [K; Q] K^T (bf16 tiles),
//     A (fp32) and M = P (Q K^T) (fp16), the inverse (diagonal 16 x 16 tiles
//     by substitution, the rest by a 2 x 2 recursion on mma.sync), then
//     D_W = K^T (T diag(beta gamma))^T on tcgen05. It writes a 32 KB record
//     {-W^T, T diag(beta), M} as ready-made fp16 operand images (128-byte
//     swizzle) and hands it to the chain CTA with one shared-memory-to-peer
//     bulk copy, two records in flight.
//   rank 0, the chain: S in TMEM (fp32) for the whole sequence, an fp16 copy
//     in shared memory as the MMA operand, and two MMA rounds per chunk:
//       R1: D_U  = V^T (T diag b)^T + S (-W^T)   (128 x 64, = Delta^T)
//           D_O  = Q~ S^T                         ( 64 x 128), Q~ = diag(gamma) Q
//       R2: D_O += M Delta                        ( 64 x 128)
//           D_S += Delta^T K~                     (128 x 128), K~ = diag(P[C-1]) K
//     with D_S pre-scaled by gamma_{C-1} when the previous chunk's state is
//     refreshed. Its tiles arrive by TMA one chunk ahead and are converted to
//     fp16 in place (Q and K rows scaled on the way) under the R1 products.
// Every product takes fp16 operands except D1 (A and B of one MMA always
// share a type); fp16 intermediates bound |q.k|, |v|, |S| to < 65504
// (unit-norm keys, as the reference specifies, keep them far below).
//
// One CTA per SM (each needs ~212 KB of shared memory), clusters persistent
// over items. Every wait is bounded; a timeout sets a sticky device flag,
// drains what is in flight (bounded), frees TMEM and returns. No load uses
// cluster multicast.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <climits>
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "chunk_common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace rhz {

// Sticky per-device flag: set when a bounded device-side wait ran out.
__device__ int g_tc_status = 0;

namespace {
using namespace sm100;
using namespace chunk;

constexpr int NT = 256;   // threads per CTA

constexpr uint32_t KQ_STAGE = 32768;  // [half][K rows | Q rows], 64 x 64 bf16 boxes
constexpr uint32_t V_STAGE = 16384;   // [half][V rows]
constexpr uint32_t KQ_BYTES = 4 * 8192;
constexpr uint32_t KQV_BYTES = 6 * 8192;

// Producer -> chain record: fp16 operand images, 128-byte swizzle.
constexpr uint32_t REC_WT = 0;        // -W^T [j = 128 rows][t = 64]     (MN-major B of R1)
constexpr uint32_t REC_TT = 16384;    // T diag(beta) [t = 64 rows][s]   (K-major B of R1)
constexpr uint32_t REC_M = 24576;     // M = P (Q K^T) [t rows][s]        (K-major A of R2)
constexpr uint32_t REC_BYTES = 32768;


// Chain CTA (cluster rank 0) shared memory.
constexpr uint32_t C_OFF_KQ = 0;             // 2 stages
constexpr uint32_t C_OFF_V = 65536;          // 2 stages
constexpr uint32_t C_OFF_REC = 98304;        // 2 record slots
constexpr uint32_t C_OFF_S = 163840;         // fp16 state [half j][128 rows i][64 j]
constexpr uint32_t C_OFF_DT = 196608;        // fp16 Delta^T [i = 128 rows][s]
constexpr uint32_t C_OFF_GATE = 212992;      // ring of 4 gate tables
constexpr uint32_t C_OFF_BAR = C_OFF_GATE + 4 * G_BYTES;
// Chain barriers: tiles landed [2], record landed [2], D_U done (R1), D_S
// done (R2), all of a chunk's products done, tiles converted [2] (warpgroup
// 1 -> 0), D_O buffer read out [2] (1 -> 0), and a barrier that only the
// failure path uses to wait for every MMA issued.
constexpr int CB_LOAD = 0, CB_FULL = 2, CB_R1 = 4, CB_R2S = 5, CB_R2 = 6, CB_CONV = 7, CB_OFREE = 9,
              CB_DRAIN = 11, CB_NUM = 12;
constexpr uint32_t C_OFF_NORM = C_OFF_BAR + 128;  // output-norm scale, HD floats
constexpr uint32_t C_USED = C_OFF_NORM + HD * 4;
static_assert(C_OFF_NORM >= C_OFF_BAR + CB_NUM * 8 + 16, "chain barriers overlap the norm scale");

// Producer CTA (cluster rank 1) shared memory.
constexpr uint32_t P_OFF_KQ = 0;             // 2 stages of K, Q tiles
constexpr uint32_t P_OFF_STG = 65536;        // 2 records being built
constexpr uint32_t P_OFF_TH = 131072;        // T diag(beta gamma) [t][s] as bf16 hi, lo (2 x 8 KB); earlier the solve's scratch
constexpr uint32_t P_OFF_AF = 147456;        // A fp32 [64][AST]
constexpr uint32_t P_OFF_TF = P_OFF_AF + 64 * AST * 4;   // T fp32 [64][AST]
constexpr uint32_t P_OFF_GATE = P_OFF_TF + 64 * AST * 4; // 2 gate tables
constexpr uint32_t P_OFF_BAR = P_OFF_GATE + 2 * G_BYTES;
// Producer barriers: tiles landed [2], D1 done, D_W done, chain slot free [2],
// failure-path drain of every MMA issued.
constexpr int PB_LOAD = 0, PB_D1 = 2, PB_MMA = 3, PB_EMPTY = 4, PB_DRAIN = 6, PB_DRAIN2 = 7,
              PB_NUM = 8;
constexpr uint32_t P_USED = P_OFF_BAR + PB_NUM * 8 + 16;  // + TMEM base

constexpr uint32_t SMEM_USED = C_USED > P_USED ? C_USED : P_USED;
constexpr size_t SMEM_ALLOC = SMEM_USED + 1024;  // slack for 1024-byte alignment
static_assert(C_OFF_GATE >= C_OFF_DT + 16384, "chain map overlaps");
static_assert(P_OFF_AF >= P_OFF_TH + 16384, "producer map overlaps");
static_assert(SMEM_ALLOC <= 232448, "exceeds the 227 KB opt-in shared memory");

// TMEM columns (f32). Chain: D_U (128 lanes x 64), D_S (128 x 128) and two
// D_O buffers (M = 64: row t in lane 32 (t / 16) + t % 16, 128 columns).
// Producer: D1 (128 x 64) and D_W (128 x 64).
constexpr uint32_t TM_U = 0, TM_S = 64, TM_O = 192, C_TM_COLS = 512;
constexpr uint32_t TM_D1 = 0, TM_W = 64, P_TM_COLS = 128;

constexpr uint32_t ID_D1 = idesc_bf16(128, 64, false, false);
constexpr uint32_t ID_MK64 = idesc_f16(128, 64, true, false);
constexpr uint32_t ID_MK64_BF = idesc_bf16(128, 64, true, false);
constexpr uint32_t ID_KM64 = idesc_f16(128, 64, false, true);
constexpr uint32_t ID_KM128 = idesc_f16(128, 128, false, true);
constexpr uint32_t ID_O = idesc_f16(64, 128, false, false);

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
    const float *norm_scale;  // non-null: groupnorm_heads on each O row in the epilogue
    float norm_eps;
};

// Chain: one stage's K, Q (32 KB) and V (16 KB) tiles bf16 -> fp16 in place,
// Q rows scaled by gamma_t and K rows by P[C-1][s]; this thread's 16-byte
// chunks are first, first + STRIDE, ... of the K/Q stage (2048 chunks) and of
// the V stage (1024). The swizzle permutes chunks within a row only, so chunk
// i of a K/Q half lies in row (i / 8) % 128 (rows 0..63 K, 64..127 Q).
template <int STRIDE>
__device__ __forceinline__ void chain_tiles_to_f16(uint8_t *kq, uint8_t *vv, const float *gm,
                                                   const float *pl, int first) {
    static_assert(2048 % (8 * STRIDE) == 0 && 1024 % (8 * STRIDE) == 0, "batches of 8 chunks");
    // Eight loads in flight, then eight converted stores (batches rolled to
    // keep the code small).
#pragma unroll 1
    for (int b = 0; b < 2048 / STRIDE; b += 8) {
        uint4 x[8];
        float sc[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int i = first + (b + m) * STRIDE;
            const int r = (i >> 3) & 127;
            x[m] = *reinterpret_cast<const uint4 *>(kq + i * 16);
            sc[m] = r < 64 ? pl[r] : gm[r - 64];
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            const int i = first + (b + m) * STRIDE;
            uint4 w = x[m];
            w.x = bf16x2_to_f16x2(w.x, sc[m]);
            w.y = bf16x2_to_f16x2(w.y, sc[m]);
            w.z = bf16x2_to_f16x2(w.z, sc[m]);
            w.w = bf16x2_to_f16x2(w.w, sc[m]);
            *reinterpret_cast<uint4 *>(kq + i * 16) = w;
        }
    }
#pragma unroll 1
    for (int b = 0; b < 1024 / STRIDE; b += 8) {
        uint4 x[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) x[m] = *reinterpret_cast<const uint4 *>(vv + (first + (b + m) * STRIDE) * 16);
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            uint4 w = x[m];
            w.x = bf16x2_to_f16x2(w.x, 1.f);
            w.y = bf16x2_to_f16x2(w.y, 1.f);
            w.z = bf16x2_to_f16x2(w.z, 1.f);
            w.w = bf16x2_to_f16x2(w.w, 1.f);
            *reinterpret_cast<uint4 *>(vv + (first + (b + m) * STRIDE) * 16) = w;
        }
    }
}

// Make thread-written smem operands and TMEM stores visible to the MMA issuer.
__device__ __forceinline__ void operands_ready() {
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
}

struct Ref {
    int64_t item, ts;  // item < 0: no chunk
    int L, h;
};

// The chunks a cluster processes, in order: items start, start + stride, ...
// and within an item its chunks of CH positions from the sequence start.
// Both CTAs of a cluster walk the same sequence; chunk k of it uses tile
// stage, record slot and gate table k & 1.
struct Walk {
    const TcParams *p;
    int64_t n_items, stride;
    int H;

    __device__ void bounds(int64_t item, int64_t &t0, int64_t &t1) const {
        const int64_t seq = item / H;
        if (p->cu_seqlens) {
            // Offsets are caller data: clamp them to the packed stream.
            t0 = p->cu_seqlens[seq];
            t1 = p->cu_seqlens[seq + 1];
            t0 = t0 < 0 ? 0 : (t0 > p->total_tokens ? p->total_tokens : t0);
            t1 = t1 < t0 ? t0 : (t1 > p->total_tokens ? p->total_tokens : t1);
        } else {
            t0 = seq * p->seq_len;
            t1 = t0 + p->seq_len;
        }
    }
    // First chunk at or after item `it` (skipping empty sequences).
    __device__ Ref first_from(int64_t it) const {
        for (; it < n_items; it += stride) {
            int64_t t0, t1;
            bounds(it, t0, t1);
            if (t1 > t0) {
                const int64_t seq = it / H;
                return Ref{it, t0, static_cast<int>((t1 - t0) < CH ? (t1 - t0) : CH),
                           static_cast<int>(it - seq * H)};
            }
        }
        return Ref{-1, 0, 0, 0};
    }
    __device__ Ref next_of(const Ref &r) const {
        int64_t t0, t1;
        bounds(r.item, t0, t1);
        const int64_t tn = r.ts + CH;
        if (tn < t1) return Ref{r.item, tn, static_cast<int>((t1 - tn) < CH ? (t1 - tn) : CH), r.h};
        return first_from(r.item + stride);
    }
    // The chunk n steps after chunk c of `item` (bounds [t0, t1), nch chunks,
    // head h): arithmetic inside the item, the walk only past its end (once
    // per item rather than once per chunk).
    __device__ Ref after(int64_t item, int h, int64_t t0, int64_t t1, int nch, int c, int n) const {
        const int cc = c + n;
        if (cc < nch) {
            const int64_t ts = t0 + static_cast<int64_t>(cc) * CH;
            return Ref{item, ts, static_cast<int>((t1 - ts) < CH ? (t1 - ts) : CH), h};
        }
        Ref r = first_from(item + stride);
        for (int i = nch; i < cc && r.item >= 0; ++i) r = next_of(r);
        return r;
    }
};

__device__ __forceinline__ GateIn gate_load(const TcParams &p, const Ref &r, int lane) {
    GateIn g{1.f, 1.f, 0.f, 0.f};
    if (r.item < 0) return g;
    const int H = p.H;
    const int p0 = 2 * lane, p1 = p0 + 1;
    if (p0 < r.L) {
        g.a0 = p.alpha[(r.ts + p0) * H + r.h];
        g.b0 = p.beta[(r.ts + p0) * H + r.h];
    }
    if (p1 < r.L) {
        g.a1 = p.alpha[(r.ts + p1) * H + r.h];
        g.b1 = p.beta[(r.ts + p1) * H + r.h];
    }
    return g;
}

struct RoleState {
    bool failed;
};

// ------------------------------------------------------------------ chain CTA
//
// Warpgroup 0 runs the serial state path of every chunk k: record k, tiles k
// converted and D_O buffer k & 1 free -> R1 -> Delta^T -> R2 -> state
// refresh. Warpgroup 1 works beside it: gate tables two chunks ahead, the
// fp16 conversion of chunk k + 1's tiles under chunk k's products, and, once
// R2(k) is done, the release of stage / record slot k & 1, the loads of chunk
// k + 2 and the O rows of chunk k from D_O[k & 1]. Every barrier phase has a
// single producer and is consumed before it can be reused, so parities never
// alias.
__device__ __forceinline__ RoleState chain_role(const CUtensorMap *tm_q, const CUtensorMap *tm_k,
                                                const CUtensorMap *tm_v, const TcParams &p,
                                                uint8_t *smem, const Walk &wk, int64_t start,
                                                uint32_t tmem) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ww = warp & 3;
    const uint32_t trow = tmem + (static_cast<uint32_t>(ww) << 21);  // lanes 32 ww .. 32 ww + 31
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C_OFF_BAR);
    uint64_t *bar_load = bars + CB_LOAD, *bar_full = bars + CB_FULL, *bar_r1 = bars + CB_R1,
             *bar_r2s = bars + CB_R2S, *bar_r2 = bars + CB_R2, *bar_conv = bars + CB_CONV,
             *bar_ofree = bars + CB_OFREE;
    const uint32_t sbase = smem_u32(smem);
    const int H = p.H;
    const int64_t tok_stride = static_cast<int64_t>(H) * HD;
    auto gates = [&](int kc) { return reinterpret_cast<float *>(smem + C_OFF_GATE) + (kc & 3) * G_SIZE; };
    RoleState rs{false};

    if (tid < 128) {
        // ------------------------------------------------ warpgroup 0: state path
        const int row = tid;  // state row i = TMEM lane
        int k = 0;
        for (int64_t item = start; item < wk.n_items && !rs.failed; item += wk.stride) {
            const int64_t seq = item / H;
            const int h = static_cast<int>(item - seq * H);
            int64_t t0, t1;
            wk.bounds(item, t0, t1);
            const int nch = static_cast<int>((t1 - t0 + CH - 1) / CH);
            int64_t slot = -1;
            if (p.state_in) slot = p.in_slots ? static_cast<int64_t>(p.in_slots[seq]) : seq;
            const bool have = p.state_in && slot >= 0 && slot < p.num_slots;
            const float *src = have ? p.state_in + ((slot * H + h) * HD + row) * HD : nullptr;
            int64_t so = -1;
            if (p.state_out) so = p.out_slots ? static_cast<int64_t>(p.out_slots[seq]) : seq;
            float *dst = (p.state_out && so >= 0 && so < p.num_slots)
                             ? p.state_out + ((so * H + h) * HD + row) * HD
                             : nullptr;
            if (nch == 0) {
                // Empty sequence: the final state is the initial state.
                if (dst)
                    for (int e = 0; e < HD; e += 4)
                        *reinterpret_cast<float4 *>(dst + e) =
                            have ? *reinterpret_cast<const float4 *>(src + e) : make_float4(0.f, 0.f, 0.f, 0.f);
                continue;
            }
            for (int c = 0; c < nch; ++c, ++k) {
                const int64_t ts = t0 + static_cast<int64_t>(c) * CH;
                (void)ts;
                const uint32_t kq = sbase + C_OFF_KQ + (k & 1) * KQ_STAGE;
                const uint32_t vb = sbase + C_OFF_V + (k & 1) * V_STAGE;
                const uint32_t rec = sbase + C_OFF_REC + (k & 1) * REC_BYTES;
                const uint32_t tO = tmem + TM_O + 128 * (k & 1);

                // ---- R1's inputs: record k (its barrier armed here; the peer's
                // copy may already have delivered its bytes), tiles k in fp16,
                // D_O buffer k & 1 read out
                if (tid == 0) mbar_arrive_expect_tx(&bar_full[k & 1], REC_BYTES);
                bool ok = mbar_wait_cluster(&bar_full[k & 1], (k >> 1) & 1);
                ok = ok && mbar_wait(&bar_conv[k & 1], (k >> 1) & 1);
                if (k >= 2) ok = ok && mbar_wait(&bar_ofree[k & 1], ((k >> 1) + 1) & 1);
                if (wg_sync_or(1, !ok)) { rs.failed = true; break; }

                // ---- first chunk of the item: fp16 copy of S0 (unscaled) and
                // D_S = gamma_{C-1} S0
                if (c == 0) {
                    const float gC = gates(k)[G_GM + 63];
#pragma unroll 1
                    for (int q4 = 0; q4 < 4; ++q4) {
                        float v[32];
#pragma unroll
                        for (int e = 0; e < 32; e += 4) {
                            const float4 f = have ? *reinterpret_cast<const float4 *>(src + 32 * q4 + e)
                                                  : make_float4(0.f, 0.f, 0.f, 0.f);
                            v[e] = f.x; v[e + 1] = f.y; v[e + 2] = f.z; v[e + 3] = f.w;
                        }
                        st_row32_f16(smem + C_OFF_S + (q4 >> 1) * 16384, row, 4 * (q4 & 1), v);
#pragma unroll
                        for (int e = 0; e < 32; ++e) v[e] *= gC;
                        tmem_st32(trow + TM_S + 32 * q4, v);
                    }
                    tmem_wait_st();
                    fence_proxy_async_smem();
                    tc_fence_before();
                    wg_sync(1);
                }

                // ---- R1: D_U = V^T (T diag b)^T + S (-W^T) ; D_O[k & 1] = Q~ S^T
                if (tid == 0) {
                    tc_fence_after();
#pragma unroll 1
                    for (int kk = 0; kk < 4; ++kk)
                        umma_f16(tmem + TM_U, sdesc_sw128(vb + kk * 2048, 8192, 1024),
                                 sdesc_sw128(rec + REC_TT + kk * 32, 16, 1024), ID_MK64, kk > 0);
#pragma unroll 1
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                        umma_f16(tmem + TM_U, sdesc_sw128(sbase + C_OFF_S + off, 16, 1024),
                                 sdesc_sw128(rec + REC_WT + kk * 2048, 8192, 1024), ID_KM64, 1);
                    }
                    umma_commit(bar_r1);  // Delta^T is ready; D_O runs on behind it
#pragma unroll 1
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
                        umma_f16(tO, sdesc_sw128(kq + off + 8192, 16, 1024),
                                 sdesc_sw128(sbase + C_OFF_S + off, 16, 1024), ID_O, kk > 0);
                    }
                }
                ok = mbar_wait(bar_r1, k & 1);
                if (wg_sync_or(1, !ok)) { rs.failed = true; break; }
                tc_fence_after();

                // ---- Delta^T (fp16): row i, all 64 positions
                {
                    float x[32], y[32];
                    tmem_ld32(trow + TM_U, x);
                    tmem_ld32(trow + TM_U + 32, y);
                    tmem_wait_ld();
                    st_row32_f16(smem + C_OFF_DT, row, 0, x);
                    st_row32_f16(smem + C_OFF_DT, row, 4, y);
                }
                fence_proxy_async_smem();
                tc_fence_before();
                wg_sync(1);

                // ---- R2: D_S += Delta^T K~ (the state refresh waits for this
                // part only), then D_O[k & 1] += M Delta
                if (tid == 0) {
                    tc_fence_after();
#pragma unroll 1
                    for (int kk = 0; kk < 4; ++kk)
                        umma_f16(tmem + TM_S, sdesc_sw128(sbase + C_OFF_DT + kk * 32, 16, 1024),
                                 sdesc_sw128(kq + kk * 2048, 16384, 1024), ID_KM128, 1);
                    umma_commit(bar_r2s);
#pragma unroll 1
                    for (int kk = 0; kk < 4; ++kk)
                        umma_f16(tO, sdesc_sw128(rec + REC_M + kk * 32, 16, 1024),
                                 sdesc_sw128(sbase + C_OFF_DT + kk * 32, 16, 1024), ID_O, 1);
                    umma_commit(bar_r2);
                }
                ok = mbar_wait(bar_r2s, k & 1);
                if (wg_sync_or(1, !ok)) { rs.failed = true; break; }
                tc_fence_after();

                // ---- state: fp16 copy for the next chunk and D_S pre-scaled
                // by its gamma_{C-1}, or the final state
                {
                    const bool more = c + 1 < nch;
                    const float gn = more ? gates(k + 1)[G_GM + 63] : 1.f;
#pragma unroll 1
                    for (int q4 = 0; q4 < 4; ++q4) {
                        float v[32];
                        tmem_ld32(trow + TM_S + 32 * q4, v);
                        tmem_wait_ld();
                        if (more) {
                            st_row32_f16(smem + C_OFF_S + (q4 >> 1) * 16384, row, 4 * (q4 & 1), v);
#pragma unroll
                            for (int e = 0; e < 32; ++e) v[e] *= gn;
                            tmem_st32(trow + TM_S + 32 * q4, v);
                        } else if (dst) {
#pragma unroll
                            for (int e = 0; e < 32; e += 4)
                                *reinterpret_cast<float4 *>(dst + 32 * q4 + e) =
                                    make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                        }
                    }
                    if (more) tmem_wait_st();
                }
                fence_proxy_async_smem();
                tc_fence_before();
                wg_sync(1);
            }
        }
        if (rs.failed && tid == 0) {
            // Every MMA this thread issued (including D_O products that no
            // commit covered yet) completes before TMEM is released.
            umma_commit(bars + CB_DRAIN);
            mbar_wait(bars + CB_DRAIN, 0, 200000000ull);
        }
    } else {
        // ------------------------------------------------ warpgroup 1: tiles, epilogue
        const int wt = tid - 128;
        const uint32_t peer_empty = mapa_shared(sbase + P_OFF_BAR + 8 * PB_EMPTY, 1);
        int loads_issued = 0, loads_waited = 0;
        GateIn gin{1.f, 1.f, 0.f, 0.f};  // warp 4: inputs of the gate table two chunks ahead
        auto issue_loads = [&](int kc, const Ref &r) {
            const uint32_t st = kc & 1;
            uint64_t *bar = &bar_load[st];
            uint8_t *kqs = smem + C_OFF_KQ + st * KQ_STAGE;
            uint8_t *vv = smem + C_OFF_V + st * V_STAGE;
            mbar_arrive_expect_tx(bar, KQV_BYTES);
            const int t32 = static_cast<int>(r.ts);
            tma_load_3d(kqs, tm_k, 0, r.h, t32, bar);
            tma_load_3d(kqs + 16384, tm_k, 64, r.h, t32, bar);
            tma_load_3d(kqs + 8192, tm_q, 0, r.h, t32, bar);
            tma_load_3d(kqs + 24576, tm_q, 64, r.h, t32, bar);
            tma_load_3d(vv, tm_v, 0, r.h, t32, bar);
            tma_load_3d(vv + 8192, tm_v, 64, r.h, t32, bar);
        };
        auto convert = [&](int kc) {
            const float *g = gates(kc);
            chain_tiles_to_f16<128>(smem + C_OFF_KQ + (kc & 1) * KQ_STAGE,
                                    smem + C_OFF_V + (kc & 1) * V_STAGE, g + G_GM, g + G_PL, wt);
            fence_proxy_async_smem();
        };

        float *nsc = reinterpret_cast<float *>(smem + C_OFF_NORM);
        const bool norm = p.norm_scale != nullptr;
        if (norm) nsc[wt] = p.norm_scale[wt];  // wt < 128 = HD
        {
            const Ref r0 = wk.first_from(start);
            const Ref r1 = r0.item >= 0 ? wk.next_of(r0) : r0;
            const Ref r2 = r1.item >= 0 ? wk.next_of(r1) : r1;
            if (wt == 0) {
                if (r0.item >= 0) issue_loads(0, r0);
                if (r1.item >= 0) issue_loads(1, r1);
            }
            loads_issued = (r0.item >= 0) + (r1.item >= 0);
            if (ww == 0) {
                gate_tables(gates(0), gate_load(p, r0, lane), lane);
                gate_tables(gates(1), gate_load(p, r1, lane), lane);
                gin = gate_load(p, r2, lane);
            }
            if (r0.item >= 0) {
                const bool ok = mbar_wait(&bar_load[0], 0);
                if (wg_sync_or(2, !ok)) {
                    rs.failed = true;
                } else {
                    ++loads_waited;
                    convert(0);
                    mbar_arrive(&bar_conv[0]);
                }
            }
        }

        int k = 0;
        for (int64_t item = start; item < wk.n_items && !rs.failed; item += wk.stride) {
            const int64_t seq = item / H;
            const int h = static_cast<int>(item - seq * H);
            int64_t t0, t1;
            wk.bounds(item, t0, t1);
            const int nch = static_cast<int>((t1 - t0 + CH - 1) / CH);
            for (int c = 0; c < nch; ++c, ++k) {
                const int64_t ts = t0 + static_cast<int64_t>(c) * CH;
                const int L = static_cast<int>((t1 - ts) < CH ? (t1 - ts) : CH);
                const Ref nxt = wk.after(item, h, t0, t1, nch, c, 1);
                const Ref nn = wk.after(item, h, t0, t1, nch, c, 2);

                // ---- gate table of chunk k + 2, then the inputs of chunk k + 3
                if (nn.item >= 0 && ww == 0) {
                    gate_tables(gates(k + 2), gin, lane);
                    gin = gate_load(p, wk.after(item, h, t0, t1, nch, c, 3), lane);
                }
                // ---- chunk k + 1's tiles -> fp16 (under chunk k's products)
                if (nxt.item >= 0) {
                    const bool ok = mbar_wait(&bar_load[(k + 1) & 1], ((k + 1) >> 1) & 1);
                    if (wg_sync_or(2, !ok)) { rs.failed = true; break; }
                    ++loads_waited;
                    convert(k + 1);
                }
                // ---- chunk k's products are done
                {
                    const bool ok = mbar_wait(bar_r2, k & 1);
                    if (wg_sync_or(2, !ok)) { rs.failed = true; break; }
                    tc_fence_after();
                }
                if (nxt.item >= 0) mbar_arrive(&bar_conv[(k + 1) & 1]);
                // Stage and record slot k & 1 are free again.
                if (wt == 0) {
                    mbar_arrive_remote_relaxed(peer_empty + 8 * (k & 1));
                    if (nn.item >= 0) issue_loads(k + 2, nn);
                }
                if (nn.item >= 0) ++loads_issued;

                // ---- O rows of chunk k (D_O row t in lane 32 (t / 16) + t % 16),
                // optionally RMS-normalised per head first (groupnorm_heads,
                // norm.rs:48-60, on the fp32 accumulator)
                {
                    const uint32_t tO = trow + TM_O + 128 * (k & 1);
                    const int t = 16 * ww + lane;
                    const bool has_row = lane < 16 && t < L;
                    __nv_bfloat16 *op = p.o + (ts + t) * tok_stride + static_cast<int64_t>(h) * HD;
                    float inv = 1.f;
                    if (norm) {
                        float ss = 0.f;
#pragma unroll 1
                        for (int q4 = 0; q4 < 4; ++q4) {
                            float o[32];
                            tmem_ld32(tO + 32 * q4, o);
                            tmem_wait_ld();
#pragma unroll
                            for (int e = 0; e < 32; ++e) ss += o[e] * o[e];
                        }
                        inv = 1.f / sqrtf(ss / static_cast<float>(HD) + p.norm_eps);
                    }
#pragma unroll 1
                    for (int q4 = 0; q4 < 4; ++q4) {
                        float o[32];
                        tmem_ld32(tO + 32 * q4, o);
                        tmem_wait_ld();
                        if (norm) {
#pragma unroll
                            for (int e = 0; e < 32; ++e) o[e] = o[e] * inv * nsc[32 * q4 + e];
                        }
                        if (has_row) {
#pragma unroll
                            for (int c8 = 0; c8 < 4; ++c8) {
                                uint4 w;
                                w.x = pack_bf16x2(o[8 * c8 + 0], o[8 * c8 + 1]);
                                w.y = pack_bf16x2(o[8 * c8 + 2], o[8 * c8 + 3]);
                                w.z = pack_bf16x2(o[8 * c8 + 4], o[8 * c8 + 5]);
                                w.w = pack_bf16x2(o[8 * c8 + 6], o[8 * c8 + 7]);
                                *reinterpret_cast<uint4 *>(op + 32 * q4 + 8 * c8) = w;
                            }
                        }
                    }
                    tc_fence_before();
                    mbar_arrive(&bar_ofree[k & 1]);
                }
            }
        }
        if (rs.failed && wt == 0)
            for (int kk = loads_waited; kk < loads_issued; ++kk)
                mbar_wait(&bar_load[kk & 1], (kk >> 1) & 1, 200000000ull);
    }
    if (rs.failed) atomicExch(&g_tc_status, 1);
    rs.failed = __syncthreads_or(rs.failed);
    return rs;
}

// ------------------------------------------------------------------ producer CTA
//
// All eight warps build chunk k's record while the tiles of chunk k + 1 land
// and its D1 runs; records alternate between two staging buffers, so building
// never waits for the copy of the previous record.
__device__ __forceinline__ RoleState producer_role(const CUtensorMap *tm_q, const CUtensorMap *tm_k,
                                                   const TcParams &p, uint8_t *smem, const Walk &wk,
                                                   int64_t start, uint32_t tmem) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row = 32 * (warp & 3) + lane;  // TMEM lane
    const int half = warp >> 2;              // column half of this thread
    const uint32_t trow = tmem + (static_cast<uint32_t>(warp & 3) << 21);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + P_OFF_BAR);
    uint64_t *bar_load = bars + PB_LOAD, *bar_d1 = bars + PB_D1, *bar_mma = bars + PB_MMA,
             *bar_empty = bars + PB_EMPTY;
    float *Af = reinterpret_cast<float *>(smem + P_OFF_AF);
    float *Tf = reinterpret_cast<float *>(smem + P_OFF_TF);
    float *Xf = reinterpret_cast<float *>(smem + P_OFF_TH);  // scratch of the solve; T^ comes later
    const uint32_t sbase = smem_u32(smem);
    const uint32_t peer_full = mapa_shared(sbase + C_OFF_BAR + 8 * CB_FULL, 0);
    const uint32_t peer_rec = mapa_shared(sbase + C_OFF_REC, 0);
    auto gates = [&](int kc) { return reinterpret_cast<float *>(smem + P_OFF_GATE) + (kc & 1) * G_SIZE; };
    auto issue_loads = [&](int kc, const Ref &r) {
        uint64_t *bar = &bar_load[kc & 1];
        uint8_t *kq = smem + P_OFF_KQ + (kc & 1) * KQ_STAGE;
        mbar_arrive_expect_tx(bar, KQ_BYTES);
        const int t32 = static_cast<int>(r.ts);
        tma_load_3d(kq, tm_k, 0, r.h, t32, bar);
        tma_load_3d(kq + 16384, tm_k, 64, r.h, t32, bar);
        tma_load_3d(kq + 8192, tm_q, 0, r.h, t32, bar);
        tma_load_3d(kq + 24576, tm_q, 64, r.h, t32, bar);
    };
    // D1 = [K; Q] K^T of chunk kc on its bf16 tiles.
    // The MMA-issue loops of both roles stay rolled: the per-chunk code of a
    // role is larger than the instruction cache keeps warm, and a rolled issue
    // loop (one thread, eight MMAs) costs nothing on the critical path while
    // the unrolled copies cost instruction-fetch stalls (4.5% of the kernel on
    // one box; the one-CTA kernel, with a different footprint, did not gain).
    auto issue_d1 = [&](int kc) {
        const uint32_t kq = sbase + P_OFF_KQ + (kc & 1) * KQ_STAGE;
#pragma unroll 1
        for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_f16(tmem + TM_D1, sdesc_sw128(kq + off, 16, 1024), sdesc_sw128(kq + off, 16, 1024),
                     ID_D1, kk > 0);
        }
        umma_commit(bar_d1);
    };

    RoleState rs{false};
    uint32_t mma_phase = 0;
    int loads_issued = 0, loads_waited = 0;
    // Record hand-over of the previous chunk, deferred into this chunk's
    // first phase (thread 128, whose warp has no table block there).
    bool ho_pending = false;
    Ref ho_nn{-1, 0, 0, 0};
    int ho_k = 0;
    auto handover = [&]() {
        if (tid == 128) {
            tc_fence_after();
            if (ho_nn.item >= 0) issue_loads(ho_k + 2, ho_nn);
            const uint32_t slot = ho_k & 1;
            bulk_copy_to_peer(peer_rec + slot * REC_BYTES, smem + P_OFF_STG + slot * REC_BYTES, REC_BYTES,
                              peer_full + 8 * slot);
        }
        if (ho_nn.item >= 0) ++loads_issued;
        ho_pending = false;
    };
    int k = 0;
    GateIn gin{1.f, 1.f, 0.f, 0.f};  // warp 4: inputs of the next chunk's gate table
    {
        const Ref cur = wk.first_from(start);
        const Ref second = cur.item >= 0 ? wk.next_of(cur) : cur;
        if (tid == 0) {
            if (cur.item >= 0) issue_loads(0, cur);
            if (second.item >= 0) issue_loads(1, second);
        }
        loads_issued = (cur.item >= 0) + (second.item >= 0);
        if (cur.item >= 0) {
            if (warp == 0) gate_tables(gates(0), gate_load(p, cur, lane), lane);
            if (warp == 4) gin = gate_load(p, second, lane);
            const bool ok = mbar_wait(&bar_load[0], 0);
            if (__syncthreads_or(!ok)) {
                rs.failed = true;
            } else {
                ++loads_waited;
                if (tid == 0) {
                    tc_fence_after();
                    issue_d1(0);
                }
            }
        }
    }

    for (int64_t item = start; item < wk.n_items && !rs.failed; item += wk.stride) {
        const int64_t seq = item / wk.H;
        const int h = static_cast<int>(item - seq * wk.H);
        int64_t t0, t1;
        wk.bounds(item, t0, t1);
        const int nch = static_cast<int>((t1 - t0 + CH - 1) / CH);
        for (int c = 0; c < nch; ++c, ++k) {
            const uint32_t kq = sbase + P_OFF_KQ + (k & 1) * KQ_STAGE;
            uint8_t *stg = smem + P_OFF_STG + (k & 1) * REC_BYTES;
            const float *g = gates(k);
            const int *gz = reinterpret_cast<const int *>(g + G_Z);

            // ---- staging buffer k & 1 is free once the chain consumed chunk k - 2;
            // D1 of this chunk (issued during the previous one)
            {
                bool ok = k < 2 || mbar_wait_cluster(&bar_empty[k & 1], ((k >> 1) + 1) & 1);
                ok = ok && mbar_wait(bar_d1, k & 1);
                if (__syncthreads_or(!ok)) { rs.failed = true; break; }
                tc_fence_after();
            }
            if (ho_pending) handover();

            // ---- A = beta P (K K^T) (fp32) and M = P (Q K^T) (record, fp16), 32 columns per thread
            {
                const bool qk = row >= 64;
                const int t = row & 63;
                const int s0 = 32 * half;
                // Warp-uniform: the whole 32 x 32 block lies above the diagonal.
                if (half == 1 && (warp & 1) == 0) {
                    if (qk) st_zero32(stg + REC_M, t, 4);
                } else {
                    const float glt = g[G_GL + t];
                    const int zt = gz[t];
                    const float bt = qk ? 1.f : g[G_BE + t];
#pragma unroll 1
                    for (int hp = 0; hp < 2; ++hp) {
                        const int sb = s0 + 16 * hp;
                        float v[16];
                        tmem_ld16(trow + TM_D1 + sb, v);
                        tmem_wait_ld();
#pragma unroll
                        for (int j4 = 0; j4 < 4; ++j4) {
                            const float4 g4 = *reinterpret_cast<const float4 *>(g + G_GL + sb + 4 * j4);
                            const int4 z4 = *reinterpret_cast<const int4 *>(gz + sb + 4 * j4);
                            const float gs[4] = {g4.x, g4.y, g4.z, g4.w};
                            const int zs[4] = {z4.x, z4.y, z4.z, z4.w};
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const int j = 4 * j4 + e, s = sb + j;
                                const float pv = zs[e] == zt ? ex2(glt - gs[e]) : 0.f;
                                const bool keep = qk ? (s <= t) : (s < t);
                                v[j] = keep ? bt * pv * v[j] : 0.f;
                            }
                        }
                        if (qk) {
                            st_row16_f16(stg + REC_M, t, 4 * half + 2 * hp, v);
                        } else {
#pragma unroll
                            for (int j4 = 0; j4 < 4; ++j4)
                                *reinterpret_cast<float4 *>(Af + t * AST + sb + 4 * j4) =
                                    make_float4(v[4 * j4], v[4 * j4 + 1], v[4 * j4 + 2], v[4 * j4 + 3]);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncthreads();

            // ---- diagonal 16 x 16 tiles of T (warps 0-3, one each) while warps
            // 4-7 zero tiles (0,1), (2,3) of T and wait for the next chunk's
            // tiles
            const Ref nxt = wk.after(item, h, t0, t1, nch, c, 1);
            const Ref nn = wk.after(item, h, t0, t1, nch, c, 2);
            bool prep_fail = false;
            if (warp < 4) {
                diag_inverse16(Af + (16 * warp) * AST + 16 * warp, Tf + (16 * warp) * AST + 16 * warp, lane);
            } else {
                const int wt = tid - 128;
                for (int e = wt; e < 512; e += 128) {
                    const int blk = e >> 8, rr = (e >> 4) & 15, cc = e & 15;
                    Tf[(32 * blk + rr) * AST + 32 * blk + 16 + cc] = 0.f;
                }
                if (nxt.item >= 0) prep_fail = !mbar_wait(&bar_load[(k + 1) & 1], ((k + 1) >> 1) & 1);
            }
            if (__syncthreads_or(prep_fail)) { rs.failed = true; break; }
            // The next D1 comes from thread 128 (warps 4-7 have no part in the
            // solve's first step; from thread 0 it delayed warp 0's).
            if (nxt.item >= 0) {
                ++loads_waited;
                if (tid == 128) {
                    tc_fence_after();
                    issue_d1(k + 1);
                }
            }
            solve_offdiag(Af, Tf, Xf, warp, lane, 0);

            // ---- T diag(beta) (record, fp16) and T diag(beta gamma) (local, as a
            // bf16 hi + lo pair so that D_W can read K's bf16 tile as it landed)
            {
                const int t = tid & 63;
                const bool hat = (tid >> 6) & 1;
                const int hh = tid >> 7;
                const int s0 = 32 * hh;
                uint8_t *dstb = hat ? smem + P_OFF_TH : stg + REC_TT;
                if (hh == 1 && t < 32) {
                    st_zero32(dstb, t, 4);
                    if (hat) st_zero32(dstb + 8192, t, 4);
                } else {
                    const float *sc = g + (hat ? G_BG : G_BE);
#pragma unroll 1
                    for (int hp = 0; hp < 2; ++hp) {
                        const int sb = s0 + 16 * hp;
                        float v[16];
#pragma unroll
                        for (int j4 = 0; j4 < 4; ++j4) {
                            const float4 tv = *reinterpret_cast<const float4 *>(Tf + t * AST + sb + 4 * j4);
                            const float4 sv = *reinterpret_cast<const float4 *>(sc + sb + 4 * j4);
                            const int s = sb + 4 * j4;
                            v[4 * j4 + 0] = s + 0 <= t ? tv.x * sv.x : 0.f;
                            v[4 * j4 + 1] = s + 1 <= t ? tv.y * sv.y : 0.f;
                            v[4 * j4 + 2] = s + 2 <= t ? tv.z * sv.z : 0.f;
                            v[4 * j4 + 3] = s + 3 <= t ? tv.w * sv.w : 0.f;
                        }
                        if (hat)
                            st_row16_bf16_split(dstb, dstb + 8192, t, 4 * hh + 2 * hp, v);
                        else
                            st_row16_f16(dstb, t, 4 * hh + 2 * hp, v);
                    }
                }
            }
            operands_ready();

            // ---- D_W = K^T (T diag bg)^T = K^T (hi + lo)^T on bf16 operands
            // (lane j, column t: W[t][j])
            if (tid == 0) {
#pragma unroll 1
                for (int kk = 0; kk < 8; ++kk)
                    umma_f16(tmem + TM_W, sdesc_sw128(kq + (kk & 3) * 2048, 16384, 1024),
                             sdesc_sw128(sbase + P_OFF_TH + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024),
                             ID_MK64_BF, kk > 0);
                umma_commit(bar_mma);
            }
            // The next chunk's gate table, under D_W (off the solve's path:
            // executed once per chunk by one warp, it ran mostly on
            // instruction-fetch stalls)
            if (warp == 4 && nxt.item >= 0) {
                gate_tables(gates(k + 1), gin, lane);
                gin = gate_load(p, nn, lane);
            }
            {
                const bool ok = mbar_wait(bar_mma, mma_phase);
                if (__syncthreads_or(!ok)) { rs.failed = true; break; }
                mma_phase ^= 1u;
                tc_fence_after();
            }
            {
                float x[32];
                tmem_ld32(trow + TM_W + 32 * half, x);
                tmem_wait_ld();
#pragma unroll
                for (int t = 0; t < 32; ++t) x[t] = -x[t];
                st_row32_f16(stg + REC_WT, row, 4 * half, x);
            }
            fence_proxy_async_smem();
            tc_fence_before();
            __syncthreads();

            // ---- stage k & 1 is free (D1 and D_W are done): fetch chunk k + 2;
            // hand the record to the chain CTA (its slot k & 1 is free: the
            // chain consumed chunk k - 2 before this staging buffer was reused)
            ho_pending = true;
            ho_nn = nn;
            ho_k = k;
        }
    }
    if (!rs.failed && ho_pending) handover();

    if (rs.failed && tid == 0) {
        for (int kk = loads_waited; kk < loads_issued; ++kk)
            mbar_wait(&bar_load[kk & 1], (kk >> 1) & 1, 200000000ull);
        umma_commit(bars + PB_DRAIN);  // every MMA thread 0 issued: D_W and the first D1
        mbar_wait(bars + PB_DRAIN, 0, 200000000ull);
        atomicExch(&g_tc_status, 1);
    }
    if (rs.failed && tid == 128) {
        umma_commit(bars + PB_DRAIN2);  // the later D1s (issued by this thread)
        mbar_wait(bars + PB_DRAIN2, 0, 200000000ull);
    }
    rs.failed = __syncthreads_or(rs.failed);
    return rs;
}

__global__ void __launch_bounds__(NT, 1)
    gdr_chunk_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v,
                        const __grid_constant__ TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tid = threadIdx.x, warp = tid >> 5;
    const uint32_t rank = cluster_ctarank();
    const bool chain = rank == 0;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + (chain ? C_OFF_BAR : P_OFF_BAR));
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + (chain ? CB_NUM : PB_NUM));
    const uint32_t ncols = chain ? C_TM_COLS : P_TM_COLS;

    if (tid == 0) {
        if (chain) {
            for (int i = 0; i < CB_NUM; ++i) mbar_init(&bars[i], 1);  // loads, R1, R2
            for (int i = 0; i < 2; ++i) {
                mbar_init(&bars[CB_CONV + i], 128);   // warpgroup 1 signals
                mbar_init(&bars[CB_OFREE + i], 128);
            }
        } else {
            for (int i = 0; i < PB_NUM; ++i) mbar_init(&bars[i], 1);
        }
        mbar_fence_init();
        prefetch_tmap(&tm_q);
        prefetch_tmap(&tm_k);
        if (chain) prefetch_tmap(&tm_v);
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, ncols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Both CTAs' barriers exist before either side touches the other's.
    cluster_sync();

    int64_t n_seq = p.n_seq;
    if (p.n_seq_dev) {
        const int64_t nd = *p.n_seq_dev;
        n_seq = nd < n_seq ? nd : n_seq;
    }
    const Walk wk{&p, n_seq * p.H, static_cast<int64_t>(cluster_count_x()), p.H};
    const int64_t start = cluster_id_x();
    const RoleState rs = chain ? chain_role(&tm_q, &tm_k, &tm_v, p, smem, wk, start, tmem)
                               : producer_role(&tm_q, &tm_k, p, smem, wk, start, tmem);

    // Teardown: past this cluster barrier neither side issues anything to the
    // other. Normally every record copy has been consumed; after a failure a
    // copy may still be in flight, so the chain pauses (bounded) to let it land
    // before its shared memory goes away.
    cluster_sync();
    if (chain && rs.failed && tid == 0) {
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 200000ull) {
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, ncols);
}

}  // namespace

bool chunk_tc_supports(int d, int dtype) { return d == HD && dtype == RHZ_DTYPE_BF16; }

int chunk_pair_status(int *flag, bool clear) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_status, sizeof(int));
    if (e == cudaSuccess && clear && v) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_tc_status, &zero, sizeof(int));
    }
    if (e != cudaSuccess) return set_error(RHZ_ERR_DEVICE, "reading the pair kernel's status: %s", cudaGetErrorString(e));
    *flag = v;
    return RHZ_OK;
}

namespace {
std::atomic<int> g_chunk_variant{RHZ_CHUNK_AUTO};
}

int set_chunk_variant(int v, int *prev) {
    if (v < RHZ_CHUNK_AUTO || v > RHZ_CHUNK_GRID)
        return set_error(RHZ_ERR_INVALID, "chunk kernel variant %d is not one of 0, 1, 2, 3", v);
    *prev = g_chunk_variant.exchange(v);
    return RHZ_OK;
}

// Work per (sequence, head) item: the cluster pair finishes an item in
// about 1/1.6 of the one-CTA kernel's time (measured on B200 at B=4, T=4096,
// H=16) but holds two SMs, so once there are more items than pairs the
// one-CTA kernel's doubled parallelism wins. Compare whole passes over the
// SMs with that cost ratio.
bool chunk_use_solo(int64_t items, int sms) {
    const int64_t pairs = sms / 2 > 0 ? sms / 2 : 1;
    const int64_t pair_passes = (items + pairs - 1) / pairs;
    const int64_t solo_passes = (items + sms - 1) / sms;
    return 10 * pair_passes > 16 * solo_passes;
}

int launch_chunk_tc(const SeqArgs &a) {
    if (!chunk_tc_supports(a.d, a.dtype))
        return set_error(RHZ_ERR_SHAPE, "tensor-core kernel needs bf16 and head_dim 128 (got %d)", a.d);
    const int v = g_chunk_variant.load();
    if (v == RHZ_CHUNK_AUTO || v == RHZ_CHUNK_GRID) return launch_chunk_grid(a);
    return v == RHZ_CHUNK_SOLO ? launch_chunk_solo(a) : launch_chunk_pair(a);
}

int launch_chunk_pair(const SeqArgs &a) {
    if (!chunk_tc_supports(a.d, a.dtype))
        return set_error(RHZ_ERR_SHAPE, "tensor-core kernel needs bf16 and head_dim 128 (got %d)", a.d);
    const int64_t tokens = a.cu_seqlens ? a.total_tokens : a.n_seq * a.seq_len;
    if (a.n_seq == 0) return RHZ_OK;
    if (tokens <= 0) {
        // Every sequence is empty: final state = initial state.
        SeqArgs b = a;
        return launch_seq(b);
    }
    if (tokens > INT_MAX - CH)
        return set_error(RHZ_ERR_SHAPE, "tensor-core kernel addresses at most %d token rows (got %lld)",
                         INT_MAX - CH, static_cast<long long>(tokens));
    CUtensorMap tq, tk, tv;
    int st = make_chunk_tmap(&tq, a.q, tokens, a.H);
    if (st == RHZ_OK) st = make_chunk_tmap(&tk, a.k, tokens, a.H);
    if (st == RHZ_OK) st = make_chunk_tmap(&tv, a.v, tokens, a.H);
    if (st != RHZ_OK) return st;
    int sms = 148;
    bool sm100 = true;
    device_info(&sms, &sm100);
    static std::once_flag attr_once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(attr_once, [] {
        attr_err = cudaFuncSetAttribute(gdr_chunk_tc_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(SMEM_ALLOC));
    });
    if (attr_err != cudaSuccess)
        return set_error(RHZ_ERR_DEVICE, "gdr_chunk_tc_kernel smem attribute: %s", cudaGetErrorString(attr_err));
    const int64_t items = a.n_seq * a.H;
    const int64_t max_clusters = sms / 2;
    const int clusters = static_cast<int>(items < max_clusters ? items : max_clusters);
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
    p.norm_scale = a.norm_scale;
    p.norm_eps = a.norm_eps;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = SMEM_ALLOC;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, gdr_chunk_tc_kernel, tq, tk, tv, p);
    if (e != cudaSuccess)
        return set_error(RHZ_ERR_DEVICE, "gdr_chunk_tc_kernel launch: %s", cudaGetErrorString(e));
    return check_launch("gdr_chunk_tc_kernel");
}

}  // namespace rhz
