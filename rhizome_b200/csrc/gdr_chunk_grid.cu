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
// Work split. Everything that depends only on one chunk's keys and gates --
// the decayed [K; Q] K^T, the unit-lower-triangular inverse T, T diag(beta)
// and W -- is independent across chunks; only the products with S form the
// sequential chain of each (sequence, head) item. The kernel is one
// cooperative launch of one CTA per SM in two roles:
//   chains (the first n_chains CTAs): item j, j + n_chains, ... one after
//     the other, S in TMEM (fp32) for the whole sequence, an fp16 image of S
//     in TMEM that the products read as their A operand, and two MMA rounds
//     per chunk:
//       R1: D_U  = V^T (T diag b)^T + S (-W^T)   (128 x 64, = Delta^T)
//           O^T  = S Q~^T                         (128 x 64), Q~ = diag(gamma) Q
//       R2: D_S += Delta^T K~                     (128 x 128), K~ = diag(P[C-1]) K
//           O^T += Delta^T M^T                    (128 x 64)
//     with Delta^T's fp16 image also in TMEM and D_S pre-scaled by
//     gamma_{C-1} while R1 runs. Neither S nor Delta passes through shared
//     memory; O^T leaves through a bf16 [t][i] staging tile. The tiles arrive
//     by TMA one chunk ahead and are converted to fp16 in place (Q and K rows
//     scaled on the way) under the R1 products.
//   producers (the other CTAs): chunk records for every chain, in
//     round-major order (round r of every chain before round r + 1 of any),
//     so all chains are fed evenly. A record is the 32 KB {-W^T, T diag(beta),
//     M = P (Q K^T)} as ready-made fp16 operand images (128-byte swizzle):
//     D1 = [K; Q] K^T (bf16 tiles), A (fp32) and M, the inverse (diagonal
//     16 x 16 tiles by the product formula, the rest by a 2 x 2 recursion on
//     mma.sync), D_W = K^T (T diag(beta gamma))^T on tcgen05.
// Records travel through a ring of RING slots per chain in the caller's
// workspace (L2-resident: a few MB): the producer writes the record's images
// with generic stores and publishes the slot with a release flag; the chain
// acquires the flag, bulk-loads the record into shared memory and releases
// the slot. Each chain's flags sit on their own 128-byte line. Every product
// takes fp16 operands except D1 (A and B of one MMA always share a type);
// fp16 intermediates bound |q.k|, |v|, |S| to < 65504 (unit-norm keys, as
// the reference specifies, keep them far below).
//
// Each chain's result depends only on its own item's inputs and every
// record is computed the same way whichever producer builds it, so outputs
// are batch invariant and bitwise deterministic. Every wait is bounded; a
// timeout sets a sticky device flag and a workspace abort flag that ends the
// other CTAs' waits, drains what is in flight (bounded), frees TMEM and
// returns. No load uses multicast.
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
__device__ int g_grid_status = 0;

namespace {
using namespace sm100;
using namespace chunk;

constexpr int NT = 512;   // threads per CTA (chain: two warpgroups work; producer: two contexts)

constexpr uint32_t KQ_STAGE = 32768;  // producer tiles: [half][K rows | Q rows], 64 x 64 bf16 boxes
constexpr uint32_t KQ_BYTES = 4 * 8192;
constexpr uint32_t KQV_BYTES = 6 * 8192;

// Producer -> chain record: fp16 operand images, 128-byte swizzle, in the
// pieces the chain's bulk copies place next to its own tiles.
constexpr uint32_t REC_W = 0;         // -W [j half][t = 64 rows][64 j]   (K-major rows 64..127 of R1's B)
constexpr uint32_t REC_MT = 16384;    // M^T [s = 64 rows][64 t]           (third MN-major atom of R2's B)
constexpr uint32_t REC_TT = 24576;    // T diag(beta) [t = 64 rows][64 s]  (K-major B of the U product)
constexpr uint32_t REC_BYTES = 32768;


// Chain CTA shared memory: two stages (chunk k in stage k & 1) of
//   B1 [j half][Q~ rows t 0..63 | -W rows t 64..127]   K-major B of R1 (N = 128)
//   B2 [K~ j 0..63 | K~ j 64..127 | M^T] (rows s)      MN-major B of R2 (N = 192, atoms 8 KB apart)
//   V  [i half][rows s]                                 MN-major A of the U product
//   TT T diag(beta) [t][s]                              K-major B of the U product
// The Q, K, V tiles come by TMA, the -W, M^T and T diag(beta) pieces by bulk
// copies from the record ring.
constexpr uint32_t CS_B1 = 0, CS_B2 = 32768, CS_V = 57344, CS_TT = 73728, C_STAGE = 81920;
constexpr uint32_t C_OFF_OST = 2 * C_STAGE;           // O rows of a chunk, bf16 [64 t][128 i] (epilogue staging)
constexpr uint32_t C_OFF_NPART = C_OFF_OST + 16384;   // output norm: per-warp partial sums [4][64], then 1/rms [64]
constexpr uint32_t C_OFF_GATE = C_OFF_NPART + 2048;   // ring of 4 gate tables
constexpr uint32_t C_OFF_BAR = C_OFF_GATE + 4 * G_BYTES;
// Chain barriers: tiles landed [2], record landed [2] (bulk copies from the
// ring), D_U done (R1), all of a chunk's products done (R2), tiles converted
// [2] (warpgroup 1 -> 0), O^T read out and cleared [2] (1 -> 0, by chunk
// parity), a barrier that only the failure path uses to wait for every MMA
// issued, and the state and Delta^T images ready (warpgroup 0 -> MMA warp).
constexpr int CB_LOAD = 0, CB_FULL = 2, CB_R1 = 4, CB_R2 = 6, CB_CONV = 7, CB_OFREE = 9,
              CB_DRAIN = 11, CB_S16 = 12, CB_D16 = 13, CB_NUM = 14;
constexpr uint32_t C_OFF_NORM = C_OFF_BAR + 128;  // output-norm scale, HD floats
constexpr uint32_t C_USED = C_OFF_NORM + HD * 4;
static_assert(C_OFF_NORM >= C_OFF_BAR + CB_NUM * 8 + 16, "chain barriers overlap the norm scale");
static_assert(C_STAGE % 1024 == 0 && CS_TT + 8192 <= C_STAGE, "chain stage map");

// Producer CTA: PCTX independent contexts of 256 threads, each building the
// records of its own task stream in its own slice of shared memory (two
// chunks in flight per SM hide each other's dependent phases).
constexpr int PCTX = 2;
constexpr uint32_t P_OFF_KQ = 0;             // 2 stages of K, Q tiles
constexpr uint32_t P_OFF_AF = 65536;         // A fp32 [64][AST]; after the solve, T diag(beta gamma) as bf16 hi, lo (2 x 8 KB)
constexpr uint32_t P_OFF_TF = P_OFF_AF + 64 * AST * 4;  // T fp32 [64][AST]
constexpr uint32_t P_OFF_X = P_OFF_TF + 64 * AST * 4;   // the solve's scratch (4 KB)
constexpr uint32_t P_OFF_GATE = P_OFF_X + 4096;         // 2 gate tables
constexpr uint32_t P_OFF_BAR = P_OFF_GATE + 2 * G_BYTES;
// Producer barriers (per context): tiles landed [2], D1 done, D_W done,
// failure-path drain of every MMA issued (one per issuing thread).
constexpr int PB_LOAD = 0, PB_D1 = 2, PB_MMA = 3, PB_DRAIN = 4, PB_DRAIN2 = 5, PB_NUM = 6;
constexpr uint32_t P_CTX_BYTES = (P_OFF_BAR + PB_NUM * 8 + 1023) / 1024 * 1024;
constexpr uint32_t P_OFF_TMEM = PCTX * P_CTX_BYTES;     // TMEM base (both contexts)
constexpr uint32_t P_USED = P_OFF_TMEM + 16;
static_assert(P_OFF_TF >= P_OFF_AF + 16384, "T diag(beta gamma) hi + lo must fit the A table");

constexpr uint32_t SMEM_USED = C_USED > P_USED ? C_USED : P_USED;
constexpr size_t SMEM_ALLOC = SMEM_USED + 1024;  // slack for 1024-byte alignment
static_assert(SMEM_ALLOC <= 232448, "exceeds the 227 KB opt-in shared memory");

// TMEM columns (32-bit). Chain: one contiguous accumulator [D_S 128 | O^T 64 |
// D_U 64] (lane i; O^T column t, D_U = Delta^T column s), so that R1 writes
// [O^T | D_U] and R2 writes [D_S | O^T] as single wide products, and the
// fp16 images of S (128 x 128 -> 64 columns) and Delta^T (128 x 64 -> 32
// columns) that the products read as their A operand straight from tensor
// memory. Producer: D1 (128 x 64) and D_W (128 x 64) per context.
constexpr uint32_t TM_DS = 0, TM_OT = 128, TM_DU = 192, TM_S16 = 256, TM_D16 = 320, C_TM_COLS = 512;
constexpr uint32_t TM_D1 = 0, TM_W = 64, P_TM_CTX = 128, P_TM_COLS = PCTX * P_TM_CTX;

constexpr uint32_t ID_D1 = idesc_bf16(128, 64, false, false);
constexpr uint32_t ID_MK64 = idesc_f16(128, 64, true, false);
constexpr uint32_t ID_MK64_BF = idesc_bf16(128, 64, true, false);
constexpr uint32_t ID_R1 = idesc_f16(128, 128, false, false);  // S [Q~ | -W]^T: A from TMEM, B K-major
constexpr uint32_t ID_R2 = idesc_f16(128, 192, false, true);   // Delta^T [K~ | M^T]: B MN-major

// Record ring: RING slots of REC_BYTES per chain; flags in the workspace.
constexpr int RING = 8;
// Each chain's flags (ready[RING], consumed) sit on their own 128-byte line:
// producers ahead of the chains poll them, and lines shared by several
// chains turned those polls into one L2 hot spot.
constexpr int FLAG_STRIDE = 32;
static_assert(RING <= FLAG_STRIDE, "a chain's ready flags fit its line");
constexpr int MAX_CHAINS = 128;

struct GParams {
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
    // grid
    uint8_t *ring;        // [n_chains][RING][REC_BYTES]
    int *ready;           // [n_chains][FLAG_STRIDE]: round + 1 of the record ring slot i holds (i < RING)
    int *consumed;        // [n_chains][FLAG_STRIDE]: rounds the chain has taken out of its ring
    int *abort_flag;      // set by any CTA whose bounded wait ran out
    const int32_t *off;   // packed streams: [items] first round of each item in its chain
    const int32_t *sched; // packed streams: [0] rounds of the longest chain, [1 + j] rounds of chain j
    const int32_t *order; // packed streams: sequences by chunk count, longest first (null: as given)
    int snake;            // chains take positions in snake order (packed streams)
    int n_chains;
    int n_prod;           // producer CTAs
    uint64_t poll_ns;     // bound of every wait on another CTA's flag
    int never_ready;      // test hook: chains wait for a record flag no producer sets
};

// One fp16 element at (row r, column e) of a block of 128-byte rows of 64
// columns stored with the 128-byte swizzle.
__device__ __forceinline__ void st_sw_f16(uint8_t *blk, int r, int e, float v) {
    *reinterpret_cast<__half *>(blk + r * 128 + (((e >> 3) ^ (r & 7)) << 4) + (e & 7) * 2) =
        __float2half_rn(v);
}

// The same place, given the fp16 bits.
__device__ __forceinline__ void st_sw_h(uint8_t *blk, int r, int e, uint16_t h) {
    *reinterpret_cast<uint16_t *>(blk + r * 128 + (((e >> 3) ^ (r & 7)) << 4) + (e & 7) * 2) = h;
}

// Two floats as an fp16 pair (round to nearest even; the first in the low half).
__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Chain: parts P0 .. P1 - 1 of one stage's Q, K and V tiles (16 KB each)
// bf16 -> fp16 in place, Q rows (in B1) scaled by gamma_t and K rows (in B2)
// by P[C-1][s]. The stage holds 3072 16-byte chunks: Q (B1 half h, rows
// 0..63), K (B2, contiguous), V; this thread's are first, first + STRIDE,
// ... The swizzle permutes chunks within a row only, so a chunk's row (and
// scale) follows from its index.
template <int STRIDE, int P0, int P1>
__device__ __forceinline__ void chain_tiles_to_f16(uint8_t *stage, const float *gm, const float *pl,
                                                   int first) {
    static_assert(1024 % (8 * STRIDE) == 0, "batches of 8 chunks");
#pragma unroll 1
    for (int part = P0; part < P1; ++part) {
#pragma unroll 1
        for (int b = 0; b < 1024 / STRIDE; b += 8) {
            uint4 x[8];
            uint8_t *ad[8];
            float sc[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const int i = first + (b + m) * STRIDE;  // chunk within the part
                const int r = (i >> 3) & 63;
                if (part == 0) {
                    ad[m] = stage + CS_B1 + (i >> 9) * 16384 + r * 128 + (i & 7) * 16;
                    sc[m] = gm[r];
                } else if (part == 1) {
                    ad[m] = stage + CS_B2 + i * 16;
                    sc[m] = pl[r];
                } else {
                    ad[m] = stage + CS_V + i * 16;
                    sc[m] = 1.f;
                }
                x[m] = *reinterpret_cast<const uint4 *>(ad[m]);
            }
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                uint4 w = x[m];
                w.x = bf16x2_to_f16x2(w.x, sc[m]);
                w.y = bf16x2_to_f16x2(w.y, sc[m]);
                w.z = bf16x2_to_f16x2(w.z, sc[m]);
                w.w = bf16x2_to_f16x2(w.w, sc[m]);
                *reinterpret_cast<uint4 *>(ad[m]) = w;
            }
        }
    }
}

struct Ref {
    int64_t item, ts;  // item < 0: no chunk
    int L, h;
    int r, j;          // producer tasks: round and chain
    int64_t m;         // the item's place in its chain's sequence
};

// The chunks chain j processes, in order: the items at positions
// pos(j, 0), pos(j, 1), ... and within an item its chunks of CH positions
// from the sequence start; the k-th chunk is the chain's round k and uses
// tile stage, record slot and gate table k & 1 (k & 3 for gate tables).
// Dense batches: position q is item q and chain j takes j, j + NC, ...
// Packed streams (lengths differ): position q is the item of the
// (q / H)-th longest sequence (`order`, longest first) and head q % H, and
// the chains take positions in snake order (row m of NC positions left to
// right when m is even, right to left when odd), which spreads the long
// sequences evenly over the chains.
struct Walk {
    const GParams *p;
    int64_t n_items, stride;
    int H;

    __device__ int64_t pos(int j, int64_t m) const {
        if (!p->snake) return j + m * stride;
        return m * stride + ((m & 1) ? stride - 1 - j : j);
    }
    __device__ int64_t item_at(int64_t q) const {
        if (!p->order) return q;
        return static_cast<int64_t>(p->order[q / H]) * H + q % H;
    }
    // Number of items chain j takes.
    __device__ int64_t count(int j) const {
        const int64_t full = n_items / stride;
        return full + ((full * stride < n_items && pos(j, full) < n_items) ? 1 : 0);
    }

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
    // First chunk of chain j's items at or after place m (skipping empty sequences).
    __device__ Ref first_from(int j, int64_t m) const {
        for (;; ++m) {
            const int64_t q = pos(j, m);
            if (q >= n_items) break;
            const int64_t it = item_at(q);
            int64_t t0, t1;
            bounds(it, t0, t1);
            if (t1 > t0) {
                const int64_t seq = it / H;
                return Ref{it, t0, static_cast<int>((t1 - t0) < CH ? (t1 - t0) : CH),
                           static_cast<int>(it - seq * H), 0, j, m};
            }
        }
        return Ref{-1, 0, 0, 0, 0, j, 0};
    }
    __device__ Ref next_of(const Ref &r) const {
        int64_t t0, t1;
        bounds(r.item, t0, t1);
        const int64_t tn = r.ts + CH;
        if (tn < t1)
            return Ref{r.item, tn, static_cast<int>((t1 - tn) < CH ? (t1 - tn) : CH), r.h, 0, r.j, r.m};
        return first_from(r.j, r.m + 1);
    }
    // The chunk n steps after chunk c of chain j's item at place m (bounds
    // [t0, t1), nch chunks, head h): arithmetic inside the item, the walk
    // only past its end (once per item rather than once per chunk).
    __device__ Ref after(int j, int64_t m, int64_t item, int h, int64_t t0, int64_t t1, int nch, int c,
                         int n) const {
        const int cc = c + n;
        if (cc < nch) {
            const int64_t ts = t0 + static_cast<int64_t>(cc) * CH;
            return Ref{item, ts, static_cast<int>((t1 - ts) < CH ? (t1 - ts) : CH), h, 0, j, m};
        }
        Ref r = first_from(j, m + 1);
        for (int i = nch; i < cc && r.item >= 0; ++i) r = next_of(r);
        return r;
    }
};

// Producer tasks in round-major order: task t is round t / n_chains of chain
// t % n_chains. Dense batches (every item has nch chunks) map a round to its
// item by arithmetic; packed streams use the per-position round offsets
// `off` that gdr_grid_sched_kernel computed (the item is the chain's last
// one whose offset is <= r; an empty item shares its offset with the next
// item, which comes later in the chain, so the search never lands on it).
struct Sched {
    const GParams *p;
    const Walk *wk;
    int64_t n_items;
    int NC;
    int nch;       // dense: chunks per item; 0: packed stream (tables)
    int64_t n_tasks;

    __device__ int rounds(int j) const {
        if (nch > 0) return static_cast<int>(wk->count(j) * nch);
        return p->sched[1 + j];
    }
    // Task t, or item < 0 if that chain has no round t / NC.
    __device__ Ref at(int64_t t) const {
        const int r = static_cast<int>(t / NC), j = static_cast<int>(t - static_cast<int64_t>(r) * NC);
        Ref out{-1, 0, 0, 0, r, j, 0};
        if (r >= rounds(j)) return out;
        int64_t item;
        int c;
        if (nch > 0) {
            const int m = r / nch;
            c = r - m * nch;
            item = wk->item_at(wk->pos(j, m));
        } else {
            int64_t lo = 0, hi = wk->count(j) - 1;  // largest m with off <= r
            while (lo < hi) {
                const int64_t mid = (lo + hi + 1) >> 1;
                if (p->off[wk->pos(j, mid)] <= r) lo = mid; else hi = mid - 1;
            }
            const int64_t q = wk->pos(j, lo);
            item = wk->item_at(q);
            c = r - p->off[q];
        }
        int64_t t0, t1;
        wk->bounds(item, t0, t1);
        const int64_t seq = item / p->H;
        out.item = item;
        out.ts = t0 + static_cast<int64_t>(c) * CH;
        out.L = static_cast<int>((t1 - out.ts) < CH ? (t1 - out.ts) : CH);
        out.h = static_cast<int>(item - seq * p->H);
        return out;
    }
    // The first non-empty task at or after t among t, t + step, ...
    __device__ Ref first_from(int64_t t, int64_t step) const {
        for (; t < n_tasks; t += step) {
            const Ref r = at(t);
            if (r.item >= 0) return r;
        }
        return Ref{-1, 0, 0, 0, 0, 0, 0};
    }
};

__device__ __forceinline__ GateIn gate_load(const GParams &p, const Ref &r, int lane) {
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
// converted and O^T of chunk k - 1 read out -> R1 -> Delta^T -> R2 -> state
// refresh. A dependent run of MMAs into one accumulator costs about the same
// per instruction for N = 64 ... 192 on B200, so each round is one wide
// product over the contiguous [D_S | O^T | D_U] accumulator: R1 (8 steps,
// N = 128) and R2 (4 steps, N = 192). Warpgroup 1 works beside it: gate
// tables two chunks ahead, the fp16 conversion of chunk k + 1's tiles under
// chunk k's products, and, once R2(k) is done, the loads of chunk k + 2 into
// stage k & 1 and the O rows of chunk k. Every barrier phase has a single
// producer and is consumed before it can be reused, so parities never alias.
__device__ __forceinline__ RoleState chain_role(const CUtensorMap *tm_q, const CUtensorMap *tm_k,
                                                const CUtensorMap *tm_v, const GParams &p,
                                                uint8_t *smem, const Walk &wk, int64_t start,
                                                uint32_t tmem) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ww = warp & 3;
    const uint32_t trow = tmem + (static_cast<uint32_t>(ww) << 21);  // lanes 32 ww .. 32 ww + 31
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C_OFF_BAR);
    uint64_t *bar_load = bars + CB_LOAD, *bar_full = bars + CB_FULL, *bar_r1 = bars + CB_R1,
             *bar_r2 = bars + CB_R2, *bar_conv = bars + CB_CONV, *bar_ofree = bars + CB_OFREE,
             *bar_s16 = bars + CB_S16, *bar_d16 = bars + CB_D16;
    const uint32_t sbase = smem_u32(smem);
    const int H = p.H;
    const int64_t tok_stride = static_cast<int64_t>(H) * HD;
    auto gates = [&](int kc) { return reinterpret_cast<float *>(smem + C_OFF_GATE) + (kc & 3) * G_SIZE; };
    auto stage = [&](int kc) { return sbase + (kc & 1) * C_STAGE; };
    const int chain = static_cast<int>(start);
    int *consumed = p.consumed + chain * FLAG_STRIDE;
    RoleState rs{false};

    if (tid < 128) {
        // ------------------------------------------------ warpgroup 0: state path
        // Moves the state and Delta^T between their fp32 accumulators and the
        // fp16 images the products read; the MMA warp issues the products.
        const int row = tid;  // state row i = TMEM lane
        int k = 0;
        // O^T starts at zero: R1 accumulates onto it (warpgroup 1 clears it
        // again after reading each chunk's rows); ordered before the first
        // R1 by the first state-image arrival.
        {
            uint32_t z[32];
#pragma unroll
            for (int e = 0; e < 32; ++e) z[e] = 0u;
            tmem_st32u(trow + TM_OT, z);
            tmem_st32u(trow + TM_OT + 32, z);
            tmem_wait_st();
        }
        // This warpgroup converts the K and V tiles of chunks 1, 2, ... and
        // the V tile of chunk 0 (warpgroup 1, busy with the O rows and the
        // records, converts every Q tile and chunk 0's K): chunk kc's, once its
        // tiles landed, into stage kc & 1, then its share of that chunk's
        // conversion barrier. K's scale (P[C-1]) is in chunk kc's gate table,
        // which warpgroup 1 wrote before its conversion arrival for chunk
        // kc - 1, which this warpgroup has waited for.
        auto convert_kv = [&](int kc) -> bool {
            const bool ok = mbar_wait(&bar_load[kc & 1], (kc >> 1) & 1, p.poll_ns);
            if (wg_sync_or(1, !ok)) return false;
            if (kc == 0)
                chain_tiles_to_f16<128, 2, 3>(smem, nullptr, nullptr, row);
            else
                chain_tiles_to_f16<128, 1, 3>(smem + (kc & 1) * C_STAGE, nullptr, gates(kc) + G_PL, row);
            fence_proxy_async_smem();
            mbar_arrive(&bar_conv[kc & 1]);
            return true;
        };
        if (wk.first_from(chain, 0).item >= 0 && !convert_kv(0)) rs.failed = true;
        for (int64_t m = 0; !rs.failed; ++m) {
            const int64_t q = wk.pos(chain, m);
            if (q >= wk.n_items) break;
            const int64_t item = wk.item_at(q);
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
                // Chunk k's gate table (gamma) is in once warpgroup 1 has
                // converted its tiles: it builds the tables ahead of that.
                {
                    const bool ok = mbar_wait(&bar_conv[k & 1], (k >> 1) & 1, p.poll_ns);
                    if (wg_sync_or(1, !ok)) { rs.failed = true; break; }
                }
                // ---- first chunk of the item: fp16 image of S0 (unscaled) and
                // D_S = gamma_{C-1} S0 (the previous item's products are done)
                if (c == 0) {
                    const float gC = gates(k)[G_GM + 63];
#pragma unroll 1
                    for (int h2 = 0; h2 < 2; ++h2) {
                        uint32_t w[32];
#pragma unroll
                        for (int q2 = 0; q2 < 2; ++q2) {
                            float v[32];
#pragma unroll
                            for (int e = 0; e < 32; e += 4) {
                                const float4 f = have ? *reinterpret_cast<const float4 *>(src + 64 * h2 + 32 * q2 + e)
                                                      : make_float4(0.f, 0.f, 0.f, 0.f);
                                v[e] = f.x; v[e + 1] = f.y; v[e + 2] = f.z; v[e + 3] = f.w;
                            }
#pragma unroll
                            for (int e = 0; e < 16; ++e) w[16 * q2 + e] = pack_f16x2(v[2 * e], v[2 * e + 1]);
#pragma unroll
                            for (int e = 0; e < 32; ++e) v[e] *= gC;
                            tmem_st32(trow + TM_DS + 64 * h2 + 32 * q2, v);
                        }
                        tmem_st32u(trow + TM_S16 + 32 * h2, w);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    mbar_arrive(bar_s16);
                } else {
                    // ---- D_S pre-scaled by this chunk's gamma_{C-1} while R1
                    // runs (R1 does not touch D_S; R2, which accumulates into
                    // it, waits for this thread's Delta^T arrival below)
                    tc_fence_after();
                    const float gC = gates(k)[G_GM + 63];
#pragma unroll 1
                    for (int q4 = 0; q4 < 4; ++q4) {
                        float v[32];
                        tmem_ld32(trow + TM_DS + 32 * q4, v);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) v[e] *= gC;
                        tmem_st32(trow + TM_DS + 32 * q4, v);
                    }
                    tmem_wait_st();
                }
                bool ok = mbar_wait(bar_r1, k & 1, p.poll_ns);
                if (wg_sync_or(1, !ok)) { rs.failed = true; break; }
                tc_fence_after();

                // ---- Delta^T (fp16) into its TMEM image: row i, all 64 positions
                {
                    float x[32], y[32];
                    tmem_ld32(trow + TM_DU, x);
                    tmem_ld32(trow + TM_DU + 32, y);
                    tmem_wait_ld();
                    uint32_t w[32];
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        w[e] = pack_f16x2(x[2 * e], x[2 * e + 1]);
                        w[16 + e] = pack_f16x2(y[2 * e], y[2 * e + 1]);
                    }
                    tmem_st32u(trow + TM_D16, w);
                    tmem_wait_st();
                }
                tc_fence_before();
                mbar_arrive(bar_d16);
                ok = mbar_wait(bar_r2, k & 1, p.poll_ns);
                if (wg_sync_or(1, !ok)) { rs.failed = true; break; }
                tc_fence_after();

                // ---- state: the fp16 image the next chunk's R1 reads (its only
                // wait on this chunk), or the final state
                if (c + 1 < nch) {
#pragma unroll 1
                    for (int h2 = 0; h2 < 2; ++h2) {
                        float v[32], x[32];
                        tmem_ld32(trow + TM_DS + 64 * h2, v);
                        tmem_ld32(trow + TM_DS + 64 * h2 + 32, x);
                        tmem_wait_ld();
                        uint32_t w[32];
#pragma unroll
                        for (int e = 0; e < 16; ++e) {
                            w[e] = pack_f16x2(v[2 * e], v[2 * e + 1]);
                            w[16 + e] = pack_f16x2(x[2 * e], x[2 * e + 1]);
                        }
                        tmem_st32u(trow + TM_S16 + 32 * h2, w);
                    }
                    tmem_wait_st();
                    tc_fence_before();
                    mbar_arrive(bar_s16);
                } else if (dst) {
#pragma unroll 1
                    for (int q4 = 0; q4 < 4; ++q4) {
                        float v[32];
                        tmem_ld32(trow + TM_DS + 32 * q4, v);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; e += 4)
                            *reinterpret_cast<float4 *>(dst + 32 * q4 + e) =
                                make_float4(v[e], v[e + 1], v[e + 2], v[e + 3]);
                    }
                }
                // ---- the next chunk's K and V tiles (under the next R1's other waits)
                if (wk.after(chain, m, item, h, t0, t1, nch, c, 1).item >= 0 && !convert_kv(k + 1)) {
                    rs.failed = true;
                    break;
                }
            }
        }
    } else if (tid == 256) {
        // ------------------------------------------------ MMA warp (one thread)
        // Issues every product of the chain, so that a thread held up by a
        // full MMA queue holds up no warpgroup.
        int k = 0;
        bool u_pre = false;  // the next R1's U part is already issued
        // D_U = V^T (T diag b)^T (starts D_U; R1 accumulates onto it)
        auto issue_u = [&](uint32_t st) {
#pragma unroll 1
            for (int kk = 0; kk < 4; ++kk)
                umma_f16(tmem + TM_DU, sdesc_sw128(st + CS_V + kk * 2048, 8192, 1024),
                         sdesc_sw128(st + CS_TT + kk * 32, 16, 1024), ID_MK64, kk > 0);
        };
        for (int64_t m = 0; !rs.failed; ++m) {
            const int64_t q = wk.pos(chain, m);
            if (q >= wk.n_items) break;
            const int64_t item = wk.item_at(q);
            int64_t t0, t1;
            wk.bounds(item, t0, t1);
            const int nch = static_cast<int>((t1 - t0 + CH - 1) / CH);
            for (int c = 0; c < nch; ++c, ++k) {
                const uint32_t st = stage(k);
                // ---- R1's inputs: record k (its ring slot is free again once
                // it has landed), tiles k in fp16, O^T of chunk k - 1 read out
                // and cleared, S's fp16 image
                bool ok = mbar_wait(&bar_full[k & 1], (k >> 1) & 1, p.poll_ns);
                ok = ok && mbar_wait(&bar_conv[k & 1], (k >> 1) & 1, p.poll_ns);
                if (k >= 1) ok = ok && mbar_wait(&bar_ofree[(k - 1) & 1], ((k - 1) >> 1) & 1, p.poll_ns);
                ok = ok && mbar_wait(bar_s16, k & 1, p.poll_ns);
                if (!ok) { rs.failed = true; break; }
                tc_fence_after();
                // ---- R1: [O^T | D_U] += S [Q~ | -W]^T, one N = 128 product (S
                // read from its fp16 image in TMEM; D_U starts as the U part)
                if (!u_pre) issue_u(st);
#pragma unroll 1
                for (int kk = 0; kk < 8; ++kk)
                    umma_f16_ta(tmem + TM_OT, tmem + TM_S16 + 8 * kk,
                                sdesc_sw128(st + CS_B1 + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024),
                                ID_R1, 1);
                umma_commit(bar_r1);
                // The record's ring slot is free again: the bulk copies that
                // read it completed before this thread's (acquiring) wait on
                // bar_full, so a relaxed store publishes it; a release store's
                // GPU-scope fence cost ~1,200-2,000 cycles on this path.
                st_relaxed_gpu(consumed, k + 1);
                // ---- R2: [D_S | O^T] += Delta^T [K~ | M^T] (one N = 192 product)
                if (!mbar_wait(bar_d16, k & 1, p.poll_ns)) { rs.failed = true; break; }
                tc_fence_after();
#pragma unroll 1
                for (int kk = 0; kk < 4; ++kk)
                    umma_f16_ta(tmem + TM_DS, tmem + TM_D16 + 8 * kk,
                                sdesc_sw128(st + CS_B2 + kk * 2048, 8192, 1024), ID_R2, 1);
                umma_commit(bar_r2);
                // ---- the next chunk's U part, under the state refresh (D_U
                // was read out before Delta^T's arrival)
                u_pre = false;
                if (c + 1 < nch) {
                    const int kn = k + 1;
                    ok = mbar_wait(&bar_full[kn & 1], (kn >> 1) & 1, p.poll_ns) &&
                         mbar_wait(&bar_conv[kn & 1], (kn >> 1) & 1, p.poll_ns);
                    if (!ok) { rs.failed = true; break; }
                    tc_fence_after();
                    issue_u(stage(kn));
                    u_pre = true;
                }
            }
        }
        if (rs.failed) {
            // Every MMA issued completes before TMEM is released.
            umma_commit(bars + CB_DRAIN);
            mbar_wait(bars + CB_DRAIN, 0, 200000000ull);
        }
    } else if (tid < 256) {
        // ------------------------------------------------ warpgroup 1: tiles, epilogue
        const int wt = tid - 128;
        int loads_issued = 0, loads_waited = 0, recs_issued = 0;
        bool rec_pending = false;  // thread 0: the next chunk's record not fetched yet
        // Round kc's record: wait until a producer has published it in ring
        // slot kc % RING, then bulk-copy its pieces next to stage kc & 1's tiles.
        // (blocking: waits, bounded, for the record; otherwise returns at once
        // with *fetched = false when it is not published yet)
        auto fetch_record = [&](int kc, bool blocking = true, bool *fetched = nullptr) -> bool {
            const int slot = kc % RING;
            const int target = p.never_ready ? kc + 1 + (1 << 30) : kc + 1;
            if (!blocking) {
                *fetched = ld_acquire_gpu(p.ready + chain * FLAG_STRIDE + slot) >= target;
                if (!*fetched) return true;
            } else if (!poll_ge(p.ready + chain * FLAG_STRIDE + slot, target, p.abort_flag, p.poll_ns)) {
                return false;
            }
            fence_proxy_async_global();
            uint64_t *bar = &bar_full[kc & 1];
            uint8_t *stp = smem + (kc & 1) * C_STAGE;
            const uint8_t *rec = p.ring + (static_cast<size_t>(chain) * RING + slot) * REC_BYTES;
            mbar_arrive_expect_tx(bar, REC_BYTES);
            bulk_load_g2s(stp + CS_B1 + 8192, rec + REC_W, 8192, bar);
            bulk_load_g2s(stp + CS_B1 + 16384 + 8192, rec + REC_W + 8192, 8192, bar);
            bulk_load_g2s(stp + CS_B2 + 16384, rec + REC_MT, 8192, bar);
            bulk_load_g2s(stp + CS_TT, rec + REC_TT, 8192, bar);
            ++recs_issued;
            return true;
        };
        GateIn gin{1.f, 1.f, 0.f, 0.f};  // warp 4: inputs of the gate table two chunks ahead
        auto issue_loads = [&](int kc, const Ref &r) {
            uint64_t *bar = &bar_load[kc & 1];
            uint8_t *stp = smem + (kc & 1) * C_STAGE;
            mbar_arrive_expect_tx(bar, KQV_BYTES);
            const int t32 = static_cast<int>(r.ts);
            tma_load_3d(stp + CS_B1, tm_q, 0, r.h, t32, bar);
            tma_load_3d(stp + CS_B1 + 16384, tm_q, 64, r.h, t32, bar);
            tma_load_3d(stp + CS_B2, tm_k, 0, r.h, t32, bar);
            tma_load_3d(stp + CS_B2 + 8192, tm_k, 64, r.h, t32, bar);
            tma_load_3d(stp + CS_V, tm_v, 0, r.h, t32, bar);
            tma_load_3d(stp + CS_V + 8192, tm_v, 64, r.h, t32, bar);
        };
        // Q tiles (chunk 0: Q and K; warpgroup 0 converts the rest).
        auto convert = [&](int kc) {
            const float *g = gates(kc);
            if (kc == 0)
                chain_tiles_to_f16<128, 0, 2>(smem, g + G_GM, g + G_PL, wt);
            else
                chain_tiles_to_f16<128, 0, 1>(smem + (kc & 1) * C_STAGE, g + G_GM, nullptr, wt);
            fence_proxy_async_smem();
        };

        float *nsc = reinterpret_cast<float *>(smem + C_OFF_NORM);
        const bool norm = p.norm_scale != nullptr;
        if (norm) nsc[wt] = p.norm_scale[wt];  // wt < 128 = HD
        {
            const Ref r0 = wk.first_from(chain, 0);
            const Ref r1 = r0.item >= 0 ? wk.next_of(r0) : r0;
            const Ref r2 = r1.item >= 0 ? wk.next_of(r1) : r1;
            bool fok = true;
            if (wt == 0) {
                if (r0.item >= 0) issue_loads(0, r0);
                if (r1.item >= 0) issue_loads(1, r1);
                if (r0.item >= 0) fok = fetch_record(0);
                if (fok && r1.item >= 0) fok = fetch_record(1);
            }
            loads_issued = (r0.item >= 0) + (r1.item >= 0);
            if (wg_sync_or(2, !fok)) rs.failed = true;
            if (ww == 0) {
                gate_tables(gates(0), gate_load(p, r0, lane), lane);
                gate_tables(gates(1), gate_load(p, r1, lane), lane);
                gin = gate_load(p, r2, lane);
            }
            if (r0.item >= 0 && !rs.failed) {
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
        for (int64_t m = 0; !rs.failed; ++m) {
            const int64_t q = wk.pos(chain, m);
            if (q >= wk.n_items) break;
            const int64_t item = wk.item_at(q);
            const int64_t seq = item / H;
            const int h = static_cast<int>(item - seq * H);
            int64_t t0, t1;
            wk.bounds(item, t0, t1);
            const int nch = static_cast<int>((t1 - t0 + CH - 1) / CH);
            for (int c = 0; c < nch; ++c, ++k) {
                const int64_t ts = t0 + static_cast<int64_t>(c) * CH;
                const int L = static_cast<int>((t1 - ts) < CH ? (t1 - ts) : CH);
                const Ref nxt = wk.after(chain, m, item, h, t0, t1, nch, c, 1);
                const Ref nn = wk.after(chain, m, item, h, t0, t1, nch, c, 2);

                // ---- gate table of chunk k + 2, then the inputs of chunk k + 3
                if (nn.item >= 0 && ww == 0) {
                    gate_tables(gates(k + 2), gin, lane);
                    gin = gate_load(p, wk.after(chain, m, item, h, t0, t1, nch, c, 3), lane);
                }
                // ---- chunk k + 1's tiles -> fp16 (under chunk k's products)
                if (nxt.item >= 0) {
                    const bool ok = mbar_wait(&bar_load[(k + 1) & 1], ((k + 1) >> 1) & 1);
                    if (wg_sync_or(2, !ok)) { rs.failed = true; break; }
                    ++loads_waited;
                    convert(k + 1);
                    mbar_arrive(&bar_conv[(k + 1) & 1]);
                }
                // ---- chunk k's products are done
                {
                    const bool ok = mbar_wait(bar_r2, k & 1);
                    if (wg_sync_or(2, !ok)) { rs.failed = true; break; }
                    tc_fence_after();
                }
                // Stage k & 1 is free again: chunk k + 2's tiles now, its
                // record after chunk k's O rows (below).
                if (wt == 0 && nn.item >= 0) issue_loads(k + 2, nn);
                if (nn.item >= 0) ++loads_issued;

                // ---- O rows of chunk k from O^T (lane i, column t), optionally
                // RMS-normalised per head first (groupnorm_heads, norm.rs:48-60,
                // on the fp32 accumulator): each thread turns its column i into
                // bf16 in a [t][i] staging tile and clears O^T for the next
                // chunk, then the rows go out as 16-byte stores.
                {
                    const uint32_t tOT = trow + TM_OT;
                    float *npart = reinterpret_cast<float *>(smem + C_OFF_NPART);
                    float *ninv = npart + 4 * 64;
                    if (norm) {
                        // sum over i of o[t][i]^2 for every t: a transposing
                        // butterfly over the warp's 32 lanes (lane l ends with
                        // t = 2l, 2l + 1), then the four warps through shared memory
                        float r[32];
                        {
                            float x[32], y[32];
                            tmem_ld32(tOT, x);
                            tmem_ld32(tOT + 32, y);
                            tmem_wait_ld();
                            const bool up = lane & 16;
#pragma unroll
                            for (int j = 0; j < 32; ++j) {
                                const float sx = x[j] * x[j], sy = y[j] * y[j];
                                r[j] = (up ? sy : sx) + __shfl_xor_sync(0xffffffffu, up ? sx : sy, 16);
                            }
                        }
#pragma unroll
                        for (int step = 0; step < 4; ++step) {
                            const int m = 8 >> step, n = 16 >> step;
                            const bool up = lane & m;
#pragma unroll
                            for (int j = 0; j < 16; ++j) {
                                if (j < n) {
                                    const float lo = r[j], hi = r[j + n];
                                    r[j] = (up ? hi : lo) + __shfl_xor_sync(0xffffffffu, up ? lo : hi, m);
                                }
                            }
                        }
                        npart[ww * 64 + 2 * lane] = r[0];
                        npart[ww * 64 + 2 * lane + 1] = r[1];
                        wg_sync(2);
                        if (wt < 64) {
                            const float ss = npart[wt] + npart[64 + wt] + npart[128 + wt] + npart[192 + wt];
                            ninv[wt] = 1.f / sqrtf(ss / static_cast<float>(HD) + p.norm_eps);
                        }
                        wg_sync(2);
                    }
                    uint16_t *stg = reinterpret_cast<uint16_t *>(smem + C_OFF_OST);
                    const float sc = norm ? nsc[wt] : 1.f;
#pragma unroll 1
                    for (int hf = 0; hf < 2; ++hf) {
                        float x[32];
                        tmem_ld32(tOT + 32 * hf, x);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const int t = 32 * hf + j;
                            const float v = norm ? x[j] * ninv[t] * sc : x[j];
                            stg[t * HD + wt] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
                        }
                    }
                    {
                        uint32_t z[32];
#pragma unroll
                        for (int e = 0; e < 32; ++e) z[e] = 0u;
                        tmem_st32u(tOT, z);
                        tmem_st32u(tOT + 32, z);
                        tmem_wait_st();
                    }
                    tc_fence_before();
                    mbar_arrive(&bar_ofree[k & 1]);
                    wg_sync(2);
                    __nv_bfloat16 *orow = p.o + ts * tok_stride + static_cast<int64_t>(h) * HD;
#pragma unroll
                    for (int c8 = 0; c8 < 8; ++c8) {
                        const int idx = wt + 128 * c8, t = idx >> 4, ch = idx & 15;
                        if (t < L)
                            *reinterpret_cast<uint4 *>(orow + t * tok_stride + 8 * ch) =
                                *reinterpret_cast<const uint4 *>(stg + t * HD + 8 * ch);
                    }
                }
                // ---- records. Chunk k + 1's, if it was not published when
                // last tried: now it is needed (the next R1 waits for it), so
                // wait for it. Chunk k + 2's into stage k & 1: taken if it is
                // published, else left for the end of the next chunk, so that
                // a late record holds up neither chunk k + 1's tile conversion
                // nor chunk k + 1's O rows. Thread 0 alone tracks the pending
                // record. (The barrier also keeps the staging tile's next
                // writes after this chunk's reads.)
                {
                    bool fok = true;
                    if (wt == 0) {
                        if (rec_pending) {
                            fok = fetch_record(k + 1);
                            rec_pending = false;
                        }
                        if (fok && nn.item >= 0) {
                            bool fetched = false;
                            fok = fetch_record(k + 2, false, &fetched);
                            rec_pending = !fetched;
                        }
                    }
                    if (wg_sync_or(2, !fok)) { rs.failed = true; break; }
                }
            }
        }
        if (rs.failed && wt == 0) {
            // Tile loads and record copies still in flight land before the
            // shared memory goes away.
            for (int kk = loads_waited; kk < loads_issued; ++kk)
                mbar_wait(&bar_load[kk & 1], (kk >> 1) & 1, 200000000ull);
            for (int kk = (recs_issued > 2 ? recs_issued - 2 : 0); kk < recs_issued; ++kk)
                mbar_wait(&bar_full[kk & 1], (kk >> 1) & 1, 200000000ull);
        }
    }
    if (rs.failed) {
        atomicExch(&g_grid_status, 1);
        atomicExch(p.abort_flag, 1);
    }
    rs.failed = __syncthreads_or(rs.failed);
    return rs;
}

// ------------------------------------------------------------------ producer CTA
//
// One context (256 threads, its own slice of shared memory, TMEM columns and
// named barrier) builds the records of its tasks one after the other: chunk
// k's record while the tiles of chunk k + 1 land and its D1 runs. A record is
// written straight into its ring slot (generic stores of the swizzled fp16
// images) once the chain has taken round r - RING out of that slot, and
// published with a release flag when complete. Thread 128, whose warp has no
// block in the A / M phase, publishes each record and then checks the next
// record's slot, under that phase; the phase's closing barrier carries its
// answer, and nothing writes the slot before it. A record is therefore always
// published before its producer waits on any chain.
__device__ __forceinline__ RoleState producer_role(const CUtensorMap *tm_q, const CUtensorMap *tm_k,
                                                   const GParams &p, uint8_t *smem, const Sched &sc,
                                                   int64_t start, int64_t step, uint32_t tmem,
                                                   int lt, int bar_id) {
    const int warp = lt >> 5, lane = lt & 31;
    const int row = 32 * (warp & 3) + lane;  // TMEM lane
    const int half = warp >> 2;              // column half of this thread
    const uint32_t trow = tmem + (static_cast<uint32_t>(warp & 3) << 21);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + P_OFF_BAR);
    uint64_t *bar_load = bars + PB_LOAD, *bar_d1 = bars + PB_D1, *bar_mma = bars + PB_MMA;
    float *Af = reinterpret_cast<float *>(smem + P_OFF_AF);
    float *Tf = reinterpret_cast<float *>(smem + P_OFF_TF);
    float *Xf = reinterpret_cast<float *>(smem + P_OFF_X);
    uint8_t *th = smem + P_OFF_AF;  // T diag(beta gamma) hi, lo: the A table is dead by then
    const uint32_t sbase = smem_u32(smem);
    auto csync = [&]() { nbar_sync(bar_id, 256); };
    auto csync_or = [&](bool x) { return nbar_sync_or(bar_id, 256, x); };
    auto task_of = [&](const Ref &r) { return static_cast<int64_t>(r.r) * sc.NC + r.j; };
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
    // The MMA-issue loops stay rolled: the per-chunk code is larger than the
    // instruction cache keeps warm, and a rolled issue loop (one thread, eight
    // MMAs) costs nothing on the critical path while unrolled copies cost
    // instruction-fetch stalls.
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
    int slot_seen = INT_MIN;  // thread 128: consumed flag of the next record's chain, read early
    int k = 0;
    GateIn gin{1.f, 1.f, 0.f, 0.f};  // warp 4: inputs of the next chunk's gate table
    Ref cur = sc.first_from(start, step);
    Ref nxt = cur.item >= 0 ? sc.first_from(task_of(cur) + step, step) : cur;
    if (cur.item >= 0) {
        if (lt == 0) {
            issue_loads(0, cur);
            if (nxt.item >= 0) issue_loads(1, nxt);
        }
        loads_issued = 1 + (nxt.item >= 0);
        if (warp == 0) gate_tables(gates(0), gate_load(p, cur, lane), lane);
        if (warp == 4) gin = gate_load(p, nxt, lane);
        const bool ok = mbar_wait(&bar_load[0], 0);
        if (csync_or(!ok)) {
            rs.failed = true;
        } else {
            ++loads_waited;
            if (lt == 0) {
                tc_fence_after();
                issue_d1(0);
            }
        }
    }

    for (; cur.item >= 0 && !rs.failed; ++k) {
        const Ref nn = nxt.item >= 0 ? sc.first_from(task_of(nxt) + step, step) : nxt;
        const uint32_t kq = sbase + P_OFF_KQ + (k & 1) * KQ_STAGE;
        const float *g = gates(k);
        const int *gz = reinterpret_cast<const int *>(g + G_Z);
        const int slot = cur.r % RING;
        uint8_t *rec = p.ring + (static_cast<size_t>(cur.j) * RING + slot) * REC_BYTES;

        // ---- D1 of this chunk (issued during the previous one), and the ring
        // slot: the chain has taken round r - RING out of it. Thread 128, whose
        // warp has no block in the A / M phase, checks the slot (after
        // publishing the previous record) and its answer joins the barrier
        // that ends the phase: nothing writes the slot before it. A flag value
        // read during the previous record skips the poll when it already
        // shows the slot free (the chain's copies out of the slot completed
        // before it stored the flag).
        const bool d1_ok = __all_sync(0xffffffffu, mbar_wait(bar_d1, k & 1));
        tc_fence_after();
        bool slot_ok = true;
        if (lt == 128 && d1_ok && slot_seen < cur.r - RING + 1)
            slot_ok = poll_ge_backoff(p.consumed + cur.j * FLAG_STRIDE, cur.r - RING + 1, p.abort_flag,
                                      p.poll_ns);

        // ---- A = beta P (K K^T) (fp32) and M = P (Q K^T) (record, fp16), 32 columns per thread
        const bool qk = row >= 64;
        // Warp-uniform: the whole 32 x 32 block lies above the diagonal.
        const bool upper = half == 1 && (warp & 1) == 0;
        uint32_t mt0[8] = {}, mt1[8] = {};  // qk threads: M^T[s][t] for s = 32 half + 0..15, + 16..31 (fp16 pairs)
        if (d1_ok && !upper) {
            const int t = row & 63;
            const int s0 = 32 * half;
            {
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
#pragma unroll
                        for (int jp = 0; jp < 8; ++jp) {
                            const uint32_t w = pack_f16x2(v[2 * jp], v[2 * jp + 1]);
                            if (hp == 0) mt0[jp] = w; else mt1[jp] = w;
                        }
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
        if (csync_or(!d1_ok || !slot_ok)) { rs.failed = true; break; }
        // M^T into the record straight from registers, now that the slot is
        // free: for each s a warp's 32 consecutive t fill one aligned 64-byte
        // half of the 128-byte row (two whole sectors per store instruction)
        if (qk) {
            const int t = row & 63;
            uint8_t *mtb = rec + REC_MT;
            if (upper) {
#pragma unroll 4
                for (int s = 32; s < 64; ++s) st_sw_h(mtb, s, t, 0);
            } else {
                const int s0 = 32 * half;
#pragma unroll
                for (int jp = 0; jp < 8; ++jp) {
                    st_sw_h(mtb, s0 + 2 * jp, t, static_cast<uint16_t>(mt0[jp]));
                    st_sw_h(mtb, s0 + 2 * jp + 1, t, static_cast<uint16_t>(mt0[jp] >> 16));
                    st_sw_h(mtb, s0 + 16 + 2 * jp, t, static_cast<uint16_t>(mt1[jp]));
                    st_sw_h(mtb, s0 + 17 + 2 * jp, t, static_cast<uint16_t>(mt1[jp] >> 16));
                }
            }
        }

        // ---- diagonal 16 x 16 tiles of T (warps 0-3, one each) while warps
        // 4-7 zero tiles (0,1), (2,3) of T and wait for the next chunk's
        // tiles
        bool prep_fail = false;
        if (warp < 4) {
            diag_inverse16(Af + (16 * warp) * AST + 16 * warp, Tf + (16 * warp) * AST + 16 * warp, lane);
        } else {
            const int wt = lt - 128;
            for (int e = wt; e < 512; e += 128) {
                const int blk = e >> 8, rr = (e >> 4) & 15, cc = e & 15;
                Tf[(32 * blk + rr) * AST + 32 * blk + 16 + cc] = 0.f;
            }
            if (nxt.item >= 0) prep_fail = !mbar_wait(&bar_load[(k + 1) & 1], ((k + 1) >> 1) & 1);
        }
        if (csync_or(prep_fail)) { rs.failed = true; break; }
        // The next D1 comes from thread 128 (warps 4-7 have no part in the
        // solve's first step).
        if (nxt.item >= 0) {
            ++loads_waited;
            if (lt == 128) {
                tc_fence_after();
                issue_d1(k + 1);
            }
        }
        solve_offdiag(Af, Tf, Xf, warp, lane, bar_id);

        // ---- T diag(beta) (record, fp16) and T diag(beta gamma) (local, as a
        // bf16 hi + lo pair so that D_W can read K's bf16 tile as it landed)
        {
            const int t = lt & 63;
            const bool hat = (lt >> 6) & 1;
            const int hh = lt >> 7;
            const int s0 = 32 * hh;
            uint8_t *dstb = hat ? th : rec + REC_TT;
            if (hh == 1 && t < 32) {
                st_zero32(dstb, t, 4);
                if (hat) st_zero32(dstb + 8192, t, 4);
            } else {
                const float *scl = g + (hat ? G_BG : G_BE);
#pragma unroll 1
                for (int hp = 0; hp < 2; ++hp) {
                    const int sb = s0 + 16 * hp;
                    float v[16];
#pragma unroll
                    for (int j4 = 0; j4 < 4; ++j4) {
                        const float4 tv = *reinterpret_cast<const float4 *>(Tf + t * AST + sb + 4 * j4);
                        const float4 sv = *reinterpret_cast<const float4 *>(scl + sb + 4 * j4);
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
        fence_proxy_async_smem();
        tc_fence_before();
        csync();
        tc_fence_after();

        // ---- D_W = K^T (T diag bg)^T = K^T (hi + lo)^T on bf16 operands
        // (lane j, column t: W[t][j])
        if (lt == 0) {
#pragma unroll 1
            for (int kk = 0; kk < 8; ++kk)
                umma_f16(tmem + TM_W, sdesc_sw128(kq + (kk & 3) * 2048, 16384, 1024),
                         sdesc_sw128(smem_u32(th) + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024),
                         ID_MK64_BF, kk > 0);
            umma_commit(bar_mma);
        }
        // The next chunk's gate table, under D_W.
        if (warp == 4 && nxt.item >= 0) {
            gate_tables(gates(k + 1), gin, lane);
            gin = gate_load(p, nn, lane);
        }
        {
            const bool ok = mbar_wait(bar_mma, mma_phase);
            if (csync_or(!ok)) { rs.failed = true; break; }
            mma_phase ^= 1u;
            tc_fence_after();
        }
        // Stage k & 1 is free (this chunk's D1 and D_W are done): chunk k + 2's
        // tiles go out now, under the W staging and the publish.
        if (nn.item >= 0) {
            if (lt == 128) issue_loads(k + 2, nn);
            ++loads_issued;
        }
        if (lt == 128 && nxt.item >= 0) slot_seen = ld_relaxed_gpu(p.consumed + nxt.j * FLAG_STRIDE);
        {
            // -W K-major [j half][t][64 j] straight into the record: lane j
            // writes its 32 t's, and for each t a warp's 32 consecutive j fill
            // one aligned 64-byte half of the 128-byte row (the swizzle
            // permutes 16-byte chunks within aligned groups of four), two
            // whole sectors per store instruction
            float x[32];
            tmem_ld32(trow + TM_W + 32 * half, x);
            tmem_wait_ld();
            uint8_t *blk = rec + REC_W + (row >> 6) * 8192;
#pragma unroll
            for (int t = 0; t < 32; ++t) st_sw_f16(blk, 32 * half + t, row & 63, -x[t]);
        }
        tc_fence_before();
        csync();
        // ---- record complete: publish it (thread 128: its fence's wait for
        // the record's stores runs under the next record's A / M phase)
        if (lt == 128) {
            fence_proxy_async_global();
            st_release_gpu(p.ready + cur.j * FLAG_STRIDE + slot, cur.r + 1);
        }
        cur = nxt;
        nxt = nn;
    }

    if (rs.failed && lt == 0) {
        for (int kk = loads_waited; kk < loads_issued; ++kk)
            mbar_wait(&bar_load[kk & 1], (kk >> 1) & 1, 200000000ull);
        umma_commit(bars + PB_DRAIN);  // every MMA thread 0 issued: D_W and the first D1
        mbar_wait(bars + PB_DRAIN, 0, 200000000ull);
        atomicExch(&g_grid_status, 1);
        atomicExch(p.abort_flag, 1);
    }
    if (rs.failed && lt == 128) {
        umma_commit(bars + PB_DRAIN2);  // the later D1s (issued by this thread)
        mbar_wait(bars + PB_DRAIN2, 0, 200000000ull);
    }
    rs.failed = csync_or(rs.failed);
    return rs;
}

__global__ void __launch_bounds__(NT, 1)
    gdr_chunk_grid_kernel(const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ GParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tid = threadIdx.x, warp = tid >> 5;
    const bool chain = static_cast<int>(blockIdx.x) < p.n_chains;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(
        chain ? smem + C_OFF_BAR + CB_NUM * 8 : smem + P_OFF_TMEM);
    const uint32_t ncols = chain ? C_TM_COLS : P_TM_COLS;

    if (tid == 0) {
        if (chain) {
            uint64_t *bars = reinterpret_cast<uint64_t *>(smem + C_OFF_BAR);
            for (int i = 0; i < CB_NUM; ++i) mbar_init(&bars[i], 1);  // loads, records, R1, R2
            for (int i = 0; i < 2; ++i) {
                mbar_init(&bars[CB_CONV + i], 256);   // both warpgroups signal (V tile by 0, Q and K by 1)
                mbar_init(&bars[CB_OFREE + i], 128);
            }
            mbar_init(&bars[CB_S16], 128);            // warpgroup 0 signals
            mbar_init(&bars[CB_D16], 128);
        } else {
            for (int c = 0; c < PCTX; ++c) {
                uint64_t *bars = reinterpret_cast<uint64_t *>(smem + c * P_CTX_BYTES + P_OFF_BAR);
                for (int i = 0; i < PB_NUM; ++i) mbar_init(&bars[i], 1);
            }
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

    int64_t n_seq = p.n_seq;
    if (p.n_seq_dev) {
        const int64_t nd = *p.n_seq_dev;
        n_seq = nd < n_seq ? nd : n_seq;
    }
    const int64_t n_items = n_seq * p.H;
    const Walk wk{&p, n_items, static_cast<int64_t>(p.n_chains), p.H};
    if (chain) {
        chain_role(&tm_q, &tm_k, &tm_v, p, smem, wk, blockIdx.x, tmem);
    } else {
        Sched sc{&p, &wk, n_items, p.n_chains, 0, 0};
        if (p.cu_seqlens == nullptr) {
            sc.nch = static_cast<int>((p.seq_len + CH - 1) / CH);
            sc.n_tasks = (n_items + p.n_chains - 1) / p.n_chains * sc.nch * p.n_chains;
        } else {
            sc.n_tasks = static_cast<int64_t>(p.sched[0]) * p.n_chains;
        }
        // Context c of producer CTA b takes tasks PCTX (b - n_chains) + c,
        // then every PCTX n_prod-th after it.
        const int ctx = tid >> 8;
        const int64_t first = static_cast<int64_t>(PCTX) * (blockIdx.x - p.n_chains) + ctx;
        producer_role(&tm_q, &tm_k, p, smem + ctx * P_CTX_BYTES, sc, first,
                      static_cast<int64_t>(PCTX) * p.n_prod, tmem + ctx * P_TM_CTX, tid & 255, 3 + ctx);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, ncols);
}

__device__ __forceinline__ int64_t seq_chunks(const int32_t *cu, int64_t seq, int64_t total_tokens) {
    int64_t t0 = cu[seq], t1 = cu[seq + 1];
    t0 = t0 < 0 ? 0 : (t0 > total_tokens ? total_tokens : t0);
    t1 = t1 < t0 ? t0 : (t1 > total_tokens ? total_tokens : t1);
    return (t1 - t0 + CH - 1) / CH;
}

__device__ __forceinline__ int64_t dev_n_seq(const int32_t *n_seq_dev, int64_t n_seq_host) {
    if (!n_seq_dev) return n_seq_host;
    const int64_t nd = *n_seq_dev;
    return nd < n_seq_host ? nd : n_seq_host;
}

// Packed streams of at most this many sequences are ordered longest first;
// longer lists keep the caller's order.
constexpr int GRID_RANK_MAX = 4096;
constexpr int GRID_RANK_THREADS = 256;
constexpr int GRID_RANK_BLOCKS = GRID_RANK_MAX / GRID_RANK_THREADS;

// Sequences of a packed stream by chunk count, longest first (ties by
// index): order[rank(i)] = i, rank(i) = #{j : n_j > n_i or (n_j = n_i and
// j < i)}. Each block holds every sequence's chunk count in shared memory and
// each thread ranks one sequence against all of them. The sequence count is
// read on the device; above GRID_RANK_MAX the order is the identity.
__global__ void __launch_bounds__(GRID_RANK_THREADS)
    gdr_grid_rank_kernel(const int32_t *cu, const int32_t *n_seq_dev, int64_t n_seq_host,
                         int64_t total_tokens, int32_t *order) {
    __shared__ int cnt[GRID_RANK_MAX];
    const int64_t n = dev_n_seq(n_seq_dev, n_seq_host);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (n > GRID_RANK_MAX) {  // the same branch for every thread of the grid
        for (int64_t i = i0; i < n; i += stride) order[i] = static_cast<int32_t>(i);
        return;
    }
    const int ni32 = static_cast<int>(n);
    for (int i = threadIdx.x; i < ni32; i += blockDim.x) cnt[i] = static_cast<int>(seq_chunks(cu, i, total_tokens));
    __syncthreads();
    for (int64_t i = i0; i < n; i += stride) {
        const int c = cnt[i];
        int rank = 0;
        for (int j = 0; j < ni32; ++j) {
            const int cj = cnt[j];
            rank += (cj > c || (cj == c && j < i)) ? 1 : 0;
        }
        order[rank] = static_cast<int32_t>(i);
    }
}

// Per-position round offsets of a packed stream: chain j takes the items at
// positions pos(j, 0), pos(j, 1), ... (snake order over positions sorted
// longest first) and off[pos] is the number of chunks of the chain's
// earlier items (one warp per chain, 32 items per step with a warp scan).
// sched[0] is the longest chain's round count, sched[1 + j] chain j's.
__global__ void gdr_grid_sched_kernel(const int32_t *cu, const int32_t *n_seq_dev, int64_t n_seq_host,
                                      int64_t total_tokens, int H, int NC, const int32_t *order,
                                      int32_t *off, int32_t *sched) {
    const int lane = threadIdx.x & 31;
    const int j = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (j >= NC) return;
    const int64_t n_items = dev_n_seq(n_seq_dev, n_seq_host) * H;
    int carry = 0;
    for (int64_t m0 = 0;; m0 += 32) {
        const int64_t m = m0 + lane;
        const int64_t q = m * NC + ((m & 1) ? NC - 1 - j : j);
        const int64_t q0 = m0 * NC + ((m0 & 1) ? NC - 1 - j : j);
        if (q0 >= n_items) break;
        int nch = 0;
        if (q < n_items) {
            const int64_t item = order ? static_cast<int64_t>(order[q / H]) * H + q % H : q;
            nch = static_cast<int>(seq_chunks(cu, item / H, total_tokens));
        }
        int incl = nch;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int x = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += x;
        }
        if (q < n_items) off[q] = carry + incl - nch;
        carry += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
        sched[1 + j] = carry;
        atomicMax(&sched[0], carry);
    }
}

}  // namespace

namespace {

struct GridWs {
    size_t ready, consumed, abort, sched, off, order, flags_end, total;
};

GridWs grid_ws(int64_t n_items, bool packed) {
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    GridWs w;
    const size_t ring = static_cast<size_t>(MAX_CHAINS) * RING * REC_BYTES;
    w.ready = up(ring);
    w.consumed = up(w.ready + static_cast<size_t>(MAX_CHAINS) * FLAG_STRIDE * sizeof(int));
    w.abort = up(w.consumed + static_cast<size_t>(MAX_CHAINS) * FLAG_STRIDE * sizeof(int));
    w.sched = up(w.abort + sizeof(int));
    w.flags_end = up(w.sched + static_cast<size_t>(1 + MAX_CHAINS) * sizeof(int));
    const size_t ni = static_cast<size_t>(n_items > 0 ? n_items : 0);
    w.off = w.flags_end;
    w.order = up(w.off + ni * sizeof(int));  // at most one entry per sequence, sized per item
    w.total = packed ? up(w.order + ni * sizeof(int)) : w.off;
    return w;
}

// Chains. Up to 45% of the SMs every item gets its own chain (one pass).
// Beyond that a chain runs several items one after another:
//   - equal-length items (the batched layout): the fewest chains that keep
//     the pass count of the 45% split, leaving the rest of the SMs to the
//     producers;
//   - packed (ragged) items, balanced by longest-first scheduling: 39% of
//     the SMs, near where a chain's per-chunk time (about 6.2K cycles)
//     matches the record rate of the producers' two contexts.
// RHZ_GRID_CHAINS overrides the split.
int grid_chains(int sms, int64_t items, bool packed) {
    static int env = -1;
    static std::once_flag once;
    std::call_once(once, [] {
        const char *e = getenv("RHZ_GRID_CHAINS");
        env = e ? atoi(e) : 0;
    });
    int64_t nc;
    if (env > 0) {
        nc = env;
    } else {
        const int64_t hi = (static_cast<int64_t>(sms) * 45 + 50) / 100;
        if (items <= hi) {
            nc = items;
        } else if (packed) {
            nc = (static_cast<int64_t>(sms) * 39 + 50) / 100;
        } else {
            const int64_t passes = (items + hi - 1) / hi;
            nc = (items + passes - 1) / passes;
        }
    }
    if (nc > items) nc = items;
    if (nc > MAX_CHAINS) nc = MAX_CHAINS;
    if (nc > sms - 1) nc = sms - 1;
    return nc < 1 ? 1 : static_cast<int>(nc);
}

// Test hook (rhz_gdr_set_wait_test): off, or every chain waits for a record
// flag that no producer sets, with cross-CTA waits bounded at g_test_ns.
std::atomic<int> g_test_mode{0};
std::atomic<int64_t> g_test_ns{0};

}  // namespace

int set_wait_test(int mode, int64_t limit_ns) {
    if (mode != 0 && mode != 1) return set_error(RHZ_ERR_INVALID, "wait test mode %d is not 0 or 1", mode);
    if (mode == 1 && (limit_ns < 1000 || limit_ns > 2000000000LL))
        return set_error(RHZ_ERR_INVALID, "wait limit %lld ns outside [1 us, 2 s]", static_cast<long long>(limit_ns));
    g_test_ns.store(mode ? limit_ns : 0);
    g_test_mode.store(mode);
    return RHZ_OK;
}

size_t chunk_grid_ws_bytes(int64_t n_items, bool packed) { return grid_ws(n_items, packed).total; }

int chunk_grid_status(int *flag, bool clear) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_grid_status, sizeof(int));
    if (e == cudaSuccess && clear && v) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_grid_status, &zero, sizeof(int));
    }
    if (e != cudaSuccess)
        return set_error(RHZ_ERR_DEVICE, "reading the chunked kernel's status: %s", cudaGetErrorString(e));
    *flag = v;
    return RHZ_OK;
}

int launch_chunk_grid(const SeqArgs &a) {
    if (a.d != HD || a.dtype != RHZ_DTYPE_BF16)
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
    const int64_t items = a.n_seq * a.H;
    const bool packed = a.cu_seqlens != nullptr;
    const GridWs w = grid_ws(items, packed);
    if (a.ws == nullptr || a.ws_bytes < w.total)
        return set_error(RHZ_ERR_INVALID, "workspace too small: need %zu bytes, got %zu", w.total, a.ws_bytes);
    if (!aligned(a.ws, 256)) return set_error(RHZ_ERR_INVALID, "workspace must be 256-byte aligned");
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
        attr_err = cudaFuncSetAttribute(gdr_chunk_grid_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(SMEM_ALLOC));
    });
    if (attr_err != cudaSuccess)
        return set_error(RHZ_ERR_DEVICE, "gdr_chunk_grid_kernel smem attribute: %s", cudaGetErrorString(attr_err));
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gdr_chunk_grid_kernel, NT, SMEM_ALLOC);
    if (e != cudaSuccess || per_sm < 1)
        return set_error(RHZ_ERR_DEVICE, "gdr_chunk_grid_kernel does not fit an SM: %s", cudaGetErrorString(e));
    const int grid = sms;  // one CTA per SM (shared memory allows no second)
    const int nc = grid_chains(sms, items, packed);

    char *ws = static_cast<char *>(a.ws);
    e = cudaMemsetAsync(ws + w.ready, 0, w.flags_end - w.ready, a.stream);
    if (e != cudaSuccess) return set_error(RHZ_ERR_DEVICE, "workspace flags: %s", cudaGetErrorString(e));
    GParams p;
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
    p.ring = reinterpret_cast<uint8_t *>(ws);
    p.ready = reinterpret_cast<int *>(ws + w.ready);
    p.consumed = reinterpret_cast<int *>(ws + w.consumed);
    p.abort_flag = reinterpret_cast<int *>(ws + w.abort);
    p.sched = reinterpret_cast<int32_t *>(ws + w.sched);
    p.off = packed ? reinterpret_cast<int32_t *>(ws + w.off) : nullptr;
    p.order = packed ? reinterpret_cast<int32_t *>(ws + w.order) : nullptr;
    p.snake = packed ? 1 : 0;
    p.n_chains = nc;
    p.n_prod = grid - nc;
    p.never_ready = g_test_mode.load();
    p.poll_ns = p.never_ready ? static_cast<uint64_t>(g_test_ns.load()) : 2000000000ull;
    if (packed) {
        gdr_grid_rank_kernel<<<GRID_RANK_BLOCKS, GRID_RANK_THREADS, 0, a.stream>>>(
            a.cu_seqlens, a.n_seq_dev, a.n_seq, tokens, const_cast<int32_t *>(p.order));
        {
            const int ls = check_launch("gdr_grid_rank_kernel");
            if (ls != RHZ_OK) return ls;
        }
        const int warps = 8;
        gdr_grid_sched_kernel<<<(nc + warps - 1) / warps, 32 * warps, 0, a.stream>>>(
            a.cu_seqlens, a.n_seq_dev, a.n_seq, tokens, a.H, nc, p.order,
            reinterpret_cast<int32_t *>(ws + w.off), reinterpret_cast<int32_t *>(ws + w.sched));
        {
            const int ls = check_launch("gdr_grid_sched_kernel");
            if (ls != RHZ_OK) return ls;
        }
    }

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(NT, 1, 1);
    cfg.dynamicSmemBytes = SMEM_ALLOC;
    cfg.stream = a.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: they wait on each other
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, gdr_chunk_grid_kernel, tq, tk, tv, p);
    if (e != cudaSuccess)
        return set_error(RHZ_ERR_DEVICE, "gdr_chunk_grid_kernel launch: %s", cudaGetErrorString(e));
    return check_launch("gdr_chunk_grid_kernel");
}

}  // namespace rhz
