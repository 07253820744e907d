// Chunked gated delta-rule prefill on the sm_100a tensor cores, one CTA per
// (sequence, head): the form used when there are more (sequence, head)
// items than SMs (e.g. the full-layer configuration), where every SM running
// a whole chain beats two SMs per chain. gdr_chunk_tc.cu (a 2-CTA cluster
// per item) serves the case with fewer items than SMs; both compute the
// same quantities with the same rounding points.
//
// Math (per sequence and head; S is d_v x d_k, row i = v index): inside a
// chunk of positions t = 0..C-1 that starts from state S0,
//   P[t][s] = prod_{r=s+1..t} alpha_r (s <= t),  gamma_t = prod_{r=0..t} alpha_r
//   A[t][s] = beta_t P[t][s] (k_t . k_s) for s < t, T = (I + A)^-1
//   U = T diag(beta) V,  W = T diag(beta gamma) K,  Delta = U - W S0^T
//   O[t] = gamma_t S0 q_t + sum_{s<=t} P[t][s] (q_t . k_s) Delta_s
//   S_C = gamma_{C-1} S0 + sum_s P[C-1][s] Delta_s k_s^T
// which equals C applications of gated_delta_step (crates/ops/src/delta.rs:
// 93-127). Decays: P[t][s] = (z_t == z_s) ? exp2(gl_t - gl_s) : 0 with gl the
// prefix sum of log2(alpha) over nonzero alphas and z the count of zeros.
//
// Products (head dimension on M = 128 so each accumulator row is one TMEM
// lane; the output is an M = 64 product stored row by row):
//   D1   = [K; Q] K^T          (128 x 64, K = d)     -> A (fp32 smem) and masked M
//   D_U  = V^T (T diag b)^T    (128 x 64, K = C)
//   D_W  = K^T (T diag bg)^T   (128 x 64, K = C)     -> -W^T (fp16 smem)
//   D_O  = Q~ S0^T             ( 64 x 128, K = d)    Q~ = diag(gamma) Q
//   D_U += S0 (-W^T)           (128 x 64, K = d)     -> Delta^T (fp16 smem)
//   D_O += M Delta             ( 64 x 128, K = C)
//   D_S += (P[C-1] Delta)^T K  (128 x 128, K = C)    (D_S pre-scaled by gamma_{C-1})
// Q, K, V tiles arrive by TMA (128-byte swizzle, double-buffered one chunk
// ahead; no multicast), are converted to fp16 in place, and every product
// after D1 takes fp16 operands. The 16 x 16 diagonal blocks of T come from
// the product formula (I + N)^-1 = (I - N)(I + N^2)(I + N^4)(I + N^8) on
// mma.sync (one warp per block), the rest from a 2 x 2 recursion on mma.sync.
// With an output-norm scale the O rows are RMS-normalised per head
// (groupnorm_heads, norm.rs:48-60) on the fp32 accumulator before the store.
//
// One CTA (256 threads) per SM, persistent over (sequence, head) items. Every
// wait is bounded; a timeout sets a sticky device flag, drains in-flight
// copies and MMAs (bounded), frees TMEM and returns.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "chunk_common.cuh"
#include "sm100.cuh"
#include "tmap.h"

namespace rhz {

// Sticky per-device flag: set when a bounded device-side wait ran out.
__device__ int g_solo_status = 0;

namespace {
using namespace sm100;
using namespace chunk;

constexpr int NT = 256;   // threads per CTA

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
constexpr uint32_t OFF_WT = OFF_R;                 //   -W^T [j][t] fp16 (16 KB)
constexpr uint32_t OFF_DT = OFF_R + 16384;         //   Delta^T [i][s] fp16 (16 KB)
constexpr uint32_t OFF_DTS = OFF_R + 32768;        //   (P[C-1] Delta)^T [i][s] fp16 (16 KB)
constexpr uint32_t OFF_AF = OFF_R;                 //   A fp32 [64][AST]   (solve phase)
constexpr uint32_t OFF_TF = OFF_AF + 64 * AST * 4; //   T fp32 [64][AST]
constexpr uint32_t OFF_XF = OFF_TF + 64 * AST * 4; //   32 x 32 fp32 partial products
constexpr uint32_t OFF_SMALL = OFF_R + 49152;      // 2 x {gl, z, beta, gamma, P[C-1][.], beta*gamma}
constexpr uint32_t OFF_BAR = OFF_SMALL + 3072;     // 4 mbarriers + TMEM base address
constexpr uint32_t OFF_NORM = OFF_BAR + 64;        // output-norm scale (HD floats)
constexpr uint32_t OFF_NRM = OFF_NORM + HD * 4;    // per-(row, half) sums of squares
constexpr uint32_t SMEM_USED = OFF_NRM + 64 * 2 * 4;
constexpr size_t SMEM_ALLOC = SMEM_USED + 1024;    // slack for 1024-byte alignment
static_assert(OFF_XF + 4 * 256 * 4 <= OFF_R + 49152, "solve scratch overflows its region");
static_assert(SMEM_ALLOC <= 232448, "exceeds the 227 KB opt-in shared memory");

// TMEM columns (f32 accumulators). D_O is an M = 64 accumulator (row t in
// lane 32 (t / 16) + t % 16) over 128 columns; the others use all 128 lanes.
constexpr uint32_t TM_D1 = 0, TM_U = 64, TM_W = 128, TM_O = 192, TM_S = 320;
constexpr uint32_t TM_COLS = 512;

// Every product runs on fp16 operands (the bf16 tiles are converted in place).
constexpr uint32_t ID_D1 = idesc_f16(128, 64, false, false);
constexpr uint32_t ID_MK64 = idesc_f16(128, 64, true, false);
constexpr uint32_t ID_KM64 = idesc_f16(128, 64, false, true);
constexpr uint32_t ID_KM128 = idesc_f16(128, 128, false, true);
constexpr uint32_t ID_O = idesc_f16(64, 128, false, false);
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
    const float *norm_scale;  // non-null: groupnorm_heads on each O row in the epilogue
    float norm_eps;
};

// bf16 -> fp16 in place on 16-byte chunks [first, 3072) of one stage's K, Q
// (32 KB) and V (16 KB) tiles, stepping by `stride`. The swizzled layout is
// elementwise, so it is unchanged; bf16 values in the fp16 normal range
// convert exactly.
__device__ __forceinline__ void tiles_to_f16(uint8_t *kq, uint8_t *vv, int first, int stride) {
    for (int i = first; i < 3072; i += stride) {
        uint4 *ptr = reinterpret_cast<uint4 *>(i < 2048 ? kq + i * 16 : vv + (i - 2048) * 16);
        uint4 w = *ptr;
        w.x = bf16x2_to_f16x2(w.x);
        w.y = bf16x2_to_f16x2(w.y);
        w.z = bf16x2_to_f16x2(w.z);
        w.w = bf16x2_to_f16x2(w.w);
        *ptr = w;
    }
}

__global__ void __launch_bounds__(NT, 1)
    gdr_chunk_solo_kernel(const __grid_constant__ CUtensorMap tm_q,
                        const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // TMEM lane (accumulator row) of this thread and the column half it owns.
    const int row = 32 * (warp & 3) + lane;
    const int half = warp >> 2;
    uint64_t *bar_load = reinterpret_cast<uint64_t *>(smem + OFF_BAR);  // [2] TMA per stage
    uint64_t *bar_mma = bar_load + 2;                                   // state-chain MMAs
    uint64_t *bar_d1 = bar_load + 3;                                    // D1 of the next chunk
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bar_load + 4);
    float *Af = reinterpret_cast<float *>(smem + OFF_AF);
    float *Tf = reinterpret_cast<float *>(smem + OFF_TF);
    float *Xf = reinterpret_cast<float *>(smem + OFF_XF);
    float *nsc = reinterpret_cast<float *>(smem + OFF_NORM);
    float *nrm = reinterpret_cast<float *>(smem + OFF_NRM);
    const bool norm = p.norm_scale != nullptr;
    if (norm && tid < HD) nsc[tid] = p.norm_scale[tid];
    const uint32_t sbase = smem_u32(smem);

    if (tid == 0) {
        mbar_init(&bar_load[0], 1);
        mbar_init(&bar_load[1], 1);
        mbar_init(bar_mma, 1);
        mbar_init(bar_d1, 1);
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
    const uint32_t trow = tmem + (static_cast<uint32_t>(warp & 3) << 21);  // lane (32 (w&3)) << 16

    const int H = p.H;
    int64_t n_seq = p.n_seq;
    if (p.n_seq_dev) {
        const int64_t nd = *p.n_seq_dev;
        n_seq = nd < n_seq ? nd : n_seq;
    }
    const int64_t n_items = n_seq * H;
    const int64_t tok_stride = static_cast<int64_t>(H) * HD;

    // The chunks this CTA processes, in order: items blockIdx.x, +gridDim.x,
    // ..., and within an item its chunks of CH positions from the sequence
    // start. Chunk k of that order uses TMA stage k & 1 and gate tables k & 1.
    auto bounds = [&](int64_t item, int64_t &t0, int64_t &t1) {
        const int64_t seq = item / H;
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
    };
    struct Ref {
        int64_t item, ts;  // item < 0: no chunk
        int L, h;
    };
    // First chunk at or after item `it` (skipping empty sequences).
    auto first_from = [&](int64_t it) -> Ref {
        for (; it < n_items; it += gridDim.x) {
            int64_t t0, t1;
            bounds(it, t0, t1);
            if (t1 > t0) {
                const int64_t seq = it / H;
                return Ref{it, t0, static_cast<int>((t1 - t0) < CH ? (t1 - t0) : CH),
                           static_cast<int>(it - seq * H)};
            }
        }
        return Ref{-1, 0, 0, 0};
    };
    auto next_of = [&](const Ref &r) -> Ref {
        int64_t t0, t1;
        bounds(r.item, t0, t1);
        const int64_t tn = r.ts + CH;
        if (tn < t1) return Ref{r.item, tn, static_cast<int>((t1 - tn) < CH ? (t1 - tn) : CH), r.h};
        return first_from(r.item + gridDim.x);
    };
    // The chunk n steps after chunk c of `item` (bounds [t0, t1), nch chunks,
    // head h): arithmetic inside the item, the walk only past its end.
    auto after = [&](int64_t item, int h, int64_t t0, int64_t t1, int nch, int c, int n) -> Ref {
        const int cc = c + n;
        if (cc < nch) {
            const int64_t ts = t0 + static_cast<int64_t>(cc) * CH;
            return Ref{item, ts, static_cast<int>((t1 - ts) < CH ? (t1 - ts) : CH), h};
        }
        Ref r = first_from(item + gridDim.x);
        for (int i = nch; i < cc && r.item >= 0; ++i) r = next_of(r);
        return r;
    };

    uint32_t mma_phase = 0;
    bool failed = false, mma_pending = false, d1_pending = false;
    int loads_issued = 0, loads_waited = 0;  // thread 0 / all threads

    auto issue_loads = [&](int k, const Ref &r) {
        const uint32_t st = k & 1;
        uint64_t *bar = &bar_load[st];
        uint8_t *kq = smem + OFF_KQ + st * KQ_STAGE;
        uint8_t *vv = smem + OFF_V + st * V_STAGE;
        mbar_arrive_expect_tx(bar, LOAD_BYTES);
        const int t32 = static_cast<int>(r.ts);
        tma_load_3d(kq, &tm_k, 0, r.h, t32, bar);
        tma_load_3d(kq + 16384, &tm_k, 64, r.h, t32, bar);
        tma_load_3d(kq + 8192, &tm_q, 0, r.h, t32, bar);
        tma_load_3d(kq + 24576, &tm_q, 64, r.h, t32, bar);
        tma_load_3d(vv, &tm_v, 0, r.h, t32, bar);
        tma_load_3d(vv + 8192, &tm_v, 64, r.h, t32, bar);
    };
    // Commit the issued state-chain MMAs and wait for them on every thread.
    auto mma_wait = [&]() -> bool {
        const bool ok = mbar_wait(bar_mma, mma_phase);
        if (__syncthreads_or(!ok)) return false;
        mma_phase ^= 1u;
        mma_pending = false;
        tc_fence_after();
        return true;
    };
    auto mma_commit = [&]() {
        if (tid == 0) umma_commit(bar_mma);
        mma_pending = true;
    };
    // Make thread-written smem operands and TMEM stores visible to the MMA issuer.
    auto operands_ready = [&]() {
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
    };

    // Gate inputs of one chunk (two positions per lane of one warp), fetched
    // a chunk ahead into registers; padded positions get alpha = 1, beta = 0
    // so they write nothing.
    auto gate_fetch = [&](const Ref &r) -> GateIn {
        GateIn g{1.f, 1.f, 0.f, 0.f};
        if (r.item < 0) return g;
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
    };
    // Gate tables of chunk k (one warp), in the table slot k & 1.
    auto gate_tables = [&](int k, const GateIn &in) {
        chunk::gate_tables(reinterpret_cast<float *>(smem + OFF_SMALL) + (k & 1) * G_SIZE, in, lane);
    };
    // D1 = [K; Q] K^T of chunk k on its (fp16) tiles, tracked by bar_d1.
    auto issue_d1 = [&](int kc) {
        const uint32_t kq = sbase + OFF_KQ + (kc & 1) * KQ_STAGE;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
            const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
            umma_f16(tmem + TM_D1, sdesc_sw128(kq + off, 16, 1024), sdesc_sw128(kq + off, 16, 1024),
                     ID_D1, kk > 0);
        }
        umma_commit(bar_d1);
    };
    // Everything chunk k needs before its first SIMT phase: gate tables, its
    // tiles landed and converted to fp16, and D1 = [K; Q] K^T issued.
    auto prepare = [&](int k, const Ref &r) -> bool {
        if (warp == 0) gate_tables(k, gate_fetch(r));
        const bool ok = mbar_wait(&bar_load[k & 1], (k >> 1) & 1);
        if (__syncthreads_or(!ok)) return false;
        ++loads_waited;
        tiles_to_f16(smem + OFF_KQ + (k & 1) * KQ_STAGE, smem + OFF_V + (k & 1) * V_STAGE, tid, NT);
        operands_ready();
        if (tid == 0) issue_d1(k);
        d1_pending = true;
        return true;
    };

    // Prime: tiles of the first two chunks, then chunk 0's preparation.
    Ref cur = first_from(blockIdx.x);
    GateIn gin{1.f, 1.f, 0.f, 0.f};  // warp 4: gate inputs of the next chunk
    {
        const Ref second = cur.item >= 0 ? next_of(cur) : cur;
        if (tid == 0) {
            if (cur.item >= 0) issue_loads(0, cur);
            if (second.item >= 0) issue_loads(1, second);
        }
        if (warp == 4) gin = gate_fetch(second);
        loads_issued = (cur.item >= 0) + (second.item >= 0);
        if (cur.item >= 0 && !prepare(0, cur)) failed = true;
    }
    int k = 0;  // index of the chunk being processed

    for (int64_t item = blockIdx.x; item < n_items && !failed; item += gridDim.x) {
        const int64_t seq = item / H;
        const int h = static_cast<int>(item - seq * H);
        int64_t t0, t1;
        bounds(item, t0, t1);
        const int nch = static_cast<int>((t1 - t0 + CH - 1) / CH);

        // ---- initial state: (row, half) -> TMEM (fp32) and the fp16 copy
        {
            int64_t slot = -1;
            if (p.state_in) slot = p.in_slots ? static_cast<int64_t>(p.in_slots[seq]) : seq;
            const bool have = p.state_in && slot >= 0 && slot < p.num_slots;
            const float *src = have ? p.state_in + ((slot * H + h) * HD + row) * HD + 64 * half : nullptr;
#pragma unroll
            for (int q2 = 0; q2 < 2; ++q2) {
                float v[32];
#pragma unroll
                for (int e = 0; e < 32; e += 4) {
                    float4 f = have ? *reinterpret_cast<const float4 *>(src + 32 * q2 + e)
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
                    v[e] = f.x; v[e + 1] = f.y; v[e + 2] = f.z; v[e + 3] = f.w;
                }
                tmem_st32(trow + TM_S + 64 * half + 32 * q2, v);
                st_row32_f16(smem + OFF_S + half * 16384, row, 4 * q2, v);
            }
            tmem_wait_st();
        }
        operands_ready();

        for (int c = 0; c < nch; ++c, ++k) {
            const int64_t ts = t0 + static_cast<int64_t>(c) * CH;
            const int L = static_cast<int>((t1 - ts) < CH ? (t1 - ts) : CH);
            const uint32_t kq = sbase + OFF_KQ + (k & 1) * KQ_STAGE;
            const uint32_t vb = sbase + OFF_V + (k & 1) * V_STAGE;
            const float *sgl = reinterpret_cast<const float *>(smem + OFF_SMALL) + (k & 1) * 384;
            const int *sz = reinterpret_cast<const int *>(sgl + 64);
            const float *sbeta = sgl + 128, *sgam = sgl + 192, *spl = sgl + 256, *sbg = sgl + 320;

            // ---- D1 of this chunk (issued during the previous chunk's tail)
            {
                const bool ok = mbar_wait(bar_d1, k & 1);
                if (__syncthreads_or(!ok)) { failed = true; break; }
                d1_pending = false;
                tc_fence_after();
            }

            // ---- A = beta P (K K^T) (fp32) and M = P (Q K^T) (fp16), 32 columns per thread
            {
                const bool qk = row >= 64;
                const int t = row & 63;
                const int s0 = 32 * half;
                // Warp-uniform: the whole 32 x 32 block lies above the diagonal.
                if (half == 1 && (warp & 1) == 0) {
                    if (qk) st_zero32(smem + OFF_M, t, 4);
                } else {
                    const float glt = sgl[t];
                    const int zt = sz[t];
                    const float bt = qk ? 1.f : sbeta[t];
#pragma unroll 1
                    for (int hp = 0; hp < 2; ++hp) {
                        const int sb = s0 + 16 * hp;
                        float v[16];
                        tmem_ld16(trow + TM_D1 + sb, v);
                        tmem_wait_ld();
#pragma unroll
                        for (int j4 = 0; j4 < 4; ++j4) {
                            const float4 g4 = *reinterpret_cast<const float4 *>(sgl + sb + 4 * j4);
                            const int4 z4 = *reinterpret_cast<const int4 *>(sz + sb + 4 * j4);
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
                            st_row16_f16(smem + OFF_M, t, 4 * half + 2 * hp, v);
                        } else {
#pragma unroll
                            for (int j4 = 0; j4 < 4; ++j4)
                                *reinterpret_cast<float4 *>(Af + t * AST + sb + 4 * j4) =
                                    make_float4(v[4 * j4], v[4 * j4 + 1], v[4 * j4 + 2], v[4 * j4 + 3]);
                        }
                    }
                }
            }
            __syncthreads();

            // ---- diagonal 16 x 16 tiles of T (warps 0-3, one each) while warps
            // 4-7 zero tiles (0,1), (2,3) of T and convert the next chunk's
            // tiles to fp16
            const Ref nxt = after(item, h, t0, t1, nch, c, 1);
            bool prep_fail = false;
            if (warp < 4) {
                diag_inverse16(Af + (16 * warp) * AST + 16 * warp, Tf + (16 * warp) * AST + 16 * warp, lane);
            } else {
                for (int e = tid - 128; e < 512; e += 128) {
                    const int blk = e >> 8, rr = (e >> 4) & 15, cc = e & 15;
                    Tf[(32 * blk + rr) * AST + 32 * blk + 16 + cc] = 0.f;
                }
                if (nxt.item >= 0) {
                    prep_fail = !mbar_wait(&bar_load[(k + 1) & 1], ((k + 1) >> 1) & 1);
                    if (!prep_fail)
                        tiles_to_f16(smem + OFF_KQ + ((k + 1) & 1) * KQ_STAGE,
                                     smem + OFF_V + ((k + 1) & 1) * V_STAGE, tid - 128, 128);
                    fence_proxy_async_smem();
                }
            }
            if (__syncthreads_or(prep_fail)) { failed = true; break; }
            if (nxt.item >= 0) {
                ++loads_waited;
                if (tid == 0) issue_d1(k + 1);
                d1_pending = true;
            }
            solve_offdiag(Af, Tf, Xf, warp, lane, 0);

            // ---- T diag(beta) and T diag(beta gamma) as fp16 operands
            {
                const int t = tid & 63;
                const bool hat = (tid >> 6) & 1;
                const int hh = tid >> 7;
                const int s0 = 32 * hh;
                uint8_t *dst = smem + (hat ? OFF_TH : OFF_TT);
                if (hh == 1 && t < 32) {
                    st_zero32(dst, t, 4);
                } else {
                    const float *sc = hat ? sbg : sbeta;
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
                        st_row16_f16(dst, t, 4 * hh + 2 * hp, v);
                    }
                }
            }
            operands_ready();

            // ---- D_U = V^T (T diag b)^T, D_W = K^T (T diag bg)^T, D_O = Q S0^T
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
                    umma_f16(tmem + TM_O, sdesc_sw128(kq + off + 8192, 16, 1024),
                             sdesc_sw128(sbase + OFF_S + off, 16, 1024), ID_O, kk > 0);
                }
            }
            mma_commit();
            // The next chunk's gate table under these products (off the solve's
            // path), and the gate inputs of the chunk after it.
            if (warp == 4 && nxt.item >= 0) {
                gate_tables(k + 1, gin);
                gin = gate_fetch(after(item, h, t0, t1, nch, c, 2));
            }
            if (!mma_wait()) { failed = true; break; }
            {
#pragma unroll 1
                for (int hp = 0; hp < 2; ++hp) {
                    float x[16];
                    tmem_ld16(trow + TM_W + 32 * half + 16 * hp, x);  // W[t][j = row], t in this half
                    tmem_wait_ld();
#pragma unroll
                    for (int t = 0; t < 16; ++t) x[t] = -x[t];
                    st_row16_f16(smem + OFF_WT, row, 4 * half + 2 * hp, x);
                }
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
            mma_commit();
            if (!mma_wait()) { failed = true; break; }
            {
#pragma unroll 1
                for (int hp = 0; hp < 2; ++hp) {
                    float x[16];
                    tmem_ld16(trow + TM_U + 32 * half + 16 * hp, x);  // Delta[s][i = row]
                    tmem_wait_ld();
                    st_row16_f16(smem + OFF_DT, row, 4 * half + 2 * hp, x);
#pragma unroll
                    for (int j4 = 0; j4 < 4; ++j4) {
                        const float4 pl = *reinterpret_cast<const float4 *>(spl + 32 * half + 16 * hp + 4 * j4);
                        x[4 * j4] *= pl.x; x[4 * j4 + 1] *= pl.y; x[4 * j4 + 2] *= pl.z; x[4 * j4 + 3] *= pl.w;
                    }
                    st_row16_f16(smem + OFF_DTS, row, 4 * half + 2 * hp, x);
                }
                // D_S <- gamma_{C-1} D_S before the rank-C update accumulates.
                const float gC = sgam[63];
#pragma unroll
                for (int q2 = 0; q2 < 2; ++q2) {
                    float v[32];
                    tmem_ld32(trow + TM_S + 64 * half + 32 * q2, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] *= gC;
                    tmem_st32(trow + TM_S + 64 * half + 32 * q2, v);
                }
                // D_O row t <- gamma_t (Q S0^T)[t] before M Delta accumulates
                // (rows live in lanes 0..15 of each subpartition; the other
                // lanes' columns here belong to no accumulator).
                const float gt = sgam[(16 * (warp & 3) + lane) & 63];
#pragma unroll
                for (int q2 = 0; q2 < 2; ++q2) {
                    float v[32];
                    tmem_ld32(trow + TM_O + 64 * half + 32 * q2, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) v[e] *= gt;
                    tmem_st32(trow + TM_O + 64 * half + 32 * q2, v);
                }
                tmem_wait_st();
            }
            operands_ready();

            // ---- D_O += M Delta ; D_S += (P[C-1] Delta)^T K
            if (tid == 0) {
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    umma_f16(tmem + TM_O, sdesc_sw128(sbase + OFF_M + kk * 32, 16, 1024),
                             sdesc_sw128(sbase + OFF_DT + kk * 32, 16, 1024), ID_O, 1);
                }
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    umma_f16(tmem + TM_S, sdesc_sw128(sbase + OFF_DTS + kk * 32, 16, 1024),
                             sdesc_sw128(kq + kk * 2048, 16384, 1024), ID_KM128, 1);
                }
            }
            mma_commit();

            if (!mma_wait()) { failed = true; break; }
            // The stage of this chunk is free again: fetch the chunk after next.
            if (nxt.item >= 0) {
                const Ref nn = after(item, h, t0, t1, nch, c, 2);
                if (nn.item >= 0) {
                    if (tid == 0) issue_loads(k + 2, nn);
                    ++loads_issued;
                }
            }

            // ---- epilogue: O rows (D_O row t sits in lane 32 (t / 16) + t % 16;
            // lanes 16..31 of each warp hold no row) go out as 16-byte stores;
            // refresh the fp16 state copy
            {
                float o[32];
                const int t = 16 * (warp & 3) + lane;
                const bool has_row = lane < 16 && t < L;
                __nv_bfloat16 *op = p.o + (ts + t) * tok_stride + static_cast<int64_t>(h) * HD + 64 * half;
                // Optional per-head RMS norm of each O row (groupnorm_heads,
                // norm.rs:48-60): warps w and w + 4 hold the row's two halves.
                float inv = 1.f;
                if (norm) {
                    float ss = 0.f;
#pragma unroll 1
                    for (int q2 = 0; q2 < 2; ++q2) {
                        tmem_ld32(trow + TM_O + 64 * half + 32 * q2, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; ++e) ss += o[e] * o[e];
                    }
                    if (lane < 16) nrm[2 * t + half] = ss;
                    __syncthreads();
                    inv = lane < 16 ? 1.f / sqrtf((nrm[2 * t] + nrm[2 * t + 1]) / static_cast<float>(HD) + p.norm_eps) : 1.f;
                }
#pragma unroll
                for (int q2 = 0; q2 < 2; ++q2) {
                    tmem_ld32(trow + TM_O + 64 * half + 32 * q2, o);
                    tmem_wait_ld();
                    if (norm) {
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] = o[e] * inv * nsc[64 * half + 32 * q2 + e];
                    }
                    if (has_row) {
#pragma unroll
                        for (int c8 = 0; c8 < 4; ++c8) {
                            uint4 w;
                            w.x = pack_bf16x2(o[8 * c8 + 0], o[8 * c8 + 1]);
                            w.y = pack_bf16x2(o[8 * c8 + 2], o[8 * c8 + 3]);
                            w.z = pack_bf16x2(o[8 * c8 + 4], o[8 * c8 + 5]);
                            w.w = pack_bf16x2(o[8 * c8 + 6], o[8 * c8 + 7]);
                            *reinterpret_cast<uint4 *>(op + 32 * q2 + 8 * c8) = w;
                        }
                    }
                }
#pragma unroll
                for (int q2 = 0; q2 < 2; ++q2) {
                    float v[32];
                    tmem_ld32(trow + TM_S + 64 * half + 32 * q2, v);
                    tmem_wait_ld();
                    st_row32_f16(smem + OFF_S + half * 16384, row, 4 * q2, v);
                }
            }
            operands_ready();
        }
        if (failed) break;

        // ---- final state
        if (p.state_out) {
            const int64_t slot = p.out_slots ? static_cast<int64_t>(p.out_slots[seq]) : seq;
            if (slot >= 0 && slot < p.num_slots) {
                float *dst = p.state_out + ((slot * H + h) * HD + row) * HD + 64 * half;
#pragma unroll
                for (int q2 = 0; q2 < 2; ++q2) {
                    float v[32];
                    tmem_ld32(trow + TM_S + 64 * half + 32 * q2, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        *reinterpret_cast<float4 *>(dst + 32 * q2 + e) =
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
            for (int kk = loads_waited; kk < loads_issued; ++kk)
                mbar_wait(&bar_load[kk & 1], (kk >> 1) & 1, 200000000ull);
            if (mma_pending) mbar_wait(bar_mma, mma_phase, 200000000ull);
            if (d1_pending) mbar_wait(bar_d1, k & 1, 200000000ull);
            atomicExch(&g_solo_status, 1);
        }
        __syncthreads();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, TM_COLS);
}

}  // namespace

int chunk_solo_status(int *flag, bool clear) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_solo_status, sizeof(int));
    if (e == cudaSuccess && clear && v) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_solo_status, &zero, sizeof(int));
    }
    if (e != cudaSuccess) return set_error(RHZ_ERR_DEVICE, "reading the one-CTA kernel's status: %s", cudaGetErrorString(e));
    *flag = v;
    return RHZ_OK;
}

int launch_chunk_solo(const SeqArgs &a) {
    if (a.d != HD || a.dtype != RHZ_DTYPE_BF16)
        return set_error(RHZ_ERR_SHAPE, "tensor-core kernel needs bf16 and head_dim 128 (got %d)", a.d);
    const int64_t tokens = a.cu_seqlens ? a.total_tokens : a.n_seq * a.seq_len;
    if (a.n_seq == 0) return RHZ_OK;
    if (tokens <= 0) {
        // Every sequence is empty: final state = initial state.
        SeqArgs b = a;
        return launch_seq(b);
    }
    CUtensorMap tq, tk, tv;
    int st = make_chunk_tmap(&tq, a.q, tokens, a.H);
    if (st == RHZ_OK) st = make_chunk_tmap(&tk, a.k, tokens, a.H);
    if (st == RHZ_OK) st = make_chunk_tmap(&tv, a.v, tokens, a.H);
    if (st != RHZ_OK) return st;
    int sms = 148;
    bool sm100 = true;
    device_info(&sms, &sm100);
    const int64_t items = a.n_seq * a.H;
    const int grid = static_cast<int>(items < sms ? items : sms);
    static std::once_flag attr_once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(attr_once, [] {
        attr_err = cudaFuncSetAttribute(gdr_chunk_solo_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(SMEM_ALLOC));
    });
    if (attr_err != cudaSuccess)
        return set_error(RHZ_ERR_DEVICE, "gdr_chunk_solo_kernel smem attribute: %s", cudaGetErrorString(attr_err));
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
    gdr_chunk_solo_kernel<<<grid, NT, SMEM_ALLOC, a.stream>>>(tq, tk, tv, p);
    return check_launch("gdr_chunk_solo_kernel");
}

}  // namespace rhz
