// Chunked backward of the gated delta rule on tensor cores (bf16 inputs,
// d = 128, dense batches from a zero state): the WY-form differentiation
// that oracle/chunked_bwd.py restates in f64, split into five launches.
//
// Per chunk of C = 64 positions from the state S0 at its start (P[t][s] =
// prod alpha over (s, t], gamma_t = P[t][-1], pL = P[C-1], A = diag(beta)
// (P . K K^T) strictly lower, T = (I + A)^-1, W = T diag(beta gamma) K,
// M = P . Q K^T lower):
//   Delta = T diag(beta) V - W S0^T,   S_C = gamma_{C-1} S0 + Delta^T diag(pL) K
// and backwards, with dSC the gradient of S_C:
//   dDelta = M^T dO + diag(pL) K dSC^T,
//   dS0 = gamma_{C-1} dSC - dDelta^T W + dO^T diag(gamma) Q.
//
//   gdr_bwdtc_scale_kernel  max |d_o| and max |d_state_final| (below).
//   gdr_bwdtc_rec_kernel    one CTA per chunk: gate tables, [K; Q] K^T, the
//                           solve for T, W; writes the chunk's fp16 record
//                           {T, T diag(beta), M, -W, diag(pL) K, diag(gamma) Q}
//                           and gamma_{C-1}.
//   gdr_bwdtc_chain_kernel  the two serial passes, one CTA per (item, half of
//                           the state's rows): forward S_c (dumping S0 and
//                           Delta^T of every chunk), then the adjoint dS_c in
//                           reverse (dumping dSC and dDelta^T). Rows of S and
//                           dS evolve independently given the records, so each
//                           warp keeps its 16 rows of the state in registers
//                           and the product of one step is the A operand of
//                           the next, straight from its accumulators.
//   gdr_bwdtc_grad_kernel   one CTA per chunk: dq, dk, dv, dalpha, dbeta from
//                           the chunk's inputs, record, S0, dSC, Delta and
//                           dDelta (chunk_bwd of oracle/chunked_bwd.py).
//
// dalpha is formed without dividing by alpha: with dP and dgamma the
// gradients of the decay table and of gamma,
//   dL/dalpha_r = sum_{t >= r} P[t][r] ((dP P^T)[t][r-1] + dgamma_t gamma_{r-1})
// (gamma_{-1} = 1), exact where some alpha is zero. Products take fp16
// operands (mma.sync m16n8k16, fp32 accumulation; bf16 operands miss the
// bf16 tolerance by up to 1.4x on dk in a rounding-point simulation, fp16
// stays under 0.5x); the solve for T uses the fp16 helpers of the forward
// kernels. Every gradient is linear in (d_o, d_state_final), so both enter
// multiplied by s = 2^-e, e the binary exponent of the larger of max |d_o|
// and max |d_state_final|, and the outputs leave multiplied by 1 / s: exact
// scalings that keep the gradient side's fp16 values near 1 whatever the
// loss scale. Inputs q, k, v convert to fp16 exactly within its range
// (|x| < 65504). Every value depends only on its own chunk's data,
// fixed-order sums and a max: the result is deterministic.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>

#include "chunk_common.cuh"
#include "common.cuh"
#include "kernels.h"
#include "mma_f16.cuh"
#include "sm100.cuh"

namespace rhz {
namespace {

using bf16 = __nv_bfloat16;
using mmah::cp16;
using mmah::f16;
using mmah::gemm;
using mmah::gemm_areg;
using mmah::pack_h2;
using mmah::zero;

constexpr int C = chunk::CH;   // 64
constexpr int D = chunk::HD;   // 128
constexpr int AST = chunk::AST;
constexpr int L128 = D + 8;    // padded row strides of shared tiles (bank spread for ldmatrix)
constexpr int L64 = C + 8;

// One chunk's record (fp16 elements, row-major, unpadded).
constexpr int R_T = 0;          // T [t][s]
constexpr int R_TB = 4096;      // T diag(beta) [t][s]
constexpr int R_M = 8192;       // M = P . Q K^T [t][s], lower incl. diagonal
constexpr int R_W = 12288;      // -W [t][j]
constexpr int R_KT = 20480;     // diag(pL) K [s][j]
constexpr int R_QT = 28672;     // diag(gamma) Q [t][j]
constexpr int R_ELEMS = 36864;
constexpr int SD_ELEMS = D * D;  // S0 / dSC dump [i][j]
constexpr int DD_ELEMS = D * C;  // Delta^T / dDelta^T dump [i][s]

struct BtParams {
    const bf16 *q, *k, *v, *d_o;
    const float *alpha, *beta;
    const float *d_state_final;  // [B][H][d][d] or null
    bf16 *dq, *dk, *dv;
    float *dalpha, *dbeta;
    f16 *rec;
    float *g63;
    f16 *s_dump, *ds_dump, *d_dump, *dd_dump;
    unsigned *gmax;              // bits of max(|d_o|, |d_state_final|)
    int64_t B, T;
    int H, nch;
};

struct ChunkPos {
    int64_t item, tok0;  // tok0: the chunk's first token row (b T + c C)
    int c, h, L;
};

__device__ __forceinline__ ChunkPos chunk_pos(const BtParams &p, int64_t chunk) {
    ChunkPos r;
    r.item = chunk / p.nch;
    r.c = static_cast<int>(chunk - r.item * p.nch);
    const int64_t b = r.item / p.H;
    r.h = static_cast<int>(r.item - b * p.H);
    r.tok0 = b * p.T + static_cast<int64_t>(r.c) * C;
    const int64_t rem = p.T - static_cast<int64_t>(r.c) * C;
    r.L = static_cast<int>(rem < C ? rem : C);
    return r;
}

__device__ __forceinline__ const bf16 *row_ptr(const bf16 *x, const BtParams &p, const ChunkPos &cp, int t) {
    return x + ((cp.tok0 + t) * p.H + cp.h) * static_cast<int64_t>(D);
}

// Rows t < L of a [tokens][H][128] bf16 array (columns col0 .. col0 + 8
// nchunk16 - 1) into a padded shared tile, still bf16 (to_f16 converts it);
// rows past L read as zeros.
__device__ __forceinline__ void load_rows(f16 *dst, int ld, const bf16 *src, const BtParams &p,
                                          const ChunkPos &cp, int col0, int nchunk16, int tid, int nthr) {
    for (int i = tid; i < C * nchunk16; i += nthr) {
        const int r = i / nchunk16, c16 = i - r * nchunk16;
        const bool in = r < cp.L;
        const bf16 *s = in ? row_ptr(src, p, cp, r) + col0 + 8 * c16 : src;
        cp16(dst + r * ld + 8 * c16, s, in ? 16 : 0);
    }
}

// rows x (8 nchunk16) fp16 block stored densely (row stride 8 nchunk16) into a padded tile.
__device__ __forceinline__ void load_dense(f16 *dst, int ld, const f16 *src, int rows, int nchunk16, int tid,
                                           int nthr) {
    for (int i = tid; i < rows * nchunk16; i += nthr) {
        const int r = i / nchunk16, c16 = i - r * nchunk16;
        cp16(dst + r * ld + 8 * c16, src + static_cast<int64_t>(r) * nchunk16 * 8 + 8 * c16, 16);
    }
}

// Gate tables of one chunk (one warp): padded positions alpha = 1, beta = 0.
__device__ __forceinline__ void chunk_gates(float *g, const BtParams &p, const ChunkPos &cp, int lane) {
    chunk::GateIn in{1.f, 1.f, 0.f, 0.f};
    const int p0 = 2 * lane, p1 = p0 + 1;
    if (p0 < cp.L) {
        const int64_t i = (cp.tok0 + p0) * p.H + cp.h;
        in.a0 = p.alpha[i];
        in.b0 = p.beta[i];
    }
    if (p1 < cp.L) {
        const int64_t i = (cp.tok0 + p1) * p.H + cp.h;
        in.a1 = p.alpha[i];
        in.b1 = p.beta[i];
    }
    chunk::gate_tables(g, in, lane);
}

// P[t][s] (s <= t) from the gate tables: 0 when a zero alpha lies in (s, t].
__device__ __forceinline__ float pdec(const float *g, int t, int s) {
    const int *z = reinterpret_cast<const int *>(g + chunk::G_Z);
    return z[t] == z[s] ? chunk::ex2(g[chunk::G_GL + t] - g[chunk::G_GL + s]) : 0.f;
}

__device__ __forceinline__ void st2(f16 *p, float a, float b) {
    *reinterpret_cast<uint32_t *>(p) = pack_h2(a, b);
}

// A shared tile loaded as bf16 (rows x cols, row stride ld) to fp16 in
// place, times `scale`.
__device__ __forceinline__ void to_f16(f16 *t, int ld, int rows, int cols, float scale, int tid, int nthr) {
    const int pairs = cols / 2;
    for (int i = tid; i < rows * pairs; i += nthr) {
        const int r = i / pairs, c = 2 * (i - r * pairs);
        uint32_t *w = reinterpret_cast<uint32_t *>(t + r * ld + c);
        const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(w));
        *w = pack_h2(f.x * scale, f.y * scale);
    }
}

// s = 2^-e for the gradient side (e the binary exponent of the max; 1 when
// every gradient is zero).
__device__ __forceinline__ float grad_scale(const unsigned *gmax) {
    const unsigned bits = *gmax;
    if (bits == 0) return 1.f;
    int e = static_cast<int>((bits >> 23) & 255u) - 127;
    e = e < -126 ? -126 : (e > 126 ? 126 : e);
    return __uint_as_float(static_cast<unsigned>(127 - e) << 23);
}

// ---------------------------------------------------------------- scale

__global__ void gdr_bwdtc_scale_kernel(const BtParams p, int64_t n_do, int64_t n_sf) {
    float m = 0.f;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 8; i < n_do; i += stride * 8) {
        const uint4 u = *reinterpret_cast<const uint4 *>(p.d_o + i);  // 8 values (n_do is a multiple of 128)
        const __nv_bfloat162 *h = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 f = __bfloat1622float2(h[e]);
            m = fmaxf(m, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
    }
    if (p.d_state_final) {
        for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_sf; i += stride)
            m = fmaxf(m, fabsf(p.d_state_final[i]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0 && m > 0.f) atomicMax(p.gmax, __float_as_uint(m));  // non-negative floats order as their bits
}

// ---------------------------------------------------------------- records

constexpr uint32_t RK_KS = 0;
constexpr uint32_t RK_QS = RK_KS + C * L128 * 2;
constexpr uint32_t RK_AF = RK_QS + C * L128 * 2;
constexpr uint32_t RK_TF = RK_AF + C * AST * 4;
constexpr uint32_t RK_XF = RK_TF + C * AST * 4;
constexpr uint32_t RK_TB = RK_XF + 4096;
constexpr uint32_t RK_G = RK_TB + C * L64 * 2;
constexpr uint32_t RK_SMEM = RK_G + chunk::G_BYTES;

__global__ void __launch_bounds__(256) gdr_bwdtc_rec_kernel(const BtParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    f16 *Ks = reinterpret_cast<f16 *>(smem + RK_KS);
    f16 *Qs = reinterpret_cast<f16 *>(smem + RK_QS);
    float *Af = reinterpret_cast<float *>(smem + RK_AF);
    float *Tf = reinterpret_cast<float *>(smem + RK_TF);
    float *Xf = reinterpret_cast<float *>(smem + RK_XF);
    f16 *Tb = reinterpret_cast<f16 *>(smem + RK_TB);
    float *gt = reinterpret_cast<float *>(smem + RK_G);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tq = lane & 3;
    const int64_t chunk = blockIdx.x;
    const ChunkPos cp = chunk_pos(p, chunk);
    f16 *rec = p.rec + chunk * R_ELEMS;

    load_rows(Ks, L128, p.k, p, cp, 0, 16, tid, 256);
    load_rows(Qs, L128, p.q, p, cp, 0, 16, tid, 256);
    mmah::cp_commit();
    if (warp == 0) chunk_gates(gt, p, cp, lane);
    mmah::cp_wait<0>();
    __syncthreads();
    to_f16(Ks, L128, C, D, 1.f, tid, 256);
    to_f16(Qs, L128, C, D, 1.f, tid, 256);
    __syncthreads();

    // ---- K K^T (warps 0-3) and Q K^T (warps 4-7), one 16-row block each
    {
        const int mt = warp & 3;
        float acc[8][4];
        zero(acc);
        gemm<8, 8, true, true>(acc, warp < 4 ? Ks : Qs, L128, 16 * mt, 0, Ks, L128, 0, 0, lane);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int t = 16 * mt + g + 8 * hh;
                const int s0 = 8 * nt + 2 * tq;
                float v[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int s = s0 + e;
                    const float x = acc[nt][2 * hh + e];
                    if (warp < 4)
                        v[e] = s < t ? gt[chunk::G_BE + t] * pdec(gt, t, s) * x : 0.f;
                    else
                        v[e] = s <= t ? pdec(gt, t, s) * x : 0.f;
                }
                if (warp < 4) {
                    Af[t * AST + s0] = v[0];
                    Af[t * AST + s0 + 1] = v[1];
                } else {
                    st2(rec + R_M + t * C + s0, v[0], v[1]);
                }
            }
    }
    __syncthreads();

    // ---- T = (I + A)^-1: diagonal 16 x 16 inverses (warps 0-3) while warps
    // 4-7 clear T's upper triangle, then the off-diagonal blocks
    if (warp < 4) {
        chunk::diag_inverse16(Af + (16 * warp) * AST + 16 * warp, Tf + (16 * warp) * AST + 16 * warp, lane);
    } else {
        for (int e = tid - 128; e < C * C; e += 128) {
            const int r = e >> 6, s = e & 63;
            if ((s >> 4) > (r >> 4)) Tf[r * AST + s] = 0.f;
        }
    }
    __syncthreads();
    chunk::solve_offdiag(Af, Tf, Xf, warp, lane, 1);

    // ---- T, T diag(beta) to the record; T diag(beta gamma) for W
    for (int i = tid; i < C * C / 2; i += 256) {
        const int t = i >> 5, s = (i & 31) * 2;
        const float x0 = s <= t ? Tf[t * AST + s] : 0.f;
        const float x1 = s + 1 <= t ? Tf[t * AST + s + 1] : 0.f;
        st2(rec + R_T + t * C + s, x0, x1);
        st2(rec + R_TB + t * C + s, x0 * gt[chunk::G_BE + s], x1 * gt[chunk::G_BE + s + 1]);
        st2(Tb + t * L64 + s, x0 * gt[chunk::G_BG + s], x1 * gt[chunk::G_BG + s + 1]);
    }
    __syncthreads();

    // ---- -W = -(T diag(beta gamma)) K
    {
        const int mt = warp & 3, n0 = 64 * (warp >> 2);
        float acc[8][4];
        zero(acc);
        gemm<8, 4, true, false>(acc, Tb, L64, 16 * mt, 0, Ks, L128, 0, n0, lane);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const int t = 16 * mt + g + 8 * hh;
                st2(rec + R_W + t * D + n0 + 8 * nt + 2 * tq, -acc[nt][2 * hh], -acc[nt][2 * hh + 1]);
            }
    }
    // ---- diag(pL) K and diag(gamma) Q
    for (int i = tid; i < C * D / 2; i += 256) {
        const int r = i >> 6, j = (i & 63) * 2;
        const float2 kk = __half22float2(*reinterpret_cast<const __half2 *>(Ks + r * L128 + j));
        const float2 qq = __half22float2(*reinterpret_cast<const __half2 *>(Qs + r * L128 + j));
        const float pl = gt[chunk::G_PL + r], gm = gt[chunk::G_GM + r];
        st2(rec + R_KT + r * D + j, pl * kk.x, pl * kk.y);
        st2(rec + R_QT + r * D + j, gm * qq.x, gm * qq.y);
    }
    if (tid == 0) p.g63[chunk] = gt[chunk::G_GM + C - 1];
}

// ---------------------------------------------------------------- chains

// Stage layouts (fp16 tiles, padded rows).
constexpr uint32_t CF_TB = 0;                       // T diag(beta), the record's [t][s]
constexpr uint32_t CF_WN = CF_TB + C * L64 * 2;     // -W [s][j]
constexpr uint32_t CF_KT = CF_WN + C * L128 * 2;    // diag(pL) K [s][j]
constexpr uint32_t CF_V = CF_KT + C * L128 * 2;     // V [t][this half's 64 i]
constexpr uint32_t CF_STAGE = CF_V + C * L64 * 2;
constexpr uint32_t CA_M = 0;                        // M [t][s]
constexpr uint32_t CA_WN = CA_M + C * L64 * 2;      // -W [s][j]
constexpr uint32_t CA_KT = CA_WN + C * L128 * 2;    // diag(pL) K [s][j]
constexpr uint32_t CA_QT = CA_KT + C * L128 * 2;    // diag(gamma) Q [t][j]
constexpr uint32_t CA_DO = CA_QT + C * L128 * 2;    // dO [t][this half's 64 i]
constexpr uint32_t CA_STAGE = CA_DO + C * L64 * 2;

template <bool ADJ>
__device__ __forceinline__ void chain_load(uint8_t *st, const BtParams &p, int64_t item, int c, int half,
                                           int tid) {
    const int64_t chunk = item * p.nch + c;
    const f16 *rec = p.rec + chunk * R_ELEMS;
    const ChunkPos cp = chunk_pos(p, chunk);
    if (!ADJ) {
        load_dense(reinterpret_cast<f16 *>(st + CF_TB), L64, rec + R_TB, C, 8, tid, 128);
        load_dense(reinterpret_cast<f16 *>(st + CF_WN), L128, rec + R_W, C, 16, tid, 128);
        load_dense(reinterpret_cast<f16 *>(st + CF_KT), L128, rec + R_KT, C, 16, tid, 128);
        load_rows(reinterpret_cast<f16 *>(st + CF_V), L64, p.v, p, cp, 64 * half, 8, tid, 128);
    } else {
        load_dense(reinterpret_cast<f16 *>(st + CA_M), L64, rec + R_M, C, 8, tid, 128);
        load_dense(reinterpret_cast<f16 *>(st + CA_WN), L128, rec + R_W, C, 16, tid, 128);
        load_dense(reinterpret_cast<f16 *>(st + CA_KT), L128, rec + R_KT, C, 16, tid, 128);
        load_dense(reinterpret_cast<f16 *>(st + CA_QT), L128, rec + R_QT, C, 16, tid, 128);
        load_rows(reinterpret_cast<f16 *>(st + CA_DO), L64, p.d_o, p, cp, 64 * half, 8, tid, 128);
    }
}

// The warp's rows (16 from row0) of an accumulator set to an fp16 dump of
// row stride ld.
template <int NT>
__device__ __forceinline__ void dump_rows(f16 *dst, int ld, const float (&x)[NT][4], int lane) {
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        st2(dst + g * ld + 8 * nt + 2 * tq, x[nt][0], x[nt][1]);
        st2(dst + (g + 8) * ld + 8 * nt + 2 * tq, x[nt][2], x[nt][3]);
    }
}

template <bool ADJ>
__global__ void __launch_bounds__(128, 1) gdr_bwdtc_chain_kernel(const BtParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr uint32_t STAGE = ADJ ? CA_STAGE : CF_STAGE;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t item = blockIdx.x >> 1;
    const int half = blockIdx.x & 1;
    const int row0 = 64 * half + 16 * warp;  // the warp's first state row
    const int n = p.nch;

    float X[16][4];  // state rows row0 .. row0 + 15, all 128 columns
    zero(X);
    const float gs = ADJ ? grad_scale(p.gmax) : 1.f;
    if (ADJ && p.d_state_final) {
        const int g = lane >> 2, tq = lane & 3;
        const float *src = p.d_state_final + item * static_cast<int64_t>(SD_ELEMS) + static_cast<int64_t>(row0) * D;
#pragma unroll
        for (int nt = 0; nt < 16; ++nt) {
            const float2 a = *reinterpret_cast<const float2 *>(src + g * D + 8 * nt + 2 * tq);
            const float2 b = *reinterpret_cast<const float2 *>(src + (g + 8) * D + 8 * nt + 2 * tq);
            X[nt][0] = gs * a.x; X[nt][1] = gs * a.y; X[nt][2] = gs * b.x; X[nt][3] = gs * b.y;
        }
    }
    // chunk order: forward 0 .. n-1, adjoint n-1 .. 0
    auto chunk_at = [&](int it) { return ADJ ? n - 1 - it : it; };
    chain_load<ADJ>(smem, p, item, chunk_at(0), half, tid);
    mmah::cp_commit();
    if (n > 1) chain_load<ADJ>(smem + STAGE, p, item, chunk_at(1), half, tid);
    mmah::cp_commit();

#pragma unroll 1
    for (int it = 0; it < n; ++it) {
        const int c = chunk_at(it);
        uint8_t *st = smem + (it & 1) * STAGE;
        mmah::cp_wait<1>();
        __syncthreads();
        // this stage's V (or dO) columns arrived as bf16
        to_f16(reinterpret_cast<f16 *>(st + (ADJ ? CA_DO : CF_V)), L64, C, 64, gs, tid, 128);
        __syncthreads();
        const int64_t chunk = item * n + c;
        float E[8][4];  // Delta^T (forward) or dDelta^T (adjoint): rows row0.., 64 columns s
        zero(E);
        if (!ADJ) {
            dump_rows(p.s_dump + chunk * SD_ELEMS + static_cast<int64_t>(row0) * D, D, X, lane);
            const f16 *Vt = reinterpret_cast<const f16 *>(st + CF_V);
            // U^T = V^T (T diag b)^T, then - S W^T
            gemm<8, 4, false, true>(E, Vt, L64, 16 * warp, 0, reinterpret_cast<const f16 *>(st + CF_TB), L64, 0, 0, lane);
            gemm_areg<8, 8, true>(E, X, reinterpret_cast<const f16 *>(st + CF_WN), L128, 0, 0, lane);
            dump_rows(p.d_dump + chunk * DD_ELEMS + static_cast<int64_t>(row0) * C, C, E, lane);
            const float gm = p.g63[chunk];
#pragma unroll
            for (int nt = 0; nt < 16; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) X[nt][e] *= gm;
            // S += Delta^T diag(pL) K
            gemm_areg<16, 4, false>(X, E, reinterpret_cast<const f16 *>(st + CF_KT), L128, 0, 0, lane);
        } else {
            dump_rows(p.ds_dump + chunk * SD_ELEMS + static_cast<int64_t>(row0) * D, D, X, lane);
            const f16 *dOt = reinterpret_cast<const f16 *>(st + CA_DO);
            // dDelta^T = dO^T M + dSC (diag(pL) K)^T
            gemm<8, 4, false, false>(E, dOt, L64, 16 * warp, 0, reinterpret_cast<const f16 *>(st + CA_M), L64, 0, 0, lane);
            gemm_areg<8, 8, true>(E, X, reinterpret_cast<const f16 *>(st + CA_KT), L128, 0, 0, lane);
            dump_rows(p.dd_dump + chunk * DD_ELEMS + static_cast<int64_t>(row0) * C, C, E, lane);
            const float gm = p.g63[chunk];
#pragma unroll
            for (int nt = 0; nt < 16; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) X[nt][e] *= gm;
            // dS0 = gamma dSC + dDelta^T (-W) + dO^T diag(gamma) Q
            gemm_areg<16, 4, false>(X, E, reinterpret_cast<const f16 *>(st + CA_WN), L128, 0, 0, lane);
            gemm<16, 4, false, false>(X, dOt, L64, 16 * warp, 0, reinterpret_cast<const f16 *>(st + CA_QT), L128, 0, 0, lane);
        }
        __syncthreads();  // every warp is done with this stage
        if (it + 2 < n) chain_load<ADJ>(st, p, item, chunk_at(it + 2), half, tid);
        mmah::cp_commit();
    }
    mmah::cp_wait<0>();
}

// ---------------------------------------------------------------- gradients

constexpr uint32_t GK_Q = 0;
constexpr uint32_t GK_K = GK_Q + C * L128 * 2;
constexpr uint32_t GK_V = GK_K + C * L128 * 2;
constexpr uint32_t GK_DO = GK_V + C * L128 * 2;
constexpr uint32_t GK_BUF = GK_DO + C * L128 * 2;     // dSC, then S0 [i][j]
constexpr uint32_t GK_DT = GK_BUF + D * L128 * 2;     // Delta^T [i][s]
constexpr uint32_t GK_DDT = GK_DT + D * L64 * 2;      // dDelta^T [i][s]
constexpr uint32_t GK_T = GK_DDT + D * L64 * 2;       // T [t][s]
constexpr uint32_t GK_DMP = GK_T + C * L64 * 2;       // dM . P [t][s]
constexpr uint32_t GK_DW = GK_DMP + C * L64 * 2;      // dW [s][j]
constexpr uint32_t GK_DTT = GK_DW + C * L128 * 2;     // dT [t][s]
constexpr uint32_t GK_E1 = GK_DTT + C * L64 * 2;      // dT T^T, later P [t][s]
constexpr uint32_t GK_DKK = GK_E1 + C * L64 * 2;      // dKK [s][u]
constexpr uint32_t GK_DP = GK_DKK + C * L64 * 2;      // dP [t][s]
constexpr uint32_t GK_GATE = GK_DP + C * L64 * 2;
constexpr uint32_t GK_RED = GK_GATE + chunk::G_BYTES;
constexpr int RED_DG = 0, RED_DB1 = 128, RED_DBG = 256, RED_DB2 = 384, RED_PD = 512, RED_DGAM = 640,
              RED_WS = 704, RED_FLOATS = 720;
constexpr uint32_t GK_SMEM = GK_RED + RED_FLOATS * 4;
constexpr uint32_t GK_G = GK_DW;                      // (dP P^T) fp32 [64][65], after dW and dT are used
static_assert(GK_G + C * 65 * 4 <= GK_E1, "G fits over dW and dT");
static_assert(GK_SMEM <= 232448, "shared memory per CTA");

// Sum of the values of the four lanes that share an accumulator row.
__device__ __forceinline__ float quad_sum(float x) {
    x += __shfl_xor_sync(0xffffffffu, x, 1);
    x += __shfl_xor_sync(0xffffffffu, x, 2);
    return x;
}

// Row sums over this warp's columns of acc (.) Y (Y an fp16 tile [row][col]),
// written to red[part][row] by the lane with tq == 0.
template <int NT>
__device__ __forceinline__ void row_dot(float *red, int part, const float (&acc)[NT][4], const f16 *Y, int ld,
                                        int m0, int c0, int lane) {
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int r = m0 + g + 8 * hh;
        float s = 0.f;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const float2 y = __half22float2(*reinterpret_cast<const __half2 *>(Y + r * ld + c0 + 8 * nt + 2 * tq));
            s += acc[nt][2 * hh] * y.x + acc[nt][2 * hh + 1] * y.y;
        }
        s = quad_sum(s);
        if (tq == 0) red[part * 64 + r] = s;
    }
}

// Rows t < L of the warp's 16 x (8 NT) block (columns from c0) times
// `scale` to a [tokens][H][128] bf16 output.
template <int NT>
__device__ __forceinline__ void store_rows(bf16 *dst, const BtParams &p, const ChunkPos &cp, const float (&acc)[NT][4],
                                           int m0, int c0, float scale, int lane) {
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const int r = m0 + g + 8 * hh;
        if (r >= cp.L) continue;
        bf16 *row = dst + ((cp.tok0 + r) * p.H + cp.h) * static_cast<int64_t>(D);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            __nv_bfloat162 v = __floats2bfloat162_rn(scale * acc[nt][2 * hh], scale * acc[nt][2 * hh + 1]);
            *reinterpret_cast<__nv_bfloat162 *>(row + c0 + 8 * nt + 2 * tq) = v;
        }
    }
}

__global__ void __launch_bounds__(256, 1) gdr_bwdtc_grad_kernel(const BtParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    f16 *Qs = reinterpret_cast<f16 *>(smem + GK_Q);
    f16 *Ks = reinterpret_cast<f16 *>(smem + GK_K);
    f16 *Vs = reinterpret_cast<f16 *>(smem + GK_V);
    f16 *dOs = reinterpret_cast<f16 *>(smem + GK_DO);
    f16 *BUF = reinterpret_cast<f16 *>(smem + GK_BUF);
    f16 *DTs = reinterpret_cast<f16 *>(smem + GK_DT);
    f16 *dDTs = reinterpret_cast<f16 *>(smem + GK_DDT);
    f16 *Ts = reinterpret_cast<f16 *>(smem + GK_T);
    f16 *dMPs = reinterpret_cast<f16 *>(smem + GK_DMP);
    f16 *dWs = reinterpret_cast<f16 *>(smem + GK_DW);
    f16 *dTs = reinterpret_cast<f16 *>(smem + GK_DTT);
    f16 *E1s = reinterpret_cast<f16 *>(smem + GK_E1);
    f16 *dKKs = reinterpret_cast<f16 *>(smem + GK_DKK);
    f16 *dPs = reinterpret_cast<f16 *>(smem + GK_DP);
    float *gt = reinterpret_cast<float *>(smem + GK_GATE);
    float *red = reinterpret_cast<float *>(smem + GK_RED);
    float *Gm = reinterpret_cast<float *>(smem + GK_G);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, tq = lane & 3;
    const int64_t chunk = blockIdx.x;
    const ChunkPos cp = chunk_pos(p, chunk);
    const f16 *rec = p.rec + chunk * R_ELEMS;
    const f16 *s0g = p.s_dump + chunk * SD_ELEMS;
    const f16 *dscg = p.ds_dump + chunk * SD_ELEMS;
    const float gs = grad_scale(p.gmax), inv_gs = 1.f / gs;

    load_rows(Qs, L128, p.q, p, cp, 0, 16, tid, 256);
    load_rows(Ks, L128, p.k, p, cp, 0, 16, tid, 256);
    load_rows(Vs, L128, p.v, p, cp, 0, 16, tid, 256);
    load_rows(dOs, L128, p.d_o, p, cp, 0, 16, tid, 256);
    load_dense(BUF, L128, dscg, D, 16, tid, 256);
    load_dense(DTs, L64, p.d_dump + chunk * DD_ELEMS, D, 8, tid, 256);
    load_dense(dDTs, L64, p.dd_dump + chunk * DD_ELEMS, D, 8, tid, 256);
    load_dense(Ts, L64, rec + R_T, C, 8, tid, 256);
    mmah::cp_commit();
    if (warp == 0) chunk_gates(gt, p, cp, lane);
    mmah::cp_wait<0>();
    __syncthreads();
    to_f16(Qs, L128, C, D, 1.f, tid, 256);
    to_f16(Ks, L128, C, D, 1.f, tid, 256);
    to_f16(Vs, L128, C, D, 1.f, tid, 256);
    to_f16(dOs, L128, C, D, gs, tid, 256);
    __syncthreads();

    // 64 x 64 blocks: rows 16 mt.., columns c64 .. c64 + 31; 64 x 128: columns c128 .. c128 + 63.
    const int mt = warp & 3, m0 = 16 * mt;
    const int c64 = 32 * (warp >> 2), c128 = 64 * (warp >> 2), part = warp >> 2;
    auto row_of = [&](int hh) { return m0 + g + 8 * hh; };
    auto col_of = [&](int nt, int e) { return 8 * nt + 2 * tq + e; };

    // ---- K K^T, Q K^T, P on this warp's 64 x 64 block
    float KKf[4][4], QKf[4][4], Pf[4][4], dPf[4][4];
    zero(KKf);
    zero(QKf);
    gemm<4, 8, true, true>(KKf, Ks, L128, m0, 0, Ks, L128, 0, c64, lane);
    gemm<4, 8, true, true>(QKf, Qs, L128, m0, 0, Ks, L128, 0, c64, lane);
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int t = row_of(e >> 1), s = c64 + col_of(nt, e & 1);
            Pf[nt][e] = s <= t ? pdec(gt, t, s) : 0.f;
        }

    // ---- dM = tril(dO Delta^T); dM . P (for dq, dk) and dP = dM . QK
    {
        float dM[4][4];
        zero(dM);
        gemm<4, 8, true, false>(dM, dOs, L128, m0, 0, DTs, L64, 0, c64, lane);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const float a = dM[nt][2 * hh] * Pf[nt][2 * hh], b = dM[nt][2 * hh + 1] * Pf[nt][2 * hh + 1];
                st2(dMPs + row_of(hh) * L64 + c64 + col_of(nt, 0), a, b);
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int t = row_of(hh), s = c64 + col_of(nt, e);
                    dPf[nt][2 * hh + e] = s <= t ? dM[nt][2 * hh + e] * QKf[nt][2 * hh + e] : 0.f;
                }
            }
    }

    // ---- Delta dSC: dk = diag(pL) (Delta dSC); dpL = rowsum(K . (Delta dSC))
    float dkf[8][4];
    {
        float DdS[8][4];
        zero(DdS);
        gemm<8, 8, false, false>(DdS, DTs, L64, m0, 0, BUF, L128, 0, c128, lane);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) dkf[nt][e] = gt[chunk::G_PL + row_of(e >> 1)] * DdS[nt][e];
        row_dot<8>(red + RED_PD, part, DdS, Ks, L128, m0, c128, lane);
    }
    // ---- sum(dSC . S0) for dgamma_{C-1}
    {
        float s = 0.f;
        const int base = tid * 64;  // 64 consecutive elements of the 128 x 128 block
        const int i = base >> 7, j0 = base & 127;
#pragma unroll
        for (int q8 = 0; q8 < 8; ++q8) {
            const uint4 a = *reinterpret_cast<const uint4 *>(s0g + base + 8 * q8);
            const uint4 b = *reinterpret_cast<const uint4 *>(BUF + i * L128 + j0 + 8 * q8);
            const __half2 *ah = reinterpret_cast<const __half2 *>(&a);
            const __half2 *bh = reinterpret_cast<const __half2 *>(&b);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 x = __half22float2(ah[e]), y = __half22float2(bh[e]);
                s += x.x * y.x + x.y * y.y;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) red[RED_WS + warp] = s;
    }
    __syncthreads();  // dSC is no longer read: S0 takes its place
    load_dense(BUF, L128, s0g, D, 16, tid, 256);
    mmah::cp_commit();
    mmah::cp_wait<0>();
    __syncthreads();

    // ---- X = dO S0: dgamma partial rowsum(X . Q); dq = diag(gamma) X + (dM . P) K
    {
        float Xf[8][4];
        zero(Xf);
        gemm<8, 8, true, false>(Xf, dOs, L128, m0, 0, BUF, L128, 0, c128, lane);
        row_dot<8>(red + RED_DG, part, Xf, Qs, L128, m0, c128, lane);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) Xf[nt][e] *= gt[chunk::G_GM + row_of(e >> 1)];
        gemm<8, 4, true, false>(Xf, dMPs, L64, m0, 0, Ks, L128, 0, c128, lane);
        store_rows<8>(p.dq, p, cp, Xf, m0, c128, inv_gs, lane);
    }
    // ---- dk += (dM . P)^T Q
    gemm<8, 4, false, false>(dkf, dMPs, L64, m0, 0, Qs, L128, 0, c128, lane);
    // ---- dW = -dDelta S0
    {
        float Wf[8][4];
        zero(Wf);
        gemm<8, 8, false, false>(Wf, dDTs, L64, m0, 0, BUF, L128, 0, c128, lane);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
                st2(dWs + row_of(hh) * L128 + c128 + col_of(nt, 0), -Wf[nt][2 * hh], -Wf[nt][2 * hh + 1]);
    }
    __syncthreads();

    // ---- dY = T^T dDelta: dv = diag(beta) dY, dbeta += rowsum(dY . V)
    {
        float Yf[8][4];
        zero(Yf);
        gemm<8, 4, false, true>(Yf, Ts, L64, m0, 0, dDTs, L64, 0, c128, lane);
        row_dot<8>(red + RED_DB1, part, Yf, Vs, L128, m0, c128, lane);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) Yf[nt][e] *= gt[chunk::G_BE + row_of(e >> 1)];
        store_rows<8>(p.dv, p, cp, Yf, m0, c128, inv_gs, lane);
    }
    // ---- dZ = T^T dW: dk += diag(beta gamma) dZ, dbg = rowsum(dZ . K)
    {
        float Zf[8][4];
        zero(Zf);
        gemm<8, 4, false, false>(Zf, Ts, L64, m0, 0, dWs, L128, 0, c128, lane);
        row_dot<8>(red + RED_DBG, part, Zf, Ks, L128, m0, c128, lane);
#pragma unroll
        for (int nt = 0; nt < 8; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) dkf[nt][e] += gt[chunk::G_BG + row_of(e >> 1)] * Zf[nt][e];
    }
    // ---- dT = dDelta Y^T + dW Z^T = (dDelta V^T) diag(beta) + (dW K^T) diag(beta gamma)
    {
        float P1[4][4], P2[4][4];
        zero(P1);
        zero(P2);
        gemm<4, 8, false, true>(P1, dDTs, L64, m0, 0, Vs, L128, 0, c64, lane);
        gemm<4, 8, true, true>(P2, dWs, L128, m0, 0, Ks, L128, 0, c64, lane);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                float v[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int s = c64 + col_of(nt, e);
                    v[e] = gt[chunk::G_BE + s] * P1[nt][2 * hh + e] + gt[chunk::G_BG + s] * P2[nt][2 * hh + e];
                }
                st2(dTs + row_of(hh) * L64 + c64 + col_of(nt, 0), v[0], v[1]);
            }
    }
    __syncthreads();
    // ---- E1 = dT T^T
    {
        float Ef[4][4];
        zero(Ef);
        gemm<4, 4, true, true>(Ef, dTs, L64, m0, 0, Ts, L64, 0, c64, lane);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
                st2(E1s + row_of(hh) * L64 + c64 + col_of(nt, 0), Ef[nt][2 * hh], Ef[nt][2 * hh + 1]);
    }
    __syncthreads();
    // ---- dA = strict_lower(-T^T E1): dbeta += rowsum(dA . P . KK), dP += dA beta KK, dKK = dA beta P
    {
        float dA[4][4];
        zero(dA);
        gemm<4, 4, false, false>(dA, Ts, L64, m0, 0, E1s, L64, 0, c64, lane);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int t = row_of(hh);
            const float bt = gt[chunk::G_BE + t];
            float rs = 0.f;
            float kk[4][2];
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int s = c64 + col_of(nt, e);
                    const float a = s < t ? -dA[nt][2 * hh + e] : 0.f;
                    rs += a * Pf[nt][2 * hh + e] * KKf[nt][2 * hh + e];
                    dPf[nt][2 * hh + e] += a * bt * KKf[nt][2 * hh + e];
                    kk[nt][e] = a * bt * Pf[nt][2 * hh + e];
                }
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) st2(dKKs + t * L64 + c64 + col_of(nt, 0), kk[nt][0], kk[nt][1]);
            rs = quad_sum(rs);
            if (tq == 0) red[RED_DB2 + part * 64 + t] = rs;
        }
    }
    __syncthreads();
    // ---- dk += dKK K + dKK^T K; dP row C-1 += dpL; dP and P as fp16 tiles
    gemm<8, 4, true, false>(dkf, dKKs, L64, m0, 0, Ks, L128, 0, c128, lane);
    gemm<8, 4, false, false>(dkf, dKKs, L64, m0, 0, Ks, L128, 0, c128, lane);
    store_rows<8>(p.dk, p, cp, dkf, m0, c128, inv_gs, lane);
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int t = row_of(hh);
            float v[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int s = c64 + col_of(nt, e);
                v[e] = dPf[nt][2 * hh + e] + (t == C - 1 ? red[RED_PD + s] + red[RED_PD + 64 + s] : 0.f);
            }
            st2(dPs + t * L64 + c64 + col_of(nt, 0), v[0], v[1]);
            st2(E1s + t * L64 + c64 + col_of(nt, 0), Pf[nt][2 * hh], Pf[nt][2 * hh + 1]);
        }
    __syncthreads();
    // ---- G = dP P^T (fp32 to shared); dgamma
    {
        float Gf[4][4];
        zero(Gf);
        gemm<4, 4, true, true>(Gf, dPs, L64, m0, 0, E1s, L64, 0, c64, lane);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) Gm[row_of(e >> 1) * 65 + c64 + col_of(nt, e & 1)] = Gf[nt][e];
    }
    if (tid < C) {
        const int t = tid;
        float w = 0.f;
        if (t == C - 1) {
#pragma unroll
            for (int i = 0; i < 8; ++i) w += red[RED_WS + i];
        }
        const float dbg = red[RED_DBG + t] + red[RED_DBG + 64 + t];
        red[RED_DGAM + t] = red[RED_DG + t] + red[RED_DG + 64 + t] + w + gt[chunk::G_BE + t] * dbg;
    }
    __syncthreads();
    // ---- dalpha_r = sum_{t >= r} P[t][r] (G[t][r-1] + dgamma_t gamma_{r-1}); dbeta
    if (tid < C) {
        const int r = tid;
        const float gprev = r > 0 ? gt[chunk::G_GM + r - 1] : 1.f;
        float da = 0.f;
        for (int t = r; t < C; ++t) {
            const float h = (r > 0 ? Gm[t * 65 + r - 1] : 0.f) + red[RED_DGAM + t] * gprev;
            da += pdec(gt, t, r) * h;
        }
        const float dbg = red[RED_DBG + r] + red[RED_DBG + 64 + r];
        const float db = red[RED_DB1 + r] + red[RED_DB1 + 64 + r] + gt[chunk::G_GM + r] * dbg + red[RED_DB2 + r] +
                         red[RED_DB2 + 64 + r];
        if (r < cp.L) {
            const int64_t i = (cp.tok0 + r) * p.H + cp.h;
            p.dalpha[i] = da * inv_gs;
            p.dbeta[i] = db * inv_gs;
        }
    }
}

struct BtWs {
    size_t gmax, rec, g63, s_dump, ds_dump, d_dump, dd_dump, total;
};

BtWs bt_ws(int64_t chunks) {
    auto up = [](size_t x) { return (x + 255) / 256 * 256; };
    const size_t n = static_cast<size_t>(chunks > 0 ? chunks : 0);
    BtWs w{};
    w.gmax = 0;
    w.rec = 256;
    w.g63 = w.rec + up(n * R_ELEMS * 2);
    w.s_dump = w.g63 + up(n * 4);
    w.ds_dump = w.s_dump + up(n * SD_ELEMS * 2);
    w.d_dump = w.ds_dump + up(n * SD_ELEMS * 2);
    w.dd_dump = w.d_dump + up(n * DD_ELEMS * 2);
    w.total = w.dd_dump + up(n * DD_ELEMS * 2);
    return w;
}

std::atomic<int> g_bwd_form{0};  // 0: tensor-core path where it applies, 1: fp32 reverse scan always

}  // namespace

bool bwd_tc_supports(const BwdArgs &a) {
    auto al16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    return g_bwd_form.load() == 0 && a.dtype == RHZ_DTYPE_BF16 && a.d == D && a.segment == nullptr &&
           al16(a.q) && al16(a.k) && al16(a.v) && al16(a.d_o) &&
           (a.d_state_final == nullptr || (reinterpret_cast<uintptr_t>(a.d_state_final) & 7u) == 0);
}

size_t bwd_tc_ws_bytes(int64_t B, int64_t T, int H, int d) {
    if (d != D || B <= 0 || T <= 0) return 0;
    return bt_ws(B * H * ((T + C - 1) / C)).total;
}

int set_bwd_form(int form, int *prev) {
    if (form < 0 || form > 1) return set_error(RHZ_ERR_INVALID, "backward form %d (0 = tensor cores where supported, 1 = fp32 scan)", form);
    const int old = g_bwd_form.exchange(form);
    if (prev) *prev = old;
    return RHZ_OK;
}

int launch_bwd_tc(const BwdArgs &a) {
    const int nch = static_cast<int>((a.T + C - 1) / C);
    const int64_t items = a.B * a.H;
    const int64_t chunks = items * nch;
    const BtWs w = bt_ws(chunks);
    uint8_t *ws = static_cast<uint8_t *>(a.workspace);
    BtParams p;
    p.q = static_cast<const bf16 *>(a.q);
    p.k = static_cast<const bf16 *>(a.k);
    p.v = static_cast<const bf16 *>(a.v);
    p.d_o = static_cast<const bf16 *>(a.d_o);
    p.alpha = a.alpha;
    p.beta = a.beta;
    p.d_state_final = a.d_state_final;
    p.dq = static_cast<bf16 *>(a.dq);
    p.dk = static_cast<bf16 *>(a.dk);
    p.dv = static_cast<bf16 *>(a.dv);
    p.dalpha = a.dalpha;
    p.dbeta = a.dbeta;
    p.gmax = reinterpret_cast<unsigned *>(ws + w.gmax);
    p.rec = reinterpret_cast<f16 *>(ws + w.rec);
    p.g63 = reinterpret_cast<float *>(ws + w.g63);
    p.s_dump = reinterpret_cast<f16 *>(ws + w.s_dump);
    p.ds_dump = reinterpret_cast<f16 *>(ws + w.ds_dump);
    p.d_dump = reinterpret_cast<f16 *>(ws + w.d_dump);
    p.dd_dump = reinterpret_cast<f16 *>(ws + w.dd_dump);
    p.B = a.B;
    p.T = a.T;
    p.H = a.H;
    p.nch = nch;
    if (chunks == 0) return RHZ_OK;

    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(gdr_bwdtc_rec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, RK_SMEM);
        if (attr == cudaSuccess)
            attr = cudaFuncSetAttribute(gdr_bwdtc_chain_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        2 * CF_STAGE);
        if (attr == cudaSuccess)
            attr = cudaFuncSetAttribute(gdr_bwdtc_chain_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        2 * CA_STAGE);
        if (attr == cudaSuccess)
            attr = cudaFuncSetAttribute(gdr_bwdtc_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GK_SMEM);
    });
    if (attr != cudaSuccess)
        return set_error(RHZ_ERR_DEVICE, "backward kernels' smem attribute: %s", cudaGetErrorString(attr));
    cudaError_t me = cudaMemsetAsync(p.gmax, 0, sizeof(unsigned), a.stream);
    if (me != cudaSuccess) return set_error(RHZ_ERR_DEVICE, "clearing the gradient max: %s", cudaGetErrorString(me));
    const int64_t n_do = a.B * a.T * a.H * D;
    gdr_bwdtc_scale_kernel<<<296, 256, 0, a.stream>>>(p, n_do, a.d_state_final ? items * SD_ELEMS : 0);
    int st = check_launch("gdr_bwdtc_scale_kernel");
    if (st != RHZ_OK) return st;
    gdr_bwdtc_rec_kernel<<<static_cast<unsigned>(chunks), 256, RK_SMEM, a.stream>>>(p);
    st = check_launch("gdr_bwdtc_rec_kernel");
    if (st != RHZ_OK) return st;
    gdr_bwdtc_chain_kernel<false><<<static_cast<unsigned>(2 * items), 128, 2 * CF_STAGE, a.stream>>>(p);
    st = check_launch("gdr_bwdtc_chain_kernel<forward>");
    if (st != RHZ_OK) return st;
    gdr_bwdtc_chain_kernel<true><<<static_cast<unsigned>(2 * items), 128, 2 * CA_STAGE, a.stream>>>(p);
    st = check_launch("gdr_bwdtc_chain_kernel<adjoint>");
    if (st != RHZ_OK) return st;
    gdr_bwdtc_grad_kernel<<<static_cast<unsigned>(chunks), 256, GK_SMEM, a.stream>>>(p);
    return check_launch("gdr_bwdtc_grad_kernel");
}

}  // namespace rhz
