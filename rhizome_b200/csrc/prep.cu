// Input producer of the Local block (SPEC.md:53-54, 61-63): the step that
// feeds the recurrence. Per token and head, for the q, k and v channels, the
// causal depthwise conv of kernel 4 (crates/ops/src/delta.rs:236-243) carried
// across each sequence from its slot's 3-sample state, then
//   q = l2norm(conv_q) * q_scale, k = l2norm(conv_k), v = conv_v
//   (crates/ops/src/elementwise.rs:125-129: x / max(|x|, 1e-12) * scale),
//   beta = sigmoid(beta_logit), alpha = exp(-softplus(a_h) softplus(alpha_logit))
//   (elementwise.rs:5-12, 36-42).
// Layouts: x*, q, k, v [tokens][H][d] (f32 or bf16); logits, alpha, beta
// [tokens][H] f32; a_head [H]; conv_w [3][H][d][4]; conv_b [3][H][d];
// conv_state [num_slots][3][H][d][3] f32 (samples oldest first).
//
// Three forms, all with conv weights in registers and a 3-sample window per
// channel sliding along consecutive tokens (restarted from the slot's carried
// samples at each sequence start), four channels per lane, norms as
// warp-shuffle sums:
//   gdr_prep_tma_kernel  bf16, d = 128, 16-byte aligned inputs: a CTA per
//                        (64 tokens, head), rows staged by TMA, each row's
//                        sequence looked up once per CTA;
//   gdr_prep_tile_kernel rows of 256 bytes otherwise (and d = 64): the same
//                        tiles staged by 16-byte loads of all threads;
//   gdr_prep_kernel      any other width: a warp per (64 tokens, head) with
//                        one token of look-ahead.
// HBM traffic is one read of x and logits (plus a 3-row halo per tile) and
// one write of q, k, v, alpha, beta. A second kernel writes each sequence's
// last three samples back to its slot once every token has read the old
// state.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "kernels.h"
#include "sm100.cuh"
#include "tmap.h"

namespace rhz {
namespace {

using namespace sm100;

constexpr int WARPS = 4;

__device__ __forceinline__ void store4(__nv_bfloat16 *p, const float (&x)[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(x[2], x[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t *>(&a);
    u.y = *reinterpret_cast<uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(p) = u;
}

__device__ __forceinline__ void store4(float *p, const float (&x)[4]) {
    *reinterpret_cast<float4 *>(p) = make_float4(x[0], x[1], x[2], x[3]);
}

// sigmoid and softplus in the reference's numerically stable forms.
__device__ __forceinline__ float sigmoid_f(float x) {
    if (x >= 0.f) return 1.f / (1.f + expf(-x));
    const float e = expf(x);
    return e / (1.f + e);
}

__device__ __forceinline__ float softplus_f(float x) { return x > 30.f ? x : log1pf(expf(x)); }

constexpr int TILE = 64;  // consecutive tokens of one head per warp

// Samples of channels c0..c0+3 at the three positions before `tok` (oldest
// first) for a sequence starting at t0: its own rows where they exist, else
// the carried state (zeros without one).
template <typename T>
__device__ __forceinline__ void load_window(const PrepArgs &p, const T *x, int a, int h, int c0,
                                            int64_t tok, int64_t t0, int64_t slot, bool have,
                                            float (&win)[3][4]) {
    const int64_t rs = static_cast<int64_t>(p.H) * p.d;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
        const int64_t t = tok - 3 + j;
        if (t >= t0) {
            load4(x + t * rs + static_cast<int64_t>(h) * p.d + c0, true, 4, win[j]);
        } else if (have) {
            const float *st = p.conv_state + (((slot * 3 + a) * p.H + h) * p.d + c0) * 3;
#pragma unroll
            for (int e = 0; e < 4; ++e) win[j][e] = st[3 * e + 3 + (t - t0)];
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) win[j][e] = 0.f;
        }
    }
}

// One warp per (tile of TILE consecutive token rows, head), four channels per
// lane and channel group: the conv weights stay in registers, a 3-sample
// window per channel slides along the tile, so every input element is read
// once (plus the 3-row halo of each tile). A sequence boundary inside the
// tile restarts the window from the next sequence's slot.
template <typename T, int NG>
__global__ void __launch_bounds__(32 * WARPS, 3) gdr_prep_kernel(const PrepArgs p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = p.H, d = p.d;
    const int64_t gw = static_cast<int64_t>(blockIdx.x) * WARPS + warp;
    const int64_t tile = gw / H;
    const int h = static_cast<int>(gw - tile * H);
    const int64_t tok0 = tile * TILE;
    if (tok0 >= p.total_tokens) return;
    const int64_t tok_end = tok0 + TILE < p.total_tokens ? tok0 + TILE : p.total_tokens;
    const int64_t rs = static_cast<int64_t>(H) * d;
    const T *xs[3] = {static_cast<const T *>(p.xq), static_cast<const T *>(p.xk),
                      static_cast<const T *>(p.xv)};
    T *ys[3] = {static_cast<T *>(p.q), static_cast<T *>(p.k), static_cast<T *>(p.v)};

    float w[3][NG][4][4], bias[3][NG][4];
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int g = 0; g < NG; ++g) {
            const int c0 = 4 * lane + 128 * g;
            if (c0 >= d) continue;
            const float *wp = p.conv_w + ((static_cast<int64_t>(a) * H + h) * d + c0) * 4;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float4 f = *reinterpret_cast<const float4 *>(wp + 4 * e);
                w[a][g][e][0] = f.x; w[a][g][e][1] = f.y; w[a][g][e][2] = f.z; w[a][g][e][3] = f.w;
            }
            const float4 bf = *reinterpret_cast<const float4 *>(p.conv_b + (static_cast<int64_t>(a) * H + h) * d + c0);
            bias[a][g][0] = bf.x; bias[a][g][1] = bf.y; bias[a][g][2] = bf.z; bias[a][g][3] = bf.w;
        }

    int64_t seq = 0, t0 = 0, t1 = 0, slot = -1;
    bool have = false, covered = true;
    auto enter = [&](int64_t tok) {  // the sequence containing `tok` (or past all of them)
        if (p.cu_seqlens) {
            int64_t lo = 0, hi = p.n_seq - 1;  // largest i with cu[i] <= tok
            while (lo < hi) {
                const int64_t mid = (lo + hi + 1) >> 1;
                if (static_cast<int64_t>(p.cu_seqlens[mid]) <= tok) lo = mid;
                else hi = mid - 1;
            }
            seq = lo;
            t0 = p.cu_seqlens[lo];
            t1 = p.cu_seqlens[lo + 1];
            t0 = t0 < 0 ? 0 : t0;  // offsets are caller data
            covered = tok >= t0 && tok < t1;
        } else {
            seq = tok / p.seq_len;
            t0 = seq * p.seq_len;
            t1 = t0 + p.seq_len;
        }
        slot = p.slots ? static_cast<int64_t>(p.slots[seq]) : seq;
        have = p.conv_state && !p.zero_init && slot >= 0 && slot < p.num_slots;
    };
    float win[3][NG][3][4];
    auto restart = [&](int64_t tok) {
        enter(tok);
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
            for (int g = 0; g < NG; ++g) {
                const int c0 = 4 * lane + 128 * g;
                if (c0 < d) load_window(p, xs[a], a, h, c0, tok, t0, slot, have, win[a][g]);
            }
    };
    restart(tok0);

    // Rows and logits of the next token are fetched while this one is
    // processed (one token of look-ahead per warp).
    float xn[3][NG][4];
    float bln = 0.f, aln = 0.f;
    auto fetch = [&](int64_t tok) {
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
            for (int g = 0; g < NG; ++g) {
                const int c0 = 4 * lane + 128 * g;
                if (c0 < d) load4(xs[a] + tok * rs + static_cast<int64_t>(h) * d + c0, true, 4, xn[a][g]);
            }
        if (lane == 0) {
            bln = p.beta_logit[tok * H + h];
            aln = p.alpha_logit[tok * H + h];
        }
    };
    fetch(tok0);
    const float sp_a = softplus_f(p.a_head[h]);

#pragma unroll 1
    for (int64_t tok = tok0; tok < tok_end; ++tok) {
        float xc[3][NG][4];
#pragma unroll
        for (int a = 0; a < 3; ++a)
#pragma unroll
            for (int g = 0; g < NG; ++g)
#pragma unroll
                for (int e = 0; e < 4; ++e) xc[a][g][e] = xn[a][g][e];
        const float blc = bln, alc = aln;
        if (tok + 1 < tok_end) fetch(tok + 1);
        if (tok >= t1 || !covered) restart(tok);  // next sequence (or still outside one)
        if (!covered) continue;                   // a row that no sequence covers
#pragma unroll
        for (int a = 0; a < 3; ++a) {
            float y[NG][4];
            float ss = 0.f;
#pragma unroll
            for (int g = 0; g < NG; ++g) {
                const int c0 = 4 * lane + 128 * g;
                if (c0 >= d) continue;
                const float *x = xc[a][g];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    // weight[0] state[0] + weight[1] state[1] + weight[2] state[2] + weight[3] x + bias
                    y[g][e] = w[a][g][e][0] * win[a][g][0][e] + w[a][g][e][1] * win[a][g][1][e] +
                              w[a][g][e][2] * win[a][g][2][e] + w[a][g][e][3] * x[e] + bias[a][g][e];
                    win[a][g][0][e] = win[a][g][1][e];
                    win[a][g][1][e] = win[a][g][2][e];
                    win[a][g][2][e] = x[e];
                    ss += y[g][e] * y[g][e];
                }
            }
            float mul = 1.f;
            if (a < 2) {
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
                mul = (a == 0 ? p.q_scale : 1.f) / fmaxf(sqrtf(ss), 1e-12f);
            }
#pragma unroll
            for (int g = 0; g < NG; ++g) {
                const int c0 = 4 * lane + 128 * g;
                if (c0 >= d) continue;
                float o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) o[e] = a < 2 ? y[g][e] * mul : y[g][e];
                store4(ys[a] + tok * rs + static_cast<int64_t>(h) * d + c0, o);
            }
        }
        if (lane == 0) {
            const int64_t i = tok * H + h;
            p.beta[i] = sigmoid_f(blc);
            p.alpha[i] = expf(-sp_a * softplus_f(alc));
        }
    }
}

// Tiled form for rows of at most 256 bytes (d = 128 in bf16): a CTA takes one
// head over TT consecutive token rows. All 256 threads first copy the tile's
// rows of xq, xk, xv plus a 3-row halo into shared memory with independent
// 16-byte loads (about 50 KB in flight per CTA), then each warp runs TT / 8
// tokens from shared memory with the conv weights in registers.
constexpr int TT = 64;
constexpr int TWARPS = 8;

template <typename T, int D>
__global__ void __launch_bounds__(32 * TWARPS, 3) gdr_prep_tile_kernel(const PrepArgs p) {
    extern __shared__ uint8_t smem_raw[];
    T *rows = reinterpret_cast<T *>(smem_raw);  // [3][TT + 3][D]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = p.H;
    constexpr int d = D;
    const int64_t tile = blockIdx.x / H;
    const int h = static_cast<int>(blockIdx.x - tile * H);
    const int64_t tok0 = tile * TT;
    const int64_t tok_end = tok0 + TT < p.total_tokens ? tok0 + TT : p.total_tokens;
    const int64_t rs = static_cast<int64_t>(H) * d;
    // q, k, v pointers by array index, as selects (no local-memory table).
    auto xsel = [&](int a) {
        return static_cast<const T *>(a == 0 ? p.xq : a == 1 ? p.xk : p.xv);
    };
    auto ysel = [&](int a) { return static_cast<T *>(a == 0 ? p.q : a == 1 ? p.k : p.v); };

    // ---- rows tok0 - 3 .. tok_end - 1 of the three arrays -> shared memory
    // (compile-time row geometry: the index splits are shifts and
    // constant-divisor multiplies)
    constexpr int CH = 16 / sizeof(T);  // elements per 16-byte chunk
    constexpr int CPR = D / CH;         // chunks per row
    constexpr int NR = TT + 3;
    for (int i = tid; i < 3 * NR * CPR; i += 32 * TWARPS) {
        const int c = i % CPR, ar = i / CPR;
        const int a = ar / NR, r = ar - a * NR;
        const int64_t tok = tok0 - 3 + r;
        if (tok < 0 || tok >= tok_end) continue;
        *reinterpret_cast<uint4 *>(rows + (a * NR + r) * D + c * CH) =
            *reinterpret_cast<const uint4 *>(xsel(a) + tok * rs + static_cast<int64_t>(h) * D + c * CH);
    }

    const int c0 = 4 * lane;
    const bool active = c0 < d;
    const float sp_a = softplus_f(p.a_head[h]);
    __syncthreads();

    // ---- tokens ta .. ta + PER - 1 of this tile, one array at a time: that
    // array's weights and a 3-sample window per channel live in registers and
    // the window slides along the tokens (restarted at a sequence start), so
    // each token reads only its own row from shared memory
    constexpr int PER = TT / TWARPS;
    const int64_t ta = tok0 + PER * warp;
    const int nt = static_cast<int>(tok_end - ta < PER ? (tok_end - ta > 0 ? tok_end - ta : 0) : PER);
    // Gate logits of the warp's tokens, one per lane, fetched up front.
    float bl = 0.f, al = 0.f;
    if (lane < nt) {
        bl = p.beta_logit[(ta + lane) * H + h];
        al = p.alpha_logit[(ta + lane) * H + h];
    }
#pragma unroll 1
    for (int a = 0; a < 3; ++a) {
        float w[4][4], bias[4];
        if (active) {
            const float *wp = p.conv_w + ((static_cast<int64_t>(a) * H + h) * d + c0) * 4;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float4 f = *reinterpret_cast<const float4 *>(wp + 4 * e);
                w[e][0] = f.x; w[e][1] = f.y; w[e][2] = f.z; w[e][3] = f.w;
            }
            const float4 bf = *reinterpret_cast<const float4 *>(p.conv_b + (static_cast<int64_t>(a) * H + h) * d + c0);
            bias[0] = bf.x; bias[1] = bf.y; bias[2] = bf.z; bias[3] = bf.w;
        }
        int64_t t0 = 0, t1 = -1, slot = -1;
        bool have = false, covered = false;
        float win[3][4];  // [sample, oldest first][channel]
        // In groups of HB tokens: pass 1, the conv outputs (the window slides
        // along them); pass 2, their L2 norms, HB shuffle trees side by side;
        // pass 3, the stores. (One token at a time, each norm's five dependent
        // shuffles sat on the path of every row.)
        constexpr int HB = 4;
#pragma unroll 1
        for (int jb = 0; jb < PER; jb += HB) {
            float y[HB][4];
            float ss[HB];
            bool ok[HB];
#pragma unroll
            for (int jj = 0; jj < HB; ++jj) {
                const int j = jb + jj;
                ok[jj] = false;
                ss[jj] = 0.f;
#pragma unroll
                for (int e = 0; e < 4; ++e) y[jj][e] = 0.f;
                if (j >= nt) continue;
                const int64_t tok = ta + j;
                if (j == 0 || tok >= t1 || !covered) {  // the sequence holding this row
                    int64_t seq;
                    if (p.cu_seqlens) {
                        int64_t lo = 0, hi = p.n_seq - 1;
                        while (lo < hi) {
                            const int64_t mid = (lo + hi + 1) >> 1;
                            if (static_cast<int64_t>(p.cu_seqlens[mid]) <= tok) lo = mid;
                            else hi = mid - 1;
                        }
                        seq = lo;
                        t0 = p.cu_seqlens[lo];
                        t1 = p.cu_seqlens[lo + 1];
                        t0 = t0 < 0 ? 0 : t0;  // offsets are caller data
                        covered = tok >= t0 && tok < t1;
                    } else {
                        seq = tok / p.seq_len;
                        t0 = seq * p.seq_len;
                        t1 = t0 + p.seq_len;
                        covered = true;
                    }
                    slot = p.slots ? static_cast<int64_t>(p.slots[seq]) : seq;
                    have = p.conv_state && !p.zero_init && slot >= 0 && slot < p.num_slots;
                    if (covered && active) {
#pragma unroll
                        for (int m = 0; m < 3; ++m) {
                            const int64_t t = tok - 3 + m;
                            if (t >= t0) {
                                load4(rows + (a * (TT + 3) + static_cast<int>(t - tok0 + 3)) * d + c0, true, 4, win[m]);
                            } else if (have) {
                                const float *st = p.conv_state + (((slot * 3 + a) * H + h) * d + c0) * 3;
#pragma unroll
                                for (int e = 0; e < 4; ++e) win[m][e] = st[3 * e + 3 + (t - t0)];
                            } else {
#pragma unroll
                                for (int e = 0; e < 4; ++e) win[m][e] = 0.f;
                            }
                        }
                    }
                }
                if (!covered) continue;  // a row that no sequence covers
                ok[jj] = true;
                if (active) {
                    float x[4];
                    load4(rows + (a * (TT + 3) + static_cast<int>(tok - tok0) + 3) * d + c0, true, 4, x);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        // weight[0] state[0] + weight[1] state[1] + weight[2] state[2] + weight[3] x + bias
                        y[jj][e] = w[e][0] * win[0][e] + w[e][1] * win[1][e] + w[e][2] * win[2][e] +
                                   w[e][3] * x[e] + bias[e];
                        win[0][e] = win[1][e];
                        win[1][e] = win[2][e];
                        win[2][e] = x[e];
                        ss[jj] += y[jj][e] * y[jj][e];
                    }
                }
            }
            if (a < 2) {
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
                    for (int jj = 0; jj < HB; ++jj) ss[jj] += __shfl_xor_sync(0xffffffffu, ss[jj], off);
                }
            }
#pragma unroll
            for (int jj = 0; jj < HB; ++jj) {
                if (!ok[jj] || !active) continue;
                const int64_t tok = ta + jb + jj;
                const float mul = a < 2 ? (a == 0 ? p.q_scale : 1.f) / fmaxf(sqrtf(ss[jj]), 1e-12f) : 1.f;
                float o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) o[e] = y[jj][e] * mul;
                store4(ysel(a) + tok * rs + static_cast<int64_t>(h) * d + c0, o);
            }
        }
    }
    // Gates of the warp's tokens, one per lane (rows that no sequence covers
    // are left alone).
    if (lane < nt) {
        const int64_t tok = ta + lane;
        bool in_seq = true;
        if (p.cu_seqlens) {
            int64_t lo = 0, hi = p.n_seq - 1;
            while (lo < hi) {
                const int64_t mid = (lo + hi + 1) >> 1;
                if (static_cast<int64_t>(p.cu_seqlens[mid]) <= tok) lo = mid;
                else hi = mid - 1;
            }
            in_seq = tok >= p.cu_seqlens[lo] && tok < p.cu_seqlens[lo + 1];
        }
        if (in_seq) {
            const int64_t i = tok * H + h;
            p.beta[i] = sigmoid_f(bl);
            p.alpha[i] = expf(-sp_a * softplus_f(al));
        }
    }
}

// TMA form for bf16 rows of d = 128 (the model's shape): one CTA per (tile
// of MT tokens, head). One thread copies the tile's rows of xq, xk and xv
// plus a 3-row halo with three TMA boxes ([MT + 3 rows][128 channels] each;
// rows above the first token or past the last read as zeros) while the
// first MT threads look up each row's sequence once: its depth (rows of the
// same sequence before it, capped at 3; DEPTH_NONE for a row no sequence
// covers) and its conv-state slot (-1: zeros). Each warp then runs its
// MPER rows of one array at a time, four channels per lane, the weights and
// a 3-sample window per channel in registers; the window slides along the
// rows and a row of depth < 3 (the first rows of a sequence) takes its
// missing samples from the slot. The norms use rsqrtf (within 2 ulp) and
// four rows' shuffle reductions run side by side.
constexpr int MT = 64;
constexpr int MROWS = MT + 3;
constexpr int MWARPS = 8;
constexpr int MPER = MT / MWARPS;
constexpr int MD = 128;
constexpr int DEPTH_NONE = 4;
constexpr uint32_t M_ARRAY_BYTES = MROWS * MD * 2;
constexpr uint32_t M_OFF_BAR = 3 * M_ARRAY_BYTES;
constexpr uint32_t M_OFF_DEPTH = M_OFF_BAR + 64;
constexpr uint32_t M_OFF_SLOT = M_OFF_DEPTH + MT * 4;
constexpr uint32_t M_SMEM = M_OFF_SLOT + MT * 4;
static_assert(M_ARRAY_BYTES % 128 == 0, "TMA destinations stay 128-byte aligned");

__device__ int g_prep_status = 0;

__device__ __forceinline__ void lds4_bf16(const __nv_bfloat16 *p, float (&x)[4]) {
    const uint2 t = *reinterpret_cast<const uint2 *>(p);
    const float2 fa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&t.x));
    const float2 fb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&t.y));
    x[0] = fa.x; x[1] = fa.y; x[2] = fb.x; x[3] = fb.y;
}

__global__ void __launch_bounds__(32 * MWARPS, 3)
    gdr_prep_tma_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const PrepArgs p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const __nv_bfloat16 *rows = reinterpret_cast<const __nv_bfloat16 *>(smem);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + M_OFF_BAR);
    int *mdepth = reinterpret_cast<int *>(smem + M_OFF_DEPTH);
    int *mslot = reinterpret_cast<int *>(smem + M_OFF_SLOT);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int H = p.H;
    const int64_t tile = blockIdx.x / H;
    const int h = static_cast<int>(blockIdx.x - tile * H);
    const int64_t tok0 = tile * MT;

    if (tid == 0) {
        mbar_init(bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0) {
        mbar_arrive_expect_tx(bar, 3 * M_ARRAY_BYTES);
        const int y0 = static_cast<int>(tok0) - 3;
        tma_load_3d(smem, &tm_q, 0, h, y0, bar);
        tma_load_3d(smem + M_ARRAY_BYTES, &tm_k, 0, h, y0, bar);
        tma_load_3d(smem + 2 * M_ARRAY_BYTES, &tm_v, 0, h, y0, bar);
    }
    // ---- each row's sequence (under the copies)
    if (tid < MT) {
        const int64_t tok = tok0 + tid;
        int depth = DEPTH_NONE, slot_out = -1;
        if (tok < p.total_tokens) {
            int64_t seq, t0, t1;
            if (p.cu_seqlens) {
                int64_t lo = 0, hi = p.n_seq - 1;  // largest i with cu[i] <= tok
                while (lo < hi) {
                    const int64_t mid = (lo + hi + 1) >> 1;
                    if (static_cast<int64_t>(p.cu_seqlens[mid]) <= tok) lo = mid;
                    else hi = mid - 1;
                }
                seq = lo;
                t0 = p.cu_seqlens[lo];
                t1 = p.cu_seqlens[lo + 1];
                t0 = t0 < 0 ? 0 : t0;  // offsets are caller data
            } else {
                seq = tok / p.seq_len;
                t0 = seq * p.seq_len;
                t1 = t0 + p.seq_len;
            }
            if (tok >= t0 && tok < t1) {
                depth = tok - t0 < 3 ? static_cast<int>(tok - t0) : 3;
                const int64_t slot = p.slots ? static_cast<int64_t>(p.slots[seq]) : seq;
                if (p.conv_state && !p.zero_init && slot >= 0 && slot < p.num_slots)
                    slot_out = static_cast<int>(slot);
            }
        }
        mdepth[tid] = depth;
        mslot[tid] = slot_out;
    }
    const int r0 = MPER * warp;  // this warp's first row, relative to tok0
    // Gate logits of the warp's rows, one per lane, fetched before the wait.
    float bl = 0.f, al = 0.f;
    const int64_t gtok = tok0 + r0 + lane;
    if (lane < MPER && gtok < p.total_tokens) {
        bl = p.beta_logit[gtok * H + h];
        al = p.alpha_logit[gtok * H + h];
    }
    const float sp_a = softplus_f(p.a_head[h]);
    __syncthreads();
    if (!mbar_wait(bar, 0)) {
        // The copies never landed: record it, and give them a last bounded
        // chance to finish before this CTA's shared memory is released.
        atomicExch(&g_prep_status, 1);
        mbar_wait(bar, 0, 200000000ull);
        return;
    }

    if (lane < MPER && mdepth[r0 + lane] != DEPTH_NONE) {
        const int64_t i = gtok * H + h;
        p.beta[i] = sigmoid_f(bl);
        p.alpha[i] = expf(-sp_a * softplus_f(al));
    }

    const int c0 = 4 * lane;
    const int64_t rs = static_cast<int64_t>(H) * MD;
#pragma unroll 1
    for (int a = 0; a < 3; ++a) {
        float w[4][4], bias[4];
        {
            const float *wp = p.conv_w + ((static_cast<int64_t>(a) * H + h) * MD + c0) * 4;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float4 f = *reinterpret_cast<const float4 *>(wp + 4 * e);
                w[e][0] = f.x; w[e][1] = f.y; w[e][2] = f.z; w[e][3] = f.w;
            }
            const float4 bf = *reinterpret_cast<const float4 *>(p.conv_b + (static_cast<int64_t>(a) * H + h) * MD + c0);
            bias[0] = bf.x; bias[1] = bf.y; bias[2] = bf.z; bias[3] = bf.w;
        }
        const __nv_bfloat16 *xr = rows + a * MROWS * MD + c0;  // smem row i = token tok0 - 3 + i
        __nv_bfloat16 *yp = static_cast<__nv_bfloat16 *>(a == 0 ? p.q : a == 1 ? p.k : p.v) +
                            (tok0 + r0) * rs + static_cast<int64_t>(h) * MD + c0;
        const float scale = a == 0 ? p.q_scale : 1.f;
        float win[3][4];  // samples of the three rows before the current one, oldest first
#pragma unroll
        for (int m = 0; m < 3; ++m) lds4_bf16(xr + (r0 + m) * MD, win[m]);
#pragma unroll
        for (int g = 0; g < MPER; g += 4) {
            float y[4][4], ss[4];
            bool live[4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int r = r0 + g + jj;
                const int depth = mdepth[r];
                live[jj] = depth != DEPTH_NONE;
                if (depth < 3) {  // the first rows of a sequence: samples before it from its slot
                    const int slot = mslot[r];
                    const float *st = slot >= 0
                        ? p.conv_state + (((static_cast<int64_t>(slot) * 3 + a) * H + h) * MD + c0) * 3
                        : nullptr;
#pragma unroll
                    for (int m = 0; m < 3; ++m) {
                        if (m < 3 - depth) {
#pragma unroll
                            for (int e = 0; e < 4; ++e) win[m][e] = st ? st[3 * e + depth + m] : 0.f;
                        }
                    }
                }
                float x[4];
                lds4_bf16(xr + (r + 3) * MD, x);
                ss[jj] = 0.f;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    // weight[0] state[0] + weight[1] state[1] + weight[2] state[2] + weight[3] x + bias
                    y[jj][e] = w[e][0] * win[0][e] + w[e][1] * win[1][e] + w[e][2] * win[2][e] +
                               w[e][3] * x[e] + bias[e];
                    win[0][e] = win[1][e];
                    win[1][e] = win[2][e];
                    win[2][e] = x[e];
                    ss[jj] += y[jj][e] * y[jj][e];
                }
            }
            if (a < 2) {
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) ss[jj] += __shfl_xor_sync(0xffffffffu, ss[jj], off);
                }
            }
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                if (!live[jj]) continue;
                // x / max(|x|, 1e-12) * scale
                const float mul = a < 2 ? scale * (ss[jj] >= 1e-24f ? rsqrtf(ss[jj]) : 1e12f) : 1.f;
                float o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) o[e] = y[jj][e] * mul;
                store4(yp + (g + jj) * rs, o);
            }
        }
    }
}

// Each sequence's last three samples (older ones from its previous state
// where it is shorter than three) back to its slot: one thread per
// (sequence, q/k/v, head, channel).
template <typename T>
__global__ void gdr_conv_state_kernel(const PrepArgs p) {
    const int64_t H = p.H, d = p.d;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= p.n_seq * 3 * H * d) return;
    const int64_t c = idx % d;
    const int64_t h = (idx / d) % H;
    const int64_t a = (idx / (d * H)) % 3;
    const int64_t seq = idx / (3 * H * d);
    const int64_t slot = p.slots ? static_cast<int64_t>(p.slots[seq]) : seq;
    if (slot < 0 || slot >= p.num_slots) return;
    int64_t t0, t1;
    if (p.cu_seqlens) {
        t0 = p.cu_seqlens[seq];
        t1 = p.cu_seqlens[seq + 1];
        t0 = t0 < 0 ? 0 : (t0 > p.total_tokens ? p.total_tokens : t0);
        t1 = t1 < t0 ? t0 : (t1 > p.total_tokens ? p.total_tokens : t1);
    } else {
        t0 = seq * p.seq_len;
        t1 = t0 + p.seq_len;
    }
    const int64_t L = t1 - t0;
    const T *x = static_cast<const T *>(a == 0 ? p.xq : a == 1 ? p.xk : p.xv);
    float *st = p.conv_state + (((slot * 3 + a) * H + h) * d + c) * 3;
    float old[3];
#pragma unroll
    for (int m = 0; m < 3; ++m) old[m] = p.zero_init ? 0.f : st[m];
    float nw[3];
#pragma unroll
    for (int m = 0; m < 3; ++m) {
        const int64_t pj = L - 3 + m;
        nw[m] = pj >= 0 ? to_f32(x[(t0 + pj) * H * d + h * d + c]) : old[L + m];
    }
#pragma unroll
    for (int m = 0; m < 3; ++m) st[m] = nw[m];
}

// The TMA form takes bf16 rows of d = 128 whose arrays start on 16-byte
// boundaries (TMA's rule) and token counts that fit its 32-bit coordinates.
bool prep_tma_fits(const PrepArgs &a) {
    auto al16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    return a.dtype == RHZ_DTYPE_BF16 && a.d == MD && a.total_tokens > 0 &&
           a.total_tokens <= static_cast<int64_t>(INT_MAX) - 2 * MT && al16(a.xq) && al16(a.xk) &&
           al16(a.xv) && a.total_tokens * a.H / MT <= static_cast<int64_t>(INT_MAX);
}

int launch_prep_tma(const PrepArgs &a) {
    CUtensorMap tm[3];
    const void *src[3] = {a.xq, a.xk, a.xv};
    const uint64_t dims[3] = {MD, static_cast<uint64_t>(a.H), static_cast<uint64_t>(a.total_tokens)};
    const uint64_t strides[2] = {MD * 2, static_cast<uint64_t>(a.H) * MD * 2};
    const uint32_t box[3] = {MD, 1, MROWS};
    for (int i = 0; i < 3; ++i) {
        const int st = encode_tmap(&tm[i], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, src[i], dims, strides, box,
                                   CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st != RHZ_OK) return st;
    }
    static std::once_flag attr_once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(attr_once, [] {
        attr_err = cudaFuncSetAttribute(gdr_prep_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(M_SMEM));
    });
    if (attr_err != cudaSuccess)
        return set_error(RHZ_ERR_DEVICE, "gdr_prep_tma_kernel smem attribute: %s", cudaGetErrorString(attr_err));
    const int64_t blocks = (a.total_tokens + MT - 1) / MT * a.H;
    gdr_prep_tma_kernel<<<static_cast<unsigned>(blocks), 32 * MWARPS, M_SMEM, a.stream>>>(tm[0], tm[1], tm[2], a);
    return check_launch("gdr_prep_tma_kernel");
}

template <typename T>
int launch_prep_t(const PrepArgs &a) {
    const size_t row_bytes = static_cast<size_t>(a.d) * sizeof(T);
    auto al16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
    // 16-byte row copies: the arrays must start on 16-byte boundaries (bf16
    // callers only guarantee 8; the warp form reads 8 bytes at a time)
    const bool tiled = ((a.d == 128 && sizeof(T) == 2) || a.d == 64) && al16(a.xq) && al16(a.xk) && al16(a.xv);
    if (prep_tma_fits(a)) {
        const int st = launch_prep_tma(a);
        if (st != RHZ_OK) return st;
    } else if (a.total_tokens > 0 && tiled) {
        const int64_t blocks = (a.total_tokens + TT - 1) / TT * a.H;
        const size_t smem = 3 * (TT + 3) * row_bytes;
        void (*kern)(const PrepArgs) = gdr_prep_tile_kernel<T, 64>;
        if constexpr (sizeof(T) == 2) {
            if (a.d == 128) kern = gdr_prep_tile_kernel<T, 128>;
        }
        static std::once_flag attr_once;
        static cudaError_t attr_err = cudaSuccess;
        std::call_once(attr_once, [] {
            attr_err = cudaFuncSetAttribute(gdr_prep_tile_kernel<T, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(3 * (TT + 3) * 256));
            if constexpr (sizeof(T) == 2) {
                if (attr_err == cudaSuccess)
                    attr_err = cudaFuncSetAttribute(gdr_prep_tile_kernel<T, 128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                    static_cast<int>(3 * (TT + 3) * 256));
            }
        });
        if (attr_err != cudaSuccess)
            return set_error(RHZ_ERR_DEVICE, "gdr_prep_tile_kernel smem attribute: %s", cudaGetErrorString(attr_err));
        kern<<<static_cast<unsigned>(blocks), 32 * TWARPS, smem, a.stream>>>(a);
        const int st = check_launch("gdr_prep_tile_kernel");
        if (st != RHZ_OK) return st;
    } else if (a.total_tokens > 0) {
        const int64_t warps = (a.total_tokens + TILE - 1) / TILE * a.H;
        const int64_t blocks = (warps + WARPS - 1) / WARPS;
        const unsigned grid = static_cast<unsigned>(blocks);
        if (a.d <= 128) gdr_prep_kernel<T, 1><<<grid, 32 * WARPS, 0, a.stream>>>(a);
        else if (a.d <= 256) gdr_prep_kernel<T, 2><<<grid, 32 * WARPS, 0, a.stream>>>(a);
        else gdr_prep_kernel<T, 4><<<grid, 32 * WARPS, 0, a.stream>>>(a);
        const int st = check_launch("gdr_prep_kernel");
        if (st != RHZ_OK) return st;
    }
    if (a.conv_state && a.write_state && a.n_seq > 0) {
        const int64_t n = a.n_seq * 3 * a.H * a.d;
        gdr_conv_state_kernel<T><<<static_cast<unsigned>((n + 255) / 256), 256, 0, a.stream>>>(a);
        return check_launch("gdr_conv_state_kernel");
    }
    return RHZ_OK;
}

}  // namespace

int prep_status(int *flag, bool clear) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_prep_status, sizeof(int));
    if (e == cudaSuccess && clear && v) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_prep_status, &zero, sizeof(int));
    }
    if (e != cudaSuccess)
        return set_error(RHZ_ERR_DEVICE, "reading the input producer's status: %s", cudaGetErrorString(e));
    *flag = v;
    return RHZ_OK;
}

int launch_prep(const PrepArgs &a) {
    return a.dtype == RHZ_DTYPE_BF16 ? launch_prep_t<__nv_bfloat16>(a) : launch_prep_t<float>(a);
}

}  // namespace rhz
