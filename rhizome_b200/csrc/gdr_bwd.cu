// Backward of the gated delta-rule scan (the adjoint the reference names as
// "reverse scan of the rank-1 update", docs/kernels.md:16; it has no code,
// so the rules follow from gated_delta_step, crates/ops/src/delta.rs:93-127).
// With P = S_{t-1} after any reset, M = alpha (I - beta k k^T) and
// S_t = P M + beta v k^T, o_t = S_t q_t, the adjoint G of S_t runs backwards:
//   G += dO_t q_t^T;  dq_t = S_t^T dO_t;  g = G k_t;  p = P k_t
//   dv_t = beta g;  dbeta_t = v.g - alpha p.g;  dalpha_t = <P, G> - beta p.g
//   dk_t = beta G^T v - alpha beta (P^T g + G^T p)
//   G <- alpha (G - beta g k^T), and G <- 0 at a reset (t = 0, segment change).
// fp32 throughout (inputs f32 or bf16), d <= 128 with d % 4 == 0.
//
// This fp32 reverse scan serves f32 inputs, segments and other widths; bf16
// inputs of d = 128 take the chunked tensor-core form (gdr_bwd_tc.cu).
//
// Rows of S and G evolve independently, so one CTA (4 warps, 4 rows each)
// owns 16 rows of one (sequence, head); a lane holds 4 consecutive columns.
// Pass 1 runs the recurrence forward and stores the CTA's rows of the state
// every CK positions. Pass 2 walks the chunks backwards: it recomputes the
// chunk's pre-states into shared memory, then applies the adjoint steps.
// dv is row-local and written directly; the column sums (dq, dk) and the
// three scalars of dalpha / dbeta are per-row-block partials that a second
// kernel adds up in a fixed order (deterministic, no atomics).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace rhz {
namespace {

constexpr int R = 16;   // state rows per CTA
constexpr int NW = 4;   // warps per CTA, 4 rows each
constexpr int CK = 8;   // positions per checkpoint
constexpr int PW = 3;   // scalar partials per position: <P,G>, p.g, v.g

struct BwdParams {
    void *dq, *dk, *dv;
    float *dalpha, *dbeta;
    const void *q, *k, *v, *d_o;
    const float *alpha, *beta;
    const int64_t *segment;
    const float *d_state_final;
    float *ckpt;  // [B*H*nrb][nck][R][d]
    float *part;  // [B*H*nrb][T][2d + PW]
    int64_t B, T;
    int H, d, nrb;
};

template <typename T>
__device__ __forceinline__ void ld4(const T *p, float (&x)[4]) {
    load4(p, true, 4, x);
}

// Dot products of four rows with one vector, reduced over the 32 lanes of the
// warp; every lane gets all four results.
__device__ __forceinline__ void dot4(const float (&a)[4][4], const float (&x)[4], float (&out)[4]) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        float s = a[r][0] * x[0] + a[r][1] * x[1] + a[r][2] * x[2] + a[r][3] * x[3];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
        out[r] = s;
    }
}

__device__ __forceinline__ bool reset_at(const BwdParams &p, int64_t b, int64_t t) {
    if (t == 0) return true;
    return p.segment && p.segment[b * p.T + t] != p.segment[b * p.T + t - 1];
}

template <typename T>
__global__ void __launch_bounds__(32 * NW) gdr_bwd_kernel(const BwdParams p) {
    extern __shared__ float smem_f[];
    float (*pbuf)[R][128] = reinterpret_cast<float (*)[R][128]>(smem_f);           // [CK][R][128]
    float (*red)[2 * 128 + PW] = reinterpret_cast<float (*)[2 * 128 + PW]>(smem_f + CK * R * 128);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = p.d, H = p.H;
    const int64_t blk = blockIdx.x;                  // (b, h, rb)
    const int rb = static_cast<int>(blk % p.nrb);
    const int64_t bh = blk / p.nrb;
    const int h = static_cast<int>(bh % H);
    const int64_t b = bh / H;
    const int row0 = rb * R + 4 * warp;  // first of this warp's 4 rows
    const int c0 = 4 * lane;
    const bool act = c0 < d;
    const int64_t ts = static_cast<int64_t>(H) * d;  // token stride
    const T *q = static_cast<const T *>(p.q), *k = static_cast<const T *>(p.k);
    const T *v = static_cast<const T *>(p.v), *dO = static_cast<const T *>(p.d_o);
    const int nck = static_cast<int>((p.T + CK - 1) / CK);
    float *ck = p.ckpt + blk * static_cast<int64_t>(nck) * R * d;
    float *part = p.part + blk * p.T * (2 * d + PW);

    auto row_ok = [&](int r) { return row0 + r < d; };
    auto tok = [&](int64_t t) { return (b * p.T + t) * ts + static_cast<int64_t>(h) * d; };
    float S[4][4];
    // One forward step on this warp's rows (rows outside d stay zero).
    auto step = [&](int64_t t) {
        float kv[4] = {0.f, 0.f, 0.f, 0.f};
        if (act) ld4(k + tok(t) + c0, kv);
        float sk[4];
        dot4(S, kv, sk);
        const float a = p.alpha[(b * p.T + t) * H + h], be = p.beta[(b * p.T + t) * H + h];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const float vi = row_ok(r) ? to_f32(v[tok(t) + row0 + r]) : 0.f;
#pragma unroll
            for (int e = 0; e < 4; ++e) S[r][e] = a * (S[r][e] - be * sk[r] * kv[e]) + be * vi * kv[e];
        }
    };
    auto zero_state = [&]() {
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int e = 0; e < 4; ++e) S[r][e] = 0.f;
    };
    auto save = [&](float *dst) {  // this warp's rows -> [R][d] buffer
        if (!act) return;
#pragma unroll
        for (int r = 0; r < 4; ++r)
            *reinterpret_cast<float4 *>(dst + (4 * warp + r) * d + c0) = make_float4(S[r][0], S[r][1], S[r][2], S[r][3]);
    };
    auto load = [&](const float *src) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            float4 f = act ? *reinterpret_cast<const float4 *>(src + (4 * warp + r) * d + c0) : make_float4(0.f, 0.f, 0.f, 0.f);
            S[r][0] = f.x; S[r][1] = f.y; S[r][2] = f.z; S[r][3] = f.w;
        }
    };

    // ---- pass 1: forward, pre-state of every CK-th position (after reset)
    zero_state();
#pragma unroll 1
    for (int64_t t = 0; t < p.T; ++t) {
        if (reset_at(p, b, t)) zero_state();
        if (t % CK == 0) save(ck + (t / CK) * R * d);
        step(t);
    }

    // ---- pass 2: adjoint, chunk by chunk from the end
    float G[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        float4 f = make_float4(0.f, 0.f, 0.f, 0.f);
        if (p.d_state_final && act && row_ok(r))
            f = *reinterpret_cast<const float4 *>(p.d_state_final + (bh * d + row0 + r) * d + c0);
        G[r][0] = f.x; G[r][1] = f.y; G[r][2] = f.z; G[r][3] = f.w;
    }
#pragma unroll 1
    for (int c = nck - 1; c >= 0; --c) {
        const int64_t t0 = static_cast<int64_t>(c) * CK;
        const int n = static_cast<int>(p.T - t0 < CK ? p.T - t0 : CK);
        // pre-states of the chunk
        load(ck + c * R * d);
#pragma unroll 1
        for (int j = 0; j < n; ++j) {
            if (reset_at(p, b, t0 + j)) zero_state();
            if (act) {
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int e = 0; e < 4; ++e) pbuf[j][4 * warp + r][c0 + e] = S[r][e];
            }
            step(t0 + j);
        }
        __syncwarp();
#pragma unroll 1
        for (int j = n - 1; j >= 0; --j) {
            const int64_t t = t0 + j;
            float P[4][4];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int e = 0; e < 4; ++e) P[r][e] = act ? pbuf[j][4 * warp + r][c0 + e] : 0.f;
            float kv[4] = {0.f, 0.f, 0.f, 0.f}, qv[4] = {0.f, 0.f, 0.f, 0.f};
            if (act) {
                ld4(k + tok(t) + c0, kv);
                ld4(q + tok(t) + c0, qv);
            }
            const float a = p.alpha[(b * p.T + t) * H + h], be = p.beta[(b * p.T + t) * H + h];
            float vi[4], di[4];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                vi[r] = row_ok(r) ? to_f32(v[tok(t) + row0 + r]) : 0.f;
                di[r] = row_ok(r) ? to_f32(dO[tok(t) + row0 + r]) : 0.f;
            }
            float pk[4];
            dot4(P, kv, pk);
            // S_t (this warp's rows), G += dO q^T
            float dqp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float st = a * (P[r][e] - be * pk[r] * kv[e]) + be * vi[r] * kv[e];
                    dqp[e] += st * di[r];
                    G[r][e] += di[r] * qv[e];
                }
            float g[4];
            dot4(G, kv, g);
            float pg = 0.f, vg = 0.f, pG = 0.f;
            float dkp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                pg += pk[r] * g[r];
                vg += vi[r] * g[r];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    pG += P[r][e] * G[r][e];
                    dkp[e] += be * G[r][e] * vi[r] - a * be * (P[r][e] * g[r] + G[r][e] * pk[r]);
                }
            }
            // dv (row-local)
            T *dv = static_cast<T *>(p.dv);
            const float gl = lane == 0 ? g[0] : lane == 1 ? g[1] : lane == 2 ? g[2] : g[3];
            if (lane < 4 && row_ok(lane)) dv[tok(t) + row0 + lane] = from_f32<T>(be * gl);
            // <P, G> summed over the lanes (pg and vg are already warp totals)
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) pG += __shfl_xor_sync(0xffffffffu, pG, off);
            // per-warp partials -> shared memory, then the CTA's partial row
            if (act) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    red[warp][c0 + e] = dqp[e];
                    red[warp][d + c0 + e] = dkp[e];
                }
            }
            if (lane == 0) {
                red[warp][2 * d + 0] = pG;
                red[warp][2 * d + 1] = pg;
                red[warp][2 * d + 2] = vg;
            }
            __syncthreads();
            for (int i = threadIdx.x; i < 2 * d + PW; i += 32 * NW)
                part[t * (2 * d + PW) + i] = red[0][i] + red[1][i] + red[2][i] + red[3][i];
            __syncthreads();
            // G <- alpha (G - beta g k^T); zero at a reset
            const bool rs = reset_at(p, b, t);
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int e = 0; e < 4; ++e) G[r][e] = rs ? 0.f : a * (G[r][e] - be * g[r] * kv[e]);
        }
        __syncwarp();
    }
}

// dq, dk, dalpha, dbeta from the row-block partials, summed in block order.
template <typename T>
__global__ void gdr_bwd_reduce_kernel(const BwdParams p) {
    const int d = p.d, H = p.H;
    const int64_t row = blockIdx.x;  // (b, h, t)
    const int64_t t = row % p.T;
    const int64_t bh = row / p.T;
    const int h = static_cast<int>(bh % H);
    const int64_t b = bh / H;
    const int64_t w = 2 * d + PW;
    const float *base = p.part + (bh * p.nrb) * p.T * w + t * w;
    const int64_t o = (b * p.T + t) * static_cast<int64_t>(H) * d + static_cast<int64_t>(h) * d;
    for (int i = threadIdx.x; i < 2 * d; i += blockDim.x) {
        float s = 0.f;
        for (int r = 0; r < p.nrb; ++r) s += base[static_cast<int64_t>(r) * p.T * w + i];
        T *dst = static_cast<T *>(i < d ? p.dq : p.dk);
        dst[o + (i < d ? i : i - d)] = from_f32<T>(s);
    }
    if (threadIdx.x == 0) {
        float pG = 0.f, pg = 0.f, vg = 0.f;
        for (int r = 0; r < p.nrb; ++r) {
            const float *x = base + static_cast<int64_t>(r) * p.T * w + 2 * d;
            pG += x[0];
            pg += x[1];
            vg += x[2];
        }
        const int64_t i = (b * p.T + t) * H + h;
        p.dalpha[i] = pG - p.beta[i] * pg;
        p.dbeta[i] = vg - p.alpha[i] * pg;
    }
}

}  // namespace

// The larger of the two forms' needs: the query does not know the dtype.
size_t bwd_ws_bytes(int64_t B, int64_t T, int H, int d) {
    const int64_t nrb = (d + R - 1) / R;
    const int64_t nck = (T + CK - 1) / CK;
    const int64_t blocks = B * H * nrb;
    const int64_t ck = blocks * nck * R * d * 4;
    const int64_t pt = blocks * T * (2 * d + PW) * 4;
    const size_t scan = static_cast<size_t>(((ck + 255) / 256) * 256 + pt);
    const size_t tc = bwd_tc_ws_bytes(B, T, H, d);
    return scan > tc ? scan : tc;
}

int launch_bwd(const BwdArgs &a) {
    if (a.B > 0 && a.T > 0 && bwd_tc_supports(a)) return launch_bwd_tc(a);
    BwdParams p;
    p.dq = a.dq; p.dk = a.dk; p.dv = a.dv; p.dalpha = a.dalpha; p.dbeta = a.dbeta;
    p.q = a.q; p.k = a.k; p.v = a.v; p.d_o = a.d_o;
    p.alpha = a.alpha; p.beta = a.beta; p.segment = a.segment; p.d_state_final = a.d_state_final;
    p.B = a.B; p.T = a.T; p.H = a.H; p.d = a.d;
    p.nrb = (a.d + R - 1) / R;
    const int64_t nck = (a.T + CK - 1) / CK;
    const int64_t blocks = a.B * a.H * p.nrb;
    const int64_t ck = blocks * nck * R * a.d * 4;
    p.ckpt = static_cast<float *>(a.workspace);
    p.part = reinterpret_cast<float *>(static_cast<char *>(a.workspace) + ((ck + 255) / 256) * 256);
    if (blocks == 0 || a.T == 0) return RHZ_OK;
    constexpr int smem = (CK * R * 128 + NW * (2 * 128 + PW)) * 4;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {
        attr = cudaFuncSetAttribute(gdr_bwd_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (attr == cudaSuccess)
            attr = cudaFuncSetAttribute(gdr_bwd_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    });
    if (attr != cudaSuccess) return set_error(RHZ_ERR_DEVICE, "gdr_bwd_kernel smem attribute: %s", cudaGetErrorString(attr));
    if (a.dtype == RHZ_DTYPE_BF16) {
        gdr_bwd_kernel<__nv_bfloat16><<<static_cast<unsigned>(blocks), 32 * NW, smem, a.stream>>>(p);
        int st = check_launch("gdr_bwd_kernel");
        if (st != RHZ_OK) return st;
        gdr_bwd_reduce_kernel<__nv_bfloat16><<<static_cast<unsigned>(a.B * a.H * a.T), 128, 0, a.stream>>>(p);
    } else {
        gdr_bwd_kernel<float><<<static_cast<unsigned>(blocks), 32 * NW, smem, a.stream>>>(p);
        int st = check_launch("gdr_bwd_kernel");
        if (st != RHZ_OK) return st;
        gdr_bwd_reduce_kernel<float><<<static_cast<unsigned>(a.B * a.H * a.T), 128, 0, a.stream>>>(p);
    }
    return check_launch("gdr_bwd_reduce_kernel");
}

}  // namespace rhz
