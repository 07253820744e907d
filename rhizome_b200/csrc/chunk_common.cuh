// Device helpers shared by the tensor-core chunked kernels (the pair form
// gdr_chunk_tc.cu, the one-CTA form gdr_chunk_solo.cu and the grid form
// gdr_chunk_grid.cu): fp16/bf16 packing into 128-byte-swizzled operand
// blocks, the mma.sync fragments of the 64 x 64 triangular solve
// T = (I + A)^-1, and the per-chunk gate tables.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>

#include "sm100.cuh"

namespace rhz {
namespace chunk {
using namespace sm100;

constexpr int CH = 64;    // chunk length
constexpr int HD = 128;   // head dim (d_k = d_v)
constexpr int AST = 68;   // fp32 row stride of the A / T tables (16-byte rows, bank spread)

// Gate table layout (floats): gl[64] z[64] (int) beta[64] gamma[64] P[C-1][.][64] beta*gamma[64].
constexpr int G_GL = 0, G_Z = 64, G_BE = 128, G_GM = 192, G_PL = 256, G_BG = 320, G_SIZE = 384;
constexpr uint32_t G_BYTES = G_SIZE * 4;

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float lg2(float x) {
    float y;
    asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
}

// 8 consecutive values as one 16-byte fp16 chunk.
__device__ __forceinline__ uint4 pack8_f16(const float *v) {
    uint4 w;
    w.x = pack_f16x2(v[0], v[1]);
    w.y = pack_f16x2(v[2], v[3]);
    w.z = pack_f16x2(v[4], v[5]);
    w.w = pack_f16x2(v[6], v[7]);
    return w;
}

// 32 values as fp16 into 16-byte chunks c0 .. c0+3 of row `row` of a
// 128-byte-swizzled block of 128-byte rows (canonical SWIZZLE_128B layout).
__device__ __forceinline__ void st_row32_f16(uint8_t *blk, uint32_t row, uint32_t c0,
                                             const float *v) {
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4 *>(blk + sw128_offset(row, c0 + c)) = pack8_f16(v + 8 * c);
}

// 16 values as fp16 into 16-byte chunks c0, c0+1 of row `row` of a
// 128-byte-swizzled block of 128-byte rows (canonical SWIZZLE_128B layout).
__device__ __forceinline__ void st_row16_f16(uint8_t *blk, uint32_t row, uint32_t c0, const float *v) {
    *reinterpret_cast<uint4 *>(blk + sw128_offset(row, c0)) = pack8_f16(v);
    *reinterpret_cast<uint4 *>(blk + sw128_offset(row, c0 + 1)) = pack8_f16(v + 8);
}

// 16 values as a bf16 pair hi = bf16(v), lo = bf16(v - hi) into chunks c0,
// c0+1 of row `row` of two blocks of the st_row16_f16 layout (hi + lo
// carries ~16 mantissa bits).
__device__ __forceinline__ void st_row16_bf16_split(uint8_t *hi_blk, uint8_t *lo_blk, uint32_t row,
                                                    uint32_t c0, const float *v) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float a = v[8 * c + 2 * e], b = v[8 * c + 2 * e + 1];
            const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
            const __nv_bfloat162 l = __floats2bfloat162_rn(a - __low2float(h), b - __high2float(h));
            hi[e] = *reinterpret_cast<const uint32_t *>(&h);
            lo[e] = *reinterpret_cast<const uint32_t *>(&l);
        }
        *reinterpret_cast<uint4 *>(hi_blk + sw128_offset(row, c0 + c)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4 *>(lo_blk + sw128_offset(row, c0 + c)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

__device__ __forceinline__ void st_zero32(uint8_t *blk, uint32_t row, uint32_t c0) {
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4 *>(blk + sw128_offset(row, c0 + c)) = make_uint4(0, 0, 0, 0);
}

__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t x, float s) {
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162 *>(&x);
    return pack_f16x2(__low2float(b) * s, __high2float(b) * s);
}

__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t x) {
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162 *>(&x);
    return pack_f16x2(__low2float(b), __high2float(b));
}

__device__ __forceinline__ uint32_t h2(float a, float b) { return pack_f16x2(a, b); }

// D (16 x 8, fp32) += A (16 x 16, fp16) * B (16 x 8, fp16) on the warp's
// legacy tensor-core path (mma.sync m16n8k16); fragments per the PTX layout
// with g = lane / 4, t = lane % 4.
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// A fragment of the 16 x 16 fp32 tile at L (row stride ls), rounded to fp16.
__device__ __forceinline__ void frag_a(const float *L, int ls, int lane, uint32_t (&a)[4]) {
    const int g = lane >> 2, t = lane & 3;
    const float2 x0 = *reinterpret_cast<const float2 *>(L + g * ls + 2 * t);
    const float2 x1 = *reinterpret_cast<const float2 *>(L + (g + 8) * ls + 2 * t);
    const float2 x2 = *reinterpret_cast<const float2 *>(L + g * ls + 2 * t + 8);
    const float2 x3 = *reinterpret_cast<const float2 *>(L + (g + 8) * ls + 2 * t + 8);
    a[0] = h2(x0.x, x0.y);
    a[1] = h2(x1.x, x1.y);
    a[2] = h2(x2.x, x2.y);
    a[3] = h2(x3.x, x3.y);
}

// B fragment of the 16 x 8 fp32 tile at R (row-major [k][n], row stride rs).
__device__ __forceinline__ void frag_b(const float *R, int rs, int lane, uint32_t (&b)[2]) {
    const int g = lane >> 2, t = lane & 3;
    b[0] = h2(R[(2 * t) * rs + g], R[(2 * t + 1) * rs + g]);
    b[1] = h2(R[(2 * t + 8) * rs + g], R[(2 * t + 9) * rs + g]);
}

// Store the 16 x 8 accumulator (times `sign`) into fp32 rows at C (stride cs).
__device__ __forceinline__ void st_frag_c(float *C, int cs, int lane, const float (&d)[4], float sign) {
    const int g = lane >> 2, t = lane & 3;
    *reinterpret_cast<float2 *>(C + g * cs + 2 * t) = make_float2(sign * d[0], sign * d[1]);
    *reinterpret_cast<float2 *>(C + (g + 8) * cs + 2 * t) = make_float2(sign * d[2], sign * d[3]);
}

// Transpose of one 8 x 8 fp16 block held in the mma fragment layout.
__device__ __forceinline__ uint32_t movtrans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

// A fragment (fp16) of a 16 x 16 matrix from its two 16 x 8 accumulator halves.
__device__ __forceinline__ void c_to_a(const float (&c0)[4], const float (&c1)[4], uint32_t (&a)[4]) {
    a[0] = h2(c0[0], c0[1]);
    a[1] = h2(c0[2], c0[3]);
    a[2] = h2(c1[0], c1[1]);
    a[3] = h2(c1[2], c1[3]);
}

// B fragments (both 16 x 8 column halves) of the matrix whose A fragment is
// `a`: the B layout of X is the A layout of X^T, block by block.
__device__ __forceinline__ void a_to_b(const uint32_t (&a)[4], uint32_t (&b0)[2], uint32_t (&b1)[2]) {
    b0[0] = movtrans(a[0]);
    b0[1] = movtrans(a[1]);
    b1[0] = movtrans(a[2]);
    b1[1] = movtrans(a[3]);
}

// Inverse of the unit-lower-triangular 16 x 16 block I + N (N strictly lower,
// fp32 in A at row stride AST) written to T (same stride), by one warp:
// (I + N)^-1 = (I - N)(I + N^2)(I + N^4)(I + N^8), exact for nilpotent N of
// order 16, as 12 mma.sync products with fp16 operands and fp32 accumulation.
__device__ __forceinline__ void diag_inverse16(const float *A, float *T, int lane) {
    const int g = lane >> 2, t = lane & 3;
    float n0[4], n1[4];
    {
        const float2 a0 = *reinterpret_cast<const float2 *>(A + g * AST + 2 * t);
        const float2 a1 = *reinterpret_cast<const float2 *>(A + (g + 8) * AST + 2 * t);
        const float2 a2 = *reinterpret_cast<const float2 *>(A + g * AST + 8 + 2 * t);
        const float2 a3 = *reinterpret_cast<const float2 *>(A + (g + 8) * AST + 8 + 2 * t);
        n0[0] = a0.x; n0[1] = a0.y; n0[2] = a1.x; n0[3] = a1.y;
        n1[0] = a2.x; n1[1] = a2.y; n1[2] = a3.x; n1[3] = a3.y;
    }
    // X = I - N in the accumulator layout (row g / g + 8, columns 8h + 2t, +1).
    float x0[4], x1[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const int r = g + 8 * (e >> 1), c = 2 * t + (e & 1);
        x0[e] = (r == c ? 1.f : 0.f) - n0[e];
        x1[e] = (r == c + 8 ? 1.f : 0.f) - n1[e];
    }
    uint32_t aP[4], bP0[2], bP1[2], aX[4];
    c_to_a(n0, n1, aP);
    a_to_b(aP, bP0, bP1);
#pragma unroll
    for (int lvl = 0; lvl < 3; ++lvl) {
        // P <- P^2 (N^2, N^4, N^8), then X <- X + X P.
        float p0[4] = {0.f, 0.f, 0.f, 0.f}, p1[4] = {0.f, 0.f, 0.f, 0.f};
        mma16816(p0, aP, bP0);
        mma16816(p1, aP, bP1);
        c_to_a(p0, p1, aP);
        a_to_b(aP, bP0, bP1);
        c_to_a(x0, x1, aX);
        mma16816(x0, aX, bP0);
        mma16816(x1, aX, bP1);
    }
    st_frag_c(T, AST, lane, x0, 1.f);
    st_frag_c(T + 8, AST, lane, x1, 1.f);
}

// Off-diagonal part of T = (I + A)^-1 once the four diagonal 16 x 16 inverses
// D_I are in Tf (and Tf's tiles (0,1) and (2,3) are zero), by a 2 x 2
// recursion: T_{2p+1,2p} = -D_{2p+1} (A_{2p+1,2p} D_{2p}) for p = 0, 1, then
// T[32:64, 0:32] = -T[32:64, 32:64] (A[32:64, 0:32] T[0:32, 0:32]). The
// products run on mma.sync with fp16 operands (T is rounded to fp16 for the
// tcgen05 products anyway), on the eight warps of one producer context
// (named barrier `bar`). Ends synchronised.
__device__ inline void solve_offdiag(const float *Af, float *Tf, float *Xf, int warp, int lane, int bar) {
    if (warp < 4) {
        const int pb = warp >> 1, nt = warp & 1;
        const int r0 = 32 * pb + 16, c0 = 32 * pb;  // tile (2p+1, 2p)
        uint32_t a[4], b[2];
        float x[4] = {0.f, 0.f, 0.f, 0.f};
        frag_a(Af + r0 * AST + c0, AST, lane, a);
        frag_b(Tf + c0 * AST + c0 + 8 * nt, AST, lane, b);
        mma16816(x, a, b);
        float *X = Xf + pb * 256 + 8 * nt;  // [16][16]
        st_frag_c(X, 16, lane, x, 1.f);
        __syncwarp();
        float y[4] = {0.f, 0.f, 0.f, 0.f};
        frag_a(Tf + r0 * AST + r0, AST, lane, a);
        frag_b(X, 16, lane, b);
        mma16816(y, a, b);
        st_frag_c(Tf + r0 * AST + c0 + 8 * nt, AST, lane, y, -1.f);
    }
    nbar_sync(bar, 256);
    const int mt = warp >> 2, nt = warp & 3;
    {
        float y[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
            uint32_t a[4], b[2];
            frag_a(Af + (32 + 16 * mt) * AST + 16 * ks, AST, lane, a);
            frag_b(Tf + (16 * ks) * AST + 8 * nt, AST, lane, b);
            mma16816(y, a, b);
        }
        st_frag_c(Xf + (16 * mt) * 32 + 8 * nt, 32, lane, y, 1.f);  // Y [32][32]
    }
    nbar_sync(bar, 256);
    {
        float y[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 2; ++ks) {
            uint32_t a[4], b[2];
            frag_a(Tf + (32 + 16 * mt) * AST + 32 + 16 * ks, AST, lane, a);
            frag_b(Xf + (16 * ks) * 32 + 8 * nt, 32, lane, b);
            mma16816(y, a, b);
        }
        st_frag_c(Tf + (32 + 16 * mt) * AST + 8 * nt, AST, lane, y, -1.f);
    }
    nbar_sync(bar, 256);
}

// Gate inputs of one chunk for one warp (two positions per lane), loaded a
// chunk ahead of their use so the global latency stays off the critical
// path. Padded positions get alpha = 1, beta = 0 so they write nothing.
struct GateIn {
    float a0, a1, b0, b1;
};

// Gate tables of one chunk (one warp): prefix sums of log2 alpha over nonzero
// alphas and of zero-alpha counts, then gamma_t, P[C-1][s], beta, beta*gamma.
__device__ __forceinline__ void gate_tables(float *g, const GateIn &in, int lane) {
    int *zz = reinterpret_cast<int *>(g + G_Z);
    const int p0 = 2 * lane, p1 = p0 + 1;
    const float a0 = in.a0, a1 = in.a1, b0 = in.b0, b1 = in.b1;
    const bool nz0 = a0 >= 1.17549435e-38f, nz1 = a1 >= 1.17549435e-38f;
    const float l0 = nz0 ? lg2(a0) : 0.f, l1 = nz1 ? lg2(a1) : 0.f;
    const int z0 = nz0 ? 0 : 1, z1 = nz1 ? 0 : 1;
    float ls = l0 + l1;
    int zs = z0 + z1;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const float lo = __shfl_up_sync(0xffffffffu, ls, off);
        const int zo = __shfl_up_sync(0xffffffffu, zs, off);
        if (lane >= off) { ls += lo; zs += zo; }
    }
    const float g1 = ls, g0 = ls - l1;  // inclusive prefix at p1, p0
    const int y1 = zs, y0 = zs - z1;
    const float g63 = __shfl_sync(0xffffffffu, g1, 31);
    const int y63 = __shfl_sync(0xffffffffu, y1, 31);
    g[G_GL + p0] = g0; g[G_GL + p1] = g1;
    zz[p0] = y0; zz[p1] = y1;
    g[G_BE + p0] = b0; g[G_BE + p1] = b1;
    const float gm0 = y0 == 0 ? ex2(g0) : 0.f, gm1 = y1 == 0 ? ex2(g1) : 0.f;
    g[G_GM + p0] = gm0; g[G_GM + p1] = gm1;
    g[G_BG + p0] = b0 * gm0; g[G_BG + p1] = b1 * gm1;
    g[G_PL + p0] = y0 == y63 ? ex2(g63 - g0) : 0.f;
    g[G_PL + p1] = y1 == y63 ? ex2(g63 - g1) : 0.f;
}

}  // namespace chunk
}  // namespace rhz
