// Warp-level fp16 products on the mma.sync m16n8k16 path (fp32 accumulate)
// with operands in shared memory fetched by ldmatrix, for the chunked
// backward. Fragment layout (PTX, g = lane / 4, t = lane % 4): accumulator
// tile n holds rows g and g + 8 of a 16 x 8 block, columns 2t and 2t + 1.
#pragma once

#include <cuda_fp16.h>

#include <cstdint>

#include "sm100.cuh"

namespace rhz {
namespace mmah {

using f16 = __half;

__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
    __half2 v = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(sm100::smem_u32(p)));
}

__device__ __forceinline__ void ldsm4t(uint32_t (&r)[4], const void *p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(sm100::smem_u32(p)));
}

// A fragment (16 x 16) of A = X[m0.., k0..]: AK -- X stored [m][k] with row
// stride ld; !AK -- X stored transposed, [k][m].
template <bool AK>
__device__ __forceinline__ void frag_a(uint32_t (&a)[4], const f16 *x, int ld, int m0, int k0, int lane) {
    if (AK) {
        ldsm4(a, x + (m0 + (lane & 15)) * ld + k0 + ((lane >> 4) << 3));
    } else {
        ldsm4t(a, x + (k0 + (lane & 7) + ((lane >> 4) << 3)) * ld + m0 + (((lane >> 3) & 1) << 3));
    }
}

// B fragments of two adjacent 8-column tiles (n0 and n0 + 8) over k0 .. k0 + 15:
// r[0], r[1] for tile n0, r[2], r[3] for n0 + 8. BN -- B stored [n][k];
// !BN -- B stored [k][n].
template <bool BN>
__device__ __forceinline__ void frag_b2(uint32_t (&r)[4], const f16 *x, int ld, int k0, int n0, int lane) {
    if (BN) {
        ldsm4(r, x + (n0 + (lane & 7) + ((lane >> 4) << 3)) * ld + k0 + (((lane >> 3) & 1) << 3));
    } else {
        ldsm4t(r, x + (k0 + (lane & 7) + (((lane >> 3) & 1) << 3)) * ld + n0 + ((lane >> 4) << 3));
    }
}

// acc[NT] (16 rows from m0, NT 8-column tiles from n0) += A[m0.., ka .. ka + 16 KS]
// * B[kb .. kb + 16 KS, n0 ..].
template <int NT, int KS, bool AK, bool BN>
__device__ __forceinline__ void gemm(float (&acc)[NT][4], const f16 *A, int lda, int m0, int ka,
                                     const f16 *B, int ldb, int kb, int n0, int lane) {
    static_assert(NT % 2 == 0, "tiles in pairs");
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
        uint32_t a[4];
        frag_a<AK>(a, A, lda, m0, ka + 16 * ks, lane);
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
            uint32_t b[4];
            frag_b2<BN>(b, B, ldb, kb + 16 * ks, n0 + 16 * np, lane);
            mma(acc[2 * np], a, b[0], b[1]);
            mma(acc[2 * np + 1], a, b[2], b[3]);
        }
    }
}

// The A fragment of k-step ks from accumulator tiles 2 ks and 2 ks + 1 (the
// accumulator of one product is the A operand of the next, rounded to fp16).
template <int NA>
__device__ __forceinline__ void areg(uint32_t (&a)[4], const float (&c)[NA][4], int ks) {
    a[0] = pack_h2(c[2 * ks][0], c[2 * ks][1]);
    a[1] = pack_h2(c[2 * ks][2], c[2 * ks][3]);
    a[2] = pack_h2(c[2 * ks + 1][0], c[2 * ks + 1][1]);
    a[3] = pack_h2(c[2 * ks + 1][2], c[2 * ks + 1][3]);
}

// acc[NT] += (the warp's accumulator rows C, KS k-steps) * B[kb .., n0 ..].
template <int NT, int KS, bool BN, int NA>
__device__ __forceinline__ void gemm_areg(float (&acc)[NT][4], const float (&c)[NA][4], const f16 *B,
                                          int ldb, int kb, int n0, int lane) {
    static_assert(2 * KS <= NA, "A from accumulator tiles");
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
        uint32_t a[4];
        areg(a, c, ks);
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
            uint32_t b[4];
            frag_b2<BN>(b, B, ldb, kb + 16 * ks, n0 + 16 * np, lane);
            mma(acc[2 * np], a, b[0], b[1]);
            mma(acc[2 * np + 1], a, b[2], b[3]);
        }
    }
}

template <int NT>
__device__ __forceinline__ void zero(float (&acc)[NT][4]) {
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[n][e] = 0.f;
}

// 16-byte asynchronous copy global -> shared; src_bytes < 16 zero-fills the rest.
__device__ __forceinline__ void cp16(void *dst, const void *src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sm100::smem_u32(dst)), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}

__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace mmah
}  // namespace rhz
