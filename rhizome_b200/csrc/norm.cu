// Per-head output norm, groupnorm_heads (crates/ops/src/norm.rs:48-60): every
// (row, head) slice of d values is RMS-normalised on its own,
//   out = x / sqrt(mean(x^2) + eps) * scale[0..d)   (norm.rs:8-13),
// with the same first d entries of `scale` for every head, as the reference
// slices scale[..dh]. One warp per (row, head), four channels per lane and
// channel group, 8/16-byte vector accesses, a shuffle sum; in place allowed.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace rhz {
namespace {

constexpr int WARPS = 8;

__device__ __forceinline__ void put4(__nv_bfloat16 *p, const float (&x)[4]) {
    __nv_bfloat162 a = __floats2bfloat162_rn(x[0], x[1]);
    __nv_bfloat162 b = __floats2bfloat162_rn(x[2], x[3]);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t *>(&a);
    u.y = *reinterpret_cast<uint32_t *>(&b);
    *reinterpret_cast<uint2 *>(p) = u;
}

__device__ __forceinline__ void put4(float *p, const float (&x)[4]) {
    *reinterpret_cast<float4 *>(p) = make_float4(x[0], x[1], x[2], x[3]);
}

template <typename T>
__global__ void __launch_bounds__(32 * WARPS) groupnorm_heads_kernel(T *out, const T *x,
                                                                     const float *scale, int64_t n,
                                                                     int d, float eps) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t slice = static_cast<int64_t>(blockIdx.x) * WARPS + warp;  // (row, head)
    if (slice >= n) return;
    const T *src = x + slice * d;
    T *dst = out + slice * d;
    float v[4][4];
    float ss = 0.f;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const int c0 = 4 * lane + 128 * g;
        if (c0 >= d) continue;
        load4(src + c0, true, 4, v[g]);
#pragma unroll
        for (int e = 0; e < 4; ++e) ss += v[g][e] * v[g][e];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = 1.f / sqrtf(ss / static_cast<float>(d) + eps);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const int c0 = 4 * lane + 128 * g;
        if (c0 >= d) continue;
        const float4 s4 = *reinterpret_cast<const float4 *>(scale + c0);
        float o[4] = {v[g][0] * inv * s4.x, v[g][1] * inv * s4.y, v[g][2] * inv * s4.z,
                      v[g][3] * inv * s4.w};
        put4(dst + c0, o);
    }
}

}  // namespace

int launch_groupnorm_heads(void *out, const void *x, const float *scale, int64_t rows, int H, int d,
                           float eps, int dtype, cudaStream_t s) {
    const int64_t n = rows * H;
    if (n == 0) return RHZ_OK;
    const unsigned grid = static_cast<unsigned>((n + WARPS - 1) / WARPS);
    if (dtype == RHZ_DTYPE_BF16)
        groupnorm_heads_kernel<__nv_bfloat16><<<grid, 32 * WARPS, 0, s>>>(
            static_cast<__nv_bfloat16 *>(out), static_cast<const __nv_bfloat16 *>(x), scale, n, d, eps);
    else
        groupnorm_heads_kernel<float><<<grid, 32 * WARPS, 0, s>>>(static_cast<float *>(out),
                                                                   static_cast<const float *>(x), scale, n, d, eps);
    return check_launch("groupnorm_heads_kernel");
}

}  // namespace rhz
