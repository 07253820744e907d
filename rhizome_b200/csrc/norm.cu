// Per-head output norm, groupnorm_heads (crates/ops/src/norm.rs:48-60): every
// (row, head) slice of d values is RMS-normalised on its own,
//   out = x / sqrt(mean(x^2) + eps) * scale[0..d)   (norm.rs:8-13),
// with the same first d entries of `scale` for every head, as the reference
// slices scale[..dh]. General d: one warp per (row, head), four channels per
// lane and channel group, 8/16-byte vector accesses, a shuffle sum. d = 128
// (the model's head width): 16-byte accesses, several slices per warp in
// flight. In place allowed.
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

// d = 128 with 16-byte rows: a slice is 128 / VEC lanes (16 for bf16, 32 for
// f32), each warp keeps U passes of loads in flight before it reduces and
// stores (the one-slice-per-warp kernel above held 256 B in flight per warp,
// too little to cover HBM latency), grid-stride over groups of slices.
template <typename T>
__global__ void __launch_bounds__(32 * WARPS) groupnorm_d128_kernel(T *out, const T *x,
                                                                    const float *scale, int64_t n,
                                                                    float eps) {
    constexpr int D = 128;
    constexpr int VEC = 16 / static_cast<int>(sizeof(T));  // elements per 16-byte access
    constexpr int LPS = D / VEC;                           // lanes per slice
    constexpr int SPP = 32 / LPS;                          // slices per pass
    constexpr int U = 4;                                   // passes in flight
    const int lane = threadIdx.x & 31;
    const int sub = lane / LPS, cl = lane % LPS;
    const int64_t wg = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nw = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    float sc[VEC];
#pragma unroll
    for (int e = 0; e < VEC; e += 4) {
        const float4 s4 = *reinterpret_cast<const float4 *>(scale + cl * VEC + e);
        sc[e] = s4.x; sc[e + 1] = s4.y; sc[e + 2] = s4.z; sc[e + 3] = s4.w;
    }
    for (int64_t base = wg * (U * SPP); base < n; base += nw * (U * SPP)) {
        uint4 raw[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t slice = base + u * SPP + sub;
            raw[u] = slice < n ? *reinterpret_cast<const uint4 *>(x + slice * D + cl * VEC)
                               : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int64_t slice = base + u * SPP + sub;
            float v[VEC];
            if constexpr (sizeof(T) == 2) {
                const uint32_t w[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[e]));
                    v[2 * e] = f.x;
                    v[2 * e + 1] = f.y;
                }
            } else {
                v[0] = __uint_as_float(raw[u].x); v[1] = __uint_as_float(raw[u].y);
                v[2] = __uint_as_float(raw[u].z); v[3] = __uint_as_float(raw[u].w);
            }
            float ss = 0.f;
#pragma unroll
            for (int e = 0; e < VEC; ++e) ss += v[e] * v[e];
#pragma unroll
            for (int off = LPS / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
            const float inv = 1.f / sqrtf(ss / static_cast<float>(D) + eps);
            if (slice < n) {
                T *dst = out + slice * D + cl * VEC;
#pragma unroll
                for (int e = 0; e < VEC; e += 4) {
                    const float o[4] = {v[e] * inv * sc[e], v[e + 1] * inv * sc[e + 1],
                                        v[e + 2] * inv * sc[e + 2], v[e + 3] * inv * sc[e + 3]};
                    put4(dst + e, o);
                }
            }
        }
    }
}

}  // namespace

int launch_groupnorm_heads(void *out, const void *x, const float *scale, int64_t rows, int H, int d,
                           float eps, int dtype, cudaStream_t s) {
    const int64_t n = rows * H;
    if (n == 0) return RHZ_OK;
    if (d == 128 && aligned(out, 16) && aligned(x, 16) && aligned(scale, 16)) {
        int sms = 148;
        bool sm100 = true;
        device_info(&sms, &sm100);
        const int64_t per_cta = WARPS * 4 * (dtype == RHZ_DTYPE_BF16 ? 2 : 1);
        int64_t grid = (n + per_cta - 1) / per_cta;
        if (grid > static_cast<int64_t>(sms) * 16) grid = static_cast<int64_t>(sms) * 16;
        if (dtype == RHZ_DTYPE_BF16)
            groupnorm_d128_kernel<__nv_bfloat16><<<static_cast<unsigned>(grid), 32 * WARPS, 0, s>>>(
                static_cast<__nv_bfloat16 *>(out), static_cast<const __nv_bfloat16 *>(x), scale, n, eps);
        else
            groupnorm_d128_kernel<float><<<static_cast<unsigned>(grid), 32 * WARPS, 0, s>>>(
                static_cast<float *>(out), static_cast<const float *>(x), scale, n, eps);
        return check_launch("groupnorm_d128_kernel");
    }
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
