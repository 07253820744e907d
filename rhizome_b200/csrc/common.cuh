// Shared host/device helpers for the GDR library (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/rhizome_gdr.h"

namespace rhz {

// ---------------------------------------------------------------- host side

// Records a printf-style message as this thread's last error; returns `code`.
int set_error(int code, const char *fmt, ...);
// Clears this thread's last error (called on entry by every API function).
void clear_error();
// Maps a pending launch error to RHZ_ERR_DEVICE (and records it).
int check_launch(const char *what);
// Current device's SM count and whether it is an sm_100 part.
int device_info(int *sm_count, bool *is_sm100);

inline bool aligned(const void *p, size_t a) {
    return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

inline cudaStream_t as_cuda(rhz_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// ---------------------------------------------------------------- device side

__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
    return __float2bfloat16_rn(x);
}

// Four consecutive elements as f32; `vec` selects one aligned vector load
// (row starts are 16-byte aligned for f32 / 8-byte for bf16 when d % 4 == 0),
// otherwise element loads masked by `n_valid` (0..4).
__device__ __forceinline__ void load4(const float *p, bool vec, int n_valid, float (&x)[4]) {
    if (vec && n_valid == 4) {
        float4 t = *reinterpret_cast<const float4 *>(p);
        x[0] = t.x; x[1] = t.y; x[2] = t.z; x[3] = t.w;
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = e < n_valid ? p[e] : 0.f;
    }
}

__device__ __forceinline__ void load4(const __nv_bfloat16 *p, bool vec, int n_valid,
                                      float (&x)[4]) {
    if (vec && n_valid == 4) {
        uint2 t = *reinterpret_cast<const uint2 *>(p);
        __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162 *>(&t.x);
        __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162 *>(&t.y);
        float2 fa = __bfloat1622float2(a), fb = __bfloat1622float2(b);
        x[0] = fa.x; x[1] = fa.y; x[2] = fb.x; x[3] = fb.y;
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) x[e] = e < n_valid ? __bfloat162float(p[e]) : 0.f;
    }
}

__device__ __forceinline__ void store4(float *p, bool vec, int n_valid, const float (&x)[4]) {
    if (vec && n_valid == 4) {
        *reinterpret_cast<float4 *>(p) = make_float4(x[0], x[1], x[2], x[3]);
    } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
            if (e < n_valid) p[e] = x[e];
    }
}

}  // namespace rhz
