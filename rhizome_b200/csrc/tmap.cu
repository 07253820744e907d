// Tensor-map encoding shared by the TMA kernels (see tmap.h).
#include "tmap.h"

#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <mutex>

#include "common.cuh"

namespace rhz {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

}  // namespace

int encode_tmap(CUtensorMap *m, CUtensorMapDataType type, int rank, const void *base,
                const uint64_t *dims, const uint64_t *strides, const uint32_t *box,
                CUtensorMapSwizzle swizzle) {
    auto fn = encode_fn();
    if (!fn) return set_error(RHZ_ERR_DEVICE, "cuTensorMapEncodeTiled is unavailable");
    if (rank < 1 || rank > 5) return set_error(RHZ_ERR_INVALID, "tensor map rank %d", rank);
    cuuint64_t d[5], s[4];
    cuuint32_t b[5], e[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = static_cast<cuuint64_t>(dims[i]);
        b[i] = static_cast<cuuint32_t>(box[i]);
        e[i] = 1;
        if (i + 1 < rank) s[i] = static_cast<cuuint64_t>(strides[i]);
    }
    CUresult r = fn(m, type, static_cast<cuuint32_t>(rank), const_cast<void *>(base), d, s, b, e,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(RHZ_ERR_DEVICE, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return RHZ_OK;
}

int make_chunk_tmap(CUtensorMap *m, const void *base, int64_t tokens, int H) {
    constexpr uint64_t HD = 128;
    const uint64_t dims[3] = {HD, static_cast<uint64_t>(H), static_cast<uint64_t>(tokens)};
    const uint64_t strides[2] = {HD * 2, static_cast<uint64_t>(H) * HD * 2};
    const uint32_t box[3] = {64, 1, 64};
    return encode_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box,
                       CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace rhz
