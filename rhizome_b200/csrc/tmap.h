// Tensor-map encoding shared by the kernels that load tiles with TMA. The
// driver's cuTensorMapEncodeTiled is reached through the runtime's
// entry-point query, so the library links no libcuda.
#pragma once

#include <cuda.h>

#include <cstdint>

namespace rhz {

// A tiled tensor map over `rank` dimensions, innermost first: dims in
// elements, strides in bytes for dimensions 1 .. rank - 1, box in elements.
// Out-of-range boxes read zeros. Returns RHZ_OK or sets the error message.
int encode_tmap(CUtensorMap *m, CUtensorMapDataType type, int rank, const void *base,
                const uint64_t *dims, const uint64_t *strides, const uint32_t *box,
                CUtensorMapSwizzle swizzle);

// q, k or v rows [tokens][H][128] bf16 as the chunked kernels read them: a
// box of 64 channels x 1 head x 64 tokens, 128-byte swizzle.
int make_chunk_tmap(CUtensorMap *m, const void *base, int64_t tokens, int H);

}  // namespace rhz
