// Tensor-core chunked GDR kernel (work in progress).
#include "common.cuh"
#include "kernels.h"

namespace rhz {
bool chunk_tc_supports(int, int) { return false; }
int launch_chunk_tc(const SeqArgs &) {
    return set_error(RHZ_ERR_SHAPE, "tensor-core chunked kernel not built");
}
}  // namespace rhz
