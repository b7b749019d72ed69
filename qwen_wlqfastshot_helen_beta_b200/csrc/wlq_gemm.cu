// Prefill GEMM (M > 16) -- placeholder until the tcgen05 kernel lands.
#include "wlq_common.cuh"
#include "wlq_internal.h"

namespace wlq {
int launch_gemm(const LinearArgs& a, cudaStream_t) {
    return fail(WLQ_ERR_UNSUPPORTED, "wlq_gemm: M=%d > 16 needs the tensor-core GEMM, not in this build", a.M);
}
}  // namespace wlq
