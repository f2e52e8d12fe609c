// tcgen05 GEMM (placeholder until the tensor-core kernel lands).
#include "gemm.cuh"

namespace ancha {
int gemm_tc(const GemmGroup&, int, const GemmEpilogue&, cudaStream_t) {
    return fail(ANCHA_E_UNSUPPORTED, "tcgen05 GEMM not built");
}
}  // namespace ancha
