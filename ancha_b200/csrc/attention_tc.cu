// tcgen05 attention (placeholder until the tensor-core kernel lands).
#include "attention.cuh"

namespace ancha {
int attention_tc(const AttnArgs&, cudaStream_t) {
    return fail(ANCHA_E_UNSUPPORTED, "tcgen05 attention not built");
}
}  // namespace ancha
