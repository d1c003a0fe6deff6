// tcgen05 3xTF32 GEMM emitter (placeholder until the tensor-core path lands:
// every GEMM currently takes the CUDA-core path).
#include "lower.hpp"

namespace porch::detail {

    int lowerer::emit_gemm_tc(int, const box&, kernel&, const kernel_arg&, const kernel_arg&,
                              int64_t, int64_t, int64_t) {
        return -1;
    }

} // namespace porch::detail
