// Compound ops (drop-in for the reference's include/porch/ops.hpp:7-9).
// They are graph builders over tensor primitives; the B200 lowering
// recognises their shapes (e.g. softmax) and runs them as fused kernels.
#pragma once

#include "porch/tensor.hpp"

namespace porch {

    [[nodiscard]] tensor_expr relu(tensor_expr value);
    [[nodiscard]] tensor_expr softmax(tensor_expr value, size_t axis);
    [[nodiscard]] tensor_expr logistic(tensor_expr value);

} // namespace porch
