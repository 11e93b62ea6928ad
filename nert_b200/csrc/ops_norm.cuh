// Softmax / LayerNormalization rows (ops_norm.cu).
#pragma once

#include "runtime.hpp"

#include <cstdint>

namespace nb2 {

// Softmax over the middle axis of an [outer, L, inner] view.
void softmax(nb2_device* dev, const float* x, float* y, int64_t outer, int64_t L, int64_t inner);

// LayerNormalization over rows of length D (the trailing axes from `axis`);
// `bias`, `mean` and `inv_std` may be null.
void layernorm(nb2_device* dev, const float* x, const float* scale, const float* bias, float* y, float* mean,
               float* inv_std, int64_t rows, int64_t D, float eps);

} // namespace nb2
