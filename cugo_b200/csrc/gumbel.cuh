// Gumbel noise of the policy samplers (sample_kernel, the fused MLP's sampling head):
// u = ((word >> 8) + 0.5) * 2^-24 in (0, 1), g = -log(-log(u)) for a Philox word.
// One definition, so both samplers draw identical noise.
#pragma once

#include <math.h>
#include <stdint.h>

namespace cb {

__device__ __forceinline__ float gumbel_of(uint32_t word) {
  const float u = (static_cast<float>(word >> 8) + 0.5f) * (1.0f / 16777216.0f);
  return -logf(-logf(u));
}

}  // namespace cb
