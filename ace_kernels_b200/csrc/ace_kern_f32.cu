// Kernel instances for float logits (one translation unit per dtype, so the
// build compiles the dtypes in parallel).
#include "ace_kernels.cuh"

namespace ace {
ACE_INSTANTIATE(float)
}  // namespace ace
