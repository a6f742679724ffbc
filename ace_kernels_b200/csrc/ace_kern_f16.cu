// Kernel instances for __half logits (one translation unit per dtype, so the
// build compiles the dtypes in parallel).
#include "ace_kernels.cuh"

namespace ace {
ACE_INSTANTIATE(__half)
}  // namespace ace
