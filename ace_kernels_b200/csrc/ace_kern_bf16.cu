// Kernel instances for __nv_bfloat16 logits (one translation unit per dtype, so the
// build compiles the dtypes in parallel).
#include "ace_kernels.cuh"

namespace ace {
ACE_INSTANTIATE(__nv_bfloat16)
}  // namespace ace
