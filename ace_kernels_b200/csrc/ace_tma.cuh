// Building blocks of the TMA-pipelined kernels (soft_fwd_kernel and
// grad_tma_kernel) on B200 (sm_100a): the CTA shape (one producer warp that
// streams tiles into a shared-memory ring with bulk copies, kPipeConsumerWarps
// consumer warps), mbarrier and bulk-copy wrappers with bounded waits, and the
// consumers' shared-memory loads of a tile. Included by ace_kernels.cuh after the
// shared helpers.
#pragma once

namespace ace {

constexpr int kPipeConsumerWarps = 16;
constexpr int kPipeThreads = (kPipeConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kPipeLaneVoxels = 4;                            // voxels per consumer lane per tile
constexpr int kPipeTileVoxels = kPipeConsumerWarps * 32 * kPipeLaneVoxels;
constexpr int kPipeMaxStages = 4;
constexpr unsigned long long kPipeWaitNs = 1000000000ull;  // bound of every barrier wait (1 s)

__device__ __forceinline__ unsigned smem_addr(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long ace_now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// mbarrier and bulk-copy primitives (shared addresses of this CTA).
__device__ __forceinline__ void mbar_init(unsigned bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(unsigned bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(unsigned bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits until the barrier's phase of parity `parity` has completed; false if
// that takes longer than kPipeWaitNs.
__device__ __forceinline__ bool mbar_wait(unsigned bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = ace_now_ns();
  while (!mbar_try_wait(bar, parity))
    if (ace_now_ns() - t0 > kPipeWaitNs) return false;
  return true;
}
// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from
// global memory into this CTA's shared memory, completing on barrier `bar`.
__device__ __forceinline__ void bulk_load(unsigned dst, const void* src, unsigned bytes,
                                          unsigned bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// Barrier of the consumer warps only (the producer runs ahead meanwhile).
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kPipeConsumerWarps * 32) : "memory");
}

// A lane's kPipeLaneVoxels logits of one channel from a stage, widened to fp32.
template <typename T>
__device__ __forceinline__ void lds_logits(unsigned a, float (&x)[4]);
template <>
__device__ __forceinline__ void lds_logits<float>(unsigned a, float (&x)[4]) {
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(x[0]), "=f"(x[1]), "=f"(x[2]), "=f"(x[3])
               : "r"(a));
}
template <>
__device__ __forceinline__ void lds_logits<__nv_bfloat16>(unsigned a, float (&x)[4]) {
  unsigned w0, w1;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(w0), "=r"(w1) : "r"(a));
  x[0] = __uint_as_float(w0 << 16);
  x[1] = __uint_as_float(w0 & 0xffff0000u);
  x[2] = __uint_as_float(w1 << 16);
  x[3] = __uint_as_float(w1 & 0xffff0000u);
}
template <>
__device__ __forceinline__ void lds_logits<__half>(unsigned a, float (&x)[4]) {
  unsigned w0, w1;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(w0), "=r"(w1) : "r"(a));
  const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&w0));
  const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&w1));
  x[0] = f0.x;
  x[1] = f0.y;
  x[2] = f1.x;
  x[3] = f1.y;
}

// The low words of a lane's kPipeLaneVoxels int64 labels from a stage.
__device__ __forceinline__ void lds_labels(unsigned a, int (&lab)[4]) {
  unsigned long long l0, l1, l2, l3;
  asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(l0), "=l"(l1) : "r"(a));
  asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(l2), "=l"(l3) : "r"(a + 16));
  lab[0] = (int)l0;
  lab[1] = (int)l1;
  lab[2] = (int)l2;
  lab[3] = (int)l3;
}

}  // namespace ace
