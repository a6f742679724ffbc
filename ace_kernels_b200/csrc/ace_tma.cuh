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

// A lane's voxel pair of one channel from a stage, widened to fp32.
template <typename T>
__device__ __forceinline__ float2 lds_pair(unsigned a);
template <>
__device__ __forceinline__ float2 lds_pair<float>(unsigned a) {
  float2 x;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(x.x), "=f"(x.y) : "r"(a));
  return x;
}
__device__ __forceinline__ unsigned lds_u32(unsigned a) {
  unsigned w;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(w) : "r"(a));
  return w;
}
// Two packed 16-bit values widened to fp32 (low half first).
template <typename T>
__device__ __forceinline__ float2 widen2(unsigned w);
template <>
__device__ __forceinline__ float2 widen2<__nv_bfloat16>(unsigned w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 widen2<__half>(unsigned w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
template <>
__device__ __forceinline__ float2 lds_pair<__nv_bfloat16>(unsigned a) {
  return widen2<__nv_bfloat16>(lds_u32(a));
}
template <>
__device__ __forceinline__ float2 lds_pair<__half>(unsigned a) {
  return widen2<__half>(lds_u32(a));
}
// Elementwise maximum of two packed 16-bit pairs (a NaN loses, as with fmaxf;
// exact, so the maximum of the widened values).
template <typename T>
__device__ __forceinline__ unsigned max2(unsigned a, unsigned b);
template <>
__device__ __forceinline__ unsigned max2<__nv_bfloat16>(unsigned a, unsigned b) {
  unsigned r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
template <>
__device__ __forceinline__ unsigned max2<__half>(unsigned a, unsigned b) {
  unsigned r;
  asm("max.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Plain loads from a stage (a pointer into this CTA's shared memory, read after
// the stage's full barrier: the compiler may schedule them like any load).
template <typename T>
__device__ __forceinline__ float2 ld_pair(const unsigned char* p) {
  if constexpr (sizeof(T) == 4) return *reinterpret_cast<const float2*>(p);
  else return widen2<T>(*reinterpret_cast<const unsigned*>(p));
}
__device__ __forceinline__ int2 ld_labels2(const unsigned char* p) {
  const int4 v = *reinterpret_cast<const int4*>(p);  // two int64, little-endian
  return make_int2(v.x, v.z);
}

// The low words of a lane's two int64 labels from a stage.
__device__ __forceinline__ int2 lds_labels2(unsigned a) {
  unsigned long long l0, l1;
  asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(l0), "=l"(l1) : "r"(a));
  return make_int2((int)l0, (int)l1);
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

// The producer thread of a forward pipeline (soft_fwd_kernel, mc_fwd_kernel).
// Tiles of TV voxels are claimed from per-batch counters `ctr` (one claim ahead,
// so its latency hides behind the stages in flight); the CTA starts on batch
// blockIdx.x * B / gridDim.x and, when a batch runs out, takes tiles of another
// one with tiles left. Each tile's C logit rows (TV * sizeof(T) bytes apart in
// the stage) and its int64 labels (after the rows) are streamed into stage i % S
// of the ring (the labels after `rows` >= C row slots), with s_meta[s] = {tile,
// batch, voxels, 0}; the last stage carries
// the end marker (tile -1, no copies). A wait that runs out sets s_abort and the
// error word; the producer then waits (bounded) for its copies still in flight.
template <typename T, int TV>
__device__ __forceinline__ void produce_claimed(const T* x, const int64_t* lab, int C, int rows,
                                                int64_t N,
                                                int B, int64_t tpb, unsigned* ctr,
                                                unsigned stage0, unsigned SB, int S,
                                                unsigned long long* s_full,
                                                unsigned long long* s_empty, int4* s_meta,
                                                volatile int* s_abort, unsigned* err) {
  constexpr unsigned XB = TV * sizeof(T);
  int b = (int)((int64_t)blockIdx.x * B / gridDim.x);
  unsigned pend = atomicAdd(ctr + b, 1u);  // claimed one tile ahead
  int pend_b = b;
  int issued = 0;
  for (int i = 0;; ++i) {
    const int s = i % S;
    const unsigned use = (unsigned)(i / S);
    int64_t tile = pend;
    int tb = pend_b;
    if (tile >= tpb) {  // this batch is done: take a tile of another one
      tile = -1;
      for (int k = 1; k < B; ++k) {
        const int bb = (pend_b + k) % B;
        const unsigned t2 = atomicAdd(ctr + bb, 1u);
        if ((int64_t)t2 < tpb) {
          tile = t2;
          tb = bb;
          break;
        }
      }
    }
    if (tile >= 0) {
      pend = atomicAdd(ctr + tb, 1u);
      pend_b = tb;
    }
    // the stage's previous tile must have been read
    if (use > 0 && !mbar_wait(smem_addr(&s_empty[s]), (use - 1) & 1u)) {
      *s_abort = 1;
      atomicExch(err, 1u);
      break;
    }
    if (*s_abort) break;
    if (tile < 0) {  // no tiles left: the end marker (no copies)
      s_meta[s] = make_int4(-1, 0, 0, 0);
      mbar_arrive(smem_addr(&s_full[s]));
      break;
    }
    const int64_t v0 = tile * TV;
    const int cnt = (int)min((int64_t)TV, N - v0);
    s_meta[s] = make_int4((int)tile, tb, cnt, 0);
    const unsigned xb = (unsigned)cnt * (unsigned)sizeof(T), lb = (unsigned)cnt * 8u;
    const unsigned full = smem_addr(&s_full[s]);
    mbar_arrive_tx(full, (unsigned)C * xb + lb);
    const unsigned dst = stage0 + (unsigned)s * SB;
    const T* gx = x + (int64_t)tb * C * N + v0;
    for (int c = 0; c < C; ++c) bulk_load(dst + c * XB, gx + (int64_t)c * N, xb, full);
    bulk_load(dst + rows * XB, lab + (int64_t)tb * N + v0, lb, full);
    issued = i + 1;
  }
  // After an abort no copy may still be in flight when the CTA leaves: wait
  // (bounded) for the last fill of every stage. (Otherwise the consumers have
  // consumed every fill before the CTA's final barrier.)
  if (*s_abort)
    for (int i = issued - S > 0 ? issued - S : 0; i < issued; ++i)
      mbar_wait(smem_addr(&s_full[i % S]), (unsigned)(i / S) & 1u);
}

}  // namespace ace
