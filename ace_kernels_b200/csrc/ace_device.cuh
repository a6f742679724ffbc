// Device-side building blocks shared by the histogram, epilogue and gradient
// kernels of the mL1-ACE loss (sm_100a).
//
// Everything that decides which bin a voxel lands in lives here, so the forward
// and the backward kernels run the same instruction sequence on the same logits
// and, for hard binning, a voxel always falls in the same bin in both passes (the
// reference states the same contract for its Triton kernels:
// ace_kernels/kernels/act.py:1-7, ace_kernels/kernels/hard_bwd.py:9-11). Soft
// binning needs no such contract: its weights are continuous in p.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string.h>

#include "ace_types.h"

namespace ace {

// ---------------------------------------------------------------------------
// Rounding-explicit fp32 arithmetic.
//
// The probability and bin-index path must not be contracted into FMAs by the
// compiler (it would round differently in different kernels). On the device the
// *_rn intrinsics are never fused; on the host (used by the CPU test hook for the
// bin index) a volatile store forces one rounding per operation.
// ---------------------------------------------------------------------------
#ifdef __CUDA_ARCH__
#define ACE_FMUL(a, b) __fmul_rn((a), (b))
#define ACE_FADD(a, b) __fadd_rn((a), (b))
#define ACE_FSUB(a, b) __fsub_rn((a), (b))
#define ACE_FDIV(a, b) __fdiv_rn((a), (b))
#else
static inline float ace_host_round(float v) {
  volatile float r = v;
  return r;
}
#define ACE_FMUL(a, b) ace_host_round((a) * (b))
#define ACE_FADD(a, b) ace_host_round((a) + (b))
#define ACE_FSUB(a, b) ace_host_round((a) - (b))
#define ACE_FDIV(a, b) ace_host_round((a) / (b))
#endif

// ---------------------------------------------------------------------------
// Bin index.
//
// Hard binning: the bin of p is torch.bucketize(p, edges, right) = the number of
// edges e_j with e_j < p (e_j <= p when `right`), edges = fp32
// linspace(0, 1 + eps32, K + 1)[1:] (reference: ace_kernels/binning.py:47-51,
// ace_reference/hardl1ace.py:70-90).
//
// Soft binning: the reference computes a half-bin index h against
// linspace(0, 1 + eps32, 2K + 1)[1:] and derives the two neighbouring bins and the
// distances to the replicated centre table (ace_kernels/common.py:43-61,
// ace_reference/softl1ace.py:87-110). Since the 2K boundaries interleave centres
// and edges, (h + 1) / 2 equals j = the number of centres counted for p, and the
// reference's left/right bins are max(j - 1, 0) and min(j, K - 1), with the
// distances taken to (centre j-1 or the -10000 sentinel) and (centre j or the
// +10000 sentinel). So both binnings need one search over a sorted K-entry table.
//
// The search is O(1): a guess from p*K (hard) or p*K + 0.5 (soft), which is
// within one of the answer because entry j is (j+1)/K (hard) or (j+0.5)/K (soft)
// up to a few ulp, then a verified correction against the table itself. The
// correction loop terminates after one or two passes; its bound only guards the
// loop. Entry i of the table holds {t[i-1], t[i]} (sentinels at both ends), so
// one shared-memory load fetches both neighbours, which the soft binning also
// needs as its interval ends.
// ---------------------------------------------------------------------------
// Guess of the count: round(p*n - 0.5) (hard) or round(p*n) (soft), via the
// 1.5 * 2^23 bias (adding it leaves the nearest integer in the low mantissa
// bits), so the guess costs FMA-pipe work only and no float<->int conversion.
// Any guess within one of the answer is corrected by the search below. An
// unsigned minimum clamps it to the table: negative guesses (NaN or negative p)
// become n and are walked down by the slow path like any other wrong guess.
__host__ __device__ __forceinline__ int ace_guess(float p, float nf, int n, bool soft) {
  const float g = soft ? ACE_FMUL(p, nf) : ACE_FSUB(ACE_FMUL(p, nf), 0.5f);
  const float b = ACE_FADD(g, 12582912.0f);
  unsigned i;
#ifdef __CUDA_ARCH__
  i = __float_as_uint(b) - 0x4B400000u;
#else
  memcpy(&i, &b, sizeof(i));
  i -= 0x4B400000u;
#endif
  return (int)(i < (unsigned)n ? i : (unsigned)n);
}

// Is i the count for p, given its table neighbours pr = {t[i-1], t[i]}? The
// table is `right`-adjusted, so "entry counted" is always t < p, and its ends
// hold the -10000 / +10000 sentinels, which need no index test for
// -10000 < p < 10000 (a NaN or an out-of-range value fails the test and takes
// the guarded slow path).
__host__ __device__ __forceinline__ bool ace_is_count(float p, float2 pr) {
  return pr.x < p && !(pr.y < p);
}


// Rare path: walk from a guess that failed ace_is_count to the count (one or two
// steps for probabilities; the bound only guards against NaN / invalid input).
// Returns the count and its neighbours by value, so the caller's registers never
// need a memory address (a reference argument would force them to local memory).
struct Located {
  int i;
  float2 pr;
};

static __host__ __device__ __noinline__ Located ace_fix_count(float p, int i, int n,
                                                              const float2* lohi, int stride) {
  float2 pr = lohi[i * stride];
#pragma unroll 1
  for (int it = 0; it <= n + 1; ++it) {
    const bool lo_ok = (i == 0) || pr.x < p;
    if (lo_ok && (i == n || !(pr.y < p))) break;
    i += lo_ok ? 1 : -1;
    i = i < 0 ? 0 : (i > n ? n : i);
    pr = lohi[i * stride];
  }
  Located r;
  r.i = i;
  r.pr = pr;
  return r;
}

// The count j in [0, n] of table entries counted for p, and its neighbours
// {t[j-1], t[j]}. `lohi_tab` has n + 1 entries `stride` apart; nf = (float)n.
__host__ __device__ __forceinline__ int ace_locate(float p, const float2* lohi_tab, int stride,
                                                   int n, float nf, bool soft, float2& lohi) {
  int i = ace_guess(p, nf, n, soft);
  float2 pr = lohi_tab[i * stride];
  if (!ace_is_count(p, pr)) {
    const Located r = ace_fix_count(p, i, n, lohi_tab, stride);
    i = r.i;
    pr = r.pr;
  }
  lohi = pr;
  return i;
}

#ifdef __CUDACC__

// ---------------------------------------------------------------------------
// Element loads. Logits are read natively (fp32 / bf16 / fp16) and widened to
// fp32; all arithmetic after the load is fp32, as the reference's kernels
// (ace_kernels/kernels/act.py:38-50).
// ---------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ float ace_to_float(T v);
template <>
__device__ __forceinline__ float ace_to_float<float>(float v) { return v; }
template <>
__device__ __forceinline__ float ace_to_float<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <>
__device__ __forceinline__ float ace_to_float<__half>(__half v) { return __half2float(v); }

template <typename T>
__device__ __forceinline__ T ace_from_float(float v);
template <>
__device__ __forceinline__ float ace_from_float<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 ace_from_float<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <>
__device__ __forceinline__ __half ace_from_float<__half>(float v) { return __float2half_rn(v); }

// Read-only vector load of V consecutive elements (V * sizeof(T) in {2..16}
// bytes), widened to fp32. The address must be aligned to V * sizeof(T).
template <typename T, int V>
struct VecIO {
  static constexpr int BYTES = V * (int)sizeof(T);
  static_assert(BYTES == 2 || BYTES == 4 || BYTES == 8 || BYTES == 16 || BYTES == 32,
                "unsupported vector width");

  __device__ __forceinline__ static void load(const T* __restrict__ p, float (&out)[V]) {
    if constexpr (BYTES == 32) {
      const uint4* q = reinterpret_cast<const uint4*>(p);
      uint4 a = __ldg(q), b = __ldg(q + 1);
      T tmp[V];
      *reinterpret_cast<uint4*>(&tmp[0]) = a;
      *reinterpret_cast<uint4*>(&tmp[V / 2]) = b;
#pragma unroll
      for (int i = 0; i < V; ++i) out[i] = ace_to_float<T>(tmp[i]);
    } else if constexpr (BYTES == 16) {
      uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
      T tmp[V];
      *reinterpret_cast<uint4*>(&tmp[0]) = a;
#pragma unroll
      for (int i = 0; i < V; ++i) out[i] = ace_to_float<T>(tmp[i]);
    } else if constexpr (BYTES == 8) {
      uint2 a = __ldg(reinterpret_cast<const uint2*>(p));
      T tmp[V];
      *reinterpret_cast<uint2*>(&tmp[0]) = a;
#pragma unroll
      for (int i = 0; i < V; ++i) out[i] = ace_to_float<T>(tmp[i]);
    } else if constexpr (BYTES == 4) {
      unsigned a = __ldg(reinterpret_cast<const unsigned*>(p));
      T tmp[V];
      *reinterpret_cast<unsigned*>(&tmp[0]) = a;
#pragma unroll
      for (int i = 0; i < V; ++i) out[i] = ace_to_float<T>(tmp[i]);
    } else {
      out[0] = ace_to_float<T>(p[0]);
    }
  }

  // Streaming store (the gradient is written once and not re-read).
  __device__ __forceinline__ static void store(T* __restrict__ p, const float (&in)[V]) {
    T tmp[V];
#pragma unroll
    for (int i = 0; i < V; ++i) tmp[i] = ace_from_float<T>(in[i]);
    if constexpr (BYTES == 32) {
      __stcs(reinterpret_cast<uint4*>(p), *reinterpret_cast<uint4*>(&tmp[0]));
      __stcs(reinterpret_cast<uint4*>(p) + 1, *reinterpret_cast<uint4*>(&tmp[V / 2]));
    } else if constexpr (BYTES == 16) {
      __stcs(reinterpret_cast<uint4*>(p), *reinterpret_cast<uint4*>(&tmp[0]));
    } else if constexpr (BYTES == 8) {
      __stcs(reinterpret_cast<uint2*>(p), *reinterpret_cast<uint2*>(&tmp[0]));
    } else if constexpr (BYTES == 4) {
      __stcs(reinterpret_cast<unsigned*>(p), *reinterpret_cast<unsigned*>(&tmp[0]));
    } else {
      p[0] = tmp[0];
    }
  }
};

// V int64 class labels -> int32. Labels are only compared with channel
// indices (never used as addresses), so the low 32 bits suffice: a class index in
// [0, C) selects its channel; the reference rejects other values, here they
// select whatever channel their low bits name, or none.
template <int V>
__device__ __forceinline__ void ace_load_labels(const int64_t* __restrict__ p, int (&out)[V]) {
  if constexpr (V >= 2) {
#pragma unroll
    for (int i = 0; i < V; i += 2) {
      const int4 a = __ldg(reinterpret_cast<const int4*>(p + i));
      out[i] = a.x;  // little-endian: the low word first
      out[i + 1] = a.z;
    }
  } else {
    out[0] = __ldg(reinterpret_cast<const int*>(p));
  }
}

// Programmatic dependent launch: wait until the grid this one depends on has
// completed and its memory is visible (a no-op without the launch attribute);
// and allow the dependent grid to be scheduled.
__device__ __forceinline__ void ace_grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void ace_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Asynchronous prefetch of [p, p + bytes) from HBM into L2 (no registers, no
// completion to wait for). p and bytes must be multiples of 16; the range must lie
// inside the allocation.
__device__ __forceinline__ void ace_prefetch_l2(const void* p, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// Prefetches into L2 the part of a tile of `count` elements of `elem` bytes
// starting at element `start` of a row of n elements at `row`: from the first
// element if its address is 16-byte aligned (else nothing), up to the last
// 16-byte boundary inside the row.
__device__ __forceinline__ void ace_prefetch_tile(const void* row, int64_t start, int64_t count,
                                                  int64_t n, int elem) {
  if (start >= n) return;
  const int64_t end = min(start + count, n);
  const uintptr_t a0 = reinterpret_cast<uintptr_t>(row) + (uintptr_t)(start * elem);
  const uintptr_t a1 = (reinterpret_cast<uintptr_t>(row) + (uintptr_t)(end * elem)) & ~(uintptr_t)15;
  if ((a0 & 15) != 0 || a1 <= a0) return;
  ace_prefetch_l2(reinterpret_cast<const void*>(a0), (unsigned)(a1 - a0));
}

// ---------------------------------------------------------------------------
// Activation. Softmax over channels: m = max_c x_c, e_c = exp(x_c - m),
// s = sum_c e_c (ascending c), p_c = e_c / s, as torch.softmax and the
// reference's fused kernels (ace_kernels/kernels/act.py:38-62). exp is CUDA's
// expf (not the fast approximation), compiled without fast-math. Sigmoid:
// 1 / (1 + exp(-x)) with IEEE division.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ace_sigmoid(float x) {
  return ACE_FDIV(1.0f, ACE_FADD(1.0f, expf(-x)));
}

// Approximate reciprocal (the hardware's, max 1 ulp error). s > 0 finite.
__device__ __forceinline__ float ace_rcp_approx(float s) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(s));
  return y;
}

// Reciprocal of s in [1, 2^64) to about half an ulp: the hardware approximation
// refined by one Newton-Raphson step, y += y (1 - s y).
__device__ __forceinline__ float ace_rcp_refined(float s) {
  const float y = ace_rcp_approx(s);
  return __fmaf_rn(__fmaf_rn(-s, y, 1.0f), y, y);
}

// a / s from y ~ 1/s with Markstein's correction step (P. Markstein,
// "Computation of elementary functions on the IBM RISC System/6000 processor",
// IBM J. Res. Dev. 34(1), 1990): q0 = a y, the remainder r = a - s q0 is exact
// with an FMA, and q = q0 + r y carries an error of about |q - q0| |1 - s y|
// before its single rounding, so q is the correctly rounded quotient unless a/s
// lies within ~2^-23 ulp of a rounding midpoint. One reciprocal per voxel then
// serves all C channels of the softmax.
__device__ __forceinline__ float ace_div_corrected(float a, float s, float y) {
  const float q0 = __fmul_rn(a, y);
  const float r = __fmaf_rn(-s, q0, a);
  return __fmaf_rn(r, y, q0);
}

// In place: x[c] (c < C, C <= CM) logits -> exp(x - max); returns the sum.
template <int CM>
__device__ __forceinline__ float ace_softmax_exp(float (&x)[CM], int C) {
  float m = x[0];
#pragma unroll
  for (int c = 1; c < CM; ++c)
    if (c < C) m = fmaxf(m, x[c]);
  float s = 0.0f;
#pragma unroll
  for (int c = 0; c < CM; ++c) {
    if (c < C) {
      const float e = expf(ACE_FSUB(x[c], m));
      x[c] = e;
      s = ACE_FADD(s, e);
    }
  }
  return s;
}

// In place: x[c] (c < C) logits -> softmax probabilities, the one routine every
// kernel uses (so a voxel's probabilities, hence its bins, are bit-identical in
// the forward and the backward). The division by the sum uses one refined
// reciprocal per voxel and the corrected quotient per channel (see
// ace_div_corrected): s is in [1, C], so no special cases arise.
template <int CM>
__device__ __forceinline__ void ace_softmax(float (&x)[CM], int C) {
  const float s = ace_softmax_exp<CM>(x, C);
  const float y = ace_rcp_refined(s);
#pragma unroll
  for (int c = 0; c < CM; ++c)
    if (c < C) x[c] = ace_div_corrected(x[c], s, y);
}

// Softmax for soft binning, where no bin has to match the reference's bit for
// bit: the soft weights are continuous in p, and the loss and gradient are
// compared with a tolerance. exp(x - m) = 2^(x log2(e) - m log2(e)): one fused
// multiply-add against the rounded m log2(e) of the voxel (a common factor that
// cancels in the normalisation) and the hardware base-2 exponential
// (ex2.approx.ftz, relative error about 2^-22); the normalisation is one
// approximate reciprocal per voxel (1 ulp). p is then within a few ulp of the
// correctly rounded softmax for the probabilities that carry weight, at about a
// third of the instructions of ace_softmax; every kernel that calls these
// functions gets the same p.
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ace_exp2_approx(float t) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(t));
  return y;
}

// exp(x - m) given mL = m * log2(e) (rounded once, ACE_FMUL).
__device__ __forceinline__ float ace_exp_fast(float x, float mL) {
  return ace_exp2_approx(__fmaf_rn(x, kLog2e, -mL));
}

template <int CM>
__device__ __forceinline__ void ace_softmax_fast(float (&x)[CM], int C) {
  float m = x[0];
#pragma unroll
  for (int c = 1; c < CM; ++c)
    if (c < C) m = fmaxf(m, x[c]);
  const float mL = ACE_FMUL(m, kLog2e);
  float s = 0.0f;
#pragma unroll
  for (int c = 0; c < CM; ++c) {
    if (c < C) {
      x[c] = ace_exp_fast(x[c], mL);
      s = ACE_FADD(s, x[c]);
    }
  }
  const float y = ace_rcp_approx(s);
#pragma unroll
  for (int c = 0; c < CM; ++c)
    if (c < C) x[c] = ACE_FMUL(x[c], y);
}

// The softmax a kernel instance uses: fast for soft binning, exact otherwise.
template <bool FAST, int CM>
__device__ __forceinline__ void ace_softmax_sel(float (&x)[CM], int C) {
  if constexpr (FAST) ace_softmax_fast<CM>(x, C);
  else ace_softmax<CM>(x, C);
}

#endif  // __CUDACC__

}  // namespace ace
