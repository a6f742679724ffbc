// Kernels of the mL1-ACE loss on B200 (sm_100a): the fused histogram (forward),
// the epilogue, and the gradient (backward). Instantiated per logit dtype in
// ace_kern_{f32,bf16,f16}.cu.
//
// All three are HBM-bound streaming kernels on CUDA cores: nothing on this path
// is a dense contraction, so there is no tensor-core work.
#pragma once

#include "ace_device.cuh"
#include "ace_types.h"

namespace ace {

// Which kernel variant a launch uses; chosen on the host (ace_api.cu).
struct Variant {
  int V;        // voxels per thread per tile (vector width of the loads)
  int CM;       // softmax: channel capacity of the register tile; pointwise: 1
  bool softmax; // activation softmax over C > 1 channels (else none / sigmoid)
  bool soft;    // soft binning
  bool labels;  // int64 labels (else dense fp32 targets)
  bool split;   // forward only: soft_fwd_kernel (softmax, CM <= 4, soft, labels)
  bool mc;      // mc_fwd_kernel / mc_grad_kernel (softmax over many channels)
  int offset;   // soft_fwd_kernel: 1 when the background channel is dropped
};

template <typename T>
cudaError_t launch_hist(const FwdParams& p, const Variant& v, dim3 grid, int smem,
                        cudaStream_t s, int dev);
template <typename T>
cudaError_t launch_grad(const BwdParams& p, const Variant& v, dim3 grid, int smem,
                        cudaStream_t s, int dev);
template <typename T>
cudaError_t launch_probs(const void* x, float* probs, int64_t B, int C, int64_t N, int act,
                         cudaStream_t s);
// Occupancy (CTAs per SM) of the variant's kernel with `smem` dynamic bytes on
// device `dev` (the current device).
template <typename T>
int hist_occupancy(const Variant& v, int smem, int dev);
template <typename T>
int grad_occupancy(const Variant& v, int smem, int dev);

// Multi-CTA epilogue on [3, B_total, CL, K] statistics; `ws` holds a counter
// (left at zero) and one partial sum per CTA.
cudaError_t launch_epilogue(const float* hist, const EpiParams& e, unsigned* counter,
                            float* partial, cudaStream_t s);
constexpr int kEpiRowsPerCta = 32;

#ifdef __CUDACC__

// ---------------------------------------------------------------------------
// Epilogue: per row (b, c) and bin k, from W, P, G:
//   nonempty = W != 0 (hard) / W >= empty_weight (soft)
//   d = P / W - G / W (two IEEE divisions, then subtract; 0 if empty)
//   f = sum_nonempty |d| / K_ne (NaN if K_ne = 0)
//   coef = sign(d) / (K_ne * W) (0 if empty)
//   present = sum_k G > 0; f *= present (if ignore_empty); f *= w_c
//   jac = [present] * w_c (/ rows for "mean"); loss = mean or sum of f
// Same formulas and operation order as v2_autograd.coefficients
// (ace_kernels/impls/v2_autograd.py:66-76), common.reduce_classes
// (ace_kernels/common.py:184-207) and the fused Triton epilogue
// (ace_kernels/kernels/epilogue.py:23-82). One warp per row, lanes over bins
// (K <= 128: up to four bins a lane), butterfly reductions; the loss is summed in
// a fixed order (rows ascending per warp, warps ascending, then CTAs ascending),
// so it is deterministic.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = ACE_FADD(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Epilogue of row r by one warp, from the row's W, P, G held by its lanes (lane
// l has bins l, l + 32, l + 64, l + 96; entries past K are ignored). Writes d,
// coef, f and jac of the row and returns f (on every lane).
__device__ __forceinline__ float epilogue_row(const EpiParams& E, int r, const float (&w)[4],
                                              const float (&p)[4], const float (&g)[4]) {
  const int lane = threadIdx.x & 31;
  const int K = E.K;
  const float nan = __int_as_float(0x7fc00000);
  float dk[4], wk[4];
  bool ne[4];
  int kne = 0;
  float err = 0.0f, gsum = 0.0f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int k = lane + 32 * q;
    dk[q] = 0.0f;
    wk[q] = 1.0f;
    ne[q] = false;
    if (k < K) {
      gsum = ACE_FADD(gsum, g[q]);
      ne[q] = E.soft ? (w[q] >= E.empty_weight) : (w[q] != 0.0f);
      if (ne[q]) {
        wk[q] = w[q];
        dk[q] = ACE_FSUB(ACE_FDIV(p[q], w[q]), ACE_FDIV(g[q], w[q]));
        err = ACE_FADD(err, fabsf(dk[q]));
        ++kne;
      }
    }
  }
  kne = warp_sum_i(kne);
  err = warp_sum(err);
  gsum = warp_sum(gsum);
  const float kf = (float)kne;
  const int64_t out = (int64_t)r * K;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int k = lane + 32 * q;
    if (k < K) {
      const float sg = dk[q] > 0.0f ? 1.0f : (dk[q] < 0.0f ? -1.0f : 0.0f);
      E.d[out + k] = dk[q];
      E.coef[out + k] = ne[q] ? ACE_FDIV(sg, ACE_FMUL(kf, wk[q])) : 0.0f;
    }
  }
  float f = kne > 0 ? ACE_FDIV(err, kf) : nan;
  const float present = gsum > 0.0f ? 1.0f : 0.0f;
  const float wc = E.class_w[r % E.CL];
  float scale = wc;
  if (E.ignore_empty) {
    f = ACE_FMUL(f, present);  // NaN stays NaN, as the reference
    scale = ACE_FMUL(present, wc);
  }
  f = ACE_FMUL(f, wc);
  if (E.reduction == ACE_B200_REDUCTION_MEAN) scale = ACE_FDIV(scale, (float)E.rows_global);
  if (lane == 0) {
    E.f[r] = f;
    E.jac[r] = scale;
  }
  return f;
}

// Sum over the CTA of each warp's `mine` (the sum of f over the rows the warp
// took), in warp order: a fixed order, so the loss is deterministic. Called by
// all threads; returns the total on every thread.
__device__ __forceinline__ float cta_sum_in_warp_order(float mine) {
  __shared__ float wsum[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  if (lane == 0) wsum[warp] = mine;
  __syncthreads();
  float total = 0.0f;
  for (int w = 0; w < nwarps; ++w) total = ACE_FADD(total, wsum[w]);
  __syncthreads();
  return total;
}

// Rows [r0, r1) of the epilogue; `st` points at [3, R_total, K] statistics
// (shared or global memory) and row r of it is statistics row r - st_row0.
// Returns (on every thread) this CTA's sum of f over its rows, in fixed order.
__device__ __forceinline__ float epilogue_rows(const EpiParams& E, const float* st, int st_rows,
                                               int st_row0, int r0, int r1) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int K = E.K;
  const int64_t RK = (int64_t)st_rows * K;
  float mine = 0.0f;
  for (int r = r0 + warp; r < r1; r += nwarps) {
    const int64_t base = (int64_t)(r - st_row0) * K;
    float w[4], p[4], g[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int k = lane + 32 * q;
      w[q] = k < K ? st[base + k] : 0.0f;
      p[q] = k < K ? st[RK + base + k] : 0.0f;
      g[q] = k < K ? st[2 * RK + base + k] : 0.0f;
    }
    mine = ACE_FADD(mine, epilogue_row(E, r, w, p, g));
  }
  return cta_sum_in_warp_order(mine);
}

__device__ __forceinline__ void write_loss(const EpiParams& E, float total) {
  if (E.reduction == ACE_B200_REDUCTION_MEAN) total = ACE_FDIV(total, (float)E.rows_global);
  E.loss[0] = total;
}

__device__ __forceinline__ void write_loss_if0(const EpiParams& E, float total) {
  if (threadIdx.x == 0) write_loss(E, total);
}

// ---------------------------------------------------------------------------
// Shared-memory statistics table: integer fixed point, lane-replicated.
//
// Values are accumulated with native 32-bit integer shared-memory atomics (a
// float atomic add there is a compare-and-swap loop, measured 3x slower). A
// value v in [0, 1] is added as the bit pattern of the float v * 2^21 +
// 1.5 * 2^23, which equals 0x4B400000 + round(v * 2^21): FMA-pipe instructions
// only, no conversion instruction. Each slot also counts its additions (n), so
// its sum of patterns minus n * 0x4B400000 (mod 2^32) is the exact sum of the
// rounded values. Where sums of a few small values matter (soft binning), every
// value is split in two words, hi = round(v * 2^21) and lo = round((v * 2^21 -
// hi) * 2^21): an absolute precision of 2^-43 per value. A word takes at most
// 1023 additions between two folds (1023 * 2^21 < 2^31); the CTA folds its table
// into the workspace every `flush_tiles` tiles and at the end. The sums are
// integers, so they do not depend on the order of the additions.
//
// Layout [row][slot][R][NW] 32-bit words, NW odd: lane l updates replica l % R,
// whose NW words are contiguous, so the accumulator offsets are immediates and
// the 32 lanes of a warp hit 32 different banks whatever their bins (R = 32).
//   hard, slot = bin k (K slots), NW 3:  0 n, 1 p, 2 y (a count for labels)
//   soft, slot = interval j (K+1 slots):  0 n, 1-2 u, 3 u^2 (one word: it only
//        enters P multiplied by the span, ~1/K), then
//        labels (NW 7): 4 ny (true-class count), 5-6 u (true class);
//        dense  (NW 9): 4-5 y, 6-7 u y, 8 unused
// Interval j lies between bin centres lo = c_{j-1} and hi = c_j; there u = t =
// (p - lo) / S with the interval's span S = hi - lo is the weight of the right
// bin and 1 - t that of the left bin (ace_kernels/common.py:43-61), and p = lo +
// S t, so the bins' W, P, G follow exactly from n, sum t, sum t^2 (the last CTA's
// reconstruction below). In the two end intervals (sentinel at one side) all the
// weight goes to one end bin: there u = p, and only n, sum p (and the target
// moments) are used.
// ---------------------------------------------------------------------------
template <bool SOFT, bool LABELS>
struct Acc {
  static constexpr int NW = SOFT ? (LABELS ? 7 : 9) : 3;  // words per slot replica (odd)
  static constexpr int NOUT = SOFT ? 6 : 3;               // global sums per slot (stride)
  static constexpr int NFOLD = SOFT ? 5 : 3;              // global sums per slot (used)
  // Global sum o of a slot: its word a (and low word b, or -1), and the word that
  // counts its additions (cw; -1: the value is itself a count).
  __device__ __forceinline__ static void words(int o, int& cw, int& a, int& b) {
    if constexpr (!SOFT) {
      cw = o == 0 || (o == 2 && LABELS) ? -1 : 0;
      a = o;
      b = -1;
    } else if constexpr (LABELS) {  // words: 0 n, 1-2 u, 3 u^2, 4 ny, 5-6 u (true class)
      cw = (o == 0 || o == 3) ? -1 : (o == 4 ? 4 : 0);
      a = o == 0 ? 0 : o == 1 ? 1 : o == 2 ? 3 : o == 3 ? 4 : 5;
      b = o == 1 ? 2 : o == 4 ? 6 : -1;
    } else {  // words: 0 n, 1-2 u, 3 u^2, 4-5 y, 6-7 u y
      cw = o == 0 ? -1 : 0;
      a = o == 0 ? 0 : o == 1 ? 1 : o == 2 ? 3 : o == 3 ? 4 : 6;
      b = o == 1 ? 2 : o == 3 ? 5 : o == 4 ? 7 : -1;
    }
  }
};

constexpr float kFixMagic = 12582912.0f;         // 1.5 * 2^23
constexpr unsigned kFixMagicBits = 0x4B400000u;  // bits of kFixMagic

__device__ __forceinline__ void sadd(unsigned* h, int a, unsigned v) { atomicAdd(h + a, v); }

// Bit patterns of the hi and lo words of v * 2^21 = vs (already scaled).
__device__ __forceinline__ uint2 fix2_scaled(float vs) {
  const float hb = __fadd_rn(vs, kFixMagic);
  const float r = __fsub_rn(vs, __fsub_rn(hb, kFixMagic));  // exact residual, |r| <= 1/2
  return make_uint2(__float_as_uint(hb), __float_as_uint(__fmaf_rn(r, kFixScale, kFixMagic)));
}
// Same for a product a * b (a scaled by 2^21): one rounding for hi, exact residual.
__device__ __forceinline__ uint2 fix2_prod(float as, float b) {
  const float hb = __fmaf_rn(as, b, kFixMagic);
  const float r = __fmaf_rn(as, b, -__fsub_rn(hb, kFixMagic));
  return make_uint2(__float_as_uint(hb), __float_as_uint(__fmaf_rn(r, kFixScale, kFixMagic)));
}
__device__ __forceinline__ unsigned fix1(float v) {
  return __float_as_uint(__fmaf_rn(v, kFixScale, kFixMagic));
}

// Folds this CTA's table into the workspace and clears it. Each global sum of a
// slot (hard: n, sum p, target count or sum y; soft: n, sum u, sum u^2, target
// count or sum y, target sum u or sum u y) is taken by a group of G = 4
// consecutive lanes (1 if R < 4): each adds R / G of the replicas exactly in
// 64-bit integers, in an order rotated by the slot (spreading a warp's reads over
// the banks), the group adds its parts with shuffles and its first lane issues
// one fp64 atomic add; then the table is zeroed. A fixed-point word w with cnt
// additions holds the exact value (int)(w - cnt * 0x4B400000); count words hold
// their value. The word selection is branch-free, so the lanes of a warp, which
// take different sums, do not diverge. Called by all threads between barriers.
template <class L>
__device__ __forceinline__ void fold_table(unsigned* hist, int CL, int slots, int R,
                                           double* accum, int64_t out_stride, int64_t row0) {
  constexpr int NW = L::NW;
  constexpr int NF = L::NFOLD;
  const int G = R >= 4 ? 4 : 1;
  const int per = R / G;
  const double unit = 1.0 / (double)kFixScale;
  const int total = CL * slots * NF * G;
  for (int i0 = 0; i0 < total; i0 += blockDim.x) {  // uniform trip count: full-warp shuffles
    const int i = i0 + threadIdx.x;
    const bool valid = i < total;
    const int out = valid ? i / G : 0, part = i - (i / G) * G;
    const int e = out / NF, o = out - e * NF;
    // cw: word counting the value's additions (-1: the value is a count); a, b:
    // its words (b < 0: one word)
    int cw, a, b;
    L::words(o, cw, a, b);
    const unsigned mul = cw < 0 ? 0u : kFixMagicBits;
    const int cwi = cw < 0 ? a : cw, bi = b < 0 ? a : b;
    const long long hs = b < 0 ? 1ll : (long long)kFixScale;
    const unsigned* base = hist + (int64_t)e * R * NW;
    long long acc = 0;
    if (valid) {
      for (int k = 0; k < per; ++k) {
        const unsigned* w = base + ((part * per + k + e) & (R - 1)) * NW;
        const unsigned offv = w[cwi] * mul;
        const long long hi = cw < 0 ? (long long)w[a] : (long long)(int)(w[a] - offv);
        const long long lo = b < 0 ? 0ll : (long long)(int)(w[bi] - offv);
        acc += hi * hs + lo;
      }
    }
    if (G == 4) {
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    }
    if (valid && part == 0 && acc != 0) {
      const double scale = cw < 0 ? 1.0 : (b >= 0 ? unit * unit : unit);
      const int row = e / slots, slot = e - row * slots;
      atomicAdd(accum + o * out_stride + (row0 + row) * slots + slot, (double)acc * scale);
    }
  }
  __syncthreads();
  const int words = CL * slots * R * NW;
  uint4* h4 = reinterpret_cast<uint4*>(hist);
  for (int i = threadIdx.x; i < words / 4; i += blockDim.x) h4[i] = make_uint4(0u, 0u, 0u, 0u);
  for (int i = (words & ~3) + threadIdx.x; i < words; i += blockDim.x) hist[i] = 0u;
}

// Channel count of a kernel instance: exact for softmax instances with CM <= 4
// (the loops then have no per-channel guard), else the runtime value (CM is a
// capacity, or 1 for the pointwise activations that loop over channels).
template <int CM, bool SOFTMAX>
__device__ __forceinline__ int channels(int runtime_c) {
  return (SOFTMAX && CM <= 4) ? CM : runtime_c;
}

// Tiles [g0, g1) of CTA blockIdx.x (see the forward's comment).
__device__ __forceinline__ void chunk_range(const Grid& G, int64_t& g0, int64_t& g1) {
  const int64_t tpc = G.tiles_per_chunk;
  if (G.chunks_per_batch > 0) {
    const int cb = G.chunks_per_batch;
    const int bx = (int)blockIdx.x / cb;
    g0 = bx * G.tiles + (int64_t)((int)blockIdx.x - bx * cb) * tpc;
    g1 = min(g0 + tpc, (bx + 1) * G.tiles);
  } else {
    g0 = (int64_t)blockIdx.x * tpc;
    g1 = min(g0 + tpc, (int64_t)G.B * G.tiles);
  }
}

// ---------------------------------------------------------------------------
// Forward: fused activation + W/P/G statistics (+ epilogue in the last CTA).
//
// Tiles of kHistThreads * V voxels are numbered over all batches (tile g is tile
// g % tpb of batch g / tpb); a 1-D grid of one wave, CTA x streams tiles
// [g0, g1): chunk x % cb of batch x / cb when the host chose chunks_per_batch =
// cb > 0, else run x of the whole sequence, which may cross into the next batch
// (the CTA then folds its table before it takes the next batch's rows). Thread t
// owns V consecutive voxels of a tile, read with 16-byte (V * sizeof(T))
// coalesced loads per channel (the channel stride is N). The logits of all C
// channels of a voxel are in registers, so the softmax needs no second read. Per
// voxel the bins of all loss channels are located first (one shared-memory load
// each, straight-line), then the table updates are issued; the true class's
// target updates are issued once per voxel. The last CTA to finish (a ticket in
// the workspace, no waiting) turns the workspace sums into W, P, G, resets the
// workspace and runs the epilogue.
// ---------------------------------------------------------------------------
template <typename T, int V, int CM, bool SOFTMAX, bool SOFT, bool LABELS>
__global__ void __launch_bounds__(kHistThreads) hist_kernel(const __grid_constant__ FwdParams P) {
  constexpr int NW = Acc<SOFT, LABELS>::NW;
  constexpr int NOUT = Acc<SOFT, LABELS>::NOUT;
  extern __shared__ __align__(16) float smem[];
  const int tid = threadIdx.x;
  const int C = channels<CM, SOFTMAX>(P.g.C), CL = P.g.CL, off = P.g.offset, K = P.tab.K;
  const int slots = SOFT ? K + 1 : K;
  const int64_t N = P.g.N;
  const int R = P.R;
  const float Kf = (float)K;

  // Bin tables in kTabCopies interleaved copies (lane l reads copy l % 16, so a
  // warp's random-index gather is bank-conflict-free), then the statistics.
  float2* lohi_t = reinterpret_cast<float2*>(smem);
  float2* map_t = lohi_t + (K + 1) * kTabCopies;
  unsigned* hist = reinterpret_cast<unsigned*>(map_t + (K + 1) * kTabCopies);
  const int table_words = CL * slots * R * NW;
  for (int i = tid; i < (K + 1) * kTabCopies; i += kHistThreads) {
    lohi_t[i] = P.tab.lohi[i / kTabCopies];
    map_t[i] = P.tab.map[i / kTabCopies];
  }
  const float2* my_lohi = lohi_t + (tid & (kTabCopies - 1));
  const float2* my_map = map_t + (tid & (kTabCopies - 1));
  {
    uint4* h4 = reinterpret_cast<uint4*>(hist);  // 16-byte aligned: (K + 1) * 256 bytes in
    for (int i = tid; i < table_words / 4; i += kHistThreads) h4[i] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = (table_words & ~3) + tid; i < table_words; i += kHistThreads) hist[i] = 0u;
  }
  // Launched with programmatic dependent launch: the setup above (parameters
  // and shared memory only) overlaps the previous kernel's tail; no global
  // memory is touched before the previous grid has completed.
  ace_grid_dependency_wait();
  __syncthreads();

  const int col = (tid & (R - 1)) * NW;
  const int slot_stride = R * NW, row_stride = slots * slot_stride;
  const int64_t out_stride = (int64_t)P.B_total * CL * slots;

  const int64_t tpb = P.g.tiles > 0 ? P.g.tiles : 1;  // (no tiles at all when N = 0)
  int64_t g0, g1;
  chunk_range(P.g, g0, g1);
  auto x_of = [&](int bb) { return static_cast<const T*>(P.x) + (int64_t)bb * C * N; };
  auto lab_of = [&](int bb) {
    return LABELS ? static_cast<const int64_t*>(P.target) + (int64_t)bb * N : nullptr;
  };
  auto y_of = [&](int bb) {
    return LABELS ? nullptr : static_cast<const float*>(P.target) + (int64_t)bb * C * N;
  };

  // One loss-channel value into the table, with its target: y (dense) or
  // whether this channel is the voxel's class (labels; the soft softmax path
  // passes false and adds the true class once per voxel with true_update).
  // Returns the soft fixed-point words of u.
  auto update = [&](int row, float p, int j, float4 q, float y, bool is_true) -> uint2 {
    if constexpr (!SOFT) {
      if (j < K) {  // p above the last edge (only for invalid p > 1 + eps) is dropped
        const int a = row * row_stride + j * slot_stride + col;
        sadd(hist, a, 1u);
        sadd(hist, a + 1, fix1(p));
        if constexpr (LABELS) {
          if (is_true) sadd(hist, a + 2, 1u);
        } else {
          sadd(hist, a + 2, fix1(y));
        }
      }
      return make_uint2(0u, 0u);
    } else {
      // u * 2^21, u = (p - lo) / S inside, u = p in the end intervals
      const float us = fminf(ACE_FMUL(ACE_FSUB(p, q.z), q.w), kFixScale);
      const int a = row * row_stride + j * slot_stride + col;
      sadd(hist, a, 1u);
      const uint2 uw = fix2_scaled(us);
      sadd(hist, a + 1, uw.x);
      sadd(hist, a + 2, uw.y);
      sadd(hist, a + 3, __float_as_uint(__fmaf_rn(us, ACE_FMUL(us, 1.0f / kFixScale), kFixMagic)));
      if constexpr (LABELS) {
        if (is_true) {
          sadd(hist, a + 4, 1u);
          sadd(hist, a + 5, uw.x);
          sadd(hist, a + 6, uw.y);
        }
      } else {
        const uint2 yw = fix2_prod(kFixScale, y);
        sadd(hist, a + 4, yw.x);
        sadd(hist, a + 5, yw.y);
        const uint2 uyw = fix2_prod(us, y);
        sadd(hist, a + 6, uyw.x);
        sadd(hist, a + 7, uyw.y);
      }
      return uw;
    }
  };
  // The voxel's class (labels): its count (and soft: its u words) in its row.
  auto true_update = [&](int row, int j, uint2 uw) {
    const int a = row * row_stride + j * slot_stride + col;
    if constexpr (!SOFT) {
      if (j < K) sadd(hist, a + 2, 1u);
    } else {
      sadd(hist, a + 4, 1u);
      sadd(hist, a + 5, uw.x);
      sadd(hist, a + 6, uw.y);
    }
  };
  // Table entry of count j: neighbours and, for soft binning, base / scale.
  auto entry = [&](int j) -> float4 {
    const float2 lh = my_lohi[j * kTabCopies];
    if constexpr (SOFT) {
      const float2 m = my_map[j * kTabCopies];
      return make_float4(lh.x, lh.y, m.x, m.y);
    } else {
      return make_float4(lh.x, lh.y, 0.0f, 0.0f);
    }
  };

  // Soft binning, softmax path: the count is the rounded p * K clamped to
  // [0, K], without the exact test. It can be one off only for p within a few
  // ulps of a bin centre, where both candidate intervals give the centre's bin a
  // weight of ~1 (t ~ 1 in the lower interval, t ~ 0 in the upper one), so the
  // sums differ by ulps; t may then be a few ulps below 0, or is clamped at 1.
  // (The gradient kernel keeps the exact interval: the derivative of the weights
  // jumps at a centre.) Only base / scale are read.
  auto soft_entry = [&](float p, int& j) -> float4 {
    int i = (int)(__float_as_uint(__fadd_rn(__fmul_rn(p, Kf), kFixMagic)) - kFixMagicBits);
    i = max(0, min(i, K));
    j = i;
    const float2 m = my_map[i * kTabCopies];
    return make_float4(0.0f, 0.0f, m.x, m.y);
  };

  int since_fold = 0;
  const int64_t tile = (int64_t)kHistThreads * V;
  // L2 prefetch of the next tile (one thread per channel row and one for the
  // labels), so the loads of the next iteration hit L2 instead of HBM
  const bool pf_x = ((reinterpret_cast<uintptr_t>(P.x) | (N * sizeof(T))) & 15) == 0;
  int b = (int)(g0 / tpb);   // batch of tile g
  int64_t t = g0 - b * tpb;  // its tile within the batch
  const T* xb = x_of(b);
  const int64_t* lb = lab_of(b);
  const float* yb = y_of(b);
  int64_t row0 = (int64_t)(P.b_offset + b) * CL;
  for (int64_t g = g0; g < g1; ++g, ++t) {
    if (t == tpb) {  // next batch: fold this batch's rows first
      __syncthreads();
      fold_table<Acc<SOFT, LABELS>>(hist, CL, slots, R, P.accum, out_stride, row0);
      __syncthreads();
      since_fold = 0;
      ++b;
      t = 0;
      xb = x_of(b);
      lb = lab_of(b);
      yb = y_of(b);
      row0 = (int64_t)(P.b_offset + b) * CL;
    }
    if (t + 1 < tpb && g + 1 < g1 && pf_x) {
      if (tid < C) ace_prefetch_tile(xb + (int64_t)tid * N, (t + 1) * tile, tile, N, sizeof(T));
      if constexpr (LABELS) {
        if (tid == C) ace_prefetch_tile(lb, (t + 1) * tile, tile, N, 8);
      }
    }
    const int64_t v0 = (t * kHistThreads + tid) * V;
    if (v0 < N) {  // V > 1 implies N % V == 0: groups are whole
      int lab[V];
      if constexpr (LABELS) ace_load_labels<V>(lb + v0, lab);
      if constexpr (SOFTMAX && CM > 4) {
        // Many channels: three passes over the channels, so that only per-voxel
        // scalars live in registers (the reloads hit L1 / L2): the maximum, the
        // sum of exponentials (ascending channels), then each probability,
        // computed as in ace_softmax (same operations, same result), is binned
        // and added.
        const T* xr = xb + v0;
        float m[V], sm[V], rc[V];
        VecIO<T, V>::load(xr, m);
#pragma unroll 4
        for (int c = 1; c < C; ++c) {
          float x[V];
          VecIO<T, V>::load(xr + (int64_t)c * N, x);
#pragma unroll
          for (int i = 0; i < V; ++i) m[i] = fmaxf(m[i], x[i]);
        }
#pragma unroll
        for (int i = 0; i < V; ++i) sm[i] = 0.0f;
#pragma unroll 4
        for (int c = 0; c < C; ++c) {
          float x[V];
          VecIO<T, V>::load(xr + (int64_t)c * N, x);
#pragma unroll
          for (int i = 0; i < V; ++i) sm[i] = ACE_FADD(sm[i], expf(ACE_FSUB(x[i], m[i])));
        }
#pragma unroll
        for (int i = 0; i < V; ++i) rc[i] = ace_rcp_refined(sm[i]);
#pragma unroll 2
        for (int c = off; c < C; ++c) {
          float x[V], yv[V];
          VecIO<T, V>::load(xr + (int64_t)c * N, x);
          if constexpr (!LABELS) VecIO<float, V>::load(yb + (int64_t)c * N + v0, yv);
#pragma unroll
          for (int i = 0; i < V; ++i) {
            const float p = ace_div_corrected(expf(ACE_FSUB(x[i], m[i])), sm[i], rc[i]);
            int j;
            float4 q;
            if constexpr (SOFT) {
              q = soft_entry(p, j);
            } else {
              float2 lh;
              j = ace_locate(p, my_lohi, kTabCopies, K, Kf, false, lh);
              q = make_float4(lh.x, lh.y, 0.0f, 0.0f);
            }
            float y = 0.0f;
            if constexpr (!LABELS) y = yv[i];
            const bool is_true = LABELS && lab[i] == c;
            const uint2 w = update(c - off, p, j, q, y, !SOFT && is_true);
            if constexpr (SOFT && LABELS) {
              if (is_true) true_update(c - off, j, w);
            }
          }
        }
      } else if constexpr (SOFTMAX) {
        float xv[CM][V];
#pragma unroll
        for (int c = 0; c < CM; ++c)
          if (c < C) VecIO<T, V>::load(xb + (int64_t)c * N + v0, xv[c]);
        float yv[CM][V];
        if constexpr (!LABELS) {
#pragma unroll
          for (int c = 0; c < CM; ++c)
            if ((c > 0 || off == 0) && c < C) VecIO<float, V>::load(yb + (int64_t)c * N + v0, yv[c]);
        }
#pragma unroll
        for (int i = 0; i < V; ++i) {
          float p[CM];
#pragma unroll
          for (int c = 0; c < CM; ++c) p[c] = xv[c][i];
          ace_softmax<CM>(p, C);
          int j[CM];
          float4 q[CM];
          if constexpr (SOFT) {
#pragma unroll
            for (int c = 0; c < CM; ++c)
              if ((c > 0 || off == 0) && c < C) q[c] = soft_entry(p[c], j[c]);
          } else {
            bool ok = true;
#pragma unroll
            for (int c = 0; c < CM; ++c) {
              if ((c > 0 || off == 0) && c < C) {
                j[c] = ace_guess(p[c], Kf, K, SOFT);
                q[c] = entry(j[c]);
                ok &= ace_is_count(p[c], make_float2(q[c].x, q[c].y));
              }
            }
            if (!ok) {
#pragma unroll
              for (int c = 0; c < CM; ++c)
                if ((c > 0 || off == 0) && c < C &&
                    !ace_is_count(p[c], make_float2(q[c].x, q[c].y))) {
                  j[c] = ace_fix_count(p[c], j[c], K, my_lohi, kTabCopies).i;
                  q[c] = entry(j[c]);
                }
            }
          }
          uint2 uw[CM];
#pragma unroll
          for (int c = 0; c < CM; ++c) {
            if ((c > 0 || off == 0) && c < C) {
              float y = 0.0f;
              if constexpr (!LABELS) y = yv[c][i];
              // hard: the class's count as one predicated add per channel
              uw[c] = update(c - off, p[c], j[c], q[c], y, !SOFT && LABELS && lab[i] == c);
            }
          }
          if constexpr (SOFT && LABELS) {
            // the voxel's class, if it is a loss channel: its bin and u words
            const int lt = lab[i];
            int jt = 0;
            uint2 wt = make_uint2(0u, 0u);
#pragma unroll
            for (int c = 0; c < CM; ++c) {
              if ((c > 0 || off == 0) && c < C && lt == c) {
                jt = j[c];
                wt = uw[c];
              }
            }
            if (lt >= off && lt < C) true_update(lt - off, jt, wt);
          }
        }
      } else {
        // none / sigmoid: channels are independent, one at a time
        for (int c = off; c < C; ++c) {
          float xv[V];
          VecIO<T, V>::load(xb + (int64_t)c * N + v0, xv);
          float yv[V];
          if constexpr (!LABELS) VecIO<float, V>::load(yb + (int64_t)c * N + v0, yv);
#pragma unroll
          for (int i = 0; i < V; ++i) {
            const float p = P.act == ACE_B200_ACT_SIGMOID ? ace_sigmoid(xv[i]) : xv[i];
            float2 lh;
            const int j = ace_locate(p, my_lohi, kTabCopies, K, Kf, SOFT, lh);
            float y = 0.0f;
            if constexpr (!LABELS) y = yv[i];
            update(c - off, p, j, entry(j), y, LABELS && lab[i] == c);
          }
        }
      }
    }
    if (++since_fold == P.flush_tiles && g + 1 < g1) {
      since_fold = 0;
      __syncthreads();
      fold_table<Acc<SOFT, LABELS>>(hist, CL, slots, R, P.accum, out_stride, row0);
      __syncthreads();
    }
  }
  ace_launch_dependents();  // a dependent launch may begin its own setup now
  __syncthreads();
  fold_table<Acc<SOFT, LABELS>>(hist, CL, slots, R, P.accum, out_stride, row0);
  __syncthreads();
  __shared__ bool s_last;
  if (tid == 0) {
    // The ticket is a release (this CTA's sums, ordered before it by the
    // barrier) and an acquire (the other CTAs' sums, for the last CTA).
    unsigned done;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                 : "=r"(done)
                 : "l"(P.counter)
                 : "memory");
    s_last = (done == gridDim.x * gridDim.y - 1);
  }
  __syncthreads();
  if (!s_last) return;

  // Last CTA: the workspace sums become W, P, G per bin. Hard: slot = bin. Soft:
  // interval j in 1..K-1 (between lo and hi = lo + S) gives bin j its t share,
  //   W += sum t,  P += lo sum t + S sum t^2,  G += target sum t,
  // and bin j-1 its 1 - t share,
  //   W += n - sum t,  P += lo (n - sum t) + S (sum t - sum t^2),  G += ny - target sum t;
  // intervals 0 and K give all of n, sum p, ny to bins 0 and K-1 (both
  // neighbours are the end bin there), as the reference's two scatters.
  const int rows = P.B_total * CL;
  const int64_t stat_stride = (int64_t)rows * K;
  const bool stage = P.do_epilogue && 3 * stat_stride <= (int64_t)table_words;
  float* staged = reinterpret_cast<float*>(hist);
  const double* acc = P.accum;
  for (int64_t e = tid; e < stat_stride; e += kHistThreads) {
    const int64_t r = e / K;
    const int k = (int)(e - r * K);
    double w, pp, g;
    if constexpr (!SOFT) {
      const int64_t gi = r * slots + k;
      w = __ldcg(acc + gi);
      pp = __ldcg(acc + out_stride + gi);
      g = __ldcg(acc + 2 * out_stride + gi);
    } else {
      w = pp = g = 0.0;
      // j = k: the t share of interval k (all of it if k == 0)
      // j = k + 1: the 1 - t share of interval k + 1 (all of it if k + 1 == K)
      for (int side = 0; side < 2; ++side) {
        const int j = k + side;
        const int64_t gi = r * slots + j;
        const double n = __ldcg(acc + gi), su = __ldcg(acc + out_stride + gi);
        const double ny = __ldcg(acc + 3 * out_stride + gi);
        const double yu = __ldcg(acc + 4 * out_stride + gi);
        if (j == 0 || j == K) {
          w += n;
          pp += su;
          g += ny;
          continue;
        }
        const double lo = P.tab.lohi[j].x, span = (double)P.tab.lohi[j].y - lo;
        const double su2 = __ldcg(acc + 2 * out_stride + gi);
        const double pt = lo * su + span * su2;  // sum t p
        if (side == 0) {
          w += su;
          pp += pt;
          g += yu;
        } else {
          w += n - su;
          pp += lo * n + span * su - pt;
          g += ny - yu;
        }
      }
    }
    const float wf = (float)w, pf = (float)pp, gf = (float)g;
    P.hist_out[e] = wf;
    P.hist_out[stat_stride + e] = pf;
    P.hist_out[2 * stat_stride + e] = gf;
    if (stage) {
      staged[e] = wf;
      staged[stat_stride + e] = pf;
      staged[2 * stat_stride + e] = gf;
    }
  }
  __syncthreads();
  double* accw = P.accum;
  for (int64_t i = tid; i < NOUT * out_stride; i += kHistThreads) __stcg(accw + i, 0.0);
  if (tid == 0) *P.counter = 0u;
  if (stage) {
    __syncthreads();
    write_loss_if0(P.epi, epilogue_rows(P.epi, staged, rows, 0, 0, rows));
  }
}

}  // namespace ace

#include "ace_tma.cuh"       // pipeline primitives
#include "ace_xchg.cuh"      // statistics exchange between ranks (multi-rank forwards)
#include "ace_soft_fwd.cuh"  // soft_fwd_kernel (uses the helpers above)
#include "ace_mc_fwd.cuh"    // mc_fwd_kernel (uses soft_fwd_kernel's pipeline)

namespace ace {

// ---------------------------------------------------------------------------
// Backward: d loss / d x in one pass (ace_kernels/impls/v2_autograd.py:88-118,
// derivation in the reference's docs/derivation.md):
//   hard: gp_c = g_bc * coef[b, c, bin(p_c)]
//   soft: gp_c = g_bc * (coef_l (lw - (p - y - d_l) / S) + coef_r (rw + (p - y - d_r) / S))
//   softmax: dx_c = p_c (gp_c - sum_c' p_c' gp_c'); sigmoid: gp p (1 - p); none: gp
// with gp = 0 on a dropped background channel. The activation and the bins are
// recomputed (hard binning: with the forward's code, so the same bins). Per CTA,
// the rows of its batch sit in shared memory with g folded in: hard, cg[row][k] =
// g coef (0 past the last bin); soft, one record {F, D} per row and interval j.
// Inside interval j (centres lo = c_{j-1}, hi = c_j, S = hi - lo, inv = 1 / S) the
// weights are rw = (p - lo) inv and lw = 1 - rw, so with A = g coef_l,
// B = g coef_r the soft formula is affine in p and y:
//   gp = A + (B - A) inv (p - lo) + (B - A) inv (p - y) + inv (A d_l - B d_r)
//      = F + D (2 p - y),  D = (B - A) inv,  F = A - D lo + inv (A d_l - B d_r).
// In the two end intervals both sides are the same bin: D = 0, F = g coef. The
// records are built in double precision and rounded once; one 8-byte load and
// two FMAs per value remain. Hard binning reads no targets.
// ---------------------------------------------------------------------------
template <bool SOFT>
__device__ __forceinline__ float grad_p(const float* __restrict__ tab, int copies, int row, int K,
                                        int j, float p, float y) {
  // `tab` points at this lane's copy; entries are `copies` apart.
  if constexpr (!SOFT) {
    return tab[(row * (K + 1) + j) * copies];
  } else {
    const float2 rec = reinterpret_cast<const float2*>(tab)[(row * (K + 1) + j) * copies];
    return __fmaf_rn(rec.y, __fmaf_rn(2.0f, p, -y), rec.x);
  }
}

template <typename T, int V, int CM, bool SOFTMAX, bool SOFT, bool LABELS>
__global__ void __launch_bounds__(kThreads) grad_kernel(const __grid_constant__ BwdParams P) {
  extern __shared__ __align__(16) float smem[];
  const int tid = threadIdx.x;
  const int b = blockIdx.y;
  const int C = channels<CM, SOFTMAX>(P.g.C), CL = P.g.CL, off = P.g.offset, K = P.tab.K;
  const int64_t N = P.g.N;
  const float Kf = (float)K;

  // Tables in interleaved copies so that the lanes of one load phase rarely share
  // banks (random-index gathers): the bin table in kTabCopies copies, the per-row
  // soft records in up to 16 copies (8-byte records, 16 lanes a phase) or the
  // hard g coef table in up to 32 copies (4-byte values, 32 lanes a phase); the
  // host lowers P.rec_copies (a power of two) when many rows would not fit.
  float* tab = smem;  // [CL][K+1][copies] floats (hard) or float2 (soft)
  const int rec_copies = P.rec_copies;
  float2* lohi_t = reinterpret_cast<float2*>(tab + (SOFT ? 2 : 1) * CL * (K + 1) * rec_copies);
  // many channels: per-thread gp of every channel, [c][thread][V] (fp32)
  float* gscratch = reinterpret_cast<float*>(lohi_t + (K + 1) * kTabCopies);
  for (int i = tid; i < (K + 1) * kTabCopies; i += kThreads) lohi_t[i] = P.tab.lohi[i / kTabCopies];
  // programmatic dependent launch: global memory only after the previous grid
  ace_grid_dependency_wait();
  const int64_t row0 = (int64_t)(P.b_offset + b) * CL;
  // One thread per (row, j) record; it writes all the record's copies (16-byte
  // stores: rec_copies * record bytes is a multiple of 16).
  for (int e = tid; e < CL * (K + 1); e += kThreads) {
    const int row = e / (K + 1), j = e - row * (K + 1);
    const float g = P.jac[row0 + row] * (P.grad_per_row ? P.grad_out[row0 + row] : P.grad_out[0]);
    const float* cf = P.coef + (row0 + row) * K;
    const float* dd = P.d + (row0 + row) * K;
    uint4 v;
    if constexpr (!SOFT) {
      const unsigned u = __float_as_uint(j < K ? g * cf[j] : 0.0f);
      v = make_uint4(u, u, u, u);
    } else {
      const int l = max(j - 1, 0), r = min(j, K - 1);
      const float a = g * cf[l], bb = g * cf[r];
      float2 rec = make_float2(a, 0.0f);
      if (j > 0 && j < K) {
        const double lo = P.tab.map[j].x, inv = (double)P.tab.map[j].y / (double)kFixScale;
        const double dd_ = ((double)bb - (double)a) * inv;
        const double e_ = inv * ((double)a * dd[l] - (double)bb * dd[r]);
        rec = make_float2((float)((double)a - dd_ * lo + e_), (float)dd_);
      }
      v = make_uint4(__float_as_uint(rec.x), __float_as_uint(rec.y), __float_as_uint(rec.x),
                     __float_as_uint(rec.y));
    }
    uint4* dst = reinterpret_cast<uint4*>(tab + (SOFT ? 2 : 1) * e * rec_copies);
    for (int q = 0; q < (SOFT ? 2 : 1) * rec_copies / 4; ++q) dst[q] = v;
  }
  __syncthreads();
  const float* my_tab = tab + (SOFT ? 2 : 1) * (tid & (rec_copies - 1));
  const float2* my_lohi = lohi_t + (tid & (kTabCopies - 1));

  auto entry = [&](int j) -> float2 { return my_lohi[j * kTabCopies]; };
  // Many-channel passes: one value's exponential and probability, the same
  // operations as ace_softmax_sel (fast for soft binning, exact for hard).
  auto expf_c = [](float x, float m) -> float {
    if constexpr (SOFT) return ace_exp_fast(x, ACE_FMUL(m, kLog2e));
    else return expf(ACE_FSUB(x, m));
  };
  auto prob_c = [](float e, float s, float r) -> float {
    if constexpr (SOFT) return ACE_FMUL(e, r);
    else return ace_div_corrected(e, s, r);
  };

  const T* xb = static_cast<const T*>(P.x) + (int64_t)b * C * N;
  T* db = static_cast<T*>(P.dx) + (int64_t)b * C * N;
  const int64_t* lb = (SOFT && LABELS) ? static_cast<const int64_t*>(P.target) + (int64_t)b * N : nullptr;
  const float* yb = (SOFT && !LABELS) ? static_cast<const float*>(P.target) + (int64_t)b * C * N : nullptr;

  const int64_t t0 = (int64_t)blockIdx.x * P.g.tiles_per_chunk;
  const int64_t t1 = min(t0 + P.g.tiles_per_chunk, P.g.tiles);
  const int64_t tile = (int64_t)kThreads * V;
  const bool pf_x = ((reinterpret_cast<uintptr_t>(xb) | (N * sizeof(T))) & 15) == 0;
  for (int64_t t = t0; t < t1; ++t) {
    if (t + 1 < t1 && pf_x) {  // L2 prefetch of the next tile
      if (tid < C) ace_prefetch_tile(xb + (int64_t)tid * N, (t + 1) * tile, tile, N, sizeof(T));
      if constexpr (SOFT && LABELS) {
        if (tid == C) ace_prefetch_tile(lb, (t + 1) * tile, tile, N, 8);
      }
    }
    const int64_t v0 = (t * kThreads + tid) * V;
    if (v0 >= N) continue;
    int lab[V];
    if constexpr (SOFT && LABELS) ace_load_labels<V>(lb + v0, lab);
    if constexpr (SOFTMAX && CM > 4) {
      // Many channels, in passes as the forward: maximum, sum of exponentials,
      // then p and gp per channel (gp kept in shared memory, the dot product in
      // registers), then dx = p (gp - dot); only per-voxel scalars in registers.
      const T* xr = xb + v0;
      float m[V], sm[V], rc[V], dot[V];
      VecIO<T, V>::load(xr, m);
#pragma unroll 4
      for (int c = 1; c < C; ++c) {
        float x[V];
        VecIO<T, V>::load(xr + (int64_t)c * N, x);
#pragma unroll
        for (int i = 0; i < V; ++i) m[i] = fmaxf(m[i], x[i]);
      }
#pragma unroll
      for (int i = 0; i < V; ++i) sm[i] = 0.0f;
#pragma unroll 4
      for (int c = 0; c < C; ++c) {
        float x[V];
        VecIO<T, V>::load(xr + (int64_t)c * N, x);
#pragma unroll
        for (int i = 0; i < V; ++i) sm[i] = ACE_FADD(sm[i], expf_c(x[i], m[i]));
      }
#pragma unroll
      for (int i = 0; i < V; ++i) {
        rc[i] = SOFT ? ace_rcp_approx(sm[i]) : ace_rcp_refined(sm[i]);
        dot[i] = 0.0f;
      }
      float* gs = gscratch + tid * V;
      const int gstride = kThreads * V;
#pragma unroll 2
      for (int c = 0; c < C; ++c) {
        float x[V], yv[V];
        VecIO<T, V>::load(xr + (int64_t)c * N, x);
        if constexpr (SOFT && !LABELS) {
          if (c >= off) VecIO<float, V>::load(yb + (int64_t)c * N + v0, yv);
        }
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const float p = prob_c(expf_c(x[i], m[i]), sm[i], rc[i]);
          float gp = 0.0f;
          if (c >= off) {
            float2 lh;
            const int jc = ace_locate(p, my_lohi, kTabCopies, K, Kf, SOFT, lh);
            float y = 0.0f;
            if constexpr (SOFT && LABELS) y = (lab[i] == c) ? 1.0f : 0.0f;
            if constexpr (SOFT && !LABELS) y = yv[i];
            gp = grad_p<SOFT>(my_tab, rec_copies, c - off, K, jc, p, y);
          }
          dot[i] += p * gp;
          gs[c * gstride + i] = gp;
        }
      }
#pragma unroll 2
      for (int c = 0; c < C; ++c) {
        float x[V], o[V];
        VecIO<T, V>::load(xr + (int64_t)c * N, x);
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const float p = prob_c(expf_c(x[i], m[i]), sm[i], rc[i]);
          o[i] = p * (gs[c * gstride + i] - dot[i]);
        }
        VecIO<T, V>::store(db + (int64_t)c * N + v0, o);
      }
    } else if constexpr (SOFTMAX) {
      float xv[CM][V];
#pragma unroll
      for (int c = 0; c < CM; ++c)
        if (c < C) VecIO<T, V>::load(xb + (int64_t)c * N + v0, xv[c]);
      float yv[CM][V];
      if constexpr (SOFT && !LABELS) {
#pragma unroll
        for (int c = 0; c < CM; ++c)
          if ((c > 0 || off == 0) && c < C) VecIO<float, V>::load(yb + (int64_t)c * N + v0, yv[c]);
      }
#pragma unroll
      for (int i = 0; i < V; ++i) {
        float p[CM];
#pragma unroll
        for (int c = 0; c < CM; ++c) p[c] = xv[c][i];
        ace_softmax_sel<SOFT, CM>(p, C);
        float gp[CM];
        float dot = 0.0f;
        int j[CM];
        bool ok = true;
#pragma unroll
        for (int c = 0; c < CM; ++c) {
          if ((c > 0 || off == 0) && c < C) {
            j[c] = ace_guess(p[c], Kf, K, SOFT);
            ok &= ace_is_count(p[c], entry(j[c]));
          }
        }
        if (!ok) {
#pragma unroll
          for (int c = 0; c < CM; ++c)
            if ((c > 0 || off == 0) && c < C && !ace_is_count(p[c], entry(j[c])))
              j[c] = ace_fix_count(p[c], j[c], K, my_lohi, kTabCopies).i;
        }
#pragma unroll
        for (int c = 0; c < CM; ++c) {
          gp[c] = 0.0f;
          if (c < C) {
            if (c > 0 || off == 0) {
              float y = 0.0f;
              if constexpr (SOFT && LABELS) y = (lab[i] == c) ? 1.0f : 0.0f;
              if constexpr (SOFT && !LABELS) y = yv[c][i];
              gp[c] = grad_p<SOFT>(my_tab, rec_copies, c - off, K, j[c], p[c], y);
            }
            dot += p[c] * gp[c];
          }
        }
#pragma unroll
        for (int c = 0; c < CM; ++c)
          if (c < C) xv[c][i] = p[c] * (gp[c] - dot);
      }
#pragma unroll
      for (int c = 0; c < CM; ++c)
        if (c < C) VecIO<T, V>::store(db + (int64_t)c * N + v0, xv[c]);
    } else {
      for (int c = 0; c < C; ++c) {
        float xv[V];
        if (c < off) {
#pragma unroll
          for (int i = 0; i < V; ++i) xv[i] = 0.0f;
          VecIO<T, V>::store(db + (int64_t)c * N + v0, xv);
          continue;
        }
        VecIO<T, V>::load(xb + (int64_t)c * N + v0, xv);
        float yv[V];
        if constexpr (SOFT && !LABELS) VecIO<float, V>::load(yb + (int64_t)c * N + v0, yv);
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const bool sig = P.act == ACE_B200_ACT_SIGMOID;
          const float p = sig ? ace_sigmoid(xv[i]) : xv[i];
          float y = 0.0f;
          if constexpr (SOFT && LABELS) y = (lab[i] == c) ? 1.0f : 0.0f;
          if constexpr (SOFT && !LABELS) y = yv[i];
          float2 lh;
          const int j = ace_locate(p, my_lohi, kTabCopies, K, Kf, SOFT, lh);
          const float gp = grad_p<SOFT>(my_tab, rec_copies, c - off, K, j, p, y);
          xv[i] = sig ? gp * p * (1.0f - p) : gp;
        }
        VecIO<T, V>::store(db + (int64_t)c * N + v0, xv);
      }
    }
  }
}

}  // namespace ace

#include "ace_grad_tma.cuh"  // grad_tma_kernel (uses grad_p above)
#include "ace_mc_grad.cuh"   // mc_grad_kernel (grad_tma_kernel's pipeline, mc_fwd_kernel's math)

namespace ace {

// ---------------------------------------------------------------------------
// Test hook: the activated probabilities, computed by the same functions as the
// two kernels above.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads) probs_kernel(const T* __restrict__ x,
                                                         float* __restrict__ out, int64_t B,
                                                         int C, int64_t N, int act) {
  const int64_t total = B * N;
  for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * kThreads) {
    const int64_t b = i / N, n = i - b * N;
    const T* xp = x + b * C * N + n;
    float* op = out + b * C * N + n;
    if (act == ACE_B200_ACT_SOFTMAX && C > 1) {
      float e[kMaxClasses];
#pragma unroll
      for (int c = 0; c < kMaxClasses; ++c) e[c] = c < C ? ace_to_float<T>(xp[(int64_t)c * N]) : 0.0f;
      ace_softmax<kMaxClasses>(e, C);
#pragma unroll
      for (int c = 0; c < kMaxClasses; ++c)
        if (c < C) op[(int64_t)c * N] = e[c];
    } else {
      for (int c = 0; c < C; ++c) {
        const float v = ace_to_float<T>(xp[(int64_t)c * N]);
        op[(int64_t)c * N] = act == ACE_B200_ACT_SIGMOID ? ace_sigmoid(v) : v;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Host-side dispatch from a runtime Variant to a template instance.
// ---------------------------------------------------------------------------
// The launchers live in an unnamed namespace: their "already opted in" state is
// then private to the translation unit that launches the kernels (a static local
// of an exported template would be merged with any other loaded copy of the
// library and could skip the opt-in).
namespace {

// Launch with programmatic stream serialization (programmatic dependent launch):
// the kernel may start while the previous kernel on the stream finishes; it waits
// for it (ace_grid_dependency_wait) before touching global memory.
template <typename K, typename Params>
cudaError_t launch_dependent(K* kernel, dim3 grid, int threads, int smem, cudaStream_t s,
                             const Params& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p);
}

// Opt a kernel in to `smem` dynamic shared-memory bytes when static + dynamic
// would exceed the default 48 KB. The attribute belongs to the current device
// only, so the size already granted is kept per device (`granted[dev]`): a
// process that drives several GPUs opts in on each of them.
template <typename K>
cudaError_t set_smem(K* kernel, int smem, int* granted, int dev) {
  if (smem <= 40 * 1024) return cudaSuccess;
  if (dev >= 0 && dev < kMaxDevices && smem <= granted[dev]) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess && dev >= 0 && dev < kMaxDevices) granted[dev] = smem;
  return e;
}

// One launcher per kernel instance: `granted` is its per-device opt-in state.
#define ACE_LAUNCHER(NAME, KERNEL, THREADS, PARAMS)                                       \
  struct NAME {                                                                          \
    static int* granted() {                                                              \
      static int bytes[kMaxDevices] = {0};                                               \
      return bytes;                                                                      \
    }                                                                                    \
    static cudaError_t run(const PARAMS& p, dim3 grid, int smem, cudaStream_t s, int dev) { \
      cudaError_t e = set_smem(KERNEL, smem, granted(), dev);                            \
      if (e != cudaSuccess) return e;                                                    \
      return launch_dependent(KERNEL, grid, THREADS, smem, s, p);                        \
    }                                                                                    \
    static int occupancy(int smem, int dev) {                                            \
      set_smem(KERNEL, smem, granted(), dev);                                            \
      int n = 0;                                                                         \
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, KERNEL, THREADS, smem) !=    \
          cudaSuccess)                                                                   \
        n = 1;                                                                           \
      return n > 0 ? n : 1;                                                              \
    }                                                                                    \
  }

template <typename T, int V, int CM, bool SM, bool SOFT, bool LAB>
ACE_LAUNCHER(HistLauncher, (hist_kernel<T, V, CM, SM, SOFT, LAB>), kHistThreads, FwdParams);

template <typename T, int C, int OFF>
ACE_LAUNCHER(SoftFwdLauncher, (soft_fwd_kernel<T, C, OFF>), kPipeThreads, FwdParams);

template <typename T, int CM, bool SOFT>
ACE_LAUNCHER(McFwdLauncher, (mc_fwd_kernel<T, CM, SOFT>), kPipeThreads, FwdParams);

template <typename T, int V, int CM, bool SM, bool SOFT, bool LAB>
ACE_LAUNCHER(GradLauncher, (grad_kernel<T, V, CM, SM, SOFT, LAB>), kThreads, BwdParams);

template <typename T, int C, int OFF, bool SOFT>
ACE_LAUNCHER(GradTmaLauncher, (grad_tma_kernel<T, C, OFF, SOFT>), kPipeThreads, BwdParams);

template <typename T, int CM, bool SOFT>
ACE_LAUNCHER(McGradLauncher, (mc_grad_kernel<T, CM, SOFT>), kPipeThreads, BwdParams);

#undef ACE_LAUNCHER

}  // namespace

// Calls L<T, V, CM, softmax, soft, labels>::F(args...) for the runtime variant.
// The (V, CM) pairs instantiated here are the ones the host chooses
// (ace_api.cu: choose_variant); any other pair returns cudaErrorInvalidValue.
#define ACE_VARIANT_CASES(L, F, T, ...)                                                   \
  do {                                                                                    \
    constexpr int VM = 16 / (int)sizeof(T);                                               \
    constexpr int V8 = (VM < 4 ? VM : 4);                                                 \
    if (v.softmax) {                                                                      \
      if (v.CM == 2 && v.V == VM) return L<T, VM, 2, true, S_, L_>::F(__VA_ARGS__);      \
      if (v.CM == 2 && v.V == 1) return L<T, 1, 2, true, S_, L_>::F(__VA_ARGS__);        \
      if (v.CM == 3 && v.V == VM) return L<T, VM, 3, true, S_, L_>::F(__VA_ARGS__);      \
      if (v.CM == 3 && v.V == 1) return L<T, 1, 3, true, S_, L_>::F(__VA_ARGS__);        \
      if (v.CM == 4 && v.V == VM) return L<T, VM, 4, true, S_, L_>::F(__VA_ARGS__);      \
      if (v.CM == 4 && v.V == 1) return L<T, 1, 4, true, S_, L_>::F(__VA_ARGS__);        \
      if (v.CM == 8 && v.V == V8) return L<T, V8, 8, true, S_, L_>::F(__VA_ARGS__);      \
      if (v.CM == 8 && v.V == 1) return L<T, 1, 8, true, S_, L_>::F(__VA_ARGS__);        \
      if (v.CM == 16 && v.V == 2) return L<T, 2, 16, true, S_, L_>::F(__VA_ARGS__);      \
      if (v.CM == 16 && v.V == 1) return L<T, 1, 16, true, S_, L_>::F(__VA_ARGS__);      \
      if (v.CM == 32 && v.V == 2) return L<T, 2, 32, true, S_, L_>::F(__VA_ARGS__);      \
      if (v.CM == 32 && v.V == 1) return L<T, 1, 32, true, S_, L_>::F(__VA_ARGS__);      \
      if (v.CM == 64 && v.V == 2) return L<T, 2, 64, true, S_, L_>::F(__VA_ARGS__);      \
      if (v.CM == 64 && v.V == 1) return L<T, 1, 64, true, S_, L_>::F(__VA_ARGS__);      \
    } else {                                                                              \
      if (v.V == VM) return L<T, VM, 1, false, S_, L_>::F(__VA_ARGS__);                  \
      if (v.V == 1) return L<T, 1, 1, false, S_, L_>::F(__VA_ARGS__);                    \
    }                                                                                     \
  } while (0)

#define ACE_FOR_SOFT_LABELS(BODY)                        \
  if (v.soft && v.labels) {                              \
    constexpr bool S_ = true, L_ = true;                 \
    BODY;                                                \
  } else if (v.soft) {                                   \
    constexpr bool S_ = true, L_ = false;                \
    BODY;                                                \
  } else if (v.labels) {                                 \
    constexpr bool S_ = false, L_ = true;                \
    BODY;                                                \
  } else {                                               \
    constexpr bool S_ = false, L_ = false;               \
    BODY;                                                \
  }

// The soft forward for labels and C <= 4: exact channel counts 2..4, background
// kept (offset 0) or dropped (offset 1); full vectors only (v.V is the dtype's
// 16-byte width: the bulk copies move 16-byte multiples).
#define ACE_SOFT_FWD_CASES(F, T, ...)                                                     \
  do {                                                                                    \
    if (v.split) {                                                                        \
      if (v.CM == 2 && v.offset == 0) return SoftFwdLauncher<T, 2, 0>::F(__VA_ARGS__);   \
      if (v.CM == 2 && v.offset == 1) return SoftFwdLauncher<T, 2, 1>::F(__VA_ARGS__);   \
      if (v.CM == 3 && v.offset == 0) return SoftFwdLauncher<T, 3, 0>::F(__VA_ARGS__);   \
      if (v.CM == 3 && v.offset == 1) return SoftFwdLauncher<T, 3, 1>::F(__VA_ARGS__);   \
      if (v.CM == 4 && v.offset == 0) return SoftFwdLauncher<T, 4, 0>::F(__VA_ARGS__);   \
      if (v.CM == 4 && v.offset == 1) return SoftFwdLauncher<T, 4, 1>::F(__VA_ARGS__);   \
    }                                                                                     \
  } while (0)

// The many-channel forward for labels: channel capacities 8, 16 and 24.
#define ACE_MC_FWD_CASES(F, T, ...)                                                      \
  do {                                                                                   \
    if (v.mc) {                                                                          \
      if (v.soft) {                                                                      \
        if (v.CM == 8) return McFwdLauncher<T, 8, true>::F(__VA_ARGS__);                 \
        if (v.CM == 16) return McFwdLauncher<T, 16, true>::F(__VA_ARGS__);              \
        if (v.CM == 24) return McFwdLauncher<T, 24, true>::F(__VA_ARGS__);              \
      } else {                                                                           \
        if (v.CM == 8) return McFwdLauncher<T, 8, false>::F(__VA_ARGS__);                \
        if (v.CM == 16) return McFwdLauncher<T, 16, false>::F(__VA_ARGS__);             \
        if (v.CM == 24) return McFwdLauncher<T, 24, false>::F(__VA_ARGS__);             \
      }                                                                                  \
    }                                                                                    \
  } while (0)

template <typename T>
cudaError_t launch_hist(const FwdParams& p, const Variant& v, dim3 grid, int smem,
                        cudaStream_t s, int dev) {
  ACE_SOFT_FWD_CASES(run, T, p, grid, smem, s, dev);
  if (v.split) return cudaErrorInvalidValue;
  ACE_MC_FWD_CASES(run, T, p, grid, smem, s, dev);
  if (v.mc) return cudaErrorInvalidValue;
  ACE_FOR_SOFT_LABELS(ACE_VARIANT_CASES(HistLauncher, run, T, p, grid, smem, s, dev));
  return cudaErrorInvalidValue;
}

// The pipelined backward: softmax over C = 2..4 channels, soft binning with
// labels or hard binning, background kept or dropped.
#define ACE_GRAD_TMA_CASES(F, T, ...)                                                    \
  do {                                                                                   \
    if (v.split) {                                                                       \
      if (v.soft) {                                                                      \
        if (v.CM == 2 && v.offset == 0) return GradTmaLauncher<T, 2, 0, true>::F(__VA_ARGS__); \
        if (v.CM == 2 && v.offset == 1) return GradTmaLauncher<T, 2, 1, true>::F(__VA_ARGS__); \
        if (v.CM == 3 && v.offset == 0) return GradTmaLauncher<T, 3, 0, true>::F(__VA_ARGS__); \
        if (v.CM == 3 && v.offset == 1) return GradTmaLauncher<T, 3, 1, true>::F(__VA_ARGS__); \
        if (v.CM == 4 && v.offset == 0) return GradTmaLauncher<T, 4, 0, true>::F(__VA_ARGS__); \
        if (v.CM == 4 && v.offset == 1) return GradTmaLauncher<T, 4, 1, true>::F(__VA_ARGS__); \
      } else {                                                                           \
        if (v.CM == 2 && v.offset == 0) return GradTmaLauncher<T, 2, 0, false>::F(__VA_ARGS__); \
        if (v.CM == 2 && v.offset == 1) return GradTmaLauncher<T, 2, 1, false>::F(__VA_ARGS__); \
        if (v.CM == 3 && v.offset == 0) return GradTmaLauncher<T, 3, 0, false>::F(__VA_ARGS__); \
        if (v.CM == 3 && v.offset == 1) return GradTmaLauncher<T, 3, 1, false>::F(__VA_ARGS__); \
        if (v.CM == 4 && v.offset == 0) return GradTmaLauncher<T, 4, 0, false>::F(__VA_ARGS__); \
        if (v.CM == 4 && v.offset == 1) return GradTmaLauncher<T, 4, 1, false>::F(__VA_ARGS__); \
      }                                                                                  \
      return cudaErrorInvalidValue;                                                      \
    }                                                                                    \
  } while (0)

// The many-channel backward: channel capacities 8, 16 and 24, soft binning with
// labels or hard binning.
#define ACE_MC_GRAD_CASES(F, T, ...)                                                     \
  do {                                                                                   \
    if (v.mc) {                                                                          \
      if (v.soft) {                                                                      \
        if (v.CM == 8) return McGradLauncher<T, 8, true>::F(__VA_ARGS__);                \
        if (v.CM == 16) return McGradLauncher<T, 16, true>::F(__VA_ARGS__);             \
        if (v.CM == 24) return McGradLauncher<T, 24, true>::F(__VA_ARGS__);             \
      } else {                                                                           \
        if (v.CM == 8) return McGradLauncher<T, 8, false>::F(__VA_ARGS__);               \
        if (v.CM == 16) return McGradLauncher<T, 16, false>::F(__VA_ARGS__);            \
        if (v.CM == 24) return McGradLauncher<T, 24, false>::F(__VA_ARGS__);            \
      }                                                                                  \
      return cudaErrorInvalidValue;                                                      \
    }                                                                                    \
  } while (0)

template <typename T>
cudaError_t launch_grad(const BwdParams& p, const Variant& v, dim3 grid, int smem,
                        cudaStream_t s, int dev) {
  ACE_GRAD_TMA_CASES(run, T, p, grid, smem, s, dev);
  ACE_MC_GRAD_CASES(run, T, p, grid, smem, s, dev);
  ACE_FOR_SOFT_LABELS(ACE_VARIANT_CASES(GradLauncher, run, T, p, grid, smem, s, dev));
  return cudaErrorInvalidValue;
}

template <typename T>
int hist_occupancy(const Variant& v, int smem, int dev) {
  ACE_SOFT_FWD_CASES(occupancy, T, smem, dev);
  if (v.split) return 1;
  ACE_MC_FWD_CASES(occupancy, T, smem, dev);
  if (v.mc) return 1;
  ACE_FOR_SOFT_LABELS(ACE_VARIANT_CASES(HistLauncher, occupancy, T, smem, dev));
  return 1;
}

template <typename T>
int grad_occupancy(const Variant& v, int smem, int dev) {
  if (v.split) return 1;
  ACE_FOR_SOFT_LABELS(ACE_VARIANT_CASES(GradLauncher, occupancy, T, smem, dev));
  return 1;
}

template <typename T>
cudaError_t launch_probs(const void* x, float* probs, int64_t B, int C, int64_t N, int act,
                         cudaStream_t s) {
  const int64_t total = B * N;
  int64_t blocks = (total + kThreads - 1) / kThreads;
  if (blocks > 4096) blocks = 4096;
  if (blocks < 1) blocks = 1;
  probs_kernel<T><<<(unsigned)blocks, kThreads, 0, s>>>(static_cast<const T*>(x), probs, B, C,
                                                        N, act);
  return cudaGetLastError();
}

#define ACE_INSTANTIATE(T)                                                                   \
  template cudaError_t launch_hist<T>(const FwdParams&, const Variant&, dim3, int,          \
                                      cudaStream_t, int);                                    \
  template cudaError_t launch_grad<T>(const BwdParams&, const Variant&, dim3, int,          \
                                      cudaStream_t, int);                                    \
  template int hist_occupancy<T>(const Variant&, int, int);                                  \
  template int grad_occupancy<T>(const Variant&, int, int);                                  \
  template cudaError_t launch_probs<T>(const void*, float*, int64_t, int, int64_t, int,     \
                                       cudaStream_t);

#endif  // __CUDACC__

}  // namespace ace
