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
};

template <typename T>
cudaError_t launch_hist(const FwdParams& p, const Variant& v, dim3 grid, int smem,
                        cudaStream_t s);
template <typename T>
cudaError_t launch_grad(const BwdParams& p, const Variant& v, dim3 grid, int smem,
                        cudaStream_t s);
template <typename T>
cudaError_t launch_probs(const void* x, float* probs, int64_t B, int C, int64_t N, int act,
                         cudaStream_t s);
// Occupancy (CTAs per SM) of the variant's kernel with `smem` dynamic bytes.
template <typename T>
int hist_occupancy(const Variant& v, int smem);
template <typename T>
int grad_occupancy(const Variant& v, int smem);

cudaError_t launch_epilogue(const float* hist, const EpiParams& e, cudaStream_t s);

#ifdef __CUDACC__

// ---------------------------------------------------------------------------
// Epilogue (one CTA): per row (b, c) and bin k, from W, P, G:
//   nonempty = W != 0 (hard) / W >= empty_weight (soft)
//   d = P / W - G / W (two IEEE divisions, then subtract; 0 if empty)
//   f = sum_nonempty |d| / K_ne (NaN if K_ne = 0)
//   coef = sign(d) / (K_ne * W) (0 if empty)
//   present = sum_k G > 0; f *= present (if ignore_empty); f *= w_c
//   jac = [present] * w_c (/ rows for "mean"); loss = mean or sum of f
// Same formulas and operation order as v2_autograd.coefficients
// (ace_kernels/impls/v2_autograd.py:66-76), common.reduce_classes
// (ace_kernels/common.py:184-207) and the fused Triton epilogue
// (ace_kernels/kernels/epilogue.py:23-82). The loss is summed in a fixed order
// (per thread ascending rows, then a fixed tree), so it is deterministic.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void epilogue_block(const EpiParams& E, const float* __restrict__ hist) {
  __shared__ float red[kThreads];
  const int tid = threadIdx.x;
  const int R = E.B_total * E.CL;
  const int K = E.K;
  const int64_t RK = (int64_t)R * K;
  const float* W = hist;
  const float* P = hist + RK;
  const float* G = hist + 2 * RK;
  const float nan = __int_as_float(0x7fc00000);
  const float rows = (float)E.rows_global;
  float mine = 0.0f;
  for (int r = tid; r < R; r += kThreads) {
    const int64_t base = (int64_t)r * K;
    int kne = 0;
    float err = 0.0f, gsum = 0.0f;
    for (int k = 0; k < K; ++k) {
      const float w = W[base + k];
      const float g = G[base + k];
      gsum = ACE_FADD(gsum, g);
      const bool ne = E.soft ? (w >= E.empty_weight) : (w != 0.0f);
      float dk = 0.0f;
      if (ne) {
        dk = ACE_FSUB(ACE_FDIV(P[base + k], w), ACE_FDIV(g, w));
        err = ACE_FADD(err, fabsf(dk));
        ++kne;
      }
      E.d[base + k] = dk;
    }
    const float kf = (float)kne;
    for (int k = 0; k < K; ++k) {
      const float w = W[base + k];
      const bool ne = E.soft ? (w >= E.empty_weight) : (w != 0.0f);
      const float dk = E.d[base + k];
      const float sg = dk > 0.0f ? 1.0f : (dk < 0.0f ? -1.0f : 0.0f);
      E.coef[base + k] = ne ? ACE_FDIV(sg, ACE_FMUL(kf, w)) : 0.0f;
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
    if (E.reduction == ACE_B200_REDUCTION_MEAN) scale = ACE_FDIV(scale, rows);
    E.f[r] = f;
    E.jac[r] = scale;
    mine = ACE_FADD(mine, f);
  }
  red[tid] = mine;
  __syncthreads();
#pragma unroll
  for (int s = kThreads / 2; s > 0; s >>= 1) {
    if (tid < s) red[tid] = ACE_FADD(red[tid], red[tid + s]);
    __syncthreads();
  }
  if (tid == 0) {
    float total = red[0];
    if (E.reduction == ACE_B200_REDUCTION_MEAN) total = ACE_FDIV(total, rows);
    E.loss[0] = total;
  }
}

// ---------------------------------------------------------------------------
// Shared-memory histogram with lane-replicated columns.
//
// Layout [stat][row][bin][R]: entry (stat, row, bin) has R consecutive words and
// lane l updates word l % R, so with R = 32 the 32 lanes of a warp always hit 32
// different banks whatever their bins are (no intra-warp conflicts, no
// serialisation on hot bins such as p < 0.05). Warps of a CTA share the table and
// update it with shared-memory atomics; hard-binning counts (W, and G with label
// targets) are exact u32 counts, the rest fp32.
// ---------------------------------------------------------------------------
struct SmemHist {
  float* h;
  int SS;     // stride between the three statistics: CL * K * R
  int RS;     // stride between rows: K * R
  int shift;  // log2(R)
  int col;    // this lane's column

  __device__ __forceinline__ int at(int row, int bin) const {
    return row * RS + (bin << shift) + col;
  }
  __device__ __forceinline__ void add_u(int a, unsigned v) const {
    atomicAdd(reinterpret_cast<unsigned*>(h + a), v);
  }
  __device__ __forceinline__ void add_f(int a, float v) const { atomicAdd(h + a, v); }
};

// One probability of loss row `row` into the histogram. `y` is the target value
// (labels: 1 for the true class, else 0).
template <bool SOFT, bool LABELS>
__device__ __forceinline__ void accumulate(const SmemHist& H, const float2* __restrict__ pairs,
                                           int K, bool right, int row, float p, float y) {
  float2 lohi;
  const int j = ace_locate(p, pairs, K, SOFT, right, lohi);
  if constexpr (!SOFT) {
    if (j < K) {  // p above the last edge (only for invalid p > 1 + eps) is dropped
      const int a = H.at(row, j);
      H.add_u(a, 1u);
      H.add_f(a + H.SS, p);
      if constexpr (LABELS) {
        if (y != 0.0f) H.add_u(a + 2 * H.SS, 1u);
      } else {
        if (y != 0.0f) H.add_f(a + 2 * H.SS, y);
      }
    }
  } else {
    const SoftW w = ace_soft_weights(p, j, lohi, K);
    const int al = H.at(row, w.l);
    const int ar = H.at(row, w.r);
    H.add_f(al, w.lw);
    H.add_f(ar, w.rw);
    H.add_f(al + H.SS, ACE_FMUL(w.lw, p));
    H.add_f(ar + H.SS, ACE_FMUL(w.rw, p));
    if constexpr (LABELS) {
      if (y != 0.0f) {
        H.add_f(al + 2 * H.SS, w.lw);
        H.add_f(ar + 2 * H.SS, w.rw);
      }
    } else {
      if (y != 0.0f) {
        H.add_f(al + 2 * H.SS, ACE_FMUL(w.lw, y));
        H.add_f(ar + 2 * H.SS, ACE_FMUL(w.rw, y));
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Forward: fused activation + W/P/G statistics (+ epilogue in the last CTA).
//
// Grid (chunks, B): CTA (x, b) streams tiles [x * tpc, (x + 1) * tpc) of batch b;
// a tile is kThreads * V voxels and thread t owns V consecutive voxels of it, read
// with 16-byte (V * sizeof(T)) coalesced loads per channel (the channel stride is
// N). The logits of all C channels of a voxel are in registers, so the softmax
// needs no second read. At the end each CTA folds its table into the workspace
// accumulators with global atomics (one per non-zero statistic), and the last CTA
// to finish (counter in the workspace, no waiting) writes the statistics, resets
// the workspace, and runs the epilogue.
// ---------------------------------------------------------------------------
template <typename T, int V, int CM, bool SOFTMAX, bool SOFT, bool LABELS>
__global__ void __launch_bounds__(kThreads) hist_kernel(const __grid_constant__ FwdParams P) {
  extern __shared__ __align__(16) float smem[];
  const int tid = threadIdx.x;
  const int b = blockIdx.y;
  const int C = P.g.C, CL = P.g.CL, off = P.g.offset, K = P.tab.K;
  const int64_t N = P.g.N;
  const int R = P.R;

  float2* pairs = reinterpret_cast<float2*>(smem);
  float* hist = smem + 2 * (kMaxBins + 1);
  const int entries = 3 * CL * K;
  for (int i = tid; i <= K; i += kThreads) pairs[i] = P.tab.pair[i];
  for (int i = tid; i < entries * R; i += kThreads) hist[i] = 0.0f;
  __syncthreads();

  SmemHist H;
  H.h = hist;
  H.shift = 31 - __clz(R);
  H.RS = K * R;
  H.SS = CL * H.RS;
  H.col = tid & (R - 1);

  const T* xb = static_cast<const T*>(P.x) + (int64_t)b * C * N;
  const int64_t* lb = LABELS ? static_cast<const int64_t*>(P.target) + (int64_t)b * N : nullptr;
  const float* yb = LABELS ? nullptr : static_cast<const float*>(P.target) + (int64_t)b * C * N;

  const int64_t t0 = (int64_t)blockIdx.x * P.g.tiles_per_chunk;
  const int64_t t1 = min(t0 + P.g.tiles_per_chunk, P.g.tiles);
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t v0 = (t * kThreads + tid) * V;
    if (v0 >= N) continue;  // V > 1 implies N % V == 0: groups are whole
    int lab[V];
    if constexpr (LABELS) ace_load_labels<V>(lb + v0, lab);
    if constexpr (SOFTMAX) {
      float xv[CM][V];
#pragma unroll
      for (int c = 0; c < CM; ++c)
        if (c < C) VecIO<T, V>::load(xb + (int64_t)c * N + v0, xv[c]);
      float yv[CM][V];
      if constexpr (!LABELS) {
#pragma unroll
        for (int c = 0; c < CM; ++c)
          if (c >= off && c < C) VecIO<float, V>::load(yb + (int64_t)c * N + v0, yv[c]);
      }
#pragma unroll
      for (int i = 0; i < V; ++i) {
        float e[CM];
#pragma unroll
        for (int c = 0; c < CM; ++c) e[c] = xv[c][i];
        const float s = ace_softmax_exp<CM>(e, C);
#pragma unroll
        for (int c = 0; c < CM; ++c) {
          if (c >= off && c < C) {
            const float p = ACE_FDIV(e[c], s);
            float y;
            if constexpr (LABELS) y = (lab[i] == c) ? 1.0f : 0.0f;
            else y = yv[c][i];
            accumulate<SOFT, LABELS>(H, pairs, K, P.right, c - off, p, y);
          }
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
          float y;
          if constexpr (LABELS) y = (lab[i] == c) ? 1.0f : 0.0f;
          else y = yv[i];
          accumulate<SOFT, LABELS>(H, pairs, K, P.right, c - off, p, y);
        }
      }
    }
  }
  __syncthreads();

  // Fold the lane columns (rotated start: conflict-free for R = 32) and add the
  // CTA's statistics to the workspace accumulators.
  const int64_t rowK = (int64_t)(P.b_offset + b) * CL * K;
  const int64_t statS = (int64_t)P.B_total * CL * K;
  for (int e = tid; e < entries; e += kThreads) {
    const int stat = e / (CL * K);
    const int rk = e - stat * CL * K;
    const bool is_u = !SOFT && (stat == 0 || (stat == 2 && LABELS));
    const float* src = hist + (int64_t)e * R;
    const int64_t gi = stat * statS + rowK + rk;
    if (is_u) {
      unsigned s = 0;
      for (int i = 0; i < R; ++i) s += __float_as_uint(src[(i + tid) & (R - 1)]);
      if (s) atomicAdd(reinterpret_cast<unsigned*>(P.accum) + gi, s);
    } else {
      float s = 0.0f;
      for (int i = 0; i < R; ++i) s += src[(i + tid) & (R - 1)];
      if (s != 0.0f) atomicAdd(P.accum + gi, s);
    }
  }
  __threadfence();
  __syncthreads();
  __shared__ bool s_last;
  if (tid == 0) {
    const unsigned done = atomicAdd(P.counter, 1u);
    s_last = (done == gridDim.x * gridDim.y - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // Last CTA: statistics out, workspace back to zero, epilogue.
  const int64_t total = 3 * statS;
  unsigned* acc_u = reinterpret_cast<unsigned*>(P.accum);
  for (int64_t i = tid; i < total; i += kThreads) {
    const int stat = (int)(i / statS);
    const bool is_u = !SOFT && (stat == 0 || (stat == 2 && LABELS));
    const unsigned raw = __ldcg(acc_u + i);
    P.hist_out[i] = is_u ? (float)raw : __uint_as_float(raw);
    __stcg(acc_u + i, 0u);
  }
  if (tid == 0) *P.counter = 0u;
  if (P.do_epilogue) {
    __syncthreads();
    epilogue_block(P.epi, P.hist_out);
  }
}

// ---------------------------------------------------------------------------
// Backward: d loss / d x in one pass (ace_kernels/impls/v2_autograd.py:88-118,
// derivation in the reference's docs/derivation.md):
//   hard: gp_c = g_bc * coef[b, c, bin(p_c)]
//   soft: gp_c = g_bc * (coef_l (lw - (p - y - d_l) / S) + coef_r (rw + (p - y - d_r) / S))
//   softmax: dx_c = p_c (gp_c - sum_c' p_c' gp_c'); sigmoid: gp p (1 - p); none: gp
// with gp = 0 on a dropped background channel. The activation is recomputed with
// the forward's code (same bins); coef / d of this CTA's batch row sit in shared
// memory as {coef, d} pairs. Hard binning reads no targets.
// ---------------------------------------------------------------------------
template <bool SOFT>
__device__ __forceinline__ float grad_p(const float2* __restrict__ pairs,
                                        const float2* __restrict__ cd, int K, bool right,
                                        int row, float g, float p, float y) {
  float2 lohi;
  const int j = ace_locate(p, pairs, K, SOFT, right, lohi);
  const float2* cr = cd + row * K;
  if constexpr (!SOFT) {
    return j < K ? g * cr[j].x : 0.0f;
  } else {
    const SoftW w = ace_soft_weights(p, j, lohi, K);
    const float inv = ACE_FDIV(1.0f, w.span);
    const float resid = p - y;
    const float2 L = cr[w.l], Rr = cr[w.r];
    const float left = L.x * (w.lw - inv * (resid - L.y));
    const float right_ = Rr.x * (w.rw + inv * (resid - Rr.y));
    return (left + right_) * g;
  }
}

template <typename T, int V, int CM, bool SOFTMAX, bool SOFT, bool LABELS>
__global__ void __launch_bounds__(kThreads) grad_kernel(const __grid_constant__ BwdParams P) {
  extern __shared__ __align__(16) float smem[];
  const int tid = threadIdx.x;
  const int b = blockIdx.y;
  const int C = P.g.C, CL = P.g.CL, off = P.g.offset, K = P.tab.K;
  const int64_t N = P.g.N;

  float2* pairs = reinterpret_cast<float2*>(smem);
  float2* cd = pairs + (kMaxBins + 1);
  float* gs = reinterpret_cast<float*>(cd + CL * K);
  const int64_t row0 = (int64_t)(P.b_offset + b) * CL;
  for (int i = tid; i <= K; i += kThreads) pairs[i] = P.tab.pair[i];
  for (int i = tid; i < CL * K; i += kThreads)
    cd[i] = make_float2(P.coef[row0 * K + i], P.d[row0 * K + i]);
  for (int i = tid; i < CL; i += kThreads)
    gs[i] = P.jac[row0 + i] * (P.grad_per_row ? P.grad_out[row0 + i] : P.grad_out[0]);
  __syncthreads();

  const T* xb = static_cast<const T*>(P.x) + (int64_t)b * C * N;
  T* db = static_cast<T*>(P.dx) + (int64_t)b * C * N;
  const int64_t* lb = (SOFT && LABELS) ? static_cast<const int64_t*>(P.target) + (int64_t)b * N : nullptr;
  const float* yb = (SOFT && !LABELS) ? static_cast<const float*>(P.target) + (int64_t)b * C * N : nullptr;

  const int64_t t0 = (int64_t)blockIdx.x * P.g.tiles_per_chunk;
  const int64_t t1 = min(t0 + P.g.tiles_per_chunk, P.g.tiles);
  for (int64_t t = t0; t < t1; ++t) {
    const int64_t v0 = (t * kThreads + tid) * V;
    if (v0 >= N) continue;
    int lab[V];
    if constexpr (SOFT && LABELS) ace_load_labels<V>(lb + v0, lab);
    if constexpr (SOFTMAX) {
      float xv[CM][V];
#pragma unroll
      for (int c = 0; c < CM; ++c)
        if (c < C) VecIO<T, V>::load(xb + (int64_t)c * N + v0, xv[c]);
      float yv[CM][V];
      if constexpr (SOFT && !LABELS) {
#pragma unroll
        for (int c = 0; c < CM; ++c)
          if (c >= off && c < C) VecIO<float, V>::load(yb + (int64_t)c * N + v0, yv[c]);
      }
#pragma unroll
      for (int i = 0; i < V; ++i) {
        float e[CM];
#pragma unroll
        for (int c = 0; c < CM; ++c) e[c] = xv[c][i];
        const float s = ace_softmax_exp<CM>(e, C);
        float gp[CM];
        float dot = 0.0f;
#pragma unroll
        for (int c = 0; c < CM; ++c) {
          gp[c] = 0.0f;
          if (c < C) {
            const float p = ACE_FDIV(e[c], s);
            e[c] = p;
            if (c >= off) {
              float y = 0.0f;
              if constexpr (SOFT && LABELS) y = (lab[i] == c) ? 1.0f : 0.0f;
              if constexpr (SOFT && !LABELS) y = yv[c][i];
              gp[c] = grad_p<SOFT>(pairs, cd, K, P.right, c - off, gs[c - off], p, y);
            }
            dot += p * gp[c];
          }
        }
#pragma unroll
        for (int c = 0; c < CM; ++c)
          if (c < C) xv[c][i] = e[c] * (gp[c] - dot);
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
        const float g = gs[c - off];
#pragma unroll
        for (int i = 0; i < V; ++i) {
          const bool sig = P.act == ACE_B200_ACT_SIGMOID;
          const float p = sig ? ace_sigmoid(xv[i]) : xv[i];
          float y = 0.0f;
          if constexpr (SOFT && LABELS) y = (lab[i] == c) ? 1.0f : 0.0f;
          if constexpr (SOFT && !LABELS) y = yv[i];
          const float gp = grad_p<SOFT>(pairs, cd, K, P.right, c - off, g, p, y);
          xv[i] = sig ? gp * p * (1.0f - p) : gp;
        }
        VecIO<T, V>::store(db + (int64_t)c * N + v0, xv);
      }
    }
  }
}

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
      const float s = ace_softmax_exp<kMaxClasses>(e, C);
#pragma unroll
      for (int c = 0; c < kMaxClasses; ++c)
        if (c < C) op[(int64_t)c * N] = ACE_FDIV(e[c], s);
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
template <typename T, int V, int CM, bool SM, bool SOFT, bool LAB>
struct HistLauncher {
  static cudaError_t run(const FwdParams& p, dim3 grid, int smem, cudaStream_t s) {
    auto k = hist_kernel<T, V, CM, SM, SOFT, LAB>;
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
    }
    k<<<grid, kThreads, smem, s>>>(p);
    return cudaGetLastError();
  }
  static int occupancy(int smem) {
    auto k = hist_kernel<T, V, CM, SM, SOFT, LAB>;
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kThreads, smem) != cudaSuccess) n = 1;
    return n > 0 ? n : 1;
  }
};

template <typename T, int V, int CM, bool SM, bool SOFT, bool LAB>
struct GradLauncher {
  static cudaError_t run(const BwdParams& p, dim3 grid, int smem, cudaStream_t s) {
    auto k = grad_kernel<T, V, CM, SM, SOFT, LAB>;
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
    }
    k<<<grid, kThreads, smem, s>>>(p);
    return cudaGetLastError();
  }
  static int occupancy(int smem) {
    auto k = grad_kernel<T, V, CM, SM, SOFT, LAB>;
    if (smem > 48 * 1024)
      cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k, kThreads, smem) != cudaSuccess) n = 1;
    return n > 0 ? n : 1;
  }
};

// Calls L<T, V, CM, softmax, soft, labels>::F(args...) for the runtime variant.
// The (V, CM) pairs instantiated here are the ones the host chooses
// (ace_api.cu: choose_variant); any other pair returns cudaErrorInvalidValue.
#define ACE_VARIANT_CASES(L, F, T, ...)                                                   \
  do {                                                                                    \
    constexpr int VM = 16 / (int)sizeof(T);                                               \
    constexpr int V8 = (VM < 4 ? VM : 4);                                                 \
    if (v.softmax) {                                                                      \
      if (v.CM == 4 && v.V == VM) return L<T, VM, 4, true, S_, L_>::F(__VA_ARGS__);      \
      if (v.CM == 4 && v.V == 1) return L<T, 1, 4, true, S_, L_>::F(__VA_ARGS__);        \
      if (v.CM == 8 && v.V == V8) return L<T, V8, 8, true, S_, L_>::F(__VA_ARGS__);      \
      if (v.CM == 8 && v.V == 1) return L<T, 1, 8, true, S_, L_>::F(__VA_ARGS__);        \
      if (v.CM == 16 && v.V == 2) return L<T, 2, 16, true, S_, L_>::F(__VA_ARGS__);      \
      if (v.CM == 16 && v.V == 1) return L<T, 1, 16, true, S_, L_>::F(__VA_ARGS__);      \
      if (v.CM == 32 && v.V == 1) return L<T, 1, 32, true, S_, L_>::F(__VA_ARGS__);      \
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

template <typename T>
cudaError_t launch_hist(const FwdParams& p, const Variant& v, dim3 grid, int smem,
                        cudaStream_t s) {
  ACE_FOR_SOFT_LABELS(ACE_VARIANT_CASES(HistLauncher, run, T, p, grid, smem, s));
  return cudaErrorInvalidValue;
}

template <typename T>
cudaError_t launch_grad(const BwdParams& p, const Variant& v, dim3 grid, int smem,
                        cudaStream_t s) {
  ACE_FOR_SOFT_LABELS(ACE_VARIANT_CASES(GradLauncher, run, T, p, grid, smem, s));
  return cudaErrorInvalidValue;
}

template <typename T>
int hist_occupancy(const Variant& v, int smem) {
  ACE_FOR_SOFT_LABELS(ACE_VARIANT_CASES(HistLauncher, occupancy, T, smem));
  return 1;
}

template <typename T>
int grad_occupancy(const Variant& v, int smem) {
  ACE_FOR_SOFT_LABELS(ACE_VARIANT_CASES(GradLauncher, occupancy, T, smem));
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
                                      cudaStream_t);                                         \
  template cudaError_t launch_grad<T>(const BwdParams&, const Variant&, dim3, int,          \
                                      cudaStream_t);                                         \
  template int hist_occupancy<T>(const Variant&, int);                                       \
  template int grad_occupancy<T>(const Variant&, int);                                       \
  template cudaError_t launch_probs<T>(const void*, float*, int64_t, int, int64_t, int,     \
                                       cudaStream_t);

#endif  // __CUDACC__

}  // namespace ace
