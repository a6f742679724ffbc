// grad_tma_kernel: the backward (d loss / d logits) of a softmax over C <= 4
// channels, soft binning with int64 labels or hard binning, on B200 (sm_100a), as
// a TMA pipeline. Included by ace_kernels.cuh after grad_kernel's helpers.
//
// Same formulas as grad_kernel (see its comment; ace_kernels/impls/
// v2_autograd.py:88-118): per value gp = F + D (2 p - y) from the per-(row,
// interval) soft records, or g coef[bin] for hard binning, then the softmax
// backward dx_c = p_c (gp_c - sum_c' p_c' gp_c'), with the forward's activation
// recomputed. The memory side is a producer thread streaming tiles (the C logit
// rows, and the labels for soft binning) into a shared-memory ring with bulk
// copies; kPipeConsumerWarps consumer warps compute and store dx straight from
// registers with streaming 16-byte stores.
//
// Soft binning recomputes exactly the forward's p (the fast softmax, saturated)
// and takes the forward's interval, the rounded p K; its records are split by
// class flag, {F - D y, 2 D} for y = 0 and 1, so gp = fma(2 D, p, F - D y) is one
// FMA, and the fp32 arithmetic runs on voxel pairs (__ffma2_rn / __fmul2_rn /
// __fadd2_rn). Hard binning recomputes the exact softmax and locates the exact
// bin with the forward's code, so every value is in the forward's bin.
//
// Tile order: the tiles of all batches are taken round-robin by the CTAs
// (tile k of the sequence by CTA k mod grid), the sequence running from the
// batches' last tiles to their first, the batches interleaved. Every CTA then
// gets an even share of tiles still in L2 from the forward (which takes each
// batch's tiles in increasing order, so its last ones are the most recently
// read), and those are read first, before this kernel's own stores evict them.
// The records of all local batches are built once per CTA (from coef, d, jac
// and the upstream gradient) into shared memory.
#pragma once

namespace ace {

// The producer thread of a backward pipeline (grad_tma_kernel, mc_grad_kernel):
// the tiles of all batches round-robin over the CTAs (tile k of the sequence by
// CTA k mod grid), the sequence running from the batches' last tiles to their
// first, the batches interleaved (k -> batch k % B, tile tpb - 1 - k / B). Each
// tile's C logit rows (TV * sizeof(T) bytes apart) and, when `lab` is given, its
// int64 labels (after `rows` >= C row slots) go into stage i % S of the ring, with s_meta[s] =
// {tile, batch, voxels, 0}; the last stage carries the end marker (tile -1). A
// wait that runs out sets s_abort; the producer then waits (bounded) for its
// copies still in flight.
template <typename T, int TV>
__device__ __forceinline__ void produce_round_robin(const T* x, const int64_t* lab, int C,
                                                    int rows, int64_t N, int B, int64_t tpb,
                                                    unsigned stage0, unsigned SB, int S,
                                                    unsigned long long* s_full,
                                                    unsigned long long* s_empty, int4* s_meta,
                                                    volatile int* s_abort) {
  constexpr unsigned XB = TV * sizeof(T);
  const int64_t total = tpb * B;
  int issued = 0;
  int64_t k = blockIdx.x;
  for (int i = 0;; ++i, k += gridDim.x) {
    const int s = i % S;
    const unsigned use = (unsigned)(i / S);
    if (use > 0 && !mbar_wait(smem_addr(&s_empty[s]), (use - 1) & 1u)) {
      *s_abort = 1;
      break;
    }
    if (*s_abort) break;
    const unsigned full = smem_addr(&s_full[s]);
    if (k >= total) {  // the end marker (no copies)
      s_meta[s] = make_int4(-1, 0, 0, 0);
      mbar_arrive(full);
      break;
    }
    const int tb = (int)(k % B);
    const int64_t tile = tpb - 1 - k / B;
    const int64_t v0 = tile * TV;
    const int cnt = (int)min((int64_t)TV, N - v0);
    s_meta[s] = make_int4((int)tile, tb, cnt, 0);
    const unsigned xb = (unsigned)cnt * (unsigned)sizeof(T);
    mbar_arrive_tx(full, (unsigned)C * xb + (lab ? (unsigned)cnt * 8u : 0u));
    const unsigned dst = stage0 + (unsigned)s * SB;
    const T* gx = x + (int64_t)tb * C * N + v0;
    for (int c = 0; c < C; ++c) bulk_load(dst + c * XB, gx + (int64_t)c * N, xb, full);
    if (lab) bulk_load(dst + rows * XB, lab + (int64_t)tb * N + v0, (unsigned)cnt * 8u, full);
    issued = i + 1;
  }
  // after an abort, no copy may still be in flight when the CTA leaves
  if (*s_abort)
    for (int i = issued - S > 0 ? issued - S : 0; i < issued; ++i)
      mbar_wait(smem_addr(&s_full[i % S]), (unsigned)(i / S) & 1u);
}

// The per-(batch, row, interval or bin) records of the pipelined backwards, built
// by the consumer threads into shared memory from coef, d, jac and the upstream
// gradient g (after the dependency wait): hard, [B][CL][K + 1][copies] floats
// g coef[k] (0 for the count K, no bin); soft, [B][CL][K + 1][2][copies] float2
// {F - D y, 2 D} for the class flags y = 0, 1 of interval j (see grad_kernel: the
// soft gradient is F + D (2 p - y) inside an interval). One thread per record
// writes all its copies with 16-byte stores (copies * record bytes is a multiple
// of 16), or 4-byte stores when a hard record has fewer than four copies.
template <bool SOFT>
__device__ __forceinline__ void build_records(const BwdParams& P, float* rec, int CL,
                                              const float2* s_map) {
  const int K = P.tab.K, B = P.g.B, copies = P.rec_copies;
  for (int e = threadIdx.x; e < B * CL * (K + 1); e += kPipeConsumerWarps * 32) {
    const int bro = e / (K + 1), j = e - bro * (K + 1);  // bro = b * CL + row
    const int b = bro / CL, row = bro - b * CL;
    const int64_t grow = (int64_t)(P.b_offset + b) * CL + row;
    const float g = P.jac[grow] * (P.grad_per_row ? P.grad_out[grow] : P.grad_out[0]);
    const float* cf = P.coef + grow * K;
    const float* dd = P.d + grow * K;
    if constexpr (!SOFT) {
      const unsigned u = __float_as_uint(j < K ? g * cf[j] : 0.0f);
      if (copies >= 4) {
        const uint4 v = make_uint4(u, u, u, u);
        uint4* dst = reinterpret_cast<uint4*>(rec + e * copies);
        for (int q = 0; q < copies / 4; ++q) dst[q] = v;
      } else {
        for (int q = 0; q < copies; ++q) rec[e * copies + q] = __uint_as_float(u);
      }
    } else {
      const int l = max(j - 1, 0), r = min(j, K - 1);
      const float a = g * cf[l], bb = g * cf[r];
      double F = a, D = 0.0;
      if (j > 0 && j < K) {
        const float2 mp = s_map[j];
        const double lo = mp.x, inv = (double)mp.y / (double)kFixScale;
        D = ((double)bb - (double)a) * inv;
        F = (double)a - D * lo + inv * ((double)a * dd[l] - (double)bb * dd[r]);
      }
      const unsigned d2 = __float_as_uint(2.0f * (float)D);
      const unsigned f0 = __float_as_uint((float)F), f1 = __float_as_uint((float)(F - D));
      const uint4 v0 = make_uint4(f0, d2, f0, d2), v1 = make_uint4(f1, d2, f1, d2);
      uint4* dst = reinterpret_cast<uint4*>(rec + 4 * e * copies);
      for (int q = 0; q < copies / 2; ++q) dst[q] = v0;
      for (int q = copies / 2; q < copies; ++q) dst[q] = v1;
    }
  }
}

template <typename T, int C, int OFF, bool SOFT>
__global__ void __launch_bounds__(kPipeThreads, 1) grad_tma_kernel(const __grid_constant__ BwdParams P) {
  constexpr int NCW = kPipeConsumerWarps, NT = kPipeThreads;
  constexpr int TV = kPipeTileVoxels, VL = kPipeLaneVoxels;
  constexpr int CL = C - OFF;
  constexpr unsigned XB = TV * sizeof(T);                 // bytes of one logit row of a stage
  constexpr unsigned SB = C * XB + (SOFT ? TV * 8 : 0);  // bytes of a stage (rows, then labels)
  static_assert(VL == 4, "lds_logits / lds_labels load four voxels");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) unsigned long long s_full[kPipeMaxStages], s_empty[kPipeMaxStages];
  __shared__ int4 s_meta[kPipeMaxStages];  // {tile, batch, voxels, 0}; tile < 0: no more tiles
  __shared__ volatile int s_abort;
  __shared__ float2 s_map[kMaxBins + 1];   // {base, scale} of interval j (soft records)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = P.tab.K, S = P.stages, B = P.g.B, copies = P.rec_copies;
  const int64_t N = P.g.N;
  const float Kf = (float)K;
  // shared memory: records [B][CL][K + 1][copies] (hard: float) or
  // [B][CL][K + 1][2][copies] (soft: float2, by class flag), the bin table
  // [K + 1][kTabCopies] float2, then the stages (128-aligned)
  float* rec = reinterpret_cast<float*>(smem_raw);
  const int rec_words = (SOFT ? 4 : 1) * B * CL * (K + 1) * copies;
  float2* lohi_t = reinterpret_cast<float2*>(rec + rec_words);
  const unsigned stage0 = smem_addr(smem_raw) + (unsigned)P.stage_offset;
  auto full_bar = [&](int s) { return smem_addr(&s_full[s]); };
  auto empty_bar = [&](int s) { return smem_addr(&s_empty[s]); };

  for (int i = tid; i < (K + 1) * kTabCopies; i += NT) lohi_t[i] = P.tab.lohi[i / kTabCopies];
  for (int j = warp; j <= K; j += NT / 32)  // warp-uniform parameter reads
    if (lane == 0) s_map[j] = P.tab.map[j];
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1u);
      mbar_init(empty_bar(s), (unsigned)NCW);
    }
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();

  const int64_t tpb = P.tiles_per_batch;

  if (warp == NCW) {
    // ---------------- producer (one thread) ----------------
    // The logits and labels are inputs of the forward too, never written by the
    // kernel this one depends on: the copies may start before that kernel ends.
    if (lane == 0)
      produce_round_robin<T, TV>(static_cast<const T*>(P.x),
                                 SOFT ? static_cast<const int64_t*>(P.target) : nullptr, C, C,
                                 N, B, tpb, stage0, SB, S, s_full, s_empty, s_meta, &s_abort);
  } else {
    // ---------------- consumers ----------------
    // coef, d and jac come from the previous kernel: records only after it
    ace_grid_dependency_wait();
    build_records<SOFT>(P, rec, CL, s_map);
    consumer_sync();
    const float2* my_lohi = lohi_t + (lane & (kTabCopies - 1));
    auto entry = [&](int j) -> float2 { return my_lohi[j * kTabCopies]; };
    const int vo = (warp * 32 + lane) * VL;  // this lane's first voxel of a tile
    T* dxp = static_cast<T*>(P.dx);
    // soft: shared byte address of the record (row rb + c, interval j, flag 0) of
    // this lane's copy is bits(t) * RS + rbase + c * CS, t = magic + j
    const unsigned RS = 2u * copies * 8u, CS = (unsigned)(K + 1) * RS;
    const unsigned rec0 = smem_addr(rec) + (unsigned)((lane & (copies - 1)) * 8) - kFixMagicBits * RS;
    for (int i = 0;; ++i) {
      const int s = i % S;
      if (!mbar_wait(full_bar(s), (unsigned)(i / S) & 1u)) {
        s_abort = 1;
        break;
      }
      const int4 m = s_meta[s];
      if (m.x < 0 || s_abort) break;
      const unsigned st = stage0 + (unsigned)s * SB;
      float xv[C][4];
      int lab[4] = {0, 0, 0, 0};
#pragma unroll
      for (int c = 0; c < C; ++c) lds_logits<T>(st + c * XB + vo * (unsigned)sizeof(T), xv[c]);
      if constexpr (SOFT) lds_labels(st + C * XB + vo * 8u, lab);
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(s));  // the stage may be refilled now
      if (vo >= m.z) continue;                    // past the batch's last voxel
      const int rb = m.y * CL - OFF;              // record row of channel c: rb + c
      if constexpr (SOFT) {
        const unsigned rbase = rec0 + (unsigned)rb * CS;
#pragma unroll
        for (int v = 0; v < VL; v += 2) {
          // the forward's softmax (soft_fwd_kernel), on the voxel pair v, v + 1
          float2 xp[C], e[C], p[C];
#pragma unroll
          for (int c = 0; c < C; ++c) xp[c] = make_float2(xv[c][v], xv[c][v + 1]);
          float2 mx = xp[0];
#pragma unroll
          for (int c = 1; c < C; ++c) mx = make_float2(fmaxf(mx.x, xp[c].x), fmaxf(mx.y, xp[c].y));
          const float2 nmL = __fmul2_rn(mx, make_float2(-kLog2e, -kLog2e));
          float2 sum;
#pragma unroll
          for (int c = 0; c < C; ++c) {
            const float2 arg = __ffma2_rn(xp[c], make_float2(kLog2e, kLog2e), nmL);
            e[c] = make_float2(ace_exp2_approx(arg.x), ace_exp2_approx(arg.y));
            sum = c == 0 ? e[0] : __fadd2_rn(sum, e[c]);
          }
          const float2 y = make_float2(ace_rcp_approx(sum.x), ace_rcp_approx(sum.y));
          float2 dot = make_float2(0.0f, 0.0f), gp[C];
#pragma unroll
          for (int c = 0; c < C; ++c) {
            p[c] = make_float2(__saturatef(__fmul_rn(e[c].x, y.x)), __saturatef(__fmul_rn(e[c].y, y.y)));
            gp[c] = make_float2(0.0f, 0.0f);
            if (c < OFF) continue;
            const float2 t = __ffma2_rn(p[c], make_float2(Kf, Kf), make_float2(kFixMagic, kFixMagic));
            unsigned a0 = __float_as_uint(t.x) * RS + rbase + (unsigned)c * CS;
            unsigned a1 = __float_as_uint(t.y) * RS + rbase + (unsigned)c * CS;
            if (lab[v] == c) a0 += copies * 8u;
            if (lab[v + 1] == c) a1 += copies * 8u;
            float2 r0, r1;
            asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(r0.x), "=f"(r0.y) : "r"(a0));
            asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(r1.x), "=f"(r1.y) : "r"(a1));
            gp[c] = make_float2(__fmaf_rn(r0.y, p[c].x, r0.x), __fmaf_rn(r1.y, p[c].y, r1.x));
            dot = __ffma2_rn(p[c], gp[c], dot);
          }
#pragma unroll
          for (int c = 0; c < C; ++c) {
            const float2 dx = __fmul2_rn(p[c], __fadd2_rn(gp[c], make_float2(-dot.x, -dot.y)));
            xv[c][v] = dx.x;
            xv[c][v + 1] = dx.y;
          }
        }
      } else {
        const float* my_rec = rec + (lane & (copies - 1));
#pragma unroll
        for (int v = 0; v < VL; ++v) {
          float p[C];
#pragma unroll
          for (int c = 0; c < C; ++c) p[c] = xv[c][v];
          ace_softmax<C>(p, C);
          int j[C];
          bool ok = true;
#pragma unroll
          for (int c = OFF; c < C; ++c) {
            j[c] = ace_guess(p[c], Kf, K, false);
            ok &= ace_is_count(p[c], entry(j[c]));
          }
          if (!ok) {
#pragma unroll
            for (int c = OFF; c < C; ++c)
              if (!ace_is_count(p[c], entry(j[c])))
                j[c] = ace_fix_count(p[c], j[c], K, my_lohi, kTabCopies).i;
          }
          float gp[C], dot = 0.0f;
#pragma unroll
          for (int c = 0; c < C; ++c) {
            gp[c] = c >= OFF ? grad_p<false>(my_rec, copies, rb + c, K, j[c], p[c], 0.0f) : 0.0f;
            dot += p[c] * gp[c];
          }
#pragma unroll
          for (int c = 0; c < C; ++c) xv[c][v] = p[c] * (gp[c] - dot);
        }
      }
      const int64_t v0 = (int64_t)m.x * TV + vo;
      T* db = dxp + (int64_t)m.y * C * N + v0;
#pragma unroll
      for (int c = 0; c < C; ++c) VecIO<T, VL>::store(db + (int64_t)c * N, xv[c]);
    }
  }
  __syncthreads();
}

}  // namespace ace
