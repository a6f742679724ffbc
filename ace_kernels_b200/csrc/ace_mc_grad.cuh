// mc_grad_kernel: the backward (d loss / d logits) of a softmax over 5 to 24
// channels, soft binning with int64 labels or hard binning, on B200 (sm_100a).
// Included by ace_kernels.cuh after ace_mc_fwd.cuh and ace_grad_tma.cuh.
//
// Same formulas as grad_kernel (ace_kernels/impls/v2_autograd.py:88-118): per
// value gp = F + D (2 p - y) from the soft records of its interval, or g coef[bin]
// for hard binning, then dx_c = p_c (gp_c - sum_c' p_c' gp_c'). The pipeline is
// grad_tma_kernel's (produce_round_robin: tiles round robin over the CTAs from the
// batches' ends, so each CTA first reads tiles the forward left in L2; records of
// all local batches built once per CTA by build_records), the arithmetic
// mc_fwd_kernel's: a consumer lane takes a voxel pair of a 1024-voxel tile, with
// the packed fp32 pairs, the same softmax (fast for soft binning, exact for hard
// binning) and the same interval or bin of every value, so each value's gradient
// is that of the interval or bin the forward counted it in.
//
// Two phases per tile, the exponentials of all channels in registers: the first
// computes p and gp per channel and the dot product sum p gp; the second writes
// dx = p (gp - dot) with streaming stores. Up to 16 channels p and gp stay in
// registers between the phases; above that (the 96 registers of a 544-thread CTA
// hold 2 C floats a lane, not 4 C) the second phase recomputes p from the
// exponentials and gp from the records, of the bins the first phase found and
// packed (hard binning) or of the interval one FMA gives (soft binning).
#pragma once

namespace ace {

// dx of a voxel pair into a row of x's dtype (streaming: written once).
template <typename T>
__device__ __forceinline__ void stg_pair(T* p, float2 v);
template <>
__device__ __forceinline__ void stg_pair<float>(float* p, float2 v) {
  __stcs(reinterpret_cast<float2*>(p), v);
}
template <>
__device__ __forceinline__ void stg_pair<__nv_bfloat16>(__nv_bfloat16* p, float2 v) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
  __stcs(reinterpret_cast<unsigned*>(p), *reinterpret_cast<const unsigned*>(&h));
}
template <>
__device__ __forceinline__ void stg_pair<__half>(__half* p, float2 v) {
  const __half2 h = __floats2half2_rn(v.x, v.y);
  __stcs(reinterpret_cast<unsigned*>(p), *reinterpret_cast<const unsigned*>(&h));
}

template <typename T, int CM, bool SOFT>
__global__ void __launch_bounds__(kPipeThreads, 1) mc_grad_kernel(const __grid_constant__ BwdParams P) {
  constexpr int NCW = kPipeConsumerWarps, NT = kPipeThreads, TV = kMcTileVoxels;
  constexpr unsigned XB = TV * sizeof(T);  // bytes of one logit row of a stage
  constexpr bool KEEP = CM <= 16;           // p and gp stay in registers between the phases
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) unsigned long long s_full[kPipeMaxStages], s_empty[kPipeMaxStages];
  __shared__ int4 s_meta[kPipeMaxStages];  // {tile, batch, voxels, 0}; tile < 0: no more tiles
  __shared__ volatile int s_abort;
  __shared__ float2 s_map[kMaxBins + 1];   // {base, scale} of interval j (soft records)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = P.g.C, OFF = P.g.offset, CL = C - OFF;
  const int K = P.tab.K, S = P.stages, B = P.g.B, copies = P.rec_copies;
  const int64_t N = P.g.N;
  const unsigned SB = (unsigned)C * XB + (SOFT ? TV * 8u : 0u);  // C rows, then labels
  // shared memory: the records (see build_records), the bin table
  // [K + 1][kTabCopies] float2 (hard), then the ring of stages (128-aligned)
  float* rec = reinterpret_cast<float*>(smem_raw);
  const int rec_words = (SOFT ? 4 : 1) * B * CL * (K + 1) * copies;
  float2* lohi_t = reinterpret_cast<float2*>(rec + rec_words);
  const unsigned stage0 = smem_addr(smem_raw) + (unsigned)P.stage_offset;
  auto full_bar = [&](int s) { return smem_addr(&s_full[s]); };
  auto empty_bar = [&](int s) { return smem_addr(&s_empty[s]); };

  if constexpr (!SOFT)
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

  if (warp == NCW) {
    // ---------------- producer (one thread) ----------------
    // The logits and labels are inputs of the forward too, never written by the
    // kernel this one depends on: the copies may start before that kernel ends.
    if (lane == 0)
      produce_round_robin<T, TV>(static_cast<const T*>(P.x),
                                 SOFT ? static_cast<const int64_t*>(P.target) : nullptr, C, C,
                                 N, B,
                                 P.tiles_per_batch, stage0, SB, S, s_full, s_empty, s_meta,
                                 &s_abort);
  } else {
    // ---------------- consumers ----------------
    // coef, d and jac come from the previous kernel: records only after it
    ace_grid_dependency_wait();
    build_records<SOFT>(P, rec, CL, s_map);
    consumer_sync();
    const float2* my_lohi = lohi_t + (lane & (kTabCopies - 1));
    const int vo = (warp * 32 + lane) * kMcLaneVoxels;  // this lane's first voxel of a tile
    T* dxp = static_cast<T*>(P.dx);
    const float Kf = (float)K;
    const float2 K2 = make_float2(Kf, Kf);
    const float2 M2 = make_float2(kFixMagic, kFixMagic);
    const float2 KR2 = make_float2(Kf * kMcRScale, Kf * kMcRScale);
    // Record addresses (bytes, this lane's copy). Soft: (row rb + c, interval j,
    // flag f) at bits(t) * RS + rbase + c * CS + f * copies * 8 with t = magic + j
    // (mod 2^32; the magic is folded into lane_rec). Hard: (row rb + c, bin k) at
    // k * RS + rbase + c * CS.
    const unsigned RS = SOFT ? 2u * copies * 8u : (unsigned)copies * 4u;
    const unsigned CS = (unsigned)(K + 1) * RS;
    // (byte offsets from the start of shared memory, where the records begin)
    const unsigned lane_rec = (unsigned)((lane & (copies - 1)) * (SOFT ? 8 : 4)) -
                              (SOFT ? kFixMagicBits * RS : 0u);
    for (int i = 0;; ++i) {
      const int s = i % S;
      if (!mbar_wait(full_bar(s), (unsigned)(i / S) & 1u)) {
        s_abort = 1;
        break;
      }
      const int4 m = s_meta[s];
      if (m.x < 0 || s_abort) break;
      const unsigned char* st = smem_raw + P.stage_offset + (size_t)s * SB;
      const unsigned char* my = st + (size_t)vo * sizeof(T);
      int2 lab = make_int2(-1, -1);
      if constexpr (SOFT) lab = ld_labels2(st + (size_t)C * XB + (size_t)vo * 8);
      float2 e[CM];  // the forward's exponentials (pair_exponentials)
      const float2 sum = pair_exponentials<T, CM, SOFT, false>(my, C, e);
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(s));  // the stage may be refilled now
      if (vo >= m.z) continue;                    // past the batch's last voxel (N is even)
      const unsigned rbase = lane_rec + (unsigned)(m.y * CL - OFF) * CS;  // channel 0's row
      const float2 y = SOFT ? make_float2(ace_rcp_approx(sum.x), ace_rcp_approx(sum.y))
                            : make_float2(ace_rcp_refined(sum.x), ace_rcp_refined(sum.y));
      const float2 ns = make_float2(-sum.x, -sum.y);
      // p of channel c from its exponential: the forward's operations
      auto prob = [&](float2 ec) -> float2 {
        if constexpr (SOFT) {
          return make_float2(__saturatef(__fmul_rn(ec.x, y.x)), __saturatef(__fmul_rn(ec.y, y.y)));
        } else {
          const float2 q0 = __fmul2_rn(ec, y);
          return __ffma2_rn(__ffma2_rn(ns, q0, ec), y, q0);
        }
      };
      // hard binning: the records of the pair's bins k in channel c's row
      auto records = [&](int c, uint2 k) -> float2 {
        const unsigned cb = rbase + (unsigned)c * CS;
        return make_float2(*reinterpret_cast<const float*>(smem_raw + (k.x * RS + cb)),
                           *reinterpret_cast<const float*>(smem_raw + (k.y * RS + cb)));
      };
      // soft binning: gp of channel c >= OFF at p, from its interval's record (the
      // interval one FMA gives, as in mc_fwd_kernel). Hard binning finds its bins
      // in the grouped search below.
      auto grad = [&](int c, float2 p) -> float2 {
        const unsigned cb = rbase + (unsigned)c * CS;
        const float2 t = __ffma2_rn(p, K2, M2);
        const unsigned a0 =
            __float_as_uint(t.x) * RS + cb + (lab.x == c ? (unsigned)copies * 8u : 0u);
        const unsigned a1 =
            __float_as_uint(t.y) * RS + cb + (lab.y == c ? (unsigned)copies * 8u : 0u);
        const float2 r0 = *reinterpret_cast<const float2*>(smem_raw + a0);
        const float2 r1 = *reinterpret_cast<const float2*>(smem_raw + a1);
        return make_float2(__fmaf_rn(r0.y, p.x, r0.x), __fmaf_rn(r1.y, p.y, r1.x));
      };
      // channels in groups of four (one uniform branch each); a channel outside the
      // loss channels (dropped background, or past C) has gp = 0, its record read
      // taken from the nearest loss channel's rows. Between the phases: p and gp
      // (KEEP), or for hard binning the bins, 8 bits each, two channels' pairs a
      // register (PACK: the second phase reads the records again but does not
      // search), or nothing (soft: its record address is one FMA from p).
      constexpr bool PACK = !KEEP && !SOFT;
      float2 dot = make_float2(0.0f, 0.0f);
      float2 gk[KEEP ? CM : 1];
      unsigned kp[PACK ? (CM + 1) / 2 : 1];
#pragma unroll
      for (int i = 0; i < (PACK ? (CM + 1) / 2 : 1); ++i) kp[i] = 0u;
#pragma unroll
      for (int c0 = 0; c0 < CM; c0 += 4) {
        if (c0 >= C) break;
        if constexpr (SOFT) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = c0 + j;
            const float2 p = prob(e[c]);
            const float2 g = grad(min(max(c, OFF), C - 1), p);
            const float2 gp = c >= OFF && c < C ? g : make_float2(0.0f, 0.0f);
            dot = __ffma2_rn(p, gp, dot);
            if constexpr (KEEP) {
              e[c] = p;
              gk[c] = gp;
            }
          }
        } else {
          // hard binning, as mc_fwd_kernel: the guesses and their proofs of a
          // group of G channels first, then one (rarely taken) branch for the
          // table search of the values near an edge; a channel outside the loss
          // channels keeps its guess (in 0..K, a valid record index; its gp is 0).
          // With PACK the exponentials stay in registers for the second phase, so
          // the groups are halves (fewer values live at once).
          constexpr int G = PACK ? 2 : 4;
#pragma unroll
          for (int h = 0; h < 4; h += G) {
          float2 p[G];
          unsigned k0[G], k1[G];
          bool ok = true;
#pragma unroll
          for (int j = 0; j < G; ++j) {
            const int c = c0 + h + j;
            p[j] = prob(e[c]);
            const float2 g =
                __fadd2_rn(__fadd2_rn(__fmul2_rn(p[j], K2), make_float2(-0.5f, -0.5f)), M2);
            k0[j] = min(__float_as_uint(g.x) - kFixMagicBits, (unsigned)K);
            k1[j] = min(__float_as_uint(g.y) - kFixMagicBits, (unsigned)K);
            const float2 w = mc_offset(p[j], k0[j], k1[j], KR2);
            const bool act = c >= OFF && c < C;
            ok = ok & (!act | (mc_proven(k0[j], w.x, K) & mc_proven(k1[j], w.y, K)));
          }
          if (!ok) {
#pragma unroll
            for (int j = 0; j < G; ++j) {
              const int c = c0 + h + j;
              if (c < OFF || c >= C) continue;
              if (!ace_is_count(p[j].x, my_lohi[k0[j] * kTabCopies]))
                k0[j] = (unsigned)ace_fix_count(p[j].x, (int)k0[j], K, my_lohi, kTabCopies).i;
              if (!ace_is_count(p[j].y, my_lohi[k1[j] * kTabCopies]))
                k1[j] = (unsigned)ace_fix_count(p[j].y, (int)k1[j], K, my_lohi, kTabCopies).i;
            }
          }
#pragma unroll
          for (int j = 0; j < G; ++j) {
            const int c = c0 + h + j;
            if constexpr (PACK) kp[c >> 1] |= (k0[j] | (k1[j] << 8)) << (16 * (c & 1));
            const float2 g = records(min(max(c, OFF), C - 1), make_uint2(k0[j], k1[j]));
            const float2 gp = c >= OFF && c < C ? g : make_float2(0.0f, 0.0f);
            dot = __ffma2_rn(p[j], gp, dot);
            if constexpr (KEEP) {
              e[c] = p[j];
              gk[c] = gp;
            }
          }
          }
        }
      }
      const float2 nd = make_float2(-dot.x, -dot.y);
      T* db = dxp + ((int64_t)m.y * C) * N + (int64_t)m.x * TV + vo;
#pragma unroll
      for (int c0 = 0; c0 < CM; c0 += 4) {
        if (c0 >= C) break;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = c0 + j;
          float2 p, gp;
          if constexpr (KEEP) {
            p = e[c];
            gp = gk[c];
          } else {
            p = prob(e[c]);
            float2 g;
            if constexpr (PACK) {
              const unsigned w = kp[c >> 1] >> (16 * (c & 1));
              g = records(min(max(c, OFF), C - 1), make_uint2(w & 0xffu, (w >> 8) & 0xffu));
            } else {
              g = grad(min(max(c, OFF), C - 1), p);
            }
            gp = c >= OFF && c < C ? g : make_float2(0.0f, 0.0f);
          }
          if (c < C) stg_pair<T>(db + (int64_t)c * N, __fmul2_rn(p, __fadd2_rn(gp, nd)));
        }
      }
    }
  }
  __syncthreads();
}

}  // namespace ace
