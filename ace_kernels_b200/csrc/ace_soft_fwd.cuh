// soft_fwd_kernel: the forward of soft binning with int64 class labels and a
// softmax over C <= 4 channels (the headline workload's case), on B200 (sm_100a).
// Included by ace_kernels.cuh after the shared helpers (epilogue, fixed point).
//
// It computes what hist_kernel computes for that case (the reference's
// binning.soft_stats, ace_kernels/binning.py:74-116, via the two-bin linear
// assignment of ace_kernels/common.py:43-61, then the epilogue) as a pipeline
// whose memory side never waits for its arithmetic side:
//
// - Warp specialisation and a TMA ring. One producer thread streams tiles of
//   kPipeTileVoxels voxels (the C logit rows and the labels of one batch) from
//   HBM into a ring of shared-memory stages with bulk copies
//   (cp.async.bulk ... mbarrier::complete_tx), up to `stages` tiles ahead (~80
//   to 120 KB in flight per SM). kPipeConsumerWarps consumer warps wait on a
//   stage's "full" barrier, read their 4 voxels with 16-byte shared loads, release
//   the stage on its "empty" barrier and add the voxels into the statistics.
// - Dynamic tile scheduler. The producer claims tiles from a per-batch global
//   counter, one claim ahead (its latency hides behind the stages in flight).
//   CTAs start spread over the batches; a CTA whose batch runs out moves on to
//   another batch with tiles left, so SMs that run faster take more tiles.
// - Interval coordinate without a table lookup. The value's interval j (between
//   bin centres j-1 and j; the end intervals 0 and K hold one end bin each) is
//   the rounded p K, and its coordinate is r = p K - j in [-1/2, 1/2], taken from
//   the same fused multiply-add (exact before its one rounding). The reference's
//   right-bin weight u = (p - c_{j-1}) / (c_j - c_{j-1}), with its fp32 centres,
//   is affine in r: u = a_j r + b_j. The kernel sums n, sum r and sum r^2 per
//   slot; the last CTA maps them to sum u and sum u^2 exactly (in double). (The
//   rounded p K can differ from the exact interval only for p within a few ulp of
//   a centre, where both intervals give the centre's bin the same weight ~1.)
// - Slots split by class flag: slot (j, channel c, f) with f = 1 when c is the
//   voxel's class. Every value makes exactly one update of three 32-bit words
//   (n, sum r, sum r^2), and the target moments of a row are its flag-1 slots:
//   no second update for the true class.
// - The words are integer fixed point in shared memory (r in 2^-22 units, r^2 in
//   2^-23 units: at most 1.2e-7 of rounding per value, against the loss's 1e-5
//   tolerance), updated with red.shared.add.u32 (native; a float shared-memory
//   add is a compare-and-swap loop), lane-replicated R ways so that the 32 lanes
//   of a warp never share a bank.
// - Folds add the replicas exactly in 64-bit integers and issue 64-bit integer
//   global atomics: the sums do not depend on the order of anything, so every
//   run gives the same bits whichever CTA took which tile.
//
// Every wait on a barrier is bounded (kPipeWaitNs); a wait that runs out sets
// the workspace's error word and the CTA leaves its loops (after the copies it
// issued have landed), and the last CTA then writes a NaN loss.
#pragma once

namespace ace {

constexpr int kSoftNW = 3;  // words per slot replica: n, r, r^2 (odd: no bank conflicts)
constexpr int kSoftMoments = 3;
constexpr float kSoftRScale = 4194304.0f;  // 2^22: unit of sum r (|r| <= 1/2: |r 2^22| <= 2^21)

// One value's three words into the slot replica at shared byte address a.
__device__ __forceinline__ void red_slot(unsigned a, unsigned n, unsigned r, unsigned q) {
  asm volatile(
      "red.shared.add.u32 [%0], %1;\n\t"
      "red.shared.add.u32 [%0+4], %2;\n\t"
      "red.shared.add.u32 [%0+8], %3;" ::"r"(a),
      "r"(n), "r"(r), "r"(q));
}

// Fold of the table into the workspace, by the consumer threads. Slot
// e = (j * C + c) * 2 + f of the (K + 1) * C * 2 slots; item i takes slot i >> gsh
// and part i & (G - 1) of its R replicas (G = 4 lanes per slot): it removes each
// replica's fixed-point bias with the replica's count, adds exactly in 64-bit
// integers, the G lanes combine their parts with shuffles and the first issues
// three 64-bit integer atomics (n, sum r, sum r^2) for a non-empty slot of a loss
// channel. acc layout: [3][rows][K + 1][2] (moment
// stride `ms`), rows = b_total * CL; `row0` is the global row of loss channel 0
// of the batch folded. `clear`: zero the table afterwards.
__device__ __forceinline__ void fold_soft(unsigned* hist, int C, int OFF, int K, int R,
                                          unsigned long long* acc, int64_t ms, int64_t row0,
                                          bool clear) {
  constexpr int NW = kSoftNW, NCT = kPipeConsumerWarps * 32;
  const int slots = (K + 1) * C * 2;
  const int gsh = R >= 4 ? 2 : (R == 2 ? 1 : 0);
  const int G = 1 << gsh, per = R >> gsh;
  const int total = slots << gsh;
  for (int i0 = 0; i0 < total; i0 += NCT) {  // uniform trip count: full-warp shuffles
    const int i = i0 + (int)threadIdx.x;
    const bool valid = i < total;
    const int e = valid ? i >> gsh : 0, part = i & (G - 1);
    const unsigned* base = hist + e * R * NW;
    long long sr = 0, q = 0;
    unsigned n = 0;
    if (valid) {
#pragma unroll 8
      for (int k = 0; k < per; ++k) {
        const unsigned* w = base + ((part * per + k + e) & (R - 1)) * NW;
        const unsigned cnt = w[0];
        const unsigned bias = cnt * kFixMagicBits;
        n += cnt;
        sr += (int)(w[1] - bias);
        q += (int)(w[2] - bias);
      }
    }
    for (int o = 1; o < G; o <<= 1) {
      n += __shfl_xor_sync(0xffffffffu, n, o);
      sr += __shfl_xor_sync(0xffffffffu, sr, o);
      q += __shfl_xor_sync(0xffffffffu, q, o);
    }
    if (valid && part == 0 && n != 0) {
      const int f = e & 1, jc = e >> 1;
      const int j = jc / C, c = jc - j * C;
      if (c >= OFF) {
        unsigned long long* a = acc + ((row0 + c - OFF) * (K + 1) + j) * 2 + f;
        atomicAdd(a, (unsigned long long)n);
        atomicAdd(a + ms, (unsigned long long)sr);
        atomicAdd(a + 2 * ms, (unsigned long long)q);
      }
    }
  }
  if (clear) {
    consumer_sync();
    const int words = slots * R * NW;
    uint4* h4 = reinterpret_cast<uint4*>(hist);
    for (int i = threadIdx.x; i < words / 4; i += NCT) h4[i] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = (words & ~3) + threadIdx.x; i < words; i += NCT) hist[i] = 0u;
  }
}

// Ticket of a CTA that has finished its tiles (all threads): true in the last
// CTA to finish. The ticket is a release (this CTA's sums, ordered before it by
// the barrier) and an acquire (the other CTAs' sums, for the last CTA).
__device__ __forceinline__ bool last_cta_ticket(unsigned* counter) {
  __shared__ bool s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned done;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                 : "=r"(done)
                 : "l"(counter)
                 : "memory");
    s_last = (done == gridDim.x - 1);
  }
  __syncthreads();
  return s_last;
}

// Interval constants of soft_finish, per interval j: {lo, span, a, b} (one warp
// lane per interval: indexing the parameters by a lane's own j would serialise
// the lanes of a warp on the constant bank).
__device__ __forceinline__ void stage_soft_intervals(const BinTable& tab, double4* s_iv) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, K = tab.K;
  for (int j = warp; j <= K; j += blockDim.x / 32) {
    if (lane == 0) {
      const double lo = tab.lohi[j].x, span = (double)tab.lohi[j].y - lo;
      const double invK = 1.0 / (double)K;
      s_iv[j] = make_double4(lo, span, invK / span, ((double)j * invK - lo) / span);
    }
  }
}

// The last CTA of soft_fwd_kernel and mc_fwd_kernel (soft binning; all threads of
// the CTA), one warp per row r: lane l takes bins k = l + 32 q. W, P, G of bin k
// come from the slots of intervals k and k + 1 (flags 0 and 1). Interval j in
// 1..K-1, between lo = c_{j-1} and lo + S = c_j: with r = p K - j, the
// reference's right-bin weight is u = (p - lo) / S = a r + b, a = 1 / (K S),
// b = (j / K - lo) / S (s_iv), so sum u = a R1 + b n and
// sum u^2 = a^2 R2 + 2 a b R1 + b^2 n. Bin j gets the u share, W += sum u,
// P += lo sum u + S sum u^2, G += the flag-1 slot's sum u; bin j - 1 the 1 - u
// share, W += n - sum u, P += lo n + S sum u - (lo sum u + S sum u^2), G += the
// flag-1 n - sum u. The end intervals (j = 0, K) give all of n,
// sum p = (R1 + j n) / K and the flag-1 n to bins 0 and K - 1, as the
// reference's two scatters. The warp then zeroes the row's accumulators and,
// when the epilogue is fused, runs the row's epilogue from registers.
__device__ __forceinline__ void soft_finish(const FwdParams& P, const double4* s_iv) {
  constexpr int NT = kPipeThreads;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = P.tab.K;
  const int rows = P.B_total * P.g.CL;
  const int64_t m = (int64_t)rows * (K + 1) * 2;  // moment stride of the workspace sums
  unsigned* err = P.counter + 1;
  const bool xg = P.xchg.world > 1;  // ranks combined here (xchg_send_row, xchg_finish)
  const unsigned long long epoch = xg ? xchg_epoch(P.xchg) : 0ull;
  const int64_t stat_stride = (int64_t)rows * K;
  unsigned long long* acc = P.iacc;
  const double ur = 1.0 / (double)kSoftRScale, uq = ur * 0.5, invK = 1.0 / (double)K;
  const bool failed = __ldcg(err) != 0u;  // a CTA's wait ran out: the sums are incomplete
  const float nan = __int_as_float(0x7fc00000);
  float mine = 0.0f;
  const int2 rr = xchg_rows(P);  // (batch shards: this rank's rows only)
  for (int r = rr.x + warp; r < rr.y; r += NT / 32) {
    float wv[4], pv[4], gv[4];
    const int64_t row_slot = (int64_t)r * (K + 1) * 2;
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) {
      const int k = lane + 32 * qq;
      wv[qq] = pv[qq] = gv[qq] = 0.0f;
      if (k >= K) continue;
      long long mo[kSoftMoments][4];  // [moment][slot (k,0), (k,1), (k+1,0), (k+1,1)]
#pragma unroll
      for (int o = 0; o < kSoftMoments; ++o)
#pragma unroll
        for (int q = 0; q < 4; ++q)
          mo[o][q] = (long long)__ldcg(acc + o * m + row_slot + 2 * k + q);
      double w = 0.0, pp = 0.0, gs = 0.0;
#pragma unroll
      for (int side = 0; side < 2; ++side) {
        const int j = k + side;
        double n[2], r1[2], r2[2];
#pragma unroll
        for (int f = 0; f < 2; ++f) {
          const int q = 2 * side + f;
          n[f] = (double)mo[0][q];
          r1[f] = (double)mo[1][q] * ur;
          r2[f] = (double)mo[2][q] * uq;
        }
        if (j == 0 || j == K) {
          w += n[0] + n[1];
          pp += (r1[0] + r1[1] + (double)j * (n[0] + n[1])) * invK;
          gs += n[1];
          continue;
        }
        const double4 iv = s_iv[j];
        const double lo = iv.x, span = iv.y, a = iv.z, bb = iv.w;
        double su[2], su2 = 0.0;
#pragma unroll
        for (int f = 0; f < 2; ++f) {
          su[f] = a * r1[f] + bb * n[f];
          su2 += a * a * r2[f] + 2.0 * a * bb * r1[f] + bb * bb * n[f];
        }
        const double nt = n[0] + n[1], sut = su[0] + su[1];
        const double pt = lo * sut + span * su2;  // sum u p
        if (side == 0) {
          w += sut;
          pp += pt;
          gs += su[1];
        } else {
          w += nt - sut;
          pp += lo * nt + span * sut - pt;
          gs += n[1] - su[1];
        }
      }
      wv[qq] = failed ? nan : (float)w;
      pv[qq] = failed ? nan : (float)pp;
      gv[qq] = failed ? nan : (float)gs;
      const int64_t e = (int64_t)r * K + k;
      P.hist_out[e] = wv[qq];
      P.hist_out[stat_stride + e] = pv[qq];
      P.hist_out[2 * stat_stride + e] = gv[qq];
    }
    __syncwarp();  // every lane has read the row's slots
    for (int j = lane; j <= K; j += 32)
#pragma unroll
      for (int o = 0; o < kSoftMoments; ++o)
#pragma unroll
        for (int f = 0; f < 2; ++f) __stcg(acc + o * m + row_slot + 2 * j + f, 0ull);
    if (xg && P.xchg.own_rows) {
      const float f = epilogue_row(P.epi, r, wv, pv, gv);
      xchg_send_f(P, epoch, r, f);
      if (lane == 0) xchg_row_f()[r] = f;
    } else if (xg) {
      xchg_send_row(P, epoch, r, wv, pv, gv);
    } else if (P.do_epilogue) {
      mine = ACE_FADD(mine, epilogue_row(P.epi, r, wv, pv, gv));
    }
  }
  if (xg) mine = P.xchg.own_rows ? xchg_finish_f(P, epoch) : xchg_finish(P, epoch);
  for (int i = tid; i < P.g.B; i += NT) P.pool_ctr[i] = 0u;
  if (P.do_epilogue) write_loss_if0(P.epi, cta_sum_in_warp_order(mine));
  __syncthreads();
  if (tid == 0) {
    *err = 0u;
    *P.counter = 0u;
  }
}

template <typename T, int C, int OFF>
__global__ void __launch_bounds__(kPipeThreads, 1) soft_fwd_kernel(const __grid_constant__ FwdParams P) {
  constexpr int NCW = kPipeConsumerWarps, NT = kPipeThreads, NW = kSoftNW;
  constexpr int TV = kPipeTileVoxels, VL = kPipeLaneVoxels;
  constexpr unsigned XB = TV * sizeof(T);  // bytes of one logit row of a stage
  constexpr unsigned SB = C * XB + TV * 8;  // bytes of a stage (rows, then labels)
  static_assert(VL == 4, "lds_logits / lds_labels load four voxels");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) unsigned long long s_full[kPipeMaxStages], s_empty[kPipeMaxStages];
  __shared__ int4 s_meta[kPipeMaxStages];  // {tile, batch, voxels, 0}; tile < 0: no more tiles
  __shared__ volatile int s_abort;
  __shared__ double4 s_iv[kMaxBins + 1];  // soft_finish's interval constants
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int CL = C - OFF;
  const int K = P.tab.K, R = P.R, S = P.stages;
  const int64_t N = P.g.N;
  unsigned* hist = reinterpret_cast<unsigned*>(smem_raw);
  const int table_words = (K + 1) * C * 2 * R * NW;
  const unsigned stage0 = smem_addr(smem_raw) + (unsigned)P.table_bytes;
  auto full_bar = [&](int s) { return smem_addr(&s_full[s]); };
  auto empty_bar = [&](int s) { return smem_addr(&s_empty[s]); };
  {
    uint4* h4 = reinterpret_cast<uint4*>(hist);
    for (int i = tid; i < table_words / 4; i += NT) h4[i] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = (table_words & ~3) + tid; i < table_words; i += NT) hist[i] = 0u;
  }
  stage_soft_intervals(P.tab, s_iv);
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1u);
      mbar_init(empty_bar(s), (unsigned)NCW);
    }
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  // programmatic dependent launch: global memory only after the previous grid
  ace_grid_dependency_wait();
  __syncthreads();

  unsigned* err = P.counter + 1;  // the workspace's error word
  auto abort_cta = [&]() {
    s_abort = 1;
    atomicExch(err, 1u);
  };
  const int64_t mstride = (int64_t)P.B_total * CL * (K + 1) * 2;
  const int B = P.g.B;
  const int64_t tpb = P.wt_batch;  // tiles per batch

  if (warp == NCW) {
    // ---------------- producer (one thread) ----------------
    if (lane == 0)
      produce_claimed<T, TV>(static_cast<const T*>(P.x), static_cast<const int64_t*>(P.target), C,
                             C, N, B, tpb, P.pool_ctr, stage0, SB, S, s_full, s_empty, s_meta,
                             &s_abort, err);
  } else {
    // ---------------- consumers ----------------
    // Shared byte address of row c, flag 0, of the interval whose rounding
    // pattern is t (bits(t) - magic = j): bits(t) * A + base[c] (mod 2^32).
    const unsigned sb = (unsigned)(R * NW * 4);  // bytes of one slot (all replicas)
    const unsigned A = 2u * C * sb;               // bytes of one interval
    unsigned base[C];
    {
      const unsigned t0 =
          smem_addr(hist) + (unsigned)((lane & (R - 1)) * NW * 4) - kFixMagicBits * A;
#pragma unroll
      for (int c = 0; c < C; ++c) base[c] = t0 + (unsigned)c * 2u * sb;
    }
    const float Kf = (float)K, KfS = (float)K * kSoftRScale;
    const int vo = (warp * 32 + lane) * VL;  // this lane's first voxel of a tile
    int cur_b = -1, since = 0;
    for (int i = 0;; ++i) {
      const int s = i % S;
      if (!mbar_wait(full_bar(s), (unsigned)(i / S) & 1u)) {
        abort_cta();
        break;
      }
      const int4 m = s_meta[s];
      if (m.x < 0 || s_abort) break;
      if (m.y != cur_b || since == P.epoch) {
        // a new batch, or the 32-bit words' range: fold the table first
        if (cur_b >= 0) {
          consumer_sync();
          fold_soft(hist, C, OFF, K, R, P.iacc, mstride, (int64_t)(P.b_offset + cur_b) * CL, true);
          consumer_sync();
        }
        cur_b = m.y;
        since = 0;
      }
      ++since;
      const unsigned st = stage0 + (unsigned)s * SB;
      float xv[C][4];
      int lab[4];
#pragma unroll
      for (int c = 0; c < C; ++c) lds_logits<T>(st + c * XB + vo * (unsigned)sizeof(T), xv[c]);
      lds_labels(st + C * XB + vo * 8u, lab);
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(s));  // the stage may be refilled now
      if (vo >= m.z) continue;                    // past the batch's last voxel
      // Two voxels at a time: the fp32 arithmetic runs as packed pairs
      // (__ffma2_rn / __fmul2_rn / __fadd2_rn, one instruction for both voxels,
      // each element rounded as its scalar form), the rest per voxel.
#pragma unroll
      for (int v = 0; v < VL; v += 2) {
        // softmax: exp(x - m) = 2^(x log2 e - m log2 e) (ace_softmax_fast)
        float2 xp[C], e[C];
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
#pragma unroll
        for (int c = OFF; c < C; ++c) {
          // p in [0, 1] (NaN -> 0); t = magic + j, j = round(p K) in [0, K]
          const float2 p = make_float2(__saturatef(__fmul_rn(e[c].x, y.x)),
                                       __saturatef(__fmul_rn(e[c].y, y.y)));
          const float2 t = __ffma2_rn(p, make_float2(Kf, Kf), make_float2(kFixMagic, kFixMagic));
          // rs = (p K - j) 2^22, exact before its one rounding (|rs| <= 2^21)
          const float2 mj = __ffma2_rn(t, make_float2(-kSoftRScale, -kSoftRScale),
                                       make_float2(kFixMagic * kSoftRScale, kFixMagic * kSoftRScale));
          const float2 rs = __ffma2_rn(p, make_float2(KfS, KfS), mj);
          // magic + round(rs); magic + round(r^2 2^23) = magic + round(rs^2 2^-21)
          const float2 rw = __fadd2_rn(rs, make_float2(kFixMagic, kFixMagic));
          const float2 q = __ffma2_rn(
              rs, __fmul2_rn(rs, make_float2(1.0f / kFixScale, 1.0f / kFixScale)),
              make_float2(kFixMagic, kFixMagic));
          unsigned a0 = __float_as_uint(t.x) * A + base[c];
          unsigned a1 = __float_as_uint(t.y) * A + base[c];
          if (lab[v] == c) a0 += sb;
          if (lab[v + 1] == c) a1 += sb;
          red_slot(a0, 1u, __float_as_uint(rw.x), __float_as_uint(q.x));
          red_slot(a1, 1u, __float_as_uint(rw.y), __float_as_uint(q.y));
        }
      }
    }
    consumer_sync();
    if (cur_b >= 0)
      fold_soft(hist, C, OFF, K, R, P.iacc, mstride, (int64_t)(P.b_offset + cur_b) * CL, false);
  }

  ace_launch_dependents();  // a dependent launch may begin its own setup now
  if (last_cta_ticket(P.counter)) soft_finish(P, s_iv);
}

}  // namespace ace
