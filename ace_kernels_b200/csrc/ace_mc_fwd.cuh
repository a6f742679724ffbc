// mc_fwd_kernel: the forward of a softmax over 5 to 24 channels with int64 class
// labels, soft or hard binning, on B200 (sm_100a). Included by ace_kernels.cuh
// after ace_soft_fwd.cuh, whose pipeline it shares: the producer thread and its
// per-batch tile claims (produce_claimed), the ring of stages filled by bulk
// copies, the bounded waits, the exact integer folds into the workspace and, for
// soft binning, the interval moments and the last CTA's reconstruction
// (soft_finish).
//
// It computes the reference's binning.hard_stats / soft_stats
// (ace_kernels/binning.py:54-116) with the activation fused, then the epilogue.
// What differs from soft_fwd_kernel is shaped by the channel count:
//
// - Voxel pairs. A consumer lane takes two voxels of a 1024-voxel tile, so the
//   fp32 arithmetic runs on packed pairs (__ffma2_rn / __fmul2_rn / __fadd2_rn,
//   each element rounded as its scalar form). The channel maximum of a 16-bit pair
//   is one max.bf16x2 / max.f16x2 per channel (exact, so equal to the maximum of
//   the widened values). The pair's exponentials of all C channels stay in
//   registers between their sum and the binning: each logit is read from shared
//   memory twice (maximum, exponential) and exponentiated once.
// - Interval-0 aggregates (soft binning, up to 16 channels). In a softmax over
//   many classes most values are tiny: in the benchmark's 14-class case about half
//   of them fall in interval 0 outside the true class. Those skip the table:
//   lane-private register words agg[c] (count from bit 26, the sum of the values'
//   2^-22 words below) take them with one add each, and a fold adds the words of
//   all lanes with two warp reductions per channel.
// - Hard binning keeps the exact softmax (CUDA's expf, the Markstein-corrected
//   quotient) of hist_kernel, so every value lands in the bin the backward and the
//   test hook give it. The bin is ace_guess's, proven by the value's in-bin offset
//   r = p K - k (one fused multiply-add from p, exact before its one rounding)
//   lying well inside the bin, and found by the table search only near an edge.
//   Per (bin k, channel) slot the kernel sums n and r in 2^-20 units (bin k's P is
//   then (k n + sum r) / K, within 2^-21 / K of the exact sum per value), and per
//   voxel it counts the true class in its bin.
// - Soft binning keeps soft_fwd_kernel's fast softmax, interval coordinate and
//   class-flag slots.
//
// Word ranges. A table word takes at most 1024 / R values a tile (R lane
// replicas), each below 2^20 + 1 units (hard) or 2^21 (soft), so 2R - 1 (hard) or
// R - 1 (soft) tiles keep its sum below 2^31 in magnitude; an aggregate takes at
// most 2 values a tile, so 15 tiles keep its sum below 2^26 and its count below
// 64. The host's epoch (tiles between folds; a fold also comes at each change of
// batch) respects both.
#pragma once

namespace ace {

constexpr int kMcLaneVoxels = 2;
constexpr int kMcTileVoxels = kPipeConsumerWarps * 32 * kMcLaneVoxels;  // 1024
constexpr int kMcMinChannels = 5, kMcMaxChannels = 24;
constexpr int kMcAggEpoch = 15;  // tiles between folds with interval-0 aggregates
constexpr float kMcRScale = 1048576.0f;  // 2^20: unit of a hard value's in-bin offset
// Offsets (2^-20 units of p K) this far from a bin's ends prove the bin: the table's
// edges lie within 2^-22 relative of (k + 1) / K, i.e. under 32 units for K <= 128.
constexpr int kMcEdgeMargin = 64;
constexpr int kMcAggShift = 26;  // interval-0 aggregate: count from bit 26, sum below

// Fold of the hard table into the workspace, by the consumer threads (as
// fold_soft). Slot e = k * C + c of the K * C slots holds, per replica, the words
// n, magic-biased sum of r, and the true-class count; acc layout [3][rows][K]
// (moment stride `ms`); `row0` is the global row of loss channel 0 of the batch.
__device__ __forceinline__ void fold_hard(unsigned* hist, int C, int OFF, int K, int R,
                                          unsigned long long* acc, int64_t ms, int64_t row0,
                                          bool clear) {
  constexpr int NW = 3, NCT = kPipeConsumerWarps * 32;
  const int slots = K * C;
  const int gsh = R >= 4 ? 2 : (R == 2 ? 1 : 0);
  const int G = 1 << gsh, per = R >> gsh;
  const int total = slots << gsh;
  for (int i0 = 0; i0 < total; i0 += NCT) {  // uniform trip count: full-warp shuffles
    const int i = i0 + (int)threadIdx.x;
    const bool valid = i < total;
    const int e = valid ? i >> gsh : 0, part = i & (G - 1);
    const unsigned* base = hist + e * R * NW;
    long long sr = 0;
    unsigned n = 0, nt = 0;
    if (valid) {
#pragma unroll 8
      for (int k = 0; k < per; ++k) {
        const unsigned* w = base + ((part * per + k + e) & (R - 1)) * NW;
        const unsigned cnt = w[0];
        n += cnt;
        sr += (int)(w[1] - cnt * kFixMagicBits);
        nt += w[2];
      }
    }
    for (int o = 1; o < G; o <<= 1) {
      n += __shfl_xor_sync(0xffffffffu, n, o);
      sr += __shfl_xor_sync(0xffffffffu, sr, o);
      nt += __shfl_xor_sync(0xffffffffu, nt, o);
    }
    if (valid && part == 0 && (n | nt) != 0u) {
      const int k = e / C, c = e - k * C;
      if (c >= OFF) {
        unsigned long long* a = acc + (row0 + c - OFF) * K + k;
        if (n != 0u) {
          atomicAdd(a, (unsigned long long)n);
          atomicAdd(a + ms, (unsigned long long)sr);
        }
        if (nt != 0u) atomicAdd(a + 2 * ms, (unsigned long long)nt);
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

// Adds the consumer warps' aggregates s_agg[warp][c] = {count, sum} of interval
// 0, flag 0, of every loss channel to the workspace's n and sum-r sums of that
// slot: one thread per channel adds the 16 warps' in 64 bits and issues two
// atomics. By the consumer threads, after a consumer barrier.
template <int CM>
__device__ __forceinline__ void add_agg_sums(const uint2 (*s_agg)[CM], int C, int OFF, int K,
                                             unsigned long long* acc, int64_t ms, int64_t row0) {
  const int c = threadIdx.x;
  if (c >= OFF && c < C) {
    unsigned long long n = 0, s = 0;
    for (int w = 0; w < kPipeConsumerWarps; ++w) {
      n += s_agg[w][c].x;
      s += s_agg[w][c].y;
    }
    if (n != 0) {
      unsigned long long* a = acc + (row0 + c - OFF) * (K + 1) * 2;
      atomicAdd(a, n);
      atomicAdd(a + ms, s);
    }
  }
}

// The last CTA of mc_fwd_kernel, hard binning (all threads of the CTA), one warp
// per row r, lane l taking bins k = l + 32 q: W = n, P = (k n + sum r 2^-20) / K
// (in double), G = the true-class count. The warp zeroes the row's sums after
// reading them and, when the epilogue is fused, runs the row's epilogue.
__device__ __forceinline__ void hard_finish(const FwdParams& P) {
  constexpr int NT = kPipeThreads;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = P.tab.K;
  const int rows = P.B_total * P.g.CL;
  const int64_t m = (int64_t)rows * K;  // moment stride of the sums, and of W, P, G
  unsigned long long* acc = P.iacc;
  unsigned* err = P.counter + 1;
  const bool failed = __ldcg(err) != 0u;  // a CTA's wait ran out: the sums are incomplete
  const float nan = __int_as_float(0x7fc00000);
  const double ur = 1.0 / (double)kMcRScale, invK = 1.0 / (double)K;
  const bool xg = P.xchg.world > 1;  // ranks combined here (xchg_send_row, xchg_finish)
  const unsigned long long epoch = xg ? xchg_epoch(P.xchg) : 0ull;
  float mine = 0.0f;
  const int2 rr = xchg_rows(P);  // (batch shards: this rank's rows only)
  for (int r = rr.x + warp; r < rr.y; r += NT / 32) {
    float wv[4], pv[4], gv[4];
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) {
      const int k = lane + 32 * qq;
      wv[qq] = pv[qq] = gv[qq] = 0.0f;
      if (k >= K) continue;
      const int64_t e = (int64_t)r * K + k;
      const unsigned long long n = __ldcg(acc + e), nt = __ldcg(acc + 2 * m + e);
      const long long sr = (long long)__ldcg(acc + m + e);
      __stcg(acc + e, 0ull);
      __stcg(acc + m + e, 0ull);
      __stcg(acc + 2 * m + e, 0ull);
      wv[qq] = failed ? nan : (float)n;
      pv[qq] = failed ? nan : (float)(((double)k * (double)n + (double)sr * ur) * invK);
      gv[qq] = failed ? nan : (float)nt;
      P.hist_out[e] = wv[qq];
      P.hist_out[m + e] = pv[qq];
      P.hist_out[2 * m + e] = gv[qq];
    }
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

// Shared-memory reductions of one value under a condition. The soft path's is a
// C++ condition (the compiler branches or predicates), the hard path's are forced
// predicated instructions: each was measured the faster one for its path.
__device__ __forceinline__ void red_slot_if(bool on, unsigned a, unsigned n, unsigned r,
                                            unsigned q) {
  if (on) red_slot(a, n, r, q);
}
__device__ __forceinline__ void red_pair_if(bool on, unsigned a, unsigned n, unsigned r) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.u32 p, %0, 0;\n\t"
      "@p red.shared.add.u32 [%1], %2;\n\t"
      "@p red.shared.add.u32 [%1+4], %3;\n\t}" ::"r"((unsigned)on),
      "r"(a), "r"(n), "r"(r));
}
__device__ __forceinline__ void red_one_if(bool on, unsigned a, unsigned n) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.u32 p, %0, 0;\n\t"
      "@p red.shared.add.u32 [%1], %2;\n\t}" ::"r"((unsigned)on),
      "r"(a), "r"(n));
}

// A stage of mc_fwd_kernel holds CM logit rows: the tile's C rows, then
// CM - C rows of -inf written once at kernel start (the bulk copies never touch
// them). A padding row leaves a pair's maximum unchanged and its exponential is
// exactly 0, so the channel loops need neither a clamp nor a select for them.
template <typename T>
struct NegInfWord;  // a 32-bit word of -inf values of type T
template <>
struct NegInfWord<float> {
  static constexpr unsigned value = 0xff800000u;
};
template <>
struct NegInfWord<__half> {
  static constexpr unsigned value = 0xfc00fc00u;
};
template <>
struct NegInfWord<__nv_bfloat16> {
  static constexpr unsigned value = 0xff80ff80u;
};

template <typename T>
__device__ __forceinline__ void fill_padding_rows(unsigned char* stage0, int S, unsigned SB,
                                                  int C, int CM) {
  constexpr unsigned XB = kMcTileVoxels * sizeof(T);
  const unsigned neg_inf = NegInfWord<T>::value;
  const int words = (int)(XB / 4) * (CM - C);
  for (int s = 0; s < S; ++s) {
    unsigned* w = reinterpret_cast<unsigned*>(stage0 + (size_t)s * SB + (size_t)C * XB);
    for (int i = threadIdx.x; i < words; i += blockDim.x) w[i] = neg_inf;
  }
}

// The pair's channel maximum and exponentials (ascending channels) and their sum,
// from a stage: `my` is the lane's pair in channel row 0. Channels go in groups of
// four with one (uniform) branch per group, so the group's four chains are
// straight-line code the compiler interleaves. A channel c >= C of the last group
// reads a -inf padding row (PAD: fill_padding_rows), or row C - 1 (a repeated row
// leaves the maximum unchanged) and is then left out of the sum; e[c] is 0 or
// unused. (The forward measured faster with the padding, the soft backward
// slower: its extra registers spill.)
// SOFT: ace_softmax_fast's 2^(x log2 e - m log2 e); else ace_softmax's expf(x - m).
template <typename T, int CM, bool SOFT, bool PAD>
__device__ __forceinline__ float2 pair_exponentials(const unsigned char* my, int C, float2 (&e)[CM]) {
  constexpr unsigned XB = kMcTileVoxels * sizeof(T);
  auto row = [&](int c) { return PAD ? c : min(c, C - 1); };
  float2 mx;
  if constexpr (sizeof(T) == 4) {
    mx = ld_pair<float>(my);
#pragma unroll
    for (int c0 = 0; c0 < CM; c0 += 4) {
      if (c0 >= C) break;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 x = ld_pair<float>(my + row(c0 + j) * XB);
        mx = make_float2(fmaxf(mx.x, x.x), fmaxf(mx.y, x.y));
      }
    }
  } else {
    unsigned mw = *reinterpret_cast<const unsigned*>(my);
#pragma unroll
    for (int c0 = 0; c0 < CM; c0 += 4) {
      if (c0 >= C) break;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        mw = max2<T>(mw, *reinterpret_cast<const unsigned*>(my + row(c0 + j) * XB));
    }
    mx = widen2<T>(mw);
  }
  const float2 nm =
      SOFT ? __fmul2_rn(mx, make_float2(-kLog2e, -kLog2e)) : make_float2(-mx.x, -mx.y);
  float2 sum = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int c0 = 0; c0 < CM; c0 += 4) {
    if (c0 >= C) break;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = c0 + j;
      const float2 x = ld_pair<T>(my + row(c) * XB);
      if constexpr (SOFT) {
        const float2 arg = __ffma2_rn(x, make_float2(kLog2e, kLog2e), nm);
        e[c] = make_float2(ace_exp2_approx(arg.x), ace_exp2_approx(arg.y));
      } else {
        const float2 d = __fadd2_rn(x, nm);
        e[c] = make_float2(expf(d.x), expf(d.y));
      }
      sum = __fadd2_rn(sum, PAD || c < C ? e[c] : make_float2(0.0f, 0.0f));
    }
  }
  return sum;
}

// magic + round((p K - k) 2^20) for the pair's bins k0, k1 (exact before its one
// rounding: magic - k 2^20 is exact, and p (K 2^20) is exact inside the FMA).
__device__ __forceinline__ float2 mc_offset(float2 p, unsigned k0, unsigned k1, float2 KR2) {
  const float2 kf = __fadd2_rn(
      make_float2(__uint_as_float(k0 + kFixMagicBits), __uint_as_float(k1 + kFixMagicBits)),
      make_float2(-kFixMagic, -kFixMagic));
  return __ffma2_rn(p, KR2, __ffma2_rn(kf, make_float2(-kMcRScale, -kMcRScale),
                                       make_float2(kFixMagic, kFixMagic)));
}

// Whether bin k of a value with offset word w is certain without the table: the
// offset lies kMcEdgeMargin units (of 2^-20) or more inside the bin's interior.
__device__ __forceinline__ bool mc_proven(unsigned k, float w, int K) {
  const int v = (int)(__float_as_uint(w) - kFixMagicBits);
  return k < (unsigned)K && v <= (1 << 20) - kMcEdgeMargin && (k == 0u || v >= kMcEdgeMargin);
}

template <typename T, int CM, bool SOFT>
__global__ void __launch_bounds__(kPipeThreads, 1) mc_fwd_kernel(const __grid_constant__ FwdParams P) {
  constexpr int NCW = kPipeConsumerWarps, NT = kPipeThreads, NW = 3;
  constexpr int TV = kMcTileVoxels;
  constexpr unsigned XB = TV * sizeof(T);  // bytes of one logit row of a stage
  static_assert(CM <= 32, "lane c keeps channel c's aggregate at fold time");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ __align__(8) unsigned long long s_full[kPipeMaxStages], s_empty[kPipeMaxStages];
  __shared__ int4 s_meta[kPipeMaxStages];  // {tile, batch, voxels, 0}; tile < 0: no more tiles
  __shared__ volatile int s_abort;
  __shared__ uint2 s_agg[SOFT && CM <= 16 ? NCW : 1][CM];  // per warp, channel: {count, sum}
  __shared__ double4 s_iv[SOFT ? kMaxBins + 1 : 1];  // soft_finish's interval constants
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int C = P.g.C, OFF = P.g.offset, CL = C - OFF;
  const int K = P.tab.K, R = P.R, S = P.stages;
  const int64_t N = P.g.N;
  const unsigned SB = (unsigned)CM * XB + TV * 8u;  // bytes of a stage (CM rows, then labels)
  // shared memory: the table [slots][R][3] words, (hard) the bin-edge table
  // [K + 1][kTabCopies] float2, then the ring of stages
  unsigned* hist = reinterpret_cast<unsigned*>(smem_raw);
  const int slots = SOFT ? (K + 1) * C * 2 : K * C;
  const int table_words = slots * R * NW;
  float2* lohi_t = reinterpret_cast<float2*>(smem_raw + P.table_bytes);
  const unsigned stage0 = smem_addr(smem_raw) + (unsigned)P.stage_offset;
  auto full_bar = [&](int s) { return smem_addr(&s_full[s]); };
  auto empty_bar = [&](int s) { return smem_addr(&s_empty[s]); };
  {
    uint4* h4 = reinterpret_cast<uint4*>(hist);
    for (int i = tid; i < table_words / 4; i += NT) h4[i] = make_uint4(0u, 0u, 0u, 0u);
    for (int i = (table_words & ~3) + tid; i < table_words; i += NT) hist[i] = 0u;
  }
  if constexpr (SOFT) {
    stage_soft_intervals(P.tab, s_iv);
  } else {
    for (int i = tid; i < (K + 1) * kTabCopies; i += NT) lohi_t[i] = P.tab.lohi[i / kTabCopies];
  }
  fill_padding_rows<T>(smem_raw + P.stage_offset, S, SB, C, CM);
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
  const int64_t mstride = SOFT ? (int64_t)P.B_total * CL * (K + 1) * 2 : (int64_t)P.B_total * CL * K;

  if (warp == NCW) {
    // ---------------- producer (one thread) ----------------
    if (lane == 0)
      produce_claimed<T, TV>(static_cast<const T*>(P.x), static_cast<const int64_t*>(P.target), C,
                             CM, N, P.g.B, P.wt_batch, P.pool_ctr, stage0, SB, S, s_full, s_empty,
                             s_meta, &s_abort, err);
  } else {
    // ---------------- consumers ----------------
    // Slot addresses (bytes, this lane's replica): hard, slot (k, c) at
    // k * A + c * CS + lane0; soft, slot (j, c, f) at bits(t) * A + c * CS + f * sb
    // + tb with t = magic + j (mod 2^32).
    const unsigned sb = (unsigned)(R * NW * 4);  // bytes of one slot (all replicas)
    const unsigned CS = SOFT ? 2u * sb : sb;      // bytes of one channel's slots of a bin
    const unsigned A = (unsigned)C * CS;          // bytes of one bin / interval
    const unsigned lane0 = smem_addr(hist) + (unsigned)((lane & (R - 1)) * NW * 4);
    const unsigned tb = SOFT ? lane0 - kFixMagicBits * A : lane0;
    const float2* my_lohi = lohi_t + (lane & (kTabCopies - 1));
    const float Kf = (float)K;
    const float2 K2 = make_float2(Kf, Kf);
    const float2 M2 = make_float2(kFixMagic, kFixMagic);
    // Interval-0 aggregates (see the file comment), soft binning with CM <= 16:
    // lane-private packed words agg[c] (with more channels they would not fit in
    // the registers beside the exponentials, and the values go to the table).
    constexpr bool AGG = SOFT && CM <= 16;
    constexpr int SH = kMcAggShift;
    unsigned agg[AGG ? CM : 1];
#pragma unroll
    for (int c = 0; c < (AGG ? CM : 1); ++c) agg[c] = 0u;
    // the lanes' aggregates into s_agg[warp][c] = {count, sum}, then zeroed
    auto stash_agg = [&]() {
      if constexpr (AGG) {
#pragma unroll
        for (int c = 0; c < CM; ++c) {
          if (c < C) {
            const unsigned n = __reduce_add_sync(0xffffffffu, agg[c] >> SH);
            const unsigned sm = __reduce_add_sync(0xffffffffu, agg[c] & ((1u << SH) - 1u));
            if (lane == 0) s_agg[warp][c] = make_uint2(n, sm);
            agg[c] = 0u;
          }
        }
      }
    };
    auto fold_all = [&](int64_t row0, bool clear) {
      if constexpr (AGG) {
        stash_agg();
        consumer_sync();
        add_agg_sums<CM>(s_agg, C, OFF, K, P.iacc, mstride, row0);
      }
      if constexpr (SOFT) fold_soft(hist, C, OFF, K, R, P.iacc, mstride, row0, clear);
      else fold_hard(hist, C, OFF, K, R, P.iacc, mstride, row0, clear);
    };
    const int vo = (warp * 32 + lane) * kMcLaneVoxels;  // this lane's first voxel of a tile
    int cur_b = -1, since = 0;
    for (int i = 0;; ++i) {
      const int s = i % S;
      if (!mbar_wait(full_bar(s), (unsigned)(i / S) & 1u)) {
        s_abort = 1;
        atomicExch(err, 1u);
        break;
      }
      const int4 m = s_meta[s];
      if (m.x < 0 || s_abort) break;
      if (m.y != cur_b || since == P.epoch) {
        // a new batch, or the 32-bit words' range: fold the aggregates and the table
        if (cur_b >= 0) {
          consumer_sync();
          fold_all((int64_t)(P.b_offset + cur_b) * CL, true);
          consumer_sync();
        }
        cur_b = m.y;
        since = 0;
      }
      ++since;
      const unsigned char* st = smem_raw + P.stage_offset + (size_t)s * SB;
      const unsigned char* my = st + (size_t)vo * sizeof(T);
      const int2 lab = ld_labels2(st + (size_t)CM * XB + (size_t)vo * 8);
      float2 e[CM];
      const float2 sum = pair_exponentials<T, CM, SOFT, true>(my, C, e);
      __syncwarp();
      if (lane == 0) mbar_arrive(empty_bar(s));  // the stage may be refilled now
      if (warp * 32 * kMcLaneVoxels >= m.z) continue;  // the whole warp is past the batch's end
      const bool valid = vo < m.z;                       // this lane's pair (N is even)
      if constexpr (SOFT) {
        const float2 y = make_float2(ace_rcp_approx(sum.x), ace_rcp_approx(sum.y));
        const float KfS = Kf * kSoftRScale;
#pragma unroll
        for (int c0 = 0; c0 < CM; c0 += 4) {
          if (c0 >= C) break;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int c = c0 + j;
            const bool act = valid && c >= OFF && c < C;
            // as soft_fwd_kernel: p in [0, 1]; t = magic + j, j = round(p K);
            // rs = (p K - j) 2^22 (exact before its one rounding)
            const float2 p = make_float2(__saturatef(__fmul_rn(e[c].x, y.x)),
                                         __saturatef(__fmul_rn(e[c].y, y.y)));
            const float2 t = __ffma2_rn(p, K2, M2);
            const float2 mj =
                __ffma2_rn(t, make_float2(-kSoftRScale, -kSoftRScale),
                           make_float2(kFixMagic * kSoftRScale, kFixMagic * kSoftRScale));
            const float2 rs = __ffma2_rn(p, make_float2(KfS, KfS), mj);
            const float2 rw = __fadd2_rn(rs, M2);
            const float2 q = __ffma2_rn(
                rs, __fmul2_rn(rs, make_float2(1.0f / kFixScale, 1.0f / kFixScale)), M2);
            const unsigned t0 = __float_as_uint(t.x), t1 = __float_as_uint(t.y);
            const bool f0 = lab.x == c, f1 = lab.y == c;
            const bool z0 = AGG && act && t0 == kFixMagicBits && !f0;
            const bool z1 = AGG && act && t1 == kFixMagicBits && !f1;
            const unsigned cb = tb + (unsigned)c * CS;
            if constexpr (AGG)
              agg[c] += (z0 ? __float_as_uint(rw.x) - kFixMagicBits + (1u << SH) : 0u) +
                        (z1 ? __float_as_uint(rw.y) - kFixMagicBits + (1u << SH) : 0u);
            red_slot_if(act && !z0, t0 * A + cb + (f0 ? sb : 0u), 1u, __float_as_uint(rw.x),
                        __float_as_uint(q.x));
            red_slot_if(act && !z1, t1 * A + cb + (f1 ? sb : 0u), 1u, __float_as_uint(rw.y),
                        __float_as_uint(q.y));
          }
        }
      } else {
        // p = e / sum with one refined reciprocal per voxel (ace_softmax)
        const float2 y = make_float2(ace_rcp_refined(sum.x), ace_rcp_refined(sum.y));
        const float2 ns = make_float2(-sum.x, -sum.y);
        const float2 KR2 = make_float2(Kf * kMcRScale, Kf * kMcRScale);
        unsigned kt0 = (unsigned)K, kt1 = (unsigned)K;  // the true class's bin (K: none)
        // Channels in groups of four (two above 8 channels, where the exponentials
        // of all channels fill most registers). The bin of a value is the guess k of
        // ace_guess; w = magic + round((p K - k) 2^20) is its in-bin offset, from one
        // fused multiply-add. An offset at least kMcEdgeMargin units inside (0, 2^20)
        // (for k = 0 only below the top) proves k: every edge of the bin table lies
        // within 2^-22 relative of its multiple of 1 / K, far less than the margin.
        // The rare values that fail (within the margin of an edge, or k = K) take
        // the table search of ace_locate, and their w is recomputed. A lane past the
        // batch's end, and a channel outside the loss channels, get bin K (no bin).
        constexpr int G = CM > 8 ? 2 : 4;
#pragma unroll
        for (int c0 = 0; c0 < CM; c0 += G) {
          if (c0 >= C) break;
          float2 p[G], w[G];
          unsigned k0[G], k1[G];
          bool ok = true;
#pragma unroll
          for (int j = 0; j < G; ++j) {
            const int c = c0 + j;
            const float2 q0 = __fmul2_rn(e[c], y);
            p[j] = __ffma2_rn(__ffma2_rn(ns, q0, e[c]), y, q0);
            const float2 g =
                __fadd2_rn(__fadd2_rn(__fmul2_rn(p[j], K2), make_float2(-0.5f, -0.5f)), M2);
            k0[j] = min(__float_as_uint(g.x) - kFixMagicBits, (unsigned)K);
            k1[j] = min(__float_as_uint(g.y) - kFixMagicBits, (unsigned)K);
            w[j] = mc_offset(p[j], k0[j], k1[j], KR2);
            const bool act = c >= OFF && c < C;
            ok = ok & (!act | (mc_proven(k0[j], w[j].x, K) & mc_proven(k1[j], w[j].y, K)));
          }
          if (!ok && valid) {
#pragma unroll
            for (int j = 0; j < G; ++j) {
              const int c = c0 + j;
              if (c < OFF || c >= C) continue;
              if (!ace_is_count(p[j].x, my_lohi[k0[j] * kTabCopies]))
                k0[j] = (unsigned)ace_fix_count(p[j].x, (int)k0[j], K, my_lohi, kTabCopies).i;
              if (!ace_is_count(p[j].y, my_lohi[k1[j] * kTabCopies]))
                k1[j] = (unsigned)ace_fix_count(p[j].y, (int)k1[j], K, my_lohi, kTabCopies).i;
              w[j] = mc_offset(p[j], k0[j], k1[j], KR2);
            }
          }
#pragma unroll
          for (int j = 0; j < G; ++j) {
            const int c = c0 + j;
            if (!valid || c < OFF || c >= C) k0[j] = k1[j] = (unsigned)K;
            const unsigned cb = tb + (unsigned)c * CS;
            red_pair_if(k0[j] < (unsigned)K, k0[j] * A + cb, 1u, __float_as_uint(w[j].x));
            red_pair_if(k1[j] < (unsigned)K, k1[j] * A + cb, 1u, __float_as_uint(w[j].y));
            kt0 = lab.x == c ? k0[j] : kt0;
            kt1 = lab.y == c ? k1[j] : kt1;
          }
        }
        // the true class's count (a label outside the loss channels has none)
        red_one_if(kt0 < (unsigned)K, kt0 * A + tb + (unsigned)lab.x * CS + 8u, 1u);
        red_one_if(kt1 < (unsigned)K, kt1 * A + tb + (unsigned)lab.y * CS + 8u, 1u);
      }
    }
    consumer_sync();
    if (cur_b >= 0) fold_all((int64_t)(P.b_offset + cur_b) * CL, false);
  }

  ace_launch_dependents();  // a dependent launch may begin its own setup now
  if (last_cta_ticket(P.counter)) {
    if constexpr (SOFT) soft_finish(P, s_iv);
    else hard_finish(P);
  }
}

}  // namespace ace
