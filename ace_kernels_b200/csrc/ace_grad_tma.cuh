// grad_tma_kernel: the backward (d loss / d logits) of a softmax over C <= 4
// channels, soft binning with int64 labels or hard binning, on B200 (sm_100a), as
// a TMA pipeline. Included by ace_kernels.cuh after grad_kernel's helpers.
//
// Same formulas as grad_kernel (see its comment; ace_kernels/impls/
// v2_autograd.py:88-118): per value gp = F + D (2 p - y) from the per-(row,
// interval) soft records, or g coef[bin] for hard binning, then the softmax
// backward dx_c = p_c (gp_c - sum_c' p_c' gp_c'), with the forward's activation
// recomputed (soft: the fast softmax; hard: the exact one, so the bins match the
// forward's). The memory side is a producer thread streaming tiles (the C logit
// rows, and the labels for soft binning) into a shared-memory ring with bulk
// copies; kPipeConsumerWarps consumer warps compute and store dx straight from
// registers with streaming 16-byte stores.
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
  // shared memory: records [B][CL][K + 1][copies] (float2 soft, float hard), the
  // bin table [K + 1][kTabCopies] float2, then the stages (128-aligned)
  float* rec = reinterpret_cast<float*>(smem_raw);
  const int rec_words = (SOFT ? 2 : 1) * B * CL * (K + 1) * copies;
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

  // Tile sequence: k -> batch k % B, tile tpb - 1 - k / B of that batch.
  const int64_t tpb = P.tiles_per_batch;
  const int64_t total = tpb * B;

  if (warp == NCW) {
    // ---------------- producer (one thread) ----------------
    // The logits and labels are inputs of the forward too, never written by the
    // kernel this one depends on: the copies may start before that kernel ends.
    if (lane == 0) {
      const T* x = static_cast<const T*>(P.x);
      const int64_t* lab = static_cast<const int64_t*>(P.target);
      int issued = 0;
      int64_t k = blockIdx.x;
      for (int i = 0;; ++i, k += gridDim.x) {
        const int s = i % S;
        const unsigned use = (unsigned)(i / S);
        if (use > 0 && !mbar_wait(empty_bar(s), (use - 1) & 1u)) {
          s_abort = 1;
          break;
        }
        if (s_abort) break;
        if (k >= total) {  // the end marker (no copies)
          s_meta[s] = make_int4(-1, 0, 0, 0);
          mbar_arrive(full_bar(s));
          break;
        }
        const int tb = (int)(k % B);
        const int64_t tile = tpb - 1 - k / B;
        const int64_t v0 = tile * TV;
        const int cnt = (int)min((int64_t)TV, N - v0);
        s_meta[s] = make_int4((int)tile, tb, cnt, 0);
        const unsigned xb = (unsigned)cnt * (unsigned)sizeof(T);
        mbar_arrive_tx(full_bar(s), C * xb + (SOFT ? (unsigned)cnt * 8u : 0u));
        const unsigned dst = stage0 + (unsigned)s * SB;
        const T* gx = x + (int64_t)tb * C * N + v0;
#pragma unroll
        for (int c = 0; c < C; ++c) bulk_load(dst + c * XB, gx + (int64_t)c * N, xb, full_bar(s));
        if constexpr (SOFT)
          bulk_load(dst + C * XB, lab + (int64_t)tb * N + v0, (unsigned)cnt * 8u, full_bar(s));
        issued = i + 1;
      }
      // after an abort, no copy may still be in flight when the CTA leaves
      if (s_abort)
        for (int i = issued - S > 0 ? issued - S : 0; i < issued; ++i)
          mbar_wait(full_bar(i % S), (unsigned)(i / S) & 1u);
    }
  } else {
    // ---------------- consumers ----------------
    // coef, d and jac come from the previous kernel: records only after it
    ace_grid_dependency_wait();
    // One consumer thread per (batch, row, j) record; it writes all the record's
    // copies (16-byte stores: copies * record bytes is a multiple of 16).
    for (int e = tid; e < B * CL * (K + 1); e += NCW * 32) {
      const int bro = e / (K + 1), j = e - bro * (K + 1);  // bro = b * CL + row
      const int b = bro / CL, row = bro - b * CL;
      const int64_t grow = (int64_t)(P.b_offset + b) * CL + row;
      const float g = P.jac[grow] * (P.grad_per_row ? P.grad_out[grow] : P.grad_out[0]);
      const float* cf = P.coef + grow * K;
      const float* dd = P.d + grow * K;
      uint4 v;
      if constexpr (!SOFT) {
        const unsigned u = __float_as_uint(j < K ? g * cf[j] : 0.0f);
        v = make_uint4(u, u, u, u);
      } else {
        const int l = max(j - 1, 0), r = min(j, K - 1);
        const float a = g * cf[l], bb = g * cf[r];
        float2 rv = make_float2(a, 0.0f);
        if (j > 0 && j < K) {
          const float2 mp = s_map[j];
          const double lo = mp.x, inv = (double)mp.y / (double)kFixScale;
          const double dd_ = ((double)bb - (double)a) * inv;
          const double e_ = inv * ((double)a * dd[l] - (double)bb * dd[r]);
          rv = make_float2((float)((double)a - dd_ * lo + e_), (float)dd_);
        }
        v = make_uint4(__float_as_uint(rv.x), __float_as_uint(rv.y), __float_as_uint(rv.x),
                       __float_as_uint(rv.y));
      }
      uint4* dst = reinterpret_cast<uint4*>(rec + (SOFT ? 2 : 1) * e * copies);
      for (int q = 0; q < (SOFT ? 2 : 1) * copies / 4; ++q) dst[q] = v;
    }
    consumer_sync();
    const float* my_rec = rec + (SOFT ? 2 : 1) * (lane & (copies - 1));
    const float2* my_lohi = lohi_t + (lane & (kTabCopies - 1));
    auto entry = [&](int j) -> float2 { return my_lohi[j * kTabCopies]; };
    const int vo = (warp * 32 + lane) * VL;  // this lane's first voxel of a tile
    T* dxp = static_cast<T*>(P.dx);
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
#pragma unroll
      for (int v = 0; v < VL; ++v) {
        float p[C];
#pragma unroll
        for (int c = 0; c < C; ++c) p[c] = xv[c][v];
        ace_softmax_sel<SOFT, C>(p, C);
        int j[C];
        bool ok = true;
#pragma unroll
        for (int c = OFF; c < C; ++c) {
          j[c] = ace_guess(p[c], Kf, K, SOFT);
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
          gp[c] = 0.0f;
          if (c >= OFF) {
            const float y = (SOFT && lab[v] == c) ? 1.0f : 0.0f;
            gp[c] = grad_p<SOFT>(my_rec, copies, rb + c, K, j[c], p[c], y);
          }
          dot += p[c] * gp[c];
        }
#pragma unroll
        for (int c = 0; c < C; ++c) xv[c][v] = p[c] * (gp[c] - dot);
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
