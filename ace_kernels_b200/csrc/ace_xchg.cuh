// Exchange of the forward's statistics between ranks inside the forward kernel
// (ace_b200_forward_exchange), on B200 (sm_100a) GPUs joined by NVLink. Run by the
// last CTA of a pipelined forward (soft_finish, hard_finish) as it reconstructs
// this rank's W, P, G; replaces an all-reduce between two launches and the
// separate epilogue launch after it.
//
// What crosses depends on the sharding. Batch shards (the ranks' samples
// disjoint, own_rows): a sample's rows are complete on the rank that holds it, so
// that rank reconstructs and runs the epilogue of its own rows only (coef, d, jac,
// f) and only each row's f crosses, for every rank to add the loss in the
// single-rank order (bit for bit the single-GPU loss). Spatial shards (every rank holds partial sums of every
// row): each rank's W, P, G cross, and every rank adds them in rank order and
// runs the epilogue of every row.
//
// Low-latency protocol: every value crosses NVLink as one 64-bit store of {its
// bits, the call's tag}, so a receiver that reads a word carrying the current tag
// has the value: no fence, no separate flag, one one-way trip. The sender stores
// a row's values from registers as soon as it has reconstructed them; the
// receiver polls the words of the rows other ranks hold (plain loads of its own
// memory, with a bound on the wait).
//
// Mailbox of a rank (every rank's mailbox is mapped in every process through
// CUDA IPC; plain loads and stores, no multicast):
//   [0, 8)       calls completed so far (the epoch counter; its own rank only)
//   [64, 128)    barrier words[world]: the number of barriers rank src has
//                entered (xchg_barrier_kernel)
//   [256, ...)   slots[2][world]: the source rank's rows, [3][rows][K] words
//                {value bits, tag} (batch shards: [rows] words of f), tag = the low
//                32 bits of the call number
// Call e (e = epoch counter + 1) uses parity e & 1: a rank writes call e's slot in
// a peer only after finishing call e - 1, which needed that peer's call e - 1
// data, sent after the peer finished call e - 2 (its last read of parity e & 1);
// so two parities never overlap. A fresh mailbox is zero-filled and call numbers
// start at 1, so a stale word never carries the current tag.
#pragma once

namespace ace {

constexpr int kXchgHeaderBytes = 256;
constexpr int kXchgBarrierOffset = 64;  // the barrier words of the header
constexpr unsigned long long kXchgWaitNs = 2000000000ull;  // bound of the wait (2 s)

// This call's number (the last CTA, any thread; the load overlaps the
// reconstruction's own loads).
__device__ __forceinline__ unsigned long long xchg_epoch(const XchgParams& X) {
  return *reinterpret_cast<volatile unsigned long long*>(X.mailbox[X.rank]) + 1ull;
}

// Word of (stat s, row r, bin k) of source `src` in `box`, parity `par`; rows are
// counted from the source's first loss row.
__device__ __forceinline__ unsigned long long* xchg_word(const XchgParams& X, unsigned char* box,
                                                         int par, int src, int s, int r, int k,
                                                         int CL, int K) {
  const int64_t rows = (int64_t)X.count[src] * CL;
  return reinterpret_cast<unsigned long long*>(box + kXchgHeaderBytes +
                                               ((int64_t)par * X.world + src) * X.slot_bytes) +
         ((int64_t)s * rows + (r - (int64_t)X.first[src] * CL)) * K + k;
}

// One warp: row r's W, P, G (lane l holds bins l + 32 q) to every rank, if this
// rank holds the row.
__device__ __forceinline__ void xchg_send_row(const FwdParams& P, unsigned long long epoch, int r,
                                              const float (&w)[4], const float (&p)[4],
                                              const float (&g)[4]) {
  const XchgParams& X = P.xchg;
  const int CL = P.g.CL, K = P.tab.K, lane = threadIdx.x & 31;
  if (r < X.first[X.rank] * CL || r >= (X.first[X.rank] + X.count[X.rank]) * CL) return;
  const int par = (int)(epoch & 1ull);
  const unsigned long long tag = (epoch & 0xffffffffull) << 32;
  for (int dst = 0; dst < X.world; ++dst) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int k = lane + 32 * q;
      if (k >= K) continue;
      const float v[3] = {w[q], p[q], g[q]};
#pragma unroll
      for (int s = 0; s < 3; ++s) {
        unsigned long long* a = xchg_word(X, X.mailbox[dst], par, X.rank, s, r, k, CL, K);
        const unsigned long long word = tag | __float_as_uint(v[s]);
        asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(word) : "memory");
      }
    }
  }
}

// All threads of the last CTA, after every row was sent: per row (one warp, the
// single-rank path's order) the values of the ranks holding the row, added in
// rank order, into hist_out and (do_epilogue) the row's epilogue. A wait that
// runs out makes the row NaN. Returns this thread's share of the loss; advances
// the epoch counter.
__device__ __forceinline__ float xchg_finish(const FwdParams& P, unsigned long long epoch) {
  const XchgParams& X = P.xchg;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x / 32;
  const int CL = P.g.CL, K = P.tab.K, rows = P.B_total * CL;
  const int64_t m = (int64_t)rows * K;
  const int par = (int)(epoch & 1ull);
  const unsigned tag = (unsigned)(epoch & 0xffffffffull);
  unsigned char* own = X.mailbox[X.rank];
  const float nan = __int_as_float(0x7fc00000);
  const unsigned long long t0 = ace_now_ns();
  float mine = 0.0f;
  for (int r = warp; r < rows; r += nw) {
    const int b = r / CL;
    float v[3][4];
    bool ok = true;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int k = lane + 32 * q;
#pragma unroll
      for (int s = 0; s < 3; ++s) v[s][q] = 0.0f;
      if (k >= K) continue;
      for (int src = 0; src < X.world; ++src) {
        if (b < X.first[src] || b >= X.first[src] + X.count[src]) continue;
#pragma unroll
        for (int s = 0; s < 3; ++s) {
          const unsigned long long* a = xchg_word(X, own, par, src, s, r, k, CL, K);
          unsigned long long word;
          asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(word) : "l"(a) : "memory");
          while ((unsigned)(word >> 32) != tag) {
            if (ace_now_ns() - t0 > kXchgWaitNs) {
              ok = false;
              break;
            }
            asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(word) : "l"(a) : "memory");
          }
          v[s][q] = ACE_FADD(v[s][q], __uint_as_float((unsigned)word));
        }
      }
      if (!ok) v[0][q] = v[1][q] = v[2][q] = nan;
      const int64_t e = (int64_t)r * K + k;
      P.hist_out[e] = v[0][q];
      P.hist_out[m + e] = v[1][q];
      P.hist_out[2 * m + e] = v[2][q];
    }
    if (P.do_epilogue) mine = ACE_FADD(mine, epilogue_row(P.epi, r, v[0], v[1], v[2]));
  }
  __syncthreads();
  if (threadIdx.x == 0) *reinterpret_cast<volatile unsigned long long*>(own) = epoch;
  return mine;
}

// Batch shards: this rank's row r, whose epilogue gave f (on every lane), to every
// rank (one lane per destination).
__device__ __forceinline__ void xchg_send_f(const FwdParams& P, unsigned long long epoch, int r,
                                            float f) {
  const XchgParams& X = P.xchg;
  const int lane = threadIdx.x & 31, CL = P.g.CL;
  const int par = (int)(epoch & 1ull);
  if (lane < X.world) {
    unsigned long long* a = xchg_word(X, X.mailbox[lane], par, X.rank, 0, r, 0, CL, 1);
    const unsigned long long word = ((epoch & 0xffffffffull) << 32) | __float_as_uint(f);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(word) : "memory");
  }
}

// The rows the last CTA reconstructs: with batch shards only this rank's (the
// other ranks' rows of its sums are empty), else all of them.
__device__ __forceinline__ int2 xchg_rows(const FwdParams& P) {
  const XchgParams& X = P.xchg;
  const int CL = P.g.CL;
  if (X.world > 1 && X.own_rows)
    return make_int2(X.first[X.rank] * CL, (X.first[X.rank] + X.count[X.rank]) * CL);
  return make_int2(0, P.B_total * CL);
}

// Every row's f in the last CTA (batch shards; at most 256 rows, the limit of
// the fused epilogue that the exchange requires).
__device__ __forceinline__ float* xchg_row_f() {
  __shared__ float s_f[8 * kEpiRowsPerCta];
  return s_f;
}

// Batch shards, all threads of the last CTA after this rank's rows were sent and
// their f put in xchg_row_f(): zeros into hist_out for the other ranks' rows, their
// f from the ranks that hold them (one thread per row, waits bounded; NaN when one
// runs out) into xchg_row_f() and f, then per warp the sum over rows warp,
// warp + warps, ... in that order, as the single-rank path adds them. Returns this
// warp's share of the loss; advances the epoch counter.
__device__ __forceinline__ float xchg_finish_f(const FwdParams& P, unsigned long long epoch) {
  const XchgParams& X = P.xchg;
  const int tid = threadIdx.x, nt = blockDim.x, warp = tid >> 5, nw = nt / 32;
  const int CL = P.g.CL, K = P.tab.K, rows = P.B_total * CL;
  const int2 mine_rows = xchg_rows(P);
  const int par = (int)(epoch & 1ull);
  const unsigned tag = (unsigned)(epoch & 0xffffffffull);
  unsigned char* own = X.mailbox[X.rank];
  float* s_f = xchg_row_f();
  for (int64_t e = tid; e < 3 * (int64_t)rows * K; e += nt) {
    const int r = (int)((e / K) % rows);
    if (r < mine_rows.x || r >= mine_rows.y) P.hist_out[e] = 0.0f;
  }
  const unsigned long long t0 = ace_now_ns();
  for (int r = tid; r < rows; r += nt) {
    if (r >= mine_rows.x && r < mine_rows.y) continue;
    const int b = r / CL;
    int src = 0;
    while (src + 1 < X.world && !(b >= X.first[src] && b < X.first[src] + X.count[src])) ++src;
    const unsigned long long* a = xchg_word(X, own, par, src, 0, r, 0, CL, 1);
    unsigned long long word;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(word) : "l"(a) : "memory");
    bool ok = true;
    while ((unsigned)(word >> 32) != tag) {
      if (ace_now_ns() - t0 > kXchgWaitNs) {
        ok = false;
        break;
      }
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(word) : "l"(a) : "memory");
    }
    const float f = ok ? __uint_as_float((unsigned)word) : __int_as_float(0x7fc00000);
    s_f[r] = f;
    P.epi.f[r] = f;
  }
  __syncthreads();
  float mine = 0.0f;
  for (int r = warp; r < rows; r += nw) mine = ACE_FADD(mine, s_f[r]);
  __syncthreads();
  if (tid == 0) *reinterpret_cast<volatile unsigned long long*>(own) = epoch;
  return mine;
}

}  // namespace ace
