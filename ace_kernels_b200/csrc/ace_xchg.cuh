// Exchange of the forward's statistics between ranks inside the forward kernel
// (ace_b200_forward_exchange), on B200 (sm_100a) GPUs joined by NVLink. Run by the
// last CTA of a pipelined forward (soft_finish, hard_finish) once it has written
// this rank's W, P, G to hist_out; replaces an all-reduce of hist_out between two
// launches and the separate epilogue launch after it.
//
// Mailbox of a rank (XchgParams: every rank's mailbox is mapped in every process
// through CUDA IPC; plain loads and stores, no multicast):
//   [0, 8)        calls completed so far (the epoch counter; read and written by
//                 its own rank only)
//   [64, 192)     flags[2][kMaxPeers]: epoch of the data in slot (parity, source)
//   [256, ...)    slots[2][world]: {b_offset, B} (two int32, 16 bytes), then W, P, G
//                 of the source's rows, [3][B][CL][K] fp32
// Call e (e = epoch counter + 1) uses parity e & 1: a rank writes call e's slot in
// a peer only after finishing call e - 1, which needed that peer's call e - 1
// data, written after the peer finished call e - 2 (its last read of parity
// e & 1); so two parities never overlap.
#pragma once

namespace ace {

constexpr int kXchgHeaderBytes = 256;
constexpr int kXchgFlagsOffset = 64;
constexpr unsigned long long kXchgWaitNs = 2000000000ull;  // bound of the wait (2 s)

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long* xchg_flag(unsigned char* box, int parity, int src) {
  return reinterpret_cast<unsigned long long*>(box + kXchgFlagsOffset) + parity * kMaxPeers + src;
}
__device__ __forceinline__ float* xchg_slot(const XchgParams& X, unsigned char* box, int parity,
                                            int src) {
  return reinterpret_cast<float*>(box + kXchgHeaderBytes +
                                  ((int64_t)parity * X.world + src) * X.slot_bytes);
}

// All threads of the last CTA, after hist_out ([3][B_total * CL][K]) holds this
// rank's sums: sends this rank's rows to every rank, waits for every rank's rows,
// and overwrites hist_out with the rank-ordered sums (a sample's rows come from
// the ranks whose {b_offset, B} covers it). False if a wait ran out.
__device__ __forceinline__ bool exchange_stats(const FwdParams& P) {
  const XchgParams& X = P.xchg;
  const int tid = threadIdx.x, nt = blockDim.x;
  const int K = P.tab.K, CL = P.g.CL;
  const int64_t row_vals = (int64_t)CL * K;              // values of one sample, one stat
  const int64_t m = (int64_t)P.B_total * row_vals;       // one stat, all samples
  unsigned char* own = X.mailbox[X.rank];
  __shared__ unsigned long long s_epoch;
  __shared__ int s_fail;
  __syncthreads();  // hist_out written by every warp
  if (tid == 0) {
    s_epoch = *reinterpret_cast<volatile unsigned long long*>(own) + 1ull;
    s_fail = 0;
  }
  __syncthreads();
  const unsigned long long epoch = s_epoch;
  const int par = (int)(epoch & 1ull);
  // this rank's rows into its slot of every mailbox
  const int64_t first = (int64_t)P.b_offset * row_vals, cnt = (int64_t)P.g.B * row_vals;
  for (int p = 0; p < X.world; ++p) {
    float* slot = xchg_slot(X, X.mailbox[p], par, X.rank);
    if (tid == 0) {
      reinterpret_cast<int*>(slot)[0] = P.b_offset;
      reinterpret_cast<int*>(slot)[1] = P.g.B;
    }
    for (int64_t i = tid; i < 3 * cnt; i += nt) {
      const int64_t st = i / cnt, j = i - st * cnt;
      slot[4 + i] = __ldcg(P.hist_out + st * m + first + j);
    }
  }
  __syncthreads();
  if (tid < X.world) {
    // every store above, ordered before the flag by the barrier and this fence
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    st_release_sys(xchg_flag(X.mailbox[tid], par, X.rank), epoch);
    // then wait for rank tid's data in this rank's mailbox
    const unsigned long long* f = xchg_flag(own, par, tid);
    if (ld_acquire_sys(f) != epoch) {
      const unsigned long long t0 = ace_now_ns();
      while (ld_acquire_sys(f) != epoch) {
        if (ace_now_ns() - t0 > kXchgWaitNs) {
          atomicExch(&s_fail, 1);
          break;
        }
      }
    }
  }
  __syncthreads();
  const bool ok = s_fail == 0;
  if (ok) {
    for (int64_t e = tid; e < 3 * m; e += nt) {
      const int64_t st = e / m, j = e - st * m;
      const int b = (int)(j / row_vals);
      float acc = 0.0f;
      for (int r = 0; r < X.world; ++r) {
        const float* slot = xchg_slot(X, own, par, r);
        const int ob = __ldcv(reinterpret_cast<const int*>(slot)), nb = __ldcv(reinterpret_cast<const int*>(slot) + 1);
        if (b >= ob && b < ob + nb)
          acc = ACE_FADD(acc, __ldcv(slot + 4 + st * nb * row_vals + (j - (int64_t)ob * row_vals)));
      }
      P.hist_out[e] = acc;
    }
  }
  __syncthreads();
  if (tid == 0) *reinterpret_cast<volatile unsigned long long*>(own) = epoch;
  return ok;
}

}  // namespace ace
