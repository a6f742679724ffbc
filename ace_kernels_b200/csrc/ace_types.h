// Parameter blocks passed by value to the mL1-ACE kernels (kernel parameter
// space: no device allocation, no host->device copy, so every launch can be
// captured in a CUDA graph).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "ace_b200.h"  // include/ (on the include path of the build)

namespace ace {

constexpr int kMaxBins = ACE_B200_MAX_BINS;        // num_bins limit of the kernels
constexpr int kMaxClasses = ACE_B200_MAX_CLASSES;  // channels limit of the kernels
constexpr int kThreads = 256;                      // threads per CTA (gradient, epilogue)
constexpr int kHistThreads = 512;                  // threads per CTA of the histogram
constexpr int kMaxDevices = 64;                    // devices a process may drive (per-device state)
constexpr int kTabCopies = 16;                     // interleaved copies of the bin tables
constexpr float kFixScale = 2097152.0f;            // 2^21: fixed-point unit of the statistics

// Sorted search table with its neighbours paired (see ace_locate): hard binning
// uses the K upper bin edges, soft binning the K bin centres; entry i holds
// {t[i-1], t[i]} and {base, scale}, with -10000 / +10000 at the two ends (the
// reference's soft sentinels, ace_reference/softl1ace.py:99-105). With `right`
// (count t <= p) each t is replaced by the next float below it, so the kernels
// always test t < p: for finite floats, t <= p exactly when prev(t) < p. The two
// halves are separate 8-byte tables (an 8-byte shared-memory gather by 32 lanes
// with random indices conflicts far less than a 16-byte one).
// Soft binning: interval i lies between t[i-1] and t[i]; base and scale map p to
// the interval's coordinate u = (p - base) * scale / 2^21 (u = t, the right-bin
// weight, inside; u = p in the two end intervals: base 0, scale 2^21).
struct BinTable {
  int K;
  float2 lohi[kMaxBins + 1];  // {t[i-1], t[i]}
  float2 map[kMaxBins + 1];   // {base, scale}
};

// Where one launch's voxels sit in the statistics: rows b_offset .. b_offset+B-1
// of a [3, B_total, CL, K] buffer (batch sharding across ranks), and which slice
// of the voxel axis (spatial sharding) is local.
struct Grid {
  int64_t N;           // voxels per (b, c) slice in this launch
  int B;               // batches in this launch
  int C;               // channels of x
  int CL;              // loss channels: C - offset
  int offset;          // 1 when the background channel is dropped
  int chunks;          // CTAs per batch
  int64_t tiles;       // tiles of threads * V voxels per batch
  int64_t tiles_per_chunk;
  int chunks_per_batch;  // > 0: chunks never cross batches; 0: flat over all tiles
};

struct EpiParams {
  int B_total;         // rows of the statistics buffer = B_total * CL
  int CL;
  int K;
  int soft;
  float empty_weight;
  int ignore_empty;
  int reduction;       // ACE_B200_REDUCTION_*
  double rows_global;  // divisor of the "mean" reduction
  float class_w[kMaxClasses];
  // outputs (device)
  float* coef;         // [B_total, CL, K]
  float* d;            // [B_total, CL, K]
  float* jac;          // [B_total, CL]
  float* f;            // [B_total, CL]
  float* loss;         // [1]
};

// Statistics exchange between ranks inside the forward (ace_b200_forward_exchange).
constexpr int kMaxPeers = ACE_B200_MAX_PEERS;
struct XchgParams {
  int world;                          // 1: no exchange
  int rank;
  int64_t slot_bytes;                 // bytes of one rank's slot in a mailbox
  unsigned char* mailbox[kMaxPeers];  // every rank's mailbox, mapped in this process
  int first[kMaxPeers];               // each rank's first sample (b_offset)
  int count[kMaxPeers];               // and its number of samples (B)
  int own_rows;                       // 1: the ranks' samples are disjoint (batch shards)
};

struct FwdParams {
  const void* x;       // [B, C, N] logits / probabilities (fp32, bf16, fp16)
  const void* target;  // [B, N] int64 labels or [B, C, N] fp32 dense targets
  Grid g;
  int act;             // ACE_B200_ACT_*
  int soft;
  int R;               // lane replicas of the shared-memory histogram (power of 2)
  int flush_tiles;     // tiles between folds of the shared table (32-bit range)
  int b_offset;        // first statistics row of this launch
  int B_total;
  double* accum;       // workspace: [NOUT, B_total, CL, slots] sums (self-cleaning)
  // the pipelined kernels (soft_fwd_kernel, mc_fwd_kernel) only (the same
  // workspace bytes as accum):
  unsigned long long* iacc;  // integer sums (self-cleaning): soft [3, B_total, CL, K + 1, 2],
                             // mc_fwd_kernel hard [3, B_total, CL, K]
  unsigned* pool_ctr;  // [B] tile-claim counters, one per batch (self-cleaning)
  int64_t wt_batch;    // tiles per batch
  int epoch;           // tiles a CTA adds between two folds (32-bit word range)
  int stages;          // shared-memory ring stages (<= kPipeMaxStages)
  int table_bytes;     // shared-memory bytes of the statistics table (128-aligned)
  int stage_offset;    // shared-memory byte offset of the ring (128-aligned)
  unsigned* counter;   // workspace: finished-CTA counter, then an error word (self-cleaning)
  float* hist_out;     // [3, B_total, CL, K] statistics (W, P, G)
  int do_epilogue;
  BinTable tab;
  EpiParams epi;
  XchgParams xchg;
};

struct BwdParams {
  const void* x;
  const void* target;
  void* dx;            // [B, C, N], dtype of x
  Grid g;
  int act;
  int soft;
  int b_offset;        // first row of coef / d / jac used by this launch
  const float* coef;   // [B_total, CL, K]
  const float* d;      // [B_total, CL, K]
  const float* jac;    // [B_total, CL]
  const float* grad_out;  // scalar, or [B_total, CL] when grad_per_row
  int grad_per_row;
  int rec_copies;      // interleaved copies of the per-row records (power of two)
  // grad_tma_kernel only:
  int stages;          // shared-memory ring stages (<= kPipeMaxStages)
  int stage_offset;    // shared-memory byte offset of the ring (128-aligned)
  int64_t tiles_per_batch;  // tiles of kPipeTileVoxels voxels per batch
  BinTable tab;
};

}  // namespace ace
