/*
 * ace_b200.h - C ABI of the B200 (sm_100a) mL1-ACE loss library (libace_b200.so).
 *
 * The mL1-ACE calibration loss (hard or soft binning) forward and backward for
 * logits x[B, C, N] (N = product of the spatial sizes), in one fused read-once
 * histogram pass, a tiny epilogue and one gradient pass that recomputes the
 * activation instead of saving it.
 *
 * Conventions, for every entry point:
 *   - all tensor pointers are DEVICE memory owned by the caller, contiguous,
 *     row-major, in the layouts stated below; `stream` is a cudaStream_t (NULL =
 *     the legacy default stream);
 *   - every call is asynchronous on `stream`, allocates nothing and never
 *     synchronises the host, so a sequence of calls can be captured in a CUDA
 *     graph;
 *   - the return value is ACE_B200_OK (0) or a negative ACE_B200_E* code;
 *     ace_b200_last_error() then gives a message (thread-local);
 *   - the library keeps no per-call state: calls are thread-safe, except that
 *     two calls sharing one `workspace` must not run concurrently.
 *
 * Reference interfaces replaced (kapitan05/ace-kernels, paths inside that
 * project): see each declaration.
 */
#ifndef ACE_B200_H
#define ACE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define ACE_B200_OK 0
#define ACE_B200_EINVAL (-1)       /* bad argument (shape, dtype, pointer) */
#define ACE_B200_EUNSUPPORTED (-2) /* valid but outside the kernels' limits */
#define ACE_B200_ECUDA (-3)        /* a CUDA runtime call failed */

/* Limits of the kernels. */
#define ACE_B200_MAX_BINS 128
#define ACE_B200_MAX_CLASSES 64

/* Logit dtypes. */
#define ACE_B200_F32 0
#define ACE_B200_BF16 1
#define ACE_B200_F16 2

/* Activations (ACEConfig.activation; softmax over one channel is the identity). */
#define ACE_B200_ACT_NONE 0
#define ACE_B200_ACT_SOFTMAX 1
#define ACE_B200_ACT_SIGMOID 2

/* Target forms. */
#define ACE_B200_TARGET_LABELS 0 /* int64 [B, N] class index per voxel */
#define ACE_B200_TARGET_DENSE 1  /* fp32 [B, C, N] (one-hot or soft targets) */

/* Reductions (ACEConfig.reduction). */
#define ACE_B200_REDUCTION_MEAN 0
#define ACE_B200_REDUCTION_SUM 1
#define ACE_B200_REDUCTION_NONE 2

/*
 * Loss options shared by the forward, statistics and backward calls; mirrors
 * ACEConfig (ace_kernels/config.py:12-31).
 *   num_bins      K, 1..ACE_B200_MAX_BINS
 *   soft          0 hard binning, 1 soft binning
 *   activation    ACE_B200_ACT_*
 *   offset        1 drops channel 0 (include_background=False with C > 1), else 0
 *   right         bucketize convention (ACEConfig.right)
 *   empty_weight  soft binning: a bin with weight below this is empty
 *   ignore_empty  mask classes absent from the target (ACEConfig.ignore_empty_classes)
 *   reduction     ACE_B200_REDUCTION_*
 *   class_weights HOST array of C - offset weights, or NULL (unweighted); read
 *                 during the call only
 */
typedef struct ace_b200_options {
  int32_t num_bins;
  int32_t soft;
  int32_t activation;
  int32_t offset;
  int32_t right;
  float empty_weight;
  int32_t ignore_empty;
  int32_t reduction;
  const float* class_weights;
} ace_b200_options;

/*
 * Inputs of one launch.
 *   x            [B, C, N] logits (probabilities with ACE_B200_ACT_NONE), dtype x_dtype
 *   target       labels int64 [B, N] or dense fp32 [B, C, N], per target_kind
 *   b_offset     first row of the statistics this launch covers (batch sharding:
 *                rank r passes the index of its first sample), 0 otherwise
 *   b_total      batches covered by the statistics buffer (>= b_offset + B)
 *   rows_global  divisor of the "mean" reduction; 0 = b_total * (C - offset)
 */
typedef struct ace_b200_inputs {
  const void* x;
  int32_t x_dtype;
  int64_t B;
  int64_t C;
  int64_t N;
  const void* target;
  int32_t target_kind;
  int64_t b_offset;
  int64_t b_total;
  double rows_global;
} ace_b200_inputs;

/* Outputs of the epilogue, all fp32 device arrays (R = b_total * (C - offset)):
 *   coef [R, K]  sign(d) / (K_nonempty * W), 0 for empty bins
 *   d    [R, K]  mean p - mean target per bin, 0 for empty bins
 *   jac  [R]     d loss / d f (mask, class weight, reduction)
 *   f    [R]     per-class error after mask and weight (the "none" reduction)
 *   loss [1]     mean or sum of f (written for every reduction)
 */
typedef struct ace_b200_epilogue_out {
  float* coef;
  float* d;
  float* jac;
  float* f;
  float* loss;
} ace_b200_epilogue_out;

/* Bytes of the workspace for a statistics buffer of b_total * cl rows and
 * num_bins bins. The workspace must be zero-filled before its first use; every
 * call leaves it zero-filled again. */
size_t ace_b200_workspace_bytes(int64_t b_total, int64_t cl, int32_t num_bins);

/*
 * Forward: fused activation + W/P/G statistics + epilogue, one launch.
 * Replaces v6_triton._forward (ace_kernels/impls/v6_triton.py:43-65), i.e.
 * hard_hist_fused / soft_hist_fused (ace_kernels/kernels/hard_hist.py:186-233,
 * ace_kernels/kernels/soft_hist.py:229-271) followed by epilogue_triton
 * (ace_kernels/kernels/epilogue.py:93-129); the statistics are
 * binning.hard_stats / soft_stats (ace_kernels/binning.py:54-116).
 *   hist  [3, b_total, C - offset, K] fp32 out: W (count / weight sum), P, G
 */
int ace_b200_forward(const ace_b200_inputs* in, const ace_b200_options* opt, float* hist,
                     ace_b200_epilogue_out out, void* workspace, size_t workspace_bytes,
                     void* stream);

/*
 * ace_b200_forward without a workspace: the scratch (accumulators and counters)
 * is a fixed device array inside the library, ACE_B200_STATIC_SCRATCH_BYTES per
 * device. No counterpart in the reference, which allocates its scratch through
 * torch on every call. It serves callers that cannot hand over device memory: a
 * host binding the library through its C ABI alone, with no device allocator
 * of its own, or one whose allocator may not run inside its step loop. This
 * call allocates nothing and calls no allocating function.
 *   - Limit: ace_b200_workspace_bytes(b_total, C - offset, num_bins) must not
 *     exceed ACE_B200_STATIC_SCRATCH_BYTES (about b_total * (C - offset) <= 780
 *     rows at K = 20); larger calls fail with ACE_B200_EUNSUPPORTED.
 *   - Setup: the first call on each device looks the array up and clears it on
 *     `stream`; it must not run under stream capture (it then fails with
 *     ACE_B200_EINVAL).
 *   - The scratch is shared by every call on a device: two calls whose kernels
 *     may overlap (different streams without ordering between them, or two
 *     threads) race on it and give wrong results. Order them on one stream.
 */
#define ACE_B200_STATIC_SCRATCH_BYTES 1048576 /* 1 MiB */
int ace_b200_forward_static(const ace_b200_inputs* in, const ace_b200_options* opt, float* hist,
                            ace_b200_epilogue_out out, void* stream);

/*
 * Ranks that hold shards of one batch (one process per GPU) can combine their
 * statistics inside the forward kernel itself instead of an all-reduce between
 * ace_b200_hist and ace_b200_epilogue. No counterpart in the reference (which
 * runs on one device); it replaces that NCCL all-reduce and the separate
 * epilogue launch.
 *
 * Each rank allocates one mailbox (ace_b200_mailbox_alloc, zero-filled), hands
 * its IPC handle (ace_b200_ipc_handle) to the others, and maps theirs
 * (ace_b200_ipc_open). The forward's last CTA then stores this rank's rows of W,
 * P, G into every rank's mailbox over NVLink, each value as one 64-bit word
 * tagged with the call's number, reads the other ranks' rows from its own
 * mailbox as their tagged words arrive (waiting at most about 2 s), adds the
 * ranks' rows in rank order, and runs the epilogue on the global statistics:
 * every rank ends with the same loss, coef, d and jac. A wait that runs out
 * writes NaN statistics and loss. All ranks must make the same sequence of these
 * calls (the mailbox counts them); the kernels of different ranks must run on
 * different GPUs.
 *   world, rank    ranks (1..ACE_B200_MAX_PEERS) and this rank's index
 *   mailbox[r]     rank r's mailbox as mapped in this process (own one at [rank])
 *   first[r]       rank r's first sample, and count[r] its number of samples: the
 *   count[r]       b_offset and B of its inputs (own entry equal to this call's)
 * A rank's rows are samples b_offset .. b_offset + B - 1 (batch shards), or all
 * b_total samples of a spatial shard (b_offset 0, B = b_total). Cases whose
 * forward is not one of the pipelined kernels (soft binning with labels and a
 * softmax; or a softmax over 5 to 24 channels with labels) return
 * ACE_B200_EUNSUPPORTED before launching anything.
 */
#define ACE_B200_MAX_PEERS 8
typedef struct ace_b200_exchange {
  int32_t world;
  int32_t rank;
  void* mailbox[ACE_B200_MAX_PEERS];
  int32_t first[ACE_B200_MAX_PEERS];
  int32_t count[ACE_B200_MAX_PEERS];
} ace_b200_exchange;

/* Bytes of one mailbox for the statistics of b_total * cl rows, num_bins bins
 * and `world` ranks. */
size_t ace_b200_mailbox_bytes(int64_t b_total, int64_t cl, int32_t num_bins, int32_t world);
/* A zero-filled device allocation of `bytes` (cudaMalloc), and its release. */
int ace_b200_mailbox_alloc(size_t bytes, void** ptr_out);
int ace_b200_mailbox_free(void* ptr);
/* The CUDA IPC handle of a mailbox (ACE_B200_IPC_HANDLE_BYTES bytes), and the
 * mapping of another process's mailbox from its handle (and its unmapping). */
#define ACE_B200_IPC_HANDLE_BYTES 64
int ace_b200_ipc_handle(void* ptr, void* handle_out);
int ace_b200_ipc_open(const void* handle, void** ptr_out);
int ace_b200_ipc_close(void* ptr);

/* ace_b200_forward with the statistics of all ranks combined in the kernel. */
int ace_b200_forward_exchange(const ace_b200_inputs* in, const ace_b200_options* opt, float* hist,
                              ace_b200_epilogue_out out, void* workspace,
                              size_t workspace_bytes, const ace_b200_exchange* xchg,
                              void* stream);

/*
 * A barrier of the ranks of an exchange on the device, over the same mailboxes
 * (one warp: a 64-bit store into every rank's mailbox, then a wait until every
 * rank's store has arrived in this rank's). It orders the ranks' kernels in time
 * only, not memory. No counterpart in the reference; it lines the ranks up
 * before a timed step more tightly than an all-reduce, whose ranks leave it at
 * different times. `wait_ns` (device, optional) receives how long this rank
 * waited, or UINT64_MAX when a rank did not arrive within about 2 s (the kernel
 * then returns). All ranks must make the same number of these calls; their
 * kernels must run on different GPUs. Only world, rank and mailbox are used.
 */
int ace_b200_exchange_barrier(const ace_b200_exchange* xchg, uint64_t* wait_ns, void* stream);

/*
 * Statistics only (the first half of ace_b200_forward), for callers that reduce
 * the statistics across ranks (NCCL all-reduce of `hist`) before the epilogue.
 * Replaces hard_hist_fused / soft_hist_fused (ace_kernels/kernels/hard_hist.py:186-233,
 * ace_kernels/kernels/soft_hist.py:229-271).
 */
int ace_b200_hist(const ace_b200_inputs* in, const ace_b200_options* opt, float* hist,
                  void* workspace, size_t workspace_bytes, void* stream);

/*
 * Epilogue on [3, b_total, cl, K] statistics (workspace as for ace_b200_hist,
 * with the same b_total, cl and num_bins). Replaces epilogue_triton
 * (ace_kernels/kernels/epilogue.py:23-129), i.e. v2_autograd.coefficients
 * (ace_kernels/impls/v2_autograd.py:66-76) + common.reduce_classes
 * (ace_kernels/common.py:184-207) + the reduction jacobian
 * (ace_kernels/impls/v2_autograd.py:138-151).
 */
int ace_b200_epilogue(const float* hist, int64_t b_total, int64_t cl, double rows_global,
                      const ace_b200_options* opt, ace_b200_epilogue_out out, void* workspace,
                      size_t workspace_bytes, void* stream);

/*
 * Backward: d loss / d x for this launch's x (dx has x's dtype and shape).
 * coef, d, jac are the epilogue outputs (rows b_offset.. are used); grad_output
 * is a device scalar, or [b_total, C - offset] when grad_per_row (reduction
 * "none"). Replaces hard_input_grad_triton / soft_input_grad_triton
 * (ace_kernels/kernels/hard_bwd.py:98-149, ace_kernels/kernels/soft_bwd.py:251-312)
 * with the formulas of v2_autograd._df_dprobs / _activation_backward
 * (ace_kernels/impls/v2_autograd.py:88-118).
 */
int ace_b200_backward(const ace_b200_inputs* in, const ace_b200_options* opt,
                      const float* coef, const float* d, const float* jac,
                      const float* grad_output, int32_t grad_per_row, void* dx, void* stream);

/*
 * Activated probabilities p[B, C, N] (fp32) exactly as the histogram and gradient
 * kernels compute them: a test hook that lets the parity tests bin the kernel's
 * own probabilities on the host. Replaces the activation half of
 * common.prepare (ace_kernels/common.py:80-140).
 */
int ace_b200_probs(const ace_b200_inputs* in, int32_t activation, float* probs, void* stream);

/* Host: the search table of the kernels (hard: the K upper edges, soft: the K
 * centres), bit-identical to the reference's fp32 linspace tables
 * (ace_kernels/common.py:17-25). `out` has num_bins floats. */
int ace_b200_bin_table(int32_t num_bins, int32_t soft, float* out);

/* Host: the kernels' bin index for n probabilities, computed by the same code
 * the device runs (hard: the bin; soft: the count j of centres below p, so the
 * bins are max(j-1, 0) and min(j, K-1)). A CPU test hook. */
int ace_b200_bin_index_host(const float* p, int64_t n, int32_t num_bins, int32_t soft,
                            int32_t right, int32_t* out);

/* Message of the last failed call on this thread ("" if none). */
const char* ace_b200_last_error(void);

/*
 * How the last successful forward, statistics or backward call on this thread
 * was launched (thread-local, like ace_b200_last_error). No counterpart in the
 * reference, whose launches are Triton's; tests use it to check which kernel and
 * which work split a case takes.
 *   kernel          ACE_B200_KERNEL_*
 *   ctas            CTAs of the launch
 *   crosses_batches 1 when a CTA may take voxels of more than one batch
 *   stages          shared-memory ring stages (pipelined kernels), else 0
 *   replicas        lane replicas of the statistics table (forward), else 0
 *   tiles_per_batch tiles of one batch (kernel-specific tile size)
 *   fused_epilogue  1 when the forward's last CTA ran the epilogue
 */
#define ACE_B200_KERNEL_HIST 0      /* hist_kernel: generic forward */
#define ACE_B200_KERNEL_SOFT_PIPE 1 /* soft_fwd_kernel: pipelined soft forward */
#define ACE_B200_KERNEL_GRAD 2      /* grad_kernel: generic backward */
#define ACE_B200_KERNEL_GRAD_PIPE 3 /* grad_tma_kernel: pipelined backward */
#define ACE_B200_KERNEL_MC_PIPE 4   /* mc_fwd_kernel: pipelined many-channel forward */
#define ACE_B200_KERNEL_MC_GRAD 5   /* mc_grad_kernel: pipelined many-channel backward */
typedef struct ace_b200_plan {
  int32_t kernel;
  int32_t ctas;
  int32_t crosses_batches;
  int32_t stages;
  int32_t replicas;
  int32_t fused_epilogue;
  int64_t tiles_per_batch;
} ace_b200_plan;
int ace_b200_last_plan(ace_b200_plan* out);

/* Library version string. */
const char* ace_b200_version(void);

#ifdef __cplusplus
}
#endif

#endif /* ACE_B200_H */
