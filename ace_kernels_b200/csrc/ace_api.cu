// C ABI of libace_b200.so: argument checks, bin tables, launch configuration.
// The kernels themselves are in ace_kernels.cuh.

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include "ace_kernels.cuh"

namespace ace {

// The kernel instances live in ace_kern_{f32,bf16,f16}.cu.
#define ACE_EXTERN(T)                                                                      \
  extern template cudaError_t launch_hist<T>(const FwdParams&, const Variant&, dim3, int, \
                                             cudaStream_t, int);                           \
  extern template cudaError_t launch_grad<T>(const BwdParams&, const Variant&, dim3, int, \
                                             cudaStream_t, int);                           \
  extern template int hist_occupancy<T>(const Variant&, int, int);                         \
  extern template int grad_occupancy<T>(const Variant&, int, int);                         \
  extern template cudaError_t launch_probs<T>(const void*, float*, int64_t, int, int64_t, \
                                              int, cudaStream_t);
ACE_EXTERN(float)
ACE_EXTERN(__nv_bfloat16)
ACE_EXTERN(__half)
#undef ACE_EXTERN

namespace {

thread_local char g_err[512] = "";
thread_local ace_b200_plan g_plan = {-1, 0, 0, 0, 0, 0, 0};

void set_plan(int kernel, int64_t ctas, bool crosses, int stages, int replicas, bool fused,
              int64_t tiles_per_batch) {
  g_plan.kernel = kernel;
  g_plan.ctas = (int32_t)ctas;
  g_plan.crosses_batches = crosses ? 1 : 0;
  g_plan.stages = stages;
  g_plan.replicas = replicas;
  g_plan.fused_epilogue = fused ? 1 : 0;
  g_plan.tiles_per_batch = tiles_per_batch;
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(ACE_B200_ECUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

// torch.linspace(0, 1 + eps32, steps) in fp32, element i. ATen computes
// step = (end - start) / (steps - 1) in fp32 and start + step * i for the first
// half, end - step * (steps - 1 - i) for the second, each with one rounding (a
// fused multiply-add); a CPU test checks the tables against torch.linspace.
float linspace_at(int steps, int i) {
  const float start = 0.0f;
  const float end = 1.0f + 1.1920928955078125e-07f;
  const float step = (end - start) / (float)(steps - 1);
  const int halfway = steps / 2;
  if (i < halfway) return fmaf(step, (float)i, start);
  return fmaf(-step, (float)(steps - 1 - i), end);
}

// Hard: the K upper edges linspace(K + 1)[1:]; soft: the K centres
// linspace(2K + 1)[1::2] (ace_kernels/common.py:17-25).
void table_values(int K, bool soft, float* out) {
  for (int j = 0; j < K; ++j)
    out[j] = soft ? linspace_at(2 * K + 1, 2 * j + 1) : linspace_at(K + 1, j + 1);
}

// With `right`, every entry becomes the next float below it (nextafterf toward
// -inf), so that the kernels' test t < p means t <= p for the true entry. Soft
// binning also gets each interval's base and scale (u = (p - base) * scale /
// 2^21): interior intervals u = (p - lo) / (hi - lo), the end intervals u = p.
void build_table(int K, bool soft, bool right, BinTable& t) {
  float v[kMaxBins];
  table_values(K, soft, v);
  if (right)
    for (int j = 0; j < K; ++j) v[j] = nextafterf(v[j], -INFINITY);
  t.K = K;
  for (int i = 0; i <= K; ++i) {
    float2& e = t.lohi[i];
    e.x = i == 0 ? -10000.0f : v[i - 1];
    e.y = i == K ? 10000.0f : v[i];
    const bool end = i == 0 || i == K;
    t.map[i].x = end ? 0.0f : e.x;
    t.map[i].y = end ? kFixScale : (float)((double)kFixScale / ((double)e.y - (double)e.x));
  }
}

struct DeviceInfo {
  int sms = 0;
};

int sm_count(int dev) {
  static int cache[64] = {0};
  if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    n = 148;
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Workspace layout, each part 256-byte aligned:
//   [accumulators: 8 * b_total * cl * (K + 1) 8-byte words: hist_kernel's
//    [6, rows, K + 1] fp64 sums, or soft_fwd_kernel's [3, rows, K + 1, 2]
//    64-bit integer moments]
//   [histogram counter][epilogue counter]
//   [tile-pool counters: one per batch]
//   [epilogue partial sums: one per epilogue CTA].
// Counters and accumulators are zero between calls.
size_t accum_bytes(int64_t b_total, int64_t cl, int K) {
  return round_up((size_t)8 * b_total * cl * (K + 1) * sizeof(double), 256);
}

size_t pool_bytes(int64_t b_total) { return round_up((size_t)b_total * sizeof(unsigned), 256); }

int64_t epi_ctas(int64_t rows) { return (rows + kEpiRowsPerCta - 1) / kEpiRowsPerCta; }

struct Workspace {
  double* accum;
  unsigned* hist_counter;
  unsigned* epi_counter;
  unsigned* pool;
  float* epi_partial;
};

Workspace carve(void* ws, int64_t b_total, int64_t cl, int K) {
  char* base = static_cast<char*>(ws);
  const size_t a = accum_bytes(b_total, cl, K);
  Workspace w;
  w.accum = reinterpret_cast<double*>(base);
  w.hist_counter = reinterpret_cast<unsigned*>(base + a);
  w.epi_counter = reinterpret_cast<unsigned*>(base + a + 256);
  w.pool = reinterpret_cast<unsigned*>(base + a + 512);
  w.epi_partial = reinterpret_cast<float*>(base + a + 512 + pool_bytes(b_total));
  return w;
}

// Per-variant occupancy, cached (the query costs a few microseconds).
struct OccKey {
  int kind, dtype, V, CM, sm, soft, labels, split, smem, dev;
  bool operator==(const OccKey& o) const { return memcmp(this, &o, sizeof(*this)) == 0; }
};
struct OccHash {
  size_t operator()(const OccKey& k) const {
    size_t h = 1469598103934665603ull;
    const unsigned char* p = reinterpret_cast<const unsigned char*>(&k);
    for (size_t i = 0; i < sizeof(k); ++i) h = (h ^ p[i]) * 1099511628211ull;
    return h;
  }
};

int occupancy(int kind, int dtype, const Variant& v, int smem, int dev) {
  static std::mutex mu;
  static std::unordered_map<OccKey, int, OccHash> cache;
  OccKey key;
  memset(&key, 0, sizeof(key));
  key.kind = kind;
  key.dtype = dtype;
  key.V = v.V;
  key.CM = v.CM;
  key.sm = v.softmax;
  key.soft = v.soft;
  key.labels = v.labels;
  key.split = v.split;
  key.smem = smem;
  key.dev = dev;
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  int n = 1;
  if (kind == 0) {
    if (dtype == ACE_B200_F32) n = hist_occupancy<float>(v, smem, dev);
    else if (dtype == ACE_B200_BF16) n = hist_occupancy<__nv_bfloat16>(v, smem, dev);
    else n = hist_occupancy<__half>(v, smem, dev);
  } else {
    if (dtype == ACE_B200_F32) n = grad_occupancy<float>(v, smem, dev);
    else if (dtype == ACE_B200_BF16) n = grad_occupancy<__nv_bfloat16>(v, smem, dev);
    else n = grad_occupancy<__half>(v, smem, dev);
  }
  std::lock_guard<std::mutex> lock(mu);
  cache[key] = n;
  return n;
}

int elem_size(int dtype) { return dtype == ACE_B200_F32 ? 4 : 2; }

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Checks shared by all entry points. Fills the loss-channel count.
int check_common(const ace_b200_inputs* in, const ace_b200_options* opt, int& CL) {
  if (!in || !opt) return fail(ACE_B200_EINVAL, "null inputs or options");
  if (!in->x) return fail(ACE_B200_EINVAL, "x is null");
  if (in->x_dtype != ACE_B200_F32 && in->x_dtype != ACE_B200_BF16 && in->x_dtype != ACE_B200_F16)
    return fail(ACE_B200_EINVAL, "x_dtype %d is not fp32/bf16/fp16", in->x_dtype);
  if (in->B < 1 || in->C < 1 || in->N < 0)
    return fail(ACE_B200_EINVAL, "bad shape B=%lld C=%lld N=%lld", (long long)in->B,
                (long long)in->C, (long long)in->N);
  if (in->B > 65535) return fail(ACE_B200_EUNSUPPORTED, "B=%lld > 65535", (long long)in->B);
  if (in->C > kMaxClasses)
    return fail(ACE_B200_EUNSUPPORTED, "C=%lld channels > %d", (long long)in->C, kMaxClasses);
  if (in->N > ((int64_t)1 << 40)) return fail(ACE_B200_EUNSUPPORTED, "N too large");
  if (opt->num_bins < 1 || opt->num_bins > kMaxBins)
    return fail(ACE_B200_EUNSUPPORTED, "num_bins=%d outside 1..%d", opt->num_bins, kMaxBins);
  if (opt->offset != 0 && opt->offset != 1) return fail(ACE_B200_EINVAL, "offset must be 0 or 1");
  if (opt->offset == 1 && in->C < 2)
    return fail(ACE_B200_EINVAL, "offset=1 needs C > 1 (the reference ignores it for C = 1)");
  if (opt->activation < 0 || opt->activation > 2) return fail(ACE_B200_EINVAL, "bad activation");
  if (opt->reduction < 0 || opt->reduction > 2) return fail(ACE_B200_EINVAL, "bad reduction");
  if (in->target_kind != ACE_B200_TARGET_LABELS && in->target_kind != ACE_B200_TARGET_DENSE)
    return fail(ACE_B200_EINVAL, "bad target_kind");
  if (in->target_kind == ACE_B200_TARGET_LABELS && in->C < 2)
    return fail(ACE_B200_EINVAL, "label targets need C > 1 (one channel takes dense targets)");
  if (!in->target) return fail(ACE_B200_EINVAL, "target is null");
  if (!aligned(in->x, elem_size(in->x_dtype)) || !aligned(in->target, 4))
    return fail(ACE_B200_EINVAL, "misaligned x or target");
  if (in->target_kind == ACE_B200_TARGET_LABELS && !aligned(in->target, 8))
    return fail(ACE_B200_EINVAL, "int64 labels must be 8-byte aligned");
  CL = (int)in->C - opt->offset;
  if (in->b_offset < 0 || in->b_total < in->b_offset + in->B)
    return fail(ACE_B200_EINVAL, "b_offset=%lld b_total=%lld do not cover B=%lld",
                (long long)in->b_offset, (long long)in->b_total, (long long)in->B);
  if (in->b_total * CL > (int64_t)1 << 24)
    return fail(ACE_B200_EUNSUPPORTED, "too many statistics rows");
  return ACE_B200_OK;
}

// Kernel variant and vector width for this launch (see ACE_VARIANT_CASES).
// `hist`: the forward's many-channel instances (CM > 4) keep only per-voxel
// scalars in registers, so they take two voxels per thread (CM >= 16) where the
// gradient's register-tile instances take one.
Variant choose_variant(const ace_b200_inputs* in, const ace_b200_options* opt, const void* out,
                       bool hist) {
  Variant v;
  v.softmax = opt->activation == ACE_B200_ACT_SOFTMAX && in->C > 1;
  v.soft = opt->soft != 0;
  v.labels = in->target_kind == ACE_B200_TARGET_LABELS;
  v.split = false;
  v.mc = false;
  const int es = elem_size(in->x_dtype);
  const int vmax = 16 / es;
  int V;
  if (v.softmax) {
    // exact channel count up to 4 (no per-channel guards), capacity buckets above
    const int C = (int)in->C;
    v.CM = C <= 4 ? C : C <= 8 ? 8 : C <= 16 ? 16 : C <= 32 ? 32 : 64;
    V = v.CM <= 4 ? vmax : v.CM == 8 ? (vmax < 4 ? vmax : 4) : (v.CM == 16 || hist) ? 2 : 1;
  } else {
    v.CM = 1;
    V = vmax;
  }
  bool ok = V > 1 && in->N % V == 0 && aligned(in->x, (size_t)V * es);
  if (ok && !v.labels) ok = aligned(in->target, (size_t)V * 4);
  if (ok && v.labels) ok = aligned(in->target, 16);
  if (ok && out) ok = aligned(out, (size_t)V * es);
  v.V = ok ? V : 1;
  return v;
}

// One wave of CTAs over the tiles of all batches. Per-batch chunks (each CTA a
// contiguous run of one batch's tiles): always when `flat` is false (the
// gradient: grid (chunks_per_batch, B)), and for the histogram (1-D grid) when a
// wave of them is as short as the flat split; else flat: the tiles of all
// batches in one sequence, each CTA a contiguous run that may cross a batch
// boundary, so that no SM runs a second CTA when B does not divide the wave.
Grid make_grid(const ace_b200_inputs* in, int CL, int offset, int V, int threads,
               int ctas_per_sm, int dev, bool flat) {
  Grid g;
  g.N = in->N;
  g.B = (int)in->B;
  g.C = (int)in->C;
  g.CL = CL;
  g.offset = offset;
  const int64_t tile = (int64_t)threads * V;
  g.tiles = (in->N + tile - 1) / tile;
  const int64_t wave = (int64_t)sm_count(dev) * (ctas_per_sm > 0 ? ctas_per_sm : 1);
  g.chunks_per_batch = 0;
  const int64_t total = g.B * g.tiles;
  const int64_t cb = wave / g.B > 0 ? wave / g.B : 1;
  if (!flat && g.tiles == 0) {  // nothing to do: one CTA per batch
    g.tiles_per_chunk = 1;
    g.chunks_per_batch = 1;
    g.chunks = g.B;
    return g;
  }
  if (g.tiles > 0 && (!flat || wave / g.B >= 1)) {
    const int64_t c = cb < g.tiles ? cb : g.tiles;
    const int64_t tpc = (g.tiles + c - 1) / c;
    if (!flat || tpc <= (total + wave - 1) / wave) {
      g.tiles_per_chunk = tpc;
      g.chunks_per_batch = (int)((g.tiles + tpc - 1) / tpc);
      g.chunks = g.chunks_per_batch * g.B;
      return g;
    }
  }
  int64_t chunks = wave;
  if (chunks > total) chunks = total;
  if (chunks < 1) chunks = 1;
  g.tiles_per_chunk = (total + chunks - 1) / chunks;
  if (g.tiles_per_chunk < 1) g.tiles_per_chunk = 1;
  chunks = (total + g.tiles_per_chunk - 1) / g.tiles_per_chunk;
  if (chunks < 1) chunks = 1;
  g.chunks = (int)chunks;
  return g;
}

int fill_epi(EpiParams& e, int64_t b_total, int CL, double rows_global,
             const ace_b200_options* opt, const ace_b200_epilogue_out& out) {
  if (!out.coef || !out.d || !out.jac || !out.f || !out.loss)
    return fail(ACE_B200_EINVAL, "null epilogue output");
  e.B_total = (int)b_total;
  e.CL = CL;
  e.K = opt->num_bins;
  e.soft = opt->soft != 0;
  e.empty_weight = opt->empty_weight;
  e.ignore_empty = opt->ignore_empty != 0;
  e.reduction = opt->reduction;
  e.rows_global = rows_global > 0 ? rows_global : (double)(b_total * CL);
  if (CL > kMaxClasses) return fail(ACE_B200_EUNSUPPORTED, "too many loss channels");
  for (int c = 0; c < CL; ++c) {
    const float w = opt->class_weights ? opt->class_weights[c] : 1.0f;
    if (!(w >= 0.0f)) return fail(ACE_B200_EINVAL, "class weight %d is negative or NaN", c);
    e.class_w[c] = w;
  }
  e.coef = out.coef;
  e.d = out.d;
  e.jac = out.jac;
  e.f = out.f;
  e.loss = out.loss;
  return ACE_B200_OK;
}

// Shared-memory budget of one soft_fwd_kernel CTA (dynamic part; its static
// barriers, interval constants and epilogue scratch take under 5 KB of the
// 227 KB).
constexpr size_t kSoftSmemBudget = 221 * 1024;

cudaError_t launch_hist_any(const FwdParams& p, const Variant& v, dim3 grid, int smem,
                            int dtype, cudaStream_t s, int dev) {
  if (dtype == ACE_B200_F32) return launch_hist<float>(p, v, grid, smem, s, dev);
  if (dtype == ACE_B200_BF16) return launch_hist<__nv_bfloat16>(p, v, grid, smem, s, dev);
  return launch_hist<__half>(p, v, grid, smem, s, dev);
}

// soft_fwd_kernel: soft binning, int64 labels, softmax over C <= 4 channels,
// inputs whose rows are whole 16-byte vectors (the bulk copies move 16-byte
// multiples). Shared memory: the table [K + 1][C][2][R][3] words (all C channels
// get rows; a dropped background row stays empty), then the ring of stages. R
// lane replicas (32: a warp's lanes never share a bank), reduced while the table
// and two stages do not fit; a replica word takes at most 4 * 16 * 32 / R
// additions per tile and 1023 between folds (values up to 2^21 units), which
// bounds the tiles of an epoch. Returns false when the case does not fit (hist_kernel then
// takes it).
bool soft_fwd_setup(const ace_b200_inputs* in, const ace_b200_options* opt, const Variant& v,
                    FwdParams& p, const Workspace& w, int dev, bool want_epilogue, int& smem,
                    dim3& grid) {
  const int K = opt->num_bins, C = (int)in->C;
  const int es = elem_size(in->x_dtype);
  if (v.V != 16 / es) return false;
  const size_t stage_bytes = (size_t)kPipeTileVoxels * (C * es + 8);
  const size_t replica_bytes = (size_t)(K + 1) * C * 2 * kSoftNW * 4;
  int R = 32;
  auto table = [&](int r) { return round_up(replica_bytes * r, 128); };
  while (R > 4 && table(R) + 2 * stage_bytes > kSoftSmemBudget) R >>= 1;
  if (table(R) + 2 * stage_bytes > kSoftSmemBudget) return false;
  int stages = (int)((kSoftSmemBudget - table(R)) / stage_bytes);
  if (stages > kPipeMaxStages) stages = kPipeMaxStages;
  const int adds_per_tile = kPipeLaneVoxels * kPipeConsumerWarps * (32 / R);
  smem = (int)(table(R) + stages * stage_bytes);
  const int64_t tiles = (in->N + kPipeTileVoxels - 1) / kPipeTileVoxels;
  int64_t ctas = (int64_t)sm_count(dev);  // one CTA per SM
  if (ctas > in->B * tiles) ctas = in->B * tiles;
  if (ctas < 1) ctas = 1;
  p.iacc = reinterpret_cast<unsigned long long*>(w.accum);
  p.pool_ctr = w.pool;
  p.wt_batch = tiles;
  p.epoch = 1023 / adds_per_tile;
  p.stages = stages;
  p.table_bytes = (int)table(R);
  p.R = R;
  p.flush_tiles = 0;
  p.g.N = in->N;
  p.g.B = (int)in->B;
  p.g.C = C;
  p.g.CL = C - opt->offset;
  p.g.offset = opt->offset;
  p.g.chunks = (int)ctas;
  p.g.tiles = tiles;
  p.g.tiles_per_chunk = 0;
  p.g.chunks_per_batch = 0;
  const int64_t rows = in->b_total * p.g.CL;
  p.do_epilogue = want_epilogue && rows <= 8 * kEpiRowsPerCta;
  grid = dim3((unsigned)ctas, 1u);
  return true;
}

// mc_fwd_kernel: int64 labels and a softmax over kMcMinChannels to
// kMcMaxChannels channels, soft or hard binning, rows of whole 16-byte vectors
// and 16-byte aligned logits and labels (the bulk copies move 16-byte multiples). Shared memory: the table (hard: [K][C][R][3] words;
// soft: [K + 1][C][2][R][3]), the bin-edge table (hard), then three or four
// stages of a 1024-voxel tile. R lane replicas (a power of two up to 32, at
// least 4 hard / 8 soft), the most that fit beside three stages, else two; the
// epoch follows from R (the kernel's word ranges). Returns false when the case
// does not fit (hist_kernel then takes it).
constexpr size_t kMcSmemBudget = 218 * 1024;

bool mc_fwd_setup(const ace_b200_inputs* in, const ace_b200_options* opt, Variant& v,
                  FwdParams& p, const Workspace& w, int dev, bool want_epilogue, int& smem,
                  dim3& grid) {
  const int K = opt->num_bins, C = (int)in->C;
  const bool soft = opt->soft != 0;
  const int es = elem_size(in->x_dtype);
  if (!v.softmax || !v.labels || C > kMcMaxChannels || C < kMcMinChannels) return false;
  if (in->N % (16 / es) != 0 || !aligned(in->x, 16) || !aligned(in->target, 16)) return false;
  const int CM = C <= 8 ? 8 : C <= 16 ? 16 : 24;  // the instance's channel capacity
  // a stage holds CM logit rows (the C of the tile, -inf padding) and the labels
  const size_t stage_bytes = (size_t)kMcTileVoxels * (CM * es + 8);
  const size_t slot_bytes = (size_t)(soft ? (K + 1) * 2 : K) * C * 3 * 4;  // one replica
  const size_t lohi_bytes = soft ? 0 : (size_t)(K + 1) * kTabCopies * sizeof(float2);
  auto table = [&](int r) { return round_up(slot_bytes * r, 128); };
  auto need = [&](int r, int st) { return round_up(table(r) + lohi_bytes, 128) + st * stage_bytes; };
  const int r_min = soft ? 8 : 4;
  int R = 0, stages = 0;
  for (int st = 3; st >= 2 && R == 0; --st)
    for (int r = 32; r >= r_min; r >>= 1)
      if (need(r, st) <= kMcSmemBudget) {
        R = r;
        stages = st;
        break;
      }
  if (R == 0) return false;
  if (stages == 3 && need(R, 4) <= kMcSmemBudget) stages = 4;
  const int64_t tiles = (in->N + kMcTileVoxels - 1) / kMcTileVoxels;
  int64_t ctas = (int64_t)sm_count(dev);  // one CTA per SM
  if (ctas > in->B * tiles) ctas = in->B * tiles;
  if (ctas < 1) ctas = 1;
  v.mc = true;
  v.CM = CM;
  smem = (int)need(R, stages);
  p.iacc = reinterpret_cast<unsigned long long*>(w.accum);
  p.pool_ctr = w.pool;
  p.wt_batch = tiles;
  // word ranges (mc_fwd_kernel): soft R - 1 tiles, and at most kMcAggEpoch with the
  // interval-0 aggregates (CM <= 16); hard 2R - 1
  p.epoch = soft ? (v.CM <= 16 && R - 1 > kMcAggEpoch ? kMcAggEpoch : R - 1) : 2 * R - 1;
  p.stages = stages;
  p.table_bytes = (int)table(R);
  p.stage_offset = (int)round_up(table(R) + lohi_bytes, 128);
  p.R = R;
  p.flush_tiles = 0;
  p.g.N = in->N;
  p.g.B = (int)in->B;
  p.g.C = C;
  p.g.CL = C - opt->offset;
  p.g.offset = opt->offset;
  p.g.chunks = (int)ctas;
  p.g.tiles = tiles;
  p.g.tiles_per_chunk = 0;
  p.g.chunks_per_batch = 0;
  const int64_t rows = in->b_total * p.g.CL;
  p.do_epilogue = want_epilogue && rows <= 8 * kEpiRowsPerCta;
  grid = dim3((unsigned)ctas, 1u);
  return true;
}

// One source rank's slot: its rows (at most all b_total * cl) of 3 K tagged 64-bit words.
size_t mailbox_slot_bytes(int64_t b_total, int64_t cl, int K) {
  return round_up((size_t)24 * b_total * cl * K, 16);
}

int hist_impl(const ace_b200_inputs* in, const ace_b200_options* opt, float* hist,
              const ace_b200_epilogue_out* out, void* workspace, size_t ws_bytes, void* stream,
              const ace_b200_exchange* xchg = nullptr) {
  int CL = 0;
  int rc = check_common(in, opt, CL);
  if (rc) return rc;
  if (!hist) return fail(ACE_B200_EINVAL, "hist is null");
  const int K = opt->num_bins;
  const size_t need = ace_b200_workspace_bytes(in->b_total, CL, K);
  if (!workspace || ws_bytes < need)
    return fail(ACE_B200_EINVAL, "workspace of %zu bytes needed, %zu given", need, ws_bytes);
  if (!aligned(workspace, 256)) return fail(ACE_B200_EINVAL, "workspace must be 256-byte aligned");

  FwdParams p;
  memset(&p, 0, sizeof(p));
  if (out) {
    rc = fill_epi(p.epi, in->b_total, CL, in->rows_global, opt, *out);
    if (rc) return rc;
  }
  Variant v = choose_variant(in, opt, nullptr, true);
  const bool soft = opt->soft != 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  const Workspace w = carve(workspace, in->b_total, CL, K);
  p.x = in->x;
  p.target = in->target;
  p.act = opt->activation;
  p.soft = soft;
  p.b_offset = (int)in->b_offset;
  p.B_total = (int)in->b_total;
  p.accum = w.accum;
  p.counter = w.hist_counter;
  p.hist_out = hist;
  build_table(K, soft, opt->right != 0, p.tab);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  p.xchg.world = 1;
  const bool multi = xchg && xchg->world > 1;
  if (multi) {
    if (!out) return fail(ACE_B200_EINVAL, "the exchange needs the epilogue outputs");
    if (xchg->world > kMaxPeers || xchg->rank < 0 || xchg->rank >= xchg->world)
      return fail(ACE_B200_EINVAL, "bad exchange world=%d rank=%d", xchg->world, xchg->rank);
    p.xchg.world = xchg->world;
    p.xchg.rank = xchg->rank;
    p.xchg.slot_bytes = (int64_t)mailbox_slot_bytes(in->b_total, CL, K);
    for (int r = 0; r < xchg->world; ++r) {
      if (!xchg->mailbox[r] || !aligned(xchg->mailbox[r], 16))
        return fail(ACE_B200_EINVAL, "mailbox %d is null or misaligned", r);
      if (xchg->first[r] < 0 || xchg->count[r] < 1 ||
          (int64_t)xchg->first[r] + xchg->count[r] > in->b_total)
        return fail(ACE_B200_EINVAL, "rank %d's samples %d + %d are outside b_total=%lld", r,
                    xchg->first[r], xchg->count[r], (long long)in->b_total);
      p.xchg.mailbox[r] = static_cast<unsigned char*>(xchg->mailbox[r]);
      p.xchg.first[r] = xchg->first[r];
      p.xchg.count[r] = xchg->count[r];
    }
    if (xchg->first[xchg->rank] != in->b_offset || xchg->count[xchg->rank] != in->B)
      return fail(ACE_B200_EINVAL, "this rank's first/count differ from its b_offset/B");
    // batch shards (disjoint samples): only each row's f crosses
    p.xchg.own_rows = 1;
    for (int a = 0; a < xchg->world; ++a)
      for (int b = a + 1; b < xchg->world; ++b)
        if (xchg->first[a] < xchg->first[b] + xchg->count[b] &&
            xchg->first[b] < xchg->first[a] + xchg->count[a])
          p.xchg.own_rows = 0;
  }

  // Soft binning with labels and a softmax over <= 4 channels: soft_fwd_kernel.
  // Its interval distances use the true centres: `right` only decides ties of p
  // with a centre, where both intervals give the same weights.
  v.split = soft && v.softmax && v.labels && v.CM <= 4;
  v.offset = opt->offset;
  int soft_smem = 0;
  dim3 soft_grid;
  if (v.split) v.split = soft_fwd_setup(in, opt, v, p, w, dev, out != nullptr, soft_smem, soft_grid);
  if (v.split && multi && !p.do_epilogue)
    return fail(ACE_B200_EUNSUPPORTED, "the exchange needs the epilogue in the forward (<= 256 rows)");
  if (v.split) {
    build_table(K, true, false, p.tab);
    e = launch_hist_any(p, v, soft_grid, soft_smem, in->x_dtype, s, dev);
    if (e != cudaSuccess) return cuda_fail(e, "soft histogram kernel launch");
    // CTAs start spread over the batches and move on to others' tiles when theirs
    // run out, so any launch with more than one batch may cross batches
    set_plan(ACE_B200_KERNEL_SOFT_PIPE, soft_grid.x, in->B > 1, p.stages, p.R, p.do_epilogue,
             p.wt_batch);
    if (out && !p.do_epilogue) {
      e = launch_epilogue(hist, p.epi, w.epi_counter, w.epi_partial, s);
      if (e != cudaSuccess) return cuda_fail(e, "epilogue kernel launch");
    }
    return ACE_B200_OK;
  }

  // Labels and a softmax over many channels: mc_fwd_kernel, with the same tables
  // as hist_kernel (build_table above).
  int mc_smem = 0;
  dim3 mc_grid;
  if (mc_fwd_setup(in, opt, v, p, w, dev, out != nullptr, mc_smem, mc_grid)) {
    if (multi && !p.do_epilogue)
      return fail(ACE_B200_EUNSUPPORTED, "the exchange needs the epilogue in the forward (<= 256 rows)");
    e = launch_hist_any(p, v, mc_grid, mc_smem, in->x_dtype, s, dev);
    if (e != cudaSuccess) return cuda_fail(e, "many-channel histogram kernel launch");
    set_plan(ACE_B200_KERNEL_MC_PIPE, mc_grid.x, in->B > 1, p.stages, p.R, p.do_epilogue,
             p.wt_batch);
    if (out && !p.do_epilogue) {
      e = launch_epilogue(hist, p.epi, w.epi_counter, w.epi_partial, s);
      if (e != cudaSuccess) return cuda_fail(e, "epilogue kernel launch");
    }
    return ACE_B200_OK;
  }

  if (multi)
    return fail(ACE_B200_EUNSUPPORTED,
                "the exchange runs in the pipelined forwards only (labels and a softmax; soft "
                "binning, or %d..%d channels)", kMcMinChannels, kMcMaxChannels);

  // hist_kernel. Shared-memory table: `entries` words per lane replica. A 32-bit
  // word of a replica takes at most (threads / R) * V additions per tile and must
  // not take more than 1023 between two folds (values up to 2^21 each), so R has
  // a floor; above it, as many replicas as fit in ~100 KB (32 = conflict-free),
  // two CTAs of kHistThreads per SM.
  const int threads = kHistThreads;
  const size_t table_budget = 100 * 1024;
  const int words = soft ? (in->target_kind == ACE_B200_TARGET_LABELS ? 7 : 9) : 3;  // odd
  const int entries = CL * (soft ? K + 1 : K) * words;
  const size_t table_bytes = (size_t)(K + 1) * kTabCopies * sizeof(float4);
  auto r_min = [&](int V) {
    int r = 1;
    while ((threads / r) * V > 1023) r <<= 1;
    return r;
  };
  if (table_bytes + (size_t)entries * r_min(v.V) * 4 > 200 * 1024) v.V = 1;
  int R = 32;
  while (R > r_min(v.V) && table_bytes + (size_t)entries * R * 4 > table_budget) R >>= 1;
  const int smem = (int)(table_bytes + (size_t)entries * R * 4);
  if (smem > 200 * 1024)
    return fail(ACE_B200_EUNSUPPORTED,
                "statistics table of %d channels x %d bins does not fit in shared memory", CL, K);

  const int occ = occupancy(0, in->x_dtype, v, smem, dev);
  p.g = make_grid(in, CL, opt->offset, v.V, threads, occ, dev, true);
  p.R = R;
  p.flush_tiles = 1023 / ((threads / R) * v.V);
  // The last CTA runs the epilogue itself when all statistics fit in its (then
  // free) shared-memory table and the rows are few; otherwise a multi-CTA
  // epilogue kernel follows.
  const int64_t stats = 3 * in->b_total * CL * K;
  const int64_t rows = in->b_total * CL;
  const bool fused = out && stats <= (int64_t)entries * R && rows <= 8 * kEpiRowsPerCta;
  p.do_epilogue = fused ? 1 : 0;

  const dim3 grid((unsigned)p.g.chunks, 1u);
  e = launch_hist_any(p, v, grid, smem, in->x_dtype, s, dev);
  if (e != cudaSuccess) return cuda_fail(e, "histogram kernel launch");
  set_plan(ACE_B200_KERNEL_HIST, p.g.chunks, p.g.chunks_per_batch == 0 && p.g.B > 1, 0, R, fused,
           p.g.tiles);
  if (out && !fused) {
    e = launch_epilogue(hist, p.epi, w.epi_counter, w.epi_partial, s);
    if (e != cudaSuccess) return cuda_fail(e, "epilogue kernel launch");
  }
  return ACE_B200_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// Epilogue over many rows: CTA x takes rows [x * rpc, (x + 1) * rpc); each CTA
// writes its sum of f to the workspace, and the last CTA to finish adds the
// partial sums in CTA order into the loss (no waiting; the counter is left at
// zero for the next call).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) epilogue_kernel(const float* __restrict__ hist,
                                                            float* __restrict__ partial,
                                                            unsigned* __restrict__ counter,
                                                            int rows_per_cta,
                                                            const __grid_constant__ EpiParams E) {
  const int rows = E.B_total * E.CL;
  const int r0 = blockIdx.x * rows_per_cta;
  const int r1 = min(r0 + rows_per_cta, rows);
  const float mine = epilogue_rows(E, hist, rows, 0, r0, r1);
  if (gridDim.x == 1) {
    write_loss_if0(E, mine);
    return;
  }
  __shared__ bool s_last;
  if (threadIdx.x == 0) {
    partial[blockIdx.x] = mine;
    __threadfence();
    s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last || threadIdx.x != 0) return;
  __threadfence();
  float total = 0.0f;
  for (unsigned i = 0; i < gridDim.x; ++i) total = ACE_FADD(total, __ldcg(partial + i));
  *counter = 0u;
  write_loss(E, total);
}

cudaError_t launch_epilogue(const float* hist, const EpiParams& e, unsigned* counter,
                            float* partial, cudaStream_t s) {
  const int rows = e.B_total * e.CL;
  const int ctas = (rows + kEpiRowsPerCta - 1) / kEpiRowsPerCta;
  epilogue_kernel<<<ctas > 0 ? ctas : 1, kThreads, 0, s>>>(hist, partial, counter, kEpiRowsPerCta,
                                                           e);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Barrier of the ranks of an exchange (ace_b200_exchange_barrier), one warp.
// Barrier n (n = this rank's own barrier word + 1): lane d stores n into word
// [rank] of rank d's mailbox header, then lane s waits until word [s] of this
// rank's mailbox reaches n (rank s entered barrier n), at most kXchgWaitNs. The
// words only grow, and each is written by one rank, so no reset is needed.
// wait_ns: the longest lane's wait, or ~0 when a wait ran out.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(32) xchg_barrier_kernel(const __grid_constant__ XchgParams X,
                                                          unsigned long long* wait_ns) {
  const int lane = threadIdx.x;
  unsigned long long* own =
      reinterpret_cast<unsigned long long*>(X.mailbox[X.rank] + kXchgBarrierOffset);
  unsigned long long n = 0ull;
  if (lane == 0) asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(n) : "l"(own + X.rank) : "memory");
  n = __shfl_sync(0xffffffffu, n, 0) + 1ull;
  if (lane < X.world) {
    unsigned long long* a =
        reinterpret_cast<unsigned long long*>(X.mailbox[lane] + kXchgBarrierOffset) + X.rank;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(a), "l"(n) : "memory");
  }
  const unsigned long long t0 = ace_now_ns();
  unsigned long long waited = 0ull;
  if (lane < X.world) {
    for (;;) {
      unsigned long long v;
      asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(own + lane) : "memory");
      const unsigned long long t = ace_now_ns() - t0;
      if (v >= n) {
        waited = t;
        break;
      }
      if (t > kXchgWaitNs) {
        waited = ~0ull;
        break;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, waited, o);
    waited = w > waited ? w : waited;
  }
  if (lane == 0 && wait_ns) *wait_ns = waited;
}

// Scratch of ace_b200_forward_static. A __device__ array has one instance per
// device context, created when the module loads; the first call on each device
// looks its address up (cudaGetSymbolAddress may load the module lazily, which a
// capturing stream does not allow) and clears it (the accumulators and the two
// counters must start at zero; every call leaves them zero again).
__device__ __align__(256) unsigned char g_static_scratch[ACE_B200_STATIC_SCRATCH_BYTES];

std::mutex g_static_mu;
void* g_static_ptr[64];

int static_scratch(cudaStream_t s, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(ACE_B200_EUNSUPPORTED, "device %d >= 64", dev);
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (!g_static_ptr[dev]) {
    cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(s, &st);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamIsCapturing");
    if (st != cudaStreamCaptureStatusNone)
      return fail(ACE_B200_EINVAL,
                  "the first ace_b200_forward_static call on device %d is being captured: "
                  "make one call outside stream capture first", dev);
    void* ptr = nullptr;
    e = cudaGetSymbolAddress((void**)&ptr, g_static_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress");
    e = cudaMemsetAsync(ptr, 0, ACE_B200_STATIC_SCRATCH_BYTES, s);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync of the static scratch");
    g_static_ptr[dev] = ptr;
  }
  *out = g_static_ptr[dev];
  return ACE_B200_OK;
}

}  // namespace ace

using namespace ace;

extern "C" {

size_t ace_b200_workspace_bytes(int64_t b_total, int64_t cl, int32_t num_bins) {
  if (b_total < 1 || cl < 1 || num_bins < 1) return 1024;
  return accum_bytes(b_total, cl, num_bins) + 512 + pool_bytes(b_total) +
         round_up((size_t)epi_ctas(b_total * cl) * sizeof(float), 256);
}

int ace_b200_forward(const ace_b200_inputs* in, const ace_b200_options* opt, float* hist,
                     ace_b200_epilogue_out out, void* workspace, size_t workspace_bytes,
                     void* stream) {
  return hist_impl(in, opt, hist, &out, workspace, workspace_bytes, stream);
}

size_t ace_b200_mailbox_bytes(int64_t b_total, int64_t cl, int32_t num_bins, int32_t world) {
  if (b_total < 1 || cl < 1 || num_bins < 1 || world < 1) return 0;
  return (size_t)kXchgHeaderBytes + 2 * (size_t)world * mailbox_slot_bytes(b_total, cl, num_bins);
}

int ace_b200_mailbox_alloc(size_t bytes, void** ptr_out) {
  if (!ptr_out || bytes == 0) return fail(ACE_B200_EINVAL, "null pointer or zero bytes");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc of the mailbox");
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "cudaMemset of the mailbox");
  }
  *ptr_out = p;
  return ACE_B200_OK;
}

int ace_b200_mailbox_free(void* ptr) {
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? ACE_B200_OK : cuda_fail(e, "cudaFree of the mailbox");
}

int ace_b200_ipc_handle(void* ptr, void* handle_out) {
  static_assert(sizeof(cudaIpcMemHandle_t) == ACE_B200_IPC_HANDLE_BYTES, "IPC handle size");
  if (!ptr || !handle_out) return fail(ACE_B200_EINVAL, "null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  memcpy(handle_out, &h, sizeof(h));
  return ACE_B200_OK;
}

int ace_b200_ipc_open(const void* handle, void** ptr_out) {
  if (!handle || !ptr_out) return fail(ACE_B200_EINVAL, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? ACE_B200_OK : cuda_fail(e, "cudaIpcOpenMemHandle");
}

int ace_b200_ipc_close(void* ptr) {
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? ACE_B200_OK : cuda_fail(e, "cudaIpcCloseMemHandle");
}

int ace_b200_forward_exchange(const ace_b200_inputs* in, const ace_b200_options* opt, float* hist,
                              ace_b200_epilogue_out out, void* workspace, size_t workspace_bytes,
                              const ace_b200_exchange* xchg, void* stream) {
  if (!xchg) return fail(ACE_B200_EINVAL, "null exchange");
  return hist_impl(in, opt, hist, &out, workspace, workspace_bytes, stream, xchg);
}

int ace_b200_exchange_barrier(const ace_b200_exchange* xchg, uint64_t* wait_ns, void* stream) {
  if (!xchg) return fail(ACE_B200_EINVAL, "null exchange");
  if (xchg->world < 1 || xchg->world > kMaxPeers || xchg->rank < 0 || xchg->rank >= xchg->world)
    return fail(ACE_B200_EINVAL, "bad exchange world=%d rank=%d", xchg->world, xchg->rank);
  XchgParams x;
  memset(&x, 0, sizeof(x));
  x.world = xchg->world;
  x.rank = xchg->rank;
  for (int r = 0; r < xchg->world; ++r) {
    if (!xchg->mailbox[r] || !aligned(xchg->mailbox[r], 16))
      return fail(ACE_B200_EINVAL, "mailbox %d is null or misaligned", r);
    x.mailbox[r] = static_cast<unsigned char*>(xchg->mailbox[r]);
  }
  if (wait_ns && !aligned(wait_ns, 8)) return fail(ACE_B200_EINVAL, "wait_ns is misaligned");
  xchg_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      x, reinterpret_cast<unsigned long long*>(wait_ns));
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? ACE_B200_OK : cuda_fail(e, "barrier kernel launch");
}

int ace_b200_forward_static(const ace_b200_inputs* in, const ace_b200_options* opt, float* hist,
                            ace_b200_epilogue_out out, void* stream) {
  int CL = 0;
  int rc = check_common(in, opt, CL);
  if (rc) return rc;
  const size_t need = ace_b200_workspace_bytes(in->b_total, CL, opt->num_bins);
  if (need > ACE_B200_STATIC_SCRATCH_BYTES)
    return fail(ACE_B200_EUNSUPPORTED,
                "b_total=%lld x %d classes x %d bins needs %zu bytes of scratch, more than the "
                "%d of the static scratch: use ace_b200_forward with a workspace",
                (long long)in->b_total, CL, opt->num_bins, need, ACE_B200_STATIC_SCRATCH_BYTES);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  void* scratch = nullptr;
  rc = static_scratch(s, &scratch);
  if (rc) return rc;
  return hist_impl(in, opt, hist, &out, scratch, ACE_B200_STATIC_SCRATCH_BYTES, stream);
}

int ace_b200_hist(const ace_b200_inputs* in, const ace_b200_options* opt, float* hist,
                  void* workspace, size_t workspace_bytes, void* stream) {
  return hist_impl(in, opt, hist, nullptr, workspace, workspace_bytes, stream);
}

int ace_b200_epilogue(const float* hist, int64_t b_total, int64_t cl, double rows_global,
                      const ace_b200_options* opt, ace_b200_epilogue_out out, void* workspace,
                      size_t workspace_bytes, void* stream) {
  if (!hist || !opt) return fail(ACE_B200_EINVAL, "null hist or options");
  if (b_total < 1 || cl < 1 || cl > kMaxClasses)
    return fail(ACE_B200_EINVAL, "bad b_total=%lld cl=%lld", (long long)b_total, (long long)cl);
  if (b_total * cl > (int64_t)1 << 24) return fail(ACE_B200_EUNSUPPORTED, "too many rows");
  if (opt->num_bins < 1 || opt->num_bins > kMaxBins)
    return fail(ACE_B200_EUNSUPPORTED, "num_bins=%d outside 1..%d", opt->num_bins, kMaxBins);
  if (opt->reduction < 0 || opt->reduction > 2) return fail(ACE_B200_EINVAL, "bad reduction");
  EpiParams e;
  memset(&e, 0, sizeof(e));
  int rc = fill_epi(e, b_total, (int)cl, rows_global, opt, out);
  if (rc) return rc;
  const size_t need = ace_b200_workspace_bytes(b_total, cl, opt->num_bins);
  if (!workspace || workspace_bytes < need)
    return fail(ACE_B200_EINVAL, "workspace of %zu bytes needed, %zu given", need, workspace_bytes);
  if (!aligned(workspace, 256)) return fail(ACE_B200_EINVAL, "workspace must be 256-byte aligned");
  const Workspace w = carve(workspace, b_total, cl, opt->num_bins);
  cudaError_t err = launch_epilogue(hist, e, w.epi_counter, w.epi_partial,
                                    static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "epilogue kernel launch");
  return ACE_B200_OK;
}

int ace_b200_backward(const ace_b200_inputs* in, const ace_b200_options* opt,
                      const float* coef, const float* d, const float* jac,
                      const float* grad_output, int32_t grad_per_row, void* dx, void* stream) {
  int CL = 0;
  int rc = check_common(in, opt, CL);
  if (rc) return rc;
  if (!coef || !d || !jac || !grad_output || !dx)
    return fail(ACE_B200_EINVAL, "null coef, d, jac, grad_output or dx");
  if (!aligned(dx, elem_size(in->x_dtype))) return fail(ACE_B200_EINVAL, "misaligned dx");
  const int K = opt->num_bins;
  BwdParams p;
  memset(&p, 0, sizeof(p));
  Variant v = choose_variant(in, opt, dx, false);
  const bool soft = opt->soft != 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  p.x = in->x;
  p.target = in->target;
  p.dx = dx;
  p.act = opt->activation;
  p.soft = soft;
  p.b_offset = (int)in->b_offset;
  p.coef = coef;
  p.d = d;
  p.jac = jac;
  p.grad_out = grad_output;
  p.grad_per_row = grad_per_row != 0;
  build_table(K, soft, opt->right != 0, p.tab);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // grad_tma_kernel: softmax over 2..4 channels, soft binning with labels or hard
  // binning, rows of whole 16-byte vectors. Shared memory: the records of all
  // local batches in `copies` interleaved copies (fewer while the records, the
  // bin table and two stages do not fit), the bin table, then the ring.
  v.offset = opt->offset;
  v.split = v.softmax && v.CM <= 4 && (!soft || v.labels) && v.V == 16 / elem_size(in->x_dtype);
  if (v.split) {
    const size_t stage_bytes =
        (size_t)kPipeTileVoxels * (in->C * elem_size(in->x_dtype) + (soft ? 8 : 0));
    const size_t table_bytes = (size_t)(K + 1) * kTabCopies * sizeof(float2);
    int copies = soft ? 16 : 32;
    const int min_copies = soft ? 2 : 4;
    // records: soft {F - D y, 2 D} for both class flags (16 bytes), hard g coef (4)
    auto fixed = [&](int c) {
      return round_up((size_t)(soft ? 16 : 4) * c * in->B * CL * (K + 1) + table_bytes, 128);
    };
    while (copies > min_copies && fixed(copies) + 2 * stage_bytes > kSoftSmemBudget) copies /= 2;
    if (fixed(copies) + 2 * stage_bytes <= kSoftSmemBudget) {
      int stages = (int)((kSoftSmemBudget - fixed(copies)) / stage_bytes);
      if (stages > kPipeMaxStages) stages = kPipeMaxStages;
      const int64_t tiles = (in->N + kPipeTileVoxels - 1) / kPipeTileVoxels;
      int64_t ctas = sm_count(dev);
      if (ctas > tiles * in->B) ctas = tiles * in->B;
      if (ctas < 1) ctas = 1;
      p.rec_copies = copies;
      p.stages = stages;
      p.stage_offset = (int)fixed(copies);
      p.tiles_per_batch = tiles;
      p.g.N = in->N;
      p.g.B = (int)in->B;
      p.g.C = (int)in->C;
      p.g.CL = CL;
      p.g.offset = opt->offset;
      const int smem = (int)(fixed(copies) + stages * stage_bytes);
      const dim3 grid((unsigned)ctas, 1u);
      if (in->x_dtype == ACE_B200_F32) e = launch_grad<float>(p, v, grid, smem, s, dev);
      else if (in->x_dtype == ACE_B200_BF16) e = launch_grad<__nv_bfloat16>(p, v, grid, smem, s, dev);
      else e = launch_grad<__half>(p, v, grid, smem, s, dev);
      if (e != cudaSuccess) return cuda_fail(e, "gradient kernel launch");
      set_plan(ACE_B200_KERNEL_GRAD_PIPE, ctas, in->B > 1, stages, 0, false, tiles);
      return ACE_B200_OK;
    }
    v.split = false;
  }

  // mc_grad_kernel: softmax over kMcMinChannels..kMcMaxChannels channels, soft
  // binning with labels or hard binning, rows of whole 16-byte vectors, 16-byte
  // aligned logits, labels and dx. Shared memory: the records of all local
  // batches in `copies` interleaved copies (the most that fit beside three
  // stages, else two), the bin table (hard), then the ring of 1024-voxel tiles.
  if (v.softmax && (!soft || v.labels) && in->C >= kMcMinChannels && in->C <= kMcMaxChannels &&
      in->N % (16 / elem_size(in->x_dtype)) == 0 && aligned(in->x, 16) && aligned(dx, 16) &&
      (!soft || aligned(in->target, 16))) {
    const int CM = in->C <= 8 ? 8 : in->C <= 16 ? 16 : 24;  // the instance's channel capacity
    const size_t stage_bytes =
        (size_t)kMcTileVoxels * (in->C * elem_size(in->x_dtype) + (soft ? 8 : 0));
    const size_t table_bytes = soft ? 0 : (size_t)(K + 1) * kTabCopies * sizeof(float2);
    auto fixed = [&](int c) {
      return round_up((size_t)(soft ? 16 : 4) * c * in->B * CL * (K + 1) + table_bytes, 128);
    };
    int copies = 0, stages = 0;
    for (int st = 3; st >= 2 && copies == 0; --st)
      for (int c = soft ? 16 : 32; c >= (soft ? 2 : 1); c /= 2)  // soft: 16-byte record pairs
        if (fixed(c) + st * stage_bytes <= kMcSmemBudget) {
          copies = c;
          stages = st;
          break;
        }
    if (copies > 0) {
      if (stages == 3 && fixed(copies) + 4 * stage_bytes <= kMcSmemBudget) stages = 4;
      const int64_t tiles = (in->N + kMcTileVoxels - 1) / kMcTileVoxels;
      int64_t ctas = sm_count(dev);
      if (ctas > tiles * in->B) ctas = tiles * in->B;
      if (ctas < 1) ctas = 1;
      v.mc = true;
      v.split = false;
      v.CM = CM;
      p.rec_copies = copies;
      p.stages = stages;
      p.stage_offset = (int)fixed(copies);
      p.tiles_per_batch = tiles;
      p.g.N = in->N;
      p.g.B = (int)in->B;
      p.g.C = (int)in->C;
      p.g.CL = CL;
      p.g.offset = opt->offset;
      const int smem = (int)(fixed(copies) + stages * stage_bytes);
      const dim3 grid((unsigned)ctas, 1u);
      if (in->x_dtype == ACE_B200_F32) e = launch_grad<float>(p, v, grid, smem, s, dev);
      else if (in->x_dtype == ACE_B200_BF16) e = launch_grad<__nv_bfloat16>(p, v, grid, smem, s, dev);
      else e = launch_grad<__half>(p, v, grid, smem, s, dev);
      if (e != cudaSuccess) return cuda_fail(e, "gradient kernel launch");
      set_plan(ACE_B200_KERNEL_MC_GRAD, ctas, in->B > 1, stages, 0, false, tiles);
      return ACE_B200_OK;
    }
  }

  // grad_kernel. Record copies: as many as fit in 96 KB (two CTAs per SM keep
  // their tables).
  int copies = soft ? 16 : 32;
  auto grad_smem = [&](int c) {
    return (size_t)(K + 1) * kTabCopies * sizeof(float2) + (size_t)(soft ? 8 : 4) * c * CL * (K + 1);
  };
  // (at least one 16-byte store of copies per record: 2 soft, 4 hard)
  const int min_copies = soft ? 2 : 4;
  while (copies > min_copies && grad_smem(copies) > 96 * 1024) copies /= 2;
  // the many-channel kernel keeps every channel's gp per thread: C x threads x V floats
  const size_t scratch =
      (v.softmax && v.CM > 4) ? (size_t)in->C * kThreads * v.V * sizeof(float) : 0;
  const int smem = (int)(grad_smem(copies) + scratch);
  if (smem > 227 * 1024) return fail(ACE_B200_EUNSUPPORTED, "gradient tables do not fit");
  p.rec_copies = copies;
  const int occ = occupancy(1, in->x_dtype, v, smem, dev);
  p.g = make_grid(in, CL, opt->offset, v.V, kThreads, occ, dev, false);
  const dim3 grid((unsigned)p.g.chunks_per_batch, (unsigned)p.g.B);
  if (in->x_dtype == ACE_B200_F32) e = launch_grad<float>(p, v, grid, smem, s, dev);
  else if (in->x_dtype == ACE_B200_BF16) e = launch_grad<__nv_bfloat16>(p, v, grid, smem, s, dev);
  else e = launch_grad<__half>(p, v, grid, smem, s, dev);
  if (e != cudaSuccess) return cuda_fail(e, "gradient kernel launch");
  set_plan(ACE_B200_KERNEL_GRAD, (int64_t)p.g.chunks_per_batch * p.g.B, false, 0, 0, false,
           p.g.tiles);
  return ACE_B200_OK;
}

int ace_b200_probs(const ace_b200_inputs* in, int32_t activation, float* probs, void* stream) {
  if (!in || !in->x || !probs) return fail(ACE_B200_EINVAL, "null x or probs");
  if (in->B < 1 || in->C < 1 || in->C > kMaxClasses || in->N < 0)
    return fail(ACE_B200_EINVAL, "bad shape");
  if (activation < 0 || activation > 2) return fail(ACE_B200_EINVAL, "bad activation");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (in->x_dtype == ACE_B200_F32)
    e = launch_probs<float>(in->x, probs, in->B, (int)in->C, in->N, activation, s);
  else if (in->x_dtype == ACE_B200_BF16)
    e = launch_probs<__nv_bfloat16>(in->x, probs, in->B, (int)in->C, in->N, activation, s);
  else if (in->x_dtype == ACE_B200_F16)
    e = launch_probs<__half>(in->x, probs, in->B, (int)in->C, in->N, activation, s);
  else
    return fail(ACE_B200_EINVAL, "bad x_dtype");
  if (e != cudaSuccess) return cuda_fail(e, "probability kernel launch");
  return ACE_B200_OK;
}

int ace_b200_bin_table(int32_t num_bins, int32_t soft, float* out) {
  if (!out) return fail(ACE_B200_EINVAL, "out is null");
  if (num_bins < 1 || num_bins > kMaxBins)
    return fail(ACE_B200_EUNSUPPORTED, "num_bins=%d outside 1..%d", num_bins, kMaxBins);
  table_values(num_bins, soft != 0, out);
  return ACE_B200_OK;
}

int ace_b200_bin_index_host(const float* p, int64_t n, int32_t num_bins, int32_t soft,
                            int32_t right, int32_t* out) {
  if ((!p || !out) && n > 0) return fail(ACE_B200_EINVAL, "null p or out");
  if (num_bins < 1 || num_bins > kMaxBins)
    return fail(ACE_B200_EUNSUPPORTED, "num_bins=%d outside 1..%d", num_bins, kMaxBins);
  BinTable t;
  build_table(num_bins, soft != 0, right != 0, t);
  for (int64_t i = 0; i < n; ++i) {
    float2 lohi;
    out[i] = ace_locate(p[i], t.lohi, 1, num_bins, (float)num_bins, soft != 0, lohi);
  }
  return ACE_B200_OK;
}

const char* ace_b200_last_error(void) { return g_err; }

int ace_b200_last_plan(ace_b200_plan* out) {
  if (!out) return fail(ACE_B200_EINVAL, "out is null");
  *out = g_plan;
  return ACE_B200_OK;
}

const char* ace_b200_version(void) { return "ace_b200 0.1.0 (sm_100a)"; }

}  // extern "C"
