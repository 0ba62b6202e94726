// openTSNE-style FFT-grid t-SNE optimizer for B200: data layout and kernels.
//
// Layout in HBM (one session = one embedding run):
//   P        symmetric CSR in the caller's order (row_ptr int32[n+1], col int32[nnz],
//            val f32[nnz]) and a copy in the internal (spatial) order with rows
//            padded to groups of four entries, streamed as int4 / float4.
//   y[2]     float2[n] double-buffered layout (the gradient of iteration t
//            reads y[cur] while the fused update writes y[cur^1]).
//   update, gains  float2[n]
//   charges  ChargeCell[G*G]  bilinear charges {1, x, y} per grid node, 64-bit fixed point
//   rowspec  float2[G][G+1][3]  x-half-spectra of the three charge planes
//   krow     float2[G][G+1]     x-transforms of the q and q^2 kernel rows
//   colspec  float2[G][G+1][4]  y-inverted products (q2, xq2, yq2, q)
//   pot      float4[G*G]   potentials {phi_q2, phi_xq2, phi_yq2, phi_q}
//   stats    LayoutStats   bounds/sums of the layout and the normaliser Z
//
// Per iteration: splat -> fft_rows_fwd -> fft_cols -> fft_rows_inv -> gradient+update
// -> layout statistics (a sharded session adds an all-reduce of the charges
// after the splat and an all-gather of the updated rows before the statistics).
#pragma once

#include "fe_common.cuh"

#include <cuda_runtime.h>

#include <vector>

namespace fe {

class RankGroup;

// Layout statistics carried between kernels (device resident).
// One grid node's charges {sum w, sum w x, sum w y} in fixed point (+ pad to 32 B).
struct ChargeCell {
  unsigned long long m, mx, my, pad;
};

struct GridGeom {
  float mean_x, mean_y;
  float lower_x, lower_y;
  float spacing, inv_spacing;  // node spacing of the (uniform) FFT grid
  int boxes;                   // Lagrange mode: boxes per side (0 in bilinear mode)
  float inv_box;               // Lagrange mode: 1 / box width
};

// Charges are accumulated in signed 64-bit fixed point, so the splat's
// atomics are associative and the result does not depend on their order
// (runs are bit-reproducible, and sharded runs sum exactly).  Scales are
// powers of two chosen so that the largest possible node total stays below
// 2^62: sum of weights <= n, and |x|, |y| <= the grid box half extent.
struct ChargeScales {
  double m;   // weight scale
  double xy;  // coordinate-weighted scale
};

struct LayoutStats {
  double sum_x, sum_y;        // sums of the raw (uncentred) layout
  float min_x, max_x;         // bounds of the raw layout
  float min_y, max_y;
  int center;                 // 1: subtract the mean before use (iterations)
  int lagrange;               // interpolation: 0 bilinear (the reference's), 1 Lagrange 3-node boxes
  double z;                   // sum_i interp(phi_q)(y_i) - n
  float inv_z;                // 1 / max(z, FLT_MIN)
  unsigned int row_groups_taken;  // grad_update_kernel work counter
  unsigned int fft_counter;       // last-block tickets
  unsigned int stats_counter;
  unsigned int stage_taken;       // staged_grad_kernel work counter
  unsigned int stage_count;       // staged row blocks (set at each reorder)
  unsigned int group_count;       // 32-row groups left to grad_update_kernel (set at each reorder)
  // Derived once per layout by the statistics kernel (grid_geometry and
  // charge_scales below) and read by every later kernel of the iteration,
  // instead of every thread re-deriving them with double divisions.
  GridGeom geom;
  ChargeScales scales;
};

#ifdef __CUDACC__
// Grid geometry of compute_gradient_fft_grid_f (src/tsne_neighbors.cpp:1084-1106),
// evaluated on the centred layout.  Rounding is monotonic, so the bounds of the
// centred layout equal the raw bounds minus the float mean, exactly.
__device__ __forceinline__ GridGeom grid_geometry(const LayoutStats& s, int n, int g) {
  GridGeom q;
  if (s.center) {
    q.mean_x = static_cast<float>(s.sum_x / static_cast<double>(n));
    q.mean_y = static_cast<float>(s.sum_y / static_cast<double>(n));
  } else {
    q.mean_x = 0.0f;
    q.mean_y = 0.0f;
  }
  const float min_x = s.min_x - q.mean_x, max_x = s.max_x - q.mean_x;
  const float min_y = s.min_y - q.mean_y, max_y = s.max_y - q.mean_y;
  q.boxes = 0;
  q.inv_box = 0.0f;
  if (s.lagrange) {
    // FIt-SNE's box grid: square boxes of about one unit of the embedding
    // (intervals_per_integer = 1), at least 50 per side, covering the layout's
    // bounding square from its lower corner; three interpolation nodes per box
    // and side at (j + 1/2) / 3, so the nodes form a uniform grid of spacing
    // box / 3 for the FFT convolution.  At most g / 3 boxes fit the grid.
    float extent = fmaxf(max_x - min_x, max_y - min_y);
    if (!isfinite(extent) || extent <= 0.0f) extent = 1.0f;
    const int boxes = max(1, min(g / 3, max(50, static_cast<int>(ceilf(extent)))));
    const float box = extent / static_cast<float>(boxes);
    q.lower_x = min_x;
    q.lower_y = min_y;
    q.boxes = boxes;
    q.inv_box = 1.0f / box;
    q.spacing = box / 3.0f;
    q.inv_spacing = 1.0f / q.spacing;
    return q;
  }
  const float cx = 0.5f * (min_x + max_x);
  const float cy = 0.5f * (min_y + max_y);
  float span = fmaxf(max_x - min_x, max_y - min_y);
  if (!isfinite(span) || span <= 0.0f) span = 1.0f;
  const float half = 0.55f * span + 1.0e-3f;
  q.lower_x = cx - half;
  q.lower_y = cy - half;
  q.spacing = (2.0f * half) / static_cast<float>(g - 1);
  q.inv_spacing = 1.0f / q.spacing;
  return q;
}

__device__ __forceinline__ double pow2_scale_for(double max_total) {
  int e = 0;
  frexp(fmax(max_total, 1.0), &e);  // max_total < 2^e
  return ldexp(1.0, 62 - e);
}
__device__ __forceinline__ ChargeScales charge_scales(const GridGeom& q, int n, int g) {
  const float extent = q.spacing * static_cast<float>(g - 1);
  const double xmax = fmax(fmax(fabs(static_cast<double>(q.lower_x)), fabs(static_cast<double>(q.lower_x) + extent)),
                           fmax(fabs(static_cast<double>(q.lower_y)), fabs(static_cast<double>(q.lower_y) + extent)));
  // Lagrange weights reach 1.875 in magnitude per dimension (3.52 per node),
  // so a node's total can exceed the bilinear bound by 4x: two more bits.
  const double headroom = q.boxes > 0 ? 4.0 : 1.0;
  ChargeScales c;
  c.m = pow2_scale_for(headroom * static_cast<double>(n));
  c.xy = pow2_scale_for(headroom * static_cast<double>(n) * (xmax + 1.0));
  return c;
}

// Lagrange mode: the box of a point and the quadratic Lagrange weights of its
// position in the box at the three nodes t_j = (j + 1/2) / 3 of each side
// (FIt-SNE's interpolation, p = 3).  Node (j, k) of box (bx, by) is grid node
// (3 bx + j, 3 by + k).  Spread and gather use these same weights.
struct LagrangeCell {
  int bx, by;
  float wx[3], wy[3];
};
__device__ __forceinline__ void lagrange_weights(float t, float* w) {
  const float t0 = 1.0f / 6.0f, t1 = 0.5f, t2 = 5.0f / 6.0f;
  w[0] = 4.5f * (t - t1) * (t - t2);
  w[1] = -9.0f * (t - t0) * (t - t2);
  w[2] = 4.5f * (t - t0) * (t - t1);
}
__device__ __forceinline__ LagrangeCell lagrange_cell(float px, float py, const GridGeom& q) {
  LagrangeCell c;
  const float ux = (px - q.lower_x) * q.inv_box;
  const float uy = (py - q.lower_y) * q.inv_box;
  c.bx = max(0, min(q.boxes - 1, static_cast<int>(floorf(ux))));
  c.by = max(0, min(q.boxes - 1, static_cast<int>(floorf(uy))));
  lagrange_weights(fminf(1.0f, fmaxf(0.0f, ux - static_cast<float>(c.bx))), c.wx);
  lagrange_weights(fminf(1.0f, fmaxf(0.0f, uy - static_cast<float>(c.by))), c.wy);
  return c;
}

// Clamped grid coordinates, cell origin and bilinear fractions of a point
// (src/tsne_neighbors.cpp:1114-1128 and 760-775 use the same expressions).
struct Cell {
  int x0, y0;
  float tx, ty;
};
__device__ __forceinline__ Cell grid_cell(float px, float py, const GridGeom& q, int g) {
  const float raw_x = (px - q.lower_x) * q.inv_spacing;
  const float raw_y = (py - q.lower_y) * q.inv_spacing;
  const float gmax = static_cast<float>(g - 1);
  const float cx = fmaxf(0.0f, fminf(gmax, raw_x));
  const float cy = fmaxf(0.0f, fminf(gmax, raw_y));
  Cell c;
  c.x0 = max(0, min(g - 2, static_cast<int>(floorf(cx))));
  c.y0 = max(0, min(g - 2, static_cast<int>(floorf(cy))));
  c.tx = cx - static_cast<float>(c.x0);
  c.ty = cy - static_cast<float>(c.y0);
  return c;
}
#endif

// A round of the attraction kernel (four rows, eight lanes each) whose longest
// row needs more passes than this is run row by row with 32 lanes instead.
constexpr int kLongRoundPasses = 6;

// Staged row blocks (staged_grad_kernel; opt-in, FASTEMBEDR_B200_STAGED_ATTRACTION=1).
// Internal rows are cut into blocks of kStageRows; a block whose entries
// reference at most kStageCap distinct points (its column union) and span at
// most kStageSpan internal indices gets its union list and 16-bit union-local
// column indices at each reorder, and its attraction gathers y_j from the
// union staged in shared memory instead of from L2.  Other blocks stay with
// grad_update_kernel.  Results are bit-identical either way.  On the
// benchmark's mixtures a union holds each point only 1.2-1.6 times, and a
// block waits for its longest round, so the staged kernel measured slower
// (0.80 ms against 0.60 ms per iteration at N = 1M); it stays off by default.
constexpr int kStageRows = 128;
constexpr int kStageRounds = kStageRows / 4;
constexpr int kStageThreads = 1024;
constexpr int kStageCap = 24576;        // 192 KB of float2 in shared memory
constexpr int kStageSpan = 1 << 20;     // bitmap of the build: 128 KB
constexpr int kStageBuildThreads = 512;

// Exactly one of these modes is run by the fused gradient kernel.
enum GradMode { kGradUpdate = 0, kGradOnly = 1 };

constexpr int kKindCountMax = 9;

struct TsneSession {
  int device = 0;
  int n = 0;
  int grid = 0;       // G
  int fft = 0;        // M = 2G
  int log_fft = 0;
  long long nnz = 0;      // symmetric entries (both directions)
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  Arena arena;

  // P in the caller's point order: unpadded CSR, columns ascending (the
  // reference's CSR exactly).  Canonical copy; never permuted.
  int* row_ptr = nullptr;
  int* col = nullptr;
  float* val = nullptr;
  // P in the internal point order, rows contiguous and padded to whole groups
  // of four entries with (col = row, val = 0): row r occupies groups
  // row_ptr4[r] .. row_ptr4[r+1]-1 of csr4_col / csr4_val (int4 / float4).
  int* row_ptr4 = nullptr;         // n + 1 offsets, in 16-byte groups
  int4* csr4_col = nullptr;
  float4* csr4_val = nullptr;
  // Staged row blocks: per entry (csr4 positions) the index of its column in
  // the block's union; per block the union list (sorted internal indices, at
  // the block's first entry position, since a union is never longer than its
  // block's entries), {union offset, union size, staged?, entries} and the
  // order of its 32 four-row rounds (most expensive first).
  uint2* stage_col16 = nullptr;    // four 16-bit indices per csr4 group
  int* stage_union = nullptr;
  int4* stage_meta = nullptr;
  unsigned char* stage_rounds = nullptr;
  unsigned int* stage_cost = nullptr;
  unsigned int* stage_cost_sorted = nullptr;
  int* stage_ids = nullptr;
  int* stage_order = nullptr;      // staged blocks, most expensive first
  bool stage_enabled = true;       // FASTEMBEDR_B200_STAGED_ATTRACTION
  long long csr4_groups = 0;       // groups in use
  long long csr4_capacity = 0;     // groups allocated
  float2* y[2] = {nullptr, nullptr};
  int cur = 0;
  float2* update = nullptr;
  float2* gains = nullptr;
  float2* grad_out = nullptr;  // kGradOnly target
  float2* attraction = nullptr;  // staged rows' attraction sums, for staged_finish_kernel
  LayoutStats* stats = nullptr;
  double* update_partials = nullptr;  // 6 per block
  double* z_partials = nullptr;       // one per grid row
  ChargeCell* charges = nullptr;
  float2* rowspec = nullptr;
  float2* krow = nullptr;
  float2* colspec = nullptr;
  float4* pot = nullptr;
  float2* twiddle = nullptr;  // FFT twiddles (fft_twiddle_table)

  int interp = 0;  // 0 bilinear (the reference's), 1 Lagrange 3-node boxes (FIt-SNE)
  int update_blocks = 0;
  int update_threads = 256;

  // Optional per-kernel CUDA-event timing (bench / profiling).
  bool profile = false;
  std::vector<cudaEvent_t> events;
  std::vector<int> event_kind;
  double kernel_ms[kKindCountMax] = {0};
  long long kernel_launches[kKindCountMax] = {0};
  long long iterations_run = 0;

  // Captured iteration chunks, keyed by chunk length, parameter set and the
  // layout double-buffer parity they start from (least recently used evicted).
  struct GraphEntry {
    cudaGraphExec_t exec;
    int iters;
    int cur;
    float params[5];
    unsigned long long used;
  };
  std::vector<GraphEntry> graphs;
  unsigned long long graph_clock = 0;
  bool use_graphs = true;

  // Reorder scratch, carved from the session arena so that a periodic
  // reorder neither allocates nor synchronises with the host.
  unsigned int* ro_keys = nullptr;
  unsigned int* ro_keys_sorted = nullptr;
  int* ro_idx = nullptr;
  int* ro_order = nullptr;
  int* ro_perm = nullptr;
  int* ro_rank = nullptr;
  int* ro_groups = nullptr;
  float2* ro_update = nullptr;
  float2* ro_gains = nullptr;
  void* ro_temp = nullptr;
  size_t ro_temp_bytes = 0;
  // The order in which grad_update_kernel's warps take 32-row groups: most
  // expensive first (longest-processing-time first), so the groups holding
  // hub rows -- rows of P with thousands of entries -- start early and
  // overlap with the many short ones instead of forming the kernel's tail.
  // Rebuilt with the internal order.
  int* group_order = nullptr;
  unsigned int* group_cost = nullptr;
  unsigned int* group_cost_sorted = nullptr;
  int* group_ids = nullptr;

  // Sharding across processes, one per GPU (session_shard).  Every rank holds
  // the whole layout; rank r owns internal rows [row_begin, row_end), the r-th
  // block of rows_per_rank rows: it splats, attracts and updates only those,
  // the charge grid is summed with one all-reduce and the updated rows are
  // all-gathered, in place, once per iteration.  Blocks are whole multiples
  // of kStageRows (128) rows, so neither a warp nor a staged row block
  // straddles two ranks and the splat combines the same lanes as an unsharded
  // run; point arrays have room for the padding of the last block (kPadRows).
  static constexpr int kMaxRanks = 256;
  static constexpr int kPadRows = kStageRows * kMaxRanks;
  bool sharded = false;
  int shard_ranks = 1;
  int shard_rank = 0;
  int rows_per_rank = 0;
  int row_begin = 0;
  int row_end = 0;
  void* comm = nullptr;  // ncclComm_t
  bool own_comm = false;  // destroyed with the session (not when lent by the caller)
  // Single-process multi-device mode (multi_device.cu): the host-side group of
  // the ranks this process runs.  Collectives then go through the group (every
  // rank agrees on the host before each one; see rank_group.h), at most one
  // collective of this rank is in flight at a time, and iterations launch
  // without graphs, so that an abort can only ever end the newest collective.
  RankGroup* group = nullptr;
  cudaEvent_t collective_done = nullptr;  // completion of the newest collective
  bool collective_pending = false;
  long long collectives_issued = 0;
  double stall_limit_s = 0.0;  // a collective taking longer is treated as a failed peer
  long long inject_failure_at = -1;  // FASTEMBEDR_B200_INJECT_HOST_FAILURE for this rank

  // Spatial ordering: internal point r is the caller's point perm[r], and
  // caller point i is internal point rank[i].
  int* perm = nullptr;
  int* rank = nullptr;
  bool identity_perm = true;
  int reorder_every = 0;          // iterations between reorders (0 = never)
  long long next_reorder = 0;
};

enum KernelKind {
  kKindSplat = 0,
  kKindFftRows = 1,
  kKindFftCols = 2,
  kKindFftRowsInv = 3,
  kKindGradUpdate = 4,
  kKindChargeSum = 5,     // sharded: all-reduce of the charge grid
  kKindLayoutGather = 6,  // sharded: all-gather of the updated rows
  kKindLayoutStats = 7,   // statistics of the new layout
  kKindStagedGrad = 8,    // attraction + update of the staged row blocks
  kKindCount = 9
};
const char* kernel_kind_name(int kind);

// ---- P construction (tsne_affinity.cu) ----
// Builds the symmetric CSR (caller order, columns ascending) on the device
// from column-major KNN.  dist_is_double selects the element type of `dist`.
// Temporaries are freed before returning; the CSR arrays are allocated with
// cudaMalloc into *out_*.
int build_p_device(const int* d_idx, const void* d_dist, bool dist_is_double, int n, int k,
                   int index_offset, float perplexity, cudaStream_t stream, int** out_row_ptr,
                   int** out_col, float** out_val, long long* out_nnz);

// Validates and uploads a host CSR (parity hooks, resume).
int upload_csr(const int* row_ptr, const int* col, const float* val, int n, cudaStream_t stream,
               int** out_row_ptr, int** out_col, float** out_val, long long* out_nnz);

// ---- session (tsne_session.cu) ----
int session_create(TsneSession** out, int n, int grid, int* d_row_ptr, int* d_col, float* d_val,
                   long long nnz, cudaStream_t stream);
void session_destroy(TsneSession* s);
int session_set_layout(TsneSession* s, const float* y, bool host, bool center);
int session_random_layout(TsneSession* s, unsigned int seed);
int session_iterate(TsneSession* s, int iters, float exaggeration, float momentum,
                    float learning_rate, float min_gain, float max_step_norm);
int session_gradient(TsneSession* s, float exaggeration, float* grad_host, double* z_out);
// Captures the iteration chunks of one parameter set now, so that a later
// session_iterate with these parameters launches without capturing.
int session_prepare(TsneSession* s, float exaggeration, float momentum, float learning_rate, float min_gain,
                    float max_step_norm);
int session_get_layout(TsneSession* s, float* out, bool host);
// Optimizer state in the caller's point order.
int session_set_state(TsneSession* s, const float* update, const float* gains, bool host);
int session_get_state(TsneSession* s, float* update, float* gains, bool host);
int session_reset_state(TsneSession* s);
// Unpadded CSR P in the caller's point order, columns ascending.
int session_get_p(TsneSession* s, int* row_ptr, int* col, float* val);

// ---- sharding (tsne_shard.cu) ----
// Makes this session rank `rank` of an nranks-way sharded run, on the
// communicator `comm` (lent by the caller, kept) or, when comm is null, on a
// new one joined with unique_id (ncclUniqueId bytes from rank 0; destroyed
// with the session).  Every rank must hold an identical session (same P,
// layout and state) and make the same calls in the same order from then on.
int session_shard(TsneSession* s, const void* unique_id, void* comm, int nranks, int rank);
// In-place all-gather of the per-rank row blocks of a point array.
int shard_gather_rows(TsneSession* s, float2* rows);
// Sum of the charge grids of all ranks, in place.
int shard_sum_charges(TsneSession* s);
// One uncaptured round of both collectives on buffers they leave unchanged
// (fresh sessions only: zero charges and zero steps).
int shard_warm_up(TsneSession* s);
// Grouped sessions: waits until this rank's newest collective has completed,
// bounded by stall_limit_s (then the group is failed, which aborts every
// communicator, and the wait resumes, bounded again).  No-op otherwise.
int shard_quiesce(TsneSession* s);
void shard_release(TsneSession* s);

// ---- one process, several GPUs (multi_device.cu) ----
// One openTSNE run from KNN as one sharded session per device, one host
// thread each, in this process; what the one-shot entry points run when
// FASTEMBEDR_B200_DEVICES lists two or more devices.
struct MultiDeviceTsne {
  std::vector<int> devices;
  const int* indices = nullptr;    // column-major n x k, host or (on_device) the caller's device
  const void* distances = nullptr;
  bool dist_double = false;
  bool on_device = false;
  int caller_device = 0;
  const float* init = nullptr;     // host, or null for the hashed random start
  unsigned int seed = 0;
  int n = 0;
  int k = 0;
  int index_offset = 0;
  float perplexity = 0.0f;
  int grid = 0;
  int early_iter = 0;
  float early_exaggeration = 0.0f;
  float initial_momentum = 0.0f;
  float lr_early = 0.0f;
  int n_iter = 0;
  float exaggeration = 0.0f;
  float final_momentum = 0.0f;
  float lr_normal = 0.0f;
  float min_gain = 0.0f;
  float max_step_norm = 0.0f;
  float* out = nullptr;            // host, row-major n x 2
  const void* unique_id = nullptr;  // set by opentsne_multi_device
};
// The devices FASTEMBEDR_B200_DEVICES lists ("0,1,..."; empty when unset);
// status 1 for a malformed list, an ordinal out of range or a repeat.
int multi_device_list(std::vector<int>* devices);
int opentsne_multi_device(MultiDeviceTsne job);

// ---- ordering and the internal copy of P (tsne_reorder.cu) ----
// Chooses the internal point order -- Morton order of the current layout when
// by_layout, else the caller's order -- permutes the point arrays, and
// rebuilds the internal-order, group-padded copy of P from the caller CSR.
// Only the first call (from session_create) sizes the padded copy and waits
// for the device; later calls are asynchronous on the session stream.
int session_reorder(TsneSession* s, bool by_layout);
// CUB temporary storage the reorder needs for n points.
int reorder_temp_bytes(int n, size_t* bytes);
// Orders this rank's 32-row groups by estimated cost, most expensive first.
int build_group_order(TsneSession* s);
// Drops every captured iteration chunk.
void drop_graphs(TsneSession* s);
// out[perm[r]] = in[r] (internal -> caller order) and out[r] = in[perm[r]].
int launch_unpermute(TsneSession* s, const float2* in, float2* out);
int launch_permute_in(TsneSession* s, const float2* in, float2* out);

// ---- kernels (tsne_kernels.cu) ----
// Raises per-kernel dynamic shared-memory limits for this session's FFT size.
int configure_kernels(TsneSession* s);
// FFT twiddle table for transforms of length 2^log_m (entries, and the table
// itself computed in double and rounded to float; layout in tsne_kernels.cu).
int fft_twiddle_entries(int log_m);
void fft_twiddle_table(int log_m, float2* out);
// Grid and block size of the fused gradient/update kernel for `rows` rows.
void grad_update_launch_shape(int rows, int* blocks, int* threads);
int launch_stats(TsneSession* s, int center);
int launch_iteration(TsneSession* s, GradMode mode, float exaggeration, float momentum,
                     float learning_rate, float min_gain, float max_step_norm);
int launch_center_output(TsneSession* s, float2* out);

// CPU grid-size policy (tsne_fft_grid_size, src/tsne_neighbors.cpp:392-398);
// in Lagrange mode twice that (up to 1024), so unit boxes fit the layouts'
// extents.
int default_grid_size(int n);
// The interpolation FASTEMBEDR_B200_INTERPOLATION selects: 1 for "lagrange",
// else 0 (bilinear).
int interpolation_from_env();
// Switches a session's interpolation (0 bilinear, 1 Lagrange boxes); drops
// its captured graphs and re-derives the grid geometry of its layout.
int session_set_interpolation(TsneSession* s, int mode);

// ---- PCA start of the PCA-initialised entry points (pca.cu) ----
// values: host, n x p column-major (double or float).  Writes the scaled
// two-component scores, row-major, to d_out (n float2) on stream st.
int pca_start_layout(const void* values, bool values_double, int n, int p, cudaStream_t st, float2* d_out);

// ---- openTSNE transform against a fixed reference layout (landmark.cu) ----
// fastembedr_cuda_landmark_tsne_from_device_knn: device KNN of the queries
// into the reference (column-major n_query x k), host data and layout in R's
// column-major order, host output row-major n_query x 2.
int landmark_tsne(const int* device_indices, const float* device_distances, int index_offset,
                  const float* reference_data, const float* query_data, const float* reference_layout,
                  int n_reference, int n_query, int n_features, int k, float perplexity, int n_iter,
                  int early_exaggeration_iter, float learning_rate, float early_exaggeration, float exaggeration,
                  float initial_momentum, float final_momentum, float max_grad_norm, float max_step_norm,
                  int n_negatives, int exact_repulsion_threshold, unsigned int seed, int affine_neighbors,
                  float affine_ridge, float max_extrapolation, float* out);

}  // namespace fe
