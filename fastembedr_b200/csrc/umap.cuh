// UMAP COO edge-SGD optimizer: parameters and run state.
//
// Layout in HBM: heads int32[E], tails int32[E], periods f32[E] (structure of
// arrays, read once per epoch with streaming loads), layout float2[n]
// (L2-resident: 0.56 MB at n = 70k, 16 MB at n = 2M), delta float2[n] in the
// Jacobi mode.
#pragma once

#include "fe_common.cuh"

namespace fe {

// kUmapInplace: Hogwild at edge granularity (the CPU replay's order within an
// edge); kUmapDelta: Jacobi; kUmapInplaceSample: Hogwild at sample granularity
// (the reference CUDA kernel's).  umap.cu says which entry point uses which.
enum UmapMode { kUmapInplace = 0, kUmapDelta = 1, kUmapInplaceSample = 2 };

struct UmapParams {
  int n;
  int n_epochs;
  int negative_sample_rate;
  int hash_key_is_tail;  // 0: negatives keyed on the edge id (CPU replay), 1: on the tail id
  unsigned int seed;
  float learning_rate;
  float a;
  float b;
  float repulsion_strength;
  // Vertices whose moves this launch applies: [own_begin, own_end).  A shard
  // of a multi-GPU run owns a block of vertices and reads the others from the
  // epoch-start copy every rank holds; unsharded runs own every vertex.
  int own_begin = 0;
  int own_end = 0x7fffffff;
};

// Per-epoch compaction of the edge list to the edges that fire in that epoch
// (umap_compaction_alloc).  A warp then carries 32 firing edges instead of the
// ~9 of 32 consecutive edges that fire on average, so four times as many
// dependent sample chains are in flight per SM; edges keep their order.
struct UmapCompaction {
  int* active = nullptr;       // firing edge ids of the current range, in order
  int* count = nullptr;        // how many
  void* temp = nullptr;        // CUB select scratch
  std::size_t temp_bytes = 0;
};

// Buffers for runs over up to n_edges edges (dev_malloc); compaction stays off
// (all pointers null) when FASTEMBEDR_B200_UMAP_COMPACT=0.
int umap_compaction_alloc(long long n_edges, UmapCompaction* c);
void umap_compaction_free(UmapCompaction* c);

struct UmapRun {
  UmapParams params;
  int mode = kUmapInplace;
  const int* heads = nullptr;
  const int* tails = nullptr;
  const float* periods = nullptr;
  long long n_edges = 0;
  float2* layout = nullptr;
  float2* delta = nullptr;
  long long* positive_count = nullptr;  // optional: positive samples applied
  cudaStream_t stream = nullptr;
  int edge_blocks = 1;
  bool use_graphs = true;
  UmapCompaction compact;  // all null: every epoch scans the whole edge list
  // Sharded runs: after each epoch the owned rows (blocks of rows_per_rank,
  // layout padded to shard_ranks * rows_per_rank rows) are all-gathered.
  void* comm = nullptr;  // ncclComm_t
  int shard_ranks = 1;
  int shard_rank = 0;
  int rows_per_rank = 0;
};

// Gathers per Hogwild epoch in a sharded run (the last one after the epoch's
// sanitize step).
constexpr int kShardGatherParts = 4;

int umap_launch_epoch(UmapRun* r, int epoch);
int umap_run_epochs(UmapRun* r, int epoch_begin, int epoch_end);
int umap_edge_blocks(long long n_edges);
// Per edge: positive and negative samples the epoch kernel applies over
// epochs [epoch_begin, epoch_end).
int umap_count_samples(const float* periods, long long n_edges, int epoch_begin, int epoch_end, int nsr,
                       long long* pos, long long* neg, cudaStream_t stream);

// ---------------------------------------------------------------- graph from KNN

// The fuzzy KNN graph of the device-KNN path as dense rows: row i holds up to
// `width` = min(256, 2k) (neighbour, weight) slots, empty slots are (i, 0).
// Slots 0..out-1 hold row i's own KNN entries in rank order, the rest the
// incoming-only neighbours in ascending order.
struct UmapDenseGraph {
  int n = 0;
  int k = 0;
  int width = 0;
  int* nbr = nullptr;   // device, n * width
  float* w = nullptr;   // device, n * width
  ~UmapDenseGraph();
  UmapDenseGraph() = default;
  UmapDenseGraph(const UmapDenseGraph&) = delete;
  UmapDenseGraph& operator=(const UmapDenseGraph&) = delete;
};

// Row capacity of the reference's device graph, min(256, max(k, 2k))
// (src/embedding_cuda_kernels.cpp:4996).
inline int umap_graph_width(int k) { return 2 * k < 256 ? 2 * k : 256; }

// Builds the graph from column-major device KNN (entry j of row i at j*n+i).
int umap_graph_build(const int* d_idx, const void* d_dist, bool dist_is_double, int n, int k,
                     int index_offset, bool binary, cudaStream_t stream, UmapDenseGraph* g);

// Packs the non-empty slots into COO arrays (device, capacity n * width):
// rank-major (all rows' slot 0, then slot 1, ...) or row-major (grouped by
// head).  epochs_per_sample = 1 / max(w, 1e-6).
int umap_graph_pack(const UmapDenseGraph& g, bool rank_major, int* heads, int* tails, float* weights,
                    float* epochs_per_sample, long long* n_edges, cudaStream_t stream);

// Diffusion start: hashed uniform start, whitened, then `iters` rounds of
// weighted neighbour averaging, each followed by whitening.
int umap_diffusion_init(const UmapDenseGraph& g, unsigned int seed, int iters, float2* layout,
                        cudaStream_t stream);

}  // namespace fe
