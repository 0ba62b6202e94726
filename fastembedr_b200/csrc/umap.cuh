// UMAP COO edge-SGD optimizer: parameters and run state.
//
// Layout in HBM: heads int32[E], tails int32[E], periods f32[E] (structure of
// arrays, read once per epoch with streaming loads), layout float2[n]
// (L2-resident: 0.56 MB at n = 70k, 16 MB at n = 2M), delta float2[n] in the
// Jacobi mode.
#pragma once

#include "fe_common.cuh"

namespace fe {

enum UmapMode { kUmapInplace = 0, kUmapDelta = 1 };

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
};

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
};

int umap_launch_epoch(UmapRun* r, int epoch);
int umap_run_epochs(UmapRun* r, int epoch_begin, int epoch_end);
int umap_edge_blocks(long long n_edges);

}  // namespace fe
