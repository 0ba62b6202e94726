// UMAP sessions: the device-KNN UMAP path of the reference
// (fastembedr_cuda_umap_from_device_knn_spectral_impl,
// src/embedding_cuda_kernels.cpp:4967-5199) split into its set-up -- fuzzy
// graph, diffusion start, rank-major COO edge list, all kept on the device --
// and epoch ranges run on demand.  The one-shot entry points in capi.cu run
// the same steps in one call; a session lets a caller time the epochs alone,
// read the layout between epoch ranges, and count the edge samples applied.
// Hidden visibility is the build default; the header's declarations export.
#pragma GCC visibility push(default)
#include "fastembedr_b200.h"
#pragma GCC visibility pop

#include "nccl_loader.cuh"
#include "umap.cuh"

#include <cub/cub.cuh>

#include <algorithm>
#include <cstring>
#include <string>

struct fe_b200_umap {
  int n = 0;
  int k = 0;
  long long n_edges = 0;
  cudaStream_t stream = nullptr;
  fe::Arena arena;
  int* heads = nullptr;
  int* tails = nullptr;
  float* periods = nullptr;
  float2* layout = nullptr;
  float2* delta = nullptr;
  long long* counts = nullptr;  // [0] positive, [1] negative totals, then per-edge counts
  void* temp = nullptr;         // CUB reduction storage
  size_t temp_bytes = 0;
  // Sharded sessions (fe_b200_umap_shard): this rank's vertex block, the
  // edges that touch it, the layout padded for the in-place all-gather.
  void* comm = nullptr;  // ncclComm_t
  bool own_comm = false;  // destroyed with the session (not when lent by the caller)
  int shard_ranks = 1;
  int shard_rank = 0;
  int rows_per_rank = 0;
  int own_begin = 0;
  int own_end = 0x7fffffff;
  long long own_edges = 0;
  void* shard_mem = nullptr;  // own heads, tails, periods and the padded layout
  int* own_heads = nullptr;
  int* own_tails = nullptr;
  float* own_periods = nullptr;
  // Firing-edge lists of the epochs (made at the first run, for every edge).
  fe::UmapCompaction compact;
  bool compact_tried = false;
  ~fe_b200_umap() {
    if (stream) cudaStreamSynchronize(stream);
    fe::umap_compaction_free(&compact);
    if (comm && own_comm) {
      const fe::NcclApi* api = fe::nccl_api();
      if (api) api->CommDestroy(static_cast<ncclComm_t>(comm));
    }
    if (shard_mem) fe::dev_free(shard_mem);
    arena.release();
    if (stream) cudaStreamDestroy(stream);
  }
};

namespace {

using fe::set_error;

int check_session(const fe_b200_umap* s) {
  if (s == nullptr) {
    set_error("invalid UMAP session");
    return 1;
  }
  return 0;
}

__global__ void touches_kernel(const int* __restrict__ heads, const int* __restrict__ tails, long long n_edges,
                               int own_begin, int own_end, char* __restrict__ flags) {
  const long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= n_edges) return;
  const int h = heads[e], t = tails[e];
  flags[e] = static_cast<char>((h >= own_begin && h < own_end) || (t >= own_begin && t < own_end));
}

}  // namespace

extern "C" {

int fe_b200_umap_create(const int* indices, const float* distances, int n, int k, int index_offset,
                        int inputs_on_device, int binary_graph, int spectral_n_iter, unsigned int seed,
                        fe_b200_umap** out) {
  fe::clear_error();
  if (out == nullptr || indices == nullptr || distances == nullptr) {
    set_error("null pointer");
    return 1;
  }
  *out = nullptr;
  if (n < 2 || k < 1 || k > 256 || spectral_n_iter < 1) {
    set_error("invalid UMAP session dimensions or parameters");
    return 1;
  }
  fe_b200_umap* s = new fe_b200_umap();
  struct Guard {
    fe_b200_umap* s;
    ~Guard() { delete s; }
  } guard{s};
  s->n = n;
  s->k = k;
  FE_CUDA(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "cudaStreamCreate(umap session)");
  fe::UmapDenseGraph g;
  {
    void* d_idx = nullptr;
    void* d_dist = nullptr;
    struct Free {
      void** p;
      ~Free() {
        if (*p) fe::dev_free(*p);
      }
    } fi{&d_idx}, fd{&d_dist};
    const int* idx_dev = indices;
    const float* dist_dev = distances;
    if (!inputs_on_device) {
      const size_t items = static_cast<size_t>(n) * k;
      FE_CUDA(fe::dev_malloc(&d_idx, items * sizeof(int)), "cudaMalloc(UMAP indices)");
      FE_CUDA(fe::dev_malloc(&d_dist, items * sizeof(float)), "cudaMalloc(UMAP distances)");
      FE_TRY(fe::h2d_copy(d_idx, indices, items * sizeof(int), s->stream, "H2D UMAP indices"));
      FE_TRY(fe::h2d_copy(d_dist, distances, items * sizeof(float), s->stream, "H2D UMAP distances"));
      idx_dev = static_cast<const int*>(d_idx);
      dist_dev = static_cast<const float*>(d_dist);
    }
    FE_TRY(fe::umap_graph_build(idx_dev, dist_dev, false, n, k, index_offset, binary_graph != 0, s->stream, &g));
    FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(umap graph)");
  }
  const size_t slots = static_cast<size_t>(n) * g.width;
  size_t reduce_bytes = 0;
  FE_CUDA(cub::DeviceReduce::Sum(nullptr, reduce_bytes, static_cast<long long*>(nullptr),
                                 static_cast<long long*>(nullptr), static_cast<int>(slots)),
          "cub::DeviceReduce(sizing)");
  fe::Arena& a = s->arena;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 0) a.begin_plan();
    else a.rewind();
    s->heads = a.take<int>(slots);
    s->tails = a.take<int>(slots);
    s->periods = a.take<float>(slots);
    s->layout = a.take<float2>(n);
    s->delta = a.take<float2>(n);
    s->counts = a.take<long long>(2 * slots + 2);
    s->temp = a.take<char>(reduce_bytes);
    if (pass == 0) {
      FE_TRY(fe::memory_preflight(a.planned(), "UMAP session preflight"));
      FE_TRY(a.commit("UMAP session"));
    }
  }
  s->temp_bytes = reduce_bytes;
  FE_TRY(fe::umap_diffusion_init(g, seed, spectral_n_iter, s->layout, s->stream));
  FE_TRY(fe::umap_graph_pack(g, true, s->heads, s->tails, nullptr, s->periods, &s->n_edges, s->stream));
  if (s->n_edges < 1 || s->n_edges > static_cast<long long>(slots)) {
    set_error("invalid UMAP graph edge count");
    return 1;
  }
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(umap session)");
  guard.s = nullptr;
  *out = s;
  return 0;
}

int fe_b200_umap_run(fe_b200_umap* s, int epoch_begin, int epoch_end, int n_epochs, int negative_sample_rate,
                     float learning_rate, float a, float b, float repulsion_strength, unsigned int seed,
                     int optimizer_mode) {
  fe::clear_error();
  FE_TRY(check_session(s));
  if (epoch_begin < 0 || epoch_end < epoch_begin || epoch_end > n_epochs || negative_sample_rate < 0 ||
      !(learning_rate > 0.0f)) {
    set_error("invalid UMAP epoch range or parameters");
    return 1;
  }
  fe::UmapRun r;
  // Negatives keyed on the tail vertex, as the reference's COO kernels key
  // them (and as a shard needs: the edge's position differs between shards).
  r.params = fe::UmapParams{s->n, n_epochs, negative_sample_rate, 1, seed, learning_rate, a, b, repulsion_strength};
  r.mode = optimizer_mode == 1 ? fe::kUmapDelta : fe::kUmapInplaceSample;
  const bool sharded = s->comm != nullptr;
  r.heads = sharded ? s->own_heads : s->heads;
  r.tails = sharded ? s->own_tails : s->tails;
  r.periods = sharded ? s->own_periods : s->periods;
  r.n_edges = sharded ? s->own_edges : s->n_edges;
  r.params.own_begin = s->own_begin;
  r.params.own_end = s->own_end;
  r.comm = s->comm;
  r.shard_ranks = s->shard_ranks;
  r.shard_rank = s->shard_rank;
  r.rows_per_rank = s->rows_per_rank;
  r.layout = s->layout;
  r.delta = r.mode == fe::kUmapDelta ? s->delta : nullptr;
  r.stream = s->stream;
  r.edge_blocks = fe::umap_edge_blocks(std::max(1ll, r.n_edges));
  r.use_graphs = fe::env_flag("FASTEMBEDR_CUDA_GRAPH_CAPTURE", true);
  if (!s->compact_tried) {
    s->compact_tried = true;
    FE_TRY(fe::umap_compaction_alloc(s->n_edges, &s->compact));
  }
  r.compact = s->compact;
  return fe::umap_run_epochs(&r, epoch_begin, epoch_end);
}

}  // extern "C"

namespace {

// Shards the session on `lent` (kept by the caller) or, when null, on a new
// communicator joined with `id` (destroyed with the session).
int umap_shard_impl(fe_b200_umap* s, const unsigned char* id, ncclComm_t lent, int nranks, int rank) {
  if (s->comm != nullptr) {
    set_error("UMAP session is already sharded");
    return 1;
  }
  if (nranks < 1 || nranks > 256 || rank < 0 || rank >= nranks) {
    set_error("UMAP shard: need 1 <= nranks <= 256 and 0 <= rank < nranks");
    return 1;
  }
  const int n = s->n;
  const int per = (n + nranks - 1) / nranks;
  const size_t padded_rows = static_cast<size_t>(per) * nranks;
  const size_t e = static_cast<size_t>(s->n_edges);
  // This rank's edges: those with an endpoint in its block (edges across
  // blocks are kept by both ranks; each applies the moves of its own end).
  size_t select_bytes = 0;
  FE_CUDA(cub::DeviceSelect::Flagged(nullptr, select_bytes, static_cast<const int*>(nullptr),
                                     static_cast<const char*>(nullptr), static_cast<int*>(nullptr),
                                     static_cast<long long*>(nullptr), static_cast<int>(e)),
          "cub::DeviceSelect(sizing)");
  fe::Arena plan;
  plan.begin_plan();
  plan.take<int>(e);
  plan.take<int>(e);
  plan.take<float>(e);
  plan.take<float2>(padded_rows);
  plan.take<char>(e);
  plan.take<long long>(1);
  plan.take<char>(select_bytes);
  FE_TRY(fe::memory_preflight(plan.planned(), "UMAP shard preflight"));
  char* mem = nullptr;
  FE_CUDA(fe::dev_malloc(&mem, plan.planned()), "cudaMalloc(UMAP shard)");
  struct Free {
    char** p;
    ~Free() {
      if (*p) fe::dev_free(*p);
    }
  } release{&mem};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    char* q = mem + off;
    off += fe::align_up(bytes);
    return q;
  };
  int* own_heads = reinterpret_cast<int*>(take(e * sizeof(int)));
  int* own_tails = reinterpret_cast<int*>(take(e * sizeof(int)));
  float* own_periods = reinterpret_cast<float*>(take(e * sizeof(float)));
  float2* layout = reinterpret_cast<float2*>(take(padded_rows * sizeof(float2)));
  char* flags = take(e);
  long long* selected = reinterpret_cast<long long*>(take(sizeof(long long)));
  void* select_temp = take(select_bytes);
  const int own_begin = std::min(n, rank * per);
  const int own_end = std::min(n, own_begin + per);
  touches_kernel<<<static_cast<unsigned>((e + 255) / 256), 256, 0, s->stream>>>(s->heads, s->tails, s->n_edges,
                                                                               own_begin, own_end, flags);
  FE_LAUNCH("touches_kernel");
  size_t tb = select_bytes;
  FE_CUDA(cub::DeviceSelect::Flagged(select_temp, tb, s->heads, flags, own_heads, selected, static_cast<int>(e),
                                     s->stream), "cub::DeviceSelect(heads)");
  tb = select_bytes;
  FE_CUDA(cub::DeviceSelect::Flagged(select_temp, tb, s->tails, flags, own_tails, selected, static_cast<int>(e),
                                     s->stream), "cub::DeviceSelect(tails)");
  tb = select_bytes;
  FE_CUDA(cub::DeviceSelect::Flagged(select_temp, tb, s->periods, flags, own_periods, selected,
                                     static_cast<int>(e), s->stream), "cub::DeviceSelect(periods)");
  FE_CUDA(cudaMemsetAsync(layout, 0, padded_rows * sizeof(float2), s->stream), "memset layout");
  FE_CUDA(cudaMemcpyAsync(layout, s->layout, sizeof(float2) * n, cudaMemcpyDeviceToDevice, s->stream),
          "copy layout");
  long long own_edges = 0;
  FE_CUDA(cudaMemcpyAsync(&own_edges, selected, sizeof(long long), cudaMemcpyDeviceToHost, s->stream), "D2H");
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(UMAP shard)");
  ncclComm_t comm = lent;
  if (comm == nullptr) FE_TRY(fe::comm_init(id, nranks, rank, &comm));
  s->comm = comm;
  s->own_comm = lent == nullptr;
  s->shard_ranks = nranks;
  s->shard_rank = rank;
  s->rows_per_rank = per;
  s->own_begin = own_begin;
  s->own_end = own_end;
  s->own_edges = own_edges;
  s->own_heads = own_heads;
  s->own_tails = own_tails;
  s->own_periods = own_periods;
  s->layout = layout;  // the arena's copy stays allocated, unused
  s->shard_mem = mem;
  mem = nullptr;
  return 0;
}

}  // namespace

extern "C" {

int fe_b200_umap_shard(fe_b200_umap* s, const unsigned char* id, int id_bytes, int nranks, int rank) {
  fe::clear_error();
  FE_TRY(check_session(s));
  if (id == nullptr || id_bytes < static_cast<int>(sizeof(ncclUniqueId))) {
    set_error("invalid UMAP shard call");
    return 1;
  }
  return umap_shard_impl(s, id, nullptr, nranks, rank);
}

int fe_b200_umap_shard_comm(fe_b200_umap* s, fe_b200_comm* comm) {
  fe::clear_error();
  FE_TRY(check_session(s));
  if (comm == nullptr || comm->comm == nullptr) {
    set_error("invalid UMAP shard call");
    return 1;
  }
  return umap_shard_impl(s, nullptr, comm->comm, comm->nranks, comm->rank);
}

int fe_b200_umap_count_samples(fe_b200_umap* s, int epoch_begin, int epoch_end, int negative_sample_rate,
                               long long* positive, long long* negative) {
  fe::clear_error();
  FE_TRY(check_session(s));
  if (epoch_begin < 0 || epoch_end < epoch_begin) {
    set_error("invalid UMAP epoch range");
    return 1;
  }
  long long* per_edge_pos = s->counts + 2;
  long long* per_edge_neg = per_edge_pos + s->n_edges;
  FE_TRY(fe::umap_count_samples(s->periods, s->n_edges, epoch_begin, epoch_end, negative_sample_rate,
                                per_edge_pos, per_edge_neg, s->stream));
  size_t tb = s->temp_bytes;
  FE_CUDA(cub::DeviceReduce::Sum(s->temp, tb, per_edge_pos, s->counts, static_cast<int>(s->n_edges), s->stream),
          "cub::DeviceReduce(positive)");
  tb = s->temp_bytes;
  FE_CUDA(cub::DeviceReduce::Sum(s->temp, tb, per_edge_neg, s->counts + 1, static_cast<int>(s->n_edges),
                                 s->stream),
          "cub::DeviceReduce(negative)");
  long long host[2] = {0, 0};
  FE_CUDA(cudaMemcpyAsync(host, s->counts, sizeof(host), cudaMemcpyDeviceToHost, s->stream), "D2H counts");
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(count)");
  if (positive) *positive = host[0];
  if (negative) *negative = host[1];
  return 0;
}

int fe_b200_umap_get_layout(fe_b200_umap* s, float* out, int on_device) {
  fe::clear_error();
  FE_TRY(check_session(s));
  if (out == nullptr) {
    set_error("null pointer");
    return 1;
  }
  FE_CUDA(cudaMemcpyAsync(out, s->layout, sizeof(float2) * s->n,
                          on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost, s->stream),
          "copy UMAP layout");
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(layout)");
  return 0;
}

int fe_b200_umap_set_layout(fe_b200_umap* s, const float* y, int on_device) {
  fe::clear_error();
  FE_TRY(check_session(s));
  if (y == nullptr) {
    set_error("null pointer");
    return 1;
  }
  FE_CUDA(cudaMemcpyAsync(s->layout, y, sizeof(float2) * s->n,
                          on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s->stream),
          "copy UMAP layout");
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(layout)");
  return 0;
}

int fe_b200_umap_info(fe_b200_umap* s, int* n, long long* n_edges) {
  FE_TRY(check_session(s));
  if (n) *n = s->n;
  if (n_edges) *n_edges = s->n_edges;
  return 0;
}

int fe_b200_umap_get_graph(fe_b200_umap* s, int* heads, int* tails, float* epochs_per_sample) {
  fe::clear_error();
  FE_TRY(check_session(s));
  const size_t e = static_cast<size_t>(s->n_edges);
  if (heads) FE_CUDA(cudaMemcpyAsync(heads, s->heads, e * sizeof(int), cudaMemcpyDeviceToHost, s->stream), "D2H");
  if (tails) FE_CUDA(cudaMemcpyAsync(tails, s->tails, e * sizeof(int), cudaMemcpyDeviceToHost, s->stream), "D2H");
  if (epochs_per_sample) {
    FE_CUDA(cudaMemcpyAsync(epochs_per_sample, s->periods, e * sizeof(float), cudaMemcpyDeviceToHost, s->stream),
            "D2H");
  }
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(graph)");
  return 0;
}

void* fe_b200_umap_stream(fe_b200_umap* s) { return s == nullptr ? nullptr : s->stream; }

void fe_b200_umap_destroy(fe_b200_umap* s) { delete s; }

}  // extern "C"
