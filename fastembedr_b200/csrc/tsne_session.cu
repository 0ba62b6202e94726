// t-SNE session: owns the device state of one optimisation run and drives the
// per-iteration kernel sequence (as CUDA graphs of iteration chunks), the
// periodic spatial reordering, and the caller-order views of its state.
#include "tsne.cuh"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <utility>
#include <vector>

namespace fe {
namespace {

// Random init of the reference CUDA path when no init is passed
// (random_init_kernel, src/embedding_cuda_kernels.cpp:1162-1167).
__global__ void random_layout_kernel(float2* y, int n, unsigned int seed) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n) return;
  y[row] = make_float2(hashed_unit(seed, row, 0), hashed_unit(seed, row, 1));
}

__global__ void fill_float2_kernel(float2* p, int n, float2 v) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

__global__ void iota_kernel(int* p, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = i;
}

int ilog2(int v) {
  int l = 0;
  while ((1 << l) < v) ++l;
  return l;
}

// Copies a caller-order float2 array (host or device) into internal order at dst.
int load_caller_order(TsneSession* s, const float* src, bool host, float2* dst, float2* scratch) {
  const size_t bytes = sizeof(float2) * s->n;
  const cudaMemcpyKind kind = host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
  if (s->identity_perm) {
    FE_CUDA(cudaMemcpyAsync(dst, src, bytes, kind, s->stream), "copy in");
    return 0;
  }
  FE_CUDA(cudaMemcpyAsync(scratch, src, bytes, kind, s->stream), "copy in");
  return launch_permute_in(s, scratch, dst);
}

// Copies an internal-order device array into caller order at dst (host or device).
int store_caller_order(TsneSession* s, const float2* src, bool host, float* dst, float2* scratch) {
  const size_t bytes = sizeof(float2) * s->n;
  const cudaMemcpyKind kind = host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
  if (!s->identity_perm) {
    FE_TRY(launch_unpermute(s, src, scratch));
    src = scratch;
  }
  FE_CUDA(cudaMemcpyAsync(dst, src, bytes, kind, s->stream), "copy out");
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(copy out)");
  return 0;
}

}  // namespace

void drop_graphs(TsneSession* s) {
  for (TsneSession::GraphEntry& e : s->graphs) cudaGraphExecDestroy(e.exec);
  s->graphs.clear();
}

int interpolation_from_env() {
  const char* v = std::getenv("FASTEMBEDR_B200_INTERPOLATION");
  return (v != nullptr && std::strcmp(v, "lagrange") == 0) ? 1 : 0;
}

int default_grid_size(int n) {
  const int fallback = n >= 50000 ? 256 : (n >= 10000 ? 128 : 64);
  const int requested = env_int("FASTEMBEDR_TSNE_FFT_GRID", fallback);
  int grid = 32;
  while (grid < requested && grid < 512) grid <<= 1;
  grid = std::max(32, std::min(512, grid));
  if (interpolation_from_env() == 1 && env_int("FASTEMBEDR_TSNE_FFT_GRID", 0) == 0) {
    grid = std::min(1024, std::max(256, 2 * grid));
  }
  return grid;
}

int session_set_interpolation(TsneSession* s, int mode) {
  if (mode != 0 && mode != 1) {
    set_error("t-SNE interpolation must be 0 (bilinear) or 1 (Lagrange boxes)");
    return 1;
  }
  if (mode == 1 && s->grid < 192) {
    set_error("Lagrange boxes need an FFT grid of at least 256 nodes per side");
    return 1;
  }
  s->interp = mode;
  drop_graphs(s);
  FE_CUDA(cudaMemcpyAsync(&s->stats->lagrange, &s->interp, sizeof(int), cudaMemcpyHostToDevice, s->stream),
          "H2D interpolation");
  // Re-derive the geometry of the current layout in the new mode (uncentred
  // statistics, as after a set_layout; the next splat centres).
  return launch_stats(s, 1);
}

int session_create(TsneSession** out, int n, int grid, int* d_row_ptr, int* d_col, float* d_val,
                   long long nnz, cudaStream_t stream) {
  *out = nullptr;
  if (grid < 4 || (grid & (grid - 1)) != 0 || grid > 1024) {
    set_error("t-SNE FFT grid size must be a power of two in [4, 1024]");
    return 1;
  }
  TsneSession* s = new TsneSession();
  cudaGetDevice(&s->device);
  s->n = n;
  s->grid = grid;
  s->fft = grid * 2;
  s->log_fft = ilog2(s->fft);
  s->nnz = nnz;
  s->row_ptr = d_row_ptr;
  s->col = d_col;
  s->val = d_val;
  s->use_graphs = env_flag("FASTEMBEDR_CUDA_GRAPH_CAPTURE", true);
  s->interp = interpolation_from_env();
  // Opt-in: measured slower than the L2 gathers on the benchmark mixtures
  // (0.80 against 0.60 ms at N = 1M; unions hold each point only 1.2-1.6 times).
  s->stage_enabled = env_flag("FASTEMBEDR_B200_STAGED_ATTRACTION", false);
  // Spatial reordering pays once gathers start missing the caches.
  s->reorder_every = env_int_nonneg("FASTEMBEDR_B200_REORDER_EVERY", n >= 4096 ? 50 : 0);
  if (!env_flag("FASTEMBEDR_B200_REORDER", true)) s->reorder_every = 0;
  s->next_reorder = s->reorder_every;
  s->row_begin = 0;
  s->row_end = n;
  s->rows_per_rank = n;
  if (stream == nullptr) {
    if (check_cuda(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "cudaStreamCreate")) {
      delete s;
      return 1;
    }
    s->own_stream = true;
  } else {
    s->stream = stream;
  }

  // Fused gradient/update kernel: a warp per block of 32 rows, persistent
  // blocks of 8 warps, 8 blocks per SM.
  grad_update_launch_shape(n, &s->update_blocks, &s->update_threads);
  if (configure_kernels(s)) {
    if (s->own_stream) cudaStreamDestroy(s->stream);
    delete s;
    return 1;
  }

  if (reorder_temp_bytes(n, &s->ro_temp_bytes)) {
    if (s->own_stream) cudaStreamDestroy(s->stream);
    delete s;
    return 1;
  }
  const int g = grid;
  const size_t cells = static_cast<size_t>(g) * g;
  const size_t spec = static_cast<size_t>(g) * (g + 1);
  const int stat_blocks = std::max(1024, s->update_blocks);
  Arena& a = s->arena;
  for (int pass = 0; pass < 2; ++pass) {
    if (pass == 0) a.begin_plan();
    else a.rewind();
    const size_t rows = static_cast<size_t>(n) + TsneSession::kPadRows;  // room for shard padding
    s->y[0] = a.take<float2>(rows);
    s->y[1] = a.take<float2>(rows);
    s->update = a.take<float2>(rows);
    s->gains = a.take<float2>(rows);
    s->grad_out = a.take<float2>(rows);
    s->attraction = a.take<float2>(rows);
    s->perm = a.take<int>(n);
    s->rank = a.take<int>(n);
    s->row_ptr4 = a.take<int>(static_cast<size_t>(n) + 1);
    s->stats = a.take<LayoutStats>(1);
    s->update_partials = a.take<double>(6 * static_cast<size_t>(stat_blocks));
    s->z_partials = a.take<double>(g);
    s->charges = a.take<ChargeCell>(cells);
    s->rowspec = a.take<float2>(3 * spec);
    s->krow = a.take<float2>(spec);
    s->colspec = a.take<float2>(4 * spec);
    s->pot = a.take<float4>(cells);
    s->twiddle = a.take<float2>(fft_twiddle_entries(s->log_fft));
    s->ro_keys = a.take<unsigned int>(n);
    s->ro_keys_sorted = a.take<unsigned int>(n);
    s->ro_idx = a.take<int>(n);
    s->ro_order = a.take<int>(n);
    s->ro_perm = a.take<int>(n);
    s->ro_rank = a.take<int>(n);
    s->ro_groups = a.take<int>(static_cast<size_t>(n) + 1);
    s->ro_update = a.take<float2>(n);
    s->ro_gains = a.take<float2>(n);
    s->ro_temp = a.take<char>(s->ro_temp_bytes);
    const size_t groups = static_cast<size_t>(n) / 32 + 2;
    s->group_order = a.take<int>(groups);
    s->group_cost = a.take<unsigned int>(groups);
    s->group_cost_sorted = a.take<unsigned int>(groups);
    s->group_ids = a.take<int>(groups);
    const size_t sblocks = static_cast<size_t>(n) / kStageRows + 2;
    s->stage_meta = a.take<int4>(sblocks);
    s->stage_rounds = a.take<unsigned char>(sblocks * kStageRounds);
    s->stage_cost = a.take<unsigned int>(sblocks);
    s->stage_cost_sorted = a.take<unsigned int>(sblocks);
    s->stage_ids = a.take<int>(sblocks);
    s->stage_order = a.take<int>(sblocks);
    if (pass == 0) {
      if (memory_preflight(a.planned(), "t-SNE workspace preflight") || a.commit("t-SNE workspace")) {
        session_destroy(s);
        return 1;
      }
    }
  }
  std::vector<float2> tw(fft_twiddle_entries(s->log_fft));
  fft_twiddle_table(s->log_fft, tw.data());
  if (check_cuda(cudaMemcpyAsync(s->twiddle, tw.data(), sizeof(float2) * tw.size(), cudaMemcpyHostToDevice,
                                 s->stream), "H2D FFT twiddles") ||
      check_cuda(cudaStreamSynchronize(s->stream), "H2D FFT twiddles") ||
      check_cuda(cudaMemsetAsync(s->stats, 0, sizeof(LayoutStats), s->stream), "memset stats") ||
      check_cuda(cudaMemcpyAsync(&s->stats->lagrange, &s->interp, sizeof(int), cudaMemcpyHostToDevice, s->stream),
                 "H2D interpolation") ||
      check_cuda(cudaMemsetAsync(s->charges, 0, sizeof(ChargeCell) * cells, s->stream), "memset charges") ||
      check_cuda(cudaMemsetAsync(s->update, 0, sizeof(float2) * n, s->stream), "memset update")) {
    session_destroy(s);
    return 1;
  }
  fill_float2_kernel<<<(n + 255) / 256, 256, 0, s->stream>>>(s->gains, n, make_float2(1.0f, 1.0f));
  iota_kernel<<<(n + 255) / 256, 256, 0, s->stream>>>(s->perm, n);
  iota_kernel<<<(n + 255) / 256, 256, 0, s->stream>>>(s->rank, n);
  if (check_cuda(cudaGetLastError(), "session init kernels") ||
      check_cuda(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(session)") ||
      session_reorder(s, false)) {
    session_destroy(s);
    return 1;
  }
  *out = s;
  return 0;
}

void session_destroy(TsneSession* s) {
  if (s == nullptr) return;
  if (s->stream) cudaStreamSynchronize(s->stream);
  const bool trace = env_flag("FASTEMBEDR_B200_TRACE", false);
  const auto t0 = std::chrono::steady_clock::now();
  drop_graphs(s);
  shard_release(s);
  for (cudaEvent_t e : s->events) cudaEventDestroy(e);
  const auto t1 = std::chrono::steady_clock::now();
  if (s->row_ptr) fe::dev_free(s->row_ptr);
  if (s->col) fe::dev_free(s->col);
  if (s->val) fe::dev_free(s->val);
  if (s->csr4_col) fe::dev_free(s->csr4_col);
  if (s->csr4_val) fe::dev_free(s->csr4_val);
  if (s->stage_col16) fe::dev_free(s->stage_col16);
  if (s->stage_union) fe::dev_free(s->stage_union);
  s->arena.release();
  if (s->own_stream && s->stream) cudaStreamDestroy(s->stream);
  if (trace) {
    const auto t2 = std::chrono::steady_clock::now();
    std::fprintf(stderr, "[fastembedr_b200 trace] session destroy: graphs and events %.3f ms, device memory %.3f ms\n",
                 std::chrono::duration<double, std::milli>(t1 - t0).count(),
                 std::chrono::duration<double, std::milli>(t2 - t1).count());
  }
  delete s;
}

int session_set_layout(TsneSession* s, const float* y, bool host, bool center) {
  s->cur = 0;
  FE_TRY(load_caller_order(s, y, host, s->y[0], s->y[1]));
  return launch_stats(s, center ? 1 : 0);
}

int session_random_layout(TsneSession* s, unsigned int seed) {
  s->cur = 0;
  // The hashed init is keyed on the caller's row index.
  random_layout_kernel<<<(s->n + 255) / 256, 256, 0, s->stream>>>(s->y[1], s->n, seed);
  FE_LAUNCH("random_layout_kernel");
  if (s->identity_perm) {
    FE_CUDA(cudaMemcpyAsync(s->y[0], s->y[1], sizeof(float2) * s->n, cudaMemcpyDeviceToDevice, s->stream),
            "copy init");
  } else {
    FE_TRY(launch_permute_in(s, s->y[1], s->y[0]));
  }
  return launch_stats(s, 1);
}

int session_set_state(TsneSession* s, const float* update, const float* gains, bool host) {
  FE_TRY(load_caller_order(s, update, host, s->update, s->grad_out));
  FE_TRY(load_caller_order(s, gains, host, s->gains, s->grad_out));
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(set state)");
  return 0;
}

int session_get_state(TsneSession* s, float* update, float* gains, bool host) {
  if (s->sharded) {
    FE_TRY(shard_gather_rows(s, s->update));
    FE_TRY(shard_gather_rows(s, s->gains));
  }
  FE_TRY(store_caller_order(s, s->update, host, update, s->grad_out));
  FE_TRY(store_caller_order(s, s->gains, host, gains, s->grad_out));
  return 0;
}

int session_reset_state(TsneSession* s) {
  FE_CUDA(cudaMemsetAsync(s->update, 0, sizeof(float2) * s->n, s->stream), "memset update");
  fill_float2_kernel<<<(s->n + 255) / 256, 256, 0, s->stream>>>(s->gains, s->n, make_float2(1.0f, 1.0f));
  FE_LAUNCH("fill gains");
  return 0;
}

namespace {

int collect_profile(TsneSession* s) {
  if (!s->profile || s->events.empty()) return 0;
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(profile)");
  for (size_t i = 0; i + 1 < s->events.size(); i += 2) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, s->events[i], s->events[i + 1]);
    const int kind = s->event_kind[i / 2];
    s->kernel_ms[kind] += ms;
    s->kernel_launches[kind] += 1;
  }
  for (cudaEvent_t e : s->events) cudaEventDestroy(e);
  s->events.clear();
  s->event_kind.clear();
  return 0;
}

constexpr int kLongChunk = 24;

// The captured chunk of `iters` iterations for this parameter set starting at
// the current buffer parity; captured on first use.  Capturing only records
// launches, so it can overlap device work already queued on the stream.
cudaGraphExec_t chunk_graph(TsneSession* s, int iters, const float key[5]) {
  for (TsneSession::GraphEntry& e : s->graphs) {
    if (e.iters == iters && e.cur == s->cur && std::memcmp(key, e.params, sizeof(e.params)) == 0) {
      e.used = ++s->graph_clock;
      return e.exec;
    }
  }
  constexpr size_t kMaxGraphs = 8;
  if (s->graphs.size() >= kMaxGraphs) {
    auto lru = std::min_element(s->graphs.begin(), s->graphs.end(),
                                [](const TsneSession::GraphEntry& a, const TsneSession::GraphEntry& b) {
                                  return a.used < b.used;
                                });
    cudaGraphExecDestroy(lru->exec);
    s->graphs.erase(lru);
  }
  const int saved_cur = s->cur;
  cudaGraph_t g = nullptr;
  if (check_cuda(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture")) {
    return nullptr;
  }
  int rc = 0;
  for (int it = 0; it < iters && rc == 0; ++it) {
    rc = launch_iteration(s, kGradUpdate, key[0], key[1], key[2], key[3], key[4]);
  }
  const cudaError_t end = cudaStreamEndCapture(s->stream, &g);
  s->cur = saved_cur;
  if (rc != 0 || end != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    if (rc == 0) check_cuda(end, "cudaStreamEndCapture");
    return nullptr;
  }
  TsneSession::GraphEntry e{};
  const cudaError_t inst = cudaGraphInstantiate(&e.exec, g, 0);
  cudaGraphDestroy(g);
  if (check_cuda(inst, "cudaGraphInstantiate")) return nullptr;
  // Upload now (at prepare time when called from session_prepare) rather
  // than on the first launch.
  if (check_cuda(cudaGraphUpload(e.exec, s->stream), "cudaGraphUpload")) {
    cudaGraphExecDestroy(e.exec);
    return nullptr;
  }
  e.iters = iters;
  e.cur = saved_cur;
  std::memcpy(e.params, key, sizeof(e.params));
  e.used = ++s->graph_clock;
  s->graphs.push_back(e);
  return e.exec;
}

// Runs `iters` iterations with one parameter set and no reorder in between.
int iterate_block(TsneSession* s, int iters, float exaggeration, float momentum, float learning_rate,
                  float min_gain, float max_step_norm) {
  if (iters <= 0) return 0;
  // Grouped (single-process multi-device) sessions launch without graphs: a
  // graph would queue many collectives at once (see rank_group.h).
  const bool graphs = s->use_graphs && !s->profile && iters > 1 && s->group == nullptr;
  if (!graphs) {
    for (int it = 0; it < iters; ++it) {
      FE_TRY(launch_iteration(s, kGradUpdate, exaggeration, momentum, learning_rate, min_gain,
                              max_step_norm));
      if (s->profile && s->events.size() > 4000) FE_TRY(collect_profile(s));
    }
    return collect_profile(s);
  }
  // Captured chunks of 24 iterations (the reference captures chunks of 25,
  // src/embedding_cuda_kernels.cpp:5902-5985) and of 2 for the rest.  Only
  // these two lengths exist, so a parameter set needs at most two captures
  // however the reorders cut the iterations, and both can be made ahead of
  // time (session_prepare).  Even lengths return the layout double buffer to
  // the parity a chunk started from.
  const float key[5] = {exaggeration, momentum, learning_rate, min_gain, max_step_norm};
  int done = 0;
  while (iters - done >= 2) {
    const int chunk = iters - done >= kLongChunk ? kLongChunk : 2;
    cudaGraphExec_t exec = chunk_graph(s, chunk, key);
    if (exec == nullptr) return 1;
    FE_CUDA(cudaGraphLaunch(exec, s->stream), "cudaGraphLaunch(t-SNE chunk)");
    done += chunk;
  }
  for (; done < iters; ++done) {
    FE_TRY(launch_iteration(s, kGradUpdate, exaggeration, momentum, learning_rate, min_gain, max_step_norm));
  }
  return 0;
}

}  // namespace

int session_iterate(TsneSession* s, int iters, float exaggeration, float momentum,
                    float learning_rate, float min_gain, float max_step_norm) {
  while (iters > 0) {
    if (s->reorder_every > 0 && s->iterations_run >= s->next_reorder) {
      FE_TRY(session_reorder(s, true));
      s->next_reorder = s->iterations_run + s->reorder_every;
    }
    long long block = iters;
    if (s->reorder_every > 0) block = std::min<long long>(block, s->next_reorder - s->iterations_run);
    FE_TRY(iterate_block(s, static_cast<int>(block), exaggeration, momentum, learning_rate, min_gain,
                         max_step_norm));
    s->iterations_run += block;
    iters -= static_cast<int>(block);
  }
  return 0;
}

int session_prepare(TsneSession* s, float exaggeration, float momentum, float learning_rate, float min_gain,
                    float max_step_norm) {
  if (!s->use_graphs) return 0;
  const float key[5] = {exaggeration, momentum, learning_rate, min_gain, max_step_norm};
  for (int chunk : {kLongChunk, 2}) {
    if (chunk_graph(s, chunk, key) == nullptr) return 1;
  }
  return 0;
}

int session_gradient(TsneSession* s, float exaggeration, float* grad_host, double* z_out) {
  // Evaluated at the stored layout exactly as given (no re-centring).
  FE_TRY(launch_stats(s, 0));
  FE_TRY(launch_iteration(s, kGradOnly, exaggeration, 0.f, 0.f, 0.f, 0.f));
  if (s->sharded) FE_TRY(shard_gather_rows(s, s->grad_out));
  LayoutStats st;
  FE_CUDA(cudaMemcpyAsync(&st, s->stats, sizeof(st), cudaMemcpyDeviceToHost, s->stream), "D2H stats");
  FE_TRY(store_caller_order(s, s->grad_out, true, grad_host, s->y[s->cur ^ 1]));
  if (z_out) *z_out = st.z;
  return launch_stats(s, 1);
}

int session_get_layout(TsneSession* s, float* out, bool host) {
  // The newest layout is uncentred until the next splat: centre into grad_out.
  FE_TRY(launch_center_output(s, s->grad_out));
  return store_caller_order(s, s->grad_out, host, out, s->y[s->cur ^ 1]);
}

int session_get_p(TsneSession* s, int* row_ptr, int* col, float* val) {
  // The caller-order CSR is kept as is; copy it out.
  const size_t nnz = static_cast<size_t>(s->nnz);
  FE_CUDA(cudaMemcpyAsync(row_ptr, s->row_ptr, sizeof(int) * (s->n + 1), cudaMemcpyDeviceToHost, s->stream), "D2H");
  FE_CUDA(cudaMemcpyAsync(col, s->col, sizeof(int) * nnz, cudaMemcpyDeviceToHost, s->stream), "D2H");
  FE_CUDA(cudaMemcpyAsync(val, s->val, sizeof(float) * nnz, cudaMemcpyDeviceToHost, s->stream), "D2H");
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(get_p)");
  return 0;
}

}  // namespace fe
