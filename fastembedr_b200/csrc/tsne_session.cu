// t-SNE session: owns the device state of one optimisation run and drives the
// per-iteration kernel sequence (optionally as a CUDA graph per phase chunk).
#include "tsne.cuh"

#include <cmath>
#include <cstring>
#include <vector>

namespace fe {
namespace {

// Random init of the reference CUDA path when no init is passed
// (random_init_kernel + deterministic_unit, src/embedding_cuda_kernels.cpp:266-274, 1162-1167).
__device__ __forceinline__ unsigned int mix_unit(unsigned int x) {
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return x;
}

__global__ void random_layout_kernel(float2* y, int n, unsigned int seed) {
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n) return;
  float v[2];
  for (unsigned int col = 0; col < 2; ++col) {
    unsigned int x = seed;
    x ^= (static_cast<unsigned int>(row) + 1u) * 0x9e3779b9u;
    x ^= (col + 1u) * 0x85ebca6bu;
    const unsigned int bits = mix_unit(x);
    v[col] = static_cast<float>(bits & 0x00ffffffu) / 8388607.5f - 1.0f;
  }
  y[row] = make_float2(v[0], v[1]);
}

__global__ void fill_float2_kernel(float2* p, int n, float2 v) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

int ilog2(int v) {
  int l = 0;
  while ((1 << l) < v) ++l;
  return l;
}

}  // namespace

int default_grid_size(int n) {
  const int fallback = n >= 50000 ? 256 : (n >= 10000 ? 128 : 64);
  const int requested = env_int("FASTEMBEDR_TSNE_FFT_GRID", fallback);
  int grid = 32;
  while (grid < requested && grid < 512) grid <<= 1;
  return std::max(32, std::min(512, grid));
}

int session_create(TsneSession** out, int n, int grid, int* d_row_ptr, int* d_col, float* d_val,
                   long long nnz, long long nnz_pad, cudaStream_t stream) {
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
  s->nnz_pad = nnz_pad;
  s->row_ptr = d_row_ptr;
  s->col = d_col;
  s->val = d_val;
  s->use_graphs = env_flag("FASTEMBEDR_CUDA_GRAPH_CAPTURE", true);
  if (stream == nullptr) {
    if (check_cuda(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "cudaStreamCreate")) {
      delete s;
      return 1;
    }
    s->own_stream = true;
  } else {
    s->stream = stream;
  }

  // Launch shape of the fused gradient/update kernel: persistent blocks sized
  // to the measured occupancy on this device.
  s->update_threads = 256;
  s->update_blocks = sm_count() * 8;  // 2048 resident threads per SM
  s->update_blocks = std::max(1, std::min(s->update_blocks, (n + 255) / 256));
  const int m = s->fft;
  s->cols_per_block = std::max(1, std::min(16, 2048 / m));
  if (configure_kernels(s)) {
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
    s->y[0] = a.take<float2>(n);
    s->y[1] = a.take<float2>(n);
    s->update = a.take<float2>(n);
    s->gains = a.take<float2>(n);
    s->grad_out = a.take<float2>(n);
    s->stats = a.take<LayoutStats>(1);
    s->update_partials = a.take<double>(6 * static_cast<size_t>(stat_blocks));
    s->z_partials = a.take<double>(g);
    s->charges = a.take<float4>(cells);
    s->rowspec = a.take<float2>(3 * spec);
    s->krow = a.take<float2>(spec);
    s->colspec = a.take<float2>(4 * spec);
    s->pot = a.take<float4>(cells);
    s->twiddle = a.take<float2>(m / 2);
    if (pass == 0) {
      if (memory_preflight(a.planned(), "t-SNE workspace preflight") || a.commit("t-SNE workspace")) {
        session_destroy(s);
        return 1;
      }
    }
  }
  std::vector<float2> tw(m / 2);
  for (int k = 0; k < m / 2; ++k) {
    const double ang = -2.0 * M_PI * static_cast<double>(k) / static_cast<double>(m);
    tw[k] = make_float2(static_cast<float>(std::cos(ang)), static_cast<float>(std::sin(ang)));
  }
  if (check_cuda(cudaMemcpyAsync(s->twiddle, tw.data(), sizeof(float2) * tw.size(),
                                 cudaMemcpyHostToDevice, s->stream), "H2D twiddles") ||
      check_cuda(cudaMemsetAsync(s->stats, 0, sizeof(LayoutStats), s->stream), "memset stats") ||
      check_cuda(cudaMemsetAsync(s->charges, 0, sizeof(float4) * cells, s->stream), "memset charges") ||
      check_cuda(cudaMemsetAsync(s->update, 0, sizeof(float2) * n, s->stream), "memset update") ||
      check_cuda(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(session)")) {
    session_destroy(s);
    return 1;
  }
  fill_float2_kernel<<<(n + 255) / 256, 256, 0, s->stream>>>(s->gains, n, make_float2(1.0f, 1.0f));
  if (check_cuda(cudaGetLastError(), "fill gains")) {
    session_destroy(s);
    return 1;
  }
  *out = s;
  return 0;
}

void session_destroy(TsneSession* s) {
  if (s == nullptr) return;
  if (s->stream) cudaStreamSynchronize(s->stream);
  if (s->graph) cudaGraphExecDestroy(s->graph);
  for (cudaEvent_t e : s->events) cudaEventDestroy(e);
  if (s->row_ptr) cudaFree(s->row_ptr);
  if (s->col) cudaFree(s->col);
  if (s->val) cudaFree(s->val);
  s->arena.release();
  if (s->own_stream && s->stream) cudaStreamDestroy(s->stream);
  delete s;
}

int session_set_layout(TsneSession* s, const float* y, bool host, bool center) {
  s->cur = 0;
  FE_CUDA(cudaMemcpyAsync(s->y[0], y, sizeof(float2) * s->n,
                          host ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice, s->stream),
          "copy layout");
  return launch_stats(s, center ? 1 : 0);
}

int session_random_layout(TsneSession* s, unsigned int seed) {
  s->cur = 0;
  random_layout_kernel<<<(s->n + 255) / 256, 256, 0, s->stream>>>(s->y[0], s->n, seed);
  FE_LAUNCH("random_layout_kernel");
  return launch_stats(s, 1);
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

}  // namespace

int session_iterate(TsneSession* s, int iters, float exaggeration, float momentum,
                    float learning_rate, float min_gain, float max_step_norm) {
  if (iters <= 0) return 0;
  const bool graphs = s->use_graphs && !s->profile && iters > 1;
  if (!graphs) {
    for (int it = 0; it < iters; ++it) {
      FE_TRY(launch_iteration(s, kGradUpdate, exaggeration, momentum, learning_rate, min_gain,
                              max_step_norm));
      s->iterations_run += 1;
      if (s->profile && s->events.size() > 4000) FE_TRY(collect_profile(s));
    }
    return collect_profile(s);
  }
  // One captured chunk of up to 25 iterations per parameter set (the chunk
  // length the reference uses, src/embedding_cuda_kernels.cpp:5902-5985).
  // Capturing an even number of iterations keeps the y double-buffer parity.
  const int chunk = std::min(iters, 24);
  const float key[5] = {exaggeration, momentum, learning_rate, min_gain, max_step_norm};
  const bool reuse = s->graph != nullptr && s->graph_iters == chunk && s->graph_cur == s->cur &&
                     std::memcmp(key, s->graph_params, sizeof(key)) == 0 && (chunk % 2 == 0);
  if (!reuse && chunk % 2 == 0) {
    if (s->graph) {
      cudaGraphExecDestroy(s->graph);
      s->graph = nullptr;
    }
    const int saved_cur = s->cur;
    cudaGraph_t g = nullptr;
    FE_CUDA(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
    int rc = 0;
    for (int it = 0; it < chunk && rc == 0; ++it) {
      rc = launch_iteration(s, kGradUpdate, exaggeration, momentum, learning_rate, min_gain, max_step_norm);
    }
    const cudaError_t end = cudaStreamEndCapture(s->stream, &g);
    s->cur = saved_cur;
    if (rc != 0 || end != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      if (rc == 0) check_cuda(end, "cudaStreamEndCapture");
      return 1;
    }
    const cudaError_t inst = cudaGraphInstantiate(&s->graph, g, 0);
    cudaGraphDestroy(g);
    FE_CUDA(inst, "cudaGraphInstantiate");
    s->graph_iters = chunk;
    s->graph_cur = saved_cur;
    std::memcpy(s->graph_params, key, sizeof(key));
  }
  int done = 0;
  if (chunk % 2 == 0) {
    while (iters - done >= chunk) {
      FE_CUDA(cudaGraphLaunch(s->graph, s->stream), "cudaGraphLaunch(t-SNE chunk)");
      done += chunk;
    }
  }
  for (; done < iters; ++done) {
    FE_TRY(launch_iteration(s, kGradUpdate, exaggeration, momentum, learning_rate, min_gain, max_step_norm));
  }
  s->iterations_run += iters;
  return 0;
}

int session_gradient(TsneSession* s, float exaggeration, float* grad_host, double* z_out) {
  FE_TRY(launch_iteration(s, kGradOnly, exaggeration, 0.f, 0.f, 0.f, 0.f));
  FE_CUDA(cudaMemcpyAsync(grad_host, s->grad_out, sizeof(float2) * s->n, cudaMemcpyDeviceToHost, s->stream),
          "D2H gradient");
  LayoutStats st;
  FE_CUDA(cudaMemcpyAsync(&st, s->stats, sizeof(st), cudaMemcpyDeviceToHost, s->stream), "D2H stats");
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(gradient)");
  if (z_out) *z_out = st.z;
  return 0;
}

int session_get_layout(TsneSession* s, float* out, bool host) {
  // The newest layout is uncentred until the next splat; centre into grad_out.
  FE_TRY(launch_center_output(s, s->grad_out));
  FE_CUDA(cudaMemcpyAsync(out, s->grad_out, sizeof(float2) * s->n,
                          host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice, s->stream),
          "copy layout out");
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(layout)");
  return 0;
}

}  // namespace fe
