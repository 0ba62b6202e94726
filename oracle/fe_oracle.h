/* CPU restatement of the reference's optimizer hot path (openTSNE FFT-grid
 * gradient + update, UMAP COO edge-SGD epoch, and the graphs they consume).
 *
 * TEST INFRASTRUCTURE ONLY: this is the parity checker for the CUDA product
 * (tests, __graft_entry__.smoke and bench.py's cpu_baseline leg).  The
 * product never links, loads or calls it.
 *
 * Every function names the reference routine (file:line, paths relative to
 * the fastEmbedR source tree) whose algorithm it restates.  Pinning: the
 * restatement is checked against the reference's own CPU code compiled
 * unmodified into oracle/_ref (see oracle/Makefile) and against golden
 * vectors generated from it (tests/golden/make_golden.py).
 *
 * Conventions: embeddings are row-major interleaved float[n*2]; KNN inputs
 * are R column-major (idx[j*n + i]); indices are 0-based unless an
 * index_offset is passed.
 */
#ifndef FE_ORACLE_H
#define FE_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------- t-SNE ---------------- */

/* tsne_fft_grid_size, src/tsne_neighbors.cpp:392-398 (grid_override<=0: env/default). */
int or_tsne_grid_size(int n, int grid_override);

/* compute_row_probabilities_float, src/tsne_neighbors.cpp:482-532. */
void or_tsne_row_probabilities(const float* dist_row, int k, double perplexity, float* row_p);

/* build_tsne_probabilities_float, src/tsne_neighbors.cpp:540-648.
 * col/val must hold 2*n*k entries.  Returns nnz, or -1 on invalid input. */
long long or_tsne_build_p(const int* idx_cm, const float* dist_cm, int n, int k,
                          int index_offset, double perplexity,
                          int* row_ptr, int* col, float* val);

/* compute_gradient_fft_grid_f, src/tsne_neighbors.cpp:1076-1182 (bilinear
 * splat on a GxG grid, linear convolution with q and q^2 kernels, bilinear
 * gather, Z = sum interp(phi_q) - n).  The convolution is evaluated with a
 * double-precision FFT (the reference uses its own float radix-2 FFT,
 * src/tsne_neighbors.cpp:650-758); inputs and outputs are float as in the
 * reference.  Optional out_z receives Z. */
void or_tsne_gradient_fft(const int* row_ptr, const int* col, const float* val, int n,
                          const float* y, float exaggeration, int grid_size,
                          float* grad, double* out_z);

/* The repulsive part only (grad overwritten), same algorithm as above. */
void or_tsne_repulsive_fft(const float* y, int n, int grid_size, float* grad, double* out_z);

/* add_sparse_attractive_gradient_f, src/tsne_neighbors.cpp:985-1012 (adds to grad). */
void or_tsne_attractive(const int* row_ptr, const int* col, const float* val, int n,
                        const float* y, float exaggeration, float* grad);

/* compute_gradient_pair_symmetric_f, src/tsne_neighbors.cpp:1014-1074 (exact O(n^2)). */
void or_tsne_gradient_exact(const int* row_ptr, const int* col, const float* val, int n,
                            const float* y, float exaggeration, float* grad);

/* apply_open_tsne_update_f + zero_mean_f, src/tsne_neighbors.cpp:1196-1245. */
void or_tsne_update(float* y, float* update, float* gains, const float* grad, int n,
                    float learning_rate, float momentum, float min_gain, float max_step_norm);
void or_tsne_zero_mean(float* y, int n);

/* evaluate_kl_f with exact Z, src/tsne_neighbors.cpp:1247-1276 and 963-983. */
double or_tsne_kl(const int* row_ptr, const int* col, const float* val, int n, const float* y);

/* run_phase loop of knn_tsne_opentsne_float_cpp, src/tsne_neighbors.cpp:1723-1805,
 * starting from a given init (zero-meaned first, :1700). */
int or_tsne_run(const int* row_ptr, const int* col, const float* val, int n, const float* init,
                int early_exaggeration_iter, int n_iter, float early_exaggeration,
                float exaggeration, float learning_rate, int learning_rate_auto,
                float initial_momentum, float final_momentum, float min_gain,
                float max_step_norm, int grid_size, float* out);

/* The run_phase loop body for `iters` iterations from a given optimizer state. */
void or_tsne_iterate(const int* row_ptr, const int* col, const float* val, int n, float* y,
                     float* update, float* gains, int iters, float exaggeration, float momentum,
                     float learning_rate, float min_gain, float max_step_norm, int grid_size);

/* ---------------- UMAP ---------------- */

/* umap_powf_fast, src/fast_knn_umap.cpp:179-206 (Schraudolph-style exponent interpolation). */
float or_umap_powf(float x, float b);

/* Schedules, src/fast_knn_umap.cpp:595-636. */
int or_umap_positive_samples(float period, int epoch);
int or_umap_negative_samples(float period, int negative_sample_rate, int epoch);

/* deterministic_vertex_cuda_style, src/fast_knn_umap.cpp:535-547 (key = edge id), and the
 * CUDA kernels' variant src/embedding_cuda_kernels.cpp:252-264 (key = tail id). */
int or_umap_negative_vertex(int n, uint32_t seed, int epoch, int head, uint32_t key, int sample);

/* find_ab_params, src/fast_knn_umap.cpp:428-488. */
void or_umap_find_ab(double spread, double min_dist, double* a, double* b);

/* One epoch in delta (Jacobi) form: every force is evaluated against the
 * layout frozen at epoch start, accumulated, then applied with NaN->0 and a
 * +-max_abs_coord clamp.  Follows embed_epoch_coo_delta_kernel +
 * apply_delta_sanitize_layout_kernel, src/embedding_cuda_kernels.cpp:3136-3222,
 * with the per-edge arithmetic of fast_knn_umap_coo_replay_cpp,
 * src/fast_knn_umap.cpp:4969-5026.  hash_key_is_tail = 0 keys negatives on
 * the edge id (CPU replay), 1 on the tail id (reference CUDA kernels).
 * Accumulation is in double. */
void or_umap_epoch_delta(const int* heads, const int* tails, const float* epochs_per_sample,
                         int n_edges, float* layout, int n, int epoch, int n_epochs,
                         int negative_sample_rate, float learning_rate, float a, float b,
                         float repulsion_strength, uint32_t seed, int hash_key_is_tail,
                         float max_abs_coord);

/* Sequential in-place replay, identical in order and arithmetic to
 * fast_knn_umap_coo_replay_cpp with n_threads = 1, src/fast_knn_umap.cpp:4904-5056. */
void or_umap_replay_serial(const int* heads, const int* tails, const float* epochs_per_sample,
                           int n_edges, float* layout, int n, int epoch_begin, int epoch_end,
                           int n_epochs, int negative_sample_rate, float learning_rate, float a,
                           float b, float repulsion_strength, uint32_t seed, int hash_key_is_tail,
                           int sanitize_each_epoch);

/* Fuzzy-union CSR graph + epochs_per_sample: smooth_knn_dist
 * (src/fast_knn_umap.cpp:867-994), directed weights and union
 * (build_graph_csr_native_direct_values, :1553-1771, with edge_budget = k),
 * attach_csr_epoch_schedule (:1255-1273).  neighbors/weights/eps hold 2*n*k.
 * Returns nnz (or -1). */
long long or_umap_graph(const int* idx_cm, const float* dist_cm, int n, int k, int index_offset,
                        int* offsets, int* neighbors, float* weights, float* epochs_per_sample,
                        float* max_weight);

/* Row capacity of the device-KNN graph, min(256, 2k) (src/embedding_cuda_kernels.cpp:4996). */
int or_umap_graph_width(int k);

/* The device-KNN path's fuzzy graph (prepare_device_knn_graph,
 * src/embedding_cuda_kernels.cpp:3241-3321, kernels :1004-1160) as dense rows
 * nbr/w[n * width]; empty slots hold (row, 0).  The reference fills slots with
 * atomics; this restatement fixes the order the B200 library uses: own
 * entries in rank order, then incoming-only entries in ascending (source row,
 * rank) order, dropped once the row is full.  Returns width (or -1). */
int or_umap_device_graph(const int* idx_cm, const float* dist_cm, int n, int k, int index_offset,
                         int binary, int* nbr, float* w);

/* Non-empty slots as COO (mark_valid_graph_entries_rank_major_kernel and
 * pack_coo_graph_from_selected_rank_major_kernel, :2983-3022): rank-major
 * (rank_major = 1) or grouped by head.  epochs_per_sample = 1 / max(w, 1e-6).
 * Outputs hold n * width.  Returns the edge count. */
long long or_umap_pack_coo(const int* nbr, const float* w, int n, int width, int rank_major, int* heads,
                           int* tails, float* weights, float* epochs_per_sample);

/* Diffusion start layout of the device-KNN path (random_init_kernel,
 * diffuse_init_kernel, normalize_device_init, :1162-1319, 3323-3337): hashed
 * uniform start, whitened, then `iters` rounds of weighted neighbour averaging,
 * each whitened.  Moments are summed in double in row order. */
void or_umap_diffusion_init(const int* nbr, const float* w, int n, int width, uint32_t seed, int iters,
                            float* out);

#ifdef __cplusplus
}
#endif

#endif
