/*
 * fastembedr_b200 -- B200-native drop-in for fastEmbedR's CUDA embedding optimizer.
 *
 * C ABI exported by libfastembedr_b200.so.  The first block reproduces, symbol
 * for symbol and argument for argument, the prototypes that the reference's
 * host wrapper src/embedding_cuda_impl.cpp declares (lines 24-380) and links
 * against; the original definitions live in src/embedding_cuda_kernels.cpp.
 * Conventions shared with the reference:
 *   - return 0 on success, 1 on failure; the message is then available from
 *     fastembedr_cuda_embedding_last_error() (thread-local);
 *   - KNN inputs are R column-major n x k (entry j of row i at j*n + i), with
 *     index_offset = 1 for 1-based indices;
 *   - layouts (init, out) are row-major interleaved float[n*2], caller-owned;
 *   - calls are synchronous and use the current CUDA device.
 * Symbols outside the optimizer hot path (landmarks, metrics, exact t-SNE,
 * legacy objectives, PCA/RAFT helpers) are exported so the wrapper links, and
 * return 1 with "not provided by the B200 backend".
 *
 * The second block (fe_b200_*) is this backend's own interface: sessions that
 * keep state resident on the device (benchmarks, checkpoint/resume), parity
 * hooks and multi-GPU sharding.  They have no counterpart in the reference.
 */
#ifndef FASTEMBEDR_B200_H
#define FASTEMBEDR_B200_H

#include <stdbool.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ===================================================================== */
/* Reference ABI (src/embedding_cuda_impl.cpp:24-380)                     */
/* ===================================================================== */

/* src/embedding_cuda_impl.cpp:25 */
bool fastembedr_cuda_available(void);
/* src/embedding_cuda_impl.cpp:26 */
const char* fastembedr_cuda_embedding_last_error(void);

/* openTSNE FFT-grid optimizer from host KNN with double distances.
 * src/embedding_cuda_impl.cpp:79-99 (definition src/embedding_cuda_kernels.cpp:6010-6037). */
int fastembedr_cuda_opentsne_fft_from_knn(const int* indices, const double* distances,
                                          const float* init, int has_init, int n, int k,
                                          int n_components, float perplexity,
                                          int early_exaggeration_iter, int n_iter,
                                          float early_exaggeration, float exaggeration,
                                          float learning_rate, int learning_rate_auto,
                                          float initial_momentum, float final_momentum,
                                          float min_gain, float max_step_norm, unsigned int seed,
                                          int index_offset, float* out);
/* Same with float32 distances.  src/embedding_cuda_impl.cpp:100-120 (kernels.cpp:6039-6066). */
int fastembedr_cuda_opentsne_fft_from_knn_float(const int* indices, const float* distances,
                                                const float* init, int has_init, int n, int k,
                                                int n_components, float perplexity,
                                                int early_exaggeration_iter, int n_iter,
                                                float early_exaggeration, float exaggeration,
                                                float learning_rate, int learning_rate_auto,
                                                float initial_momentum, float final_momentum,
                                                float min_gain, float max_step_norm,
                                                unsigned int seed, int index_offset, float* out);
/* Device-resident KNN (the GPU-KNN object's borrowed pointers).
 * src/embedding_cuda_impl.cpp:121-141 (kernels.cpp:6068-6095). */
int fastembedr_cuda_opentsne_fft_from_device_knn_float(
    const int* indices, const float* distances, const float* init, int has_init, int n, int k,
    int n_components, float perplexity, int early_exaggeration_iter, int n_iter,
    float early_exaggeration, float exaggeration, float learning_rate, int learning_rate_auto,
    float initial_momentum, float final_momentum, float min_gain, float max_step_norm,
    unsigned int seed, int index_offset, float* out);
/* Device-KNN with a PCA init computed on the device from the host data matrix
 * pca_init_values (n x pca_init_p, R column-major): the reference's RAFT TSVD start
 * (src/embedding_cuda_kernels.cpp:3357-3495, used at :5692-5724), here a double
 * covariance eigen-decomposition; the scores are signed so that each component's
 * largest-magnitude score is positive, then centred and scaled to sd 1e-4.
 * src/embedding_cuda_impl.cpp:142-183. */
int fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_double(
    const int* indices, const float* distances, const double* pca_init_values, int pca_init_p,
    int n, int k, int n_components, float perplexity, int early_exaggeration_iter, int n_iter,
    float early_exaggeration, float exaggeration, float learning_rate, int learning_rate_auto,
    float initial_momentum, float final_momentum, float min_gain, float max_step_norm,
    unsigned int seed, int index_offset, float* out);
int fastembedr_cuda_opentsne_fft_from_device_knn_float_pca_float(
    const int* indices, const float* distances, const float* pca_init_values, int pca_init_p,
    int n, int k, int n_components, float perplexity, int early_exaggeration_iter, int n_iter,
    float early_exaggeration, float exaggeration, float learning_rate, int learning_rate_auto,
    float initial_momentum, float final_momentum, float min_gain, float max_step_norm,
    unsigned int seed, int index_offset, float* out);

/* UMAP over a host COO graph.  optimizer_mode 0: in-place (Hogwild) atomics;
 * 1: Jacobi delta.  src/embedding_cuda_impl.cpp:243-258 (kernels.cpp:5325-5450). */
int fastembedr_cuda_umap_optimize_coo(const int* heads, const int* tails, const float* weights,
                                      const float* epochs_per_sample, const float* init, int n,
                                      int n_edges_capacity, int n_epochs, int negative_sample_rate,
                                      float learning_rate, float a, float b,
                                      float repulsion_strength, unsigned int seed,
                                      int optimizer_mode, float* out);

/* UMAP from KNN with graph build and diffusion ("spectral") init on the device.
 * src/embedding_cuda_impl.cpp:184-229 (kernels.cpp:5258-5323). */
int fastembedr_cuda_umap_from_knn_spectral(const int* indices, const double* distances, int n,
                                           int k, int n_epochs, int negative_sample_rate,
                                           float learning_rate, float a, float b,
                                           float repulsion_strength, int spectral_n_iter,
                                           unsigned int seed, int index_offset,
                                           int optimizer_mode, float* out);
int fastembedr_cuda_umap_from_knn_spectral_float(const int* indices, const float* distances,
                                                 int n, int k, int n_epochs,
                                                 int negative_sample_rate, float learning_rate,
                                                 float a, float b, float repulsion_strength,
                                                 int spectral_n_iter, unsigned int seed,
                                                 int index_offset, int optimizer_mode, float* out);
int fastembedr_cuda_umap_from_device_knn_spectral_float(
    const int* device_indices, const float* device_distances, int n, int k, int n_epochs,
    int negative_sample_rate, float learning_rate, float a, float b, float repulsion_strength,
    int spectral_n_iter, unsigned int seed, int index_offset, int optimizer_mode, int binary_graph,
    float* out);
/* The device-KNN fuzzy graph as a rank-major COO list (every row's slot 0, then
 * slot 1, ...).  The out arrays hold n * min(256, 2k) entries; *out_width gets
 * min(256, 2k) and *out_capacity the number of edges written.
 * src/embedding_cuda_impl.cpp:232-242 (kernels.cpp:4804-4964). */
int fastembedr_cuda_umap_graph_dump_from_knn(const int* indices, const double* distances, int n,
                                             int k, int index_offset, int* out_heads,
                                             int* out_tails, float* out_weights,
                                             float* out_epochs_per_sample, int* out_width,
                                             int* out_capacity);

/* ---- out of scope: exported for linking, return 1 (src/embedding_cuda_impl.cpp:27-78, 259-379) ---- */
int fastembedr_cuda_embed(const int* neighbors, const float* weights, const float* init, int n,
                          int k, int objective, int n_epochs, int negative_sample_rate,
                          float learning_rate, float a, float b, float max_weight,
                          unsigned int seed, float* out);
int fastembedr_cuda_embed_from_knn(const int* indices, const double* distances, const float* init,
                                   int n, int k, int objective, int n_epochs,
                                   int negative_sample_rate, float learning_rate, float a, float b,
                                   unsigned int seed, int index_offset, float* out);
int fastembedr_cuda_spectral_init_from_knn(const int* indices, const double* distances, int n,
                                           int k, int spectral_n_iter, unsigned int seed,
                                           int index_offset, float* out);
int fastembedr_cuda_exact_tsne_from_knn(const int* indices, const double* distances,
                                        const float* init, int n, int k, int n_epochs,
                                        float perplexity, float learning_rate, int stop_lying_iter,
                                        int mom_switch_iter, float momentum, float final_momentum,
                                        float exaggeration_factor, unsigned int seed,
                                        int index_offset, float* out);
int fastembedr_cuda_landmark_tsne_from_device_knn(
    const int* device_indices, const float* device_distances, int index_offset,
    const float* reference_data, const float* query_data, const float* reference_layout,
    int n_reference, int n_query, int n_features, int k, float perplexity, int n_iter,
    int early_exaggeration_iter, float learning_rate, float early_exaggeration, float exaggeration,
    float initial_momentum, float final_momentum, float max_grad_norm, float max_step_norm,
    int n_negatives, int exact_repulsion_threshold, unsigned int seed, int affine_neighbors,
    float affine_ridge, float max_extrapolation, float* out);
int fastembedr_cuda_landmark_umap_from_device_knn(
    const int* device_indices, const float* device_distances, int index_offset,
    const float* reference_data, const float* query_data, const float* reference_layout,
    const int* landmark_rows, const int* query_rows, int n_total, int n_reference, int n_query,
    int n_features, int k, int n_epochs, int negative_sample_rate, float learning_rate, float a,
    float b, float repulsion_strength, unsigned int seed, int affine_neighbors, float affine_ridge,
    float max_extrapolation, float* out);
int fastembedr_cuda_standardize_matrix(const double* values, int n, int p, double* out,
                                       double* center, double* scale);
int fastembedr_cuda_project_embedding(const double* reference_layout, const int* projection_indices,
                                      const double* projection_distances, int n_reference,
                                      int n_query, int k, int n_components, double* out);
int fastembedr_cuda_interpolate_landmark_layout(const double* landmark_layout,
                                                const int* landmark_indices,
                                                const int* projection_indices,
                                                const double* projection_distances,
                                                int n_landmarks, int n, int k, int n_components,
                                                double* out);
int fastembedr_cuda_landmark_project_interpolate_knn_confidence(
    const double* landmark_data, const double* query_data, const double* landmark_layout,
    const int* landmark_indices, int n_landmarks, int n, int n_features, int k, int n_components,
    double* out, int* projection_indices, double* projection_distances, double* confidence);
int fastembedr_cuda_knn_structure_score(const double* layout, const int* indices, const int* keep,
                                        const int* labels, int n, int index_rows,
                                        int high_rank_limit, int preserve_k, int keep_n,
                                        int compact_indices, int n_label_levels, double* totals);
int fastembedr_cuda_silhouette_score(const double* layout, const int* labels, const int* counts,
                                     int n, int n_label_levels, double* score);
int fastembedr_cuda_matrix_multiply(const double* left, const double* right, int left_rows,
                                    int left_cols, int right_cols, int transpose_left, double* out);
int fastembedr_cuda_raft_tsvd_pca_init(const double* values, int n, int p, int n_components,
                                       float* out);

/* ===================================================================== */
/* B200 backend extensions (no counterpart in the reference)              */
/* ===================================================================== */

/* Version string of this backend. */
const char* fe_b200_version(void);

/* Device memory retained between calls.  Every call draws its device buffers
 * from one memory pool per GPU that keeps freed blocks mapped for the next
 * call, up to FASTEMBEDR_B200_RETAIN_MB (default 32768; 0 = plain
 * cudaMalloc/cudaFree, nothing retained): unmapping the several GB of a
 * large call took the driver from milliseconds to more than half a second.
 * This returns every GPU's retained, unused memory to the driver (for a
 * caller about to need it elsewhere).  Returns 0, or 1 with fe_b200 /
 * fastembedr_cuda last-error text set. */
int fe_b200_release_memory(void);

/* ---- t-SNE sessions: device-resident state across calls ---- */
typedef struct fe_b200_tsne fe_b200_tsne;

/* Builds P on the device from column-major KNN (host or device pointers,
 * float32 distances), uploads init (row-major float[n*2]; NULL = the reference
 * CUDA path's hashed uniform init), and keeps everything resident.
 * grid_size 0 selects the reference CPU policy (64/128/256 by n, env
 * FASTEMBEDR_TSNE_FFT_GRID honoured). */
int fe_b200_tsne_create(const int* indices, const float* distances, int n, int k,
                        int index_offset, float perplexity, const float* init, unsigned int seed,
                        int grid_size, int inputs_on_device, fe_b200_tsne** out);
/* Same from an already symmetrised CSR P (host arrays; parity and resume). */
int fe_b200_tsne_create_csr(const int* row_ptr, const int* col, const float* val, int n,
                            const float* init, int grid_size, fe_b200_tsne** out);
/* Runs n_iter optimizer iterations with fixed phase parameters. */
int fe_b200_tsne_iterate(fe_b200_tsne* s, int n_iter, float exaggeration, float momentum,
                         float learning_rate, float min_gain, float max_step_norm);
/* Captures the CUDA graphs that fe_b200_tsne_iterate launches for this
 * parameter set, ahead of the first iterate with it (no iteration is run). */
int fe_b200_tsne_prepare(fe_b200_tsne* s, float exaggeration, float momentum, float learning_rate,
                         float min_gain, float max_step_norm);
/* Gradient at the current layout without updating it (grad: host float[n*2]). */
int fe_b200_tsne_gradient(fe_b200_tsne* s, float exaggeration, float* grad, double* z);
/* Current (centred) layout to host (on_device = 0) or device memory. */
int fe_b200_tsne_get_layout(fe_b200_tsne* s, float* out, int on_device);
/* Replaces the layout (and resets optimizer state when reset_state != 0). */
int fe_b200_tsne_set_layout(fe_b200_tsne* s, const float* y, int on_device, int reset_state);
/* Optimizer state (update, gains) to/from host, for checkpoint/resume. */
int fe_b200_tsne_get_state(fe_b200_tsne* s, float* update, float* gains);
int fe_b200_tsne_set_state(fe_b200_tsne* s, const float* update, const float* gains);
/* Sizes: n, grid G, nnz (symmetric entries), padded nnz. */
int fe_b200_tsne_info(fe_b200_tsne* s, int* n, int* grid, long long* nnz, long long* nnz_padded);
/* Copies the (unpadded) CSR P to host arrays of size n+1 / nnz / nnz. */
int fe_b200_tsne_get_p(fe_b200_tsne* s, int* row_ptr, int* col, float* val);
/* Row blocks of this session's rows (128 internal rows each) and how many of
 * them are staged: their attraction gathers y from the block's column union in
 * shared memory (set at each spatial reorder; the rest gather from L2).
 * Synchronises the session stream. */
int fe_b200_tsne_staged_blocks(fe_b200_tsne* s, int* staged, int* blocks);
/* Repulsion interpolation of a session: 0 = bilinear on the reference's G x G grid
 * (default; the reference's scheme, src/tsne_neighbors.cpp:1076-1182), 1 = FIt-SNE
 * boxes: square boxes of about one layout unit (at least 50 per side, at most G/3),
 * three nodes per box and side, quadratic Lagrange spread and gather.  No
 * counterpart in the reference; FASTEMBEDR_B200_INTERPOLATION=lagrange selects 1
 * for every session and one-shot call (and doubles the default G). */
int fe_b200_tsne_set_interpolation(fe_b200_tsne* s, int mode);
/* Exact Euclidean KNN on the device: the producer of the GPU-KNN object the
 * device-KNN entry points consume (the reference's native_cuda_knn_impl with its
 * exact route and finalize step, src/native_knn_cuda_impl.cpp:511-700, 418-470;
 * src/embedding_cuda_kernels.cpp:1412-1464).  data: n x p, R column-major,
 * double when data_double, on the device when data_on_device else on the host.
 * Writes the k nearest non-self points (exclude_self: the query's own index is
 * skipped) into caller-allocated device arrays, column-major n x k: indices
 * 1-based int32 (0 where fewer than k exist) and float32 Euclidean distances,
 * ascending (ties by index).  1 <= k <= min(n - 1, 247). */
int fe_b200_knn_exact(const void* data, int data_double, int data_on_device, int n, int p, int k,
                      int exclude_self, int* d_indices, float* d_distances);
/* The PCA start of the _pca_ entry points on its own: host data (n x p, R
 * column-major, double when values_double else float) to a host layout
 * out[2n] (row-major), on the current device. */
int fe_b200_pca_start(const void* values, int values_double, int n, int p, float* out);
/* The cudaStream_t the session launches on. */
void* fe_b200_tsne_stream(fe_b200_tsne* s);
/* Per-kernel CUDA-event timing: enable, then read per-kind totals
 * (kinds: 0 splat, 1 fft rows, 2 fft cols, 3 fft rows inverse, 4 gradient+update (gather),
 * 7 layout statistics, 8 gradient+update of staged row blocks, and for sharded
 * sessions 5 charge all-reduce, 6 layout all-gather). */
int fe_b200_tsne_profile(fe_b200_tsne* s, int enable);
int fe_b200_tsne_kernel_times(fe_b200_tsne* s, double* ms, long long* launches, int kinds);
const char* fe_b200_tsne_kernel_name(int kind);
void fe_b200_tsne_destroy(fe_b200_tsne* s);

/* ---- UMAP sessions (no counterpart in the reference) ----
 * The device-KNN UMAP path of fastembedr_cuda_umap_from_device_knn_spectral_float
 * split into set-up and epoch ranges.  fe_b200_umap_create builds the fuzzy
 * graph from column-major KNN (host or device pointers, float32 distances),
 * the diffusion start (spectral_n_iter rounds) and the rank-major COO edge
 * list, all resident on the device.  fe_b200_umap_run applies epochs
 * [epoch_begin, epoch_end) of an n_epochs schedule (optimizer_mode 0: Hogwild
 * per sample, 1: Jacobi), negatives keyed on the tail vertex as in the
 * reference's COO kernels.  fe_b200_umap_count_samples returns the positive
 * and negative edge samples that an epoch range applies. */
typedef struct fe_b200_umap fe_b200_umap;
int fe_b200_umap_create(const int* indices, const float* distances, int n, int k, int index_offset,
                        int inputs_on_device, int binary_graph, int spectral_n_iter, unsigned int seed,
                        fe_b200_umap** out);
int fe_b200_umap_run(fe_b200_umap* s, int epoch_begin, int epoch_end, int n_epochs, int negative_sample_rate,
                     float learning_rate, float a, float b, float repulsion_strength, unsigned int seed,
                     int optimizer_mode);
int fe_b200_umap_count_samples(fe_b200_umap* s, int epoch_begin, int epoch_end, int negative_sample_rate,
                               long long* positive, long long* negative);
/* Layout (row-major float[n*2]) to/from host (on_device = 0) or device memory. */
int fe_b200_umap_get_layout(fe_b200_umap* s, float* out, int on_device);
int fe_b200_umap_set_layout(fe_b200_umap* s, const float* y, int on_device);
int fe_b200_umap_info(fe_b200_umap* s, int* n, long long* n_edges);
/* The COO edge list (host arrays of n_edges entries; any may be NULL). */
int fe_b200_umap_get_graph(fe_b200_umap* s, int* heads, int* tails, float* epochs_per_sample);
void* fe_b200_umap_stream(fe_b200_umap* s);
void fe_b200_umap_destroy(fe_b200_umap* s);
/* Makes the session rank `rank` of an nranks-way run, one process per GPU
 * (id: bytes from fe_b200_nccl_unique_id made on one rank; blocks until every
 * rank has joined).  Rank r owns the r-th block of ceil(n / nranks) vertices
 * and keeps the edges that touch it; every epoch it applies the moves of its
 * own vertices against the epoch-start positions of the others, and the
 * blocks are then all-gathered.  Every rank must hold an identical session and
 * make the same calls in the same order.  In Jacobi mode the sharded epoch is
 * the unsharded one (up to float summation order); in Hogwild mode a rank
 * sees other ranks' moves from the next epoch on. */
int fe_b200_umap_shard(fe_b200_umap* s, const unsigned char* id, int id_bytes, int nranks, int rank);
/* The same on a communicator lent by fe_b200_comm_create (declared below). */
struct fe_b200_comm;
int fe_b200_umap_shard_comm(fe_b200_umap* s, struct fe_b200_comm* comm);

/* ---- sharding one t-SNE run across GPUs (one process per GPU) ----
 * No counterpart in the reference's C ABI: the reference's multi-GPU build
 * keeps one process and picks devices itself (src/embedding_cuda_impl.cpp:24-380
 * declares no such call).  NCCL is loaded at run time ("libnccl.so.2", or the
 * path in FASTEMBEDR_B200_NCCL_LIB).
 *
 * fe_b200_nccl_unique_id writes the id_bytes (>= 128) byte identifier of a new
 * communicator; one rank makes it and the host hands the bytes to every rank.
 * fe_b200_tsne_shard then joins the communicator (blocking until all nranks
 * ranks have joined) and makes the session rank `rank` of the run: each rank
 * spreads, attracts and updates its own block of points, the charge grid is
 * all-reduced and the updated points all-gathered every iteration.  Every
 * rank must create an identical session (same P, layout, grid) on its own
 * GPU, and from then on make the same session calls with the same arguments
 * in the same order.  Results are bit-identical for any number of ranks. */
int fe_b200_nccl_unique_id(unsigned char* id, int id_bytes);
int fe_b200_tsne_shard(fe_b200_tsne* s, const unsigned char* id, int id_bytes, int nranks, int rank);
/* A communicator made once per process and lent to sessions in turn (a session
 * sharded with fe_b200_*_shard_comm keeps using it and never destroys it), so
 * that repeated runs do not pay NCCL's set-up each time.  Sessions that share
 * one communicator must not run concurrently, and the communicator must
 * outlive them.  fe_b200_comm_create blocks until every rank has joined. */
typedef struct fe_b200_comm fe_b200_comm;
int fe_b200_comm_create(const unsigned char* id, int id_bytes, int nranks, int rank, fe_b200_comm** out);
void fe_b200_comm_destroy(fe_b200_comm* comm);
int fe_b200_tsne_shard_comm(fe_b200_tsne* s, fe_b200_comm* comm);

/* ---- UMAP parity hook ---- */
/* Runs epochs [epoch_begin, epoch_end) of the COO optimizer on layout
 * (row-major float[n*2], host, in/out).  hash_key_is_tail selects the
 * negative-sample key (0: edge id as the CPU replay, 1: tail id as the
 * reference CUDA kernels).  positive_samples (optional) receives the number of
 * positive edge samples applied. */
int fe_b200_umap_epochs(const int* heads, const int* tails, const float* epochs_per_sample,
                        long long n_edges, float* layout, int n, int epoch_begin, int epoch_end,
                        int n_epochs, int negative_sample_rate, float learning_rate, float a,
                        float b, float repulsion_strength, unsigned int seed, int optimizer_mode,
                        int hash_key_is_tail, long long* positive_samples);

/* ---- UMAP epochs without any device allocation ----
 * No counterpart in the reference.  For callers that cannot let a library
 * allocate device memory (a framework that owns the device heap through its
 * own allocator or pool, real-time loops where cudaMalloc/cudaFree would
 * synchronise the device, embedders with a fixed memory budget): runs epochs
 * [epoch_begin, epoch_end) of the COO optimizer in Jacobi (delta) mode --
 * optimizer_mode 1 of fe_b200_umap_epochs, same results -- entirely on
 * caller-owned DEVICE buffers (heads, tails, epochs_per_sample: n_edges each;
 * layout: row-major float[n*2], updated in place), on `stream`
 * (cudaStream_t; NULL = the legacy default stream), and returns after the work
 * has finished.  It calls no cudaMalloc, cudaFree or allocating library
 * routine: its only scratch, one float2 per vertex, is a fixed 8 MiB static
 * device array that every GPU loading this library holds until exit, so n is
 * limited to 1,048,576 vertices (larger n returns 1 with a message).  The
 * first call on a device looks up the array's address on that device; make
 * that first call before any stream capture.  All calls share the array and
 * clear it on entry; calls that overlap on the GPU race on it. */
int fe_b200_umap_epochs_noalloc(const int* heads, const int* tails,
                                const float* epochs_per_sample, long long n_edges, float* layout,
                                int n, int epoch_begin, int epoch_end, int n_epochs,
                                int negative_sample_rate, float learning_rate, float a, float b,
                                float repulsion_strength, unsigned int seed, int hash_key_is_tail,
                                void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FASTEMBEDR_B200_H */
