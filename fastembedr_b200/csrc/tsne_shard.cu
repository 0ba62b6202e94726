// Sharding one t-SNE run across GPUs, one process per GPU.
//
// Decomposition (the optimizer's data flow, src/tsne_neighbors.cpp:1076-1256,
// split by rows of P):
//   * every rank keeps the whole layout y, the grid and the potentials;
//   * rank r owns the r-th block of rows_per_rank internal (Morton-ordered)
//     rows: it spreads their charges, streams their rows of P, and updates
//     their positions, gains and steps;
//   * the charge grids are summed with one in-place all-reduce.  Charges are
//     64-bit fixed point, so the sum is exact and independent of the number
//     of ranks; every rank then runs the (small) FFT convolution itself and Z
//     follows from the grid identity Z = sum_nodes m * phi_q - n, with no
//     second collective;
//   * the updated rows are all-gathered in place, then every rank reduces the
//     statistics of the whole new layout in the same fixed order.
// Two collectives per iteration, both captured in the iteration graphs.  A
// run on any number of ranks produces the same bits as a one-rank sharded run.
#include "nccl_loader.cuh"
#include "tsne.cuh"

#include <algorithm>
#include <cstring>
#include <string>

namespace fe {

int session_shard(TsneSession* s, const void* unique_id, void* lent_comm, int nranks, int rank) {
  if (s->sharded) {
    set_error("t-SNE session is already sharded");
    return 1;
  }
  if (nranks < 1 || nranks > TsneSession::kMaxRanks || rank < 0 || rank >= nranks) {
    set_error("t-SNE shard: need 1 <= nranks <= " + std::to_string(TsneSession::kMaxRanks) +
              " and 0 <= rank < nranks");
    return 1;
  }
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(shard)");
  ncclComm_t comm = static_cast<ncclComm_t>(lent_comm);
  if (comm == nullptr) FE_TRY(comm_init(unique_id, nranks, rank, &comm));
  s->comm = comm;
  s->own_comm = lent_comm == nullptr;
  s->sharded = true;
  s->shard_ranks = nranks;
  s->shard_rank = rank;
  const int per = (s->n + nranks - 1) / nranks;
  s->rows_per_rank = (per + 31) & ~31;
  s->row_begin = std::min(s->n, rank * s->rows_per_rank);
  s->row_end = std::min(s->n, s->row_begin + s->rows_per_rank);
  // The attraction grid covers this rank's rows only.
  const int rows = std::max(1, s->row_end - s->row_begin);
  grad_update_launch_shape(rows, &s->update_blocks, &s->update_threads);
  // The internal copy of P still holds every row, a superset of this rank's;
  // the next reorder rebuilds only the owned rows.
  drop_graphs(s);
  return build_group_order(s);
}

int shard_gather_rows(TsneSession* s, float2* rows) {
  if (s->shard_ranks == 1) return 0;  // one rank holds every row already
  const NcclApi* api = nccl_api();
  if (api == nullptr) return 1;
  const size_t count = 2 * static_cast<size_t>(s->rows_per_rank);  // floats per rank
  float* base = reinterpret_cast<float*>(rows);
  ncclComm_t comm = static_cast<ncclComm_t>(s->comm);
  return check_nccl_call(comm, api->AllGather(base + count * s->shard_rank, base, count, ncclFloat32, comm, s->stream),
                         "ncclAllGather(layout rows)");
}

int shard_sum_charges(TsneSession* s) {
  if (s->shard_ranks == 1) return 0;  // the local grid is the sum
  const NcclApi* api = nccl_api();
  if (api == nullptr) return 1;
  const size_t words = 4 * static_cast<size_t>(s->grid) * s->grid;  // ChargeCell = 4 x u64
  // Two's-complement sums of the fixed-point words: exactly the unsharded atomics.
  ncclComm_t comm = static_cast<ncclComm_t>(s->comm);
  return check_nccl_call(comm, api->AllReduce(s->charges, s->charges, words, ncclUint64, ncclSum, comm, s->stream),
                         "ncclAllReduce(charges)");
}

int shard_warm_up(TsneSession* s) {
  // Both collectives of an iteration, outside any graph capture, on buffers
  // they leave unchanged: the charge grid is all zeros between iterations and
  // the step buffer of a fresh session is zero on every rank.  NCCL sets up
  // its connections here rather than inside the first captured iteration.
  FE_TRY(shard_sum_charges(s));
  FE_TRY(shard_gather_rows(s, s->update));
  FE_CUDA(cudaStreamSynchronize(s->stream), "cudaStreamSynchronize(shard warm-up)");
  return 0;
}

void shard_release(TsneSession* s) {
  if (s->comm == nullptr) return;
  const NcclApi* api = nccl_api();
  if (api != nullptr && s->own_comm) api->CommDestroy(static_cast<ncclComm_t>(s->comm));
  s->comm = nullptr;
  s->sharded = false;
}

}  // namespace fe
