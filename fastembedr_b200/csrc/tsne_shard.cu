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
#include "rank_group.h"
#include "tsne.cuh"

#include <algorithm>
#include <chrono>
#include <cstring>
#include <string>
#include <thread>

namespace fe {
namespace {

// Polls the newest collective's completion event for up to limit_s seconds
// (0: no limit).  1: completed; 0: still running at the limit; -1: CUDA error.
int await_collective(TsneSession* s, double limit_s) {
  using clock = std::chrono::steady_clock;
  const auto start = clock::now();
  for (long long spin = 0;; ++spin) {
    const cudaError_t q = cudaEventQuery(s->collective_done);
    if (q == cudaSuccess) return 1;
    if (q != cudaErrorNotReady) {
      check_cuda(q, "collective completion");
      return -1;
    }
    if (limit_s > 0.0 && std::chrono::duration<double>(clock::now() - start).count() >= limit_s) return 0;
    // Spin briefly (the device usually finishes within microseconds), then nap.
    if (spin < 2000) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// One collective of this rank.  Ungrouped sessions call NCCL directly (their
// collectives are also captured into iteration graphs).  Grouped sessions
// first wait for their previous collective to complete, then go through the
// group: every rank arrives before any enqueues, and nothing is enqueued on a
// communicator after its abort.
template <typename Call>
int shard_collective(TsneSession* s, const char* what, Call&& call) {
  if (s->group == nullptr) return call(static_cast<ncclComm_t>(s->comm));
  FE_TRY(shard_quiesce(s));
  if (s->collectives_issued == s->inject_failure_at) {
    // A host-side failure of this rank between two collectives, with none of
    // its collectives in flight (FASTEMBEDR_B200_INJECT_HOST_FAILURE).
    s->group->fail();
    set_error(std::string(what) + ": injected host failure of rank " + std::to_string(s->shard_rank) +
              " before collective " + std::to_string(s->collectives_issued));
    return 1;
  }
  int rc = 0;
  const RankGroup::Status st = s->group->collective(s->shard_rank, [&](void* comm) {
    rc = call(static_cast<ncclComm_t>(comm));
    if (rc == 0) rc = check_cuda(cudaEventRecord(s->collective_done, s->stream), "cudaEventRecord(collective)");
    return rc;
  });
  switch (st) {
    case RankGroup::kOk:
      s->collective_pending = true;
      ++s->collectives_issued;
      return 0;
    case RankGroup::kPeerFailed:
      set_error(std::string(what) + ": not issued, another rank of this process failed");
      return 1;
    case RankGroup::kAborted:
      set_error(std::string(what) + ": not issued, the communicator was aborted");
      return 1;
    default:
      return 1;  // the call's own message
  }
}

}  // namespace

int shard_quiesce(TsneSession* s) {
  if (s->group == nullptr || !s->collective_pending) return 0;
  const int done = await_collective(s, s->stall_limit_s);
  if (done == 1) {
    s->collective_pending = false;
    return 0;
  }
  // A collective that errs or does not complete in time: fail the group and ask
  // for the abort that ends every rank's collective, then wait (bounded again)
  // for ours to end, so that no kernel of this rank still uses the communicator.
  s->group->fail(true);
  if (done == 0) {
    set_error("a collective did not complete within " + std::to_string(s->stall_limit_s) +
              " s; the communicators of every rank were aborted");
  }
  if (await_collective(s, s->stall_limit_s) == 1) s->collective_pending = false;
  return 1;
}

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
  // Whole staged row blocks (kStageRows, a multiple of 32) per rank, so every
  // block and 32-row group is the same on any rank count.
  const int per = (s->n + nranks - 1) / nranks;
  s->rows_per_rank = (per + kStageRows - 1) / kStageRows * kStageRows;
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
  return shard_collective(s, "ncclAllGather(layout rows)", [&](ncclComm_t comm) {
    return check_nccl_call(comm, api->AllGather(base + count * s->shard_rank, base, count, ncclFloat32, comm,
                                                s->stream),
                           "ncclAllGather(layout rows)");
  });
}

int shard_sum_charges(TsneSession* s) {
  if (s->shard_ranks == 1) return 0;  // the local grid is the sum
  const NcclApi* api = nccl_api();
  if (api == nullptr) return 1;
  const size_t words = 4 * static_cast<size_t>(s->grid) * s->grid;  // ChargeCell = 4 x u64
  // Two's-complement sums of the fixed-point words: exactly the unsharded atomics.
  return shard_collective(s, "ncclAllReduce(charges)", [&](ncclComm_t comm) {
    return check_nccl_call(comm, api->AllReduce(s->charges, s->charges, words, ncclUint64, ncclSum, comm,
                                                s->stream),
                           "ncclAllReduce(charges)");
  });
}

int shard_warm_up(TsneSession* s) {
  // Both collectives of an iteration, outside any graph capture, on buffers
  // they leave unchanged: the charge grid is all zeros between iterations and
  // the step buffer of a fresh session is zero on every rank.  NCCL sets up
  // its connections here rather than inside the first captured iteration.
  FE_TRY(shard_sum_charges(s));
  FE_TRY(shard_gather_rows(s, s->update));
  FE_TRY(shard_quiesce(s));
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
