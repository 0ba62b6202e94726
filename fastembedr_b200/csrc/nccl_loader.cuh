// NCCL, resolved at run time.
//
// The library does not link NCCL: single-GPU callers never need it, and a
// process that already holds a libnccl.so.2 (PyTorch bundles one) must not
// load a second copy.  The first sharded call opens "libnccl.so.2" (or the
// path in FASTEMBEDR_B200_NCCL_LIB) with dlopen, which returns the copy
// already loaded in the process when there is one, and resolves the handful of
// entry points used below.  Types and enum values come from nccl.h; they are
// part of NCCL's stable C ABI.
#pragma once

#include <nccl.h>

namespace fe {

struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*);
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t);
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  const char* (*GetErrorString)(ncclResult_t);
};

// The resolved table, or nullptr with the error text set.
const NcclApi* nccl_api();

// 0 on ncclSuccess; otherwise sets "<where>: <NCCL message>" and returns 1.
int check_nccl(ncclResult_t code, const char* where);

// check_nccl for a call on `comm`: a nonblocking communicator may answer
// ncclInProgress while NCCL finishes the call on its own threads (connection
// set-up at the first collective, for one); that is waited out, bounded by the
// join limit below, before the outcome is checked.
int check_nccl_call(ncclComm_t comm, ncclResult_t code, const char* where);

// Seconds a rank waits for the others to join a communicator:
// FASTEMBEDR_B200_NCCL_INIT_TIMEOUT_S, else the calling thread's JoinLimit,
// else 0 (as long as they take).
double join_timeout_seconds();

// A join limit for the calling thread while in scope (used where a library
// component joins several ranks itself and must never wait for good).
class JoinLimit {
 public:
  explicit JoinLimit(double seconds);
  ~JoinLimit();
  JoinLimit(const JoinLimit&) = delete;
  JoinLimit& operator=(const JoinLimit&) = delete;

 private:
  double prev_;
};

// Joins the communicator `unique_id` (ncclUniqueId bytes) as rank `rank` of
// `nranks`, on the current device, and returns once every rank has joined.
// With a join limit set the communicator is made nonblocking and polled; a
// rank whose peers have not all joined within the limit aborts it and returns
// 1 ("... timed out ...") instead of waiting for good.
int comm_init(const void* unique_id, int nranks, int rank, ncclComm_t* out);

}  // namespace fe

// A communicator made once and lent to any number of sessions in turn
// (fe_b200_comm_create); sessions never destroy it.
struct fe_b200_comm {
  ncclComm_t comm = nullptr;
  int nranks = 0;
  int rank = 0;
};
