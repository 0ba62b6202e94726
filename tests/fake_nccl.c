/* A stand-in NCCL for failure-path tests (built by tests/test_nccl_faults_cpu.py).
 *
 * Every entry point the library resolves exists and fails: ncclGetUniqueId
 * returns ncclSystemError (2), as a host without a usable network interface
 * would, and the communicator calls return ncclRemoteError (6), as when a peer
 * has gone away.  Built with -DFAKE_NCCL_MISSING_ALLGATHER it lacks
 * ncclAllGather, like an incompatible library.  No GPU is touched. */
#include <string.h>

typedef struct { char internal[128]; } fake_unique_id;
typedef void* fake_comm;

static const char* const kMessages[] = {"no error", "unhandled cuda error", "fake: no usable network interface",
                                        "internal error", "invalid argument", "invalid usage",
                                        "fake: remote process exited", "operation in progress"};

const char* ncclGetErrorString(int code) {
  return code >= 0 && code < 8 ? kMessages[code] : "unknown";
}

int ncclGetUniqueId(fake_unique_id* id) {
  memset(id, 0, sizeof(*id));
  return 2;
}

int ncclCommInitRank(fake_comm* comm, int nranks, fake_unique_id id, int rank) {
  (void)nranks;
  (void)id;
  (void)rank;
  *comm = 0;
  return 6;
}

int ncclCommDestroy(fake_comm comm) {
  (void)comm;
  return 0;
}

int ncclCommAbort(fake_comm comm) {
  (void)comm;
  return 0;
}

int ncclAllReduce(const void* s, void* r, unsigned long n, int t, int op, fake_comm c, void* st) {
  (void)s; (void)r; (void)n; (void)t; (void)op; (void)c; (void)st;
  return 6;
}

#ifndef FAKE_NCCL_MISSING_ALLGATHER
int ncclAllGather(const void* s, void* r, unsigned long n, int t, fake_comm c, void* st) {
  (void)s; (void)r; (void)n; (void)t; (void)c; (void)st;
  return 6;
}
#endif
