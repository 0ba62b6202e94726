/* A stand-in NCCL for failure-path tests (built by tests/test_nccl_faults_cpu.py).
 *
 * Default build: every entry point the library resolves exists and fails:
 * ncclGetUniqueId returns ncclSystemError (2), as a host without a usable
 * network interface would, and the communicator calls return ncclRemoteError
 * (6), as when a peer has gone away.  Built with -DFAKE_NCCL_MISSING_ALLGATHER
 * it lacks ncclAllGather, like an incompatible library.
 *
 * Built with -DFAKE_NCCL_JOIN_POLLS=n it models the join of a communicator
 * instead: ncclGetUniqueId succeeds, ncclCommInitRankConfig answers
 * ncclInProgress (7), and ncclCommGetAsyncError reports ncclInProgress for the
 * first n polls and ncclSuccess after them; n < 0 is a peer that never joins.
 * The blocking ncclCommInitRank succeeds at once when n >= 0 and returns
 * ncclInvalidUsage (5) when n < 0 (the real call would wait for good).
 * fake_nccl_aborts / _polls / _last_blocking count what the caller did.
 * No GPU is touched.
 *
 * Built with -DFAKE_NCCL_TRACK it models live communicators for the rank
 * coordination test (tests/rank_group_harness.cpp): ncclCommInitRank hands out
 * a distinct communicator per rank, collectives succeed and are counted per
 * rank, fake_nccl_fail_call(rank, call) makes that rank's call number `call`
 * fail (ncclRemoteError), ncclCommAbort marks its communicator aborted, and
 * any later call on an aborted communicator is counted as a violation
 * (fake_nccl_calls_after_abort). */
#include <stddef.h>
#include <string.h>

typedef struct { char internal[128]; } fake_unique_id;
typedef void* fake_comm;
/* The leading fields of ncclConfig_t (NCCL's stable C ABI). */
typedef struct { size_t size; unsigned int magic; unsigned int version; int blocking; } fake_config_prefix;

#ifdef FAKE_NCCL_TRACK
#include <pthread.h>

#define FAKE_MAX_RANKS 64
typedef struct {
  int rank;
  int aborted;
  int destroyed;
} fake_tracked_comm;

static fake_tracked_comm g_comms[FAKE_MAX_RANKS];
static int g_calls[FAKE_MAX_RANKS];
static int g_fail_call[FAKE_MAX_RANKS];
static int g_after_abort = 0;
static int g_aborts = 0;
static pthread_mutex_t g_lock = PTHREAD_MUTEX_INITIALIZER;

void fake_nccl_reset(void) {
  pthread_mutex_lock(&g_lock);
  for (int r = 0; r < FAKE_MAX_RANKS; ++r) {
    g_comms[r].rank = r;
    g_comms[r].aborted = 0;
    g_comms[r].destroyed = 0;
    g_calls[r] = 0;
    g_fail_call[r] = -1;
  }
  g_after_abort = 0;
  g_aborts = 0;
  pthread_mutex_unlock(&g_lock);
}
void fake_nccl_fail_call(int rank, int call) { g_fail_call[rank] = call; }
int fake_nccl_calls(int rank) { return g_calls[rank]; }
int fake_nccl_calls_after_abort(void) { return g_after_abort; }
int fake_nccl_aborts(void) { return g_aborts; }
int fake_nccl_aborted(int rank) { return g_comms[rank].aborted; }

const char* ncclGetErrorString(int code) { return code == 0 ? "no error" : "fake: remote process exited"; }
int ncclGetUniqueId(fake_unique_id* id) {
  memset(id, 0, sizeof(*id));
  return 0;
}
int ncclCommInitRank(fake_comm* comm, int nranks, fake_unique_id id, int rank) {
  (void)nranks;
  (void)id;
  *comm = (fake_comm)&g_comms[rank];
  return 0;
}
int ncclCommInitRankConfig(fake_comm* comm, int nranks, fake_unique_id id, int rank, fake_config_prefix* config) {
  (void)config;
  return ncclCommInitRank(comm, nranks, id, rank);
}
int ncclCommGetAsyncError(fake_comm comm, int* state) {
  fake_tracked_comm* c = (fake_tracked_comm*)comm;
  pthread_mutex_lock(&g_lock);
  if (c->aborted) ++g_after_abort;
  pthread_mutex_unlock(&g_lock);
  *state = 0;
  return 0;
}
static int tracked_call(fake_comm comm) {
  fake_tracked_comm* c = (fake_tracked_comm*)comm;
  int rc = 0;
  pthread_mutex_lock(&g_lock);
  if (c->aborted || c->destroyed) {
    ++g_after_abort;
    rc = 6;
  } else if (g_calls[c->rank] == g_fail_call[c->rank]) {
    rc = 6;
  } else {
    ++g_calls[c->rank];
  }
  pthread_mutex_unlock(&g_lock);
  return rc;
}
int ncclCommDestroy(fake_comm comm) {
  fake_tracked_comm* c = (fake_tracked_comm*)comm;
  pthread_mutex_lock(&g_lock);
  if (c->aborted) ++g_after_abort;
  c->destroyed = 1;
  pthread_mutex_unlock(&g_lock);
  return 0;
}
int ncclCommAbort(fake_comm comm) {
  fake_tracked_comm* c = (fake_tracked_comm*)comm;
  pthread_mutex_lock(&g_lock);
  if (c->aborted) ++g_after_abort;  /* a second abort is a use after free too */
  c->aborted = 1;
  ++g_aborts;
  pthread_mutex_unlock(&g_lock);
  return 0;
}
int ncclAllReduce(const void* s, void* r, unsigned long n, int t, int op, fake_comm c, void* st) {
  (void)s; (void)r; (void)n; (void)t; (void)op; (void)st;
  return tracked_call(c);
}
int ncclAllGather(const void* s, void* r, unsigned long n, int t, fake_comm c, void* st) {
  (void)s; (void)r; (void)n; (void)t; (void)st;
  return tracked_call(c);
}
#else

static const char* const kMessages[] = {"no error", "unhandled cuda error", "fake: no usable network interface",
                                        "internal error", "invalid argument", "invalid usage",
                                        "fake: remote process exited", "operation in progress"};

static int g_aborts = 0;
static int g_polls = 0;
static int g_last_blocking = -1;
static int g_comm_storage = 0;

int fake_nccl_aborts(void) { return g_aborts; }
int fake_nccl_polls(void) { return g_polls; }
int fake_nccl_last_blocking(void) { return g_last_blocking; }

const char* ncclGetErrorString(int code) {
  return code >= 0 && code < 8 ? kMessages[code] : "unknown";
}

int ncclGetUniqueId(fake_unique_id* id) {
  memset(id, 0, sizeof(*id));
#ifdef FAKE_NCCL_JOIN_POLLS
  return 0;
#else
  return 2;
#endif
}

int ncclCommInitRank(fake_comm* comm, int nranks, fake_unique_id id, int rank) {
  (void)nranks;
  (void)id;
  (void)rank;
#ifdef FAKE_NCCL_JOIN_POLLS
  *comm = FAKE_NCCL_JOIN_POLLS >= 0 ? (fake_comm)&g_comm_storage : 0;
  return FAKE_NCCL_JOIN_POLLS >= 0 ? 0 : 5;
#else
  *comm = 0;
  return 6;
#endif
}

int ncclCommInitRankConfig(fake_comm* comm, int nranks, fake_unique_id id, int rank, fake_config_prefix* config) {
  (void)nranks;
  (void)id;
  (void)rank;
  g_last_blocking = config ? config->blocking : -1;
#ifdef FAKE_NCCL_JOIN_POLLS
  *comm = (fake_comm)&g_comm_storage;
  g_polls = 0;
  return 7;
#else
  *comm = 0;
  return 6;
#endif
}

int ncclCommGetAsyncError(fake_comm comm, int* state) {
  (void)comm;
  ++g_polls;
#ifdef FAKE_NCCL_JOIN_POLLS
  *state = (FAKE_NCCL_JOIN_POLLS < 0 || g_polls <= FAKE_NCCL_JOIN_POLLS) ? 7 : 0;
#else
  *state = 6;
#endif
  return 0;
}

int ncclCommDestroy(fake_comm comm) {
  (void)comm;
  return 0;
}

int ncclCommAbort(fake_comm comm) {
  (void)comm;
  ++g_aborts;
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
#endif  /* FAKE_NCCL_TRACK */
