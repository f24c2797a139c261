// The one exchange of the HADS path: a float64 sum all-reduce of per-head entropy sums across
// ranks (calibration), for callers that have no torch.distributed (a JAX FFI handler, a C++
// trainer).  The reference gets it from jax.lax.pmean inside pmap (distributed/pmap_trainer.py:
// 54-55) and computes calibration on one device (training/trainer.py:79-117).
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, or of the file XSAKE_NCCL_LIBRARY names)
// rather than linked: inside a PyTorch or JAX process this returns the NCCL the framework already
// loaded, so two NCCL builds never meet in one process, and the library still loads on machines
// without NCCL (the calls then return XSAKE_EUNSUPPORTED).  Only the NCCL types come from nccl.h.
//
// Communicators are non-blocking (ncclConfig_t.blocking = 0) and every host-side wait is bounded:
// initialisation polls ncclCommGetAsyncError against a deadline (a rank that never joins), and
// xsake_comm_wait polls the stream and the communicator's error state (a rank that died or left
// a collective).  On expiry the communicator is aborted (ncclCommAbort, which also ends the
// communicator's kernels still waiting on the stream) and XSAKE_ETIMEOUT is returned; the
// process and its device stay usable, the communicator does not.
#include "common.cuh"

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <dlfcn.h>
#include <mutex>
#include <nccl.h>
#include <thread>
#include <type_traits>

namespace xsake {
namespace {

struct Nccl {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
  char why[512] = {0};
};

Nccl g_nccl;
std::once_flag g_nccl_once;

const Nccl& nccl() {
  std::call_once(g_nccl_once, [] {
    const char* path = getenv("XSAKE_NCCL_LIBRARY");
    void* h = dlopen(path && *path ? path : "libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h && !(path && *path)) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      snprintf(g_nccl.why, sizeof(g_nccl.why), "NCCL not found (%s): %s", path && *path ? path : "libnccl.so.2",
               dlerror());
      return;
    }
    auto sym = [&](auto& fn, const char* name) { fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name)); };
    sym(g_nccl.get_unique_id, "ncclGetUniqueId");
    sym(g_nccl.comm_init_rank_config, "ncclCommInitRankConfig");
    sym(g_nccl.all_reduce, "ncclAllReduce");
    sym(g_nccl.get_async_error, "ncclCommGetAsyncError");
    sym(g_nccl.comm_abort, "ncclCommAbort");
    sym(g_nccl.comm_destroy, "ncclCommDestroy");
    sym(g_nccl.error_string, "ncclGetErrorString");
    g_nccl.ok = g_nccl.get_unique_id && g_nccl.comm_init_rank_config && g_nccl.all_reduce && g_nccl.get_async_error &&
                g_nccl.comm_abort && g_nccl.comm_destroy && g_nccl.error_string;
    if (!g_nccl.ok) snprintf(g_nccl.why, sizeof(g_nccl.why), "the NCCL library lacks an expected symbol");
  });
  return g_nccl;
}

// The handle the C ABI hands out.
struct Comm {
  ncclComm_t c = nullptr;
  int timeout_ms = 0;      // bound of every host-side wait (<= 0: none)
  bool aborted = false;
};

constexpr int kDefaultTimeoutMs = 300000;

using Clock = std::chrono::steady_clock;

// Polls the communicator until its asynchronous state leaves ncclInProgress; aborts it when the
// deadline passes.  Returns XSAKE_OK, XSAKE_ECUDA (an NCCL error) or XSAKE_ETIMEOUT.
int settle(Comm* cm, const char* what, Clock::time_point deadline) {
  const Nccl& n = nccl();
  const auto spin_until = Clock::now() + std::chrono::microseconds(500);   // then back off
  for (;;) {
    ncclResult_t st = ncclInProgress;
    ncclResult_t r = n.get_async_error(cm->c, &st);
    if (r != ncclSuccess) {
      n.comm_abort(cm->c);
      cm->aborted = true;
      return set_error(XSAKE_ECUDA, "%s: ncclCommGetAsyncError failed: %s (communicator aborted)", what,
                       n.error_string(r));
    }
    if (st == ncclSuccess) return XSAKE_OK;
    if (st != ncclInProgress) {
      n.comm_abort(cm->c);
      cm->aborted = true;
      return set_error(XSAKE_ECUDA, "%s: %s (communicator aborted)", what, n.error_string(st));
    }
    if (cm->timeout_ms > 0 && Clock::now() > deadline) {
      n.comm_abort(cm->c);
      cm->aborted = true;
      return set_error(XSAKE_ETIMEOUT, "%s: no progress within %d ms (a rank did not join); communicator aborted",
                       what, cm->timeout_ms);
    }
    if (Clock::now() < spin_until)
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

Clock::time_point deadline_of(int timeout_ms) { return Clock::now() + std::chrono::milliseconds(timeout_ms); }

#define XSAKE_NCCL_TRY(expr)                                                                 \
  do {                                                                                       \
    ncclResult_t r__ = (expr);                                                               \
    if (r__ != ncclSuccess && r__ != ncclInProgress)                                         \
      return ::xsake::set_error(XSAKE_ECUDA, "%s failed: %s", #expr, nccl().error_string(r__)); \
  } while (0)

static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id size");

}  // namespace
}  // namespace xsake

using namespace xsake;

extern "C" int xsake_comm_unique_id(uint8_t id_out[128]) {
  clear_error();
  XSAKE_REQUIRE(id_out != nullptr, XSAKE_EINVAL, "id_out is NULL");
  const Nccl& n = nccl();
  XSAKE_REQUIRE(n.ok, XSAKE_EUNSUPPORTED, "%s", n.why);
  ncclUniqueId id;
  XSAKE_NCCL_TRY(n.get_unique_id(&id));
  memcpy(id_out, id.internal, sizeof(id.internal));
  return XSAKE_OK;
}

extern "C" int xsake_comm_init_ex(const uint8_t id[128], int nranks, int rank, int timeout_ms, void** comm_out) {
  clear_error();
  XSAKE_REQUIRE(id != nullptr && comm_out != nullptr, XSAKE_EINVAL, "NULL argument");
  XSAKE_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, XSAKE_EINVAL, "rank %d of %d", rank, nranks);
  *comm_out = nullptr;
  const Nccl& n = nccl();
  XSAKE_REQUIRE(n.ok, XSAKE_EUNSUPPORTED, "%s", n.why);
  ncclUniqueId uid;
  memcpy(uid.internal, id, sizeof(uid.internal));
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  Comm* cm = new Comm;
  cm->timeout_ms = timeout_ms;
  const auto deadline = deadline_of(timeout_ms);
  ncclResult_t r = n.comm_init_rank_config(&cm->c, nranks, uid, rank, &config);
  if (r != ncclSuccess && r != ncclInProgress) {
    if (cm->c) n.comm_abort(cm->c);
    delete cm;
    return set_error(XSAKE_ECUDA, "ncclCommInitRankConfig failed: %s", n.error_string(r));
  }
  int st = settle(cm, "xsake_comm_init", deadline);
  if (st) {
    delete cm;   // aborted by settle
    return st;
  }
  *comm_out = cm;
  return XSAKE_OK;
}

extern "C" int xsake_comm_init(const uint8_t id[128], int nranks, int rank, void** comm_out) {
  return xsake_comm_init_ex(id, nranks, rank, kDefaultTimeoutMs, comm_out);
}

extern "C" int xsake_comm_allreduce_sum_f64(void* comm, double* buf_dev, size_t count, void* stream) {
  clear_error();
  XSAKE_REQUIRE(comm != nullptr, XSAKE_EINVAL, "comm is NULL");
  XSAKE_REQUIRE(buf_dev != nullptr || count == 0, XSAKE_EINVAL, "buffer is NULL");
  const Nccl& n = nccl();
  XSAKE_REQUIRE(n.ok, XSAKE_EUNSUPPORTED, "%s", n.why);
  Comm* cm = static_cast<Comm*>(comm);
  XSAKE_REQUIRE(!cm->aborted, XSAKE_EINVAL, "communicator was aborted; destroy it");
  if (count == 0) return XSAKE_OK;
  const auto deadline = deadline_of(cm->timeout_ms);
  XSAKE_NCCL_TRY(n.all_reduce(buf_dev, buf_dev, count, ncclFloat64, ncclSum, cm->c, as_stream(stream)));
  return settle(cm, "xsake_comm_allreduce_sum_f64 (enqueue)", deadline);
}

extern "C" int xsake_comm_wait(void* comm, void* stream, int timeout_ms) {
  clear_error();
  XSAKE_REQUIRE(comm != nullptr, XSAKE_EINVAL, "comm is NULL");
  const Nccl& n = nccl();
  XSAKE_REQUIRE(n.ok, XSAKE_EUNSUPPORTED, "%s", n.why);
  Comm* cm = static_cast<Comm*>(comm);
  XSAKE_REQUIRE(!cm->aborted, XSAKE_EINVAL, "communicator was aborted; destroy it");
  const auto deadline = deadline_of(timeout_ms);
  const auto spin_until = Clock::now() + std::chrono::microseconds(500);
  for (;;) {
    const cudaError_t q = cudaStreamQuery(as_stream(stream));
    if (q == cudaSuccess) return XSAKE_OK;
    if (q != cudaErrorNotReady) return set_error(XSAKE_ECUDA, "cudaStreamQuery: %s", cudaGetErrorString(q));
    ncclResult_t st = ncclSuccess;
    if (n.get_async_error(cm->c, &st) == ncclSuccess && st != ncclSuccess && st != ncclInProgress) {
      n.comm_abort(cm->c);
      cm->aborted = true;
      return set_error(XSAKE_ECUDA, "xsake_comm_wait: %s (communicator aborted)", n.error_string(st));
    }
    if (timeout_ms > 0 && Clock::now() > deadline) {
      n.comm_abort(cm->c);
      cm->aborted = true;
      return set_error(XSAKE_ETIMEOUT, "xsake_comm_wait: the stream did not finish within %d ms; communicator "
                       "aborted", timeout_ms);
    }
    if (Clock::now() < spin_until)
      std::this_thread::yield();
    else
      std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

extern "C" int xsake_comm_destroy(void* comm) {
  clear_error();
  if (comm == nullptr) return XSAKE_OK;
  const Nccl& n = nccl();
  XSAKE_REQUIRE(n.ok, XSAKE_EUNSUPPORTED, "%s", n.why);
  Comm* cm = static_cast<Comm*>(comm);
  ncclResult_t r = ncclSuccess;
  if (!cm->aborted) r = n.comm_destroy(cm->c);   // an aborted communicator is already released
  delete cm;
  if (r != ncclSuccess && r != ncclInProgress)
    return set_error(XSAKE_ECUDA, "ncclCommDestroy failed: %s", n.error_string(r));
  return XSAKE_OK;
}
