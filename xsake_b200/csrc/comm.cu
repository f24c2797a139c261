// The one exchange of the HADS path: a float64 sum all-reduce of per-head entropy sums across
// ranks (calibration), for callers that have no torch.distributed (a JAX FFI handler, a C++
// trainer).  The reference gets it from jax.lax.pmean inside pmap (distributed/pmap_trainer.py:
// 54-55) and computes calibration on one device (training/trainer.py:79-117).
//
// NCCL is loaded at run time (dlopen of libnccl.so.2) rather than linked: inside a PyTorch or
// JAX process this returns the NCCL the framework already loaded, so two NCCL builds never
// meet in one process, and the library still loads on machines without NCCL (the calls then
// return XSAKE_EUNSUPPORTED).  Only the NCCL types come from nccl.h.
#include "common.cuh"

#include <cstring>
#include <dlfcn.h>
#include <mutex>
#include <nccl.h>

namespace xsake {
namespace {

struct Nccl {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
  char why[256] = {0};
};

Nccl g_nccl;
std::once_flag g_nccl_once;

const Nccl& nccl() {
  std::call_once(g_nccl_once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) {
      snprintf(g_nccl.why, sizeof(g_nccl.why), "libnccl.so.2 not found: %s", dlerror());
      return;
    }
    g_nccl.get_unique_id = reinterpret_cast<decltype(g_nccl.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    g_nccl.comm_init_rank = reinterpret_cast<decltype(g_nccl.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    g_nccl.all_reduce = reinterpret_cast<decltype(g_nccl.all_reduce)>(dlsym(h, "ncclAllReduce"));
    g_nccl.comm_destroy = reinterpret_cast<decltype(g_nccl.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    g_nccl.error_string = reinterpret_cast<decltype(g_nccl.error_string)>(dlsym(h, "ncclGetErrorString"));
    g_nccl.ok = g_nccl.get_unique_id && g_nccl.comm_init_rank && g_nccl.all_reduce && g_nccl.comm_destroy &&
                g_nccl.error_string;
    if (!g_nccl.ok) snprintf(g_nccl.why, sizeof(g_nccl.why), "libnccl.so.2 lacks an expected symbol");
  });
  return g_nccl;
}

#define XSAKE_NCCL_TRY(expr)                                                                 \
  do {                                                                                       \
    ncclResult_t r__ = (expr);                                                               \
    if (r__ != ncclSuccess)                                                                  \
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

extern "C" int xsake_comm_init(const uint8_t id[128], int nranks, int rank, void** comm_out) {
  clear_error();
  XSAKE_REQUIRE(id != nullptr && comm_out != nullptr, XSAKE_EINVAL, "NULL argument");
  XSAKE_REQUIRE(nranks >= 1 && rank >= 0 && rank < nranks, XSAKE_EINVAL, "rank %d of %d", rank, nranks);
  const Nccl& n = nccl();
  XSAKE_REQUIRE(n.ok, XSAKE_EUNSUPPORTED, "%s", n.why);
  ncclUniqueId uid;
  memcpy(uid.internal, id, sizeof(uid.internal));
  ncclComm_t c = nullptr;
  XSAKE_NCCL_TRY(n.comm_init_rank(&c, nranks, uid, rank));
  *comm_out = c;
  return XSAKE_OK;
}

extern "C" int xsake_comm_allreduce_sum_f64(void* comm, double* buf_dev, size_t count, void* stream) {
  clear_error();
  XSAKE_REQUIRE(comm != nullptr, XSAKE_EINVAL, "comm is NULL");
  XSAKE_REQUIRE(buf_dev != nullptr || count == 0, XSAKE_EINVAL, "buffer is NULL");
  const Nccl& n = nccl();
  XSAKE_REQUIRE(n.ok, XSAKE_EUNSUPPORTED, "%s", n.why);
  if (count == 0) return XSAKE_OK;
  XSAKE_NCCL_TRY(n.all_reduce(buf_dev, buf_dev, count, ncclFloat64, ncclSum, reinterpret_cast<ncclComm_t>(comm),
                              as_stream(stream)));
  return XSAKE_OK;
}

extern "C" int xsake_comm_destroy(void* comm) {
  clear_error();
  if (comm == nullptr) return XSAKE_OK;
  const Nccl& n = nccl();
  XSAKE_REQUIRE(n.ok, XSAKE_EUNSUPPORTED, "%s", n.why);
  XSAKE_NCCL_TRY(n.comm_destroy(reinterpret_cast<ncclComm_t>(comm)));
  return XSAKE_OK;
}
