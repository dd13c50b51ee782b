// NCCL collectives on raw device pointers, for the tensor-parallel paths
// (the reference has a single device and no collectives; this is new).
//
// NCCL is resolved with dlopen at first use: an already-loaded libnccl.so.2
// (PyTorch's) is preferred so the process holds one NCCL, then the path in
// TVARANT_NCCL_LIBRARY, then the default search.  Without NCCL every entry
// point returns TVR_ERR_NCCL.
#include "internal.h"

#include <dlfcn.h>

#include <climits>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace tvr {
namespace {

using nccl_result = int;
using nccl_comm = void*;
struct NcclId {
  char internal[128];
};

// Layout of ncclConfig_t as NCCL 2.28 defines it (the struct is part of
// NCCL's ABI: size, magic and version lead, then the tunable fields).
struct NcclConfig {
  size_t size;
  unsigned int magic;
  unsigned int version;
  int blocking;
  int cgaClusterSize;
  int minCTAs;
  int maxCTAs;
  const char* netName;
  int splitShare;
  int trafficClass;
  const char* commName;
  int collnetEnable;
  int CTAPolicy;
  int shrinkShare;
  int nvlsCTAs;
  int nChannelsPerNetPeer;
  int nvlinkCentricSched;
};
constexpr int kNcclUndef = INT_MIN;

struct NcclApi {
  nccl_result (*getUniqueId)(NcclId*) = nullptr;
  nccl_result (*commInitRank)(nccl_comm*, int, NcclId, int) = nullptr;
  nccl_result (*commInitRankConfig)(nccl_comm*, int, NcclId, int, NcclConfig*) = nullptr;
  nccl_result (*getVersion)(int*) = nullptr;
  nccl_result (*allReduce)(const void*, void*, size_t, int, int, nccl_comm, cudaStream_t) = nullptr;
  nccl_result (*allGather)(const void*, void*, size_t, int, nccl_comm, cudaStream_t) = nullptr;
  nccl_result (*commDestroy)(nccl_comm) = nullptr;
  nccl_result (*commAbort)(nccl_comm) = nullptr;
  const char* (*getErrorString)(nccl_result) = nullptr;
};

std::once_flag g_once;
NcclApi g_api;
bool g_ok = false;

void load() {
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (h == nullptr) {
    const char* path = std::getenv("TVARANT_NCCL_LIBRARY");
    if (path != nullptr && path[0] != '\0') h = dlopen(path, RTLD_NOW | RTLD_GLOBAL);
  }
  if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (h == nullptr) return;
  bool ok = true;
  auto sym = [&](const char* name, auto* fn) {
    void* p = dlsym(h, name);
    if (p == nullptr) ok = false;
    *fn = reinterpret_cast<std::remove_pointer_t<decltype(fn)>>(p);
  };
  sym("ncclGetUniqueId", &g_api.getUniqueId);
  sym("ncclCommInitRank", &g_api.commInitRank);
  sym("ncclAllReduce", &g_api.allReduce);
  sym("ncclAllGather", &g_api.allGather);
  sym("ncclCommDestroy", &g_api.commDestroy);
  sym("ncclCommAbort", &g_api.commAbort);
  sym("ncclGetErrorString", &g_api.getErrorString);
  g_ok = ok;
  // optional: configured communicators (NCCL 2.14+; the 2.28 layout is used)
  g_api.commInitRankConfig = reinterpret_cast<decltype(g_api.commInitRankConfig)>(
      dlsym(h, "ncclCommInitRankConfig"));
  g_api.getVersion = reinterpret_cast<decltype(g_api.getVersion)>(dlsym(h, "ncclGetVersion"));
}

const NcclApi* api() {
  std::call_once(g_once, load);
  return g_ok ? &g_api : nullptr;
}

int nccl_fail(const NcclApi* a, nccl_result r, const char* what) {
  return fail(TVR_ERR_NCCL, "%s failed: %s", what, a->getErrorString ? a->getErrorString(r) : "?");
}

// tvarant dtype ids -> ncclDataType_t
int nccl_dtype(int dtype) {
  switch (dtype) {
    case 0: return 7;  // ncclFloat32
    case 1: return 8;  // ncclFloat64
    case 2: return 2;  // ncclInt32
    case 3: return 4;  // ncclInt64
    default: return -1;
  }
}

}  // namespace
}  // namespace tvr

using namespace tvr;

extern "C" {

int tvr_nccl_available(int* available) {
  TVR_CHECK(available != nullptr, "tvr_nccl_available: null output");
  *available = api() != nullptr ? 1 : 0;
  return TVR_OK;
}

int tvr_nccl_get_unique_id(void* id128) {
  TVR_CHECK(id128 != nullptr, "tvr_nccl_get_unique_id: null output");
  const NcclApi* a = api();
  if (a == nullptr) return fail(TVR_ERR_NCCL, "NCCL library not found");
  NcclId id;
  nccl_result r = a->getUniqueId(&id);
  if (r != 0) return nccl_fail(a, r, "ncclGetUniqueId");
  memcpy(id128, &id, sizeof(id));
  return TVR_OK;
}

int tvr_nccl_comm_init(void** comm, int nranks, const void* id128, int rank, int device) {
  TVR_CHECK(comm != nullptr && id128 != nullptr, "tvr_nccl_comm_init: null argument");
  TVR_CHECK(nranks > 0 && rank >= 0 && rank < nranks, "tvr_nccl_comm_init: bad rank %d of %d",
            rank, nranks);
  const NcclApi* a = api();
  if (a == nullptr) return fail(TVR_ERR_NCCL, "NCCL library not found");
  int rc = tvr_set_device(device);
  if (rc != TVR_OK) return rc;
  NcclId id;
  memcpy(&id, id128, sizeof(id));
  nccl_comm c = nullptr;
  nccl_result r = a->commInitRank(&c, nranks, id, rank);
  if (r != 0) return nccl_fail(a, r, "ncclCommInitRank");
  *comm = c;
  return TVR_OK;
}

int tvr_nccl_comm_init_ctas(void** comm, int nranks, const void* id128, int rank, int device,
                            int max_ctas) {
  TVR_CHECK(comm != nullptr && id128 != nullptr, "tvr_nccl_comm_init_ctas: null argument");
  const NcclApi* a = api();
  if (a == nullptr) return fail(TVR_ERR_NCCL, "NCCL library not found");
  int version = 0;
  if (max_ctas <= 0 || a->commInitRankConfig == nullptr || a->getVersion == nullptr ||
      a->getVersion(&version) != 0 || version < 22800) {
    return tvr_nccl_comm_init(comm, nranks, id128, rank, device);
  }
  TVR_CHECK(nranks > 0 && rank >= 0 && rank < nranks, "tvr_nccl_comm_init_ctas: bad rank %d of %d",
            rank, nranks);
  int rc = tvr_set_device(device);
  if (rc != TVR_OK) return rc;
  NcclConfig cfg;
  cfg.size = sizeof(NcclConfig);
  cfg.magic = 0xcafebeef;
  cfg.version = static_cast<unsigned int>(version);
  cfg.blocking = cfg.cgaClusterSize = cfg.minCTAs = kNcclUndef;
  cfg.maxCTAs = max_ctas;
  cfg.netName = nullptr;
  cfg.splitShare = cfg.trafficClass = kNcclUndef;
  cfg.commName = nullptr;
  cfg.collnetEnable = cfg.CTAPolicy = cfg.shrinkShare = cfg.nvlsCTAs = kNcclUndef;
  cfg.nChannelsPerNetPeer = cfg.nvlinkCentricSched = kNcclUndef;
  NcclId id;
  memcpy(&id, id128, sizeof(id));
  nccl_comm c = nullptr;
  nccl_result r = a->commInitRankConfig(&c, nranks, id, rank, &cfg);
  if (r != 0) return nccl_fail(a, r, "ncclCommInitRankConfig");
  *comm = c;
  return TVR_OK;
}

int tvr_nccl_all_reduce(const void* send, void* recv, int64_t count, int dtype, int op,
                        void* comm, void* stream) {
  const NcclApi* a = api();
  if (a == nullptr) return fail(TVR_ERR_NCCL, "NCCL library not found");
  TVR_CHECK(comm != nullptr, "tvr_nccl_all_reduce: null communicator");
  TVR_CHECK(count >= 0, "tvr_nccl_all_reduce: negative count");
  const int dt = nccl_dtype(dtype);
  TVR_CHECK(dt >= 0, "tvr_nccl_all_reduce: unsupported dtype %d", dtype);
  TVR_CHECK(op == 0, "tvr_nccl_all_reduce: only sum (0) is supported");
  nccl_result r = a->allReduce(send, recv, static_cast<size_t>(count), dt, 0, comm,
                               as_stream(stream));
  if (r != 0) return nccl_fail(a, r, "ncclAllReduce");
  return TVR_OK;
}

int tvr_nccl_all_gather(const void* send, void* recv, int64_t send_count, int dtype, void* comm,
                        void* stream) {
  const NcclApi* a = api();
  if (a == nullptr) return fail(TVR_ERR_NCCL, "NCCL library not found");
  TVR_CHECK(comm != nullptr, "tvr_nccl_all_gather: null communicator");
  const int dt = nccl_dtype(dtype);
  TVR_CHECK(dt >= 0, "tvr_nccl_all_gather: unsupported dtype %d", dtype);
  nccl_result r = a->allGather(send, recv, static_cast<size_t>(send_count), dt, comm,
                               as_stream(stream));
  if (r != 0) return nccl_fail(a, r, "ncclAllGather");
  return TVR_OK;
}

int tvr_nccl_comm_destroy(void* comm) {
  if (comm == nullptr) return TVR_OK;
  const NcclApi* a = api();
  if (a == nullptr) return fail(TVR_ERR_NCCL, "NCCL library not found");
  nccl_result r = a->commDestroy(comm);
  if (r != 0) return nccl_fail(a, r, "ncclCommDestroy");
  return TVR_OK;
}

int tvr_nccl_comm_abort(void* comm) {
  if (comm == nullptr) return TVR_OK;
  const NcclApi* a = api();
  if (a == nullptr) return fail(TVR_ERR_NCCL, "NCCL library not found");
  nccl_result r = a->commAbort(comm);
  if (r != 0) return nccl_fail(a, r, "ncclCommAbort");
  return TVR_OK;
}

}  // extern "C"
