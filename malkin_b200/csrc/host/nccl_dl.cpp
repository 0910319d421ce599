// NCCL entry points resolved at first use with dlopen, not linked: a process that also loads PyTorch must share
// PyTorch's libnccl.so.2 (a second, older NCCL bound first breaks PyTorch's symbol lookup). dlopen of the SONAME
// returns the copy already loaded, else the system one.
#include "nccl_dl.hpp"

#include <dlfcn.h>

#include <mutex>
#include <stdexcept>
#include <string>

namespace mkb {

namespace {

struct Api {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclBroadcast) broadcast = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
};

Api g_api;
std::once_flag g_once;
std::string g_load_error;

template <typename T>
void sym(void* h, const char* name, T& out) {
  out = reinterpret_cast<T>(dlsym(h, name));
  if (!out) throw std::runtime_error(std::string("nccl: symbol ") + name + " not found");
}

void load() {
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
  if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    g_load_error = std::string("nccl: cannot load libnccl.so.2: ") + dlerror();
    return;
  }
  try {
    sym(h, "ncclGetUniqueId", g_api.get_unique_id);
    sym(h, "ncclCommInitRank", g_api.comm_init_rank);
    sym(h, "ncclCommDestroy", g_api.comm_destroy);
    sym(h, "ncclAllReduce", g_api.all_reduce);
    sym(h, "ncclAllGather", g_api.all_gather);
    sym(h, "ncclBroadcast", g_api.broadcast);
    sym(h, "ncclGroupStart", g_api.group_start);
    sym(h, "ncclGroupEnd", g_api.group_end);
    sym(h, "ncclGetErrorString", g_api.error_string);
  } catch (const std::exception& e) {
    g_load_error = e.what();
    g_api = Api{};
  }
}

const Api& api() {
  std::call_once(g_once, load);
  if (!g_api.get_unique_id) throw std::runtime_error(g_load_error);
  return g_api;
}

}  // namespace

ncclResult_t dl_get_unique_id(ncclUniqueId* id) { return api().get_unique_id(id); }
ncclResult_t dl_comm_init_rank(ncclComm_t* c, int n, ncclUniqueId id, int r) { return api().comm_init_rank(c, n, id, r); }
ncclResult_t dl_comm_destroy(ncclComm_t c) { return api().comm_destroy(c); }
ncclResult_t dl_all_reduce(const void* s, void* r, size_t n, ncclDataType_t t, ncclRedOp_t op, ncclComm_t c,
                           cudaStream_t st) {
  return api().all_reduce(s, r, n, t, op, c, st);
}
ncclResult_t dl_all_gather(const void* s, void* r, size_t n, ncclDataType_t t, ncclComm_t c, cudaStream_t st) {
  return api().all_gather(s, r, n, t, c, st);
}
ncclResult_t dl_broadcast(const void* s, void* r, size_t n, ncclDataType_t t, int root, ncclComm_t c,
                          cudaStream_t st) {
  return api().broadcast(s, r, n, t, root, c, st);
}
ncclResult_t dl_group_start() { return api().group_start(); }
ncclResult_t dl_group_end() { return api().group_end(); }
const char* dl_error_string(ncclResult_t r) { return api().error_string(r); }

}  // namespace mkb
