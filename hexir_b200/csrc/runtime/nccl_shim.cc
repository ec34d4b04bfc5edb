// nccl_shim.cc -- dlopen of libnccl.so.2 (see nccl_shim.h).

#include "nccl_shim.h"

#include <dlfcn.h>

#include <mutex>

namespace hexir {

namespace {

Nccl g_nccl;
std::once_flag g_once;

template <typename Fn>
bool bind(void *lib, Fn &slot, const char *symbol, std::string &error) {
  void *p = dlsym(lib, symbol);
  if (!p) {
    error = std::string("libnccl is missing ") + symbol;
    return false;
  }
  slot = reinterpret_cast<Fn>(p);
  return true;
}

void load() {
  Nccl &n = g_nccl;
  // An NCCL already loaded into the process (e.g. by PyTorch) is reused.
  void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
  if (!lib)
    lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!lib)
    lib = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!lib) {
    const char *why = dlerror();
    n.error = std::string("cannot load libnccl: ") + (why ? why : "unknown");
    return;
  }
  std::string &e = n.error;
  n.ok = bind(lib, n.GetUniqueId, "ncclGetUniqueId", e) &&
         bind(lib, n.CommInitRank, "ncclCommInitRank", e) &&
         bind(lib, n.CommInitAll, "ncclCommInitAll", e) &&
         bind(lib, n.CommDestroy, "ncclCommDestroy", e) &&
         bind(lib, n.GroupStart, "ncclGroupStart", e) &&
         bind(lib, n.GroupEnd, "ncclGroupEnd", e) &&
         bind(lib, n.Broadcast, "ncclBroadcast", e) &&
         bind(lib, n.Send, "ncclSend", e) && bind(lib, n.Recv, "ncclRecv", e) &&
         bind(lib, n.AllReduce, "ncclAllReduce", e) &&
         bind(lib, n.GetErrorString, "ncclGetErrorString", e);
}

}  // namespace

const Nccl &nccl() {
  std::call_once(g_once, load);
  return g_nccl;
}

std::string nccl_message(const char *call, ncclResult_t result) {
  const Nccl &n = g_nccl;
  const char *msg = n.GetErrorString ? n.GetErrorString(result) : nullptr;
  return std::string(call) + " failed: " +
         (msg ? msg : ("NCCL error " + std::to_string(result)));
}

}  // namespace hexir
