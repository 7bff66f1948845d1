// nccl_dyn.cpp -- NCCL resolved at run time, only when tensor parallelism is used.
//
// The engine does not link libnccl: a process may already hold a different NCCL
// build under the same soname (PyTorch ships its own), and whichever loads first
// wins. The first tensor-parallel call resolves the API from, in order:
//   1. $EVELYN_NCCL_LIBRARY (a path),
//   2. a libnccl.so.2 already loaded in the process,
//   3. the system libnccl.so.2.
// The calls used (unique id, communicator init/destroy/abort, all-reduce, broadcast,
// all-gather, group start/end) are stable across NCCL 2.x.
#include <dlfcn.h>

#include <cstdlib>
#include <mutex>

#include "engine.hpp"

namespace evl {

namespace {
Nccl g_nccl;
std::once_flag g_once;
std::string g_nccl_error;

template <class F> bool sym(void* h, const char* name, F* out) {
    *out = reinterpret_cast<F>(dlsym(h, name));
    return *out != nullptr;
}

void load() {
    void* h = nullptr;
    if (const char* p = std::getenv("EVELYN_NCCL_LIBRARY")) h = dlopen(p, RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        const char* e = dlerror();
        g_nccl_error = std::string("cannot load libnccl.so.2: ") + (e ? e : "unknown error");
        return;
    }
    Nccl n;
    bool ok = sym(h, "ncclGetUniqueId", &n.GetUniqueId) && sym(h, "ncclCommInitRank", &n.CommInitRank) &&
              sym(h, "ncclCommDestroy", &n.CommDestroy) && sym(h, "ncclCommAbort", &n.CommAbort) &&
              sym(h, "ncclAllReduce", &n.AllReduce) && sym(h, "ncclBroadcast", &n.Broadcast) &&
              sym(h, "ncclAllGather", &n.AllGather) &&
              sym(h, "ncclGroupStart", &n.GroupStart) && sym(h, "ncclGroupEnd", &n.GroupEnd) &&
              sym(h, "ncclGetErrorString", &n.GetErrorString);
    if (!ok) {
        g_nccl_error = "libnccl.so.2 lacks a required symbol";
        return;
    }
    n.loaded = true;
    g_nccl = n;
}
}  // namespace

const Nccl& nccl() {
    std::call_once(g_once, load);
    if (!g_nccl.loaded) raise(EVL_ERR_NCCL, g_nccl_error);
    return g_nccl;
}

void nccl_check(ncclResult_t r, const char* what) {
    if (r != ncclSuccess) raise(EVL_ERR_NCCL, std::string(what) + ": " + nccl().GetErrorString(r));
}

}  // namespace evl
