// nccl_dl.cpp -- run-time binding of the NCCL calls used by the expert-parallel path.
#include "nccl_dl.h"

#include <dlfcn.h>

#include <mutex>

namespace jmoe {

namespace {

std::once_flag g_once;
NcclApi g_api;
bool g_ok = false;
const char *g_why = "NCCL not loaded";

template <typename F>
bool bind(void *h, const char *name, F &fn)
{
    fn = reinterpret_cast<F>(dlsym(h, name));
    return fn != nullptr;
}

void load()
{
    // RTLD_NOLOAD first: reuse an NCCL the process already has
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        g_why = "libnccl.so.2 could not be loaded";
        return;
    }
    bool ok = bind(h, "ncclGetUniqueId", g_api.GetUniqueId) && bind(h, "ncclCommInitRank", g_api.CommInitRank) &&
              bind(h, "ncclCommDestroy", g_api.CommDestroy) && bind(h, "ncclAllGather", g_api.AllGather) &&
              bind(h, "ncclSend", g_api.Send) && bind(h, "ncclRecv", g_api.Recv) &&
              bind(h, "ncclGroupStart", g_api.GroupStart) && bind(h, "ncclGroupEnd", g_api.GroupEnd) &&
              bind(h, "ncclGetErrorString", g_api.GetErrorString);
    if (!ok) {
        g_why = "libnccl.so.2 lacks an expected symbol";
        return;
    }
    g_ok = true;
    g_why = nullptr;
}

}  // namespace

const NcclApi *nccl_api(const char **why)
{
    std::call_once(g_once, load);
    if (why) *why = g_why;
    return g_ok ? &g_api : nullptr;
}

}  // namespace jmoe
