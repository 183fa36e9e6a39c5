#include "engine/nccl_shim.h"

#include <dlfcn.h>

#include <cstring>
#include <mutex>

namespace fb {

namespace {
struct IdByValue {
    char internal[kNcclIdBytes];
};
using InitRankFn = int (*)(NcclComm*, int, IdByValue, int);
InitRankFn g_init_rank = nullptr;

template <typename F>
bool sym(void* h, const char* name, F* out) {
    *out = reinterpret_cast<F>(dlsym(h, name));
    return *out != nullptr;
}
}  // namespace

Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        // Prefer an instance already loaded in the process (e.g. by torch).
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            n.error = std::string("cannot load libnccl.so.2: ") + dlerror();
            return;
        }
        bool ok = sym(h, "ncclGetUniqueId", &n.GetUniqueId) && sym(h, "ncclAllReduce", &n.AllReduce) &&
                  sym(h, "ncclAllGather", &n.AllGather) && sym(h, "ncclCommDestroy", &n.CommDestroy) &&
                  sym(h, "ncclCommAbort", &n.CommAbort) &&
                  sym(h, "ncclCommGetAsyncError", &n.CommGetAsyncError) &&
                  sym(h, "ncclGetErrorString", &n.GetErrorString) && sym(h, "ncclCommInitRank", &g_init_rank);
        if (!ok) {
            n.error = "libnccl.so.2 lacks a required symbol";
            return;
        }
        n.ok = true;
    });
    return n;
}

int nccl_comm_init_rank(NcclComm* comm, int nranks, const void* id, int rank) {
    if (!nccl().ok) return -1;
    IdByValue v;
    std::memcpy(v.internal, id, kNcclIdBytes);
    return g_init_rank(comm, nranks, v, rank);
}

}  // namespace fb
