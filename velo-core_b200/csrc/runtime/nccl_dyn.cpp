// nccl_dyn.cpp -- run-time binding of the NCCL functions the tensor-parallel
// verify step uses.
#include "runtime/nccl_dyn.h"

#include <dlfcn.h>

#include <cstdlib>
#include <mutex>

#include "runtime/context.h"

namespace velo {

const NcclApi* nccl_api() {
    static NcclApi api;
    static bool ok = false;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* env = std::getenv("VELO_NCCL_LIB");
        const char* names[] = {env, "libnccl.so.2", "libnccl.so"};
        void* h = nullptr;
        for (const char* n : names) {
            if (!n) continue;
            h = dlopen(n, RTLD_NOW | RTLD_LOCAL);
            if (h) break;
        }
        if (!h) return;
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
        api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
        api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(dlsym(h, "ncclAllReduce"));
        api.AllGather = reinterpret_cast<decltype(api.AllGather)>(dlsym(h, "ncclAllGather"));
        api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
        api.CommSplit = reinterpret_cast<decltype(api.CommSplit)>(dlsym(h, "ncclCommSplit"));
        ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllReduce && api.AllGather &&
             api.GetErrorString;
    });
    if (!ok) {
        set_last_error("NCCL (libnccl.so.2) could not be loaded; set VELO_NCCL_LIB");
        return nullptr;
    }
    return &api;
}

}  // namespace velo
