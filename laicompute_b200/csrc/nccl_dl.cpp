// Run-time binding of the NCCL calls used for tensor parallelism.
#include "nccl_dl.h"

#include <dlfcn.h>

#include <mutex>

namespace laic {

const NcclApi* nccl_api(std::string& why) {
    static std::once_flag once;
    static NcclApi api;
    static bool ok = false;
    static std::string err;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            const char* e = dlerror();
            err = std::string("cannot load libnccl.so.2: ") + (e ? e : "unknown error");
            return;
        }
        auto get = [&](const char* name) -> void* {
            void* f = dlsym(h, name);
            if (!f && err.empty()) err = std::string("libnccl.so.2 lacks ") + name;
            return f;
        };
        api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(get("ncclGetUniqueId"));
        api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(get("ncclCommInitRank"));
        api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(get("ncclCommDestroy"));
        api.AllReduce = reinterpret_cast<decltype(api.AllReduce)>(get("ncclAllReduce"));
        api.AllGather = reinterpret_cast<decltype(api.AllGather)>(get("ncclAllGather"));
        api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(get("ncclGetErrorString"));
        ok = err.empty();
    });
    if (!ok) {
        why = err;
        return nullptr;
    }
    return &api;
}

}  // namespace laic
