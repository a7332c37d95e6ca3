#include "nccl_shim.h"

#include <dlfcn.h>
#include <mutex>
#include <string.h>

#include "jinf/common.h"
#include "jinf/engine.h"

namespace jinf {

const NcclApi* nccl_api() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            JINF_LOG("NCCL unavailable: %s", dlerror());
            return;
        }
#define JINF_NCCL_SYM(field, name) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name))
        JINF_NCCL_SYM(GetUniqueId, "ncclGetUniqueId");
        JINF_NCCL_SYM(CommInitRank, "ncclCommInitRank");
        JINF_NCCL_SYM(CommDestroy, "ncclCommDestroy");
        JINF_NCCL_SYM(CommAbort, "ncclCommAbort");
        JINF_NCCL_SYM(CommGetAsyncError, "ncclCommGetAsyncError");
        JINF_NCCL_SYM(AllReduce, "ncclAllReduce");
        JINF_NCCL_SYM(AllGather, "ncclAllGather");
        JINF_NCCL_SYM(GetErrorString, "ncclGetErrorString");
#undef JINF_NCCL_SYM
        api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllReduce && api.AllGather &&
                 api.GetErrorString;
        if (!api.ok) JINF_LOG("NCCL library is missing symbols");
    });
    return api.ok ? &api : nullptr;
}

}  // namespace jinf

extern "C" jinf_status jinf_nccl_get_unique_id(void* out128) {
    if (!out128) return JINF_ERR_INVALID;
    const jinf::NcclApi* n = jinf::nccl_api();
    if (!n) return JINF_ERR_CUDA;
    ncclUniqueId id;
    if (n->GetUniqueId(&id) != ncclSuccess) return JINF_ERR_CUDA;
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId is 128 bytes");
    memcpy(out128, &id, sizeof id);
    return JINF_OK;
}
