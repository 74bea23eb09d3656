// nccl_dyn.h -- NCCL entry points resolved at run time (dlopen), so the
// library links no NCCL and a process that never uses tensor parallelism
// needs none.  Inside a PyTorch process the already-loaded libnccl.so.2 is
// reused; VELO_NCCL_LIB names another file.
#pragma once
#include <nccl.h>

namespace velo {

struct NcclApi {
    decltype(&ncclGetUniqueId) GetUniqueId = nullptr;
    decltype(&ncclCommInitRank) CommInitRank = nullptr;
    decltype(&ncclCommDestroy) CommDestroy = nullptr;
    decltype(&ncclAllReduce) AllReduce = nullptr;
    decltype(&ncclAllGather) AllGather = nullptr;
    decltype(&ncclGetErrorString) GetErrorString = nullptr;
    decltype(&ncclCommSplit) CommSplit = nullptr;  // optional (NCCL >= 2.18)
};

// The resolved API, or nullptr (message via set_last_error) if NCCL cannot be loaded.
const NcclApi* nccl_api();

}  // namespace velo
